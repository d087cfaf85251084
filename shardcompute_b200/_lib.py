"""ctypes binding of libsc_b200.so (the C ABI declared in include/sc_b200.h).

The library is loaded from the package directory (built in-tree by
``shardcompute_b200.build``).  There is no fallback: if the library is
missing or does not load, every op raises ``RuntimeError``.

Status codes map to the exception types the reference raises at the same
boundary (``parallel/quantized_linear.py:71-74,164-165``): shape and argument
errors -> ``ValueError``, CUDA / NCCL errors -> ``RuntimeError``, collective
timeouts -> ``TimeoutError``.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsc_b200.so")

SC_OK, SC_ERR_SHAPE, SC_ERR_CUDA, SC_ERR_NCCL, SC_ERR_TIMEOUT, SC_ERR_ARG, SC_ERR_UNSUPPORTED, SC_ERR_WORKSPACE = range(8)
SC_F16, SC_F32, SC_I32, SC_U8 = 0, 1, 2, 3
SC_EPI_STORE, SC_EPI_RESIDUAL, SC_EPI_SWIGLU = 0, 1, 2
SC_OP_SUM, SC_OP_MAX, SC_OP_MIN, SC_OP_AVG = 0, 1, 2, 3
ABI_VERSION = 1

_vp, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
_pp = C.POINTER(C.c_void_p)

# name -> (restype, argtypes), mirroring include/sc_b200.h
SIGNATURES = {
    "sc_abi_version": (_i, []),
    "sc_status_name": (C.c_char_p, [_i]),
    "sc_last_error": (C.c_char_p, []),
    "sc_launch_count": (C.c_ulonglong, []),
    "sc_qlinear_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "sc_qlinear_noalloc": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _i, _i, _vp]),
    "sc_qgemv_device_error": (_i, [_i]),
    "sc_qgemv_probe_stamps": (_i, [_vp]),
    "sc_l2_prefetch": (_i, [_pp, C.POINTER(_sz), _i, _sz, _vp]),
    "sc_qlinear": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    "sc_qlinear_fused": (_i, [_vp, _i, _i, _i, _i, _vp, _f, _i, _pp, _pp, _pp, C.POINTER(_i), _i, _i, _vp, _i,
                              _vp, _i, _i, _vp, _i, _vp, _sz, _vp]),
    "sc_qlinear_fused_prefetch": (_i, [_vp, _i, _i, _i, _i, _vp, _f, _i, _pp, _pp, _pp, C.POINTER(_i), _i, _i, _vp,
                                       _i, _vp, _i, _i, _vp, _i, _vp, _sz, _pp, C.POINTER(_sz), _i, _sz, _vp]),
    "sc_qlinear_allreduce": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    "sc_embed_gather_q": (_i, [_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i, _vp]),
    "sc_embed_gather_f16": (_i, [_vp, _i, _vp, _i, _i, _i, _vp, _i, _vp]),
    "sc_dequantize": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "sc_quantize": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "sc_rope_append": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _vp]),
    "sc_flash_decode_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "sc_flash_decode": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _i, _vp, _sz, _vp]),
    "sc_attn_decode_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "sc_attn_device_error": (_i, [_i]),
    "sc_attn_decode": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _i, _f, _i, _vp, _i, _vp, _sz, _vp,
                            _vp]),
    "sc_rmsnorm": (_i, [_vp, _i, _i, _i, _vp, _f, _vp, _i, _vp]),
    "sc_silu_mul": (_i, [_vp, _vp, _i, _sz, _vp, _i, _vp]),
    "sc_add": (_i, [_vp, _i, _vp, _i, _sz, _vp, _i, _vp]),
    "sc_argmax_workspace_bytes": (_sz, [_i, _i]),
    "sc_argmax": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _sz, _vp]),
    "sc_argmax_merge": (_i, [_vp, _vp, _i, _i, _vp, _vp, _i, _vp]),
    "sc_comm_unique_id": (_i, [_vp, _sz]),
    "sc_comm_init": (_i, [_vp, _sz, _i, _i, _pp]),
    "sc_comm_destroy": (_i, [_vp]),
    "sc_comm_abort": (_i, [_vp]),
    "sc_comm_poll": (_i, [_vp, C.POINTER(_i)]),
    "sc_allreduce": (_i, [_vp, _vp, _sz, _i, _i, _vp, _vp]),
    "sc_allgather": (_i, [_vp, _vp, _sz, _i, _vp, _vp]),
    "sc_broadcast": (_i, [_vp, _vp, _sz, _i, _i, _vp, _vp]),
    "sc_send": (_i, [_vp, _sz, _i, _i, _vp, _vp]),
    "sc_recv": (_i, [_vp, _sz, _i, _i, _vp, _vp]),
    "sc_p2p_handle_bytes": (_sz, []),
    "sc_p2p_create": (_i, [_i, _i, _sz, _pp, _vp, _sz]),
    "sc_p2p_open": (_i, [_vp, _vp, _sz]),
    "sc_p2p_open_loopback": (_i, [_vp]),
    "sc_p2p_set_timeout": (_i, [_vp, C.c_uint64]),
    "sc_p2p_status": (_i, [_vp, C.POINTER(_i)]),
    "sc_p2p_destroy": (_i, [_vp]),
    "sc_p2p_allreduce": (_i, [_vp, _vp, _sz, _i, _vp, _vp]),
    "sc_p2p_allgather": (_i, [_vp, _vp, _sz, _i, _vp, _vp]),
    "sc_p2p_arenas": (_i, [_vp, _pp, C.POINTER(_sz)]),
    "sc_step_create": (_i, [_i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _f, _i, _i, _i, _pp]),
    "sc_step_set_layer": (_i, [_vp, _i, _vp, _vp, _pp, _pp, _pp, _vp, _vp]),
    "sc_step_set_head": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "sc_step_set_io": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "sc_step_arena_bytes": (_sz, [_i, _i]),
    "sc_step_set_peers": (_i, [_vp, _pp, _sz]),
    "sc_step_workspace_bytes": (_sz, [_vp]),
    "sc_step_finalize": (_i, [_vp, _vp, _sz, _vp]),
    "sc_step_run": (_i, [_vp, _vp]),
    "sc_step_error": (_i, [_vp, _i]),
    "sc_step_error_info": (_i, [_vp, C.POINTER(_i), _i]),
    "sc_step_set_timing": (_i, [_vp, _vp]),
    "sc_step_timing_count": (C.c_size_t, [_vp]),
    "sc_step_fit": (_i, [_vp, C.POINTER(_i)]),
    "sc_qgemm_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "sc_qgemm": (_i, [_vp, _i, _i, _i, _i, _vp, _f, _i, _pp, _pp, _pp, C.POINTER(_i), _i, _i, _vp, _i, _vp, _i, _i,
                      _vp, _i, _vp, _sz, _vp]),
    "sc_qgemm_device_error": (_i, [_i]),
    "sc_sample_workspace_bytes": (_sz, [_i]),
    "sc_sample_topp": (_i, [_vp, _i, _i, _i, _f, _f, _vp, _i, _vp, _vp, _sz, _vp]),
    "sc_sample_phase": (_i, [_vp, _i, _i, _i, _f, _f, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "sc_sample_combine": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp]),
    "sc_sample_uniforms": (_i, [C.c_uint64, _vp, _i, _vp, _vp]),
    "sc_step_destroy": (_i, [_vp]),
}

_lib = None
_lock = threading.Lock()


class ScError(RuntimeError):
    """Raised for CUDA/NCCL failures reported by libsc_b200."""


def load() -> C.CDLL:
    """Load (once) and type the library; raise RuntimeError if unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libsc_b200.so not found at {LIB_PATH}; build it with `python -m shardcompute_b200.build` "
                "(there is no CPU fallback for the quantized decode path)")
        lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        v = lib.sc_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f"libsc_b200.so ABI {v} != expected {ABI_VERSION}; rebuild the library")
        _lib = lib
        return lib


def check(status: int, what: str = "") -> None:
    """Raise the exception type matching a nonzero status."""
    if status == SC_OK:
        return
    lib = load()
    msg = (lib.sc_last_error() or b"").decode(errors="replace")
    name = (lib.sc_status_name(status) or b"").decode()
    text = f"{what}: {name}: {msg}" if what else f"{name}: {msg}"
    if status in (SC_ERR_SHAPE, SC_ERR_ARG, SC_ERR_WORKSPACE):
        raise ValueError(text)
    if status == SC_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    if status == SC_ERR_TIMEOUT:
        raise TimeoutError(text)
    raise ScError(text)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def last_error() -> str:
    """The library's message for the last failure on this thread."""
    return (load().sc_last_error() or b"").decode(errors="replace")
