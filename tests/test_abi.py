"""The C ABI: libsc_b200.so loads, exports every symbol include/sc_b200.h
declares, and the binding's signature table matches the header.  Only
host-side entry points (no GPU work) are called here."""

import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sc_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    names = re.findall(r"\b(sc_[a-z0-9_]+)\s*\(", src)
    return sorted(set(names))


def test_header_declares_the_path():
    names = header_functions()
    for must in ("sc_qlinear", "sc_qlinear_fused", "sc_embed_gather_q", "sc_embed_gather_f16", "sc_flash_decode",
                 "sc_rope_append", "sc_argmax", "sc_argmax_merge", "sc_allreduce", "sc_allgather", "sc_comm_init"):
        assert must in names


def test_library_loads_and_exports_every_declared_symbol():
    from shardcompute_b200 import _lib

    lib = _lib.load()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_table_matches_header():
    from shardcompute_b200 import _lib

    assert sorted(_lib.SIGNATURES) == header_functions()


def test_exported_symbols_are_c_linkage():
    from shardcompute_b200 import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    for n in header_functions():
        assert n in exported, f"{n} missing or C++-mangled"


def test_host_only_entry_points():
    from shardcompute_b200 import _lib

    lib = _lib.load()
    assert lib.sc_abi_version() == _lib.ABI_VERSION
    assert lib.sc_status_name(_lib.SC_ERR_SHAPE) == b"SC_ERR_SHAPE"
    # workspace sizing is pure host arithmetic: bounded, zero for invalid shapes
    assert lib.sc_qlinear_workspace_bytes(0, 4096, 4096, 4) == 0
    assert lib.sc_qlinear_workspace_bytes(1, 4096, 14336, 3) == 0
    ws = lib.sc_qlinear_workspace_bytes(16, 14336, 4096, 4)
    assert 0 <= ws <= 64 * 16 * 4096 * 4 * 2
    assert lib.sc_flash_decode_workspace_bytes(1, 1, 32, 128, 1) >= 0
    assert lib.sc_argmax_workspace_bytes(1, 128256) > 0


def test_errors_map_to_reference_exception_types():
    from shardcompute_b200 import _lib

    with pytest.raises(ValueError):
        _lib.check(_lib.SC_ERR_SHAPE, "x")
    with pytest.raises(TimeoutError):
        _lib.check(_lib.SC_ERR_TIMEOUT, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.SC_ERR_CUDA, "x")
    _lib.check(_lib.SC_OK)


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: every op demands CUDA tensors."""
    import torch

    from shardcompute_b200 import ops

    x = torch.zeros(1, 64, dtype=torch.float16)
    wq = torch.zeros(8, 8, dtype=torch.int32)
    s = torch.zeros(8, 1, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.qlinear(x, wq, s, s, 64, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.embed_gather_q(torch.zeros(3, dtype=torch.int32), wq, s, s, 0, 8, 64, 64, 4)
