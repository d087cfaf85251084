"""Tensor-level wrappers over the C ABI (torch tensors are only handles).

Every function checks devices, dtypes and shapes on the host, passes raw
pointers plus the current CUDA stream to ``libsc_b200.so`` and raises the
reference's exception types on failure.  All tensors must live on a CUDA
device; there is no CPU path.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Optional, Sequence

import torch

from . import _lib as L

_F16, _F32 = torch.float16, torch.float32


def _dt(t: torch.Tensor) -> int:
    if t.dtype == _F16:
        return L.SC_F16
    if t.dtype == _F32:
        return L.SC_F32
    if t.dtype == torch.int32:
        return L.SC_I32
    raise ValueError(f"unsupported dtype {t.dtype}")


def _cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("libsc_b200 ops take CUDA tensors only (no CPU path)")


def _f32_cache(*ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != torch.float32:
            raise ValueError(f"KV cache must be float32 (the reference caches fp32 keys/values), got {t.dtype}")


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def stream_handle(device: Optional[torch.device] = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def as_u32(t: torch.Tensor) -> torch.Tensor:
    """Packed words are handled as 4-byte storage; int32/uint32 both accepted."""
    if t.dtype in (torch.int32, getattr(torch, "uint32", torch.int32)):
        return t
    raise ValueError(f"packed weights must be uint32/int32, got {t.dtype}")


class Workspace:
    """Grow-only device scratch buffer, one per device.

    Sized before a CUDA graph capture so the captured pointer stays valid.
    """

    _bufs: dict = {}

    @classmethod
    def get(cls, nbytes: int, device: torch.device) -> Optional[torch.Tensor]:
        if nbytes <= 0:
            return None
        key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
        buf = cls._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            cls._bufs[key] = buf
        return buf


# ---------------------------------------------------------------- K1

def qlinear_workspace_bytes(M: int, K: int, N: int, bits: int) -> int:
    return int(L.load().sc_qlinear_workspace_bytes(M, K, N, bits))


def qlinear(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int,
            bits: int, bias: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ dequant(wq, scales, biases).T (+ bias)`` — mx.quantized_matmul(transpose=True)."""
    _cuda(x, wq, scales, biases, bias, out)
    wq = as_u32(wq)
    K = x.shape[-1]
    N = wq.shape[0]
    if wq.shape[1] * (32 // bits) != K:
        raise ValueError(f"weight packs {wq.shape[1] * (32 // bits)} inputs, x has {K}")
    if scales.shape != (N, K // group_size) or biases.shape != scales.shape:
        raise ValueError(f"scales {tuple(scales.shape)} / biases {tuple(biases.shape)} do not match "
                         f"[{N}, {K // group_size}]")
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = out if out is not None else torch.empty(M, N, dtype=out_dtype or x.dtype, device=x.device)
    ws_bytes = qlinear_workspace_bytes(M, K, N, bits)
    ws = Workspace.get(ws_bytes, x.device)
    L.call("sc_qlinear", _p(x2), _dt(x2), M, K, K, _p(wq), _p(scales), _p(biases), N, group_size, bits,
           _p(bias), _p(y), _dt(y), N, _p(ws), ws_bytes, stream_handle(x.device))
    return y.reshape(*x.shape[:-1], N)


def qlinear_fused(x: torch.Tensor, segments: Sequence, group_size: int, bits: int, epilogue: int = L.SC_EPI_STORE,
                  norm_weight: Optional[torch.Tensor] = None, eps: float = 1e-5,
                  bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = _F32) -> torch.Tensor:
    """Fused RMSNorm -> segments of quantized linears -> epilogue.

    ``segments`` is a list of ``(wq, scales, biases)`` sharing ``x``.
    """
    _cuda(x, norm_weight, bias, residual, out)
    n = len(segments)
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    rows = [int(s[0].shape[0]) for s in segments]
    N = rows[0] if epilogue == L.SC_EPI_SWIGLU else sum(rows)
    for wq, sc, bi in segments:
        _cuda(wq, sc, bi)
        if wq.shape[1] * (32 // bits) != K:
            raise ValueError("segment K mismatch")
    y = out if out is not None else torch.empty(M, N, dtype=out_dtype, device=x.device)
    W = (C.c_void_p * n)(*[s[0].data_ptr() for s in segments])
    S = (C.c_void_p * n)(*[s[1].data_ptr() for s in segments])
    B = (C.c_void_p * n)(*[s[2].data_ptr() for s in segments])
    R = (C.c_int * n)(*rows)
    ws_bytes = qlinear_workspace_bytes(M, K, N, bits)
    ws = Workspace.get(ws_bytes, x.device)
    res = residual.reshape(-1, N) if residual is not None else None
    L.call("sc_qlinear_fused", _p(x2), _dt(x2), M, K, K, _p(norm_weight), float(eps), n,
           C.cast(W, L._pp), C.cast(S, L._pp), C.cast(B, L._pp), R, group_size, bits, _p(bias), epilogue,
           _p(y), _dt(y), N, _p(res), N if res is not None else 0, _p(ws), ws_bytes, stream_handle(x.device))
    return y


# ---------------------------------------------------------------- K3

def embed_gather_q(ids: torch.Tensor, wq, scales, biases, vocab_start: int, vocab_end: int, hidden: int,
                   group_size: int, bits: int, out_dtype=_F16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _cuda(ids, wq, scales, biases, out)
    if wq.shape[0] < vocab_end - vocab_start or scales.shape[0] < vocab_end - vocab_start:
        raise ValueError(f"table has {wq.shape[0]} rows, vocab range needs {vocab_end - vocab_start}")
    if wq.shape[1] * (32 // bits) != hidden:
        raise ValueError(f"table packs {wq.shape[1] * (32 // bits)} values per row, hidden is {hidden}")
    ids32 = ids.reshape(-1).to(torch.int32).contiguous()
    n = ids32.numel()
    y = out if out is not None else torch.empty(n, hidden, dtype=out_dtype, device=ids.device)
    L.call("sc_embed_gather_q", _p(ids32), n, _p(as_u32(wq)), _p(scales), _p(biases), vocab_start, vocab_end,
           hidden, group_size, bits, _p(y), _dt(y), stream_handle(ids.device))
    return y.reshape(*ids.shape, hidden)


def embed_gather_f16(ids: torch.Tensor, table: torch.Tensor, vocab_start: int, vocab_end: int,
                     out_dtype=_F16) -> torch.Tensor:
    _cuda(ids, table)
    if table.shape[0] < vocab_end - vocab_start:
        raise ValueError(f"table has {table.shape[0]} rows, vocab range needs {vocab_end - vocab_start}")
    ids32 = ids.reshape(-1).to(torch.int32).contiguous()
    H = table.shape[1]
    y = torch.empty(ids32.numel(), H, dtype=out_dtype, device=ids.device)
    L.call("sc_embed_gather_f16", _p(ids32), ids32.numel(), _p(table), vocab_start, vocab_end, H, _p(y), _dt(y),
           stream_handle(ids.device))
    return y.reshape(*ids.shape, H)


def dequantize(wq, scales, biases, group_size: int, bits: int) -> torch.Tensor:
    _cuda(wq, scales, biases)
    rows = wq.shape[0]
    K = wq.shape[1] * (32 // bits)
    out = torch.empty(rows, K, dtype=_F16, device=wq.device)
    L.call("sc_dequantize", _p(as_u32(wq)), _p(scales), _p(biases), rows, K, group_size, bits, _p(out),
           stream_handle(wq.device))
    return out


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """fp16 [rows, K] -> (wq int32 [rows, K*bits/32], scales fp16, biases fp16)."""
    _cuda(w)
    w = w.to(_F16).contiguous()
    rows, K = w.shape
    wq = torch.empty(rows, K * bits // 32, dtype=torch.int32, device=w.device)
    s = torch.empty(rows, K // group_size, dtype=_F16, device=w.device)
    b = torch.empty_like(s)
    L.call("sc_quantize", _p(w), rows, K, group_size, bits, _p(wq), _p(s), _p(b), stream_handle(w.device))
    return wq, s, b


# ---------------------------------------------------------------- K4

def rope_append(qkv: torch.Tensor, B: int, S: int, Hq: int, Hkv: int, hd: int, pos: torch.Tensor,
                cos_tab: torch.Tensor, sin_tab: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor) -> None:
    _cuda(qkv, pos, cos_tab, sin_tab, q_out, k_cache, v_cache)
    _f32_cache(k_cache, v_cache)
    Lmax = k_cache.shape[2]
    L.call("sc_rope_append", _p(qkv), B, S, Hq, Hkv, hd, _p(pos), _p(cos_tab), _p(sin_tab), cos_tab.shape[0],
           _p(q_out), _p(k_cache), _p(v_cache), Lmax, stream_handle(qkv.device))


def flash_decode_workspace_bytes(B: int, S: int, Hq: int, hd: int, splits: int) -> int:
    return int(L.load().sc_flash_decode_workspace_bytes(B, S, Hq, hd, splits))


def flash_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor, B: int, S: int,
                 Hq: int, Hkv: int, hd: int, splits: int, out: torch.Tensor,
                 workspace: Optional[torch.Tensor] = None, scale: Optional[float] = None) -> torch.Tensor:
    _cuda(q, k_cache, v_cache, pos, out)
    _f32_cache(k_cache, v_cache)
    nbytes = flash_decode_workspace_bytes(B, S, Hq, hd, splits)
    if workspace is None:
        workspace = Workspace.get(nbytes, q.device)
    sc = (1.0 / math.sqrt(hd)) if scale is None else scale
    L.call("sc_flash_decode", _p(q), _p(k_cache), _p(v_cache), _p(pos), B, S, Hq, Hkv, hd, k_cache.shape[2],
           float(sc), splits, _p(out), _dt(out), _p(workspace), nbytes if workspace is not None else 0,
           stream_handle(q.device))
    return out


def attn_decode_workspace_bytes(B: int, Hq: int, hd: int, splits: int) -> int:
    return int(L.load().sc_attn_decode_workspace_bytes(B, Hq, hd, splits))


def attn_decode(qkv: torch.Tensor, B: int, Hq: int, Hkv: int, hd: int, pos: torch.Tensor, cos_tab: torch.Tensor,
                sin_tab: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, splits: int, out: torch.Tensor,
                tickets: torch.Tensor, workspace: Optional[torch.Tensor] = None,
                scale: Optional[float] = None) -> torch.Tensor:
    """One decode token per sequence: RoPE + KV append + split-KV attention
    (+ merge) in one launch.  ``tickets`` is int32 [B*Hkv], zero on entry
    and left zero."""
    _cuda(qkv, pos, cos_tab, sin_tab, k_cache, v_cache, out, tickets, workspace)
    _f32_cache(k_cache, v_cache)
    nbytes = attn_decode_workspace_bytes(B, Hq, hd, splits)
    if workspace is None:
        workspace = Workspace.get(nbytes, qkv.device)
    sc = (1.0 / math.sqrt(hd)) if scale is None else scale
    L.call("sc_attn_decode", _p(qkv), B, Hq, Hkv, hd, _p(pos), _p(cos_tab), _p(sin_tab), cos_tab.shape[0],
           _p(k_cache), _p(v_cache), k_cache.shape[2], float(sc), splits, _p(out), _dt(out), _p(workspace),
           nbytes if workspace is not None else 0, _p(tickets), stream_handle(qkv.device))
    return out


# ---------------------------------------------------------------- K5 / K7

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    _cuda(x, w)
    H = x.shape[-1]
    x2 = x.reshape(-1, H).contiguous()
    y = torch.empty(x2.shape, dtype=out_dtype or x.dtype, device=x.device)
    L.call("sc_rmsnorm", _p(x2), _dt(x2), x2.shape[0], H, _p(w.to(_F16).contiguous()), float(eps), _p(y), _dt(y),
           stream_handle(x.device))
    return y.reshape(x.shape)


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    _cuda(gate, up)
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError("gate/up shape or dtype mismatch")
    g, u = gate.contiguous(), up.contiguous()
    y = torch.empty(g.shape, dtype=out_dtype or g.dtype, device=g.device)
    L.call("sc_silu_mul", _p(g), _p(u), _dt(g), g.numel(), _p(y), _dt(y), stream_handle(g.device))
    return y


def add(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
        out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    _cuda(a, b, out)
    if a.shape != b.shape:
        raise ValueError(f"add: shapes {tuple(a.shape)} vs {tuple(b.shape)}")
    a, b = a.contiguous(), b.contiguous()
    y = out if out is not None else torch.empty(a.shape, dtype=out_dtype or torch.promote_types(a.dtype, b.dtype),
                                                device=a.device)
    L.call("sc_add", _p(a), _dt(a), _p(b), _dt(b), a.numel(), _p(y), _dt(y), stream_handle(a.device))
    return y


def argmax_workspace_bytes(M: int, N: int) -> int:
    return int(L.load().sc_argmax_workspace_bytes(M, N))


def argmax(logits: torch.Tensor, index_offset: int = 0, val: Optional[torch.Tensor] = None,
           idx: Optional[torch.Tensor] = None):
    """Per-row (max value, lowest index of it + offset) of fp32 logits [M, N]."""
    _cuda(logits)
    if logits.dtype != _F32:
        logits = logits.float()
    N = logits.shape[-1]
    lg = logits.reshape(-1, N).contiguous()
    M = lg.shape[0]
    val = val if val is not None else torch.empty(M, dtype=_F32, device=lg.device)
    idx = idx if idx is not None else torch.empty(M, dtype=torch.int32, device=lg.device)
    nb = argmax_workspace_bytes(M, N)
    ws = Workspace.get(nb, lg.device)
    L.call("sc_argmax", _p(lg), M, N, N, index_offset, _p(val), _p(idx), _p(ws), nb, stream_handle(lg.device))
    return val, idx


def argmax_merge(vals: torch.Tensor, idxs: torch.Tensor, world: int, token_out: torch.Tensor,
                 pos: Optional[torch.Tensor] = None, pos_advance: int = 0) -> torch.Tensor:
    _cuda(vals, idxs, token_out, pos)
    M = token_out.numel()
    L.call("sc_argmax_merge", _p(vals), _p(idxs), M, world, _p(token_out), _p(pos), pos_advance,
           stream_handle(vals.device))
    return token_out


# ---------------------------------------------------------------- K7b: temperature + top-p sampling

_ST_N, _ST_MAX, _ST_Z, _ST_KEPT, _ST_TOKEN = 8, 0, 1, 4, 7


def sample_workspace_bytes(B: int) -> int:
    return int(L.load().sc_sample_workspace_bytes(B))


def sample_uniforms(seed: int, counter: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """Fill ``u`` (float32 [B]) with uniforms from (seed, the int64 device
    ``counter``), advancing the counter on the device (capturable)."""
    _cuda(counter, u)
    if counter.dtype != torch.int64 or u.dtype != torch.float32:
        raise ValueError("counter must be int64 and u float32")
    L.call("sc_sample_uniforms", C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), _p(counter), u.numel(), _p(u),
           stream_handle(u.device))
    return u


def sample_topp(logits: torch.Tensor, temperature: float, top_p: float, u: torch.Tensor, tok: torch.Tensor,
                comm=None, vocab_start: int = 0, workspace: Optional[torch.Tensor] = None,
                gather: Optional[torch.Tensor] = None):
    """Temperature + top-p draw from ``logits`` (float32 [B, V_local]) into
    ``tok`` (int32 [B]) -- the sampled branch of the reference's generate
    (worker/executor.py:270-306).  ``comm`` (tensor parallel): each rank
    passes its vocab slice and the ranks exchange only per-row scalars and
    256-bin histograms (all-gather / all-reduce on the current stream), never
    the logits; every rank ends with the same token in ``tok`` (global ids).
    ``tok`` keeps its value for a row whose draw found no token."""
    _cuda(logits, u, tok, workspace, gather)
    if logits.dtype != torch.float32 or logits.dim() != 2 or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous float32 [B, V] tensor")
    if temperature <= 0.0 or top_p <= 0.0:
        raise ValueError("temperature and top_p must be positive (temperature 0 is the greedy argmax)")
    B, V = logits.shape
    nbytes = sample_workspace_bytes(B)
    if workspace is None:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=logits.device)
    stream = stream_handle(logits.device)
    ws = workspace.data_ptr()
    world = 1 if comm is None else comm.world_size
    if world == 1:
        L.call("sc_sample_topp", _p(logits), B, V, V, float(temperature), float(top_p), _p(u), int(vocab_start),
               _p(tok), ws, nbytes, stream)
        return tok
    rank = comm.rank
    st = workspace[: _ST_N * B * 4].view(torch.float32).view(_ST_N, B)
    hist = workspace[_ST_N * B * 4: nbytes].view(torch.float32)
    if gather is None:
        gather = torch.empty(world, B, dtype=torch.float32, device=logits.device)

    def phase(ph, level=0):
        L.call("sc_sample_phase", _p(logits), B, V, V, float(temperature), float(top_p), _p(u), int(vocab_start), ph,
               level, ws, nbytes, stream)

    phase(0)
    comm.allgather_into(st[_ST_MAX], gather)
    L.call("sc_sample_combine", ws, _p(gather), B, world, rank, 0, None, stream)
    phase(1)
    comm.allreduce_into(st[_ST_Z], st[_ST_Z], "sum")
    for level in range(4):
        phase(2, level)
        comm.allreduce_into(hist, hist, "sum")
        phase(3, level)
    phase(4)
    comm.allgather_into(st[_ST_KEPT], gather)
    L.call("sc_sample_combine", ws, _p(gather), B, world, rank, 1, None, stream)
    phase(5)
    comm.allreduce_into(st[_ST_TOKEN], st[_ST_TOKEN], "sum")
    L.call("sc_sample_combine", ws, None, B, world, rank, 2, _p(tok), stream)
    return tok
