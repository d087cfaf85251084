"""MLX group-wise affine quantization, restated in numpy (test oracle only).

The reference never implements this arithmetic itself; it calls MLX:

* ``mx.quantize``          parallel/quantized_linear.py:116,353; parallel/embedding.py:303
* ``mx.dequantize``        parallel/embedding.py:343-349,373-379
* ``mx.quantized_matmul``  parallel/quantized_linear.py:168-176,206-214,435-443,472-480

On-disk format (MLX's published affine format):

* ``wq``     uint32 ``[rows, K*bits/32]``; element j of a word sits at bits
  ``[bits*j, bits*(j+1))`` (little-endian packing).
* ``scales`` and ``biases``: ``[rows, K/group_size]`` (fp16 in every shard the
  reference loads).
* dequant: ``w_hat = scale*q + bias``.  The comment at
  parallel/embedding.py:342 ("(quantized - bias) * scale") is wrong; the
  reference's own docs (PIPELINE_PARALLELISM_PLAN.md:64-67,
  debug_quantization_error.md:20-29) state ``scale*q + bias``.

Rounding contract used by this build:

* ``dequantize``: the exact value ``s*q + b`` rounded ONCE to fp16 (the output
  dtype is the scales' dtype).  Computed here in float64, where ``s*q + b`` of
  fp16 operands is exact, then cast.
* ``quantized_matmul``: ``x @ (s*q + b).T`` with the dequantized weight kept
  exact (no fp16 rounding), accumulated in float64.  MLX accumulates
  ``scale*sum(x*q) + bias*sum(x)`` per group in fp32, which is the same value
  up to fp32 rounding.
"""

from __future__ import annotations

import numpy as np

SUPPORTED_BITS = (4, 8)
SUPPORTED_GROUPS = (32, 64, 128)


def pack_factor(bits: int) -> int:
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"bits must be one of {SUPPORTED_BITS}, got {bits}")
    return 32 // bits


def pack(q: np.ndarray, bits: int) -> np.ndarray:
    """Pack integer codes ``q[..., K]`` (values < 2**bits) into uint32 words."""
    pf = pack_factor(bits)
    q = np.asarray(q, dtype=np.uint64)
    if q.shape[-1] % pf:
        raise ValueError(f"last dim {q.shape[-1]} not a multiple of {pf}")
    if q.size and int(q.max()) >= (1 << bits):
        raise ValueError("code out of range")
    q = q.reshape(*q.shape[:-1], q.shape[-1] // pf, pf)
    shifts = (np.arange(pf, dtype=np.uint64) * bits)
    words = np.bitwise_or.reduce(q << shifts, axis=-1)
    return words.astype(np.uint32)


def unpack(wq: np.ndarray, bits: int) -> np.ndarray:
    """Inverse of :func:`pack`: uint32 ``[..., W]`` -> uint8 codes ``[..., W*pf]``."""
    pf = pack_factor(bits)
    w = np.asarray(wq, dtype=np.uint32).astype(np.uint64)
    shifts = (np.arange(pf, dtype=np.uint64) * bits)
    mask = np.uint64((1 << bits) - 1)
    q = (w[..., None] >> shifts) & mask
    return q.reshape(*w.shape[:-1], w.shape[-1] * pf).astype(np.uint8)


def _expand_groups(a: np.ndarray, group_size: int) -> np.ndarray:
    return np.repeat(np.asarray(a), group_size, axis=-1)


def dequantize_exact(wq, scales, biases, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """``s*q + b`` in float64 with no rounding (fp16 operands make it exact)."""
    q = unpack(wq, bits).astype(np.float64)
    s = _expand_groups(np.asarray(scales, dtype=np.float64), group_size)
    b = _expand_groups(np.asarray(biases, dtype=np.float64), group_size)
    if s.shape != q.shape:
        raise ValueError(f"scales {np.shape(scales)} do not match codes {q.shape} at group {group_size}")
    return s * q + b


def dequantize(wq, scales, biases, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """``mx.dequantize`` restated: exact ``s*q + b`` rounded once to fp16."""
    return dequantize_exact(wq, scales, biases, group_size, bits).astype(np.float16)


def quantize(w, group_size: int = 64, bits: int = 4):
    """Affine min/max quantization per group (offline data prep).

    Per group: ``b = min``, ``s = (max - min) / (2**bits - 1)`` (both stored
    as fp16), ``q = clip(rint((w - b16) / s16), 0, 2**bits - 1)`` computed in
    float64 against the stored fp16 values.  A constant group gets ``s = 0``
    and ``q = 0``.
    """
    w = np.asarray(w, dtype=np.float32)
    K = w.shape[-1]
    if group_size not in SUPPORTED_GROUPS:
        raise ValueError(f"group_size must be one of {SUPPORTED_GROUPS}")
    if K % group_size:
        raise ValueError(f"K={K} not a multiple of group_size={group_size}")
    n_bins = (1 << bits) - 1
    g = w.reshape(-1, K // group_size, group_size).astype(np.float64)
    wmin = g.min(axis=-1)
    wmax = g.max(axis=-1)
    s16 = ((wmax - wmin) / n_bins).astype(np.float16)
    b16 = wmin.astype(np.float16)
    s = s16.astype(np.float64)[..., None]
    b = b16.astype(np.float64)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s > 0, np.rint((g - b) / np.where(s > 0, s, 1.0)), 0.0)
    q = np.clip(q, 0, n_bins).astype(np.uint8).reshape(*w.shape)
    out_shape = w.shape[:-1] + (K // group_size,)
    return pack(q, bits), s16.reshape(out_shape), b16.reshape(out_shape)


def quantized_matmul(x, wq, scales, biases, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """``mx.quantized_matmul(x, w, s, b, transpose=True)``: ``x @ dequant(w).T`` (float64)."""
    w = dequantize_exact(wq, scales, biases, group_size, bits)
    return np.asarray(x, dtype=np.float64) @ w.T


def gemv_bytes(M: int, K: int, N: int, bits: int, group_size: int = 64,
               x_bytes: int = 2, y_bytes: int = 2) -> int:
    """Algorithmic HBM bytes of one dequant-matmul: packed weights + fp16
    scale/bias per group + activations in + activations out."""
    return K * N * bits // 8 + (K // group_size) * N * 2 * 2 + M * K * x_bytes + M * N * y_bytes
