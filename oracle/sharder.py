"""Shard layout of the reference's ``WeightSharder`` (test oracle only).

Restates ``model/sharder.py:51-98`` (``shard_weights``), ``:100-180``
(``_shard_quantized_weight``) and ``:182-255`` (``_shard_weight``) so the
product's layout writer and loader can be checked against it.

Quantized triples (``X.weight`` uint32 ``[out, in*bits/32]`` plus ``X.scales`` /
``X.biases`` ``[out, in/g]``) are split:

* column layers (q/k/v/up/gate, and embed_tokens / lm_head, which are therefore
  vocab-split): dim 0 of all three (:134-138);
* row layers (o_proj / down_proj): dim 1 of all three; scales/biases are
  replicated when their dim 1 does not divide by world size (:139-161);
* anything else: replicated (:162-167).

Unquantized tensors follow ``_shard_weight``: 1-D and ``bias`` tensors are
replicated; HF ``[out, in]`` linears are transposed to ``[in, out]`` then
column-split on dim 1 (q/k/v/up/gate, lm_head) or row-split on dim 0
(o_proj, down_proj); embed_tokens is split on dim 1 (hidden) without a
transpose; norms are replicated.
"""

from __future__ import annotations

import numpy as np

_COLUMN_Q = ("q_proj", "k_proj", "v_proj", "query", "key", "value",
             "up_proj", "gate_proj", "fc1", "w1", "w3", "embed_tokens", "wte", "lm_head")


def _is_row_parallel_q(name: str) -> bool:
    # model/sharder.py:127-131: for o_proj/out_proj names the test is
    # "any row marker and 'mlp' not in name"; otherwise down_proj/fc2/w2.
    if "o_proj" in name or "out_proj" in name:
        return any(x in name for x in ("o_proj", "out_proj", "down_proj", "fc2", "w2")) and "mlp" not in name.lower()
    return any(x in name for x in ("down_proj", "fc2", "w2"))


def _split(a: np.ndarray, world: int, rank: int, dim: int) -> np.ndarray:
    if a.ndim == 1:
        return a.copy()
    size = a.shape[dim] // world
    sl = [slice(None)] * a.ndim
    sl[dim] = slice(rank * size, (rank + 1) * size)
    return a[tuple(sl)].copy()


def shard_quantized(name: str, w, s, b, world: int, rank: int):
    if any(x in name for x in _COLUMN_Q):
        return _split(w, world, rank, 0), _split(s, world, rank, 0), _split(b, world, rank, 0)
    if _is_row_parallel_q(name):
        sw = _split(w, world, rank, 1)
        ss = _split(s, world, rank, 1) if s.ndim > 1 and s.shape[1] % world == 0 else s.copy()
        sb = _split(b, world, rank, 1) if b.ndim > 1 and b.shape[1] % world == 0 else b.copy()
        return sw, ss, sb
    return w.copy(), s.copy(), b.copy()


def shard_dense(name: str, w: np.ndarray, world: int, rank: int) -> np.ndarray:
    if w.ndim == 1 or "bias" in name.lower():
        return w.copy()
    if "embed_tokens" in name or "wte" in name:
        return _split(w, world, rank, 1)
    if "lm_head" in name:
        return _split(w.T, world, rank, 1)
    if any(x in name for x in ("q_proj", "k_proj", "v_proj", "query", "key", "value")):
        return _split(w.T, world, rank, 1)
    if any(x in name for x in ("o_proj", "out_proj", "dense")) and "mlp" not in name.lower():
        return _split(w.T, world, rank, 0)
    if any(x in name for x in ("up_proj", "gate_proj", "fc1", "w1", "w3")):
        return _split(w.T, world, rank, 1)
    if any(x in name for x in ("down_proj", "fc2", "w2")):
        return _split(w.T, world, rank, 0)
    return w.copy()


def shard_weights(weights: dict, world: int, rank: int) -> dict:
    """``WeightSharder.shard_weights`` (model/sharder.py:51-98)."""
    out = {}
    done = set()
    for name, w in weights.items():
        if name in done:
            continue
        sk = name.replace(".weight", ".scales") if ".weight" in name else f"{name}.scales"
        bk = name.replace(".weight", ".biases") if ".weight" in name else f"{name}.biases"
        if sk in weights and bk in weights:
            sw, ss, sb = shard_quantized(name, w, weights[sk], weights[bk], world, rank)
            wk = name if ".weight" in name else f"{name}.weight"
            out[wk], out[sk], out[bk] = sw, ss, sb
            done.update((sk, bk))
        elif name.endswith(".scales") or name.endswith(".biases"):
            continue
        else:
            out[name] = shard_dense(name, w, world, rank)
    return out
