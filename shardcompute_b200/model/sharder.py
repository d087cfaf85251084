"""Shard layout writer/reader, format-identical to the reference's WeightSharder.

Output directory (``model/sharder.py:318-364`` of the reference)::

    shard_dir/config.json                {"model": {...}, "parallel": {...}}
    shard_dir/rank_{r}/model.safetensors HF tensor names, per-rank slices
    shard_dir/rank_{r}/metadata.json     rank, world_size, num_tensors, tensor_shapes

Split rules (``_shard_quantized_weight`` :100-180, ``_shard_weight`` :182-255):
quantized ``X.weight/.scales/.biases`` triples of column layers (q/k/v/up/gate
and embed_tokens/lm_head, i.e. vocab-split) are sliced on dim 0, row layers
(o_proj/down_proj) on dim 1; unquantized HF ``[out, in]`` linears are
transposed to ``[in, out]`` then column-split on dim 1 or row-split on dim 0;
an unquantized embedding is split on its hidden dim; 1-D tensors and norms
are replicated.
"""

from __future__ import annotations

import json
import logging
from pathlib import Path
from typing import Dict, Tuple

import numpy as np

from .config import ModelConfig, ParallelConfig

logger = logging.getLogger(__name__)

COLUMN_MARKERS = ("q_proj", "k_proj", "v_proj", "query", "key", "value", "up_proj", "gate_proj", "fc1", "w1",
                  "w3", "embed_tokens", "wte", "lm_head")


def _row_parallel_quantized(name: str) -> bool:
    if "o_proj" in name or "out_proj" in name:
        return "mlp" not in name.lower()
    return any(x in name for x in ("down_proj", "fc2", "w2"))


def _slice(a: np.ndarray, world: int, rank: int, dim: int) -> np.ndarray:
    if a.ndim == 1:
        return a.copy()
    n = a.shape[dim] // world
    idx = [slice(None)] * a.ndim
    idx[dim] = slice(rank * n, (rank + 1) * n)
    return np.ascontiguousarray(a[tuple(idx)])


class WeightSharder:
    """Tensor-parallel sharder (reference ``model/sharder.py:17-401``)."""

    def __init__(self, model_config: ModelConfig, parallel_config: ParallelConfig):
        parallel_config.validate(model_config)
        self.model_config = model_config
        self.parallel_config = parallel_config
        self.world_size = parallel_config.tensor_parallel_size

    def shard_weights(self, weights: Dict[str, np.ndarray], rank: int) -> Dict[str, np.ndarray]:
        out: Dict[str, np.ndarray] = {}
        consumed = set()
        for name, w in weights.items():
            if name in consumed:
                continue
            sk = name.replace(".weight", ".scales") if ".weight" in name else f"{name}.scales"
            bk = name.replace(".weight", ".biases") if ".weight" in name else f"{name}.biases"
            if sk in weights and bk in weights:
                out.update(self._shard_quantized(name, w, weights[sk], weights[bk], rank))
                consumed.update((sk, bk))
            elif name.endswith(".scales") or name.endswith(".biases"):
                continue
            else:
                out[name] = self._shard_dense(name, w, rank)
        return out

    def _shard_quantized(self, name, w, s, b, rank) -> Dict[str, np.ndarray]:
        W = self.world_size
        if any(x in name for x in COLUMN_MARKERS):
            sw, ss, sb = _slice(w, W, rank, 0), _slice(s, W, rank, 0), _slice(b, W, rank, 0)
        elif _row_parallel_quantized(name):
            sw = _slice(w, W, rank, 1)
            ss = _slice(s, W, rank, 1) if s.ndim > 1 and s.shape[1] % W == 0 else s.copy()
            sb = _slice(b, W, rank, 1) if b.ndim > 1 and b.shape[1] % W == 0 else b.copy()
        else:
            logger.warning("Unknown quantized weight %s, replicating", name)
            sw, ss, sb = w.copy(), s.copy(), b.copy()
        wk = name if ".weight" in name else f"{name}.weight"
        return {wk: sw, wk.replace(".weight", ".scales"): ss, wk.replace(".weight", ".biases"): sb}

    def _shard_dense(self, name: str, w: np.ndarray, rank: int) -> np.ndarray:
        W = self.world_size
        if w.ndim == 1 or "bias" in name.lower():
            return w.copy()
        if "embed_tokens" in name or "wte" in name:
            return _slice(w, W, rank, 1)
        if "lm_head" in name:
            return _slice(w.T, W, rank, 1)
        if any(x in name for x in ("q_proj", "k_proj", "v_proj", "query", "key", "value")):
            return _slice(w.T, W, rank, 1)
        if any(x in name for x in ("o_proj", "out_proj", "dense")) and "mlp" not in name.lower():
            return _slice(w.T, W, rank, 0)
        if any(x in name for x in ("up_proj", "gate_proj", "fc1", "w1", "w3")):
            return _slice(w.T, W, rank, 1)
        if any(x in name for x in ("down_proj", "fc2", "w2")):
            return _slice(w.T, W, rank, 0)
        return w.copy()

    def save_shards(self, weights: Dict[str, np.ndarray], output_dir: str) -> None:
        from safetensors.numpy import save_file

        out = Path(output_dir)
        out.mkdir(parents=True, exist_ok=True)
        cfg = {"model": self.model_config.to_dict(),
               "parallel": {"world_size": self.world_size,
                            "tensor_parallel_size": self.parallel_config.tensor_parallel_size}}
        with open(out / "config.json", "w") as f:
            json.dump(cfg, f, indent=2)
        for rank in range(self.world_size):
            rd = out / f"rank_{rank}"
            rd.mkdir(exist_ok=True)
            sh = self.shard_weights(weights, rank)
            save_file(sh, str(rd / "model.safetensors"))
            meta = {"rank": rank, "world_size": self.world_size, "num_tensors": len(sh),
                    "tensor_shapes": {k: list(v.shape) for k, v in sh.items()}}
            with open(rd / "metadata.json", "w") as f:
                json.dump(meta, f, indent=2)

    @staticmethod
    def load_shards(shard_dir: str, rank: int) -> Tuple[Dict[str, np.ndarray], Dict]:
        from safetensors.numpy import load_file

        rd = Path(shard_dir) / f"rank_{rank}"
        if not rd.exists():
            raise FileNotFoundError(f"Shard directory not found: {rd}")
        with open(rd / "metadata.json") as f:
            meta = json.load(f)
        return load_file(str(rd / "model.safetensors")), meta
