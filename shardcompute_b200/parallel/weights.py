"""Per-rank device weights of a quantized, tied-embedding Llama.

Built from a shard dictionary in the reference's layout (HF tensor names,
``model/sharder.py`` split rules) -- loaded from ``rank_{r}/model.safetensors``
or produced in memory -- or generated directly on the GPU for synthetic
benchmarks (random N(0, 0.02) fp16 weights quantized by ``sc_quantize``).

Packed words are kept as int32 storage (same bytes as the shards' uint32);
scales/biases/norms stay fp16; nothing is repacked, so the kernels read the
MLX layout exactly as the reference stores it.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..model.config import ModelConfig

QTriple = Tuple[torch.Tensor, torch.Tensor, torch.Tensor]


def _dev_words(a, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        t = a
        if t.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
            raise ValueError(f"packed weights must be 32-bit, got {t.dtype}")
        return t.view(torch.int32).to(device).contiguous()
    a = np.ascontiguousarray(a)
    if a.dtype not in (np.uint32, np.int32):
        raise ValueError(f"packed weights must be uint32, got {a.dtype}")
    return torch.from_numpy(a.view(np.int32)).to(device)


def _dev_f16(a, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=torch.float16).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).to(device)


@dataclass
class LayerWeights:
    ln1: torch.Tensor
    ln2: torch.Tensor
    q: QTriple
    k: QTriple
    v: QTriple
    o: QTriple
    gate: QTriple
    up: QTriple
    down: QTriple


@dataclass
class RankWeights:
    cfg: ModelConfig
    world: int
    rank: int
    bits: int
    group: int
    embed: QTriple
    norm: torch.Tensor
    layers: List[LayerWeights] = field(default_factory=list)

    @property
    def vocab_start(self) -> int:
        return self.rank * (self.cfg.vocab_size // self.world)

    @property
    def vocab_end(self) -> int:
        return (self.rank + 1) * (self.cfg.vocab_size // self.world)

    def nbytes(self) -> int:
        n = 0
        for t in self.tensors():
            n += t.numel() * t.element_size()
        return n

    def tensors(self):
        yield from self.embed
        yield self.norm
        for L in self.layers:
            yield L.ln1
            yield L.ln2
            for tri in (L.q, L.k, L.v, L.o, L.gate, L.up, L.down):
                yield from tri

    # ------------------------------------------------------------ constructors

    @classmethod
    def from_shard(cls, cfg: ModelConfig, shard: Dict[str, object], world: int, rank: int, bits: int,
                   group: int, device: torch.device) -> "RankWeights":
        """Upload one rank's shard dict (reference layout) to ``device``.

        Row-parallel scales kept at full K (replicated by the sharder when
        their group count did not divide) are sliced to this rank, as
        ``QuantizedRowParallelLinear.load_quantized_shard`` does
        (parallel/quantized_linear.py:385-414).
        """
        pf = 32 // bits

        def tri(prefix: str, row_parallel: bool = False) -> QTriple:
            w = shard[f"{prefix}.weight"]
            s = shard[f"{prefix}.scales"]
            b = shard[f"{prefix}.biases"]
            if row_parallel:
                local_groups = tuple(w.shape)[1] * pf // group
                if tuple(s.shape)[1] == local_groups * world and world > 1:
                    sl = slice(rank * local_groups, (rank + 1) * local_groups)
                    s, b = s[:, sl], b[:, sl]
            return _dev_words(w, device), _dev_f16(s, device), _dev_f16(b, device)

        layers = []
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}"
            layers.append(LayerWeights(
                ln1=_dev_f16(shard[f"{p}.input_layernorm.weight"], device),
                ln2=_dev_f16(shard[f"{p}.post_attention_layernorm.weight"], device),
                q=tri(f"{p}.self_attn.q_proj"), k=tri(f"{p}.self_attn.k_proj"), v=tri(f"{p}.self_attn.v_proj"),
                o=tri(f"{p}.self_attn.o_proj", True),
                gate=tri(f"{p}.mlp.gate_proj"), up=tri(f"{p}.mlp.up_proj"),
                down=tri(f"{p}.mlp.down_proj", True)))
        return cls(cfg=cfg, world=world, rank=rank, bits=bits, group=group,
                   embed=tri("model.embed_tokens"), norm=_dev_f16(shard["model.norm.weight"], device),
                   layers=layers)

    @classmethod
    def from_safetensors(cls, cfg: ModelConfig, shard_dir: str, world: int, rank: int, bits: int, group: int,
                         device: torch.device) -> "RankWeights":
        """Load ``shard_dir/rank_{rank}/model.safetensors`` straight into one
        device allocation (``model.loader.load_rank_shard``) and build the
        rank's weights from those views (no host copy of any tensor)."""
        from ..model.loader import load_rank_shard

        return cls.from_shard(cfg, load_rank_shard(shard_dir, rank, device), world, rank, bits, group, device)

    SYNTH_SLICES = 8  # the finest tensor-parallel split the synthetic model is drawn for

    @classmethod
    def synthetic(cls, cfg: ModelConfig, world: int, rank: int, bits: int = 4, group: int = 64,
                  device: Optional[torch.device] = None, seed: int = 0, std: float = 0.02) -> "RankWeights":
        """Random-init N(0, std) fp16 weights of this rank's shard of ONE full
        model, quantized on the GPU.

        Every full tensor is drawn as 8 slices along the axis the sharder
        splits it on (output rows of the column-parallel linears and of the
        vocab-split embedding, input columns of the row-parallel o / down),
        slice j from its own seed (tensor, j).  A rank of a world dividing 8
        draws exactly its slices, so TP 1, 2, 4 and 8 hold shards of the same
        model (their greedy tokens agree up to the reduction order).  Other
        world sizes draw each rank's shard from seeds of (tensor, rank).
        """
        device = device or torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=device)
        H, F, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        Hq, Hkv = cfg.num_heads // world, cfg.kv_heads // world
        nsl = cls.SYNTH_SLICES
        sliced = nsl % world == 0
        per = nsl // world if sliced else 1
        tensor_id = [0]

        def draw(rows: int, cols: int, sd: int) -> torch.Tensor:
            gen.manual_seed(sd)
            return (torch.randn(rows, cols, generator=gen, device=device) * std).to(torch.float16)

        def q(rows: int, cols: int, split_cols: bool = False) -> QTriple:
            """This rank's [rows, cols] shard; slices along cols for row-parallel tensors."""
            tensor_id[0] += 1
            base = (seed * 1000003 + tensor_id[0]) * 1009
            out_w = torch.empty(rows, cols * bits // 32, dtype=torch.int32, device=device)
            out_s = torch.empty(rows, cols // group, dtype=torch.float16, device=device)
            out_b = torch.empty_like(out_s)
            even = (cols % (per * group) == 0) if split_cols else (rows % per == 0)
            if not (sliced and even):  # one draw per rank
                pieces = [(0, rows, 0, cols, base + 7919 * (rank + 1))]
            elif split_cols:
                c = cols // per
                pieces = [(0, rows, j * c, c, base + rank * per + j) for j in range(per)]
            else:
                r = rows // per
                pieces = [(j * r, r, 0, cols, base + rank * per + j) for j in range(per)]
            for (r0, nr, c0, nc, sd) in pieces:
                w = draw(nr, nc, sd)
                a, b_, c_ = ops.quantize(w, group, bits)
                del w
                out_w[r0:r0 + nr, c0 * bits // 32:(c0 + nc) * bits // 32] = a
                out_s[r0:r0 + nr, c0 // group:(c0 + nc) // group] = b_
                out_b[r0:r0 + nr, c0 // group:(c0 + nc) // group] = c_
            return out_w, out_s, out_b

        ones = torch.ones(H, dtype=torch.float16, device=device)
        layers = []
        for _ in range(cfg.num_layers):
            layers.append(LayerWeights(ln1=ones.clone(), ln2=ones.clone(), q=q(Hq * hd, H), k=q(Hkv * hd, H),
                                       v=q(Hkv * hd, H), o=q(H, Hq * hd, True), gate=q(F // world, H),
                                       up=q(F // world, H), down=q(H, F // world, True)))
        return cls(cfg=cfg, world=world, rank=rank, bits=bits, group=group,
                   embed=q(cfg.vocab_size // world, H), norm=ones.clone(), layers=layers)
