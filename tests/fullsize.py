"""Full-size parity helpers (test infrastructure only).

The numpy oracle (``oracle/tp.py``) cannot hold a dequantized 8B-parameter
model on the host in float64, so the full-depth tests use ``TorchRef``: the
same tensor-parallel math restated op for op in torch float64, run on the
GPU next to the engine.  ``tests/test_torch_ref.py`` pins it to the numpy
oracle on small shapes (CPU), so it carries the oracle's semantics:

* quantized linears: exact ``s*q + b`` in float64, ``x @ W^T``
  (``oracle.mlx_affine.quantized_matmul``);
* embedding gather and tied LM head: fp16-rounded ``dequantize``
  (``oracle.tp.embed_rank`` / ``TPModel.lm_head``);
* RMSNorm, rotate-half RoPE with fp32 tables, GQA softmax attention over a
  float64 KV cache, SwiGLU, rank-order all-reduce, rank-order all-gather
  (``oracle.tp``).

``gpu_checkpoint`` draws a full (unsharded) seeded checkpoint on the GPU in
the reference's layout (HF names, packed uint32 words as int32, fp16 scales
and biases, fp16 norms) with the library's quantizer (bit-exact against
``oracle.mlx_affine.quantize``); ``shard`` splits it by the reference's
sharder rules (``oracle.sharder``).
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional

import numpy as np
import torch

from oracle import sharder as osh
from oracle.tp import LlamaShape, rope_tables

LLAMA3_8B = dict(vocab_size=128256, hidden_size=4096, num_layers=32, num_heads=32, num_kv_heads=8,
                 intermediate_size=14336, rms_norm_eps=1e-5, rope_theta=5e5)
TINYLLAMA = dict(vocab_size=32000, hidden_size=2048, num_layers=22, num_heads=32, num_kv_heads=4,
                 intermediate_size=5632, rms_norm_eps=1e-5, rope_theta=1e4)


def gpu_checkpoint(shape: LlamaShape, seed: int, device, std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Seeded full checkpoint drawn on ``device`` (deterministic per seed)."""
    from shardcompute_b200 import ops

    gen = torch.Generator(device=device)
    H, F, hd = shape.hidden_size, shape.intermediate_size, shape.head_dim
    out: Dict[str, torch.Tensor] = {}
    counter = [seed * 1000003]

    def q(name: str, rows: int, cols: int):
        counter[0] += 1
        gen.manual_seed(counter[0])
        ws, ss, bs = [], [], []
        step = max(1, (32 << 20) // cols)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            w = (torch.randn(r1 - r0, cols, generator=gen, device=device) * std).to(torch.float16)
            a, b, c = ops.quantize(w, shape.group_size, shape.bits)
            ws.append(a)
            ss.append(b)
            bs.append(c)
        out[f"{name}.weight"] = torch.cat(ws)
        out[f"{name}.scales"] = torch.cat(ss)
        out[f"{name}.biases"] = torch.cat(bs)

    def norm(name: str):
        counter[0] += 1
        gen.manual_seed(counter[0])
        out[name] = (1.0 + 0.1 * torch.randn(H, generator=gen, device=device)).to(torch.float16)

    q("model.embed_tokens", shape.vocab_size, H)
    for i in range(shape.num_layers):
        p = f"model.layers.{i}"
        norm(f"{p}.input_layernorm.weight")
        norm(f"{p}.post_attention_layernorm.weight")
        q(f"{p}.self_attn.q_proj", shape.num_heads * hd, H)
        q(f"{p}.self_attn.k_proj", shape.num_kv_heads * hd, H)
        q(f"{p}.self_attn.v_proj", shape.num_kv_heads * hd, H)
        q(f"{p}.self_attn.o_proj", H, shape.num_heads * hd)
        q(f"{p}.mlp.gate_proj", F, H)
        q(f"{p}.mlp.up_proj", F, H)
        q(f"{p}.mlp.down_proj", H, F)
    norm("model.norm.weight")
    return out


def _split(t: torch.Tensor, world: int, rank: int, dim: int) -> torch.Tensor:
    n = t.shape[dim] // world
    return t.narrow(dim, rank * n, n).contiguous()


def shard(ckpt: Dict[str, torch.Tensor], world: int, rank: int) -> Dict[str, torch.Tensor]:
    """``oracle.sharder.shard_weights`` for a checkpoint of device tensors."""
    if world == 1:
        return dict(ckpt)
    out = {}
    for name, t in ckpt.items():
        base = name[: -len(".weight")] if name.endswith(".weight") else None
        if base is not None and f"{base}.scales" in ckpt:
            w, s, b = t, ckpt[f"{base}.scales"], ckpt[f"{base}.biases"]
            if any(x in name for x in osh._COLUMN_Q):
                w, s, b = _split(w, world, rank, 0), _split(s, world, rank, 0), _split(b, world, rank, 0)
            elif osh._is_row_parallel_q(name):
                w = _split(w, world, rank, 1)
                if s.shape[1] % world == 0:
                    s, b = _split(s, world, rank, 1), _split(b, world, rank, 1)
            out[name], out[f"{base}.scales"], out[f"{base}.biases"] = w, s, b
        elif name.endswith((".scales", ".biases")):
            continue
        else:
            out[name] = t
    return out


def _codes(words: torch.Tensor, bits: int) -> torch.Tensor:
    """Packed int32 words [R, W] -> codes [R, W * 32/bits] (element j at bits [bits*j, bits*(j+1)))."""
    pf = 32 // bits
    shifts = torch.arange(0, 32, bits, device=words.device, dtype=torch.int64)
    w = words.to(torch.int64) & 0xFFFFFFFF
    return ((w.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(words.shape[0], -1)


def dequant_exact(w: torch.Tensor, s: torch.Tensor, b: torch.Tensor, group: int, bits: int) -> torch.Tensor:
    """``s*q + b`` in float64 (``oracle.mlx_affine.dequantize_exact``), row slabs to bound memory."""
    R = w.shape[0]
    out = torch.empty(R, w.shape[1] * (32 // bits), dtype=torch.float64, device=w.device)
    step = max(1, (16 << 20) // out.shape[1])
    for r0 in range(0, R, step):
        r1 = min(R, r0 + step)
        q = _codes(w[r0:r1], bits).to(torch.float64)
        ss = s[r0:r1].to(torch.float64).repeat_interleave(group, dim=1)
        bb = b[r0:r1].to(torch.float64).repeat_interleave(group, dim=1)
        out[r0:r1] = ss * q + bb
    return out


def dequant_f16(w, s, b, group: int, bits: int) -> torch.Tensor:
    """``mx.dequantize``: exact value rounded once to fp16 (``oracle.mlx_affine.dequantize``)."""
    return dequant_exact(w, s, b, group, bits).to(torch.float16)


class TorchRef:
    """``oracle.tp.TPModel`` in torch float64 (all ranks in one process)."""

    def __init__(self, shards: List[Dict[str, torch.Tensor]], shape: LlamaShape, max_len: int, device=None):
        self.cfg = shape
        self.world = len(shards)
        self.device = device or shards[0]["model.norm.weight"].device
        g, bits = shape.group_size, shape.bits
        dev = self.device

        def lin(sd, name):
            return dequant_exact(sd[f"{name}.weight"].to(dev), sd[f"{name}.scales"].to(dev),
                                 sd[f"{name}.biases"].to(dev), g, bits)

        self.ranks = []
        for sd in shards:
            r = {"embed": dequant_f16(sd["model.embed_tokens.weight"].to(dev), sd["model.embed_tokens.scales"].to(dev),
                                      sd["model.embed_tokens.biases"].to(dev), g, bits),
                 "norm": sd["model.norm.weight"].to(dev).to(torch.float64), "layers": []}
            for i in range(shape.num_layers):
                p = f"model.layers.{i}"
                r["layers"].append({
                    "ln1": sd[f"{p}.input_layernorm.weight"].to(dev).to(torch.float64),
                    "ln2": sd[f"{p}.post_attention_layernorm.weight"].to(dev).to(torch.float64),
                    "q": lin(sd, f"{p}.self_attn.q_proj"), "k": lin(sd, f"{p}.self_attn.k_proj"),
                    "v": lin(sd, f"{p}.self_attn.v_proj"), "o": lin(sd, f"{p}.self_attn.o_proj"),
                    "gate": lin(sd, f"{p}.mlp.gate_proj"), "up": lin(sd, f"{p}.mlp.up_proj"),
                    "down": lin(sd, f"{p}.mlp.down_proj")})
            self.ranks.append(r)
        cos, sin = rope_tables(shape.head_dim, max_len, shape.rope_theta)
        self.cos = torch.from_numpy(np.concatenate([cos, cos], axis=-1)).to(dev, torch.float64)
        self.sin = torch.from_numpy(np.concatenate([sin, sin], axis=-1)).to(dev, torch.float64)
        self.cache: Optional[list] = None

    def reset(self):
        self.cache = None

    def _rms(self, x, w):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w

    def _rope(self, x, off: int):
        S, hd = x.shape[-2], x.shape[-1]
        c, s = self.cos[off:off + S], self.sin[off:off + S]
        rot = torch.cat([-x[..., hd // 2:], x[..., : hd // 2]], dim=-1)
        return x * c + rot * s

    def _embed(self, ids):
        cfg, W = self.cfg, self.world
        lv = cfg.vocab_size // W
        h = None
        for r in range(W):
            v0 = r * lv
            inr = (ids >= v0) & (ids < v0 + lv)
            e = self.ranks[r]["embed"][(ids - v0).clamp(0, lv - 1)]
            e = torch.where(inr[..., None], e, torch.zeros((), dtype=e.dtype, device=e.device)).to(torch.float64)
            h = e if h is None else h + e
        return h

    def forward(self, ids: torch.Tensor, return_hidden: bool = False):
        """Logits ``[B, S, V]`` float64 (and the hidden state after the embedding and each layer)."""
        cfg, W = self.cfg, self.world
        ids = ids.to(self.device, torch.int64)
        B, S = ids.shape
        hd = cfg.head_dim
        nh, nkv = cfg.num_heads // W, cfg.num_kv_heads // W
        h = self._embed(ids)
        hidden = [h.clone()] if return_hidden else None
        off = 0 if self.cache is None else self.cache[0][0][0].shape[2]
        new_cache = [[None] * cfg.num_layers for _ in range(W)]
        for i in range(cfg.num_layers):
            parts = []
            for r in range(W):
                L = self.ranks[r]["layers"][i]
                x = self._rms(h, L["ln1"])
                q = (x @ L["q"].T).view(B, S, nh, hd).transpose(1, 2)
                k = (x @ L["k"].T).view(B, S, nkv, hd).transpose(1, 2)
                v = (x @ L["v"].T).view(B, S, nkv, hd).transpose(1, 2)
                q, k = self._rope(q, off), self._rope(k, off)
                if self.cache is not None:
                    pk, pv = self.cache[r][i]
                    k, v = torch.cat([pk, k], dim=2), torch.cat([pv, v], dim=2)
                new_cache[r][i] = (k, v)
                Lk = k.shape[2]
                rep = nh // nkv
                kk, vv = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
                sc = (q @ kk.transpose(-1, -2)) * (1.0 / math.sqrt(hd))
                if S > 1:
                    sc = sc + torch.triu(torch.full((S, Lk), float("-inf"), dtype=sc.dtype, device=sc.device),
                                         diagonal=Lk - S + 1)
                o = torch.softmax(sc, dim=-1) @ vv
                o = o.transpose(1, 2).reshape(B, S, nh * hd)
                parts.append(o @ L["o"].T)
            h = h + self._sum(parts)
            parts = []
            for r in range(W):
                L = self.ranks[r]["layers"][i]
                x = self._rms(h, L["ln2"])
                g, u = x @ L["gate"].T, x @ L["up"].T
                parts.append((g / (1.0 + torch.exp(-g)) * u) @ L["down"].T)
            h = h + self._sum(parts)
            if return_hidden:
                hidden.append(h.clone())
        self.cache = new_cache
        logits = torch.cat([self._rms(h, R["norm"]) @ R["embed"].to(torch.float64).T for R in self.ranks], dim=-1)
        return (logits, hidden) if return_hidden else logits

    @staticmethod
    def _sum(parts):
        out = parts[0]
        for p in parts[1:]:
            out = out + p
        return out


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.to(torch.float64).reshape(-1)
    b = b.to(torch.float64).reshape(-1).to(a.device)
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-300))
