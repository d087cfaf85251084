"""Timed CPU stand-in for the reference's decode step (host cores, torch fp32).

TEST INFRASTRUCTURE ONLY: used by ``bench.py`` for its ``cpu_baseline`` leg
and its ``--impl reference`` arm, never by the product package.

The reference runs the quantized decode step on MLX's CPU path
(``mx.quantized_matmul`` per linear, ``parallel/quantized_linear.py:168-176``;
attention over the concatenated cache, ``parallel/attention.py:403-467``;
tied LM head via ``dequantize_weight``, ``parallel/transformer.py:565-573``).
MLX is not installed on either machine, so this module restates the same work
in torch fp32 on all host threads: every step dequantizes each linear's packed
words group-wise (``s*q + b``) and multiplies, runs softmax attention over a
KV cache of ``ctx`` positions, and dequantizes its share of the tied head.

One *sample* is 1/L of a token on one rank's shard: one decoder layer plus
1/L of the LM-head rows (L = number of layers).  At TP degree N the host
runs all N ranks' shards one after another on the same cores (the reference
would need N hosts), so tokens/s of the full model is
``batch / (L * N * seconds_per_sample)``.  Unlike MLX's fused
``quantized_matmul``, this stand-in dequantizes every weight to fp32 on
every step, which makes it slower than MLX would be.  Packed words are uniform random (the
timing does not depend on the values); scales/biases are small fp16 numbers.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass

import torch


@dataclass
class DecodeShape:
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    ffn: int = 14336
    vocab: int = 128256
    bits: int = 4
    group: int = 64
    ctx: int = 2048
    batch: int = 1
    world: int = 1  # TP degree: one rank's shard of every linear

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def _qtensor(rows: int, cols: int, bits: int, group: int, gen: torch.Generator):
    words = torch.randint(-(2 ** 31), 2 ** 31 - 1, (rows, cols * bits // 32), dtype=torch.int32, generator=gen)
    s = (torch.rand(rows, cols // group, generator=gen) * 0.01 + 0.001).to(torch.float16)
    b = (torch.rand(rows, cols // group, generator=gen) * -0.05).to(torch.float16)
    return words, s, b


def dequant_f32(words: torch.Tensor, s: torch.Tensor, b: torch.Tensor, bits: int, group: int) -> torch.Tensor:
    """Group-wise affine dequantize (element j of a word at bits [bits*j, bits*(j+1)))."""
    pf = 32 // bits
    shifts = torch.arange(0, 32, bits, dtype=torch.int32)
    q = (words.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)  # [rows, words, pf]
    rows = words.shape[0]
    q = q.reshape(rows, -1, group).to(torch.float32)
    w = q * s.to(torch.float32).unsqueeze(-1) + b.to(torch.float32).unsqueeze(-1)
    return w.reshape(rows, words.shape[1] * pf)


class CpuDecodeSample:
    """One layer's decode work (+1/L of the tied head) on the host cores."""

    def __init__(self, shape: DecodeShape, threads: int = 0, seed: int = 0):
        self.sh = shape
        self.threads = threads or os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        gen = torch.Generator().manual_seed(seed)
        H, F, hd, W = shape.hidden, shape.ffn, shape.head_dim, shape.world
        hq, hkv = shape.heads // W, shape.kv_heads // W
        q = lambda r, c: _qtensor(r, c, shape.bits, shape.group, gen)  # noqa: E731
        self.lin = {"q": q(hq * hd, H), "k": q(hkv * hd, H), "v": q(hkv * hd, H), "o": q(H, hq * hd),
                    "gate": q(F // W, H), "up": q(F // W, H), "down": q(H, F // W)}
        head_rows = math.ceil(shape.vocab // W / shape.layers)
        self.head = q(head_rows, H)
        self.kc = torch.randn(shape.batch, hkv, shape.ctx, hd, generator=gen)
        self.vc = torch.randn(shape.batch, hkv, shape.ctx, hd, generator=gen)
        self.x = torch.randn(shape.batch, H, generator=gen)
        self.hq, self.hkv = hq, hkv

    def _lin(self, x, name):
        w = dequant_f32(*self.lin[name], self.sh.bits, self.sh.group)
        return x @ w.T

    @staticmethod
    def _rms(x):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-5)

    def run(self) -> torch.Tensor:
        sh, B, hd = self.sh, self.sh.batch, self.sh.head_dim
        h = self.x
        x = self._rms(h)
        q = self._lin(x, "q").view(B, self.hq, 1, hd)
        k = self._lin(x, "k").view(B, self.hkv, 1, hd)
        v = self._lin(x, "v").view(B, self.hkv, 1, hd)
        kk = torch.cat([self.kc, k], dim=2).repeat_interleave(self.hq // self.hkv, dim=1)
        vv = torch.cat([self.vc, v], dim=2).repeat_interleave(self.hq // self.hkv, dim=1)
        p = torch.softmax((q @ kk.transpose(-1, -2)) / math.sqrt(hd), dim=-1)
        a = (p @ vv).reshape(B, self.hq * hd)
        h = h + self._lin(a, "o")
        x = self._rms(h)
        g, u = self._lin(x, "gate"), self._lin(x, "up")
        h = h + self._lin(torch.nn.functional.silu(g) * u, "down")
        logits = self._rms(h) @ dequant_f32(*self.head, sh.bits, sh.group).T
        return logits.argmax(-1)

    def time_samples(self, n: int) -> float:
        """Seconds per sample, averaged over ``n`` samples (after one warm-up)."""
        self.run()
        t0 = time.perf_counter()
        for _ in range(n):
            self.run()
        return (time.perf_counter() - t0) / n

    def tokens_per_s(self, sec_per_sample: float) -> float:
        """Whole-model tokens/s on this host: L layers x N rank shards per token."""
        return self.sh.batch / (self.sh.layers * self.sh.world * sec_per_sample)
