"""Tensor-parallel GQA attention with a preallocated device KV cache
(reference ``parallel/attention.py``).

``ParallelAttention.forward`` keeps the reference signature
``(hidden_states, attention_mask=None, position_ids=None,
past_key_value=None, use_cache=False) -> (output, cache)`` (:381-471) and the
same math -- head split across ranks, rotate-half RoPE at
``position_offset = cached length`` before the cache append, GQA head
``h -> h // (Hq/Hkv)``, scale ``1/sqrt(hd)`` after ``q.k``, causal mask
``triu(k = L - S + 1)`` for S > 1, o_proj row-parallel with all-reduce -- but
runs it as four kernels: the q|k|v GEMV (one fused launch over three weight
segments), ``sc_rope_append`` (RoPE + cache write), ``sc_flash_decode``
(split-KV online softmax) and the o_proj GEMV.

The cache is a ``KVCache`` handle over preallocated ``[B, Hkv/TP, Lmax, hd]``
fp32 buffers (the reference caches fp32: RoPE's fp32 tables promote k) with
the position kept on the device; ``cache[0]`` / ``cache[1]``
return the filled ``[B, Hkv/TP, L, hd]`` views, so code that reads
``past_key_value[0].shape[2]`` as the cached length keeps working.
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

from .. import ops
from .linear import ColumnParallelLinear, RowParallelLinear
from .quantized_linear import QuantizedColumnParallelLinear, QuantizedRowParallelLinear


class RoPE:
    """Rotary tables (parallel/attention.py:19-151): ``inv_freq =
    1 / base**(arange(0, hd, 2)/hd)`` in fp32, positions divided by
    ``scaling_factor``; ``__call__`` applies rotate-half to ``[B, H, S, hd]``."""

    def __init__(self, head_dim: int, max_position_embeddings: int = 2048, base: float = 10000.0,
                 scaling_factor: float = 1.0, device: Optional[torch.device] = None):
        self.head_dim = head_dim
        self.max_position_embeddings = max_position_embeddings
        self.base = base
        self.scaling_factor = scaling_factor
        self.device = device
        self.inv_freq = (np.float32(1.0) / (np.float32(base) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                                                   / np.float32(head_dim)))).astype(np.float32)
        self._cos: Optional[torch.Tensor] = None
        self._sin: Optional[torch.Tensor] = None
        self._cache_seq_len = 0

    def tables(self, seq_len: int, device: torch.device):
        """fp32 cos/sin halves ``[len, hd/2]`` covering ``seq_len`` positions
        (grown like the reference: max(seq, 2 * old, 256))."""
        if seq_len > self._cache_seq_len or self._cos is None or self._cos.device != device:
            n = max(seq_len, self._cache_seq_len * 2, 256)
            t = np.arange(n, dtype=np.float32)
            if self.scaling_factor != 1.0:
                t = (t / np.float32(self.scaling_factor)).astype(np.float32)
            f = np.outer(t, self.inv_freq).astype(np.float32)
            self._cos = torch.from_numpy(np.cos(f).astype(np.float32)).to(device)
            self._sin = torch.from_numpy(np.sin(f).astype(np.float32)).to(device)
            self._cache_seq_len = n
        return self._cos, self._sin

    def __call__(self, q: torch.Tensor, k: torch.Tensor, position_offset: int = 0):
        S = q.shape[2]
        cos, sin = self.tables(position_offset + S, q.device)
        c = torch.cat([cos, cos], -1)[position_offset:position_offset + S][None, None]
        s = torch.cat([sin, sin], -1)[position_offset:position_offset + S][None, None]

        def rot(x):
            h = x.shape[-1] // 2
            xf = x.float()
            return (xf * c + torch.cat([-xf[..., h:], xf[..., :h]], -1) * s).to(x.dtype)

        return rot(q), rot(k)


class KVCache:
    """Preallocated per-layer KV cache with a device-side length counter."""

    def __init__(self, batch: int, kv_heads: int, max_len: int, head_dim: int, device: torch.device):
        self.k = torch.zeros(batch, kv_heads, max_len, head_dim, dtype=torch.float32, device=device)
        self.v = torch.zeros_like(self.k)
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        self.length = 0
        self.max_len = max_len

    def __getitem__(self, i: int) -> torch.Tensor:
        return (self.k if i == 0 else self.v)[:, :, : self.length]

    def __len__(self) -> int:
        return 2

    def advance(self, n: int):
        if self.length + n > self.max_len:
            raise ValueError(f"KV cache full: {self.length} + {n} > {self.max_len}")
        self.length += n
        self.pos += n


class ParallelAttention:
    def __init__(self, hidden_size: int, num_heads: int, world_size: int, rank: int, communicator,
                 num_kv_heads: Optional[int] = None, head_dim: Optional[int] = None, bias: bool = False,
                 attention_dropout: float = 0.0, max_position_embeddings: int = 2048, rope_base: float = 10000.0,
                 rope_scaling_factor: float = 1.0, use_quantized: bool = False, quantization_bits: int = 4,
                 quantization_group_size: int = 64):
        if num_heads % world_size != 0:
            raise ValueError(f"num_heads ({num_heads}) must be divisible by world_size ({world_size})")
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.world_size = world_size
        self.rank = rank
        self.communicator = communicator
        self.local_num_heads = num_heads // world_size
        self.head_dim = head_dim if head_dim else hidden_size // num_heads
        self.local_hidden = self.local_num_heads * self.head_dim
        self.num_kv_heads = num_kv_heads if num_kv_heads else num_heads
        if self.num_kv_heads % world_size != 0:
            raise ValueError(f"num_kv_heads ({self.num_kv_heads}) must be divisible by world_size")
        self.local_num_kv_heads = self.num_kv_heads // world_size
        self.local_kv_hidden = self.local_num_kv_heads * self.head_dim
        self.scale = 1.0 / math.sqrt(self.head_dim)
        self.max_position_embeddings = max_position_embeddings
        self.rope = RoPE(self.head_dim, max_position_embeddings, rope_base, rope_scaling_factor)
        self.use_quantized = use_quantized
        self.bits = quantization_bits
        self.group_size = quantization_group_size
        kv_out = self.num_kv_heads * self.head_dim
        if use_quantized:
            mk = lambda o: QuantizedColumnParallelLinear(hidden_size, o, world_size, rank, bias=bias,  # noqa: E731
                                                         group_size=quantization_group_size, bits=quantization_bits)
            self.q_proj, self.k_proj, self.v_proj = mk(num_heads * self.head_dim), mk(kv_out), mk(kv_out)
            self.o_proj = QuantizedRowParallelLinear(num_heads * self.head_dim, hidden_size, world_size, rank,
                                                     bias=bias, communicator=communicator,
                                                     group_size=quantization_group_size, bits=quantization_bits)
        else:
            mk = lambda o: ColumnParallelLinear(hidden_size, o, world_size, rank, bias=bias)  # noqa: E731
            self.q_proj, self.k_proj, self.v_proj = mk(num_heads * self.head_dim), mk(kv_out), mk(kv_out)
            self.o_proj = RowParallelLinear(num_heads * self.head_dim, hidden_size, world_size, rank, bias=bias,
                                            communicator=communicator)

    # ------------------------------------------------------------ loading

    def load_shards(self, q_weight, k_weight, v_weight, o_weight, q_bias=None, k_bias=None, v_bias=None,
                    o_bias=None):
        self.q_proj.load_shard_direct(q_weight, q_bias)
        self.k_proj.load_shard_direct(k_weight, k_bias)
        self.v_proj.load_shard_direct(v_weight, v_bias)
        self.o_proj.load_shard_direct(o_weight, o_bias)

    def load_quantized_shards(self, q, k, v, o):
        """Each argument is a ``(weight, scales, biases)`` triple of this rank's shard."""
        self.q_proj.load_quantized_shard(*q)
        self.k_proj.load_quantized_shard(*k)
        self.v_proj.load_quantized_shard(*v)
        self.o_proj.load_quantized_shard(*o)

    def new_cache(self, batch: int, max_len: Optional[int] = None, device: Optional[torch.device] = None):
        dev = device or torch.device("cuda", torch.cuda.current_device())
        return KVCache(batch, self.local_num_kv_heads, max_len or self.max_position_embeddings, self.head_dim, dev)

    # ------------------------------------------------------------ compute

    def _qkv(self, x2: torch.Tensor) -> torch.Tensor:
        """``[M, (Hq + 2 Hkv) hd]`` fp32 projections of this rank's heads."""
        if self.use_quantized:
            segs = []
            for p in (self.q_proj, self.k_proj, self.v_proj):
                if p.quantized_weight is None:
                    raise RuntimeError("Weight not loaded")
                segs.append((p.quantized_weight, p.scales, p.biases_quant))
            qkv = ops.qlinear_fused(x2, segs, self.group_size, self.bits)
            biases = [p.bias for p in (self.q_proj, self.k_proj, self.v_proj)]
            if any(b is not None for b in biases):
                qkv = qkv + torch.cat([(b if b is not None else torch.zeros(p.local_out_features, device=qkv.device))
                                       .float() for b, p in zip(biases, (self.q_proj, self.k_proj, self.v_proj))])
            return qkv
        return torch.cat([p.forward_sync(x2).float() for p in (self.q_proj, self.k_proj, self.v_proj)], dim=-1)

    def forward_sync_partial(self, hidden_states: torch.Tensor, past_key_value: Optional[KVCache] = None,
                             use_cache: bool = False):
        """Attention up to this rank's o_proj partial (no all-reduce)."""
        B, S, _ = hidden_states.shape
        dev = hidden_states.device
        cache = past_key_value
        if cache is None:
            cache = self.new_cache(B, max(S, self.max_position_embeddings), dev)
        elif not isinstance(cache, KVCache):
            raise TypeError("past_key_value must be the KVCache this layer returned")
        if cache.length + S > cache.max_len:
            raise ValueError(f"KV cache full: {cache.length} + {S} > {cache.max_len}")
        x2 = hidden_states.reshape(B * S, -1)
        qkv = self._qkv(x2).contiguous()
        cos, sin = self.rope.tables(cache.max_len, dev)
        q = torch.empty(B * S, self.local_hidden, dtype=torch.float32, device=dev)
        ops.rope_append(qkv, B, S, self.local_num_heads, self.local_num_kv_heads, self.head_dim, cache.pos, cos, sin,
                        q, cache.k, cache.v)
        attn = torch.empty(B * S, self.local_hidden, dtype=torch.float32, device=dev)
        splits = 1 if S > 1 else max(1, min(64, math.ceil(296 / max(1, self.local_num_kv_heads * B)),
                                            math.ceil((cache.length + 1) / 64)))
        ops.flash_decode(q, cache.k, cache.v, cache.pos, B, S, self.local_num_heads, self.local_num_kv_heads,
                         self.head_dim, splits, attn, scale=self.scale)
        cache.advance(S)
        attn = attn.view(B, S, self.local_hidden)
        part = self.o_proj.forward_partial(attn)
        return part, (cache if use_cache else None)

    async def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                      position_ids: Optional[torch.Tensor] = None, past_key_value: Optional[KVCache] = None,
                      use_cache: bool = False):
        if attention_mask is not None:
            raise NotImplementedError("additive attention masks are not supported; the causal mask is built in")
        part, cache = self.forward_sync_partial(hidden_states, past_key_value, use_cache=True)
        out = part
        if self.communicator is not None and self.world_size > 1:
            out = await self.communicator.all_reduce(part, op="sum")
        bias = getattr(self.o_proj, "bias", None)
        if bias is not None and self.rank == 0:
            out = out + bias.to(out.dtype)
        return out, (cache if use_cache else None)

    @property
    def num_parameters(self) -> int:
        return sum(p.num_parameters for p in (self.q_proj, self.k_proj, self.v_proj, self.o_proj))

