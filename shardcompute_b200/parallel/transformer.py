"""Tensor-parallel decoder model (reference ``parallel/transformer.py``).

``RMSNorm`` (:17-61), ``ParallelTransformerBlock`` (:64-336) and
``ParallelTransformer`` (:339-596) with the reference's constructor
arguments, loaders and ``forward(input_ids, attention_mask=None,
past_key_values=None, use_cache=False) -> (logits, cache)``.  The residual
stream is fp32 on the device; logits are fp32 and all-gathered over the
vocabulary split (tied LM head = ``h @ dequantize(embed).T`` per rank,
computed as one fused RMSNorm + dequant-GEMV launch without materialising the
dequantized table).

This layer-by-layer object is the drop-in API.  For decoding,
``ParallelExecutor.generate`` drives ``DecodeEngine``, which runs the same
kernels with all-device state and replays each step as one CUDA graph.
"""

from __future__ import annotations

import logging
from typing import Dict, List, Optional

import torch

from .. import ops
from ._tensors import as_device
from .attention import KVCache, ParallelAttention
from .embedding import ParallelEmbedding, QuantizedParallelEmbedding
from .linear import ColumnParallelLinear
from .mlp import ParallelMLP

logger = logging.getLogger(__name__)


class RMSNorm:
    """``x / sqrt(mean(x^2) + eps) * w`` over the last dim (one CTA per row)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight: Optional[torch.Tensor] = None
        self.bias: Optional[torch.Tensor] = None

    def load_weights(self, weight, bias=None):
        self.weight = as_device(weight, torch.float16)
        self.bias = as_device(bias, torch.float16) if bias is not None else None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("RMSNorm weight not loaded")
        y = ops.rmsnorm(x, self.weight, self.eps)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y


class ParallelTransformerBlock:
    def __init__(self, layer_idx: int, hidden_size: int, num_heads: int, intermediate_size: int, world_size: int,
                 rank: int, communicator, num_kv_heads: Optional[int] = None, rms_norm_eps: float = 1e-5,
                 attention_bias: bool = False, mlp_bias: bool = False, max_position_embeddings: int = 2048,
                 rope_base: float = 10000.0, mlp_activation: str = "silu", use_gated_mlp: bool = True,
                 use_quantized: bool = False, quantization_bits: int = 4, quantization_group_size: int = 64):
        self.layer_idx = layer_idx
        self.hidden_size = hidden_size
        self.world_size = world_size
        self.rank = rank
        self.communicator = communicator
        self.use_quantized = use_quantized
        self.input_layernorm = RMSNorm(hidden_size, eps=rms_norm_eps)
        self.attention = ParallelAttention(hidden_size, num_heads, world_size, rank, communicator,
                                           num_kv_heads=num_kv_heads, bias=attention_bias,
                                           max_position_embeddings=max_position_embeddings, rope_base=rope_base,
                                           use_quantized=use_quantized, quantization_bits=quantization_bits,
                                           quantization_group_size=quantization_group_size)
        self.post_attention_layernorm = RMSNorm(hidden_size, eps=rms_norm_eps)
        self.mlp = ParallelMLP(hidden_size, intermediate_size, world_size, rank, communicator,
                               activation=mlp_activation, bias=mlp_bias, use_gated=use_gated_mlp,
                               use_quantized=use_quantized, quantization_bits=quantization_bits,
                               quantization_group_size=quantization_group_size)

    def load_weights(self, input_ln_weight, post_attn_ln_weight, attn_weights: Dict, mlp_weights: Dict):
        self.input_layernorm.load_weights(input_ln_weight)
        self.post_attention_layernorm.load_weights(post_attn_ln_weight)
        self.attention.load_shards(q_weight=attn_weights["q_weight"], q_bias=attn_weights.get("q_bias"),
                                   k_weight=attn_weights["k_weight"], k_bias=attn_weights.get("k_bias"),
                                   v_weight=attn_weights["v_weight"], v_bias=attn_weights.get("v_bias"),
                                   o_weight=attn_weights["o_weight"], o_bias=attn_weights.get("o_bias"))
        self.mlp.load_shards(up_weight=mlp_weights["up_weight"], up_bias=mlp_weights.get("up_bias"),
                             down_weight=mlp_weights["down_weight"], down_bias=mlp_weights.get("down_bias"),
                             gate_weight=mlp_weights.get("gate_weight"), gate_bias=mlp_weights.get("gate_bias"))

    def load_quantized_weights(self, input_ln_weight, post_attn_ln_weight, q, k, v, o, gate, up, down):
        """Each projection is a ``(weight, scales, biases)`` triple of this rank's shard."""
        self.input_layernorm.load_weights(input_ln_weight)
        self.post_attention_layernorm.load_weights(post_attn_ln_weight)
        self.attention.load_quantized_shards(q, k, v, o)
        self.mlp.load_quantized_shards(up=up, down=down, gate=gate)

    async def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                      past_key_value: Optional[KVCache] = None, use_cache: bool = False):
        h = hidden_states.float()
        attn, cache = await self.attention.forward(self.input_layernorm(h), attention_mask=attention_mask,
                                                   past_key_value=past_key_value, use_cache=True)
        h = h + attn.float()
        h = h + (await self.mlp.forward(self.post_attention_layernorm(h))).float()
        return h, (cache if use_cache else None)

    @property
    def num_parameters(self) -> int:
        return self.attention.num_parameters + self.mlp.num_parameters + 2 * self.hidden_size


class ParallelTransformer:
    def __init__(self, vocab_size: int, hidden_size: int, num_layers: int, num_heads: int, intermediate_size: int,
                 world_size: int, rank: int, communicator, num_kv_heads: Optional[int] = None,
                 max_position_embeddings: int = 2048, rms_norm_eps: float = 1e-5, tie_word_embeddings: bool = False,
                 rope_base: float = 10000.0, mlp_activation: str = "silu", use_gated_mlp: bool = True,
                 use_quantized: bool = False, quantization_bits: int = 4, quantization_group_size: int = 64):
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.num_layers = num_layers
        self.world_size = world_size
        self.rank = rank
        self.communicator = communicator
        self.tie_word_embeddings = tie_word_embeddings
        self.use_quantized = use_quantized
        self.quantization_bits = quantization_bits
        self.quantization_group_size = quantization_group_size
        self.max_position_embeddings = max_position_embeddings
        if use_quantized:
            self.embed_tokens = QuantizedParallelEmbedding(vocab_size, hidden_size, world_size, rank, communicator,
                                                           group_size=quantization_group_size,
                                                           bits=quantization_bits)
        else:
            self.embed_tokens = ParallelEmbedding(vocab_size, hidden_size, world_size, rank, communicator,
                                                  gather_output=True)
        self.layers: List[ParallelTransformerBlock] = [
            ParallelTransformerBlock(i, hidden_size, num_heads, intermediate_size, world_size, rank, communicator,
                                     num_kv_heads=num_kv_heads, rms_norm_eps=rms_norm_eps,
                                     max_position_embeddings=max_position_embeddings, rope_base=rope_base,
                                     mlp_activation=mlp_activation, use_gated_mlp=use_gated_mlp,
                                     use_quantized=use_quantized, quantization_bits=quantization_bits,
                                     quantization_group_size=quantization_group_size)
            for i in range(num_layers)]
        self.norm = RMSNorm(hidden_size, eps=rms_norm_eps)
        self.lm_head = None
        if not tie_word_embeddings:
            self.lm_head = ColumnParallelLinear(hidden_size, vocab_size, world_size, rank, bias=False,
                                                gather_output=True, communicator=communicator)

    @classmethod
    def from_config(cls, cfg, world_size: int, rank: int, communicator=None) -> "ParallelTransformer":
        q = cfg.quantization
        return cls(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, num_layers=cfg.num_layers,
                   num_heads=cfg.num_heads, intermediate_size=cfg.intermediate_size, world_size=world_size,
                   rank=rank, communicator=communicator, num_kv_heads=cfg.kv_heads,
                   max_position_embeddings=cfg.max_position_embeddings, rms_norm_eps=cfg.rms_norm_eps,
                   tie_word_embeddings=cfg.tie_word_embeddings, rope_base=cfg.rope_theta,
                   mlp_activation=cfg.hidden_act, use_gated_mlp=cfg.use_gated_mlp,
                   use_quantized=bool(q and q.enabled), quantization_bits=q.bits if q else 4,
                   quantization_group_size=q.group_size if q else 64)

    def load_embedding_weights(self, weight):
        self.embed_tokens.load_shard_direct(weight)

    def load_quantized_embedding_weights(self, weight, scales, biases):
        if not self.use_quantized:
            raise RuntimeError("Cannot load quantized embeddings into non-quantized model")
        self.embed_tokens.load_quantized_shard(weight, scales, biases)

    def load_lm_head_weights(self, weight):
        if self.lm_head is not None:
            self.lm_head.load_shard_direct(weight)

    def load_norm_weights(self, weight):
        self.norm.load_weights(weight)

    def load_rank_weights(self, w) -> "ParallelTransformer":
        """Load a ``RankWeights`` (per-rank device shard) into the layer objects."""
        self.load_quantized_embedding_weights(*w.embed)
        self.load_norm_weights(w.norm)
        for layer, lw in zip(self.layers, w.layers):
            layer.load_quantized_weights(lw.ln1, lw.ln2, lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down)
        return self

    def new_cache(self, batch: int, max_len: Optional[int] = None) -> List[KVCache]:
        return [layer.attention.new_cache(batch, max_len or self.max_position_embeddings) for layer in self.layers]

    async def logits_local(self, hidden: torch.Tensor) -> torch.Tensor:
        """This rank's vocab slice of the logits ``[B, S, V/TP]`` (fp32)."""
        B, S, H = hidden.shape
        if self.tie_word_embeddings:
            e = self.embed_tokens
            if e.quantized_weight is None:
                raise RuntimeError("Embedding weights not loaded")
            if not self.use_quantized:
                raise NotImplementedError("tied head over an unquantized hidden-split table")
            return ops.qlinear_fused(hidden.reshape(B * S, H).float(),
                                     [(e.quantized_weight, e.scales, e.biases_quant)], e.group_size, e.bits,
                                     norm_weight=self.norm.weight, eps=self.norm.eps).view(B, S, -1)
        return self.lm_head.forward_sync(self.norm(hidden)).float()

    async def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                      past_key_values: Optional[List[KVCache]] = None, use_cache: bool = False,
                      return_hidden: bool = False):
        h = (await self.embed_tokens.forward(input_ids)).float()
        hidden = [h] if return_hidden else None
        new_cache = [] if use_cache else None
        for i, layer in enumerate(self.layers):
            past = past_key_values[i] if past_key_values else None
            h, cache = await layer.forward(h, attention_mask=attention_mask, past_key_value=past, use_cache=True)
            if use_cache:
                new_cache.append(cache)
            if return_hidden:
                hidden.append(h)
        logits = await self.logits_local(h)
        if self.tie_word_embeddings and self.communicator is not None and self.world_size > 1:
            logits = await self.communicator.all_gather(logits, dim=-1)
        elif not self.tie_word_embeddings and self.world_size > 1:
            logits = await self.communicator.all_gather(logits, dim=-1)
        if return_hidden:
            return logits, new_cache, hidden
        return logits, new_cache

    @property
    def num_parameters(self) -> int:
        n = self.embed_tokens.num_parameters + sum(layer.num_parameters for layer in self.layers) + self.hidden_size
        return n + (self.lm_head.num_parameters if self.lm_head is not None else 0)

    def get_layer(self, idx: int) -> ParallelTransformerBlock:
        if not 0 <= idx < self.num_layers:
            raise IndexError(f"Layer index {idx} out of range [0, {self.num_layers})")
        return self.layers[idx]
