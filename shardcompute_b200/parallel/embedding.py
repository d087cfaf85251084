"""Tensor-parallel embeddings (reference ``parallel/embedding.py``).

* ``QuantizedParallelEmbedding`` (:191-394): vocab-split MLX-quantized table;
  ``forward`` = masked row gather + dequant (``sc_embed_gather_q``, one kernel,
  bit-exact with ``mx.dequantize``) then an all-reduce sum across ranks;
  ``dequantize_weight`` backs the tied LM head.
* ``VocabParallelEmbedding``: the same vocab split for an fp16 table
  (``sc_embed_gather_f16``).  The reference declares this class but leaves it
  unimplemented (:397-440); here it is the working fp16-row variant.
* ``ParallelEmbedding`` (:12-188): fp table split on the hidden dimension,
  local gather + all-gather of the slices.
"""

from __future__ import annotations

import logging
from typing import Optional

import torch

from .. import ops
from ._tensors import as_device, as_words

logger = logging.getLogger(__name__)


class QuantizedParallelEmbedding:
    def __init__(self, vocab_size: int, embedding_dim: int, world_size: int, rank: int, communicator=None,
                 group_size: int = 64, bits: int = 4):
        if vocab_size % world_size != 0:
            raise ValueError(f"vocab_size ({vocab_size}) must be divisible by world_size ({world_size})")
        self.vocab_size = vocab_size
        self.embedding_dim = embedding_dim
        self.world_size = world_size
        self.rank = rank
        self.communicator = communicator
        self.group_size = group_size
        self.bits = bits
        self.local_vocab_size = vocab_size // world_size
        self.vocab_start = rank * self.local_vocab_size
        self.vocab_end = self.vocab_start + self.local_vocab_size
        self.quantized_weight: Optional[torch.Tensor] = None
        self.scales: Optional[torch.Tensor] = None
        self.biases_quant: Optional[torch.Tensor] = None

    def load_quantized_shard(self, quantized_weight, scales, biases):
        qw = as_words(quantized_weight)
        if qw.shape[0] != self.local_vocab_size or qw.shape[1] * (32 // self.bits) != self.embedding_dim:
            raise ValueError(f"quantized embedding {tuple(qw.shape)} does not pack [{self.local_vocab_size}, "
                             f"{self.embedding_dim}] at {self.bits} bits")
        self.quantized_weight = qw
        self.scales = as_device(scales, torch.float16, qw.device)
        self.biases_quant = as_device(biases, torch.float16, qw.device)

    def load_shard_direct(self, weight_shard):
        """Quantize an fp ``[local_vocab, dim]`` shard on the GPU (``sc_quantize``)."""
        if weight_shard is None:
            logger.warning("load_shard_direct called with None weight, skipping")
            return
        if tuple(weight_shard.shape) != (self.local_vocab_size, self.embedding_dim):
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected "
                             f"{(self.local_vocab_size, self.embedding_dim)}. For quantized embeddings, use "
                             f"load_quantized_shard() with weight, scales, and biases.")
        w = as_device(weight_shard, torch.float16)
        self.quantized_weight, self.scales, self.biases_quant = ops.quantize(w, self.group_size, self.bits)

    def forward_local(self, input_ids: torch.Tensor) -> torch.Tensor:
        """This rank's masked, dequantized rows ``[B, S, dim]`` (fp16, zeros off-shard)."""
        if self.quantized_weight is None:
            raise RuntimeError("Embedding weights not loaded")
        ids = input_ids.to(device=self.quantized_weight.device)
        return ops.embed_gather_q(ids, self.quantized_weight, self.scales, self.biases_quant, self.vocab_start,
                                  self.vocab_end, self.embedding_dim, self.group_size, self.bits)

    async def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        emb = self.forward_local(input_ids)
        if self.communicator is not None:
            emb = await self.communicator.all_reduce(emb, op="sum")
        return emb

    @property
    def weight(self) -> Optional[torch.Tensor]:
        return self.quantized_weight

    def dequantize_weight(self) -> torch.Tensor:
        if self.quantized_weight is None or self.scales is None or self.biases_quant is None:
            raise RuntimeError("Quantized embedding weights not loaded")
        return ops.dequantize(self.quantized_weight, self.scales, self.biases_quant, self.group_size, self.bits)

    @property
    def num_parameters(self) -> int:
        return self.local_vocab_size * self.embedding_dim

    def __repr__(self) -> str:
        return (f"QuantizedParallelEmbedding(vocab_size={self.vocab_size}, local_vocab_size={self.local_vocab_size}, "
                f"embedding_dim={self.embedding_dim}, rank={self.rank}/{self.world_size}, bits={self.bits})")


class VocabParallelEmbedding:
    """fp16 table split by vocabulary: masked gather + all-reduce sum."""

    def __init__(self, vocab_size: int, embedding_dim: int, world_size: int, rank: int, communicator=None):
        if vocab_size % world_size != 0:
            raise ValueError(f"vocab_size ({vocab_size}) must be divisible by world_size ({world_size})")
        self.vocab_size = vocab_size
        self.embedding_dim = embedding_dim
        self.world_size = world_size
        self.rank = rank
        self.communicator = communicator
        self.local_vocab_size = vocab_size // world_size
        self.vocab_start = rank * self.local_vocab_size
        self.vocab_end = self.vocab_start + self.local_vocab_size
        self.weight: Optional[torch.Tensor] = None

    def load_shard(self, full_weight):
        w = full_weight[self.vocab_start:self.vocab_end]
        self.load_shard_direct(w)

    def load_shard_direct(self, weight_shard):
        if tuple(weight_shard.shape) != (self.local_vocab_size, self.embedding_dim):
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected "
                             f"{(self.local_vocab_size, self.embedding_dim)}")
        self.weight = as_device(weight_shard, torch.float16)

    def forward_local(self, input_ids: torch.Tensor) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("Embedding weights not loaded")
        return ops.embed_gather_f16(input_ids.to(self.weight.device), self.weight, self.vocab_start, self.vocab_end)

    async def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        emb = self.forward_local(input_ids)
        if self.communicator is not None:
            emb = await self.communicator.all_reduce(emb, op="sum")
        return emb

    @property
    def num_parameters(self) -> int:
        return self.local_vocab_size * self.embedding_dim


class ParallelEmbedding:
    """Unquantized table split on the hidden dimension (each rank holds
    ``dim / world`` columns of every row); slices are all-gathered."""

    def __init__(self, vocab_size: int, embedding_dim: int, world_size: int, rank: int, communicator=None,
                 gather_output: bool = True, padding_idx: Optional[int] = None):
        if embedding_dim % world_size != 0:
            raise ValueError(f"embedding_dim ({embedding_dim}) must be divisible by world_size ({world_size})")
        self.vocab_size = vocab_size
        self.embedding_dim = embedding_dim
        self.world_size = world_size
        self.rank = rank
        self.gather_output = gather_output
        self.communicator = communicator
        self.padding_idx = padding_idx
        self.local_embedding_dim = embedding_dim // world_size
        self.col_start = rank * self.local_embedding_dim
        self.col_end = self.col_start + self.local_embedding_dim
        self.weight: Optional[torch.Tensor] = None

    def load_shard(self, full_weight):
        self.load_shard_direct(full_weight[:, self.col_start:self.col_end])

    def load_shard_direct(self, weight_shard):
        if weight_shard is None:
            logger.warning("load_shard_direct called with None weight, skipping")
            return
        if tuple(weight_shard.shape) != (self.vocab_size, self.local_embedding_dim):
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected "
                             f"{(self.vocab_size, self.local_embedding_dim)}")
        self.weight = as_device(weight_shard, torch.float16)

    def forward_sync(self, input_ids: torch.Tensor) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("Weight not loaded")
        # every id is in range on every rank (the split is on the hidden dim)
        return ops.embed_gather_f16(input_ids.to(self.weight.device), self.weight, 0, self.vocab_size)

    async def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        emb = self.forward_sync(input_ids)
        if self.gather_output:
            if self.communicator is None:
                raise RuntimeError("Communicator required for gather_output=True")
            emb = await self.communicator.all_gather(emb, dim=-1)
        return emb

    @property
    def num_parameters(self) -> int:
        return self.vocab_size * self.local_embedding_dim
