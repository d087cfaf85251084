"""Unquantized tensor-parallel linears (reference ``parallel/column_linear.py``,
``parallel/row_linear.py``).

Weights are kept in the reference's ``[in, out]`` orientation (column shard
``[in, out/TP]``, row shard ``[in/TP, out]``) as fp16 CUDA tensors, and the
product is a plain cuBLAS GEMM (``torch.matmul`` on the device) -- these
layers carry unquantized checkpoints and are not part of the quantized decode
path, whose linears are ``QuantizedColumnParallelLinear`` /
``QuantizedRowParallelLinear``.
"""

from __future__ import annotations

import logging
from typing import Optional

import torch

from ._tensors import as_device

logger = logging.getLogger(__name__)


class ColumnParallelLinear:
    """parallel/column_linear.py:12-207."""

    def __init__(self, in_features: int, out_features: int, world_size: int, rank: int, bias: bool = True,
                 gather_output: bool = False, communicator=None):
        if out_features % world_size != 0:
            raise ValueError(f"out_features ({out_features}) must be divisible by world_size ({world_size})")
        self.in_features = in_features
        self.out_features = out_features
        self.world_size = world_size
        self.rank = rank
        self.gather_output = gather_output
        self.communicator = communicator
        self.local_out_features = out_features // world_size
        self.col_start = rank * self.local_out_features
        self.col_end = self.col_start + self.local_out_features
        self.weight: Optional[torch.Tensor] = None
        self.bias: Optional[torch.Tensor] = None
        self.has_bias = bias

    def load_shard(self, full_weight, full_bias=None):
        self.weight = as_device(full_weight[:, self.col_start:self.col_end], torch.float16)
        if self.has_bias and full_bias is not None:
            self.bias = as_device(full_bias[self.col_start:self.col_end], torch.float16)

    def load_shard_direct(self, weight_shard, bias_shard=None):
        if weight_shard is None:
            logger.warning("load_shard_direct called with None weight, skipping")
            return
        expected = (self.in_features, self.local_out_features)
        if tuple(weight_shard.shape) != expected:
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected {expected}")
        self.weight = as_device(weight_shard, torch.float16)
        if self.has_bias and bias_shard is not None:
            self.bias = as_device(bias_shard, torch.float16)

    def forward_sync(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("Weight not loaded. Call load_shard() or load_shard_direct() first.")
        y = torch.matmul(x.to(self.weight.dtype), self.weight)
        if self.has_bias and self.bias is not None:
            y = y + self.bias
        return y

    async def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.forward_sync(x)
        if self.gather_output:
            if self.communicator is None:
                raise RuntimeError("Communicator required for gather_output=True")
            y = await self.communicator.all_gather(y, dim=-1)
        return y

    @property
    def num_parameters(self) -> int:
        return self.in_features * self.local_out_features + (self.local_out_features if self.has_bias else 0)


class RowParallelLinear:
    """parallel/row_linear.py:12-217: K-split partial product, all-reduce,
    bias once on rank 0."""

    def __init__(self, in_features: int, out_features: int, world_size: int, rank: int, bias: bool = True,
                 input_is_partitioned: bool = True, communicator=None):
        if in_features % world_size != 0:
            raise ValueError(f"in_features ({in_features}) must be divisible by world_size ({world_size})")
        self.in_features = in_features
        self.out_features = out_features
        self.world_size = world_size
        self.rank = rank
        self.input_is_partitioned = input_is_partitioned
        self.communicator = communicator
        self.local_in_features = in_features // world_size
        self.row_start = rank * self.local_in_features
        self.row_end = self.row_start + self.local_in_features
        self.weight: Optional[torch.Tensor] = None
        self.bias: Optional[torch.Tensor] = None
        self.has_bias = bias

    def load_shard(self, full_weight, full_bias=None):
        self.weight = as_device(full_weight[self.row_start:self.row_end, :], torch.float16)
        if self.has_bias and full_bias is not None and self.rank == 0:
            self.bias = as_device(full_bias, torch.float16)

    def load_shard_direct(self, weight_shard, bias_shard=None):
        if weight_shard is None:
            logger.warning("load_shard_direct called with None weight, skipping")
            return
        expected = (self.local_in_features, self.out_features)
        if tuple(weight_shard.shape) != expected:
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected {expected}")
        self.weight = as_device(weight_shard, torch.float16)
        if self.has_bias and bias_shard is not None and self.rank == 0:
            self.bias = as_device(bias_shard, torch.float16)

    def forward_partial(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight is None:
            raise RuntimeError("Weight not loaded")
        if not self.input_is_partitioned:
            x = x[..., self.row_start:self.row_end]
        return torch.matmul(x.to(self.weight.dtype), self.weight)

    def add_bias(self, x: torch.Tensor) -> torch.Tensor:
        if self.has_bias and self.bias is not None and self.rank == 0:
            return x + self.bias.to(x.dtype)
        return x

    async def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.forward_partial(x)
        if self.communicator is not None and self.world_size > 1:
            y = await self.communicator.all_reduce(y, op="sum")
        return self.add_bias(y)

    @property
    def num_parameters(self) -> int:
        return self.local_in_features * self.out_features + (self.out_features if self.has_bias and self.rank == 0
                                                             else 0)
