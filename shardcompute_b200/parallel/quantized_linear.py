"""Quantized tensor-parallel linears (reference ``parallel/quantized_linear.py``).

Same constructor arguments, attributes, loading methods, sync/async forward
split and error behaviour as the reference classes; the weights stay in the
MLX affine layout (``uint32`` packed codes + fp16 scales/biases, output rows
first) and every product runs through ``sc_qlinear`` on the GPU.  Tensors are
torch CUDA tensors where the reference takes ``mx.array``.
"""

from __future__ import annotations

import logging
from typing import Optional

import torch

from .. import ops
from ._tensors import as_device, as_words

logger = logging.getLogger(__name__)


def _qmatmul(x: torch.Tensor, w, s, b, group: int, bits: int) -> torch.Tensor:
    """``mx.quantized_matmul(x, w, s, b, transpose=True)``: fp32 output for
    fp32 input, fp16 for fp16 (the input's dtype, as MLX returns)."""
    return ops.qlinear(x, w, s, b, group, bits, out_dtype=x.dtype if x.dtype == torch.float32 else torch.float16)


class QuantizedColumnParallelLinear:
    """Column-parallel linear (output features split), quantized weights.

    Reference: parallel/quantized_linear.py:17-251.  Local weight: packed
    ``[out_features / world, in_features * bits / 32]`` with scales/biases
    ``[out_features / world, in_features / group]``.
    """

    def __init__(self, in_features: int, out_features: int, world_size: int, rank: int, bias: bool = True,
                 gather_output: bool = False, communicator=None, group_size: int = 64, bits: int = 4):
        if out_features % world_size != 0:
            raise ValueError(f"out_features ({out_features}) must be divisible by world_size ({world_size})")
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self.in_features = in_features
        self.out_features = out_features
        self.world_size = world_size
        self.rank = rank
        self.gather_output = gather_output
        self.communicator = communicator
        self.group_size = group_size
        self.bits = bits
        self.local_out_features = out_features // world_size
        self.col_start = rank * self.local_out_features
        self.col_end = self.col_start + self.local_out_features
        self.quantized_weight: Optional[torch.Tensor] = None
        self.scales: Optional[torch.Tensor] = None
        self.biases_quant: Optional[torch.Tensor] = None
        self.bias: Optional[torch.Tensor] = None
        self.has_bias = bias

    def load_shard_and_quantize(self, weight_shard: torch.Tensor, bias_shard: Optional[torch.Tensor] = None):
        """Quantize a full-precision shard on the GPU (``sc_quantize``).

        The shard is taken in the output-rows-first layout ``[local_out,
        in_features]`` the kernels read (the reference's ``[in, local_out]``
        argument is quantized along its last axis and then applied with
        ``transpose=True``, which only lines up for square shards).
        """
        expected = (self.local_out_features, self.in_features)
        if tuple(weight_shard.shape) != expected:
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected {expected}")
        w = as_device(weight_shard, torch.float16)
        self.quantized_weight, self.scales, self.biases_quant = ops.quantize(w, self.group_size, self.bits)
        if self.has_bias and bias_shard is not None:
            self.bias = as_device(bias_shard, torch.float16)

    def load_quantized_shard(self, quantized_weight, scales, biases, linear_bias=None):
        """Load a pre-quantized shard (parallel/quantized_linear.py:127-150)."""
        qw = as_words(quantized_weight)
        sc = as_device(scales, torch.float16)
        bi = as_device(biases, torch.float16)
        if qw.shape[0] != self.local_out_features or qw.shape[1] * (32 // self.bits) != self.in_features:
            raise ValueError(f"quantized weight {tuple(qw.shape)} does not pack [{self.local_out_features}, "
                             f"{self.in_features}] at {self.bits} bits")
        self.quantized_weight, self.scales, self.biases_quant = qw, sc, bi
        if self.has_bias and linear_bias is not None:
            self.bias = as_device(linear_bias, torch.float16)

    def _matmul(self, x: torch.Tensor) -> torch.Tensor:
        if self.quantized_weight is None:
            raise RuntimeError("Weight not loaded. Call load_shard_and_quantize() first.")
        y = _qmatmul(x, self.quantized_weight, self.scales, self.biases_quant, self.group_size, self.bits)
        if self.has_bias and self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y

    async def forward(self, x: torch.Tensor) -> torch.Tensor:
        """``[..., in]`` -> ``[..., local_out]`` (or all-gathered ``[..., out]``)."""
        y = self._matmul(x)
        if self.gather_output:
            if self.communicator is None:
                raise RuntimeError("Communicator required for gather_output=True")
            y = await self.communicator.all_gather(y, dim=-1)
        return y

    def forward_sync(self, x: torch.Tensor) -> torch.Tensor:
        if self.quantized_weight is None:
            raise RuntimeError("Weight not loaded")
        return self._matmul(x)

    @property
    def num_parameters(self) -> int:
        return self.in_features * self.local_out_features + (self.local_out_features if self.has_bias else 0)

    @property
    def memory_bytes(self) -> int:
        if self.quantized_weight is None:
            return 0
        n = sum(t.numel() * t.element_size() for t in (self.quantized_weight, self.scales, self.biases_quant))
        return n + (self.bias.numel() * self.bias.element_size() if self.bias is not None else 0)

    def __repr__(self) -> str:
        return (f"QuantizedColumnParallelLinear(in_features={self.in_features}, out_features={self.out_features}, "
                f"local_out_features={self.local_out_features}, rank={self.rank}/{self.world_size}, "
                f"bits={self.bits})")


class QuantizedRowParallelLinear:
    """Row-parallel linear (input features split), quantized weights.

    Reference: parallel/quantized_linear.py:254-518.  Local weight: packed
    ``[out_features, in_features / world * bits / 32]``; scales/biases
    ``[out_features, in_features / world / group]`` (full-K scales are sliced
    to this rank on load, :385-414).  The linear bias lives on rank 0 only and
    is added after the all-reduce (:359-361, :416-417, :451-453).
    """

    def __init__(self, in_features: int, out_features: int, world_size: int, rank: int, bias: bool = True,
                 input_is_partitioned: bool = True, communicator=None, group_size: int = 64, bits: int = 4):
        if in_features % world_size != 0:
            raise ValueError(f"in_features ({in_features}) must be divisible by world_size ({world_size})")
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self.in_features = in_features
        self.out_features = out_features
        self.world_size = world_size
        self.rank = rank
        self.input_is_partitioned = input_is_partitioned
        self.communicator = communicator
        self.group_size = group_size
        self.bits = bits
        self.local_in_features = in_features // world_size
        self.row_start = rank * self.local_in_features
        self.row_end = self.row_start + self.local_in_features
        self.quantized_weight: Optional[torch.Tensor] = None
        self.scales: Optional[torch.Tensor] = None
        self.biases_quant: Optional[torch.Tensor] = None
        self.bias: Optional[torch.Tensor] = None
        self.has_bias = bias

    def load_shard_and_quantize(self, weight_shard: torch.Tensor, bias_shard: Optional[torch.Tensor] = None):
        """Quantize ``[out_features, local_in]`` on the GPU; bias kept on rank 0 only."""
        expected = (self.out_features, self.local_in_features)
        if tuple(weight_shard.shape) != expected:
            raise ValueError(f"Weight shard shape {tuple(weight_shard.shape)} doesn't match expected {expected}")
        w = as_device(weight_shard, torch.float16)
        self.quantized_weight, self.scales, self.biases_quant = ops.quantize(w, self.group_size, self.bits)
        if self.has_bias and bias_shard is not None and self.rank == 0:
            self.bias = as_device(bias_shard, torch.float16)

    def load_quantized_shard(self, quantized_weight, scales, biases, linear_bias=None):
        qw = as_words(quantized_weight)
        sc = as_device(scales, torch.float16)
        bi = as_device(biases, torch.float16)
        if qw.shape[0] == self.out_features and sc.dim() == 2:
            local_k = qw.shape[1] * (32 // self.bits)
            if local_k % self.group_size == 0:
                expected = local_k // self.group_size
                full = sc.shape[1]
                if full == expected * self.world_size and self.world_size > 1:
                    sl = slice(self.rank * expected, (self.rank + 1) * expected)
                    sc = sc[:, sl].contiguous()
                    if bi.dim() == 2:
                        bi = bi[:, sl].contiguous()
                elif full != expected:
                    logger.warning("row-parallel shard: %d scale columns fit neither this rank's %d groups nor the "
                                   "full-K count; using the scales and biases as given", full, expected)
            else:
                logger.warning("row-parallel shard: local K=%d is not a whole number of %d-wide groups; "
                               "using the scales and biases as given", local_k, self.group_size)
        self.quantized_weight, self.scales, self.biases_quant = qw, sc, bi
        if self.has_bias and linear_bias is not None and self.rank == 0:
            self.bias = as_device(linear_bias, torch.float16)

    def forward_partial(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's partial product (no all-reduce, no bias)."""
        if self.quantized_weight is None:
            raise RuntimeError("Weight not loaded")
        return _qmatmul(x, self.quantized_weight, self.scales, self.biases_quant, self.group_size, self.bits)

    def add_bias(self, x: torch.Tensor) -> torch.Tensor:
        if self.has_bias and self.bias is not None and self.rank == 0:
            return x + self.bias.to(x.dtype)
        return x

    async def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.forward_partial(x)
        if self.communicator is not None:
            y = await self.communicator.all_reduce(y, op="sum")
        if self.has_bias and self.bias is not None and self.rank == 0:
            y = y + self.bias.to(y.dtype)
        return y

    @property
    def num_parameters(self) -> int:
        return self.local_in_features * self.out_features + (self.out_features if self.has_bias and self.rank == 0
                                                             else 0)

    @property
    def memory_bytes(self) -> int:
        if self.quantized_weight is None:
            return 0
        n = sum(t.numel() * t.element_size() for t in (self.quantized_weight, self.scales, self.biases_quant))
        return n + (self.bias.numel() * self.bias.element_size() if self.bias is not None else 0)

    def __repr__(self) -> str:
        return (f"QuantizedRowParallelLinear(in_features={self.in_features}, out_features={self.out_features}, "
                f"local_in_features={self.local_in_features}, rank={self.rank}/{self.world_size}, "
                f"bits={self.bits})")
