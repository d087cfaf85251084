"""Tensor-parallel gated MLP (reference ``parallel/mlp.py:18-280``).

Quantized Llama path: gate and up are column-parallel, down is
row-parallel with one all-reduce.  The gate and up GEMVs run as ONE kernel
launch over both weight sets whose epilogue writes ``silu(gate) * up`` in
fp16 -- the activation never round-trips through HBM in fp32 -- and the down
GEMV follows.  Unquantized and non-gated configurations use the dense
layers and an elementwise activation on the device.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _lib as L
from .. import ops
from .linear import ColumnParallelLinear, RowParallelLinear
from .quantized_linear import QuantizedColumnParallelLinear, QuantizedRowParallelLinear


def _activation(name: str):
    if name in ("silu", "swish"):
        return lambda x: x * torch.sigmoid(x)
    if name == "gelu":
        return lambda x: x * torch.sigmoid(1.702 * x)
    if name == "gelu_new":
        return lambda x: 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))
    if name == "relu":
        return lambda x: torch.clamp_min(x, 0)
    if name == "gelu_exact":
        return lambda x: 0.5 * x * (1 + torch.erf(x / math.sqrt(2)))
    raise ValueError(f"Unknown activation: {name}")


class ParallelMLP:
    def __init__(self, hidden_size: int, intermediate_size: int, world_size: int, rank: int, communicator,
                 activation: str = "silu", bias: bool = False, use_gated: bool = True, use_quantized: bool = False,
                 quantization_bits: int = 4, quantization_group_size: int = 64):
        if intermediate_size % world_size != 0:
            raise ValueError(f"intermediate_size ({intermediate_size}) must be divisible by world_size")
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.world_size = world_size
        self.rank = rank
        self.communicator = communicator
        self.use_gated = use_gated
        self.use_quantized = use_quantized
        self.bits = quantization_bits
        self.group_size = quantization_group_size
        self.local_intermediate = intermediate_size // world_size
        self.activation_name = activation
        self.activation = _activation(activation)
        if use_quantized:
            col = lambda: QuantizedColumnParallelLinear(hidden_size, intermediate_size, world_size, rank,  # noqa
                                                        bias=bias, group_size=quantization_group_size,
                                                        bits=quantization_bits)
            self.up_proj = col()
            self.gate_proj = col() if use_gated else None
            self.down_proj = QuantizedRowParallelLinear(intermediate_size, hidden_size, world_size, rank, bias=bias,
                                                        input_is_partitioned=True, communicator=communicator,
                                                        group_size=quantization_group_size, bits=quantization_bits)
        else:
            col = lambda: ColumnParallelLinear(hidden_size, intermediate_size, world_size, rank, bias=bias)  # noqa
            self.up_proj = col()
            self.gate_proj = col() if use_gated else None
            self.down_proj = RowParallelLinear(intermediate_size, hidden_size, world_size, rank, bias=bias,
                                               input_is_partitioned=True, communicator=communicator)

    def load_shards(self, up_weight, up_bias, down_weight, down_bias, gate_weight=None, gate_bias=None):
        self.up_proj.load_shard_direct(up_weight, up_bias)
        self.down_proj.load_shard_direct(down_weight, down_bias)
        if self.use_gated and gate_weight is not None:
            self.gate_proj.load_shard_direct(gate_weight, gate_bias)

    def load_quantized_shards(self, up, down, gate=None):
        """Each argument is a ``(weight, scales, biases)`` triple."""
        self.up_proj.load_quantized_shard(*up)
        self.down_proj.load_quantized_shard(*down)
        if self.use_gated and gate is not None:
            self.gate_proj.load_quantized_shard(*gate)

    def _fused_ok(self) -> bool:
        return (self.use_quantized and self.use_gated and self.activation_name in ("silu", "swish")
                and self.gate_proj.bias is None and self.up_proj.bias is None)

    def intermediate(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """``act(gate(x)) * up(x)`` (or ``act(up(x))``) for this rank's slice."""
        if self._fused_ok():
            g, u = self.gate_proj, self.up_proj
            if g.quantized_weight is None or u.quantized_weight is None:
                raise RuntimeError("Weight not loaded")
            shp = hidden_states.shape
            y = ops.qlinear_fused(hidden_states.reshape(-1, shp[-1]),
                                  [(g.quantized_weight, g.scales, g.biases_quant),
                                   (u.quantized_weight, u.scales, u.biases_quant)],
                                  self.group_size, self.bits, epilogue=L.SC_EPI_SWIGLU, out_dtype=torch.float16)
            return y.view(*shp[:-1], self.local_intermediate)
        up = self.up_proj.forward_sync(hidden_states)
        if self.use_gated:
            return (self.activation(self.gate_proj.forward_sync(hidden_states).float()) * up.float()).to(up.dtype)
        return self.activation(up.float()).to(up.dtype)

    def forward_sync_partial(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """This rank's down-projection partial (no all-reduce, no bias)."""
        return self.down_proj.forward_partial(self.intermediate(hidden_states))

    async def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return await self.down_proj.forward(self.intermediate(hidden_states))

    @property
    def num_parameters(self) -> int:
        n = self.up_proj.num_parameters + self.down_proj.num_parameters
        return n + (self.gate_proj.num_parameters if self.gate_proj is not None else 0)
