"""Tensor-parallel layers with the reference's ``parallel/`` API, on the
sm_100a kernels of ``libsc_b200.so``, plus the fused decode engine."""

from .attention import KVCache, ParallelAttention, RoPE
from .decode_engine import DecodeEngine
from .embedding import ParallelEmbedding, QuantizedParallelEmbedding, VocabParallelEmbedding
from .linear import ColumnParallelLinear, RowParallelLinear
from .mlp import ParallelMLP
from .quantized_linear import QuantizedColumnParallelLinear, QuantizedRowParallelLinear
from .transformer import ParallelTransformer, ParallelTransformerBlock, RMSNorm
from .weights import LayerWeights, RankWeights

__all__ = ["KVCache", "ParallelAttention", "RoPE", "DecodeEngine", "ParallelEmbedding", "QuantizedParallelEmbedding",
           "VocabParallelEmbedding", "ColumnParallelLinear", "RowParallelLinear", "ParallelMLP",
           "QuantizedColumnParallelLinear", "QuantizedRowParallelLinear", "ParallelTransformer",
           "ParallelTransformerBlock", "RMSNorm", "LayerWeights", "RankWeights"]
