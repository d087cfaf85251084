"""Model config, shard layout and loading (reference ``model/``)."""

from .config import ModelConfig, ParallelConfig, QuantizationConfig
from .loader import load_rank_shard, load_safetensors
from .sharder import WeightSharder

__all__ = ["ModelConfig", "ParallelConfig", "QuantizationConfig", "WeightSharder", "load_rank_shard",
           "load_safetensors"]
