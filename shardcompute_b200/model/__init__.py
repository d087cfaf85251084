"""Model config, shard layout and loading (reference ``model/``)."""

from .config import ModelConfig, ParallelConfig, QuantizationConfig
from .sharder import WeightSharder

__all__ = ["ModelConfig", "ParallelConfig", "QuantizationConfig", "WeightSharder"]
