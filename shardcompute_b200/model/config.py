"""Model / parallel / quantization config, field-compatible with the reference.

Mirrors ``model/config.py`` of the reference: ``ModelConfig`` (:9-106),
``ParallelConfig`` (:109-223, tensor mode only is in scope here),
``QuantizationConfig`` (:268-308).  ``from_dict`` accepts the HF key names the
reference accepts, and ``to_dict`` writes the same keys, so a shard
directory's ``config.json`` reads the same in both.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Optional
import json


@dataclass
class QuantizationConfig:
    enabled: bool = False
    bits: int = 4
    group_size: int = 64
    quantize_attention: bool = True
    quantize_mlp: bool = True
    quantize_embeddings: bool = False
    quantize_lm_head: bool = False

    @classmethod
    def from_dict(cls, data: Optional[Dict[str, Any]]) -> "QuantizationConfig":
        if not data:
            return cls(enabled=False)
        return cls(enabled=True, bits=data.get("bits", 4), group_size=data.get("group_size", 64),
                   quantize_attention=data.get("quantize_attention", True),
                   quantize_mlp=data.get("quantize_mlp", True),
                   quantize_embeddings=data.get("quantize_embeddings", False),
                   quantize_lm_head=data.get("quantize_lm_head", False))

    def to_dict(self) -> Dict[str, Any]:
        return {"enabled": self.enabled, "bits": self.bits, "group_size": self.group_size,
                "quantize_attention": self.quantize_attention, "quantize_mlp": self.quantize_mlp,
                "quantize_embeddings": self.quantize_embeddings, "quantize_lm_head": self.quantize_lm_head}


@dataclass
class ModelConfig:
    vocab_size: int = 32000
    hidden_size: int = 2048
    num_layers: int = 22
    num_heads: int = 32
    num_kv_heads: Optional[int] = None
    intermediate_size: int = 5632
    max_position_embeddings: int = 2048
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    tie_word_embeddings: bool = False
    hidden_act: str = "silu"
    use_gated_mlp: bool = True
    model_type: str = "llama"
    quantization: Optional[QuantizationConfig] = None

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "ModelConfig":
        model_type = data.get("model_type", "llama")
        act, gated = ("gelu_new", False) if model_type == "phi" else ("silu", True)
        q = data.get("quantization")
        return cls(vocab_size=data.get("vocab_size", 32000), hidden_size=data.get("hidden_size", 2048),
                   num_layers=data.get("num_hidden_layers", data.get("num_layers", 22)),
                   num_heads=data.get("num_attention_heads", data.get("num_heads", 32)),
                   num_kv_heads=data.get("num_key_value_heads"),
                   intermediate_size=data.get("intermediate_size", 5632),
                   max_position_embeddings=data.get("max_position_embeddings", 2048),
                   rms_norm_eps=data.get("rms_norm_eps", 1e-5), rope_theta=data.get("rope_theta", 10000.0),
                   tie_word_embeddings=data.get("tie_word_embeddings", False),
                   hidden_act=data.get("hidden_act", act), use_gated_mlp=data.get("use_gated_mlp", gated),
                   model_type=model_type, quantization=QuantizationConfig.from_dict(q) if q else None)

    @classmethod
    def from_pretrained(cls, model_path: str) -> "ModelConfig":
        p = Path(model_path) / "config.json"
        if not p.exists():
            raise FileNotFoundError(f"Config not found at {p}")
        with open(p) as f:
            return cls.from_dict(json.load(f))

    def to_dict(self) -> Dict[str, Any]:
        d = {"vocab_size": self.vocab_size, "hidden_size": self.hidden_size, "num_hidden_layers": self.num_layers,
             "num_attention_heads": self.num_heads, "num_key_value_heads": self.num_kv_heads,
             "intermediate_size": self.intermediate_size, "max_position_embeddings": self.max_position_embeddings,
             "rms_norm_eps": self.rms_norm_eps, "rope_theta": self.rope_theta,
             "tie_word_embeddings": self.tie_word_embeddings, "hidden_act": self.hidden_act,
             "use_gated_mlp": self.use_gated_mlp, "model_type": self.model_type}
        if self.quantization:
            d["quantization"] = self.quantization.to_dict()
        return d

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads or self.num_heads


@dataclass
class ParallelConfig:
    world_size: int = 2
    rank: int = 0
    mode: str = "tensor"
    tensor_parallel_size: int = 2
    pipeline_parallel_size: int = 2
    row_parallel_size: int = 1
    col_parallel_size: int = 1

    @classmethod
    def from_dict(cls, data: Dict[str, Any], rank: int = 0) -> "ParallelConfig":
        mode = data.get("mode", "tensor")
        tp = data.get("tensor_parallel_size", 2)
        pp = data.get("pipeline_parallel_size", 2)
        return cls(world_size=pp if mode == "pipeline" else tp, rank=rank, mode=mode, tensor_parallel_size=tp,
                   pipeline_parallel_size=pp, row_parallel_size=data.get("row_parallel_size", 1),
                   col_parallel_size=data.get("col_parallel_size", 1))

    def validate(self, model_config: ModelConfig) -> None:
        """Tensor-mode divisibility rules (model/config.py:156-185)."""
        if self.mode != "tensor":
            raise NotImplementedError("only tensor parallelism is implemented for the B200 decode path")
        tp = self.tensor_parallel_size
        for name, val in (("num_heads", model_config.num_heads), ("hidden_size", model_config.hidden_size),
                          ("intermediate_size", model_config.intermediate_size)):
            if val % tp:
                raise ValueError(f"{name} ({val}) must be divisible by tensor_parallel_size ({tp})")
        if model_config.num_kv_heads and model_config.num_kv_heads % tp:
            raise ValueError(f"num_kv_heads ({model_config.num_kv_heads}) must be divisible by "
                             f"tensor_parallel_size ({tp})")

    @property
    def is_tensor(self) -> bool:
        return self.mode == "tensor"
