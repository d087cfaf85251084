"""Seeded synthetic quantized Llama checkpoints (test infrastructure only).

Builds the full (unsharded) tensor dictionary in the layout the reference's
``scripts/shard_weights.py`` consumes from an MLX-quantized checkpoint: HF
tensor names, every linear and the tied embedding as ``.weight`` (uint32
packed) / ``.scales`` / ``.biases`` (fp16) triples, norms as fp16 vectors.
Weights are ``N(0, std)`` rounded to fp16 and quantized by
``oracle.mlx_affine.quantize``; norms are 1 + small noise so that the norm
multiply is exercised.
"""

from __future__ import annotations

import numpy as np

from . import mlx_affine as qa
from .tp import LlamaShape


def tiny_shape(**kw) -> LlamaShape:
    """A small Llama whose GEMVs still take the TMA kernel path
    (K/g a multiple of 8, K*bits/32 a multiple of 32)."""
    base = dict(vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=4,
                intermediate_size=1024, rms_norm_eps=1e-5, rope_theta=10000.0, bits=4, group_size=64)
    base.update(kw)
    return LlamaShape(**base)


def checkpoint(cfg: LlamaShape, seed: int = 0, std: float = 0.02) -> dict:
    rng = np.random.Generator(np.random.PCG64(seed))
    H, F, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    out = {}

    def q(name: str, rows: int, cols: int):
        w = (rng.standard_normal((rows, cols)) * std).astype(np.float16)
        wq, s, b = qa.quantize(w, cfg.group_size, cfg.bits)
        out[f"{name}.weight"], out[f"{name}.scales"], out[f"{name}.biases"] = wq, s, b

    def norm(name: str):
        out[name] = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float16)

    q("model.embed_tokens", cfg.vocab_size, H)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}"
        norm(f"{p}.input_layernorm.weight")
        norm(f"{p}.post_attention_layernorm.weight")
        q(f"{p}.self_attn.q_proj", cfg.num_heads * hd, H)
        q(f"{p}.self_attn.k_proj", cfg.num_kv_heads * hd, H)
        q(f"{p}.self_attn.v_proj", cfg.num_kv_heads * hd, H)
        q(f"{p}.self_attn.o_proj", H, cfg.num_heads * hd)
        q(f"{p}.mlp.gate_proj", F, H)
        q(f"{p}.mlp.up_proj", F, H)
        q(f"{p}.mlp.down_proj", H, F)
    norm("model.norm.weight")
    return out


def model_config_dict(cfg: LlamaShape) -> dict:
    """The ``config.json["model"]`` block the reference writes for this shape."""
    return {"vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_layers,
            "num_attention_heads": cfg.num_heads, "num_key_value_heads": cfg.num_kv_heads,
            "intermediate_size": cfg.intermediate_size, "max_position_embeddings": 4096,
            "rms_norm_eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta, "tie_word_embeddings": True,
            "quantization": {"enabled": True, "bits": cfg.bits, "group_size": cfg.group_size}}
