"""Tensor-parallel quantized Llama decode, restated in numpy (test oracle only).

All ranks run in one process and collectives are simulated the way the
reference's tests do it (sum of per-rank partials for all-reduce, rank-order
concatenation for all-gather).  Compute is float64 except where the reference
defines a step in another precision (fp16 dequantize, fp32 RoPE tables).

Op-for-op sources (reference paths):

* RMSNorm                 parallel/transformer.py:46-61
* block / residuals       parallel/transformer.py:214-254
* model forward, tied head parallel/transformer.py:516-577
* attention               parallel/attention.py:381-471 (RoPE :19-151)
* MLP (SwiGLU)            parallel/mlp.py:228-254 (silu = x*sigmoid(x), :161-162)
* quantized linears       parallel/quantized_linear.py:152-219, 419-486
* vocab-split embedding   parallel/embedding.py:309-379
* greedy step             worker/executor.py:267-325 (argmax :276-278)
* all-reduce / all-gather collectives/all_reduce.py:58-193, all_gather.py:54-162
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import mlx_affine as qa


@dataclass
class LlamaShape:
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    intermediate_size: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    bits: int = 4
    group_size: int = 64

    @property
    def head_dim(self) -> int:
        # model/config.py:103-106: head_dim = hidden / heads
        return self.hidden_size // self.num_heads


# ---------------------------------------------------------------- elementwise

def rmsnorm(x, w, eps):
    """RMSNorm.__call__ (parallel/transformer.py:46-61)."""
    x = np.asarray(x, dtype=np.float64)
    rms = np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return (x / rms) * np.asarray(w, dtype=np.float64)


def silu(x):
    return x / (1.0 + np.exp(-x))


def rope_tables(head_dim: int, length: int, base: float):
    """RoPE cos/sin tables (parallel/attention.py:56-59,66-92) in fp32.

    Returns ``[length, head_dim//2]`` halves; the reference concatenates the
    half with itself, so element d and d+head_dim/2 share an angle.
    """
    inv_freq = (np.float32(1.0) / (np.float32(base) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                                         / np.float32(head_dim)))).astype(np.float32)
    t = np.arange(length, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def apply_rope(x, cos_h, sin_h):
    """RoPE._rotate (parallel/attention.py:130-151): x*cos + [-x2, x1]*sin.

    ``x`` is ``[..., S, hd]``; ``cos_h``/``sin_h`` are ``[S, hd/2]``.
    """
    x = np.asarray(x, dtype=np.float64)
    hd = x.shape[-1]
    cos = np.concatenate([cos_h, cos_h], axis=-1).astype(np.float64)
    sin = np.concatenate([sin_h, sin_h], axis=-1).astype(np.float64)
    x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
    rot = np.concatenate([-x2, x1], axis=-1)
    return x * cos + rot * sin


def softmax(s, axis=-1):
    m = np.max(s, axis=axis, keepdims=True)
    e = np.exp(s - m)
    return e / np.sum(e, axis=axis, keepdims=True)


# ---------------------------------------------------------------- collectives

def all_reduce_sum(parts):
    """Simulated all-reduce: rank-order sum (collectives/all_reduce.py:90-110)."""
    out = np.array(parts[0], dtype=np.float64, copy=True)
    for p in parts[1:]:
        out = out + p
    return out


def all_gather(parts, dim=-1):
    """Simulated all-gather: rank-order concat (collectives/all_gather.py:90-162)."""
    return np.concatenate(parts, axis=dim)


# ---------------------------------------------------------------- layers

def qlinear(x, shard: dict, prefix: str, cfg: LlamaShape, bias=None):
    """Quantized{Column,Row}ParallelLinear.forward_sync / forward_partial."""
    y = qa.quantized_matmul(x, shard[f"{prefix}.weight"], shard[f"{prefix}.scales"],
                            shard[f"{prefix}.biases"], cfg.group_size, cfg.bits)
    if bias is not None:
        y = y + bias
    return y


def embed_rank(ids, shard: dict, cfg: LlamaShape, world: int, rank: int):
    """QuantizedParallelEmbedding.forward before its all-reduce (embedding.py:322-356)."""
    local_v = cfg.vocab_size // world
    v0, v1 = rank * local_v, (rank + 1) * local_v
    ids = np.asarray(ids)
    in_range = (ids >= v0) & (ids < v1)
    local = np.clip(ids - v0, 0, local_v - 1).reshape(-1)
    w = shard["model.embed_tokens.weight"][local]
    s = shard["model.embed_tokens.scales"][local]
    b = shard["model.embed_tokens.biases"][local]
    e = qa.dequantize(w, s, b, cfg.group_size, cfg.bits).reshape(*ids.shape, cfg.hidden_size)
    return np.where(in_range[..., None], e, np.float16(0))


def attention_rank(h, shard, layer: int, cfg: LlamaShape, world: int, past, cos_t, sin_t):
    """ParallelAttention.forward up to o_proj's partial (attention.py:403-467)."""
    B, S, _ = h.shape
    hd = cfg.head_dim
    nh, nkv = cfg.num_heads // world, cfg.num_kv_heads // world
    p = f"model.layers.{layer}.self_attn"
    q = qlinear(h, shard, f"{p}.q_proj", cfg).reshape(B, S, nh, hd).transpose(0, 2, 1, 3)
    k = qlinear(h, shard, f"{p}.k_proj", cfg).reshape(B, S, nkv, hd).transpose(0, 2, 1, 3)
    v = qlinear(h, shard, f"{p}.v_proj", cfg).reshape(B, S, nkv, hd).transpose(0, 2, 1, 3)
    off = 0 if past is None else past[0].shape[2]
    q = apply_rope(q, cos_t[off:off + S], sin_t[off:off + S])
    k = apply_rope(k, cos_t[off:off + S], sin_t[off:off + S])
    if past is not None:
        k = np.concatenate([past[0], k], axis=2)
        v = np.concatenate([past[1], v], axis=2)
    cache = (k, v)
    L = k.shape[2]
    rep = nh // nkv
    kk = np.repeat(k, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    scores = (q @ kk.transpose(0, 1, 3, 2)) * (1.0 / np.sqrt(hd))
    if S > 1:
        scores = scores + np.triu(np.full((S, L), -np.inf), k=L - S + 1)
    o = softmax(scores) @ vv
    o = o.transpose(0, 2, 1, 3).reshape(B, S, nh * hd)
    return qlinear(o, shard, f"{p}.o_proj", cfg), cache


def mlp_rank(h, shard, layer: int, cfg: LlamaShape):
    """ParallelMLP.forward before the down_proj all-reduce (mlp.py:239-252)."""
    p = f"model.layers.{layer}.mlp"
    g = qlinear(h, shard, f"{p}.gate_proj", cfg)
    u = qlinear(h, shard, f"{p}.up_proj", cfg)
    return qlinear(silu(g) * u, shard, f"{p}.down_proj", cfg)


# ---------------------------------------------------------------- model

class TPModel:
    """All ranks of a quantized, tied-embedding Llama in one process."""

    def __init__(self, shards: list, cfg: LlamaShape, max_len: int = 4096):
        self.shards = shards
        self.cfg = cfg
        self.world = len(shards)
        self.cos, self.sin = rope_tables(cfg.head_dim, max_len, cfg.rope_theta)
        self.cache = None  # [rank][layer] -> (k, v)

    def reset(self):
        self.cache = None

    def forward(self, ids, use_cache=True, return_hidden=False):
        """ParallelTransformer.forward for every rank (transformer.py:516-577).

        Returns logits ``[B, S, V]`` (float64) and, when asked, the hidden
        state after the embedding and after each layer.
        """
        cfg, W = self.cfg, self.world
        ids = np.asarray(ids)
        h = all_reduce_sum([embed_rank(ids, self.shards[r], cfg, W, r).astype(np.float64) for r in range(W)])
        hidden = [h]
        new_cache = [[None] * cfg.num_layers for _ in range(W)]
        for i in range(cfg.num_layers):
            ln1 = f"model.layers.{i}.input_layernorm.weight"
            ln2 = f"model.layers.{i}.post_attention_layernorm.weight"
            parts = []
            for r in range(W):
                x = rmsnorm(h, self.shards[r][ln1], cfg.rms_norm_eps)
                past = None if self.cache is None else self.cache[r][i]
                part, kv = attention_rank(x, self.shards[r], i, cfg, W, past, self.cos, self.sin)
                parts.append(part)
                new_cache[r][i] = kv
            h = h + all_reduce_sum(parts)
            parts = []
            for r in range(W):
                x = rmsnorm(h, self.shards[r][ln2], cfg.rms_norm_eps)
                parts.append(mlp_rank(x, self.shards[r], i, cfg))
            h = h + all_reduce_sum(parts)
            hidden.append(h)
        logits = self.lm_head(h)
        if use_cache:
            self.cache = new_cache
        return (logits, hidden) if return_hidden else logits

    def lm_head(self, h):
        """Tied head: ``h @ dequantize_weight().T`` per rank, then all-gather."""
        cfg = self.cfg
        parts = []
        for r in range(self.world):
            x = rmsnorm(h, self.shards[r]["model.norm.weight"], cfg.rms_norm_eps)
            e = qa.dequantize(self.shards[r]["model.embed_tokens.weight"],
                              self.shards[r]["model.embed_tokens.scales"],
                              self.shards[r]["model.embed_tokens.biases"],
                              cfg.group_size, cfg.bits).astype(np.float64)
            parts.append(x @ e.T)
        return all_gather(parts, dim=-1)

    def generate(self, prompt, steps: int):
        """Greedy branch of ParallelExecutor.generate (executor.py:258-325)."""
        self.reset()
        logits = self.forward(prompt)
        out = []
        for _ in range(steps):
            tok = np.argmax(logits[:, -1, :], axis=-1)
            out.append(tok)
            logits = self.forward(tok[:, None])
        return np.stack(out, axis=1)


def distributed_argmax(local_logits: list, vocab_per_rank: int):
    """Greedy token from vocab-split logits without gathering them.

    Each rank contributes (max value, lowest local index of that max); the
    winner is the largest value, ties broken by the lowest global index, which
    equals ``argmax`` of the all-gathered logits (executor.py:276-278).
    """
    best_v, best_i = None, None
    for r, lg in enumerate(local_logits):
        i = np.argmax(lg, axis=-1)
        v = np.take_along_axis(lg, i[..., None], axis=-1)[..., 0]
        gi = i + r * vocab_per_rank
        if best_v is None:
            best_v, best_i = v, gi
        else:
            take = (v > best_v) | ((v == best_v) & (gi < best_i))
            best_v = np.where(take, v, best_v)
            best_i = np.where(take, gi, best_i)
    return best_i
