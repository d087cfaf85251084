"""Tensor-parallel executor (reference ``worker/executor.py:67-373``).

``forward`` runs the layer-by-layer ``ParallelTransformer`` (the drop-in
API) with the executor-held cache, exactly as the reference does.
``generate`` with ``temperature == 0`` (the greedy branch,
:267-325) runs on ``DecodeEngine``: the prompt is prefilled once, then each
step is one CUDA-graph replay whose argmax works on the vocab-split logits
(each rank contributes its (max, lowest index); ties resolve to the lowest
global index, as ``argmax`` of the gathered logits does) and writes the next
token on the device; the host reads one int32 per sequence per step for the
stop check (:308-313).  ``temperature > 0`` gathers the logits and samples
top-p on the device with torch.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Awaitable, Callable, Dict, List, Optional

import torch

from .. import ops
from ..parallel.decode_engine import DecodeEngine
from ..parallel.transformer import ParallelTransformer

TokenCallback = Callable[[int, int, bool], Awaitable[None]]


@dataclass
class LayerTiming:
    layer_idx: int
    compute_ms: float = 0.0
    comm_ms: float = 0.0

    @property
    def total_ms(self) -> float:
        return self.compute_ms + self.comm_ms


@dataclass
class ExecutionMetrics:
    total_time_ms: float
    layer_timings: List[LayerTiming] = field(default_factory=list)
    input_tokens: int = 0
    output_shape: List[int] = field(default_factory=list)

    @property
    def compute_time_ms(self) -> float:
        return sum(t.compute_ms for t in self.layer_timings)

    @property
    def comm_time_ms(self) -> float:
        return sum(t.comm_ms for t in self.layer_timings)

    @property
    def compute_fraction(self) -> float:
        tot = self.compute_time_ms + self.comm_time_ms
        return self.compute_time_ms / tot if tot > 0 else 0.0

    def to_dict(self) -> Dict[str, Any]:
        return {"total_time_ms": self.total_time_ms, "compute_time_ms": self.compute_time_ms,
                "comm_time_ms": self.comm_time_ms, "compute_fraction": self.compute_fraction,
                "input_tokens": self.input_tokens, "output_shape": self.output_shape,
                "num_layers": len(self.layer_timings)}


class ParallelExecutor:
    def __init__(self, rank: int, world_size: int, communicator, model: Optional[ParallelTransformer] = None,
                 engine: Optional[DecodeEngine] = None):
        if model is None and engine is None:
            raise ValueError("ParallelExecutor needs a model, an engine, or both")
        self.rank = rank
        self.world_size = world_size
        self.communicator = communicator
        self.model = model
        self.engine = engine
        self.last_metrics: Optional[ExecutionMetrics] = None
        self._past_key_values = None
        self.seed = 0  # seed of the sampled branch's uniform stream

    async def forward(self, input_ids: torch.Tensor, attention_mask=None, use_cache: bool = False) -> torch.Tensor:
        if self.model is None:
            raise RuntimeError("forward needs the layer model")
        t0 = time.perf_counter()
        logits, cache = await self.model.forward(input_ids, attention_mask=attention_mask,
                                                 past_key_values=self._past_key_values, use_cache=use_cache)
        if use_cache:
            self._past_key_values = cache
        torch.cuda.current_stream(logits.device).synchronize()
        self.last_metrics = ExecutionMetrics(total_time_ms=(time.perf_counter() - t0) * 1000,
                                             input_tokens=input_ids.numel(), output_shape=list(logits.shape))
        return logits

    async def forward_with_timing(self, input_ids: torch.Tensor, attention_mask=None):
        logits = await self.forward(input_ids, attention_mask=attention_mask)
        return logits, self.last_metrics

    async def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 100, temperature: float = 0.7,
                       top_p: float = 0.9, stop_tokens: Optional[List[int]] = None,
                       token_callback: Optional[TokenCallback] = None) -> torch.Tensor:
        """Prompt ``[B, S]`` -> ``[B, S + generated]`` (same device as the input)."""
        stop_tokens = list(stop_tokens or [])
        t0 = time.perf_counter()
        if temperature == 0 and self.engine is not None:
            generated = await self._generate_greedy(input_ids, max_new_tokens, stop_tokens, token_callback)
        else:
            generated = await self._generate_sampled(input_ids, max_new_tokens, temperature, top_p, stop_tokens,
                                                     token_callback)
        n = len(generated)
        if n:
            self.last_metrics = ExecutionMetrics(total_time_ms=(time.perf_counter() - t0) * 1000, input_tokens=n,
                                                 output_shape=[1, n])
            gen = torch.stack([g.to(input_ids.device, input_ids.dtype) for g in generated], dim=1)
            return torch.cat([input_ids, gen], dim=1)
        return input_ids

    async def _generate_greedy(self, input_ids, max_new_tokens, stop_tokens, token_callback):
        eng = self.engine
        B = input_ids.shape[0]
        dev = eng.device
        eng.reset()
        eng.prefill(input_ids.to(dev))
        host = torch.empty(B, dtype=torch.int32, pin_memory=True)
        out = []
        for i in range(max_new_tokens):
            host.copy_(eng.tok[:B], non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            tok = host.clone()
            out.append(tok)
            tid = int(tok[0])
            is_stop = tid in stop_tokens
            is_last = is_stop or i == max_new_tokens - 1
            if token_callback is not None:
                await token_callback(tid, i, is_last)
            if is_last:
                break
            if B == eng.B:
                eng.replay()
            else:
                eng.decode_step()
        return out

    async def _generate_sampled(self, input_ids, max_new_tokens, temperature, top_p, stop_tokens, token_callback):
        """The sampled branch (worker/executor.py:270-306): with the decode
        engine every draw runs on the GPU inside the captured step (tensor
        parallel: a distributed top-p over the vocab-split logits); without
        it, the layer model's gathered logits go through the same sampling
        kernel."""
        if self.engine is not None:
            self.engine.set_sampling(temperature, top_p, seed=self.seed)
            try:
                return await self._generate_greedy(input_ids, max_new_tokens, stop_tokens, token_callback)
            finally:
                self.engine.set_sampling(0.0)
        if self.model is None:
            raise RuntimeError("sampling needs the decode engine or the layer model")
        self._past_key_values = None
        logits = await self.forward(input_ids, use_cache=True)
        out = []
        B = logits.shape[0]
        dev = logits.device
        counter = torch.zeros(1, dtype=torch.int64, device=dev)
        u = torch.empty(B, dtype=torch.float32, device=dev)
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        for i in range(max_new_tokens):
            nl = logits[:, -1, :].float().contiguous()
            if temperature == 0:
                tok.copy_(torch.argmax(nl, dim=-1))
            else:
                ops.sample_uniforms(self.seed, counter, u)
                ops.sample_topp(nl, temperature, top_p, u, tok)
            nxt = tok.clone()
            out.append(nxt)
            tid = int(nxt[0])
            is_stop = tid in stop_tokens
            is_last = is_stop or i == max_new_tokens - 1
            if token_callback is not None:
                await token_callback(tid, i, is_last)
            if is_last:
                break
            logits = await self.forward(nxt[:, None], use_cache=True)
        return out

    def reset_cache(self):
        self._past_key_values = None
        if self.engine is not None:
            self.engine.reset()

    def get_metrics(self) -> Optional[Dict[str, Any]]:
        return self.last_metrics.to_dict() if self.last_metrics else None

    def get_timing_summary(self) -> Dict[str, Any]:
        if not self.last_metrics:
            return {}
        m = self.last_metrics
        return {"total_ms": m.total_time_ms, "compute_ms": m.compute_time_ms, "comm_ms": m.comm_time_ms,
                "compute_fraction": m.compute_fraction,
                "tokens_per_second": m.input_tokens / (m.total_time_ms / 1000) if m.total_time_ms > 0 else 0.0}
