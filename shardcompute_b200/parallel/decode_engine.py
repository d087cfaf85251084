"""Fused per-rank forward of the tensor-parallel quantized decoder.

This is the hot path behind ``ParallelTransformer.forward`` /
``ParallelExecutor.generate`` (reference parallel/transformer.py:516-577,
worker/executor.py:229-325), re-laid for B200:

* one step = embedding gather (K3) -> per layer [RMSNorm+q|k|v GEMV (K1) ->
  fused RoPE + KV append + split-KV attention (K4) -> o GEMV + residual (K1)
  -> RMSNorm+gate|up GEMV with SiLU*mul (K1) -> down GEMV + residual (K1)] ->
  RMSNorm+tied LM-head GEMV (K1) -> argmax (K7); optionally (``prefetch_mb``)
  each GEMV's producer also pulls a share of the next GEMV's weights into L2
  once its own have landed;
* TP > 1: the embedding and the two row-parallel outputs per layer are
  all-reduced through NVLink peer memory (one-shot, NCCL for messages above
  the transport's limit); rank 0 folds the residual into its partial so the
  all-reduce output *is* the new hidden state; greedy sampling gathers only
  (max, index) per rank instead of the vocab-split logits;
* the residual stream and every GEMV input are fp32 (the GEMV splits them into exact fp16 hi / lo parts), KV cache fp32
  ``[L, 2, B, Hkv/TP, Lmax, hd]`` (as the reference's: RoPE's fp32 tables promote k), preallocated;
* positions and token ids live in device buffers, so one decode step is
  captured once in a CUDA graph and replayed; each replay reads the token the
  previous replay wrote and advances the position counter on the device;
* at batch 1 with 4-bit group-64 weights the whole decode step is ONE
  persistent kernel (``sc_step_run``, ``csrc/sc_step.cu``): the weights of
  every GEMV and the cached keys / values stream through one shared-memory
  ring per SM without stopping at op boundaries, the row-parallel
  all-reduces run inside it over NVLink, and the last CTA writes the sampled
  token.  Opt-in (``one_kernel_step=True`` or ``SC_STEP=1``, batch 1, 4-bit
  g64); the per-kernel step above is the default.
"""

from __future__ import annotations

import ctypes as C
import math
import os
from typing import List, Optional

import numpy as np
import torch

from .. import _lib as L
from .. import ops
from ..model.config import ModelConfig
from .weights import RankWeights


def rope_table(head_dim: int, length: int, base: float):
    """fp32 cos/sin ``[length, head_dim/2]`` computed as the reference does
    (inv_freq = 1 / base**(arange(0, hd, 2)/hd), angles = outer(t, inv_freq);
    parallel/attention.py:56-92)."""
    inv = (np.float32(1.0) / (np.float32(base) ** (np.arange(0, head_dim, 2, dtype=np.float32)
                                                    / np.float32(head_dim)))).astype(np.float32)
    ang = np.outer(np.arange(length, dtype=np.float32), inv).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class DecodeEngine:
    """One rank's decoder state: weights, KV cache, buffers, captured step."""

    def __init__(self, weights: RankWeights, comm=None, max_batch: int = 1, max_seq: int = 2048,
                 device: Optional[torch.device] = None, attn_splits: Optional[int] = None,
                 prefetch_mb: Optional[float] = None, one_kernel_step: Optional[bool] = None,
                 fused_allreduce: Optional[bool] = None):
        cfg: ModelConfig = weights.cfg
        self.cfg = cfg
        self.w = weights
        self.comm = comm
        self.world = weights.world
        self.rank = weights.rank
        if self.world > 1 and comm is None:
            raise RuntimeError("Communicator required for tensor parallelism (world_size > 1)")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.B = max_batch
        self.Lmax = max_seq
        self.H = cfg.hidden_size
        self.hd = cfg.head_dim
        self.Hq = cfg.num_heads // self.world
        self.Hkv = cfg.kv_heads // self.world
        self.F = cfg.intermediate_size // self.world
        self.Vl = cfg.vocab_size // self.world
        self.bits, self.group = weights.bits, weights.group
        self.eps = cfg.rms_norm_eps
        nl = cfg.num_layers
        self.kv = torch.zeros(nl, 2, self.B, self.Hkv, self.Lmax, self.hd, dtype=torch.float32, device=dev)
        cos, sin = rope_table(self.hd, self.Lmax, cfg.rope_theta)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.host_pos = 0  # host mirror of pos: bounds every step against the cache length
        self.tok = torch.zeros(self.B, dtype=torch.int32, device=dev)  # decode input / sampled output
        self.tickets = torch.zeros(self.B * self.Hkv, dtype=torch.int32, device=dev)  # attention split merge
        self.fused_attn = os.environ.get("SC_ATTN_FUSED", "1") != "0"
        if attn_splits is None and os.environ.get("SC_ATTN_SPLITS"):
            attn_splits = int(os.environ["SC_ATTN_SPLITS"])
        if attn_splits is None:  # ~2 CTAs per SM
            attn_splits = max(1, min(64, math.ceil(2 * 148 / max(1, self.Hkv * self.B)), math.ceil(self.Lmax / 64)))
        self.splits = attn_splits
        self._bufs = {}
        # L2 prefetch of the next GEMV's weights (bytes per GEMV; 0 = off)
        if prefetch_mb is None:
            prefetch_mb = float(os.environ.get("SC_PREFETCH_MB", "0"))
        self.prefetch_bytes = int(prefetch_mb * (1 << 20))
        self._pf_lists = {}
        self._probe: Optional[list] = None  # (start, end, bytes) per GEMV while instrumenting
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self._graph_stream: Optional[torch.cuda.Stream] = None
        # decode scratch: fixed for the engine's lifetime (a captured graph keeps its address)
        self.workspace = torch.empty(self._workspace_bytes(self.B, 1), dtype=torch.uint8, device=dev)
        self._ws = self.workspace
        # the persistent one-kernel decode step (built at the first decode step);
        # opt-in (argument, or SC_STEP=1): its GEMV consumers are slower than
        # the per-kernel step's today
        if one_kernel_step is None:
            one_kernel_step = os.environ.get("SC_STEP", "0") == "1"
        self.use_step = (one_kernel_step and self.B == 1 and self.bits == 4 and self.group == 64
                         and cfg.hidden_size % 512 == 0 and (self.Hq * self.hd) % 512 == 0 and self.F % 256 == 0
                         and self.F >= 512 and self.hd in (64, 128) and (self.Hq // self.Hkv) in (1, 2, 4, 8))
        # TP > 1: the o / down GEMVs run their all-reduce in the epilogue
        # (sc_qlinear_allreduce, over a transport of their own) where the
        # pass allows it (argument, or SC_FUSED_AR=0 to keep the pair)
        if fused_allreduce is None:
            fused_allreduce = os.environ.get("SC_FUSED_AR", "1") != "0"
        self._ar_p2p = None
        if (fused_allreduce and self.world > 1 and not self.use_step and getattr(comm, "backend", None) == "nccl"
                and comm.p2p_enabled):
            self._ar_p2p = comm.fused_transport(self.B * self.H * 4)
        self.fused_ar_calls = 0  # row-parallel GEMVs that ran with the all-reduce in the epilogue
        self._step = None
        self._step_ws: Optional[torch.Tensor] = None
        self.step_trace: Optional[torch.Tensor] = None   # [L+1, H] hidden states of the last step (debug)
        # [V/TP] logits of the last one-kernel step (the sampler's input)
        self.step_logits = torch.zeros(self.Vl, dtype=torch.float32, device=dev)
        self._step_debug = False
        # sampling (temperature 0: greedy argmax); uniforms from a device counter
        self.temperature, self.top_p, self.seed = 0.0, 1.0, 0
        self._u = torch.zeros(self.B, dtype=torch.float32, device=dev)
        self._rng_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self._sample_ws = torch.empty(ops.sample_workspace_bytes(self.B), dtype=torch.uint8, device=dev)
        self._sample_gather = torch.zeros(self.world, self.B, dtype=torch.float32, device=dev)

    # ------------------------------------------------------------ buffers

    def _workspace_bytes(self, B: int, S: int) -> int:
        M = B * S
        qkvN = (self.Hq + 2 * self.Hkv) * self.hd
        need = [ops.qlinear_workspace_bytes(M, self.H, qkvN, self.bits),
                ops.qlinear_workspace_bytes(M, self.Hq * self.hd, self.H, self.bits),
                ops.qlinear_workspace_bytes(M, self.H, self.F, self.bits) * 2,
                ops.qlinear_workspace_bytes(M, self.F, self.H, self.bits),
                ops.qlinear_workspace_bytes(M, self.H, self.Vl, self.bits),
                ops.flash_decode_workspace_bytes(B, S, self.Hq, self.hd, self.splits if S == 1 else 1),
                ops.attn_decode_workspace_bytes(B, self.Hq, self.hd, self.splits),
                ops.argmax_workspace_bytes(B, self.Vl)]
        return max(max(need), 1 << 16)

    def _use_workspace(self, B: int, S: int):
        """Select scratch for a (B, S) pass: the decode workspace when it is
        big enough, else a transient one (prefill), never the captured one resized."""
        need = self._workspace_bytes(B, S)
        if need <= self.workspace.numel():
            self._ws = self.workspace
        else:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)

    def _buffers(self, B: int, S: int):
        key = (B, S)
        if key in self._bufs:
            return self._bufs[key]
        dev, M = self.device, B * S
        b = {
            "ids": torch.zeros(M, dtype=torch.int32, device=dev),
            "h": torch.zeros(M, self.H, dtype=torch.float32, device=dev),
            "part": torch.zeros(M, self.H, dtype=torch.float32, device=dev),
            "qkv": torch.zeros(M, (self.Hq + 2 * self.Hkv) * self.hd, dtype=torch.float32, device=dev),
            "q": torch.zeros(M, self.Hq * self.hd, dtype=torch.float32, device=dev),
            # GEMV inputs stay fp32: the factored GEMV splits them into exact fp16
            # hi / lo parts, so only the fp16 KV cache rounds activations
            "attn": torch.zeros(M, self.Hq * self.hd, dtype=torch.float32, device=dev),
            "act": torch.zeros(M, self.F, dtype=torch.float32, device=dev),
            "hlast": torch.zeros(B, self.H, dtype=torch.float32, device=dev),
            "logits": torch.zeros(B, self.Vl, dtype=torch.float32, device=dev),
            "val": torch.zeros(B, dtype=torch.float32, device=dev),
            "idx": torch.zeros(B, dtype=torch.int32, device=dev),
            "gval": torch.zeros(self.world, B, dtype=torch.float32, device=dev),
            "gidx": torch.zeros(self.world, B, dtype=torch.int32, device=dev),
        }
        if S > 1 and S * B > 64:  # prefill buffers are transient; keep only decode-sized ones cached
            return b
        self._bufs[key] = b
        return b

    # ------------------------------------------------------------ kernels of one step

    def _qlin(self, x, segs, out, epilogue=L.SC_EPI_STORE, norm=None, residual=None, prefetch=None):
        """Fused GEMV through the C ABI with the engine's workspace.

        ``prefetch``: the next GEMV's weight segments; a budget's share of them
        is pulled into L2 by this GEMV's producer once its own weights have
        landed (decode steps only; see ``prefetch_mb``)."""
        n = len(segs)

        M, K = x.shape
        rows = [int(s[0].shape[0]) for s in segs]
        N = rows[0] if epilogue == L.SC_EPI_SWIGLU else sum(rows)
        W = (C.c_void_p * n)(*[s[0].data_ptr() for s in segs])
        Sp = (C.c_void_p * n)(*[s[1].data_ptr() for s in segs])
        Bp = (C.c_void_p * n)(*[s[2].data_ptr() for s in segs])
        R = (C.c_int * n)(*rows)
        if self._probe is not None:
            slot = len(self._probe)
            L.call("sc_qgemv_probe_stamps", self._stamps[slot].data_ptr())
        args = (x.data_ptr(), ops._dt(x), M, K, K, None if norm is None else norm.data_ptr(), float(self.eps), n,
                C.cast(W, L._pp), C.cast(Sp, L._pp), C.cast(Bp, L._pp), R, self.group, self.bits, None, epilogue,
                out.data_ptr(), ops._dt(out), N, None if residual is None else residual.data_ptr(),
                N if residual is not None else 0, self._ws.data_ptr(), self._ws.numel())
        pf = self._pf_list(prefetch) if prefetch else None
        if pf is None:
            L.call("sc_qlinear_fused", *args, ops.stream_handle(self.device))
        else:
            L.call("sc_qlinear_fused_prefetch", *args, C.cast(pf[0], L._pp), pf[1], pf[2], 0,
                   ops.stream_handle(self.device))
        if self._probe is not None:
            L.call("sc_qgemv_probe_stamps", None)
            # algorithmic bytes: packed words + fp16 scale/bias of every segment,
            # the activations in, the norm weight, the outputs (and residual) once
            nbytes = (sum(r * K * self.bits // 8 + r * (K // self.group) * 4 for r in rows) +
                      M * K * x.element_size() + (0 if norm is None else K * 2) +
                      M * N * out.element_size() + (M * N * residual.element_size() if residual is not None else 0))
            self._probe.append((slot, nbytes))

    def _pf_list(self, segs):
        """(ptrs, sizes, n) for an L2 prefetch of a budget's share of ``segs``:
        every tensor of the next GEMV from its start, in proportion to the
        budget, so the first tiles of every CTA are covered.  None when off."""
        if self.prefetch_bytes <= 0:
            return None
        key = tuple(t.data_ptr() for tri in segs for t in tri)
        lst = self._pf_lists.get(key)
        if lst is None:
            tensors = [t for tri in segs for t in tri]
            sizes = [t.numel() * t.element_size() for t in tensors]
            frac = min(1.0, self.prefetch_bytes / max(1, sum(sizes)))
            n = len(tensors)
            lst = ((C.c_void_p * n)(*[t.data_ptr() for t in tensors]),
                   (C.c_size_t * n)(*[int(z * frac) for z in sizes]), n)
            self._pf_lists[key] = lst
        return lst

    def _allreduce(self, send, recv):
        if self.world == 1:
            if send.data_ptr() != recv.data_ptr():
                recv.copy_(send)
            return
        self.comm.allreduce_into(send, recv, "sum")

    def _layers(self, bf, B: int, S: int, hidden: Optional[List[torch.Tensor]] = None):
        """Embedding + all layers for M = B*S tokens at positions pos..pos+S-1."""
        w, M = self.w, B * S
        h = bf["h"]
        ops.embed_gather_q(bf["ids"], *w.embed, w.vocab_start, w.vocab_end, self.H, self.group, self.bits,
                           out=h)
        self._allreduce(h, h)
        if hidden is not None:
            hidden.append(h.clone())
        splits = self.splits if S == 1 else 1
        nl = len(w.layers)
        pf = S == 1  # decode steps prefetch; a prefill reads each weight many times anyway
        for i, lw in enumerate(w.layers):
            kc, vc = self.kv[i, 0], self.kv[i, 1]
            self._qlin(h, [lw.q, lw.k, lw.v], bf["qkv"], norm=lw.ln1, prefetch=[lw.o] if pf else None)
            if S == 1 and self.fused_attn:
                ops.attn_decode(bf["qkv"], B, self.Hq, self.Hkv, self.hd, self.pos, self.cos, self.sin, kc, vc,
                                splits, bf["attn"], self.tickets[: B * self.Hkv], workspace=self._ws)
            else:
                ops.rope_append(bf["qkv"], B, S, self.Hq, self.Hkv, self.hd, self.pos, self.cos, self.sin, bf["q"],
                                kc, vc)
                ops.flash_decode(bf["q"], kc, vc, self.pos, B, S, self.Hq, self.Hkv, self.hd, splits, bf["attn"],
                                 workspace=self._ws)
            self._row_out(bf["attn"], lw.o, h, bf["part"], [lw.gate, lw.up] if pf else None)
            self._qlin(h, [lw.gate, lw.up], bf["act"], epilogue=L.SC_EPI_SWIGLU, norm=lw.ln2,
                       prefetch=[lw.down] if pf else None)
            nxt = None
            if pf:
                nxt = [w.layers[i + 1].q, w.layers[i + 1].k, w.layers[i + 1].v] if i + 1 < nl else [w.embed]
            self._row_out(bf["act"], lw.down, h, bf["part"], nxt)
            if hidden is not None:
                hidden.append(h.clone())

    def _qlin_allreduce(self, x, tri, h) -> bool:
        """h = sum over ranks (rank order) of x.W_r^T, + h on rank 0, by one
        GEMV whose epilogue exchanges the partials over NVLink.  False (and
        nothing launched, on every rank alike) when the pass does not allow it."""
        M, K = x.shape
        N = int(tri[0].shape[0])
        if self._probe is not None:
            slot = len(self._probe)
            L.call("sc_qgemv_probe_stamps", self._stamps[slot].data_ptr())
        st = L.load().sc_qlinear_allreduce(
            x.data_ptr(), ops._dt(x), M, K, K, tri[0].data_ptr(), tri[1].data_ptr(), tri[2].data_ptr(), N,
            self.group, self.bits, None, h.data_ptr(), h.data_ptr() if self.rank == 0 else None, self._ar_p2p,
            ops.stream_handle(self.device))
        if self._probe is not None:
            L.call("sc_qgemv_probe_stamps", None)
        if st == L.SC_ERR_UNSUPPORTED:
            return False
        L.check(st, "sc_qlinear_allreduce")
        if self._probe is not None:
            nbytes = (N * K * self.bits // 8 + N * (K // self.group) * 4 + M * K * x.element_size() +
                      M * N * 4 + (M * N * 4 if self.rank == 0 else 0))
            self._probe.append((slot, nbytes))
        self.fused_ar_calls += 1
        return True

    def _row_out(self, x, tri, h, part, prefetch_next=None):
        """Row-parallel linear + residual.  TP=1: h += x.W^T in place.  TP>1:
        one GEMV with the all-reduce in its epilogue where the pass allows it;
        otherwise rank 0 writes h + x.W^T, others x.W^T, and the all-reduce of
        those partials lands in h (the residual is added exactly once).  The
        next GEMV's weights are prefetched by this GEMV's producer."""
        if self.world > 1 and self._ar_p2p is not None and self._qlin_allreduce(x, tri, h):
            return
        if self.world == 1:
            self._qlin(x, [tri], h, epilogue=L.SC_EPI_RESIDUAL, residual=h, prefetch=prefetch_next)
        elif self.rank == 0:
            self._qlin(x, [tri], part, epilogue=L.SC_EPI_RESIDUAL, residual=h, prefetch=prefetch_next)
        else:
            self._qlin(x, [tri], part, prefetch=prefetch_next)
        if self.world > 1:
            self._allreduce(part, h)

    def _sample(self, bf, hlast, B: int, advance: int):
        """Tied LM head on the last position of each sequence + greedy argmax."""
        w = self.w
        nxt = None
        if B == self.B and hlast.shape[0] == self.B and w.layers:
            lw = w.layers[0]
            nxt = [lw.q, lw.k, lw.v]  # the next step starts with layer 0's q|k|v
        self._qlin(hlast, [w.embed], bf["logits"], norm=w.norm, prefetch=nxt)
        ops.argmax(bf["logits"], index_offset=w.vocab_start, val=bf["val"], idx=bf["idx"])
        if self.world > 1:
            self.comm.allgather_into(bf["val"], bf["gval"])
            self.comm.allgather_into(bf["idx"], bf["gidx"])
            ops.argmax_merge(bf["gval"], bf["gidx"], self.world, self.tok[:B], self.pos, advance)
        else:
            ops.argmax_merge(bf["val"].view(1, B), bf["idx"].view(1, B), 1, self.tok[:B], self.pos, advance)
        self._draw(bf["logits"][:B], B)

    # ------------------------------------------------------------ public steps

    def reset(self):
        self.pos.zero_()
        self.host_pos = 0

    def _advance(self, n: int):
        if self.host_pos + n > self.Lmax:
            raise ValueError(f"KV cache full: position {self.host_pos} + {n} exceeds max_seq {self.Lmax}")
        self.host_pos += n

    def weight_bytes_per_step(self) -> int:
        """Bytes of this rank's weights one decode step streams: every
        linear's packed words, scales and biases, and the tied head's."""
        n = sum(t.numel() * t.element_size() for t in self.w.embed)
        for lw in self.w.layers:
            for tri in (lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down):
                n += sum(t.numel() * t.element_size() for t in tri)
        return n

    def kv_bytes_per_step(self) -> int:
        """KV-cache bytes one decode step reads at the current length (all layers)."""
        return self.cfg.num_layers * 2 * self.B * self.Hkv * self.host_pos * self.hd * self.kv.element_size()

    def prefill(self, input_ids: torch.Tensor):
        """Run the prompt ``[B, S]`` through the model; the first generated
        token lands in ``self.tok`` and the position counter advances by S."""
        B, S = input_ids.shape
        if B > self.B:
            raise ValueError(f"batch {B} > engine max_batch {self.B}")
        self._advance(S)
        bf = self._buffers(B, S)
        self._use_workspace(B, S)
        bf["ids"].copy_(input_ids.reshape(-1).to(torch.int32), non_blocking=True)
        self._layers(bf, B, S)
        hl = bf["h"].view(B, S, self.H)[:, -1] if S > 1 else bf["h"]
        bf["hlast"][:B].copy_(hl)
        self._sample(bf, bf["hlast"][:B], B, S)

    # ------------------------------------------------------------ the one-kernel step

    def enable_step_debug(self):
        """Have the one-kernel step also write the hidden state after the
        embedding and every layer (``step_trace``) and its logits
        (``step_logits``); call before the first decode step."""
        if self._step is not None:
            raise RuntimeError("enable_step_debug must come before the first decode step")
        self._step_debug = True

    def _build_step(self):
        lib = L.load()
        cfg, dev = self.cfg, self.device
        h = C.c_void_p()
        L.check(lib.sc_step_create(self.H, self.Hq, self.Hkv, self.hd, self.F, self.Vl, self.w.vocab_start,
                                   cfg.num_layers, self.bits, self.group, float(self.eps), self.Lmax, self.world,
                                   self.rank, C.byref(h)), "sc_step_create")
        try:
            for i, lw in enumerate(self.w.layers):
                tris = [lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down]
                arr = [(C.c_void_p * 7)(*[t[j].data_ptr() for t in tris]) for j in range(3)]
                L.check(lib.sc_step_set_layer(h, i, lw.ln1.data_ptr(), lw.ln2.data_ptr(), C.cast(arr[0], L._pp),
                                              C.cast(arr[1], L._pp), C.cast(arr[2], L._pp),
                                              self.kv[i, 0].data_ptr(), self.kv[i, 1].data_ptr()), "sc_step_set_layer")
            L.check(lib.sc_step_set_head(h, *[t.data_ptr() for t in self.w.embed], self.w.norm.data_ptr()),
                    "sc_step_set_head")
            if self._step_debug:
                self.step_trace = torch.zeros(cfg.num_layers + 1, self.H, dtype=torch.float32, device=dev)
            L.check(lib.sc_step_set_io(h, self.tok.data_ptr(), self.pos.data_ptr(), self.cos.data_ptr(),
                                       self.sin.data_ptr(), self.cos.shape[0],
                                       None if self.step_trace is None else self.step_trace.data_ptr(),
                                       self.step_logits.data_ptr()),
                    "sc_step_set_io")
            if self.world > 1:
                bases, size = self.comm.step_arena(int(lib.sc_step_arena_bytes(self.H, self.world)))
                arr = (C.c_void_p * self.world)(*bases)
                L.check(lib.sc_step_set_peers(h, C.cast(arr, L._pp), size), "sc_step_set_peers")
            nbytes = int(lib.sc_step_workspace_bytes(h))
            self._step_ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            L.check(lib.sc_step_finalize(h, self._step_ws.data_ptr(), nbytes, ops.stream_handle(dev)),
                    "sc_step_finalize")
        except BaseException:
            lib.sc_step_destroy(h)
            raise
        self._step = h

    # ------------------------------------------------------------ sampling

    def set_sampling(self, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0):
        """Sampled decoding (the reference's generate with temperature > 0,
        worker/executor.py:270-306): every token is drawn from the
        temperature + top-p distribution on the GPU, inside the captured
        step; temperature 0 is greedy.  Restarts the uniform stream."""
        if temperature < 0.0 or not (0.0 < top_p <= 1.0):
            raise ValueError("temperature must be >= 0 and top_p in (0, 1]")
        if (temperature, top_p, seed) != (self.temperature, self.top_p, self.seed):
            self.graph = None  # the captured step changes
        self.temperature, self.top_p, self.seed = float(temperature), float(top_p), int(seed)
        self._rng_counter.zero_()

    def _draw(self, logits: torch.Tensor, B: int):
        """Overwrite the greedy token with a temperature + top-p draw from
        this rank's vocab-split ``logits`` [B, V/TP] (a no-op when greedy)."""
        if self.temperature <= 0.0:
            return
        ops.sample_uniforms(self.seed, self._rng_counter, self._u[:B])
        gather = self._sample_gather if B == self.B else self._sample_gather[:, :B].contiguous()
        ops.sample_topp(logits, self.temperature, self.top_p, self._u[:B], self.tok[:B],
                        comm=self.comm if self.world > 1 else None, vocab_start=self.w.vocab_start,
                        workspace=self._sample_ws, gather=gather)

    def step_error(self, reset: bool = False) -> int:
        """The one-kernel step's device error word (0: fine); synchronises."""
        if self._step is None:
            return 0
        return int(L.load().sc_step_error(self._step, 1 if reset else 0))

    STEP_ERRORS = {1: "position outside the cache", 2: "weight ring", 3: "peer exchange", 4: "q|k|v not complete",
                   5: "GEMV input not complete", 6: "output slot", 7: "argmax exchange"}

    def step_profile(self, steps: int = 4) -> dict:
        """Time the one-kernel step's ops from inside the kernel (per-CTA
        %globaltimer stamps) over `steps` eager steps; returns, per op kind,
        the step time spent on the critical path (the latest CTA's finish of
        that op minus the latest finish of the op before it), summed over the
        layers, plus per-op medians (input wait, weight stream) of the last
        step.  Advances the decode position by `steps`."""
        if not self.use_step:
            raise RuntimeError("step_profile: this engine does not run the one-kernel step")
        if self._step is None:
            self._build_step()
        lib = L.load()
        nsm = torch.cuda.get_device_properties(self.device).multi_processor_count
        nops = 2 + 5 * self.cfg.num_layers
        stamps = torch.zeros(int(lib.sc_step_timing_count(self._step)), dtype=torch.int64, device=self.device)
        L.check(lib.sc_step_set_timing(self._step, stamps.data_ptr()), "sc_step_set_timing")
        try:
            for _ in range(steps):
                self.decode_step()
            torch.cuda.synchronize(self.device)
        finally:
            L.check(lib.sc_step_set_timing(self._step, None), "sc_step_set_timing")
        self.check_step()
        t = stamps.view(nsm, nops, 4).cpu().numpy().astype(np.float64)
        kinds = ["embed"] + ["qkv", "attn", "o", "gateup", "down"] * self.cfg.num_layers + ["head"]
        valid = t > 0
        done = np.where(valid[:, :, 3], t[:, :, 3], -np.inf).max(axis=0)
        start0 = np.where(valid[:, 0, 0], t[:, 0, 0], np.inf).min()
        crit, prev = {}, start0
        per_op = []
        for i, k in enumerate(kinds):
            d = max(done[i], prev)
            crit[k] = crit.get(k, 0.0) + (d - prev) / 1e3
            prev = d
            w = t[:, i, 1] - t[:, i, 0]
            sdur = t[:, i, 2] - t[:, i, 1]
            ok1 = valid[:, i, 1] & valid[:, i, 0]
            ok2 = valid[:, i, 2] & valid[:, i, 1]
            per_op.append({"op": i, "kind": k, "ctas": int(valid[:, i, 3].sum()),
                           "wait_us_med": float(np.median(w[ok1])) / 1e3 if ok1.any() else None,
                           "stream_us_med": float(np.median(sdur[ok2])) / 1e3 if ok2.any() else None,
                           "stream_us_max": float(np.max(sdur[ok2])) / 1e3 if ok2.any() else None,
                           "finish_us": (done[i] - start0) / 1e3})
        return {"step_us": (prev - start0) / 1e3, "critical_us_by_kind": crit, "ops": per_op}

    def step_error_info(self) -> dict:
        """Where the step kernel's first error was raised (op index and kind,
        CTA, warp, counter seen / target) and the op each CTA last started."""
        if self._step is None:
            return {}
        nsm = torch.cuda.get_device_properties(self.device).multi_processor_count
        nops = 2 + 5 * self.cfg.num_layers
        n = 8 + nsm + nops
        buf = (C.c_int * n)()
        L.check(L.load().sc_step_error_info(self._step, buf, n), "sc_step_error_info")
        kinds = ["embed"] + ["qkv", "attn", "o", "gateup", "down"] * self.cfg.num_layers + ["head"]
        op = buf[0]
        prog = list(buf[8:8 + nsm])
        where = {}
        for c, v in enumerate(prog):
            if v != nops:
                where.setdefault(v, []).append(c)
        return {"op": op, "kind": kinds[op] if 0 <= op < nops else "?", "layer": (op - 1) // 5 if 0 < op < nops - 1
                else -1, "cta": buf[1], "warp": buf[2], "seen": buf[3], "target": buf[4],
                "ctas_by_op": {f"{k}:{kinds[k] if 0 <= k < nops else '?'}": (len(v), v[:6]) for k, v in
                               sorted(where.items())},
                "input_counts": list(buf[8 + nsm:8 + nsm + nops])}

    def check_step(self):
        code = self.step_error()
        if code:
            raise TimeoutError(f"rank {self.rank}: the decode step kernel gave up on a wait (error {code}: "
                               f"{self.STEP_ERRORS.get(code, '?')}; {self.step_error_info()})")

    def __del__(self):
        try:
            if self._step is not None:
                L.load().sc_step_destroy(self._step)
                self._step = None
        except Exception:  # noqa: BLE001 - interpreter teardown
            pass

    def decode_step(self):
        """One greedy step for the engine's full batch (eager)."""
        self._advance(1)
        if self.use_step:
            if self._step is None:
                self._build_step()
            L.call("sc_step_run", self._step, ops.stream_handle(self.device))
            self._draw(self.step_logits.view(1, self.Vl), 1)
            return
        B = self.B
        bf = self._buffers(B, 1)
        self._ws = self.workspace
        bf["ids"].copy_(self.tok[:B])
        self._layers(bf, B, 1)
        self._sample(bf, bf["h"], B, 1)

    def capture(self):
        """Capture decode_step in a CUDA graph (after one eager warm-up)."""
        self._graph_stream = torch.cuda.Stream(device=self.device)
        self._graph_stream.wait_stream(torch.cuda.current_stream(self.device))
        pos0 = self.pos.clone()
        tok0 = self.tok.clone()
        rng0 = self._rng_counter.clone()
        hp0 = self.host_pos
        with torch.cuda.stream(self._graph_stream):
            self.decode_step()  # warm-up: plans, tensor maps, lazy module loads
        torch.cuda.current_stream(self.device).wait_stream(self._graph_stream)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self._graph_stream):
            self.decode_step()
        torch.cuda.synchronize(self.device)
        self.host_pos = hp0
        # the eager warm-up advanced the position, wrote one cache slot that
        # the next real step overwrites and drew one uniform (sampled decoding);
        # put the position, token and uniform stream back
        self.pos.copy_(pos0)
        self.tok.copy_(tok0)
        self._rng_counter.copy_(rng0)
        return self.graph

    def capture_probe(self):
        """Capture a second copy of the decode step whose dequant-GEMV
        launches carry in-kernel time stamps (``sc_qgemv_probe_stamps``: the
        first consumer past the dependency wait, the last CTA's exit), so
        programmatic dependent launch stays on and the GEMVs run as they do
        in the step; ``replay_probe`` then returns their summed in-step time
        and algorithmic bytes."""
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        nmax = 4 * self.cfg.num_layers + 8
        init = torch.zeros(nmax, 2, dtype=torch.int64, device=self.device)
        init[:, 0] = -1  # UINT64_MAX: the stamps lower it
        self._stamps_init = init
        self._stamps = init.clone()
        self._probe = []
        g = torch.cuda.CUDAGraph()
        hp0 = self.host_pos
        try:
            with torch.cuda.graph(g, stream=stream):
                self._stamps.copy_(self._stamps_init)
                self.decode_step()
        finally:
            probe, self._probe = self._probe, None
            self.host_pos = hp0
            L.call("sc_qgemv_probe_stamps", None)
        torch.cuda.synchronize(self.device)
        self._probe_graph, self._probe_slots = g, probe
        return g

    def replay_probe(self):
        """Replay the instrumented step; returns (gemv_ms, gemv_bytes,
        launches): the sum over the step's GEMVs of (last exit - first
        consumer start), all on the device clock."""
        self._advance(1)
        self._probe_graph.replay()
        torch.cuda.synchronize(self.device)
        st = self._stamps.cpu().numpy().view(np.uint64)
        ns, nbytes, n = 0, 0, 0
        self.probe_last = []  # (slot, ns, bytes) of the last replay, in launch order
        for slot, b in self._probe_slots:
            t0, t1 = int(st[slot, 0]), int(st[slot, 1])
            if t0 != 0xFFFFFFFFFFFFFFFF and t1 >= t0:
                ns += t1 - t0
                nbytes += b
                n += 1
                self.probe_last.append((slot, t1 - t0, b))
        return ns / 1e6, nbytes, n

    def decode_host(self, tokens: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """One greedy step driven from host memory: copy ``tokens`` (pinned
        int32 [B]) to the device, replay the step, copy the sampled tokens
        back into ``out`` (pinned int32 [B]) and wait for them."""
        self.tok[: tokens.numel()].copy_(tokens, non_blocking=True)
        self.replay()
        out.copy_(self.tok[: out.numel()], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out

    def replay(self):
        if self.graph is None:
            self.capture()
        self._advance(1)
        self.graph.replay()

    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, stop_tokens=(), use_graph: bool = True):
        """Greedy generation: prefill, then one token per step, each read back
        to the host (the reference's per-token stop check,
        worker/executor.py:308-313)."""
        self.reset()
        self.prefill(input_ids)
        B = input_ids.shape[0]
        out = []
        host_tok = torch.empty(B, dtype=torch.int32, pin_memory=True)
        for t in range(max_new_tokens):
            host_tok.copy_(self.tok[:B], non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            out.append(host_tok.clone())
            if int(host_tok[0]) in stop_tokens or t == max_new_tokens - 1:
                break
            if use_graph and B == self.B:
                self.replay()
            else:
                self.decode_step()
        if self.world > 1:
            self.comm.check_health()  # a timed-out peer-memory collective leaves undefined tokens
        self.check_step()
        return torch.stack(out, dim=1)

    def forward_logits(self, input_ids: torch.Tensor, return_hidden: bool = False):
        """Full forward of ``[B, S]`` ids at the current position (cache
        updated): logits for every position, gathered over the vocab split
        (``ParallelTransformer.forward`` semantics), optionally with the hidden
        state after the embedding and after each layer."""
        B, S = input_ids.shape
        self._advance(S)
        bf = self._buffers(B, S)
        self._use_workspace(B, S)
        bf["ids"].copy_(input_ids.reshape(-1).to(torch.int32))
        hidden = [] if return_hidden else None
        self._layers(bf, B, S, hidden)
        logits = torch.empty(B * S, self.Vl, dtype=torch.float32, device=self.device)
        self._qlin(bf["h"], [self.w.embed], logits, norm=self.w.norm)
        if self.world > 1:
            g = torch.empty(self.world, B * S, self.Vl, dtype=torch.float32, device=self.device)
            self.comm.allgather_into(logits, g)
            logits = g.permute(1, 0, 2).reshape(B * S, self.world * self.Vl)
        with torch.no_grad():
            self.pos += S
        logits = logits.view(B, S, -1)
        return (logits, hidden) if return_hidden else logits
