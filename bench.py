#!/usr/bin/env python
"""Decode throughput of the tensor-parallel 4-bit Llama-3-8B path on B200.

Workload (default): Llama-3-8B shapes (hidden 4096, 32 layers, 32 q / 8 kv
heads, ffn 14336, vocab 128256, RoPE theta 5e5), random-init N(0, 0.02)
weights quantized 4-bit g64 on the GPU, tied embedding/LM head, batch 1, KV
cache pre-filled by a 2048-token random prompt, greedy decode.  One *step* is
one decode token for the whole batch: embedding, 32 layers, LM head, argmax,
all captured in one CUDA graph.  Per step every rank streams its whole weight
shard (4.5 GB at TP1), far more than the 126 MB L2, so no L2 flush is needed.

``python bench.py --gpus N --steps K --warmup W``; for N > 1 it runs under
torchrun (one process per GPU, tensor parallel, NCCL for the data path, gloo
for timing control).  Rank 0 prints one JSON line.

``--impl reference`` times the CPU stand-in of the reference's MLX CPU decode
(torch fp32 on all host threads; MLX is not installed) on rank 0 only.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

MODELS = {
    "llama3-8b": dict(vocab_size=128256, hidden_size=4096, num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                      intermediate_size=14336, max_position_embeddings=8192, rms_norm_eps=1e-5, rope_theta=5e5,
                      tie_word_embeddings=True),
    "tinyllama": dict(vocab_size=32000, hidden_size=2048, num_hidden_layers=22, num_attention_heads=32, num_key_value_heads=4,
                      intermediate_size=5632, max_position_embeddings=2048, rms_norm_eps=1e-5, rope_theta=1e4,
                      tie_word_embeddings=True),
    "llama3-70b": dict(vocab_size=128256, hidden_size=8192, num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8,
                       intermediate_size=28672, max_position_embeddings=8192, rms_norm_eps=1e-5, rope_theta=5e5,
                       tie_word_embeddings=True),
}
METRIC = "decode tok/s bs1 Llama-3-8B 4-bit at TP 1/2/4/8; dequant-GEMV HBM GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=sorted(MODELS), default="llama3-8b")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--bits", type=int, default=4, choices=[4, 8])
    ap.add_argument("--group", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: build this many decoder layers instead of the model's")
    ap.add_argument("--workload", choices=["cfg3", "cfg2", "cfg4"], default="cfg3",
                    help="cfg3: the decode step (default, the headline); cfg2: the isolated quantized-linear sweep; "
                         "cfg4: the vocab-parallel embedding + LM head (one JSON line per case)")
    ap.add_argument("--kernel-gemv", default="",
                    help="profiling only: N,K,epilogue (store|residual|swiglu) -- time --steps launches of one "
                         "decode GEMV over 5 rotating weight sets and print one JSON line")
    return ap.parse_args()


def run_gemv(args) -> int:
    """Isolated decode-GEMV launches (the shape an ncu capture of the top kernel uses)."""
    from shardcompute_b200 import _lib as L
    from shardcompute_b200 import ops

    n, k, mode = args.kernel_gemv.split(",")
    N, K = int(n), int(k)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    nseg = 2 if mode == "swiglu" else 1
    ws = [[ops.quantize((torch.randn(N, K, device=dev) * 0.02).half(), args.group, args.bits) for _ in range(nseg)]
          for _ in range(5)]
    x = torch.randn(1, K, device=dev)
    nw = torch.ones(K, device=dev, dtype=torch.float16) if mode != "residual" else None
    y = torch.zeros(1, N, device=dev, dtype=torch.float32)

    def one(i):
        segs = ws[i % 5]
        if mode == "swiglu":
            ops.qlinear_fused(x, segs, args.group, args.bits, epilogue=L.SC_EPI_SWIGLU, norm_weight=nw, out=y)
        elif mode == "residual":
            ops.qlinear_fused(x, segs, args.group, args.bits, epilogue=L.SC_EPI_RESIDUAL, residual=y, out=y)
        else:
            ops.qlinear_fused(x, segs, args.group, args.bits, norm_weight=nw, out=y)

    for i in range(args.warmup):
        one(i)
    torch.cuda.synchronize(dev)
    # one CUDA graph of a launch per weight set, so host launch overhead does not
    # sit between the kernels (as in the decode step; PDL on between them)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(5):
            one(i)
    graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / (args.steps * 5)
    nbytes = nseg * (N * K * args.bits // 8 + N * (K // args.group) * 4) + K * 4 + N * 4
    print(json.dumps({"kernel": "qgemv_fx", "N": N, "K": K, "epilogue": mode, "us_per_launch": us,
                      "algorithmic_bytes": nbytes, "GB/s": nbytes / us / 1e3,
                      "device_error": L.load().sc_qgemv_device_error(1)}), flush=True)
    return 0


def _graph_time(fn, n_calls: int, reps: int, dev, sync=None) -> float:
    """Mean device time (ms) of one call: `n_calls` calls captured in one CUDA
    graph, replayed `reps` times between CUDA events on the replay stream
    (`sync` lines the ranks up before the timed replays)."""
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(n_calls):  # warm-up: plans, lazy loads, collective rendezvous
            fn(i)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for i in range(n_calls):
            fn(i)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize(dev)
    if sync:
        sync()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / (reps * n_calls)
    del g
    return ms


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _setup_dist(local: int, world: int, rank: int):
    import torch.distributed as dist

    from shardcompute_b200.collectives import Communicator

    torch.cuda.set_device(local)
    comm = None
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
        comm = Communicator(rank, world, backend="nccl")
        comm.initialize_sync(timeout=300)
    return comm


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sync(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def run_linear_sweep(args) -> int:
    """cfg2: the isolated quantized linear, fp16 activations N(0,1) [M, 4096]
    times 4- / 8-bit g64 weights N(0,0.02) [14336, 4096], column-parallel (N
    split, no collective) and row-parallel (K split + all-reduce of the fp32
    partial), M in {1, 4, 16, 256}.  Weight sets rotate so every call streams
    from HBM (the sets together exceed 3x the L2).  One JSON line per case:
    device time per call (max over ranks), algorithmic bytes (weights,
    scales, biases, x in, y out) and FLOPs per rank, fractions of the
    measured HBM and bf16 peaks."""
    from shardcompute_b200 import ops

    rank, world, local = dist_env()
    comm = _setup_dist(local, world, rank)
    dev = torch.device("cuda", local)
    hbm, tf, kind = _peaks()
    K, N = 4096, 14336
    torch.manual_seed(0)
    modes = ["column"] if world == 1 else ["column", "row"]
    for bits in (4, 8):
        for mode in modes:
            n_r, k_r = (N // world, K) if mode == "column" else (N, K // world)
            wbytes = n_r * k_r * bits // 8 + n_r * (k_r // args.group) * 4
            nsets = max(2, min(48, -(-3 * 126 * 2 ** 20 // wbytes)))
            sets = [ops.quantize((torch.randn(n_r, k_r, device=dev) * 0.02).half(), args.group, bits)
                    for _ in range(nsets)]
            for M in (1, 4, 16, 256):
                x = torch.randn(M, k_r, device=dev).half()
                y = torch.empty(M, n_r, device=dev, dtype=torch.float16 if mode == "column" else torch.float32)
                red = torch.empty_like(y) if mode == "row" else None

                def call(i, x=x, y=y, red=red):
                    wq, sc, bi = sets[i % nsets]
                    ops.qlinear(x, wq, sc, bi, args.group, bits, out=y)
                    if red is not None:
                        comm.allreduce_into(y, red)

                ms = _max_over_ranks(_graph_time(call, nsets, max(4, args.steps // 8), dev, lambda: _sync(world)),
                                     world)
                nbytes = wbytes + M * k_r * 2 + M * n_r * y.element_size()
                flops = 2 * M * n_r * k_r
                gbs, tfs = nbytes / (ms / 1e3) / 1e9, flops / (ms / 1e3) / 1e12
                if rank == 0:
                    print(json.dumps({"workload": "cfg2", "mode": mode, "tp": world, "bits": bits, "group": args.group,
                                      "M": M, "K": K, "N": N, "rank_shape": [n_r, k_r], "us_per_call": ms * 1e3,
                                      "algorithmic_bytes": nbytes, "GB/s": gbs, "hbm_frac": gbs / hbm,
                                      "TFLOP/s": tfs, "tensor_frac": tfs / tf, "peak_kind": kind,
                                      "collective": "all-reduce of the fp32 partial [M, N]" if mode == "row" else None,
                                      "weight_sets": nsets,
                                      "kernel": "qgemv (decode GEMV)" if M <= 16 else "qgemm_tc (tcgen05)"}),
                          flush=True)
            del sets
            torch.cuda.empty_cache()
    if comm is not None:
        comm.shutdown_sync()
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def zipf_ids(n: int, vocab: int, s: float, seed: int) -> torch.Tensor:
    """n token ids with P(id = k) proportional to (k + 1)^-s over the vocabulary."""
    import numpy as np

    p = np.arange(1, vocab + 1, dtype=np.float64) ** -s
    p /= p.sum()
    return torch.from_numpy(np.random.default_rng(seed).choice(vocab, size=n, p=p).astype(np.int32))


def run_embed_head(args) -> int:
    """cfg4: vocab-parallel embedding + LM head, 4096 Zipf(1.1) token ids per
    step: masked fp16 row gather from this rank's [V/TP, 4096] table (K3) +
    all-reduce, then the rank's 4-bit g64 head [V/TP, 4096] over the 4096
    gathered rows (tcgen05 dequant-GEMM, K2), per-row argmax of the rank's
    logits, all-gather of (max, index) and the merge (distributed argmax).
    Prints one JSON line: tokens/s and each part's device time."""
    from shardcompute_b200 import _lib as L
    from shardcompute_b200 import ops

    rank, world, local = dist_env()
    comm = _setup_dist(local, world, rank)
    dev = torch.device("cuda", local)
    hbm, tf, kind = _peaks()
    V, H, T = 128256, 4096, 4096
    Vl = V // world
    v0 = rank * Vl
    torch.manual_seed(rank)
    table = (torch.randn(Vl, H, device=dev) * 0.02).half()
    head = ops.quantize((torch.randn(Vl, H, device=dev) * 0.02).half(), args.group, args.bits)
    ids = zipf_ids(T, V, 1.1, seed=3).to(dev)
    h_part = torch.empty(T, H, device=dev)
    h = torch.empty(T, H, device=dev)
    logits = torch.empty(T, Vl, device=dev)
    val = torch.empty(T, device=dev)
    idx = torch.empty(T, dtype=torch.int32, device=dev)
    gv = torch.empty(world, T, device=dev)
    gi = torch.empty(world, T, dtype=torch.int32, device=dev)
    tok = torch.empty(T, dtype=torch.int32, device=dev)

    def gather(_):
        L.call("sc_embed_gather_f16", ids.data_ptr(), T, table.data_ptr(), v0, v0 + Vl, H, h_part.data_ptr(),
               L.SC_F32, ops.stream_handle(dev))
        if comm is not None:
            comm.allreduce_into(h_part, h)

    def head_gemm(_):
        ops.qlinear(h if comm is not None else h_part, *head, args.group, args.bits, out=logits)

    def pick(_):
        ops.argmax(logits, v0, val, idx)
        if comm is not None:
            comm.allgather_into(val, gv)
            comm.allgather_into(idx, gi)
        else:
            gv[0].copy_(val)
            gi[0].copy_(idx)
        ops.argmax_merge(gv, gi, world, tok)

    reps = max(4, args.steps // 8)
    t_g = _max_over_ranks(_graph_time(gather, 4, reps, dev, lambda: _sync(world)), world)
    t_h = _max_over_ranks(_graph_time(head_gemm, 2, reps, dev, lambda: _sync(world)), world)
    t_p = _max_over_ranks(_graph_time(pick, 4, reps, dev, lambda: _sync(world)), world)

    def step(i):
        gather(i)
        head_gemm(i)
        pick(i)

    t_s = _max_over_ranks(_graph_time(step, 2, reps, dev, lambda: _sync(world)), world)
    in_range = int(((ids >= v0) & (ids < v0 + Vl)).sum())
    g_bytes = in_range * H * 2 + T * H * 4 + T * 4  # rows read, fp32 rows written, ids
    hw_bytes = Vl * H * args.bits // 8 + Vl * (H // args.group) * 4
    flops = 2 * T * Vl * H
    if rank == 0:
        print(json.dumps({
            "workload": "cfg4", "metric": "embedding + LM head tokens/s (4096 Zipf(1.1) ids per step)",
            "value": T / (t_s / 1e3), "unit": "tok/s", "tp": world, "bits": args.bits, "group": args.group,
            "ms_per_step": t_s, "parts_ms": {"gather+allreduce": t_g, "head_gemm": t_h, "argmax+gather+merge": t_p},
            "gather": {"rows_in_range_rank0": in_range, "algorithmic_bytes": g_bytes,
                       "GB/s_incl_allreduce": g_bytes / (t_g / 1e3) / 1e9},
            "head": {"flops": flops, "TFLOP/s": flops / (t_h / 1e3) / 1e12,
                     "tensor_frac": flops / (t_h / 1e3) / 1e12 / tf, "weight_bytes": hw_bytes, "peak_kind": kind,
                     "kernel": "qgemm_tc (tcgen05, exact weights as fp16 hi + lo, x hi + lo: 3 MMAs per k-step)"},
            "data": "synthetic (N(0,0.02) table and head, Zipf(1.1) ids, seed 3)"}), flush=True)
    if comm is not None:
        comm.shutdown_sync()
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# DRAM bytes (read + written) of the GEMV launches of one decode step, measured
# by ncu (dram__bytes_read.sum + dram__bytes_write.sum over the timed graph
# replays of `python bench.py --steps 2 --warmup 3 --no-cpu-baseline`).
NCU_GEMV_TRAFFIC = {("llama3-8b", 1, 1, 4, 64, 2048): 4235.6e6}

# The first 8 greedy tokens of sequence 0 after the prompt, from a TP1 run of
# the same command (synthetic weights are one model at TP 1/2/4/8, so every N
# should reproduce them); keyed by (model, bits, group, ctx, batch, layers).
TP1_FIRST_TOKENS = {("llama3-8b", 4, 64, 2048, 1, 32): [72726, 111630, 23418, 10603, 90257, 89492, 83690, 73369]}


def probe_mlx() -> str:
    """Whether the reference's CPU backend (MLX) imports on this host."""
    try:
        import mlx.core  # noqa: F401
        return "importable"
    except Exception as e:  # noqa: BLE001 - any failure means the reference path cannot run
        return f"not importable: {type(e).__name__}: {e}"


def load_peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        sel = []
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = ["-i", uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"]
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"] + sel, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- reference arm

def cpu_sample(args, world: int, budget_s: float):
    """Time the CPU stand-in of the reference decode; returns (tok/s, threads, description)."""
    from oracle.cpu_decode import CpuDecodeSample, DecodeShape

    m = MODELS[args.model]
    sh = DecodeShape(hidden=m["hidden_size"], layers=m["num_hidden_layers"], heads=m["num_attention_heads"],
                     kv_heads=m["num_key_value_heads"],
                     ffn=m["intermediate_size"], vocab=m["vocab_size"], bits=args.bits, group=args.group,
                     ctx=args.ctx, batch=args.batch, world=world)
    s = CpuDecodeSample(sh)
    t1 = s.time_samples(1)
    n = max(1, min(64, int(budget_s / max(t1, 1e-3))))
    sec = s.time_samples(n)
    desc = (f"{n} samples of 1/{sh.layers} token (one decoder layer + 1/{sh.layers} of the tied head) at "
            f"ctx {sh.ctx}, batch {sh.batch}, one TP{world} rank shard; torch fp32 on {s.threads} threads, every "
            f"weight dequantized to fp32 on every step; tok/s = batch / ({sh.layers} x {world} shards x s/sample)")
    return s.tokens_per_s(sec), s.threads, desc, s, sec


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    from oracle.cpu_decode import CpuDecodeSample, DecodeShape

    m = MODELS[args.model]
    sh = DecodeShape(hidden=m["hidden_size"], layers=m["num_hidden_layers"], heads=m["num_attention_heads"],
                     kv_heads=m["num_key_value_heads"], ffn=m["intermediate_size"], vocab=m["vocab_size"],
                     bits=args.bits, group=args.group, ctx=args.ctx, batch=args.batch, world=world)
    s = CpuDecodeSample(sh)
    threads = s.threads
    desc = (f"each step = 1/{sh.layers} token (one decoder layer + 1/{sh.layers} of the tied head) at ctx {sh.ctx}, "
            f"batch {sh.batch}, one TP{world} rank shard, torch fp32 on {threads} threads, every weight dequantized "
            f"to fp32 on every step; all {world} shards run on this host: tok/s = batch / "
            f"({sh.layers} x {world} x s/step)")
    for _ in range(args.warmup):
        s.run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        s.run()
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    tok_s = s.tokens_per_s(sec)
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "mlx": probe_mlx(),
            "note": "MLX (the reference's CPU backend) does not import here; the oracle's torch-fp32 restatement "
                    "of the same per-token work is timed instead"}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args, world: int):
    extra = {"layers": args.layers, "note": "profiling case: reduced layer count"} if args.layers else {}
    return {**extra, "workload": f"cfg3 {args.model} {args.bits}-bit g{args.group} decode, batch {args.batch}, "
                        f"KV prefilled to {args.ctx}, TP{world}",
            "model": args.model, "global_batch": args.batch, "ctx": args.ctx, "bits": args.bits,
            "group": args.group, "parallelism": f"tp{world}",
            "l2": "no flush: every step streams the rank's full weight shard (> 126 MB L2)"}


# ---------------------------------------------------------------- our arm

def main():
    args = parse()
    rank, world, local = dist_env()
    if args.gpus != world and world > 1:
        print(f"--gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
        return 2
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.kernel_gemv:
        return run_gemv(args)
    if args.workload == "cfg2":
        return run_linear_sweep(args)
    if args.workload == "cfg4":
        return run_embed_head(args)
    if args.warmup < 3:
        print("--warmup must be >= 3", file=sys.stderr)
        return 2

    import torch.distributed as dist

    from shardcompute_b200 import _lib
    from shardcompute_b200.collectives import Communicator
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
        comm = Communicator(rank, world, backend="nccl")
        comm.initialize_sync(timeout=300)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    mdict = dict(MODELS[args.model])
    if args.layers:
        mdict["num_hidden_layers"] = args.layers
    cfg = ModelConfig.from_dict(mdict)
    weights = RankWeights.synthetic(cfg, world, rank, bits=args.bits, group=args.group, device=dev, seed=0)
    B = args.batch
    n_replays = 1 + 2 * (args.warmup + args.steps) + args.steps + 8 + 8
    eng = DecodeEngine(weights, comm, max_batch=B, max_seq=args.ctx + n_replays + 16, device=dev)
    gen = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg.vocab_size, (B, args.ctx), generator=gen, dtype=torch.int64).to(torch.int32)
    prompt_dev = prompt.to(dev)
    # prefill (untimed for the decode metric): one warm-up, then one timed with CUDA events
    eng.reset()
    eng.prefill(prompt_dev)
    torch.cuda.synchronize(dev)
    eng.reset()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    eng.prefill(prompt_dev)
    p1.record()
    barrier()
    prefill_ms = max_over_ranks(p0.elapsed_time(p1))
    # one eager step: count this library's launches per step
    c0 = _lib.load().sc_launch_count()
    eng.decode_step()
    torch.cuda.synchronize(dev)
    launches_per_step = int(_lib.load().sc_launch_count() - c0)
    eng.capture()

    # ---- the first greedy tokens after the prompt (untimed), for cross-N agreement
    host_in = torch.zeros(B, dtype=torch.int32).pin_memory()
    host_out = torch.zeros(B, dtype=torch.int32).pin_memory()
    host_out.copy_(eng.tok[:B])
    first = [int(host_out[0])]
    for _ in range(7):
        host_in.copy_(host_out)
        eng.decode_host(host_in, host_out)
        first.append(int(host_out[0]))

    # ---- timed region: K graph replays, inputs resident on the device
    for _ in range(args.warmup):
        eng.replay()
    barrier()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)  # graph replays launch on the current stream
    # one untimed replay right before e0: its collectives line the ranks up on
    # the device, so no rank's window includes waiting for a late peer
    eng.replay()
    torch.cuda.nvtx.range_push("timed")
    e0.record(stream)
    for _ in range(args.steps):
        eng.replay()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clk = clocks.stop()
    ms_step = ms / args.steps
    value = B * args.steps / (ms / 1e3)

    # ---- end to end: host token in (pinned), device step, host token out, each step
    host_out.copy_(eng.tok[:B])
    for _ in range(3):
        host_in.copy_(host_out)
        eng.decode_host(host_in, host_out)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_in.copy_(host_out)
        eng.decode_host(host_in, host_out)
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": B * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": host_in.numel() * 4,
           "d2h_bytes_per_step": host_out.numel() * 4,
           "path": "DecodeEngine.decode_host: pinned ids -> device, graph step, sampled ids -> pinned host, sync"}

    peak, peak_kind = load_peaks()
    if eng.use_step:
        # one kernel per step: its algorithmic bytes (weights, scales and biases
        # of every linear and of the tied head, the KV cache it reads) over the
        # measured step time, which bounds the kernel's own duration from above
        step_bytes = eng.weight_bytes_per_step() + eng.kv_bytes_per_step()
        achieved = step_bytes / (ms_step / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": "decode_step_kernel (the whole decode step in one launch)",
                    "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": None, "traffic_unit": "bytes per step",
                    "launches_per_step": launches_per_step, "algorithmic_bytes_per_step": step_bytes,
                    "ms_per_step": ms_step, "share_of_step": 1.0, "step_bytes": step_bytes,
                    "step_frac": achieved / peak}
    else:
        # per-kernel step: in-kernel %globaltimer stamps of every dequant-GEMV
        # of a step (first consumer past the dependency wait .. last CTA's
        # exit), in a second capture of the same step with PDL left on
        eng.capture_probe()
        eng.replay_probe()
        g_ms, g_bytes, g_n = 0.0, 0, 0
        kinds = {}  # launch order per step: per layer q|k|v, o, gate|up, down; then the head
        for _ in range(args.steps):
            a, b, n = eng.replay_probe()
            g_ms += a
            g_bytes += b
            g_n += n
            nl = cfg.num_layers
            for slot, ns, nb in eng.probe_last:
                k = ("qkv", "o", "gate_up", "down")[slot % 4] if slot < 4 * nl else "lm_head"
                e = kinds.setdefault(k, [0, 0, 0])
                e[0] += ns
                e[1] += nb
                e[2] += 1
        if g_n == 0:  # no decode-GEMV launch in the step (more than 16 rows: the tensor-core GEMM)
            g_ms, g_bytes, g_n = ms_step * args.steps, int(eng.weight_bytes_per_step()) * args.steps, args.steps
            kinds = {}
        achieved = g_bytes / (g_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": "qgemv_fx (fused RMSNorm/dequant-GEMV/epilogue)" if kinds else
                    "whole decode step (more than 16 rows per linear: the tensor-core GEMM; weights over the step time)",
                    "achieved": achieved,
                    "time_source": "in-kernel %globaltimer stamps per GEMV launch inside the graph step (PDL on)"
                    if kinds else "step time (CUDA events)",
                    "by_kind": {k: {"us_per_launch": v[0] / 1e3 / v[2], "GB/s": v[1] / v[0], "frac": v[1] / v[0] / peak}
                                for k, v in kinds.items() if v[0] > 0},
                    "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": NCU_GEMV_TRAFFIC.get((args.model, world, args.batch, args.bits, args.group, args.ctx)),
                    "traffic_unit": "bytes per step", "launches_per_step": g_n // args.steps,
                    "algorithmic_bytes_per_step": g_bytes // args.steps, "ms_per_step": g_ms / args.steps,
                    "share_of_step": g_ms / args.steps / ms_step}
        step_bytes = g_bytes / args.steps + eng.kv_bytes_per_step()
        roofline["step_bytes"] = step_bytes
        roofline["step_frac"] = step_bytes / (ms_step / 1e3) / 1e9 / peak

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tok_s, threads, desc, _, _ = cpu_sample(args, world, args.cpu_seconds)
        cpu = {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f16", "weights": f"u{args.bits} g{args.group} affine",
                "data": "synthetic (random-init N(0,0.02) weights, uniform random prompt ids)",
                "config": workload_config(args, world), "clocks": clk, "e2e": e2e,
                "gpu_launches": launches_per_step * args.steps, "roofline": roofline, "cpu_baseline": cpu,
                "first_tokens": first,
                "first_tokens_match_tp1": (None if (key := (args.model, args.bits, args.group, args.ctx, B,
                                                            args.layers or cfg.num_layers)) not in TP1_FIRST_TOKENS
                                           else first == TP1_FIRST_TOKENS[key]),
                "prefill": {"tokens": B * args.ctx, "ms": prefill_ms, "tok_per_s": B * args.ctx / (prefill_ms / 1e3),
                            "note": "the prompt through every layer (tensor-core GEMM for more than 16 rows, "
                                    "flash attention), CUDA events, after one warm-up prefill"}}
        print(json.dumps(line), flush=True)
    eng.graph = None
    eng._probe_graph = None
    if comm is not None:
        comm.shutdown_sync()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
