"""Temperature + top-p sampling on the GPU (``sc_sample_*``) against the CPU
restatement of the reference's sampled branch (``oracle/sample.py``,
worker/executor.py:270-306): the same token for the same uniform, the same
distribution, the distributed (vocab-split) phases equal to the one-rank
draw, the device uniform stream, and the engine's sampled generate."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import sample as osample
from oracle import sharder as osh
from oracle import synth
from shardcompute_b200 import _lib as L
from shardcompute_b200 import ops

pytestmark = pytest.mark.gpu

MASK64 = (1 << 64) - 1


def splitmix64(x):
    x = (x + 0x9E3779B97F4A7C15) & MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK64
    return x ^ (x >> 31)


def uniforms(seed, counter, B):
    out = []
    for b in range(B):
        z = splitmix64((seed + ((counter * B + b) * 0x9E3779B97F4A7C15)) & MASK64)
        f = np.float32((z >> 11) * (1.0 / 9007199254740992.0))
        out.append(f if f < 1 else np.float32(0.99999994))
    return np.array(out, dtype=np.float32)


@pytest.mark.parametrize("V", [1000, 32000])
@pytest.mark.parametrize("T,p", [(0.7, 0.9), (1.0, 0.5), (1.5, 1.0), (0.3, 0.95)])
def test_topp_matches_cpu_draw(cuda, V, T, p):
    rng = np.random.default_rng(V + int(T * 10) + int(p * 100))
    B = 64
    logits = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    u = rng.random(B).astype(np.float32)
    tok = torch.full((B,), -7, dtype=torch.int32, device=cuda)
    ops.sample_topp(torch.from_numpy(logits).to(cuda), T, p, torch.from_numpy(u).to(cuda), tok)
    got = tok.cpu().numpy()
    ref = osample.draw(logits, T, p, u)
    agree = float(np.mean(got == ref))
    # only rows whose uniform lands within fp32 rounding of a cumulative-mass boundary may differ
    assert agree >= 0.97, (agree, got[:10], ref[:10])
    q = osample.kept_distribution(logits, T, p)
    assert bool(np.all(q[np.arange(B), got] > 0)), "a drawn token outside the kept set"


def test_topp_distribution(cuda):
    rng = np.random.default_rng(1)
    V, N, T, p = 64, 20000, 0.8, 0.85
    row = (rng.standard_normal(V) * 2).astype(np.float32)
    logits = np.tile(row, (N, 1))
    u = ((np.arange(N) + 0.5) / N).astype(np.float32)  # stratified: counts follow the CDF to 1/N
    tok = torch.zeros(N, dtype=torch.int32, device=cuda)
    ops.sample_topp(torch.from_numpy(logits).to(cuda), T, p, torch.from_numpy(u).to(cuda), tok)
    counts = np.bincount(tok.cpu().numpy(), minlength=V) / N
    q = osample.kept_distribution(row[None], T, p)[0]
    assert np.max(np.abs(counts - q)) <= 3.0 / N
    assert np.all(counts[q == 0] == 0)


@pytest.mark.parametrize("world", [2, 4])
def test_topp_distributed_phases_equal_one_rank(cuda, world):
    """The vocab-split phases (each simulated rank on its slice, the
    exchanges done here as the communicator would) give the one-rank token."""
    lib = L.load()
    rng = np.random.default_rng(world)
    B, V, T, p = 16, 4096, 0.9, 0.8
    Vl = V // world
    logits = torch.from_numpy((rng.standard_normal((B, V)) * 2.5).astype(np.float32)).to(cuda)
    u = torch.from_numpy(rng.random(B).astype(np.float32)).to(cuda)
    one = torch.full((B,), -1, dtype=torch.int32, device=cuda)
    ops.sample_topp(logits, T, p, u, one)
    nbytes = ops.sample_workspace_bytes(B)
    ws = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(world)]
    st = [w[: 8 * B * 4].view(torch.float32).view(8, B) for w in ws]
    hist = [w[8 * B * 4:].view(torch.float32) for w in ws]
    sl = [logits[:, r * Vl:(r + 1) * Vl].contiguous() for r in range(world)]
    stream = torch.cuda.current_stream().cuda_stream

    def phase(r, ph, level=0):
        L.call("sc_sample_phase", sl[r].data_ptr(), B, Vl, Vl, T, p, u.data_ptr(), r * Vl, ph, level,
               ws[r].data_ptr(), nbytes, stream)

    def combine(r, what, gathered=None, tok=None):
        L.call("sc_sample_combine", ws[r].data_ptr(), None if gathered is None else gathered.data_ptr(), B, world, r,
               what, None if tok is None else tok.data_ptr(), stream)

    for r in range(world):
        phase(r, 0)
    g = torch.stack([st[r][0] for r in range(world)]).contiguous()
    for r in range(world):
        combine(r, 0, g)
        phase(r, 1)
    zs = sum(st[r][1].clone() for r in range(world))
    for r in range(world):
        st[r][1].copy_(zs)
    for level in range(4):
        for r in range(world):
            phase(r, 2, level)
        hs = sum(hist[r].clone() for r in range(world))
        for r in range(world):
            hist[r].copy_(hs)
            phase(r, 3, level)
    for r in range(world):
        phase(r, 4)
    g = torch.stack([st[r][4] for r in range(world)]).contiguous()
    for r in range(world):
        combine(r, 1, g)
        phase(r, 5)
    ts = sum(st[r][7].clone() for r in range(world))
    toks = []
    for r in range(world):
        st[r][7].copy_(ts)
        t = torch.full((B,), -1, dtype=torch.int32, device=cuda)
        combine(r, 2, tok=t)
        toks.append(t.cpu().numpy())
    for r in range(world):
        np.testing.assert_array_equal(toks[r], one.cpu().numpy())


def test_device_uniforms_follow_splitmix64(cuda):
    counter = torch.zeros(1, dtype=torch.int64, device=cuda)
    u = torch.zeros(7, dtype=torch.float32, device=cuda)
    for c in range(3):
        ops.sample_uniforms(12345, counter, u)
        np.testing.assert_array_equal(u.cpu().numpy(), uniforms(12345, c, 7))
    assert int(counter[0]) == 3


@pytest.mark.parametrize("one_kernel", [False, True])
def test_engine_sampled_generate(cuda, one_kernel):
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    shape = synth.tiny_shape(num_layers=2)
    shard = osh.shard_weights(synth.checkpoint(shape, seed=4, std=0.05), 1, 0)
    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    w = RankWeights.from_shard(cfg, shard, 1, 0, shape.bits, shape.group_size, cuda)
    eng = DecodeEngine(w, None, max_batch=1, max_seq=96, device=cuda, one_kernel_step=one_kernel)
    assert eng.use_step == one_kernel
    prompt = torch.from_numpy(np.random.default_rng(2).integers(0, shape.vocab_size, size=(1, 8))).to(cuda)
    greedy = eng.generate(prompt, 24).cpu().numpy()
    eng.set_sampling(1.0, 1e-6, seed=3)  # top_p -> 0 keeps only the most likely token: greedy
    assert np.array_equal(eng.generate(prompt, 24).cpu().numpy(), greedy)
    eng.set_sampling(1.2, 0.95, seed=3)
    a = eng.generate(prompt, 24).cpu().numpy()
    eng.set_sampling(1.2, 0.95, seed=3)
    b = eng.generate(prompt, 24).cpu().numpy()
    assert np.array_equal(a, b), "same seed, same tokens"
    eng.set_sampling(1.2, 0.95, seed=4)
    c = eng.generate(prompt, 24).cpu().numpy()
    assert not np.array_equal(a, c), "another seed, other tokens"
    assert (a >= 0).all() and (a < shape.vocab_size).all()
    assert eng.step_error() == 0, eng.step_error_info()
