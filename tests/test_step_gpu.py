"""The persistent one-kernel decode step (``sc_step_run``) against the float64
oracle: the hidden state after the embedding and after every layer of one
decode step (1e-3 relative L2), its logits, and greedy agreement over 128
steps; the same step through a CUDA graph; and its bounded failure path (a
position past the cache makes every CTA stop, the error word says why, and
the token and position are left as they were)."""

import numpy as np
import pytest
import torch

from oracle import sharder as osh
from oracle import synth
from oracle.tp import TPModel

pytestmark = pytest.mark.gpu

TOL = 1e-3

SHAPES = {
    # hidden, heads / kv heads (GQA group), head_dim, ffn
    "tiny-g2-hd64": synth.tiny_shape(num_layers=2),
    "llama3-8b-dims-2L": synth.tiny_shape(vocab_size=8192, hidden_size=4096, num_layers=2, num_heads=32,
                                          num_kv_heads=8, intermediate_size=14336, rope_theta=5e5),
    "tinyllama-dims-2L": synth.tiny_shape(vocab_size=32000, hidden_size=2048, num_layers=2, num_heads=32,
                                          num_kv_heads=4, intermediate_size=5632),
    "g1-hd128": synth.tiny_shape(hidden_size=1024, num_heads=8, num_kv_heads=8, intermediate_size=1536),
    # a 512-row head over a 4096-deep input (as on a TP8 rank): that GEMV runs on fewer CTAs
    # than SMs, so a tile's 16 units cross at most 4 CTAs
    "head512-4096deep": synth.tiny_shape(vocab_size=512, hidden_size=4096, num_heads=32, num_kv_heads=8,
                                         intermediate_size=512),
}


def _engine(shape, shard, max_seq, dev):
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    w = RankWeights.from_shard(cfg, shard, 1, 0, shape.bits, shape.group_size, dev)
    return DecodeEngine(w, None, max_batch=1, max_seq=max_seq, device=dev, one_kernel_step=True)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", list(SHAPES))
def test_step_kernel_hidden_states_and_logits(cuda, name):
    shape = SHAPES[name]
    shard = osh.shard_weights(synth.checkpoint(shape, seed=3), 1, 0)
    eng = _engine(shape, shard, 128, cuda)
    assert eng.use_step
    eng.enable_step_debug()
    ref = TPModel([shard], shape, max_len=128)
    prompt = np.random.Generator(np.random.PCG64(7)).integers(0, shape.vocab_size, size=(1, 11))
    ref_logits = ref.forward(prompt)
    eng.reset()
    eng.prefill(torch.from_numpy(prompt).to(cuda))
    tok = int(eng.tok[0])
    assert tok == int(np.argmax(ref_logits[0, -1]))
    for step in range(3):
        eng.decode_step()  # one launch: embedding of tok ... argmax
        torch.cuda.synchronize()
        assert eng.step_error() == 0, eng.step_error_info()
        rl, rh = ref.forward(np.array([[tok]]), return_hidden=True)
        trace = eng.step_trace.double().cpu().numpy()
        for i, r in enumerate(rh):
            err = _rel(trace[i], r[0, 0])
            assert err <= TOL, f"{name} step {step}: hidden {i} rel L2 {err:.3e}"
        err = _rel(eng.step_logits.double().cpu().numpy(), rl[0, 0])
        assert err <= TOL, f"{name} step {step}: logits rel L2 {err:.3e}"
        nxt = int(eng.tok[0])
        assert nxt == int(np.argmax(rl[0, 0])), f"{name} step {step}: token {nxt}"
        assert int(eng.pos[0]) == 11 + step + 1
        tok = nxt


def test_step_kernel_greedy_128_graph(cuda):
    shape = synth.tiny_shape(num_layers=2)
    full = synth.checkpoint(shape, seed=5, std=0.05)
    shard = osh.shard_weights(full, 1, 0)
    eng = _engine(shape, shard, 192, cuda)
    assert eng.use_step
    ref = TPModel([shard], shape, max_len=192)
    prompt = np.random.Generator(np.random.PCG64(11)).integers(0, shape.vocab_size, size=(1, 16))
    steps = 128
    ref_tok = ref.generate(prompt, steps)[0]
    out = eng.generate(torch.from_numpy(prompt).to(cuda), steps).cpu().numpy()[0]  # CUDA-graph replays
    assert float(np.mean(out == ref_tok)) >= 0.99, f"{out[:20]} vs {ref_tok[:20]}"
    assert eng.step_error() == 0, eng.step_error_info()


def test_step_kernel_stops_cleanly_past_the_cache(cuda):
    """A position at the end of the cache: every CTA skips its work, the
    error word reads 1, token and position are left as they were, and after
    a reset the engine decodes again."""
    shape = synth.tiny_shape(num_layers=1)
    shard = osh.shard_weights(synth.checkpoint(shape, seed=1), 1, 0)
    eng = _engine(shape, shard, 32, cuda)
    eng.reset()
    eng.prefill(torch.zeros(1, 8, dtype=torch.int64, device=cuda))
    eng.decode_step()
    torch.cuda.synchronize()
    assert eng.step_error() == 0, eng.step_error_info()
    tok0 = int(eng.tok[0])
    eng.pos.fill_(32)  # == max_seq: outside the cache
    eng.host_pos = 0
    eng.decode_step()
    torch.cuda.synchronize()
    assert eng.step_error(reset=True) == 1
    assert int(eng.pos[0]) == 32 and int(eng.tok[0]) == tok0
    eng.reset()
    eng.prefill(torch.zeros(1, 8, dtype=torch.int64, device=cuda))
    eng.decode_step()
    torch.cuda.synchronize()
    assert eng.step_error() == 0 and int(eng.pos[0]) == 9
