"""The reference-shaped layer API (``shardcompute_b200.parallel``) on the GPU.

Mirrors the reference's own layer tests (tests/test_parallel_layers.py,
tests/test_integration.py) with ranks simulated in one process (partials summed
/ concatenated by hand, as those tests do), then checks the full
``ParallelTransformer`` and ``ParallelExecutor.generate`` against the oracle.
"""

import asyncio

import numpy as np
import pytest
import torch

from oracle import mlx_affine as qa
from oracle import sharder as osh
from oracle import synth
from oracle.tp import TPModel
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu


def run(coro):
    return asyncio.run(coro)


def _qshard(name, wq, s, b, world, rank):
    return osh.shard_quantized(name, wq, s, b, world, rank)


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_column_then_row_split_equals_full(cuda, rng, bits):
    from shardcompute_b200.parallel import QuantizedColumnParallelLinear, QuantizedRowParallelLinear

    H, F, g, world = 512, 1024, 64, 2
    up = qa.quantize((rng.standard_normal((F, H)) * 0.02).astype(np.float16), g, bits)
    down = qa.quantize((rng.standard_normal((H, F)) * 0.02).astype(np.float16), g, bits)
    x = rng.standard_normal((2, 3, H)).astype(np.float32)
    full_inter = np.maximum(qa.quantized_matmul(x.reshape(-1, H), *up, g, bits), 0)
    full = qa.quantized_matmul(full_inter, *down, g, bits)
    parts = []
    for r in range(world):
        col = QuantizedColumnParallelLinear(H, F, world, r, bias=False, group_size=g, bits=bits)
        col.load_quantized_shard(*_qshard("mlp.up_proj.weight", *up, world, r))
        row = QuantizedRowParallelLinear(F, H, world, r, bias=False, group_size=g, bits=bits)
        row.load_quantized_shard(*_qshard("mlp.down_proj.weight", *down, world, r))
        assert col.local_out_features == F // world and row.local_in_features == F // world
        inter = torch.clamp_min(col.forward_sync(torch.from_numpy(x).to(cuda)), 0)
        parts.append(row.forward_partial(inter).double().cpu().numpy().reshape(-1, H))
    assert rel_l2(parts[0] + parts[1], full) <= 1e-3


def test_row_bias_added_once_on_rank0(cuda, rng):
    from shardcompute_b200.parallel import QuantizedRowParallelLinear

    K, N, g = 256, 64, 64
    w = qa.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float16), g, 4)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float16)
    layers = []
    for r in range(2):
        lay = QuantizedRowParallelLinear(K, N, 2, r, bias=True, group_size=g)
        lay.load_quantized_shard(*_qshard("self_attn.o_proj.weight", *w, 2, r), linear_bias=bias)
        layers.append(lay)
    assert layers[0].bias is not None and layers[1].bias is None
    x = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float32)).to(cuda)
    tot = sum(layers[r].forward_partial(x[:, r * 128:(r + 1) * 128]) for r in range(2))
    out = layers[0].add_bias(tot).double().cpu().numpy()
    ref = qa.quantized_matmul(x.cpu().numpy(), *w, g, 4) + bias
    assert rel_l2(out, ref) <= 1e-3


def test_full_k_scales_are_sliced_on_load(cuda, rng):
    """parallel/quantized_linear.py:385-414: a row shard carrying full-K
    scales/biases is sliced to the rank's K range."""
    from shardcompute_b200.parallel import QuantizedRowParallelLinear

    K, N, g = 512, 32, 64
    wq, s, b = qa.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float16), g, 4)
    lay = QuantizedRowParallelLinear(K, N, 2, 1, bias=False, group_size=g)
    lay.load_quantized_shard(wq[:, wq.shape[1] // 2:], s, b)
    assert tuple(lay.scales.shape) == (N, K // g // 2)
    np.testing.assert_array_equal(lay.scales.cpu().numpy(), s[:, K // g // 2:])


def test_quantized_embedding_ranks_sum_to_full(cuda, rng):
    from shardcompute_b200.parallel import QuantizedParallelEmbedding

    V, H, world = 1000, 256, 4
    wq, s, b = qa.quantize((rng.standard_normal((V, H)) * 0.02).astype(np.float16), 64, 4)
    ids = torch.from_numpy(rng.integers(0, V, size=(2, 9))).to(cuda)
    tot = None
    for r in range(world):
        e = QuantizedParallelEmbedding(V, H, world, r, group_size=64, bits=4)
        e.load_quantized_shard(*_qshard("model.embed_tokens.weight", wq, s, b, world, r))
        part = e.forward_local(ids)
        tot = part.float() if tot is None else tot + part.float()
    ref = qa.dequantize(wq, s, b, 64, 4)[ids.cpu().numpy()]
    np.testing.assert_array_equal(tot.half().cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_dense_column_row_and_hidden_split_embedding(cuda, rng):
    from shardcompute_b200.parallel import ColumnParallelLinear, ParallelEmbedding, RowParallelLinear

    x = torch.from_numpy(rng.standard_normal((2, 4, 256)).astype(np.float16)).to(cuda)
    W1 = torch.from_numpy((rng.standard_normal((256, 512)) * 0.05).astype(np.float16)).to(cuda)
    W2 = torch.from_numpy((rng.standard_normal((512, 256)) * 0.05).astype(np.float16)).to(cuda)
    full = (x.float() @ W1.float()).clamp_min(0) @ W2.float()
    tot = 0
    for r in range(2):
        c = ColumnParallelLinear(256, 512, 2, r, bias=False)
        c.load_shard(W1)
        rw = RowParallelLinear(512, 256, 2, r, bias=False)
        rw.load_shard(W2)
        tot = tot + rw.forward_partial(c.forward_sync(x).clamp_min(0)).float()
    assert rel_l2(tot.cpu().numpy(), full.cpu().numpy()) <= 2e-3
    table = torch.from_numpy(rng.standard_normal((1000, 256)).astype(np.float16)).to(cuda)
    ids = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8]], device=cuda)
    parts = []
    for r in range(2):
        e = ParallelEmbedding(1000, 256, 2, r, gather_output=False)
        e.load_shard(table)
        parts.append(e.forward_sync(ids))
    assert torch.equal(torch.cat(parts, -1), table[ids])


def _tiny():
    shape = synth.tiny_shape(num_layers=2)
    full = synth.checkpoint(shape, seed=21)
    return shape, full, osh.shard_weights(full, 1, 0)


def _model(shape, shard, cuda):
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel import ParallelTransformer, RankWeights

    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    w = RankWeights.from_shard(cfg, shard, 1, 0, shape.bits, shape.group_size, cuda)
    return ParallelTransformer.from_config(cfg, 1, 0, None).load_rank_weights(w), w, cfg


def test_parallel_transformer_forward_matches_oracle(cuda):
    shape, full, shard = _tiny()
    model, _, _ = _model(shape, shard, cuda)
    ref = TPModel([shard], shape, max_len=64)
    prompt = np.random.default_rng(3).integers(0, shape.vocab_size, size=(1, 7))
    ref_logits, ref_hidden = ref.forward(prompt, return_hidden=True)
    logits, cache, hidden = run(model.forward(torch.from_numpy(prompt).to(cuda), use_cache=True,
                                              return_hidden=True))
    for i, (h, r) in enumerate(zip(hidden, ref_hidden)):
        assert rel_l2(h.cpu().numpy(), r) <= 1e-3, i
    assert rel_l2(logits.cpu().numpy(), ref_logits) <= 1e-3
    assert cache[0][0].shape[2] == 7  # reference-style cached length
    tok = np.argmax(ref_logits[:, -1], -1)[:, None]
    ref2 = ref.forward(tok)
    logits2, _ = run(model.forward(torch.from_numpy(tok).to(cuda), past_key_values=cache, use_cache=True))
    assert rel_l2(logits2.cpu().numpy(), ref2) <= 1e-3


def test_executor_generate_greedy_engine_and_layers(cuda):
    from shardcompute_b200.parallel import DecodeEngine
    from shardcompute_b200.worker import ParallelExecutor

    shape, full, shard = _tiny()
    model, w, _ = _model(shape, shard, cuda)
    eng = DecodeEngine(w, None, max_batch=1, max_seq=96, device=cuda)
    prompt = np.random.default_rng(5).integers(0, shape.vocab_size, size=(1, 10))
    ref_tok = TPModel([shard], shape, max_len=96).generate(prompt, 16)
    ex = ParallelExecutor(0, 1, None, model=model, engine=eng)
    out = run(ex.generate(torch.from_numpy(prompt).to(cuda), max_new_tokens=16, temperature=0))
    assert out.shape == (1, 26)
    assert float(np.mean(out[:, 10:].cpu().numpy() == ref_tok)) >= 0.99
    # the layer path (no engine) gives the same greedy tokens
    ex2 = ParallelExecutor(0, 1, None, model=model)
    out2 = run(ex2.generate(torch.from_numpy(prompt).to(cuda), max_new_tokens=16, temperature=0))
    assert torch.equal(out2.cpu(), out.cpu())
    # stop token ends generation early
    stop = int(ref_tok[0, 3])
    out3 = run(ex.generate(torch.from_numpy(prompt).to(cuda), max_new_tokens=16, temperature=0,
                           stop_tokens=[stop]))
    assert out3.shape[1] <= 14 and int(out3[0, -1]) == stop
    # top-p sampling runs and returns in-vocab ids
    out4 = run(ex2.generate(torch.from_numpy(prompt).to(cuda), max_new_tokens=4, temperature=0.7, top_p=0.9))
    assert out4.shape == (1, 14) and int(out4.max()) < shape.vocab_size
