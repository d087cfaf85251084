"""Oracle (CPU) and CUDA path (GPU) against the committed golden fixtures.

``affine_kat.npz`` holds known answers written from the format definition;
``oracle_small.npz`` freezes seeded oracle outputs (see tests/golden/make_golden.py).
"""

import os

import numpy as np
import pytest

from oracle import mlx_affine as qa
from oracle import sharder as osh
from oracle import synth, tp

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kat():
    return dict(np.load(os.path.join(G, "affine_kat.npz")))


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(os.path.join(G, "oracle_small.npz")))


# ---------------------------------------------------------------- CPU: oracle pinned

def test_oracle_unpack_known_answers(kat):
    np.testing.assert_array_equal(qa.unpack(kat["w4_words"], 4), kat["w4_codes"])
    np.testing.assert_array_equal(qa.unpack(kat["w8_words"], 8), kat["w8_codes"])
    np.testing.assert_array_equal(qa.pack(kat["w4_codes"], 4), kat["w4_words"])
    np.testing.assert_array_equal(qa.pack(kat["w8_codes"], 8), kat["w8_words"])
    # every code appears at every position
    c4 = kat["w4_codes"].reshape(-1, 8)
    assert all(set(c4[:, j]) == set(range(16)) for j in range(8))
    c8 = kat["w8_codes"].reshape(-1, 4)
    assert all(set(c8[:, j]) == set(range(256)) for j in range(4))


def test_oracle_dequant_known_answers(kat):
    d = qa.dequantize(kat["w4_words"], kat["w4_scales_g32"], kat["w4_biases_g32"], 32, 4)
    np.testing.assert_array_equal(d.view(np.uint16), kat["w4_dequant_g32"].view(np.uint16))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("g", [32, 64, 128])
def test_oracle_quant_fixtures(gold, bits, g):
    k = f"b{bits}_g{g}"
    wq, s, b = qa.quantize(gold[f"{k}_w"], g, bits)
    np.testing.assert_array_equal(wq, gold[f"{k}_wq"])
    np.testing.assert_array_equal(s.view(np.uint16), gold[f"{k}_s"].view(np.uint16))
    np.testing.assert_array_equal(b.view(np.uint16), gold[f"{k}_b"].view(np.uint16))
    assert s[3, 0] == 0 and (qa.unpack(wq, bits)[3, :g] == 0).all()  # constant group
    deq = qa.dequantize(wq, s, b, g, bits)
    np.testing.assert_array_equal(deq.view(np.uint16), gold[f"{k}_deq"].view(np.uint16))
    np.testing.assert_array_equal(qa.quantized_matmul(gold[f"{k}_x"], wq, s, b, g, bits), gold[f"{k}_y"])
    # quantization error bounded by half a step (plus fp16 rounding of the stored scale/bias)
    err = np.abs(qa.dequantize_exact(wq, s, b, g, bits) - gold[f"{k}_w"].astype(np.float64))
    step = np.repeat(s.astype(np.float64), g, 1)
    assert (err <= 0.5 * step + 2e-3 * np.abs(gold[f"{k}_w"]) + 1e-6).all()


def test_oracle_embedding_fixture(gold):
    cfg = tp.LlamaShape(vocab_size=256, hidden_size=128, num_layers=1, num_heads=2, num_kv_heads=2,
                        intermediate_size=256)
    for world in (1, 4):
        for r in range(world):
            sh = dict(zip(("model.embed_tokens.weight", "model.embed_tokens.scales", "model.embed_tokens.biases"),
                          osh.shard_quantized("model.embed_tokens.weight", gold["emb_wq"], gold["emb_s"],
                                              gold["emb_b"], world, r)))
            got = tp.embed_rank(gold["emb_ids"], sh, cfg, world, r)
            np.testing.assert_array_equal(got.view(np.uint16), gold[f"emb_w{world}_r{r}"].view(np.uint16))


def _llama():
    shape = synth.tiny_shape(vocab_size=512, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                             intermediate_size=512)
    return shape, synth.checkpoint(shape, seed=17)


@pytest.mark.parametrize("world", [1, 2])
def test_oracle_llama_fixture(gold, world):
    shape, full = _llama()
    shards = [osh.shard_weights(full, world, r) for r in range(world)]
    m = tp.TPModel(shards, shape, max_len=64)
    logits, hidden = m.forward(gold["llama_prompt"], return_hidden=True)
    np.testing.assert_allclose(logits, gold[f"llama_tp{world}_logits"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(np.stack(hidden), gold[f"llama_tp{world}_hidden"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(m.generate(gold["llama_prompt"], 6), gold[f"llama_tp{world}_greedy"])


def test_tp1_and_tp2_oracles_agree(gold):
    """Sharding does not change the model: TP 2 matches TP 1 to float64 rounding."""
    np.testing.assert_allclose(gold["llama_tp2_logits"], gold["llama_tp1_logits"], rtol=1e-4, atol=1e-6)
    np.testing.assert_array_equal(gold["llama_tp2_greedy"], gold["llama_tp1_greedy"])


# ---------------------------------------------------------------- GPU: CUDA path against the fixtures

@pytest.mark.gpu
def test_gpu_dequant_known_answers(cuda, kat):
    import torch

    from shardcompute_b200 import ops

    wq = torch.from_numpy(kat["w4_words"].view(np.int32)).to(cuda)
    s = torch.from_numpy(kat["w4_scales_g32"]).to(cuda)
    b = torch.from_numpy(kat["w4_biases_g32"]).to(cuda)
    got = ops.dequantize(wq, s, b, 32, 4).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint16), kat["w4_dequant_g32"].view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("g", [32, 64, 128])
def test_gpu_quant_fixtures(cuda, gold, bits, g):
    import torch

    from shardcompute_b200 import ops

    k = f"b{bits}_g{g}"
    wq, s, b = ops.quantize(torch.from_numpy(gold[f"{k}_w"]).to(cuda), g, bits)
    np.testing.assert_array_equal(wq.cpu().numpy().view(np.uint32), gold[f"{k}_wq"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), gold[f"{k}_s"].view(np.uint16))
    np.testing.assert_array_equal(b.cpu().numpy().view(np.uint16), gold[f"{k}_b"].view(np.uint16))
    deq = ops.dequantize(wq, s, b, g, bits).cpu().numpy()
    np.testing.assert_array_equal(deq.view(np.uint16), gold[f"{k}_deq"].view(np.uint16))
    y = ops.qlinear(torch.from_numpy(gold[f"{k}_x"]).to(cuda), wq, s, b, g, bits, out_dtype=torch.float32)
    ref = gold[f"{k}_y"]
    assert np.linalg.norm(y.cpu().numpy() - ref) / np.linalg.norm(ref) <= 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 4])
def test_gpu_embedding_fixture(cuda, gold, world):
    import torch

    from shardcompute_b200 import ops

    for r in range(world):
        sw, ss, sb = osh.shard_quantized("model.embed_tokens.weight", gold["emb_wq"], gold["emb_s"], gold["emb_b"],
                                         world, r)
        v0, v1 = r * 256 // world, (r + 1) * 256 // world
        got = ops.embed_gather_q(torch.from_numpy(gold["emb_ids"]).to(cuda),
                                 torch.from_numpy(sw.view(np.int32)).to(cuda), torch.from_numpy(ss).to(cuda),
                                 torch.from_numpy(sb).to(cuda), v0, v1, 128, 64, 4).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint16), gold[f"emb_w{world}_r{r}"].view(np.uint16))


@pytest.mark.gpu
def test_gpu_llama_fixture(cuda, gold):
    import torch

    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    shape, full = _llama()
    shard = osh.shard_weights(full, 1, 0)
    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    w = RankWeights.from_shard(cfg, shard, 1, 0, shape.bits, shape.group_size, cuda)
    eng = DecodeEngine(w, None, max_batch=1, max_seq=64, device=cuda)
    prompt = torch.from_numpy(gold["llama_prompt"]).to(cuda)
    logits, hidden = eng.forward_logits(prompt, return_hidden=True)
    ref_h = gold["llama_tp1_hidden"]
    for i, h in enumerate(hidden):
        r = ref_h[i].astype(np.float64)
        err = np.linalg.norm(h.view(r.shape).cpu().numpy() - r) / np.linalg.norm(r)
        assert err <= 1e-3, f"hidden {i}: {err:.2e}"
    toks = eng.generate(prompt, 6).cpu().numpy()
    np.testing.assert_array_equal(toks, gold["llama_tp1_greedy"])
