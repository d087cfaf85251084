"""Parity of the CUDA decode path at the headline configurations.

cfg3 (Llama-3-8B shapes, all 32 layers, 4-bit g64, tied head, full 128256
vocab): a 2048-token prompt (the KV length the benchmark decodes at), then
128 greedy decode steps through the CUDA-graph engine; cfg3 at batch 8 and
32 through the batched GEMV; the same model end to end in 8-bit.  The
reference is ``tests/fullsize.TorchRef`` (the numpy oracle's math in torch
float64 on the GPU, pinned to the oracle by ``tests/test_torch_ref.py``).

Tolerances (the path's contract): the hidden state after the embedding and
after every layer within 1e-3 relative L2 of the float64 reference (prefill
and the first decode step); greedy tokens agree on at least 99 % of the
decode steps.
"""

import numpy as np
import pytest
import torch

from oracle import synth
from oracle.tp import LlamaShape
from tests.fullsize import LLAMA3_8B, TorchRef, gpu_checkpoint, rel_l2

pytestmark = pytest.mark.gpu

HIDDEN_TOL = 1e-3
AGREE = 0.99


def _engine(shape, shard, max_batch, max_seq, dev, world=1, rank=0, comm=None):
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    w = RankWeights.from_shard(cfg, shard, world, rank, shape.bits, shape.group_size, dev)
    return DecodeEngine(w, comm, max_batch=max_batch, max_seq=max_seq, device=dev)


def _layer_errors(hid_e, hid_r, B, S):
    return [rel_l2(e.view(B, S, -1), r) for e, r in zip(hid_e, hid_r)]


def run_parity(shape, B, ctx, steps, dev, seed=0):
    """Prefill + one decode step (per-layer hidden states) + greedy decode."""
    torch.manual_seed(seed)
    ckpt = gpu_checkpoint(shape, seed, dev)
    eng = _engine(shape, ckpt, B, ctx + steps + 8, dev)
    ref = TorchRef([ckpt], shape, max_len=ctx + steps + 8, device=dev)
    prompt = torch.randint(0, shape.vocab_size, (B, ctx), generator=torch.Generator().manual_seed(2))

    eng.reset()
    le, he = eng.forward_logits(prompt.to(dev), return_hidden=True)
    lr, hr = ref.forward(prompt, return_hidden=True)
    pre = _layer_errors(he, hr, B, ctx)
    pre_logits = rel_l2(le, lr)
    del le, he, hr

    toks_r = [lr[:, -1].argmax(-1)]
    del lr
    le2, he2 = eng.forward_logits(toks_r[0][:, None].to(dev), return_hidden=True)
    lr2, hr2 = ref.forward(toks_r[0][:, None], return_hidden=True)
    dec = _layer_errors(he2, hr2, B, 1)
    dec_logits = rel_l2(le2, lr2)
    toks_r.append(lr2[:, -1].argmax(-1))
    del le2, he2, hr2
    for _ in range(steps - 2):
        toks_r.append(ref.forward(toks_r[-1][:, None])[:, -1].argmax(-1))
    ref_tok = torch.stack(toks_r, dim=1).cpu().numpy()
    del ref
    torch.cuda.empty_cache()

    out = eng.generate(prompt.to(dev), steps).cpu().numpy()
    agree = float(np.mean(out == ref_tok))
    return dict(prefill_layers=pre, prefill_logits=pre_logits, decode_layers=dec, decode_logits=dec_logits,
                agree=agree, tokens=out, ref_tokens=ref_tok)


def _check(res, name):
    msg = (f"{name}: prefill max layer err {max(res['prefill_layers']):.2e} (logits {res['prefill_logits']:.2e}), "
           f"decode max layer err {max(res['decode_layers']):.2e} (logits {res['decode_logits']:.2e}), "
           f"greedy agreement {res['agree']:.3f}")
    print(msg)
    assert max(res["prefill_layers"]) <= HIDDEN_TOL, msg + f"\nprefill per layer: {res['prefill_layers']}"
    assert res["prefill_logits"] <= HIDDEN_TOL, msg
    assert max(res["decode_layers"]) <= HIDDEN_TOL, msg + f"\ndecode per layer: {res['decode_layers']}"
    assert res["decode_logits"] <= HIDDEN_TOL, msg
    assert res["agree"] >= AGREE, msg + f"\n{res['tokens'][0, :24]}\n{res['ref_tokens'][0, :24]}"


def test_cfg3_llama3_8b_32_layers_ctx2048(cuda):
    shape = LlamaShape(**LLAMA3_8B, bits=4, group_size=64)
    _check(run_parity(shape, B=1, ctx=2048, steps=128, dev=cuda), "cfg3 b1 ctx2048")


@pytest.mark.parametrize("B", [8, 32])
def test_cfg3_llama3_8b_batched(cuda, B):
    shape = LlamaShape(**LLAMA3_8B, bits=4, group_size=64)
    _check(run_parity(shape, B=B, ctx=128, steps=32, dev=cuda), f"cfg3 b{B}")


def test_cfg3_llama3_8b_8bit(cuda):
    shape = LlamaShape(**LLAMA3_8B, bits=8, group_size=64)
    _check(run_parity(shape, B=1, ctx=512, steps=128, dev=cuda), "cfg3 8-bit")
