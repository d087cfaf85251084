"""Parity of the CUDA decode path at the headline configurations.

cfg3 (Llama-3-8B shapes, all 32 layers, 4-bit g64, tied head, full 128256
vocab): a 2048-token prompt (the KV length the benchmark decodes at), then
128 greedy decode steps through the CUDA-graph engine; cfg3 at batch 8 and
32 through the batched GEMV; the same model end to end in 8-bit.  The
reference is ``tests/fullsize.TorchRef`` (the numpy oracle's math in torch
float64 on the GPU, pinned to the oracle by ``tests/test_torch_ref.py``).

Tolerances (the path's contract): the hidden state after the embedding and
after every layer within 1e-3 relative L2 of the float64 reference (prefill
and the first decode step), and the one-kernel step's logits on every
decode step at batch 1; greedy tokens, each step teacher-forced with the
reference's previous token through the production decode step, agree on at
least 99 % of the decode steps.
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


def _engine(shape, shard, max_batch, max_seq, dev, world=1, rank=0, comm=None, one_kernel=False):
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    w = RankWeights.from_shard(cfg, shard, world, rank, shape.bits, shape.group_size, dev)
    return DecodeEngine(w, comm, max_batch=max_batch, max_seq=max_seq, device=dev, one_kernel_step=one_kernel)


def _layer_errors(hid_e, hid_r, B, S):
    return [rel_l2(e.view(B, S, -1), r) for e, r in zip(hid_e, hid_r)]


def run_parity(shape, B, ctx, steps, dev, seed=0, one_kernel=False):
    """Prefill + one decode step (per-layer hidden states), then `steps`
    greedy steps teacher-forced through the production decode step (each
    step fed the reference's previous token from pinned host memory, the
    graph replayed, its argmax read back), compared token by token with the
    float64 reference's argmax; at batch 1 (the one-kernel step) also that
    step's logits.  A free-running generate is reported beside it (its first
    divergence), not asserted: with random weights the top-2 logits of some
    steps sit closer than any fp32 path's error, and one flip changes every
    later token."""
    torch.manual_seed(seed)
    ckpt = gpu_checkpoint(shape, seed, dev)
    eng = _engine(shape, ckpt, B, ctx + 2 * steps + 8, dev, one_kernel=one_kernel)
    ref = TorchRef([ckpt], shape, max_len=ctx + steps + 8, device=dev)
    prompt = torch.randint(0, shape.vocab_size, (B, ctx), generator=torch.Generator().manual_seed(2))

    eng.reset()
    le, he = eng.forward_logits(prompt.to(dev), return_hidden=True)
    lr, hr = ref.forward(prompt, return_hidden=True)
    pre = _layer_errors(he, hr, B, ctx)
    pre_logits = rel_l2(le, lr)
    del le, he, hr

    toks_r = [lr[:, -1].argmax(-1)]
    gaps = [lr[:, -1].topk(2, dim=-1).values.diff(dim=-1).abs()[:, 0]]
    del lr
    le2, he2 = eng.forward_logits(toks_r[0][:, None].to(dev), return_hidden=True)
    lr2, hr2 = ref.forward(toks_r[0][:, None], return_hidden=True)
    dec = _layer_errors(he2, hr2, B, 1)
    dec_logits = rel_l2(le2, lr2)
    del le2, he2, hr2
    step_ref = [lr2[:, -1]]
    for _ in range(steps - 1):
        toks_r.append(step_ref[-1].argmax(-1))
        gaps.append(step_ref[-1].topk(2, dim=-1).values.diff(dim=-1).abs()[:, 0])
        if len(toks_r) < steps:
            step_ref.append(ref.forward(toks_r[-1][:, None])[:, -1])
    ref_tok = torch.stack(toks_r, dim=1).cpu().numpy()
    ref_gap = torch.stack(gaps, dim=1).cpu().numpy()
    del ref
    torch.cuda.empty_cache()

    # teacher-forced through the production step (CUDA graph; the one-kernel step at batch 1)
    eng.reset()
    eng.prefill(prompt.to(dev))
    forced = np.zeros_like(ref_tok)
    forced[:, 0] = eng.tok[:B].cpu().numpy()
    host_in = torch.zeros(B, dtype=torch.int32).pin_memory()
    host_out = torch.zeros(B, dtype=torch.int32).pin_memory()
    step_logit_err = []
    for t in range(1, steps):
        host_in.copy_(torch.from_numpy(ref_tok[:, t - 1].astype(np.int32)))
        eng.decode_host(host_in, host_out)
        forced[:, t] = host_out.numpy()
        if eng.use_step:
            step_logit_err.append(rel_l2(eng.step_logits.view(1, -1), step_ref[t - 1]))
    eng.check_step()
    agree = float(np.mean(forced == ref_tok))
    miss = forced != ref_tok

    out = eng.generate(prompt.to(dev), steps).cpu().numpy()
    diverge = [int(np.argmax(o != r)) if (o != r).any() else steps for o, r in zip(out, ref_tok)]
    return dict(prefill_layers=pre, prefill_logits=pre_logits, decode_layers=dec, decode_logits=dec_logits,
                agree=agree, tokens=forced, ref_tokens=ref_tok, miss_gaps=ref_gap[miss].tolist(),
                median_gap=float(np.median(ref_gap)), step_logits=step_logit_err, free_run_divergence=diverge)


def _check(res, name):
    sl = res["step_logits"]
    msg = (f"{name}: prefill max layer err {max(res['prefill_layers']):.2e} (logits {res['prefill_logits']:.2e}), "
           f"decode max layer err {max(res['decode_layers']):.2e} (logits {res['decode_logits']:.2e}), "
           f"teacher-forced greedy agreement {res['agree']:.4f} (reference top-2 gaps at the misses "
           f"{[round(g, 5) for g in res['miss_gaps'][:8]]}, median gap {res['median_gap']:.4f})"
           + (f", one-kernel step logits max err {max(sl):.2e}" if sl else "")
           + f", free-running first divergence {res['free_run_divergence'][:8]}")
    print(msg)
    assert max(res["prefill_layers"]) <= HIDDEN_TOL, msg + f"\nprefill per layer: {res['prefill_layers']}"
    assert res["prefill_logits"] <= HIDDEN_TOL, msg
    assert max(res["decode_layers"]) <= HIDDEN_TOL, msg + f"\ndecode per layer: {res['decode_layers']}"
    assert res["decode_logits"] <= HIDDEN_TOL, msg
    assert not sl or max(sl) <= HIDDEN_TOL, msg
    assert res["agree"] >= AGREE, msg + f"\n{res['tokens'][0, :24]}\n{res['ref_tokens'][0, :24]}"


@pytest.mark.parametrize("one_kernel", [False, True])
def test_cfg3_llama3_8b_32_layers_ctx2048(cuda, one_kernel):
    shape = LlamaShape(**LLAMA3_8B, bits=4, group_size=64)
    res = run_parity(shape, B=1, ctx=2048, steps=128, dev=cuda, one_kernel=one_kernel)
    assert bool(res["step_logits"]) == one_kernel
    _check(res, f"cfg3 b1 ctx2048 {'one-kernel' if one_kernel else 'per-kernel'} step")


@pytest.mark.parametrize("B", [8, 32])
def test_cfg3_llama3_8b_batched(cuda, B):
    shape = LlamaShape(**LLAMA3_8B, bits=4, group_size=64)
    _check(run_parity(shape, B=B, ctx=128, steps=32, dev=cuda), f"cfg3 b{B}")


def test_cfg3_llama3_8b_8bit(cuda):
    shape = LlamaShape(**LLAMA3_8B, bits=8, group_size=64)
    _check(run_parity(shape, B=1, ctx=512, steps=128, dev=cuda), "cfg3 8-bit")
