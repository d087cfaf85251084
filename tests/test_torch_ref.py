"""Pins ``tests/fullsize.TorchRef`` (the float64 torch restatement used by the
full-size GPU parity tests) and its torch sharder to the numpy oracle, on
CPU: same logits and hidden states to float64 round-off, same greedy tokens,
same shard tensors."""

import numpy as np
import pytest
import torch

from oracle import sharder as osh
from oracle import synth
from oracle.tp import TPModel
from tests.fullsize import TorchRef, shard


def _torch_shard(sd):
    out = {}
    for k, v in sd.items():
        a = np.ascontiguousarray(v)
        if a.dtype == np.uint32:
            a = a.view(np.int32)
        out[k] = torch.from_numpy(a)
    return out


@pytest.mark.parametrize("world", [1, 2])
def test_torch_ref_matches_numpy_oracle(world):
    shape = synth.tiny_shape(num_layers=2, num_heads=8, num_kv_heads=4)
    full = synth.checkpoint(shape, seed=21)
    np_shards = [osh.shard_weights(full, world, r) for r in range(world)]
    ref = TPModel(np_shards, shape, max_len=64)
    tref = TorchRef([_torch_shard(s) for s in np_shards], shape, max_len=64, device=torch.device("cpu"))
    prompt = np.random.default_rng(5).integers(0, shape.vocab_size, size=(2, 6))
    lo, ho = ref.forward(prompt, return_hidden=True)
    lt, ht = tref.forward(torch.from_numpy(prompt), return_hidden=True)
    assert np.allclose(lt.numpy(), lo, rtol=1e-10, atol=1e-12)
    for a, b in zip(ht, ho):
        assert np.allclose(a.numpy(), b, rtol=1e-10, atol=1e-12)
    tok = np.argmax(lo[:, -1], axis=-1)[:, None]
    lo2 = ref.forward(tok)
    lt2 = tref.forward(torch.from_numpy(tok))
    assert np.allclose(lt2.numpy(), lo2, rtol=1e-10, atol=1e-12)


def test_torch_sharder_matches_oracle_sharder():
    shape = synth.tiny_shape(num_layers=1)
    full = synth.checkpoint(shape, seed=2)
    tfull = _torch_shard(full)
    for world in (2, 4):
        for r in range(world):
            a = osh.shard_weights(full, world, r)
            b = shard(tfull, world, r)
            assert sorted(a) == sorted(b)
            for k in a:
                av = np.ascontiguousarray(a[k])
                if av.dtype == np.uint32:
                    av = av.view(np.int32)
                assert np.array_equal(av, b[k].numpy()), k
