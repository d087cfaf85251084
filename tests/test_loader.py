"""Direct safetensors -> device loading (``shardcompute_b200.model.loader``)
against the ``safetensors`` package's own reader: every tensor bit-equal,
dtypes and shapes kept (packed ``U32`` words as ``int32`` of the same
bytes), 256-byte aligned placement, tensors split across staging chunks;
then a rank shard in the reference's directory layout loaded on the GPU
gives the same model output as the in-memory shard."""

import os

import numpy as np
import pytest
import torch

from shardcompute_b200.model.loader import load_rank_shard, load_safetensors, read_header


def _write(path, tensors):
    from safetensors.numpy import save_file

    save_file(tensors, path)


def _mixed(rng):
    return {
        "model.embed_tokens.weight": rng.integers(0, 2**32, size=(33, 7), dtype=np.uint32),
        "model.embed_tokens.scales": rng.standard_normal((33, 1)).astype(np.float16),
        "odd.f16": rng.standard_normal((3, 5)).astype(np.float16),  # 30 bytes
        "vec.f32": rng.standard_normal(11).astype(np.float32),
        "ids.i64": rng.integers(-5, 5, size=(2, 3), dtype=np.int64),
        "scalar.f32": np.array(1.25, dtype=np.float32),
        "bytes.u8": rng.integers(0, 255, size=(17,), dtype=np.uint8),
        "big.f16": rng.standard_normal((300, 200)).astype(np.float16),  # 120 KB: several chunks
    }


@pytest.mark.parametrize("chunk", [1 << 16, 1 << 20])
def test_load_matches_the_safetensors_reader(tmp_path, chunk):
    from safetensors.numpy import load_file

    rng = np.random.default_rng(0)
    path = str(tmp_path / "m.safetensors")
    _write(path, _mixed(rng))
    ref = load_file(path)
    got = load_safetensors(path, "cpu", chunk_bytes=chunk)
    assert set(got) == set(ref)
    base = next(iter(got.values())).untyped_storage().data_ptr()
    for name, r in ref.items():
        t = got[name]
        assert tuple(t.shape) == r.shape, name
        a = t.numpy()
        if r.dtype == np.uint32:
            assert t.dtype == torch.int32
            a = a.view(np.uint32)
        assert a.dtype == r.dtype, name
        assert np.array_equal(a, r), name
        assert (t.data_ptr() - base) % 256 == 0, name


def test_subset_and_header_checks(tmp_path):
    rng = np.random.default_rng(1)
    path = str(tmp_path / "m.safetensors")
    _write(path, _mixed(rng))
    entries, data0 = read_header(path)
    assert data0 > 8 and "odd.f16" in entries
    got = load_safetensors(path, "cpu", names=["vec.f32", "odd.f16"])
    assert set(got) == {"vec.f32", "odd.f16"}
    with pytest.raises(KeyError):
        load_safetensors(path, "cpu", names=["nope"])
    bad = str(tmp_path / "bad.safetensors")
    with open(bad, "wb") as f:
        f.write(b"\x01\x02")
    with pytest.raises(ValueError):
        load_safetensors(bad, "cpu")


def _tiny_shards(tmp_path, world=2):
    from oracle import sharder as osh
    from oracle import synth

    shape = synth.tiny_shape(num_layers=2)
    full = synth.checkpoint(shape, seed=6)
    shards = [osh.shard_weights(full, world, r) for r in range(world)]
    for r, sh in enumerate(shards):
        d = tmp_path / f"rank_{r}"
        d.mkdir()
        _write(str(d / "model.safetensors"), {k: np.ascontiguousarray(v) for k, v in sh.items()})
    return shape, shards


def test_rank_shard_directory_layout(tmp_path):
    shape, shards = _tiny_shards(tmp_path)
    for r in range(2):
        got = load_rank_shard(str(tmp_path), r, "cpu")
        assert set(got) == set(shards[r])
        for k, v in shards[r].items():
            a = got[k].numpy()
            if v.dtype == np.uint32:
                a = a.view(np.uint32)
            assert np.array_equal(a, v), k
    with pytest.raises(FileNotFoundError):
        load_rank_shard(str(tmp_path), 5, "cpu")


@pytest.mark.gpu
def test_device_load_gives_the_same_model_output(cuda, tmp_path):
    from oracle import synth
    from shardcompute_b200.model.config import ModelConfig
    from shardcompute_b200.parallel.decode_engine import DecodeEngine
    from shardcompute_b200.parallel.weights import RankWeights

    shape, shards = _tiny_shards(tmp_path, world=1)
    cfg = ModelConfig.from_dict(synth.model_config_dict(shape))
    a = RankWeights.from_shard(cfg, shards[0], 1, 0, shape.bits, shape.group_size, cuda)
    b = RankWeights.from_safetensors(cfg, str(tmp_path), 1, 0, shape.bits, shape.group_size, cuda)
    for ta, tb in zip(a.tensors(), b.tensors()):
        assert tb.is_cuda and torch.equal(ta, tb)
    prompt = torch.from_numpy(np.random.default_rng(3).integers(0, shape.vocab_size, size=(1, 9))).to(cuda)
    outs = []
    for w in (a, b):
        eng = DecodeEngine(w, None, max_batch=1, max_seq=48, device=cuda)
        outs.append(eng.generate(prompt, 12).cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
