"""Communicator host logic at world size 2 on CPU (gloo backend).

Restates the reference's collective tests (tests/test_collectives.py:69-249:
sum / mean / max all-reduce, 2-D tensors, all-gather on dim 0 and the last
dim, random tensors against numpy) plus the control ops the worker loop uses
(broadcast, barrier, send/recv, reduce-scatter, batched and split-phase
all-reduce), and one tensor-parallel step: a quantized row-parallel linear
whose per-rank partials are all-reduced (parallel/quantized_linear.py:419-455).
Each case runs as two spawned processes rendezvousing on 127.0.0.1.
"""

import asyncio
import datetime
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    try:
        sys.path.insert(0, ROOT)
        from shardcompute_b200.collectives import Communicator

        comm = Communicator(rank, world, host="127.0.0.1", port=port, backend="gloo")
        comm.initialize_sync(timeout=60)
        asyncio.run(CASES[case](comm, rank, world))
        comm.shutdown_sync()
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException:  # noqa: BLE001 - report any failure to the parent
        q.put((rank, traceback.format_exc()))


def _run(case, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in ps:
        p.start()
    results = {}
    for _ in ps:
        r, msg = q.get(timeout=120)
        results[r] = msg
    for p in ps:
        p.join(timeout=30)
    bad = {r: m for r, m in results.items() if m != "ok"}
    assert not bad, "\n".join(f"rank {r}:\n{m}" for r, m in bad.items())


# ---------------------------------------------------------------- cases (run inside the ranks)

async def case_all_reduce_ops(comm, rank, world):
    t = torch.tensor([1.0, 2.0, 3.0]) if rank == 0 else torch.tensor([4.0, 5.0, 6.0])
    assert torch.allclose(await comm.all_reduce(t, "sum"), torch.tensor([5.0, 7.0, 9.0]))
    t = torch.tensor([2.0, 4.0]) if rank == 0 else torch.tensor([6.0, 8.0])
    assert torch.allclose(await comm.all_reduce(t, "mean"), torch.tensor([4.0, 6.0]))
    t = torch.tensor([1.0, 5.0, 3.0]) if rank == 0 else torch.tensor([4.0, 2.0, 6.0])
    assert torch.allclose(await comm.all_reduce(t, "max"), torch.tensor([4.0, 5.0, 6.0]))
    t = torch.tensor([[1.0, 2.0], [3.0, 4.0]]) if rank == 0 else torch.tensor([[5.0, 6.0], [7.0, 8.0]])
    out = await comm.all_reduce(t, "sum")
    assert out.shape == (2, 2) and torch.allclose(out, torch.tensor([[6.0, 8.0], [10.0, 12.0]]))
    with pytest.raises(ValueError):
        await comm.all_reduce(t, "prod")


async def case_all_reduce_random(comm, rank, world):
    parts = [np.random.default_rng(100 + r).standard_normal((10, 20)).astype(np.float32) for r in range(world)]
    out = await comm.all_reduce(torch.from_numpy(parts[rank]), "sum")
    np.testing.assert_allclose(out.numpy(), parts[0] + parts[1], rtol=1e-5)


async def case_all_gather(comm, rank, world):
    t = torch.tensor([1.0, 2.0]) if rank == 0 else torch.tensor([3.0, 4.0])
    out = await comm.all_gather(t, dim=0)
    assert torch.equal(out, torch.tensor([1.0, 2.0, 3.0, 4.0]))
    t = torch.tensor([[[1.0, 2.0], [3.0, 4.0]]]) if rank == 0 else torch.tensor([[[5.0, 6.0], [7.0, 8.0]]])
    out = await comm.all_gather(t, dim=-1)
    assert out.shape == (1, 2, 4)
    assert torch.equal(out, torch.tensor([[[1.0, 2.0, 5.0, 6.0], [3.0, 4.0, 7.0, 8.0]]]))
    assert comm.get_stats()["total_all_gather_calls"] == 2


async def case_control_ops(comm, rank, world):
    b = await comm.broadcast(torch.arange(6, dtype=torch.float32).view(2, 3) if rank == 0 else None, root=0)
    assert torch.equal(b, torch.arange(6, dtype=torch.float32).view(2, 3))
    await comm.barrier()
    if rank == 0:
        await comm.send(torch.tensor([7, 8, 9], dtype=torch.int32), dest=1)
        got = await comm.recv(source=1)
        assert torch.equal(got, torch.tensor([1.5, 2.5]))
    else:
        got = await comm.recv(source=0)
        assert torch.equal(got, torch.tensor([7, 8, 9], dtype=torch.int32))
        await comm.send(torch.tensor([1.5, 2.5]), dest=0)
    rs = await comm.reduce_scatter(torch.ones(4, 6) * (rank + 1), dim=-1)
    assert rs.shape == (4, 3) and torch.allclose(rs, torch.full((4, 3), 3.0))
    outs = await comm.all_reduce_batch([torch.ones(3) * (rank + 1), torch.ones(2, 2)])
    assert torch.allclose(outs[0], torch.full((3,), 3.0)) and torch.allclose(outs[1], torch.full((2, 2), 2.0))
    op = comm.start_all_reduce(torch.full((5,), float(rank)))
    assert torch.allclose(await comm.wait_all_reduce(op), torch.full((5,), 1.0))
    with pytest.raises(ValueError):
        await comm.wait_all_reduce("nope")
    with pytest.raises(ValueError):
        await comm.send(torch.ones(1), dest=rank)


async def case_row_parallel_quantized(comm, rank, world):
    """K-split quantized linear: partial per rank, all-reduce, bias once (rank 0)."""
    from oracle import mlx_affine as qa
    from oracle import sharder as osh

    rng = np.random.default_rng(5)
    K, N, g = 512, 128, 64
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    wq, s, b = qa.quantize(w, g, 4)
    bias = rng.standard_normal(N)
    x = rng.standard_normal((2, K))
    full = qa.quantized_matmul(x, wq, s, b, g, 4) + bias
    sw, ss, sb = osh.shard_quantized("model.layers.0.self_attn.o_proj.weight", wq, s, b, world, rank)
    kl = K // world
    part = qa.quantized_matmul(x[:, rank * kl:(rank + 1) * kl], sw, ss, sb, g, 4)
    out = (await comm.all_reduce(torch.from_numpy(part), "sum")).numpy()
    if rank == 0:
        out = out + bias
        np.testing.assert_allclose(out, full, rtol=1e-9, atol=1e-12)


CASES = {f.__name__[5:]: f for f in (case_all_reduce_ops, case_all_reduce_random, case_all_gather, case_control_ops,
                                       case_row_parallel_quantized)}


@pytest.mark.parametrize("case", sorted(CASES))
def test_world2(case):
    _run(case)


def test_missing_peer_times_out():
    """A rank whose peer never joins fails the rendezvous within its timeout
    instead of hanging (host-side failure detection)."""
    from shardcompute_b200.collectives import Communicator

    comm = Communicator(0, 2, host="127.0.0.1", port=_free_port(), backend="gloo")
    t0 = datetime.datetime.now()
    with pytest.raises(Exception):
        comm.initialize_sync(timeout=2)
    assert (datetime.datetime.now() - t0).total_seconds() < 60
    assert not comm.is_initialized


def test_uninitialized_raises():
    from shardcompute_b200.collectives import Communicator

    comm = Communicator(0, 2, backend="gloo")
    with pytest.raises(RuntimeError, match="Communicator not initialized"):
        asyncio.run(comm.all_reduce(torch.ones(2)))
