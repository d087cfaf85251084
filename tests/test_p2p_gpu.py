"""NVLink peer-memory collectives (sc_p2p_*): bounded wait on one GPU, and
all-reduce / all-gather parity across 2 (and 4) GPUs.

The all-reduce sums in rank order with fp32 accumulation, so its results are
compared bit for bit with the same sum on the CPU; the all-gather is a copy
and compared exactly.  Messages cover odd counts (partial 16-byte lines),
in-place calls, alternating sizes (per-block epochs and the double-buffered
regions), CUDA-graph replays, and messages above the transport limit (NCCL).
"""

import ctypes as C
import os
import socket
import sys
import time
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_wait_for_silent_peer_times_out(cuda):
    """A rank whose peer never sends: every wait gives up after the timeout,
    the status flips to 1 without a GPU call, later calls return at once and
    the context stays usable."""
    from shardcompute_b200 import _lib as L

    lib = L.load()
    hb = int(lib.sc_p2p_handle_bytes())
    h = C.c_void_p()
    buf = (C.c_char * hb)()
    L.check(lib.sc_p2p_create(2, 0, 1 << 16, C.byref(h), buf, hb), "create")
    try:
        L.check(lib.sc_p2p_open_loopback(h), "loopback")
        L.check(lib.sc_p2p_set_timeout(h, 50_000_000), "timeout")  # 50 ms
        st = C.c_int(-1)
        L.check(lib.sc_p2p_status(h, C.byref(st)), "status")
        assert st.value == 0
        x = torch.arange(1000, dtype=torch.float32, device=cuda)
        y = torch.empty_like(x)
        stream = torch.cuda.current_stream(cuda).cuda_stream
        t0 = time.perf_counter()
        L.call("sc_p2p_allreduce", x.data_ptr(), y.data_ptr(), x.numel(), L.SC_F32, h, stream)
        torch.cuda.synchronize(cuda)
        first = time.perf_counter() - t0
        L.check(lib.sc_p2p_status(h, C.byref(st)), "status")
        assert st.value == 1
        assert 0.04 < first < 5.0, first
        t0 = time.perf_counter()
        for _ in range(3):
            L.call("sc_p2p_allreduce", x.data_ptr(), y.data_ptr(), x.numel(), L.SC_F32, h, stream)
        torch.cuda.synchronize(cuda)
        assert time.perf_counter() - t0 < 0.04  # sticky error: no further waiting
        assert float((x * 2).sum()) == 999000.0  # the context still runs work
        with pytest.raises(ValueError):
            L.call("sc_p2p_allreduce", x.data_ptr(), y.data_ptr(), 1 << 15, L.SC_F32, h, stream)  # > limit
        with pytest.raises(NotImplementedError):
            L.call("sc_p2p_allreduce", x.data_ptr(), y.data_ptr(), 4, L.SC_I32, h, stream)
    finally:
        L.check(lib.sc_p2p_destroy(h), "destroy")


def _inputs(rank, it, n, dtype):
    g = np.random.default_rng(1000 * it + rank)
    if dtype == torch.int32:
        return torch.from_numpy(g.integers(-2**31, 2**31 - 1, size=n, dtype=np.int64).astype(np.int32))
    v = g.standard_normal(n).astype(np.float32)
    return torch.from_numpy(v).to(dtype)


def _ref_sum(world, it, n, dtype):
    acc = np.zeros(n, dtype=np.float32)
    for q in range(world):
        acc = acc + _inputs(q, it, n, dtype).float().numpy()  # rank order, fp32
    return torch.from_numpy(acc).to(dtype)


def _rank_main(rank, world, port, q):
    try:
        sys.path.insert(0, ROOT)
        import torch

        from shardcompute_b200.collectives import Communicator

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        comm = Communicator(rank, world, host="127.0.0.1", port=port, backend="nccl")
        comm.initialize_sync(timeout=60)
        assert comm.p2p_enabled, "peer-memory transport not set up"
        limit = comm._p2p_max
        it = 0
        cases = [(1, torch.float32), (3, torch.float16), (7, torch.float32), (4096, torch.float32),
                 (4096, torch.float16), (16389, torch.float32), (5, torch.float16), (limit // 4, torch.float32),
                 (limit // 2, torch.float16), (limit // 4 + 1, torch.float32), (2, torch.float32)]
        for rep in range(2):
            for n, dt in cases:
                it += 1
                x = _inputs(rank, it, n, dt).to(dev)
                out = torch.empty_like(x)
                if rep == 1:
                    out = x  # in place
                comm.allreduce_into(x, out)
                ref = _ref_sum(world, it, n, dt)
                got = out.cpu()
                if n * x.element_size() <= limit:
                    assert torch.equal(got.view(torch.int16) if dt == torch.float16 else got.view(torch.int32),
                                       ref.view(torch.int16) if dt == torch.float16 else ref.view(torch.int32)), \
                        f"allreduce n={n} {dt} rep={rep}"
                else:  # NCCL path: its own summation order
                    assert torch.allclose(got.float(), ref.float(), rtol=1e-5, atol=1e-5)
        for n, dt in [(1, torch.int32), (2, torch.float32), (3, torch.int32), (5000, torch.float32),
                      (limit // 4, torch.int32)]:
            it += 1
            x = _inputs(rank, it, n, dt).to(dev)
            out = torch.empty((world, n), dtype=dt, device=dev)
            comm.allgather_into(x, out)
            ref = torch.stack([_inputs(r, it, n, dt) for r in range(world)])
            assert torch.equal(out.cpu(), ref), f"allgather n={n} {dt}"
        # graph replays: two all-reduces and an all-gather per replay, fresh data each time
        xs = torch.empty(4096, dtype=torch.float32, device=dev)
        ys = torch.empty_like(xs)
        zs = torch.empty((world, 3), dtype=torch.int32, device=dev)
        ids = torch.empty(3, dtype=torch.int32, device=dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            comm.allreduce_into(xs, ys)
            comm.allreduce_into(ys, ys)
            comm.allgather_into(ids, zs)
        for r in range(20):
            it += 1
            xs.copy_(_inputs(rank, it, 4096, torch.float32))
            ids.fill_(rank * 100 + r)
            graph.replay()
            part = _ref_sum(world, it, 4096, torch.float32).numpy()
            ref = np.zeros_like(part)
            for _ in range(world):  # the in-place second all-reduce sums identical partials
                ref = ref + part
            np.testing.assert_array_equal(ys.cpu().numpy(), ref)
            assert zs[:, 0].tolist() == [q * 100 + r for q in range(world)]
        del graph
        torch.cuda.synchronize(dev)
        assert comm.poll() == 0
        comm.shutdown_sync()
        q.put((rank, "ok"))
    except BaseException:  # noqa: BLE001 - report to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_p2p_collectives_match_cpu(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    bad = {r: m for r, m in res.items() if m != "ok"}
    assert not bad, "\n".join(f"rank {r}:\n{m}" for r, m in bad.items())
