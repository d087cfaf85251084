"""sc_qlinear_noalloc: the quantized linear with its split-K scratch in a
static device array.  Compared, through the C ABI, with sc_qlinear (caller
workspace) on two calls in a row, and on a shape too wide for the
tensor-core GEMM's scratch (it then runs decode-GEMV passes).  Named to
be collected last: it must pass both alone and after the other GPU tests."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import mlx_affine as qa
from shardcompute_b200 import _lib as L
from shardcompute_b200 import ops
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

SCRATCH = 4 << 20


def _dev(a, cuda):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(cuda)


def _noalloc(x, wq, s, b, group, bits, y):
    lib = L.load()
    M, K = x.shape
    N = wq.shape[0]
    return lib.sc_qlinear_noalloc(x.data_ptr(), ops._dt(x), M, K, K, wq.data_ptr(), s.data_ptr(), b.data_ptr(), N,
                                  group, bits, None, y.data_ptr(), ops._dt(y), N,
                                  torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,K,N,bits,group", [(1, 14336, 1024, 4, 64), (1, 4096, 6144, 4, 64),
                                              (3, 4096, 1024, 8, 32), (1, 256, 80, 4, 32)])
def test_noalloc_matches_workspace_entry_point(cuda, M, K, N, bits, group):
    rng = np.random.default_rng(7)
    wq, s, b = qa.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float16), group, bits)
    x = rng.standard_normal((M, K)).astype(np.float16)
    xd, wd, sd, bd = _dev(x, cuda), _dev(wq, cuda), _dev(s, cuda), _dev(b, cuda)
    ref = ops.qlinear(xd, wd, sd, bd, group, bits, out_dtype=torch.float32).cpu().numpy()
    exact = qa.quantized_matmul(x, wq, s, b, group, bits)
    # a call with other activations first, so the static scratch holds stale,
    # nonzero partials: a partial the checked calls failed to write would show
    stale = _dev(rng.standard_normal((M, K)).astype(np.float16) * 3, cuda)
    junk = torch.empty((M, N), dtype=torch.float32, device=cuda)
    assert _noalloc(stale, wd, sd, bd, group, bits, junk) == L.SC_OK, L.load().sc_last_error()
    for _ in range(2):  # two calls in a row reuse the same static scratch
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
        st = _noalloc(xd, wd, sd, bd, group, bits, y)
        assert st == L.SC_OK, L.load().sc_last_error()
        got = y.cpu().numpy()
        assert rel_l2(got, ref) <= 2e-5
        assert rel_l2(got, exact) <= 1e-3
    assert L.load().sc_qgemv_device_error(1) == 0


def test_noalloc_uses_the_scratch_for_split_k(cuda):
    """The first shape above is planned as split-K: its call enqueues the GEMV
    and the reduce kernel (two launches), and its partials live in the static
    scratch (a nonzero need that fits)."""
    lib = L.load()
    M, K, N, bits, group = 1, 14336, 1024, 4, 64
    assert 0 < lib.sc_qlinear_workspace_bytes(M, K, N, bits) <= SCRATCH
    rng = np.random.default_rng(3)
    wq, s, b = qa.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float16), group, bits)
    xd, wd, sd, bd = (_dev(a, cuda) for a in (rng.standard_normal((M, K)).astype(np.float16), wq, s, b))
    y = torch.empty((M, N), dtype=torch.float32, device=cuda)
    n0 = lib.sc_launch_count()
    assert _noalloc(xd, wd, sd, bd, group, bits, y) == L.SC_OK, lib.sc_last_error()
    assert lib.sc_launch_count() - n0 == 2, "expected a split-K GEMV plus its reduce kernel"
    torch.cuda.synchronize()
    exact = qa.quantized_matmul(xd.cpu().numpy(), wq, s, b, group, bits)
    assert rel_l2(y.cpu().numpy(), exact) <= 1e-3


def test_noalloc_runs_many_rows_as_gemv_passes(cuda):
    """More than 16 rows: the tensor-core GEMM's x parts and scratch (here
    4.5 MB) do not fit the 4 MiB static array, so the entry point runs
    decode-GEMV passes instead, whose split-K scratch stays far below it,
    and matches the exact product; the documented refusal (a plan needing
    more than 4 MiB) guards the limit."""
    M, K, N, bits, group = 48, 14336, 1024, 4, 64
    rng = np.random.default_rng(11)
    wq, s, b = qa.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float16), group, bits)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
    st = _noalloc(_dev(x, cuda), _dev(wq, cuda), _dev(s, cuda), _dev(b, cuda), group, bits, y)
    assert st == 0, L.load().sc_last_error().decode()
    exact = qa.quantized_matmul(x, wq, s, b, group, bits)
    assert rel_l2(y.cpu().numpy(), exact) <= 1e-3
    assert L.load().sc_qgemv_device_error(1) == 0
