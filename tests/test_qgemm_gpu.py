"""K2, the tcgen05 tensor-core dequant-GEMM (``sc_qgemm``), against the float64
oracle: y = x . (s*q + b)^T with exact weights (the kernel carries w and x
as fp16 high + low parts, fp32 accumulation in TMEM), every epilogue,
4- and 8-bit codes, group sizes 32 / 64 / 128, partial tiles in both the
token and the weight-row dimension.  Tolerance: 2e-5 relative L2 (the
fp16-rounded-weight definition sits near 1.5e-4, rounding x to fp16 near
3e-4, so the bound separates them)."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import mlx_affine as qa
from oracle import tp as otp
from shardcompute_b200 import _lib as L
from shardcompute_b200 import ops
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-5


def _dev(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(dev)


def _qgemm(x, segs, group, bits, epi=L.SC_EPI_STORE, norm=None, eps=1e-5, bias=None, residual=None, out=None,
           out_dtype=torch.float32):
    lib = L.load()
    M, K = x.shape
    n = len(segs)
    rows = [int(s[0].shape[0]) for s in segs]
    N = rows[0] if epi == L.SC_EPI_SWIGLU else sum(rows)
    y = out if out is not None else torch.empty(M, N, dtype=out_dtype, device=x.device)
    W = (C.c_void_p * n)(*[s[0].data_ptr() for s in segs])
    S = (C.c_void_p * n)(*[s[1].data_ptr() for s in segs])
    B = (C.c_void_p * n)(*[s[2].data_ptr() for s in segs])
    R = (C.c_int * n)(*rows)
    nbytes = int(lib.sc_qgemm_workspace_bytes(M, K, N, epi))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    L.check(lib.sc_qgemm(x.data_ptr(), ops._dt(x), M, K, K, None if norm is None else norm.data_ptr(), eps, n,
                         C.cast(W, L._pp), C.cast(S, L._pp), C.cast(B, L._pp), R, group, bits,
                         None if bias is None else bias.data_ptr(), epi, y.data_ptr(), ops._dt(y), N,
                         None if residual is None else residual.data_ptr(), N if residual is not None else 0,
                         ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream), "sc_qgemm")
    return y


def _q(rng, N, K, bits, group):
    return qa.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float16), group, bits)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("M,K,N", [(5, 512, 128), (16, 1024, 384), (130, 4096, 256), (300, 512, 1000)])
def test_qgemm_matches_exact_product(cuda, bits, group, M, K, N):
    rng = np.random.default_rng(M * 7 + K + N + bits + group)
    wq, s, b = _q(rng, N, K, bits, group)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = _qgemm(_dev(x, cuda), [(_dev(wq, cuda), _dev(s, cuda), _dev(b, cuda))], group, bits).cpu().numpy()
    ref = qa.quantized_matmul(x, wq, s, b, group, bits)
    assert rel_l2(y, ref) <= TOL
    assert L.load().sc_qgemm_device_error(1) == 0


def test_qgemm_epilogues_and_segments(cuda):
    rng = np.random.default_rng(3)
    group, bits, K, M = 64, 4, 2048, 200
    # q | k | v segments (multiples of 128 rows but the last), norm prologue, bias
    segs = [_q(rng, n, K, bits, group) for n in (512, 128, 96)]
    h = rng.standard_normal((M, K)).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    bias = (0.1 * rng.standard_normal(736)).astype(np.float16)
    y = _qgemm(_dev(h, cuda), [tuple(_dev(a, cuda) for a in sg) for sg in segs], group, bits,
               norm=_dev(nw, cuda), bias=_dev(bias, cuda)).cpu().numpy()
    xn = otp.rmsnorm(h, nw, 1e-5)
    ref = np.concatenate([qa.quantized_matmul(xn, *sg, group, bits) for sg in segs], axis=1) + bias
    assert rel_l2(y, ref) <= TOL
    # residual, in place
    wq, s, b = _q(rng, 512, K, bits, group)
    res = rng.standard_normal((M, 512)).astype(np.float32)
    r_dev = _dev(res, cuda)
    _qgemm(_dev(h, cuda), [(_dev(wq, cuda), _dev(s, cuda), _dev(b, cuda))], group, bits, epi=L.SC_EPI_RESIDUAL,
           residual=r_dev, out=r_dev)
    assert rel_l2(r_dev.cpu().numpy(), res + qa.quantized_matmul(h, wq, s, b, group, bits)) <= TOL
    # SwiGLU pair
    g, u = _q(rng, 640, K, bits, group), _q(rng, 640, K, bits, group)
    y = _qgemm(_dev(h, cuda), [tuple(_dev(a, cuda) for a in g), tuple(_dev(a, cuda) for a in u)], group, bits,
               epi=L.SC_EPI_SWIGLU).cpu().numpy()
    ref = otp.silu(qa.quantized_matmul(h, *g, group, bits)) * qa.quantized_matmul(h, *u, group, bits)
    assert rel_l2(y, ref) <= TOL
    assert L.load().sc_qgemm_device_error(1) == 0


def test_qlinear_routes_many_rows_to_the_tensor_cores(cuda):
    """sc_qlinear with more rows than the decode GEMV serves gives the
    exact-weight product (the tensor-core GEMM), not the fp16-rounded one."""
    rng = np.random.default_rng(9)
    group, bits, K, N, M = 64, 4, 4096, 512, 64
    wq, s, b = _q(rng, N, K, bits, group)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = ops.qlinear(_dev(x, cuda), _dev(wq, cuda), _dev(s, cuda), _dev(b, cuda), group, bits,
                    out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, qa.quantized_matmul(x, wq, s, b, group, bits)) <= TOL
