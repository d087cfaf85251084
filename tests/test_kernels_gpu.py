"""Parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Tolerances:
* unpack / dequantize / embedding gather / quantize: bit-exact;
* quantized matmul: relative L2 <= 1e-3 against the oracle's exact-dequant
  float64 product, and <= 2e-5 against the
  float64 product the kernel is defined on: exact weights for the decode
  kernel (scale * sum(q x) + bias * sum(x) with x split into fp16 high and
  low parts), fp16-dequantized weights for the batched kernel (checks the
  in-register arithmetic is exact and accumulation is fp32);
* attention: relative L2 <= 1e-4 against the float64 oracle.
"""

import math

import numpy as np
import pytest
import torch

from oracle import mlx_affine as qa
from oracle import tp as otp
from shardcompute_b200 import _lib as L
from shardcompute_b200 import ops
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu


def make_q(rng, N, K, bits, group, std=0.02):
    w = (rng.standard_normal((N, K)) * std).astype(np.float16)
    return qa.quantize(w, group, bits)


def to_dev(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(dev)


def ref16(x, wq, s, b, group, bits):
    return np.asarray(x, np.float64) @ qa.dequantize(wq, s, b, group, bits).astype(np.float64).T


def ref_exact(x, wq, s, b, group, bits):
    return np.asarray(x, np.float64) @ qa.dequantize_exact(wq, s, b, group, bits).T


def assert_kernel_close(y, refs, tol):
    """The decode kernel (M * groups-per-chunk <= 4) keeps the weights exact;
    the batched kernel rounds them once to fp16 (``mx.dequantize``).  Both
    carry x to ~22 bits (fp16 high + low parts).  ``refs`` holds the float64
    product for each definition; the output must match one of them."""
    y = np.asarray(y)
    rows = y.reshape(-1, y.shape[-1])
    refs = [np.asarray(r).reshape(rows.shape) for r in refs]
    # a pass of up to 16 rows runs one kernel, so each row matches one definition
    for m in range(rows.shape[0]):
        errs = [rel_l2(rows[m], r[m]) for r in refs]
        assert min(errs) <= tol, (m, errs)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("M,K,N", [(1, 256, 80), (3, 512, 48), (8, 1024, 200), (9, 384, 33),
                                   (16, 2048, 64), (17, 256, 40), (1, 4096, 1024)])
def test_qlinear_matches_oracle(cuda, rng, bits, group, M, K, N):
    if K % group:
        pytest.skip("K not a multiple of group")
    wq, s, b = make_q(rng, N, K, bits, group)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = ops.qlinear(to_dev(x, cuda), to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda), group, bits,
                    out_dtype=torch.float32)
    y = y.cpu().numpy()
    ref = qa.quantized_matmul(x, wq, s, b, group, bits)
    assert rel_l2(y, ref) <= 1e-3
    # 5e-5 (the fp16-rounded-weight definition sits near 2e-4): the decode GEMV's mma
    # accumulates (1024 + q) * x against a -1024 * sum(x) start, so fp32 rounding is
    # magnified ~70x before the offset cancels
    assert_kernel_close(y, [ref, ref16(x, wq, s, b, group, bits)], 5e-5)
    assert L.load().sc_qgemv_device_error(1) == 0


@pytest.mark.parametrize("bits", [4, 8])
def test_qlinear_edge_shapes(cuda, rng, bits):
    # K with a partial last chunk, N not a multiple of 16, tiny N forcing split-K,
    # and Llama-like shapes on both kernels (direct-load and TMA)
    for (M, K, N) in [(1, 96, 7), (2, 160, 1), (5, 4096 + 64, 16), (1, 14336, 24), (4, 8192, 130),
                      (1, 1792, 300), (2, 14336, 100), (1, 4096, 6144)]:
        group = 32
        wq, s, b = make_q(rng, N, K, bits, group)
        x = rng.standard_normal((M, K)).astype(np.float16)
        bias = (rng.standard_normal(N) * 0.1).astype(np.float16)
        y = ops.qlinear(to_dev(x, cuda), to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda), group, bits,
                        bias=to_dev(bias, cuda), out_dtype=torch.float32).cpu().numpy()
        # fp32 accumulation over K terms: the bound grows like sqrt(K) past K = 4096
        # (the tensor-core GEMM takes M > 1 with 32-groups; its fp32 accumulator
        # sums K = 14336 products in 224 MMAs)
        assert_kernel_close(y, [ref16(x, wq, s, b, group, bits) + bias, ref_exact(x, wq, s, b, group, bits) + bias],
                            2e-5 * max(1.0, (K / 4096) ** 0.5))


def test_qlinear_rejects_bad_shapes(cuda, rng):
    wq, s, b = make_q(rng, 32, 128, 4, 64)
    x = torch.zeros(1, 64, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        ops.qlinear(x, to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda), 64, 4)
    x = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        ops.qlinear(x, to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda), 48, 4)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("rows", [[64, 24, 24], [512, 128, 128]])
def test_qlinear_fused_segments_norm_residual(cuda, rng, bits, rows):
    K, group, M, eps = 512, 64, 3, 1e-5
    segs = [make_q(rng, n, K, bits, group) for n in rows]
    h = rng.standard_normal((M, K)).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    y = ops.qlinear_fused(to_dev(h, cuda), [tuple(to_dev(a, cuda) for a in sg) for sg in segs], group, bits,
                          norm_weight=to_dev(nw, cuda), eps=eps).cpu().numpy()
    xn64 = otp.rmsnorm(h, nw, eps)
    ref = np.concatenate([ref16(xn64, *sg, group, bits) for sg in segs], axis=1)
    ref_x = np.concatenate([ref_exact(xn64, *sg, group, bits) for sg in segs], axis=1)
    # x is normalised in fp32 and carried as fp16 high + low parts
    assert_kernel_close(y, [ref, ref_x], 5e-5)
    # residual epilogue, in place
    for K2 in (256, 4096):
        wq, s, b = make_q(rng, K, K2, bits, group)
        x = rng.standard_normal((M, K2)).astype(np.float16)
        res = rng.standard_normal((M, K)).astype(np.float32)
        r_dev = to_dev(res, cuda)
        ops.qlinear_fused(to_dev(x, cuda), [(to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda))], group, bits,
                          epilogue=L.SC_EPI_RESIDUAL, residual=r_dev, out=r_dev)
        assert_kernel_close(r_dev.cpu().numpy(), [res + ref16(x, wq, s, b, group, bits),
                                                  res + ref_exact(x, wq, s, b, group, bits)], 5e-5)


@pytest.mark.parametrize("M", [1, 4, 12])
@pytest.mark.parametrize("K,F", [(1024, 352), (4096, 1024)])
def test_qlinear_swiglu(cuda, rng, M, K, F):
    group, bits = 64, 4
    g = make_q(rng, F, K, bits, group)
    u = make_q(rng, F, K, bits, group)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = ops.qlinear_fused(to_dev(x, cuda), [tuple(to_dev(a, cuda) for a in g), tuple(to_dev(a, cuda) for a in u)],
                          group, bits, epilogue=L.SC_EPI_SWIGLU, out_dtype=torch.float32).cpu().numpy()
    refs = [otp.silu(f(x, *g, group, bits)) * f(x, *u, group, bits) for f in (ref16, ref_exact)]
    # the product of two GEMV outputs doubles their relative error
    assert_kernel_close(y, refs, 1e-4)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [3, 8, 16, 21])
def test_batched_kernel_fp32_input_keeps_x(cuda, rng, bits, M):
    """fp32 activations in batches: up to 16 rows run decode-GEMV passes
    (exact weights, x carried as fp16 high + low parts), more run the
    tensor-core GEMM (the same definition); the product matches the float64
    exact-weight one to 5e-5, where rounding x to fp16 alone sits near 3e-4
    and rounding the weights to fp16 near 2e-4."""
    K, N, group = 4096, 512, 64
    wq, s, b = make_q(rng, N, K, bits, group)
    x = rng.standard_normal((M, K)).astype(np.float32)
    for epi in ("store", "residual"):
        if epi == "store":
            y = ops.qlinear_fused(to_dev(x, cuda), [(to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda))], group,
                                  bits, out_dtype=torch.float32).cpu().numpy()
            refs = [ref16(x, wq, s, b, group, bits), ref_exact(x, wq, s, b, group, bits)]
        else:
            res = rng.standard_normal((M, N)).astype(np.float32)
            r_dev = to_dev(res, cuda)
            ops.qlinear_fused(to_dev(x, cuda), [(to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda))], group, bits,
                              epilogue=L.SC_EPI_RESIDUAL, residual=r_dev, out=r_dev)
            y = r_dev.cpu().numpy()
            refs = [res + ref16(x, wq, s, b, group, bits), res + ref_exact(x, wq, s, b, group, bits)]
        assert_kernel_close(y, refs, 5e-5)
    assert L.load().sc_qgemv_device_error(1) == 0


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("M", [1, 2, 4])
def test_decode_kernel_exact_weights_fp32_input(cuda, rng, bits, group, M):
    """fp32 activations through the decode kernel: weights exact and x carried
    as fp16 high + low parts, so the product matches float64 to a few 1e-5
    (the fp16-rounding kernel sits near 1e-4).  The bound allows for the low
    parts of small |x| landing in the fp16 subnormal range, most of all in
    the x/16 slots of odd 4-bit codes; |x| here spans e^-3 .. e^3."""
    K, N = 4096, 1024
    ngc = max(1, (128 if bits == 4 else 64) // group)
    if M * ngc > 4:
        pytest.skip("batched kernel")
    wq, s, b = make_q(rng, N, K, bits, group)
    x = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-3, 3, size=(M, K)))).astype(np.float32)
    y = ops.qlinear_fused(to_dev(x, cuda), [(to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda))], group, bits,
                          out_dtype=torch.float32).cpu().numpy()
    ref = ref_exact(x, wq, s, b, group, bits)
    assert rel_l2(y, ref) <= 5e-5
    assert L.load().sc_qgemv_device_error(1) == 0


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_dequantize_and_embedding_bit_exact(cuda, rng, bits, group):
    V, H = 300, 512
    wq, s, b = make_q(rng, V, H, bits, group, std=0.5)
    dq = ops.dequantize(to_dev(wq, cuda), to_dev(s, cuda), to_dev(b, cuda), group, bits).cpu().numpy()
    assert np.array_equal(dq.view(np.uint16), qa.dequantize(wq, s, b, group, bits).view(np.uint16))
    world, rank = 3, 1
    v0, v1 = 100, 200
    ids = np.array([[0, 99, 100, 150], [199, 200, 299, 123]], dtype=np.int32)
    e = ops.embed_gather_q(to_dev(ids, cuda), to_dev(wq[v0:v1], cuda), to_dev(s[v0:v1], cuda),
                           to_dev(b[v0:v1], cuda), v0, v1, H, group, bits).cpu().numpy()
    cfg = otp.LlamaShape(vocab_size=V, hidden_size=H, num_layers=0, num_heads=1, num_kv_heads=1,
                         intermediate_size=1, bits=bits, group_size=group)
    shard = {"model.embed_tokens.weight": wq[v0:v1], "model.embed_tokens.scales": s[v0:v1],
             "model.embed_tokens.biases": b[v0:v1]}
    ref = otp.embed_rank(ids, shard, cfg, world, rank)
    assert np.array_equal(e.view(np.uint16), ref.view(np.uint16))


def test_embedding_f16_rows(cuda, rng):
    V, H = 64, 136
    table = rng.standard_normal((V, H)).astype(np.float16)
    ids = rng.integers(0, 3 * V, size=(3, 5)).astype(np.int32)
    v0, v1 = V, 2 * V
    e = ops.embed_gather_f16(to_dev(ids, cuda), to_dev(table, cuda), v0, v1).cpu().numpy()
    ref = np.where(((ids >= v0) & (ids < v1))[..., None], table[np.clip(ids - v0, 0, V - 1)], np.float16(0))
    assert np.array_equal(e.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_bit_exact(cuda, rng, bits):
    w = (rng.standard_normal((40, 256)) * 0.02).astype(np.float16)
    w[3, :64] = np.float16(0.25)  # a constant group
    wq, s, b = ops.quantize(to_dev(w, cuda), 64, bits)
    rq, rs, rb = qa.quantize(w, 64, bits)
    assert np.array_equal(wq.cpu().numpy().view(np.uint32), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))
    assert np.array_equal(b.cpu().numpy().view(np.uint16), rb.view(np.uint16))


@pytest.mark.parametrize("hd,Hq,Hkv", [(128, 8, 2), (64, 8, 1), (128, 4, 4), (64, 4, 2)])
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_rope_append_and_flash_decode(cuda, rng, hd, Hq, Hkv, splits):
    B, Lmax, past, S = 2, 96, 37, 1
    cos, sin = otp.rope_tables(hd, 128, 10000.0)
    k_cache = torch.zeros(B, Hkv, Lmax, hd, dtype=torch.float32, device=cuda)
    v_cache = torch.zeros_like(k_cache)
    kp = (rng.standard_normal((B, Hkv, past, hd))).astype(np.float32)
    vp = (rng.standard_normal((B, Hkv, past, hd))).astype(np.float32)
    k_cache[:, :, :past] = torch.from_numpy(kp).to(cuda)
    v_cache[:, :, :past] = torch.from_numpy(vp).to(cuda)
    qkv = rng.standard_normal((B * S, (Hq + 2 * Hkv) * hd)).astype(np.float32)
    pos = torch.tensor([past], dtype=torch.int32, device=cuda)
    q_out = torch.empty(B * S, Hq * hd, dtype=torch.float32, device=cuda)
    ops.rope_append(to_dev(qkv, cuda), B, S, Hq, Hkv, hd, pos, to_dev(cos, cuda), to_dev(sin, cuda), q_out,
                    k_cache, v_cache)
    out = torch.empty(B * S, Hq * hd, dtype=torch.float32, device=cuda)
    ops.flash_decode(q_out, k_cache, v_cache, pos, B, S, Hq, Hkv, hd, splits, out)
    q = qkv[:, :Hq * hd].reshape(B, S, Hq, hd).transpose(0, 2, 1, 3)
    k = qkv[:, Hq * hd:(Hq + Hkv) * hd].reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
    v = qkv[:, (Hq + Hkv) * hd:].reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
    qr = otp.apply_rope(q, cos[past:past + S], sin[past:past + S])
    kr = otp.apply_rope(k, cos[past:past + S], sin[past:past + S])
    assert rel_l2(q_out.cpu().numpy().reshape(B, S, Hq, hd).transpose(0, 2, 1, 3), qr) <= 1e-6
    # the cache holds the fp32 rotation (fp32 arithmetic against the float64 oracle)
    np.testing.assert_allclose(k_cache[:, :, past:past + S].cpu().numpy().astype(np.float64), kr,
                               rtol=1e-5, atol=1e-5)
    kall = np.concatenate([kp.astype(np.float64), kr], axis=2)
    vall = np.concatenate([vp.astype(np.float64), v.astype(np.float64)], axis=2)
    rep = Hq // Hkv
    sc = (qr @ np.repeat(kall, rep, axis=1).transpose(0, 1, 3, 2)) / math.sqrt(hd)
    o = otp.softmax(sc) @ np.repeat(vall, rep, axis=1)
    ref = o.transpose(0, 2, 1, 3).reshape(B * S, Hq * hd)
    assert rel_l2(out.cpu().numpy(), ref) <= 1e-4


def test_flash_decode_causal_prefill(cuda, rng):
    B, S, Hq, Hkv, hd, Lmax = 1, 5, 4, 2, 64, 32
    past = 3
    cos, sin = otp.rope_tables(hd, 64, 10000.0)
    k_cache = torch.zeros(B, Hkv, Lmax, hd, dtype=torch.float32, device=cuda)
    v_cache = torch.zeros_like(k_cache)
    kp = rng.standard_normal((B, Hkv, past, hd)).astype(np.float32)
    vp = rng.standard_normal((B, Hkv, past, hd)).astype(np.float32)
    k_cache[:, :, :past] = torch.from_numpy(kp).to(cuda)
    v_cache[:, :, :past] = torch.from_numpy(vp).to(cuda)
    qkv = rng.standard_normal((B * S, (Hq + 2 * Hkv) * hd)).astype(np.float32)
    pos = torch.tensor([past], dtype=torch.int32, device=cuda)
    q_out = torch.empty(B * S, Hq * hd, dtype=torch.float32, device=cuda)
    ops.rope_append(to_dev(qkv, cuda), B, S, Hq, Hkv, hd, pos, to_dev(cos, cuda), to_dev(sin, cuda), q_out,
                    k_cache, v_cache)
    out = torch.empty(B * S, Hq * hd, dtype=torch.float32, device=cuda)
    ops.flash_decode(q_out, k_cache, v_cache, pos, B, S, Hq, Hkv, hd, 2, out)
    q = qkv[:, :Hq * hd].reshape(B, S, Hq, hd).transpose(0, 2, 1, 3)
    k = qkv[:, Hq * hd:(Hq + Hkv) * hd].reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
    v = qkv[:, (Hq + Hkv) * hd:].reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
    qr = otp.apply_rope(q, cos[past:past + S], sin[past:past + S])
    kr = otp.apply_rope(k, cos[past:past + S], sin[past:past + S])
    kall = np.concatenate([kp.astype(np.float64), kr], axis=2)
    vall = np.concatenate([vp, v], axis=2).astype(np.float64)
    Lt = past + S
    sc = (qr @ np.repeat(kall, 2, axis=1).transpose(0, 1, 3, 2)) / math.sqrt(hd)
    sc = sc + np.triu(np.full((S, Lt), -np.inf), k=Lt - S + 1)
    ref = (otp.softmax(sc) @ np.repeat(vall, 2, axis=1)).transpose(0, 2, 1, 3).reshape(B * S, Hq * hd)
    assert rel_l2(out.cpu().numpy(), ref) <= 1e-4


def test_rmsnorm_silu_add_argmax(cuda, rng):
    x = rng.standard_normal((3, 1000)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(1000)).astype(np.float16)
    y = ops.rmsnorm(to_dev(x, cuda), to_dev(w, cuda), 1e-5).cpu().numpy()
    assert rel_l2(y, otp.rmsnorm(x, w, 1e-5)) <= 1e-6
    g = rng.standard_normal(777).astype(np.float32)
    u = rng.standard_normal(777).astype(np.float32)
    assert rel_l2(ops.silu_mul(to_dev(g, cuda), to_dev(u, cuda)).cpu().numpy(), otp.silu(g) * u) <= 1e-6
    assert np.allclose(ops.add(to_dev(g, cuda), to_dev(u, cuda)).cpu().numpy(), g + u)
    lg = rng.standard_normal((2, 10007)).astype(np.float32)
    lg[0, 17] = lg[0, 9000] = 50.0  # tie: lowest index wins
    v, i = ops.argmax(to_dev(lg, cuda), index_offset=5)
    assert i.cpu().tolist() == [17 + 5, int(np.argmax(lg[1])) + 5]
    parts = [rng.standard_normal((2, 50)).astype(np.float32) for _ in range(3)]
    parts[2][1, 0] = parts[0][1].max() + 1
    vals = torch.stack([ops.argmax(to_dev(p, cuda), index_offset=r * 50)[0] for r, p in enumerate(parts)])
    idxs = torch.stack([ops.argmax(to_dev(p, cuda), index_offset=r * 50)[1] for r, p in enumerate(parts)])
    tok = torch.empty(2, dtype=torch.int32, device=cuda)
    pos = torch.tensor([7], dtype=torch.int32, device=cuda)
    ops.argmax_merge(vals, idxs, 3, tok, pos, 1)
    assert tok.cpu().tolist() == otp.distributed_argmax(parts, 50).tolist()
    assert int(pos.item()) == 8


def test_l2_prefetch_is_a_pure_hint(cuda, rng):
    """sc_l2_prefetch touches no data: buffers are unchanged, unaligned starts
    are rounded, empty lists are a no-op and more than 12 regions are refused."""
    import ctypes as C

    lib = L.load()
    bufs = [torch.randn(n, device=cuda) for n in (1000, 4096, 77)]
    before = [b.clone() for b in bufs]
    ptrs = [b.data_ptr() for b in bufs] + [bufs[0].data_ptr() + 4]
    sizes = [b.numel() * 4 for b in bufs] + [100]
    P = (C.c_void_p * 4)(*ptrs)
    Z = (C.c_size_t * 4)(*sizes)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.sc_l2_prefetch(C.cast(P, L._pp), Z, 4, 0, stream) == L.SC_OK
    assert lib.sc_l2_prefetch(C.cast(P, L._pp), Z, 4, 1024, stream) == L.SC_OK
    assert lib.sc_l2_prefetch(None, None, 0, 0, stream) == L.SC_OK
    P13 = (C.c_void_p * 13)(*([ptrs[0]] * 13))
    Z13 = (C.c_size_t * 13)(*([64] * 13))
    assert lib.sc_l2_prefetch(C.cast(P13, L._pp), Z13, 13, 0, stream) == L.SC_ERR_ARG
    torch.cuda.synchronize()
    for a, b in zip(bufs, before):
        assert torch.equal(a, b)


@pytest.mark.parametrize("hd,Hq,Hkv", [(128, 32, 8), (64, 8, 1), (128, 4, 4), (64, 16, 2), (128, 16, 2)])
@pytest.mark.parametrize("splits,past", [(1, 37), (3, 37), (33, 2047), (8, 0), (64, 5)])
def test_attn_decode_matches_rope_append_plus_flash(cuda, rng, hd, Hq, Hkv, splits, past):
    """The fused decode attention appends exactly what sc_rope_append writes
    and matches sc_rope_append + sc_flash_decode (and the float64 oracle)."""
    B, Lmax = 2, 2112
    cos, sin = otp.rope_tables(hd, 4096, 5e5)
    cos_t, sin_t = torch.from_numpy(cos).to(cuda), torch.from_numpy(sin).to(cuda)
    kc = torch.from_numpy((rng.standard_normal((B, Hkv, Lmax, hd))).astype(np.float32)).to(cuda)
    vc = torch.from_numpy((rng.standard_normal((B, Hkv, Lmax, hd))).astype(np.float32)).to(cuda)
    kc2, vc2 = kc.clone(), vc.clone()
    qkv = torch.from_numpy(rng.standard_normal((B, (Hq + 2 * Hkv) * hd)).astype(np.float32)).to(cuda)
    pos = torch.tensor([past], dtype=torch.int32, device=cuda)
    out = torch.empty(B, Hq * hd, dtype=torch.float32, device=cuda)
    tickets = torch.zeros(B * Hkv, dtype=torch.int32, device=cuda)
    ws = torch.empty(max(1, ops.attn_decode_workspace_bytes(B, Hq, hd, splits)), dtype=torch.uint8, device=cuda)
    for _ in range(2):  # twice: the tickets must come back to zero
        ops.attn_decode(qkv, B, Hq, Hkv, hd, pos, cos_t, sin_t, kc, vc, splits, out, tickets, workspace=ws)
    assert int(tickets.abs().sum()) == 0
    q2 = torch.empty(B, Hq * hd, dtype=torch.float32, device=cuda)
    ops.rope_append(qkv, B, 1, Hq, Hkv, hd, pos, cos_t, sin_t, q2, kc2, vc2)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    ref = torch.empty_like(out)
    ops.flash_decode(q2, kc2, vc2, pos, B, 1, Hq, Hkv, hd, max(1, splits), ref)
    assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
    # float64 oracle over the cache as the kernel left it
    k64 = kc[:, :, : past + 1].double().cpu().numpy()
    v64 = vc[:, :, : past + 1].double().cpu().numpy()
    q64 = q2.double().cpu().numpy().reshape(B, Hq, 1, hd)
    G = Hq // Hkv
    kk, vv = np.repeat(k64, G, 1), np.repeat(v64, G, 1)
    o64 = otp.softmax(q64 @ kk.transpose(0, 1, 3, 2) / math.sqrt(hd)) @ vv
    assert rel_l2(out.cpu().numpy(), o64.reshape(B, Hq * hd)) <= 1e-4
