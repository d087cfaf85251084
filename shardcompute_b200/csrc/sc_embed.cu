// K3: vocab-split embedding gather (4/8-bit MLX affine rows or fp16 rows),
// whole-table dequantize, and group-wise affine quantize.
//
// Dequantization everywhere is fma.rn.f16x2(q, scale, bias): the exact value
// scale*q + bias rounded once to fp16, which is the rounding contract of the
// reference's mx.dequantize output (fp16, the scales' dtype).
#include <algorithm>

#include "sc_common.cuh"

namespace sc {

// Dequantise one 4-word (16-byte) slice into natural-order halves.
// 4-bit: 32 values; 8-bit: 16 values.
template <int BITS>
__device__ __forceinline__ void dequant_v4(const uint4 w, __half2 s, __half2 b, __half2 (&out)[BITS == 4 ? 16 : 8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (BITS == 4) {
      __half2 P[4];
      unpack_u4(ws[j], P);
#pragma unroll
      for (int q = 0; q < 4; ++q) P[q] = hfma2_rn(P[q], s, b);
      // P[q] = (v_q, v_{q+4}) -> natural order v0..v7
      out[4 * j + 0] = __lows2half2(P[0], P[1]);
      out[4 * j + 1] = __lows2half2(P[2], P[3]);
      out[4 * j + 2] = __highs2half2(P[0], P[1]);
      out[4 * j + 3] = __highs2half2(P[2], P[3]);
    } else {
      __half2 P[2];
      unpack_u8(ws[j], P);
      P[0] = hfma2_rn(P[0], s, b);
      P[1] = hfma2_rn(P[1], s, b);
      // P0 = (v0, v2), P1 = (v1, v3)
      out[2 * j + 0] = __lows2half2(P[0], P[1]);
      out[2 * j + 1] = __highs2half2(P[0], P[1]);
    }
  }
}

template <typename OT>
__device__ __forceinline__ void store_h2s(OT* dst, const __half2* v, int n2);
template <>
__device__ __forceinline__ void store_h2s<__half>(__half* dst, const __half2* v, int n2) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = 0; i < n2 / 4; ++i)
    d[i] = make_uint4(h2_as_u32(v[4 * i]), h2_as_u32(v[4 * i + 1]), h2_as_u32(v[4 * i + 2]), h2_as_u32(v[4 * i + 3]));
}
template <>
__device__ __forceinline__ void store_h2s<float>(float* dst, const __half2* v, int n2) {
  float4* d = reinterpret_cast<float4*>(dst);
  for (int i = 0; i < n2 / 2; ++i) {
    const float2 a = __half22float2(v[2 * i]), b = __half22float2(v[2 * i + 1]);
    d[i] = make_float4(a.x, a.y, b.x, b.y);
  }
}

// grid: one CTA per token row; each thread handles 16-byte slices of the row.
template <int BITS, typename OT>
__global__ void embed_gather_q_kernel(const int32_t* __restrict__ ids, const uint32_t* __restrict__ wq,
                                      const uint16_t* __restrict__ scales, const uint16_t* __restrict__ biases,
                                      int v0, int v1, int H, int group, OT* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  constexpr int PF = 32 / BITS;
  constexpr int VPS = 4 * PF;  // values per 16-byte slice
  const int row = blockIdx.x;
  const int id = ids[row];
  OT* o = out + (size_t)row * H;
  const int nslice = H / VPS;
  if (id < v0 || id >= v1) {
    for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = from_f32<OT>(0.f);
    return;
  }
  const int local = id - v0;
  const int KG = H / group;
  const uint4* wr = reinterpret_cast<const uint4*>(wq + (size_t)local * (H / PF));
  for (int sl = threadIdx.x; sl < nslice; sl += blockDim.x) {
    const int gi = (sl * VPS) / group;
    const __half2 s = __half2half2(__ushort_as_half(scales[(size_t)local * KG + gi]));
    const __half2 b = __half2half2(__ushort_as_half(biases[(size_t)local * KG + gi]));
    __half2 v[VPS / 2];
    dequant_v4<BITS>(wr[sl], s, b, v);
    store_h2s<OT>(o + sl * VPS, v, VPS / 2);
  }
}

template <typename OT>
__global__ void embed_gather_f16_kernel(const int32_t* __restrict__ ids, const uint16_t* __restrict__ table,
                                        int v0, int v1, int H, OT* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int id = ids[row];
  OT* o = out + (size_t)row * H;
  const bool ok = id >= v0 && id < v1;
  const __half* src = reinterpret_cast<const __half*>(table) + (size_t)(ok ? id - v0 : 0) * H;
  if ((H & 7) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
      uint4 v = ok ? s4[i] : make_uint4(0, 0, 0, 0);
      const __half2 hv[4] = {u32_as_h2(v.x), u32_as_h2(v.y), u32_as_h2(v.z), u32_as_h2(v.w)};
      store_h2s<OT>(o + 8 * i, hv, 4);
    }
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x)
      o[i] = from_f32<OT>(ok ? __half2float(src[i]) : 0.f);
  }
}

template <int BITS>
__global__ void dequantize_kernel(const uint32_t* __restrict__ wq, const uint16_t* __restrict__ scales,
                                  const uint16_t* __restrict__ biases, int rows, int K, int group,
                                  __half* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  constexpr int PF = 32 / BITS;
  constexpr int VPS = 4 * PF;
  const size_t nsl_row = K / VPS;
  const size_t total = (size_t)rows * nsl_row;
  const int KG = K / group;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const size_t r = e / nsl_row, sl = e % nsl_row;
    const int gi = (int)(sl * VPS) / group;
    const __half2 s = __half2half2(__ushort_as_half(scales[r * KG + gi]));
    const __half2 b = __half2half2(__ushort_as_half(biases[r * KG + gi]));
    const uint4 w = reinterpret_cast<const uint4*>(wq + r * (K / PF))[sl];
    __half2 v[VPS / 2];
    dequant_v4<BITS>(w, s, b, v);
    store_h2s<__half>(out + r * K + sl * VPS, v, VPS / 2);
  }
}

// One warp per group of `group` values.  Scale/bias/codes computed in double
// so they match an IEEE double restatement bit for bit.
template <int BITS>
__global__ void quantize_kernel(const __half* __restrict__ w, int rows, int K, int group,
                                uint32_t* __restrict__ wq, uint16_t* __restrict__ scales,
                                uint16_t* __restrict__ biases) {
  pdl_trigger();
  pdl_wait();
  constexpr int PF = 32 / BITS;
  constexpr int NB = (1 << BITS) - 1;
  const int KG = K / group;
  const size_t ngroups = (size_t)rows * KG;
  const int lane = threadIdx.x & 31;
  const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t gidx = warp; gidx < ngroups; gidx += nwarps) {
    const size_t r = gidx / KG, gi = gidx % KG;
    const __half* src = w + r * K + gi * group;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = lane; i < group; i += 32) {
      const float v = __half2float(src[i]);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const __half s16 = __double2half(((double)mx - (double)mn) / (double)NB);
    const __half b16 = __double2half((double)mn);
    const double s = (double)__half2float(s16), b = (double)__half2float(b16);
    if (lane == 0) {
      scales[gidx] = __half_as_ushort(s16);
      biases[gidx] = __half_as_ushort(b16);
    }
    const int nwords = group / PF;
    for (int wi = lane; wi < nwords; wi += 32) {
      uint32_t word = 0;
#pragma unroll
      for (int e = 0; e < PF; ++e) {
        const double v = (double)__half2float(src[wi * PF + e]);
        double q = s > 0.0 ? rint((v - b) / s) : 0.0;
        q = fmin(fmax(q, 0.0), (double)NB);
        word |= ((uint32_t)q) << (BITS * e);
      }
      wq[r * (K / PF) + gi * nwords + wi] = word;
    }
  }
}

}  // namespace sc

extern "C" {

int sc_embed_gather_q(const int32_t* ids, int n, const uint32_t* wq, const uint16_t* scales,
                      const uint16_t* biases, int vocab_start, int vocab_end, int H, int group_size, int bits,
                      void* out, int out_dtype, cudaStream_t stream) {
  SC_REQUIRE(bits == 4 || bits == 8, SC_ERR_SHAPE, "embed_gather_q: bits must be 4 or 8");
  SC_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, SC_ERR_SHAPE,
             "embed_gather_q: group_size must be 32, 64 or 128");
  SC_REQUIRE(H > 0 && H % group_size == 0, SC_ERR_SHAPE, "embed_gather_q: H=%d not a multiple of group %d", H,
             group_size);
  SC_REQUIRE(vocab_end >= vocab_start, SC_ERR_SHAPE, "embed_gather_q: empty vocab range");
  SC_REQUIRE(out_dtype == SC_F16 || out_dtype == SC_F32, SC_ERR_ARG, "embed_gather_q: out dtype");
  if (n <= 0) return SC_OK;
  SC_REQUIRE(ids && wq && scales && biases && out, SC_ERR_ARG, "embed_gather_q: null pointer");
  const int threads = 128;
  if (bits == 4) {
    if (out_dtype == SC_F16)
      ::sc::launch(sc::embed_gather_q_kernel<4, __half>, n, threads, 0, stream, ids, wq, scales, biases, vocab_start, vocab_end,
                                                                      H, group_size, (__half*)out);
    else
      ::sc::launch(sc::embed_gather_q_kernel<4, float>, n, threads, 0, stream, ids, wq, scales, biases, vocab_start, vocab_end,
                                                                     H, group_size, (float*)out);
  } else {
    if (out_dtype == SC_F16)
      ::sc::launch(sc::embed_gather_q_kernel<8, __half>, n, threads, 0, stream, ids, wq, scales, biases, vocab_start, vocab_end,
                                                                      H, group_size, (__half*)out);
    else
      ::sc::launch(sc::embed_gather_q_kernel<8, float>, n, threads, 0, stream, ids, wq, scales, biases, vocab_start, vocab_end,
                                                                     H, group_size, (float*)out);
  }
  return sc::check_launch("embed_gather_q");
}

int sc_embed_gather_f16(const int32_t* ids, int n, const uint16_t* table, int vocab_start, int vocab_end, int H,
                        void* out, int out_dtype, cudaStream_t stream) {
  SC_REQUIRE(H > 0, SC_ERR_SHAPE, "embed_gather_f16: H must be positive");
  SC_REQUIRE(vocab_end >= vocab_start, SC_ERR_SHAPE, "embed_gather_f16: empty vocab range");
  SC_REQUIRE(out_dtype == SC_F16 || out_dtype == SC_F32, SC_ERR_ARG, "embed_gather_f16: out dtype");
  if (n <= 0) return SC_OK;
  SC_REQUIRE(ids && table && out, SC_ERR_ARG, "embed_gather_f16: null pointer");
  const int threads = std::min(256, std::max(32, ((H / 8) + 31) / 32 * 32));
  if (out_dtype == SC_F16)
    ::sc::launch(sc::embed_gather_f16_kernel<__half>, n, threads, 0, stream, ids, table, vocab_start, vocab_end, H, (__half*)out);
  else
    ::sc::launch(sc::embed_gather_f16_kernel<float>, n, threads, 0, stream, ids, table, vocab_start, vocab_end, H, (float*)out);
  return sc::check_launch("embed_gather_f16");
}

int sc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int rows, int K,
                  int group_size, int bits, uint16_t* out, cudaStream_t stream) {
  SC_REQUIRE(bits == 4 || bits == 8, SC_ERR_SHAPE, "dequantize: bits must be 4 or 8");
  SC_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, SC_ERR_SHAPE,
             "dequantize: group_size must be 32, 64 or 128");
  SC_REQUIRE(K > 0 && K % group_size == 0, SC_ERR_SHAPE, "dequantize: K=%d not a multiple of group %d", K,
             group_size);
  if (rows <= 0) return SC_OK;
  SC_REQUIRE(wq && scales && biases && out, SC_ERR_ARG, "dequantize: null pointer");
  const int blocks = 4 * sc::sm_count();
  if (bits == 4)
    ::sc::launch(sc::dequantize_kernel<4>, blocks, 256, 0, stream, wq, scales, biases, rows, K, group_size, (__half*)out);
  else
    ::sc::launch(sc::dequantize_kernel<8>, blocks, 256, 0, stream, wq, scales, biases, rows, K, group_size, (__half*)out);
  return sc::check_launch("dequantize");
}

int sc_quantize(const uint16_t* w, int rows, int K, int group_size, int bits, uint32_t* wq, uint16_t* scales,
                uint16_t* biases, cudaStream_t stream) {
  SC_REQUIRE(bits == 4 || bits == 8, SC_ERR_SHAPE, "quantize: bits must be 4 or 8");
  SC_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, SC_ERR_SHAPE,
             "quantize: group_size must be 32, 64 or 128");
  SC_REQUIRE(K > 0 && K % group_size == 0, SC_ERR_SHAPE, "quantize: K=%d not a multiple of group %d", K,
             group_size);
  if (rows <= 0) return SC_OK;
  SC_REQUIRE(w && wq && scales && biases, SC_ERR_ARG, "quantize: null pointer");
  const int blocks = 8 * sc::sm_count();
  if (bits == 4)
    ::sc::launch(sc::quantize_kernel<4>, blocks, 256, 0, stream, (const __half*)w, rows, K, group_size, wq, scales, biases);
  else
    ::sc::launch(sc::quantize_kernel<8>, blocks, 256, 0, stream, (const __half*)w, rows, K, group_size, wq, scales, biases);
  return sc::check_launch("quantize");
}

}  // extern "C"
