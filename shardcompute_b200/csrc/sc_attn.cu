// K4: RoPE + KV-cache append, and split-KV GQA flash-decode.
//
// KV cache layout (per layer, per rank): fp32 [B, Hkv, Lmax, hd], preallocated
// once; token positions come from a device counter so one captured CUDA graph
// serves every decode step.  The cache is fp32 because the reference's is:
// RoPE multiplies q and k by fp32 cos/sin tables and the hidden state is fp32
// after the first residual, so MLX's type promotion caches fp32 keys and
// values (parallel/attention.py:427-436); an fp16 cache moved the hidden state
// of a 32-layer Llama-3-8B about 6e-3 (relative L2) away from the reference.
//
// Flash-decode: grid (splits, Hkv, B*S).  A CTA owns one KV head and the G =
// Hq/Hkv query heads that share it (GQA packed: K/V are read once for the
// whole group, never repeated), and a contiguous range of keys.  Inside the
// CTA, 4 warps interleave over key steps; a key row (hd fp16) is spread over
// hd/8 lanes with two 16-byte loads each, so a warp covers 32*8/hd keys per
// step.  Each lane group keeps an online-softmax state (max, sum, o[8]) per
// query head; the states are merged in shared memory and written as one
// (max, sum, o[hd]) partial per split, which a second kernel merges.
#include <algorithm>

#include "sc_common.cuh"

namespace sc {

// 8 consecutive fp32 values (two 16-byte loads), zeros for a null pointer.
__device__ __forceinline__ void ld_f8(const float* p, float (&v)[8]) {
  if (!p) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return;
  }
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__global__ void rope_append_kernel(const float* __restrict__ qkv, int S, int Hq, int Hkv, int hd,
                                   const int32_t* __restrict__ pos_ptr, const float* __restrict__ cos_tab,
                                   const float* __restrict__ sin_tab, int max_pos, float* __restrict__ q_out,
                                   float* __restrict__ kc, float* __restrict__ vc, int Lmax) {
  pdl_trigger();
  pdl_wait();
  const int tok = blockIdx.x;  // b*S + s
  const int b = tok / S, s = tok % S;
  const int pos = *pos_ptr + s;
  const int half = hd / 2;
  const int width = (Hq + 2 * Hkv) * hd;
  const float* src = qkv + (size_t)tok * width;
  const bool pos_ok = pos >= 0 && pos < max_pos && pos < Lmax;
  const int items = (Hq + Hkv) * half + Hkv * hd;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    if (it < (Hq + Hkv) * half) {
      const int h = it / half, d = it % half;
      const float x1 = src[h * hd + d], x2 = src[h * hd + d + half];
      const float c = pos_ok ? cos_tab[(size_t)pos * half + d] : 1.f;
      const float sn = pos_ok ? sin_tab[(size_t)pos * half + d] : 0.f;
      // x*cos + rotate_half(x)*sin, rotate_half = [-x2, x1], products unfused
      const float o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, sn));
      const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
      if (h < Hq) {
        q_out[(size_t)tok * Hq * hd + h * hd + d] = o1;
        q_out[(size_t)tok * Hq * hd + h * hd + d + half] = o2;
      } else if (pos_ok) {
        const int kh = h - Hq;
        float* dst = kc + (((size_t)b * Hkv + kh) * Lmax + pos) * hd;
        dst[d] = o1;
        dst[d + half] = o2;
      }
    } else if (pos_ok) {
      const int r = it - (Hq + Hkv) * half;
      const int vh = r / hd, d = r % hd;
      vc[(((size_t)b * Hkv + vh) * Lmax + pos) * hd + d] = src[(Hq + Hkv) * hd + vh * hd + d];
    }
  }
}

constexpr int FD_WARPS = 4;

template <int HD, int G, typename OT>
__global__ void __launch_bounds__(FD_WARPS * 32)
flash_decode_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                    const int32_t* __restrict__ pos_ptr, int S, int Hq, int Hkv, int Lmax, float scale,
                    int splits, float* __restrict__ part, OT* __restrict__ out, int tok0) {
  pdl_trigger();
  pdl_wait();
  constexpr int LPK = HD / 8;    // lanes per key
  constexpr int KPS = 32 / LPK;  // keys per warp step
  const int split = blockIdx.x, kvh = blockIdx.y, tok = tok0 + (int)blockIdx.z;
  const int b = tok / S, s = tok % S;
  // keys visible to this query, never past the cache (a position beyond
  // Lmax was not appended by sc_rope_append either)
  const int L = min(*pos_ptr + s + 1, Lmax);
  const int chunk = (L + splits - 1) / splits;
  const int k_beg = split * chunk;
  const int k_end = min(L, k_beg + chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPK, dl = lane % LPK;
  const int d0 = dl * 8;

  float qr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float* qp = q + (size_t)tok * Hq * HD + (size_t)(kvh * G + g) * HD + d0;
    const float4 a = *reinterpret_cast<const float4*>(qp);
    const float4 c = *reinterpret_cast<const float4*>(qp + 4);
    qr[g][0] = a.x; qr[g][1] = a.y; qr[g][2] = a.z; qr[g][3] = a.w;
    qr[g][4] = c.x; qr[g][5] = c.y; qr[g][6] = c.z; qr[g][7] = c.w;
  }
  float m[G], l[G], o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
  }
  const float* kbase = kc + ((size_t)b * Hkv + kvh) * Lmax * HD;
  const float* vbase = vc + ((size_t)b * Hkv + kvh) * Lmax * HD;

  for (int k0 = k_beg + warp * KPS; k0 < k_end; k0 += FD_WARPS * KPS) {
    const int key = k0 + sub;
    const bool valid = key < k_end;
    float kf[8], vf[8];
    ld_f8(valid ? kbase + (size_t)key * HD + d0 : nullptr, kf);
    ld_f8(valid ? vbase + (size_t)key * HD + d0 : nullptr, vf);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(qr[g][i], kf[i], dot);
#pragma unroll
      for (int off = LPK / 2; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      if (valid) {
        const float sc = dot * scale;
        const float mn = fmaxf(m[g], sc);
        const float corr = expf(m[g] - mn);
        const float pr = expf(sc - mn);
        l[g] = l[g] * corr + pr;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[g][i] = fmaf(pr, vf[i], o[g][i] * corr);
        m[g] = mn;
      }
    }
  }

  // merge the FD_WARPS*KPS lane-group states
  __shared__ float sm_m[FD_WARPS * KPS][G], sm_l[FD_WARPS * KPS][G];
  __shared__ float sm_o[FD_WARPS * KPS][G][HD];
  const int grp = warp * KPS + sub;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (dl == 0) {
      sm_m[grp][g] = m[g];
      sm_l[grp][g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) sm_o[grp][g][d0 + i] = o[g][i];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += FD_WARPS * 32) {
    const int g = e / HD, d = e % HD;
    float M = -INFINITY;
    for (int r = 0; r < FD_WARPS * KPS; ++r) M = fmaxf(M, sm_m[r][g]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int r = 0; r < FD_WARPS * KPS; ++r) {
        const float w = expf(sm_m[r][g] - M);
        Ls = fmaf(sm_l[r][g], w, Ls);
        O = fmaf(sm_o[r][g][d], w, O);
      }
    }
    const int qh = kvh * G + g;
    if (splits == 1) {
      out[(size_t)tok * Hq * HD + (size_t)qh * HD + d] = from_f32<OT>(O / Ls);
    } else {
      float* pp = part + (((size_t)tok * Hq + qh) * splits + split) * (HD + 2);
      pp[2 + d] = O;
      if (d == 0) {
        pp[0] = M;
        pp[1] = Ls;
      }
    }
  }
}

// Merge of split-KV partials {m, l, o[HD]} for G heads by one CTA of NT
// threads.  The split maxima and sums are read once, in parallel, into shared
// memory; each output element then sums its splits with AM_BATCH loads in
// flight (the merge is a chain of L2 round trips, so fewer rounds is faster).
constexpr int FD_MAX_SPLITS = 64;
constexpr int AM_BATCH = 16;

template <int HD, int G, int NT, typename OT>
__device__ __forceinline__ void merge_partials(const float* pbase, size_t sstride, size_t gstride, int splits,
                                               OT* outp, float (*s_w)[G], float (*s_l)[G], float* s_inv) {
  for (int i = threadIdx.x; i < splits * G; i += NT) {
    const int sp = i / G, g = i % G;
    const float* pp = pbase + sp * sstride + g * gstride;
    s_w[sp][g] = __ldcg(pp);
    s_l[sp][g] = __ldcg(pp + 1);
  }
  __syncthreads();
  if (threadIdx.x < G) {  // the head's maximum over the splits (cheap: no exp)
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, s_w[sp][g]);
    s_inv[g] = M;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < splits * G; i += NT) {  // the splits' weights, in parallel
    const int sp = i / G, g = i % G;
    const float mw = s_w[sp][g];
    s_w[sp][g] = mw == -INFINITY ? 0.f : expf(mw - s_inv[g]);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float Ls = 0.f;
    for (int sp = 0; sp < splits; ++sp) Ls = fmaf(s_l[sp][g], s_w[sp][g], Ls);
    s_inv[g] = 1.f / Ls;
  }
  __syncthreads();
  constexpr int EPT = (G * HD + NT - 1) / NT;  // outputs per thread
  float acc[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) acc[j] = 0.f;
  for (int s0 = 0; s0 < splits; s0 += AM_BATCH) {
    float v[EPT][AM_BATCH];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const int e = threadIdx.x + j * NT;
      const int g = e / HD, d = e % HD;
#pragma unroll
      for (int u = 0; u < AM_BATCH; ++u)
        v[j][u] = (e < G * HD && s0 + u < splits) ? __ldcg(pbase + (s0 + u) * sstride + g * gstride + 2 + d) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const int e = threadIdx.x + j * NT;
      const int g = (e < G * HD ? e : 0) / HD;
#pragma unroll
      for (int u = 0; u < AM_BATCH; ++u)
        if (s0 + u < splits) acc[j] = fmaf(v[j][u], s_w[s0 + u][g], acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int e = threadIdx.x + j * NT;
    if (e < G * HD) outp[(size_t)(e / HD) * HD + e % HD] = from_f32<OT>(acc[j] * s_inv[e / HD]);
  }
}

// Split merge of the fused decode kernel in one round of loads, by one CTA of
// NT threads.  Partials are {m, l, -, -, o[HD]} per (split, head): 16-byte
// aligned, so a thread's 8 dims of one split are two 16-byte loads.  Thread
// (unit, subset) owns 8 output dims of one head and the splits congruent to
// its subset modulo S; it issues all their loads (up to MR_BATCH) at once,
// folds them in with a running maximum, and the S subsets are folded through
// shared memory (`s_red`, NT * 10 floats).  Output = sum(w o) / sum(w l).
constexpr int MR_BATCH = 10;
constexpr int AD_PSTRIDE_PAD = 4;  // floats before o[] in a fused-kernel partial

template <int HD, int G, int NT, typename OT>
__device__ __forceinline__ void merge_partials_1r(const float* pbase, int splits, OT* outp, float* s_red) {
  constexpr int UNITS = G * HD / 8;
  constexpr int S = NT / UNITS;
  constexpr int PS = HD + AD_PSTRIDE_PAD;  // floats per (split, head)
  static_assert(S >= 1, "one thread per 8 output dims at least");
  const int u = threadIdx.x % UNITS, j = threadIdx.x / UNITS;
  const int g = u / (HD / 8), d8 = (u % (HD / 8)) * 8;
  float M = -INFINITY, Ls = 0.f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (j < S) {
    for (int s0 = j; s0 < splits; s0 += S * MR_BATCH) {
      float2 ml[MR_BATCH];
      float4 oa[MR_BATCH], ob[MR_BATCH];
#pragma unroll
      for (int r = 0; r < MR_BATCH; ++r) {
        const int sp = s0 + r * S;
        ml[r] = make_float2(-INFINITY, 0.f);
        oa[r] = ob[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (sp < splits) {
          const float* pp = pbase + ((size_t)sp * G + g) * PS;
          ml[r] = __ldcg(reinterpret_cast<const float2*>(pp));
          oa[r] = __ldcg(reinterpret_cast<const float4*>(pp + AD_PSTRIDE_PAD + d8));
          ob[r] = __ldcg(reinterpret_cast<const float4*>(pp + AD_PSTRIDE_PAD + d8 + 4));
        }
      }
#pragma unroll
      for (int r = 0; r < MR_BATCH; ++r) {
        if (ml[r].x == -INFINITY) continue;  // an empty split (or past the last)
        const float mn = fmaxf(M, ml[r].x);
        const float co = M == -INFINITY ? 0.f : expf(M - mn);
        const float w = expf(ml[r].x - mn);
        Ls = Ls * co + ml[r].y * w;
        const float ov[8] = {oa[r].x, oa[r].y, oa[r].z, oa[r].w, ob[r].x, ob[r].y, ob[r].z, ob[r].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = acc[i] * co + ov[i] * w;
        M = mn;
      }
    }
  }
  float* me = s_red + (size_t)threadIdx.x * 10;
  me[0] = M;
  me[1] = Ls;
#pragma unroll
  for (int i = 0; i < 8; ++i) me[2 + i] = acc[i];
  __syncthreads();
  if (j == 0) {
    for (int jj = 1; jj < S; ++jj) {
      const float* o = s_red + (size_t)(jj * UNITS + u) * 10;
      if (o[0] == -INFINITY) continue;
      const float mn = fmaxf(M, o[0]);
      const float co = M == -INFINITY ? 0.f : expf(M - mn);
      const float w = expf(o[0] - mn);
      Ls = Ls * co + o[1] * w;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = acc[i] * co + o[2 + i] * w;
      M = mn;
    }
    const float inv = 1.f / Ls;
#pragma unroll
    for (int i = 0; i < 8; ++i) outp[(size_t)g * HD + d8 + i] = from_f32<OT>(acc[i] * inv);
  }
}

template <int HD, typename OT>
__global__ void flash_decode_merge_kernel(const float* __restrict__ part, int Hq, int splits, OT* __restrict__ out,
                                          int tok0) {
  pdl_trigger();
  pdl_wait();
  const int qh = blockIdx.x, tok = tok0 + (int)blockIdx.y;
  __shared__ float s_w[FD_MAX_SPLITS][1], s_l[FD_MAX_SPLITS][1], s_inv[1];
  merge_partials<HD, 1, HD, OT>(part + ((size_t)tok * Hq + qh) * splits * (HD + 2), HD + 2, 0, splits,
                                out + (size_t)tok * Hq * HD + (size_t)qh * HD, s_w, s_l, s_inv);
}

template <int HD, int G, typename OT>
static int launch_fd(const float* q, const float* kc, const float* vc, const int32_t* pos, int B, int S, int Hq,
                     int Hkv, int Lmax, float scale, int splits, float* part, OT* out, cudaStream_t stream) {
  // tokens go on the grid's y / z axes (at most 65535 each): launches of up to 32768 tokens
  const int T = B * S;
  for (int t0 = 0; t0 < T; t0 += 32768) {
    const int nt = std::min(32768, T - t0);
    ::sc::launch(flash_decode_kernel<HD, G, OT>, dim3(splits, Hkv, nt), FD_WARPS * 32, 0, stream, q, kc, vc, pos, S, Hq,
                 Hkv, Lmax, scale, splits, part, out, t0);
    int st = check_launch("flash_decode");
    if (st != SC_OK) return st;
    if (splits == 1) continue;
    ::sc::launch(flash_decode_merge_kernel<HD, OT>, dim3(Hq, nt), HD, 0, stream, part, Hq, splits, out, t0);
    st = check_launch("flash_decode_merge");
    if (st != SC_OK) return st;
  }
  return SC_OK;
}

template <int HD, typename OT>
static int dispatch_g(int G, const float* q, const float* kc, const float* vc, const int32_t* pos, int B, int S,
                      int Hq, int Hkv, int Lmax, float scale, int splits, float* part, OT* out, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_fd<HD, 1, OT>(q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, out, stream);
    case 2: return launch_fd<HD, 2, OT>(q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, out, stream);
    case 4: return launch_fd<HD, 4, OT>(q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, out, stream);
    case 8: return launch_fd<HD, 8, OT>(q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, out, stream);
  }
  set_error("flash_decode: GQA group %d unsupported (1, 2, 4, 8)", G);
  return SC_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Fused decode attention (one new token per sequence): RoPE of q and the new
// k, append of k and v to the cache, split-KV online softmax over the cache,
// and the merge of the splits -- one launch instead of three.
//
// grid (splits, Hkv, B), AD_WARPS warps.  A CTA's keys are one contiguous
// range of the cache ([B][Hkv][Lmax][hd] rows), so they stream into shared
// memory as 1-D bulk copies of AD_TK keys (K and V), AD_NB tiles in flight,
// issued before anything else so the HBM latency overlaps the rotation work.
// Every CTA rotates its G query heads itself (a few hundred floats); the CTA
// whose key range holds the new position also rotates the new k, writes k
// and v into the cache and uses those fp16 values for that key (its tile's
// copy of that row may predate the write).  Partials go to the workspace; the
// last CTA of a (sequence, kv head) -- an atomic ticket per pair -- merges the
// splits and writes the output, then resets its ticket to zero for the next
// call.  Tile waits are bounded; a timeout raises g_attn_error and the CTA
// stops computing (its output is undefined).

constexpr int AD_WARPS = 8;
constexpr int AD_TK = 32;  // keys per tile (fp32 K and V: 32 KB per tile pair)
constexpr int AD_NB = 2;   // tiles in flight
__device__ int g_attn_error = 0;

__host__ __device__ constexpr int ad_groups(int hd) { return AD_WARPS * (32 / (hd / 8)); }  // lane groups of a CTA
__host__ __device__ constexpr size_t ad_kv_bytes(int hd) { return (size_t)AD_NB * 2 * AD_TK * hd * 4; }
__host__ __device__ constexpr size_t ad_smem_bytes(int hd, int G) {
  // the tile buffers, reused after the last tile for the lane groups' partial outputs
  return ad_kv_bytes(hd) > (size_t)ad_groups(hd) * G * hd * 4 ? ad_kv_bytes(hd) : (size_t)ad_groups(hd) * G * hd * 4;
}

template <int HD>
__device__ __forceinline__ void rope_pair(float x1, float x2, float c, float sn, float& o1, float& o2) {
  // x*cos + rotate_half(x)*sin, rotate_half = [-x2, x1]; products unfused, as sc_rope_append
  o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, sn));
  o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
}

template <int HD, int G, typename OT>
__global__ void __launch_bounds__(AD_WARPS * 32)
attn_decode_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ pos_ptr,
                   const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int max_pos, int Hq,
                   int Hkv, int Lmax, float scale, int splits, float* __restrict__ kc, float* __restrict__ vc,
                   float* __restrict__ part, int* __restrict__ tickets, OT* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  constexpr int LPK = HD / 8;    // lanes per key (8 halves each)
  constexpr int KPS = 32 / LPK;  // keys per warp step
  constexpr int HALF = HD / 2;
  constexpr int NT = AD_WARPS * 32;
  constexpr int STEP = AD_WARPS * KPS;  // keys per CTA step
  constexpr int NGRP = ad_groups(HD);
  static_assert(G <= LPK, "the score butterfly needs a lane per head in a key's lane group");
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPK, dl = lane % LPK;
  const int d0 = dl * 8;

  const int pos = *pos_ptr;
  const bool append = pos >= 0 && pos < Lmax && pos < max_pos;
  const int L = append ? pos + 1 : min(max(pos, 0), Lmax);
  const int chunk = (L + splits - 1) / splits;
  const int k_beg = min(L, split * chunk);
  const int k_end = min(L, k_beg + chunk);
  const int ntiles = (k_end - k_beg + AD_TK - 1) / AD_TK;
  const bool owner = append && pos >= k_beg && pos < k_end;
  const int width = (Hq + 2 * Hkv) * HD;
  const float* src = qkv + (size_t)b * width;
  const float* kbase = kc + ((size_t)b * Hkv + kvh) * Lmax * HD;
  const float* vbase = vc + ((size_t)b * Hkv + kvh) * Lmax * HD;

  extern __shared__ __align__(128) unsigned char ad_smem[];
  float* s_kv = reinterpret_cast<float*>(ad_smem);  // [AD_NB][2][AD_TK][HD]
  __shared__ __align__(8) uint64_t s_full[AD_NB];
  __shared__ int s_abort;
  __shared__ float s_q[G][HD];
  __shared__ __align__(16) float s_knew[HD], s_vnew[HD];

  auto issue = [&](int t) {  // thread 0: bulk copies of tile t's K and V rows
    const int kt = k_beg + t * AD_TK;
    const uint32_t bytes = (uint32_t)(min(AD_TK, k_end - kt) * HD * 4);
    const int bi = t % AD_NB;
    float* dk = s_kv + (size_t)(bi * 2) * AD_TK * HD;
    mbar_arrive_expect_tx(&s_full[bi], 2 * bytes);
    bulk_load(dk, kbase + (size_t)kt * HD, bytes, &s_full[bi]);
    bulk_load(dk + AD_TK * HD, vbase + (size_t)kt * HD, bytes, &s_full[bi]);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < AD_NB; ++i) mbar_init(&s_full[i], 1);
    s_abort = 0;
    fence_mbar_init();
    for (int t = 0; t < min(AD_NB, ntiles); ++t) issue(t);
  }

  // rotated queries (and, for the owner, the new key / value) while the tiles stream in
  for (int e = threadIdx.x; e < G * HALF; e += NT) {
    const int g = e / HALF, d = e % HALF;
    const float* qh = src + (size_t)(kvh * G + g) * HD;
    float o1 = qh[d], o2 = qh[d + HALF];
    if (append) rope_pair<HD>(qh[d], qh[d + HALF], cos_tab[(size_t)pos * HALF + d], sin_tab[(size_t)pos * HALF + d],
                              o1, o2);
    s_q[g][d] = o1;
    s_q[g][d + HALF] = o2;
  }
  if (owner) {
    const float* kh = src + (size_t)(Hq + kvh) * HD;
    const float* vh = src + (size_t)(Hq + Hkv + kvh) * HD;
    float* kdst = kc + (((size_t)b * Hkv + kvh) * Lmax + pos) * HD;
    float* vdst = vc + (((size_t)b * Hkv + kvh) * Lmax + pos) * HD;
    for (int d = threadIdx.x; d < HALF; d += NT) {
      float o1, o2;
      rope_pair<HD>(kh[d], kh[d + HALF], cos_tab[(size_t)pos * HALF + d], sin_tab[(size_t)pos * HALF + d], o1, o2);
      s_knew[d] = o1;
      s_knew[d + HALF] = o2;
      kdst[d] = o1;
      kdst[d + HALF] = o2;
    }
    for (int d = threadIdx.x; d < HD; d += NT) {
      const float v = vh[d];
      s_vnew[d] = v;
      vdst[d] = v;
    }
  }
  __syncthreads();

  // Per tile: (1) scores of all its keys into s_s, (2) one softmax update per
  // head (running max / sum in shared memory, probabilities back into s_s),
  // (3) o += p . V with the tile's rescale applied once.  Every lane group
  // shares the running max, so the groups' outputs merge by a plain sum.
  __shared__ float s_s[G][AD_TK];
  __shared__ float s_rm[G], s_rl[G], s_corr[G];  // running max / sum per head
  if (threadIdx.x < G) {
    s_rm[threadIdx.x] = -INFINITY;
    s_rl[threadIdx.x] = 0.f;
  }
  float qr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) qr[g][i] = s_q[g][d0 + i];
  float o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
  int t = 0;
  for (; t < ntiles; ++t) {
    const int bi = t % AD_NB;
    mbar_wait_bounded(&s_full[bi], (t / AD_NB) & 1, &s_abort, 1000000000ull);  // a timeout raises s_abort
    __syncthreads();  // every thread's wait has ended: the abort decision below is uniform
    if (s_abort) break;
    const int kt = k_beg + t * AD_TK;
    const int nk = min(AD_TK, k_end - kt);
    const float* tk = s_kv + (size_t)(bi * 2) * AD_TK * HD;
    const float* tv = tk + AD_TK * HD;
    // (1) scores: only the steps that hold keys; the G per-lane dot products
    // are summed over the LPK lanes of a key with a transposing butterfly
    // (G - 1 + log2(LPK / G) shuffles instead of G * log2(LPK))
    const int steps = (nk + STEP - 1) / STEP;
    for (int st = 0; st < steps; ++st) {
      const int kk = st * STEP + warp * KPS + sub;
      const bool valid = kk < nk;
      float kf[8];
      ld_f8(valid ? (owner && kt + kk == pos ? s_knew : tk + (size_t)kk * HD) + d0 : nullptr, kf);
      float dv[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(qr[g][i], kf[i], dot);
        dv[g] = dot;
      }
      int h = 0;  // head whose sum this lane ends up holding
#pragma unroll
      for (int half = G / 2, off = LPK / 2; half >= 1; half >>= 1, off >>= 1) {
        const bool up = (dl & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = up ? dv[i] : dv[i + half];
          const float keep = up ? dv[i + half] : dv[i];
          dv[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
        h += up ? half : 0;
      }
#pragma unroll
      for (int off = LPK / (2 * G); off >= 1; off >>= 1) dv[0] += __shfl_xor_sync(0xffffffffu, dv[0], off);
      if ((dl & (LPK / G - 1)) == 0) s_s[h][kk] = valid ? dv[0] * scale : -INFINITY;
    }
    __syncthreads();
    // (2) softmax update: warp g owns head g
    if (warp < G) {
      const int g = warp;
      float v[AD_TK / 32];
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < AD_TK / 32; ++j) {
        v[j] = lane + 32 * j < nk ? s_s[g][lane + 32 * j] : -INFINITY;  // slots past nk were not written
        mt = fmaxf(mt, v[j]);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_old = s_rm[g];
      const float mn = fmaxf(m_old, mt);
      const bool none = mn == -INFINITY;  // no key so far: keep zeros, no NaN
      float lt = 0.f;
#pragma unroll
      for (int j = 0; j < AD_TK / 32; ++j) {
        const float pj = none ? 0.f : expf(v[j] - mn);
        s_s[g][lane + 32 * j] = pj;
        lt += pj;
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
      if (lane == 0) {
        const float corr = none ? 1.f : expf(m_old - mn);
        s_corr[g] = corr;
        s_rl[g] = s_rl[g] * corr + lt;
        s_rm[g] = mn;
      }
    }
    __syncthreads();
    // (3) o = o * corr + p . V
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float c = s_corr[g];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[g][i] *= c;
    }
#pragma unroll
    for (int kk = warp * KPS + sub; kk < AD_TK; kk += STEP) {
      if (kk >= nk) break;  // keys ascend with kk for this lane
      float vf[8];
      ld_f8((owner && kt + kk == pos ? s_vnew : tv + (size_t)kk * HD) + d0, vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = s_s[g][kk];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[g][i] = fmaf(pr, vf[i], o[g][i]);
      }
    }
    __syncthreads();  // every warp is done with buffer bi and with s_s
    if (threadIdx.x == 0 && t + AD_NB < ntiles) issue(t + AD_NB);
  }
  if (s_abort) {
    if (threadIdx.x == 0) {
      atomicExch(&g_attn_error, 1);
      // let the copies still in flight (tiles t .. t + AD_NB - 1) land before the CTA exits
      for (int u = t; u < min(t + AD_NB, ntiles); ++u) {
        int dummy = 0;
        mbar_wait_bounded(&s_full[u % AD_NB], (u / AD_NB) & 1, (volatile int*)&dummy, 250000000ull);
      }
    }
    return;  // every thread returns: no barrier below is left waiting
  }

  // sum the lane groups' outputs (they reuse the tile buffers)
  float* sm_o = reinterpret_cast<float*>(ad_smem);  // [NGRP][G][HD]
  const int grp = warp * KPS + sub;
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) sm_o[((size_t)grp * G + g) * HD + d0 + i] = o[g][i];
  __syncthreads();
  constexpr int PS = HD + AD_PSTRIDE_PAD;
  float* pbase = part + (((size_t)b * Hkv + kvh) * splits) * G * PS;
  for (int e = threadIdx.x; e < G * HD; e += NT) {
    const int g = e / HD, d = e % HD;
    float O = 0.f;
    for (int r = 0; r < NGRP; ++r) O += sm_o[((size_t)r * G + g) * HD + d];
    const float M = s_rm[g], Ls = s_rl[g];
    if (splits == 1) {
      out[(size_t)b * Hq * HD + (size_t)(kvh * G + g) * HD + d] = from_f32<OT>(O / Ls);
    } else {
      float* pp = pbase + ((size_t)split * G + g) * PS;
      pp[AD_PSTRIDE_PAD + d] = O;
      if (d == 0) {
        pp[0] = M;
        pp[1] = Ls;
      }
    }
  }
  if (splits == 1) return;

  // the last CTA of this (sequence, kv head) merges the splits
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int tk = atomicAdd(&tickets[b * Hkv + kvh], 1);
    s_last = (tk == splits - 1);
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  merge_partials_1r<HD, G, NT, OT>(pbase, splits, out + (size_t)b * Hq * HD + (size_t)kvh * G * HD,
                                   reinterpret_cast<float*>(ad_smem));
  if (threadIdx.x == 0) tickets[b * Hkv + kvh] = 0;
}

template <int HD, int G, typename OT>
static int launch_ad(const float* qkv, const int32_t* pos, const float* cos_tab, const float* sin_tab, int max_pos,
                     int B, int Hq, int Hkv, int Lmax, float scale, int splits, float* kc, float* vc, float* part,
                     int* tickets, OT* out, cudaStream_t stream) {
  auto kern = attn_decode_kernel<HD, G, OT>;
  const size_t smem = ad_smem_bytes(HD, G);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = true;
  }
  ::sc::launch(kern, dim3(splits, Hkv, B), AD_WARPS * 32, smem, stream, qkv, pos, cos_tab, sin_tab, max_pos, Hq, Hkv,
               Lmax, scale, splits, kc, vc, part, tickets, out);
  return check_launch("attn_decode");
}

template <int HD, typename OT>
static int dispatch_ad(int G, const float* qkv, const int32_t* pos, const float* cos_tab, const float* sin_tab,
                       int max_pos, int B, int Hq, int Hkv, int Lmax, float scale, int splits, float* kc, float* vc,
                       float* part, int* tickets, OT* out, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_ad<HD, 1, OT>(qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc, part, tickets, out, stream);
    case 2: return launch_ad<HD, 2, OT>(qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc, part, tickets, out, stream);
    case 4: return launch_ad<HD, 4, OT>(qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc, part, tickets, out, stream);
    case 8: return launch_ad<HD, 8, OT>(qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc, part, tickets, out, stream);
  }
  set_error("attn_decode: GQA group %d unsupported (1, 2, 4, 8)", G);
  return SC_ERR_UNSUPPORTED;
}

}  // namespace sc

extern "C" {

int sc_rope_append(const float* qkv, int B, int S, int Hq, int Hkv, int hd, const int32_t* pos,
                   const float* cos_tab, const float* sin_tab, int max_pos, float* q_out, float* k_cache,
                   float* v_cache, int Lmax, cudaStream_t stream) {
  SC_REQUIRE(hd > 0 && hd % 2 == 0, SC_ERR_SHAPE, "rope_append: head_dim must be even");
  SC_REQUIRE(Hq > 0 && Hkv > 0 && B > 0 && S > 0, SC_ERR_SHAPE, "rope_append: empty shape");
  SC_REQUIRE(qkv && pos && cos_tab && sin_tab && q_out && k_cache && v_cache, SC_ERR_ARG,
             "rope_append: null pointer");
  ::sc::launch(sc::rope_append_kernel, B * S, 256, 0, stream, qkv, S, Hq, Hkv, hd, pos, cos_tab, sin_tab, max_pos, q_out,
                                                    k_cache, v_cache, Lmax);
  return sc::check_launch("rope_append");
}

size_t sc_flash_decode_workspace_bytes(int B, int S, int Hq, int hd, int splits) {
  if (splits <= 1) return 0;
  return (size_t)B * S * Hq * splits * (hd + 2) * sizeof(float);
}

int sc_flash_decode(const float* q, const float* k_cache, const float* v_cache, const int32_t* pos, int B,
                    int S, int Hq, int Hkv, int hd, int Lmax, float scale, int splits, void* out, int out_dtype,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  SC_REQUIRE(hd == 64 || hd == 128, SC_ERR_UNSUPPORTED, "flash_decode: head_dim %d unsupported (64, 128)", hd);
  SC_REQUIRE(Hkv > 0 && Hq % Hkv == 0, SC_ERR_SHAPE, "flash_decode: Hq=%d not a multiple of Hkv=%d", Hq, Hkv);
  SC_REQUIRE(B > 0 && S > 0 && splits >= 1 && splits <= sc::FD_MAX_SPLITS, SC_ERR_SHAPE,
             "flash_decode: bad B/S/splits (splits 1..%d)", sc::FD_MAX_SPLITS);
  SC_REQUIRE(q && k_cache && v_cache && pos && out, SC_ERR_ARG, "flash_decode: null pointer");
  SC_REQUIRE(out_dtype == SC_F16 || out_dtype == SC_F32, SC_ERR_ARG, "flash_decode: out dtype");
  const size_t need = sc_flash_decode_workspace_bytes(B, S, Hq, hd, splits);
  SC_REQUIRE(workspace_bytes >= need && (need == 0 || workspace), SC_ERR_WORKSPACE,
             "flash_decode: workspace of %zu bytes needed (got %zu)", need, workspace_bytes);
  const int G = Hq / Hkv;
  const float* kc = k_cache;
  const float* vc = v_cache;
  float* part = (float*)workspace;
  if (hd == 128) {
    if (out_dtype == SC_F16)
      return sc::dispatch_g<128, __half>(G, q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, (__half*)out,
                                         stream);
    return sc::dispatch_g<128, float>(G, q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, (float*)out,
                                      stream);
  }
  if (out_dtype == SC_F16)
    return sc::dispatch_g<64, __half>(G, q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, (__half*)out,
                                      stream);
  return sc::dispatch_g<64, float>(G, q, kc, vc, pos, B, S, Hq, Hkv, Lmax, scale, splits, part, (float*)out, stream);
}

size_t sc_attn_decode_workspace_bytes(int B, int Hq, int hd, int splits) {
  if (splits <= 1) return 0;
  return (size_t)B * Hq * splits * (hd + sc::AD_PSTRIDE_PAD) * sizeof(float);
}

int sc_attn_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sc::g_attn_error, sizeof(int));
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(sc::g_attn_error, &z, sizeof(int));
  }
  return v;
}

int sc_attn_decode(const float* qkv, int B, int Hq, int Hkv, int hd, const int32_t* pos, const float* cos_tab,
                   const float* sin_tab, int max_pos, float* k_cache, float* v_cache, int Lmax, float scale,
                   int splits, void* out, int out_dtype, void* workspace, size_t workspace_bytes, int32_t* tickets,
                   cudaStream_t stream) {
  SC_REQUIRE(hd == 64 || hd == 128, SC_ERR_UNSUPPORTED, "attn_decode: head_dim %d unsupported (64, 128)", hd);
  SC_REQUIRE(Hkv > 0 && Hq % Hkv == 0, SC_ERR_SHAPE, "attn_decode: Hq=%d not a multiple of Hkv=%d", Hq, Hkv);
  SC_REQUIRE(B > 0 && splits >= 1 && splits <= sc::FD_MAX_SPLITS && Lmax > 0, SC_ERR_SHAPE,
             "attn_decode: bad B/splits/Lmax (splits 1..%d)", sc::FD_MAX_SPLITS);
  SC_REQUIRE(qkv && pos && cos_tab && sin_tab && k_cache && v_cache && out, SC_ERR_ARG,
             "attn_decode: null pointer");
  SC_REQUIRE(out_dtype == SC_F16 || out_dtype == SC_F32, SC_ERR_ARG, "attn_decode: out dtype");
  const size_t need = sc_attn_decode_workspace_bytes(B, Hq, hd, splits);
  SC_REQUIRE(workspace_bytes >= need && (need == 0 || workspace), SC_ERR_WORKSPACE,
             "attn_decode: workspace of %zu bytes needed (got %zu)", need, workspace_bytes);
  SC_REQUIRE(splits == 1 || tickets, SC_ERR_ARG, "attn_decode: split-KV needs the ticket array");
  const int G = Hq / Hkv;
  float* kc = k_cache;
  float* vc = v_cache;
  float* part = (float*)workspace;
  if (hd == 128) {
    if (out_dtype == SC_F16)
      return sc::dispatch_ad<128, __half>(G, qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc,
                                          vc, part, tickets, (__half*)out, stream);
    return sc::dispatch_ad<128, float>(G, qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc,
                                       part, tickets, (float*)out, stream);
  }
  if (out_dtype == SC_F16)
    return sc::dispatch_ad<64, __half>(G, qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc,
                                       part, tickets, (__half*)out, stream);
  return sc::dispatch_ad<64, float>(G, qkv, pos, cos_tab, sin_tab, max_pos, B, Hq, Hkv, Lmax, scale, splits, kc, vc,
                                    part, tickets, (float*)out, stream);
}

}  // extern "C"
