// K1: group-wise affine 4/8-bit dequant-GEMV for decode (M <= 16 per pass).
//
// y[m, n] = sum_k x[m, k] * w_hat[n, k],  w_hat = fp16(scale*q + bias) (exact,
// one rounding), fp32 accumulation on the tensor cores (mma.m16n8k16).
//
// Layout read (unchanged MLX format of the reference's shards):
//   wq     uint32 [N, K*bits/32], row n contiguous
//   scales fp16   [N, K/group]
//   biases fp16   [N, K/group]
//
// Vocabulary: a "chunk" is 16 consecutive uint32 words (64 B) of one weight
// row; a "tile" is 16 weight rows.  Lane (g = lane/4, t = lane%4) of a warp
// dequantises words [4t, 4t+4) of a chunk for tile rows g and g+8 into the A
// registers of mma.m16n8k16; the activation x is the B operand, staged once
// per CTA in shared memory in exactly the permuted k order the A registers
// come out in, so no shuffle is needed.  fp16 dequantisation is
// fma.rn.f16x2(q, scale, bias): bit-identical to the oracle's dequantize.
//
// Two kernels:
//   * qgemv_tma_kernel (main path): warp-specialised TMA pipeline, below.
//   * qgemv_kernel (fallback for shapes the tensor maps cannot describe:
//     K*bits/32 not a multiple of 32 words, K/group not a multiple of 8,
//     unaligned bases, segments not multiples of 16 rows): 128-bit
//     non-allocating loads straight from HBM into registers.
// Both split K across CTAs (grid.y) when x's K-slice does not fit in shared
// memory or there are too few tiles for the SMs; fp32 partials then go to a
// caller-provided workspace (summed by a second kernel), or, for an in-place
// fp32 residual epilogue, are added atomically.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sc_p2p.cuh"

namespace sc {

constexpr int QG_WARPS = 8;
constexpr int QG_THREADS = QG_WARPS * 32;
constexpr int QG_MAX_SEG = 3;
constexpr int QG_XS_MAX = 96 * 1024;  // shared-memory budget for the staged x slice (fallback)

struct QSeg {
  const uint32_t* wq;
  const uint16_t* s;
  const uint16_t* b;
  int rows;
};

struct QGemvParams {
  const void* x;
  int ldx;
  int M;   // rows of the B tile in this pass (<= 16): 2 * Mr when hilo
  int Mr;  // rows of x in this pass
  int hilo;  // batched kernel: B rows [0, Mr) carry fp16(x), rows [Mr, 2 Mr) the fp16 remainder x - fp16(x)
  int K;
  const uint16_t* norm_w;
  float eps;
  QSeg seg[QG_MAX_SEG];
  int nseg;
  int N;   // output columns: sum of segment rows (or rows of one segment for SwiGLU)
  int group;
  const uint16_t* bias;
  void* y;
  int ldy;
  const float* residual;
  int ldr;
  float* partial;        // [nacc][splits][M][N] when splits > 1
  int splits;
  int chunks_per_split;  // chunk count of each K split
  int tiles;             // ceil(N / 16)
  int lg_group;          // log2(group)
  int x_vec;             // x rows start on 16 bytes: 8 values load as one or two 16-byte vectors
  PrefetchList pf;       // the next kernel's weights, pulled into L2 by the decode kernel's producer
  unsigned long long* stamp;  // null, or {first consumer start after the dependency wait, last exit} (%globaltimer)
  // Row-parallel all-reduce in the epilogue (the transport's device copy of
  // its P2PArgs; null: off): every CTA pushes its outputs to every peer as
  // {value, epoch} half lines, then sums each output over the ranks in rank
  // order into y (fp32).  Only the kernel instances built with AR read it.
  const P2PArgs* ar;
};

// The stamp pointer the next sc_qlinear* launches of this host thread carry
// (sc_qgemv_probe_stamps).
static thread_local unsigned long long* t_next_stamp = nullptr;

template <int BITS>
struct QTraits;
template <>
struct QTraits<4> {
  static constexpr int PF = 8;    // codes per word
  static constexpr int NMMA = 8;  // mma per chunk per 16-row tile
  static constexpr int KPC = 128; // k values per chunk
};
template <>
struct QTraits<8> {
  static constexpr int PF = 4;
  static constexpr int NMMA = 4;
  static constexpr int KPC = 64;
};

// Shared-memory slot (in halves) of x[m][k] for a K-slice starting at k0.
// Row (kc_local, t) holds M * NMMA * 4 halves plus 8 halves of padding.
template <int BITS>
__device__ __forceinline__ int xslot(int kl, int m, int M) {
  using T = QTraits<BITS>;
  const int w = kl / T::PF, e = kl % T::PF;
  const int kc = w >> 4, t = (w >> 2) & 3, j = w & 3;
  int i, h;
  if (BITS == 4) {
    const int p = e & 3, hi = e >> 2;
    i = 2 * j + (p >> 1);
    h = 2 * (p & 1) + hi;
  } else {
    const int p = e & 1, hi = e >> 1;
    i = j;
    h = 2 * p + hi;
  }
  const int rowlen = M * T::NMMA * 4 + 8;
  return (kc * 4 + t) * rowlen + (m * T::NMMA + i) * 4 + h;
}

template <typename T>
__device__ __forceinline__ float ld_x(const void* x, size_t idx) {
  return to_f32<T>(reinterpret_cast<const T*>(x)[idx]);
}

// Stage x (optionally RMS-normalised) for chunks [kc0, kc1) into `xs`.
// Threads [0, nthreads) of the CTA take part; `s_rms` holds 16 floats.
template <int BITS, bool NORM, typename XT>
__device__ __forceinline__ void stage_x(const QGemvParams& p, __half* xs, float* s_rms, int kc0, int kc1, int tid,
                                        int nthreads, int bar_id) {
  using TR = QTraits<BITS>;
  const int M = p.M, Mr = p.Mr;
  const int rowlen = M * TR::NMMA * 4 + 8;
  const int warp = tid >> 5, lane = tid & 31, nwarps = nthreads >> 5;
  if (NORM) {
    for (int m = warp; m < Mr; m += nwarps) {
      float ss = 0.f;
      for (int k = lane; k < p.K; k += 32) {
        const float v = ld_x<XT>(p.x, (size_t)m * p.ldx + k);
        ss = fmaf(v, v, ss);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) s_rms[m] = sqrtf(ss / (float)p.K + p.eps);
    }
    named_bar_sync(bar_id, nthreads);
  }
  const int nkc = kc1 - kc0;
  const int k0 = kc0 * TR::KPC;
  const int span = nkc * TR::KPC;
  for (int idx = tid; idx < span * Mr; idx += nthreads) {
    const int m = idx / span, kl = idx % span;
    const int k = k0 + kl;
    float v = 0.f;
    if (k < p.K) {
      v = ld_x<XT>(p.x, (size_t)m * p.ldx + k);
      if (NORM) v = (v / s_rms[m]) * __half2float(__ushort_as_half(p.norm_w[k]));
    }
    const __half h = __float2half_rn(v);
    xs[xslot<BITS>(kl, m, M)] = h;
    if (p.hilo) xs[xslot<BITS>(kl, m + Mr, M)] = __float2half_rn(v - __half2float(h));
  }
  // zero the padding halves so no uninitialised value is ever read
  for (int r = tid; r < nkc * 4; r += nthreads)
    for (int h = M * TR::NMMA * 4; h < rowlen; ++h) xs[r * rowlen + h] = __float2half_rn(0.f);
  named_bar_sync(bar_id, nthreads);
}

// Epilogue of one output element (row, col) of a tile, from its summed
// accumulators v[NACC].
template <int EPI, typename YT>
__device__ __forceinline__ void epilogue(const QGemvParams& p, int split, bool atomic_out, int row, int col,
                                         const float* v) {
  constexpr bool DUAL = (EPI == SC_EPI_SWIGLU);
  if (atomic_out) {
    // split-K into an fp32 output that already holds the residual
    float add = v[0];
    if (split == 0 && p.bias) add += __half2float(__ushort_as_half(p.bias[row]));
    atomicAdd(reinterpret_cast<float*>(p.y) + (size_t)col * p.ldy + row, add);
    return;
  }
  if (p.splits > 1) {
    p.partial[(((size_t)0 * p.splits + split) * p.Mr + col) * p.N + row] = v[0];
    if (DUAL) p.partial[(((size_t)1 * p.splits + split) * p.Mr + col) * p.N + row] = v[DUAL ? 1 : 0];
    return;
  }
  float out;
  if (DUAL) {
    out = silu_f32(v[0]) * v[DUAL ? 1 : 0];
  } else {
    out = v[0];
    if (p.bias) out += __half2float(__ushort_as_half(p.bias[row]));
    if (EPI == SC_EPI_RESIDUAL) out += p.residual[(size_t)col * p.ldr + row];
  }
  reinterpret_cast<YT*>(p.y)[(size_t)col * p.ldy + row] = from_f32<YT>(out);
}

// ---------------------------------------------------------------------------
// Fallback: direct 128-bit loads from HBM into registers.  A CTA (8 warps)
// owns a tile at a time; its warps split the tile's chunks along K (warp w
// takes chunks w, w+8, ...) and the partial tiles are summed through shared
// memory.
template <int BITS, int MT, int EPI, bool NORM, typename XT, typename YT>
__global__ void __launch_bounds__(QG_THREADS)
qgemv_kernel(const QGemvParams p) {
  pdl_trigger();
  pdl_wait();
  using TR = QTraits<BITS>;
  constexpr int NMMA = TR::NMMA;
  constexpr bool DUAL = (EPI == SC_EPI_SWIGLU);
  constexpr int NACC = DUAL ? 2 : 1;
  constexpr int UNR = DUAL ? 2 : 4;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ float s_rms[16];
  const int M = p.M;
  const int rowlen = M * NMMA * 4 + 8;  // halves
  const int split = blockIdx.y;
  const int kc0 = split * p.chunks_per_split;
  const int KW = p.K / TR::PF;
  const int KC = (KW + 15) / 16;
  const int kc1 = min(KC, kc0 + p.chunks_per_split);
  const int nkc = kc1 - kc0;
  __half* xs = reinterpret_cast<__half*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw + (size_t)nkc * 4 * rowlen * sizeof(__half));

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;

  stage_x<BITS, NORM, XT>(p, xs, s_rms, kc0, kc1, tid, QG_THREADS, 0);

  const int gsize = p.group;
  const int KG = p.K / gsize;

  for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
    const int n0 = tile * 16;
    // resolve the two rows of this lane to (segment pointer, local row)
    const uint32_t* wrow[NACC][2];
    const uint16_t* srow[NACC][2];
    const uint16_t* brow[NACC][2];
    bool rvalid[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = n0 + g + 8 * h;
      rvalid[h] = n < p.N;
      int sidx = 0, local = n;
      if (!DUAL) {
#pragma unroll
        for (int s = 0; s < QG_MAX_SEG - 1; ++s)
          if (s + 1 < p.nseg && local >= p.seg[sidx].rows) { local -= p.seg[sidx].rows; ++sidx; }
      }
      if (!rvalid[h]) local = 0;
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        const QSeg& sg = p.seg[DUAL ? a : sidx];
        wrow[a][h] = sg.wq + (size_t)local * KW;
        srow[a][h] = sg.s + (size_t)local * KG;
        brow[a][h] = sg.b + (size_t)local * KG;
      }
    }

    float acc[NACC][MT][4];
#pragma unroll
    for (int a = 0; a < NACC; ++a)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[a][mt][r] = 0.f;

    for (int base = kc0 + warp; base < kc1; base += QG_WARPS * UNR) {
      uint4 wv[UNR][NACC][2];
      uint32_t sb[UNR][NACC][2];  // (scale | bias << 16) per row
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int kc = base + u * QG_WARPS;
        const int word = kc * 16 + 4 * t;
        const bool kval = (kc < kc1) && (word < KW);
        const int gi = kval ? (word * TR::PF) / gsize : 0;
#pragma unroll
        for (int a = 0; a < NACC; ++a)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (kval && rvalid[h]) {
              wv[u][a][h] = ldg_stream_v4(wrow[a][h] + word);
              sb[u][a][h] = (uint32_t)ldg_u16(srow[a][h] + gi) | ((uint32_t)ldg_u16(brow[a][h] + gi) << 16);
            } else {
              wv[u][a][h] = make_uint4(0, 0, 0, 0);
              sb[u][a][h] = 0u;  // scale = bias = 0 -> w_hat = 0
            }
          }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int kc = base + u * QG_WARPS;
        if (kc >= kc1) break;
        uint32_t bf[MT][NMMA][2];
        const int kcl = kc - kc0;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int m = min(mt * 8 + g, M - 1);
          const uint4* src = reinterpret_cast<const uint4*>(xs + (kcl * 4 + t) * rowlen + m * NMMA * 4);
#pragma unroll
          for (int q = 0; q < NMMA / 2; ++q) {
            const uint4 v = src[q];
            bf[mt][2 * q][0] = v.x;
            bf[mt][2 * q][1] = v.y;
            bf[mt][2 * q + 1][0] = v.z;
            bf[mt][2 * q + 1][1] = v.w;
          }
        }
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          const __half2 s0 = __half2half2(__ushort_as_half((uint16_t)(sb[u][a][0] & 0xffffu)));
          const __half2 b0 = __half2half2(__ushort_as_half((uint16_t)(sb[u][a][0] >> 16)));
          const __half2 s1 = __half2half2(__ushort_as_half((uint16_t)(sb[u][a][1] & 0xffffu)));
          const __half2 b1 = __half2half2(__ushort_as_half((uint16_t)(sb[u][a][1] >> 16)));
          const uint32_t w0[4] = {wv[u][a][0].x, wv[u][a][0].y, wv[u][a][0].z, wv[u][a][0].w};
          const uint32_t w1[4] = {wv[u][a][1].x, wv[u][a][1].y, wv[u][a][1].z, wv[u][a][1].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (BITS == 4) {
              __half2 P0[4], P1[4];
              unpack_u4(w0[j], P0);
              unpack_u4(w1[j], P1);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                P0[q] = hfma2_rn(P0[q], s0, b0);
                P1[q] = hfma2_rn(P1[q], s1, b1);
              }
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int i = 2 * j + hh;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                  mma_16816(acc[a][mt], h2_as_u32(P0[2 * hh]), h2_as_u32(P1[2 * hh]),
                            h2_as_u32(P0[2 * hh + 1]), h2_as_u32(P1[2 * hh + 1]), bf[mt][i][0],
                            bf[mt][i][1]);
              }
            } else {
              __half2 P0[2], P1[2];
              unpack_u8(w0[j], P0);
              unpack_u8(w1[j], P1);
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                P0[q] = hfma2_rn(P0[q], s0, b0);
                P1[q] = hfma2_rn(P1[q], s1, b1);
              }
#pragma unroll
              for (int mt = 0; mt < MT; ++mt)
                mma_16816(acc[a][mt], h2_as_u32(P0[0]), h2_as_u32(P1[0]), h2_as_u32(P0[1]),
                          h2_as_u32(P1[1]), bf[mt][j][0], bf[mt][j][1]);
            }
          }
        }
      }
    }

    // ---- cross-warp reduction of the tile ----
    constexpr int RPL = NACC * MT * 4;  // floats per lane per warp
#pragma unroll
    for (int a = 0; a < NACC; ++a)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 4; ++r) red[(warp * 32 + lane) * RPL + (a * MT + mt) * 4 + r] = acc[a][mt][r];
    __syncthreads();
    for (int e = tid; e < 32 * MT * 4; e += QG_THREADS) {
      const int l = e & 31, rr = e >> 5;  // rr = mt*4 + r
      const int mt = rr >> 2, r = rr & 3;
      const int row = n0 + (l >> 2) + 8 * (r >> 1);
      const int col = mt * 8 + 2 * (l & 3) + (r & 1);
      if (row >= p.N || col >= p.Mr) continue;
      // the remainder column of a hi / lo pass: same tile row, B column col + Mr
      const int cl = col + p.Mr;
      const int l2 = (l & ~3) | ((cl & 7) >> 1), mt2 = cl >> 3, r2 = (r & 2) | (cl & 1);
      float v[NACC];
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        float sacc = 0.f, slo = 0.f;
#pragma unroll
        for (int w = 0; w < QG_WARPS; ++w) sacc += red[(w * 32 + l) * RPL + (a * MT + mt) * 4 + r];
        if (p.hilo) {
#pragma unroll
          for (int w = 0; w < QG_WARPS; ++w) slo += red[(w * 32 + l2) * RPL + (a * MT + mt2) * 4 + r2];
        }
        v[a] = sacc + slo;
      }
      epilogue<EPI, YT>(p, split, false, row, col, v);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised TMA pipeline (the main decode path).
//
// One producer warp streams each tile's K-range into a ring of NST
// shared-memory stages with tensor-map TMA: per stage ONE
// cp.async.bulk.tensor brings 16 rows x (cps*16) packed words (a 3-D box,
// 128-byte swizzled), and one each brings the matching 16 x (groups) fp16
// scales and biases (swizzled to their row width).  All complete on the
// stage's "full" mbarrier by byte count; a TMA copy has a fixed issue cost,
// so a stage is a few large boxes rather than many row copies.  Sixteen
// consumer warps wait on "full", dequantise from shared memory exactly as the
// fallback does from registers, feed mma.m16n8k16 and release the stage on
// its "empty" mbarrier, so the producer runs up to NST stages ahead.  Tile
// rows are read in a permuted order (mma row m <-> tile row tile_row(m)) so
// the 128-bit shared loads of one quarter-warp hit different swizzle phases
// and never conflict.  Every wait is bounded in time; on timeout the CTA
// stops, drains its in-flight copies and records an error readable through
// sc_qgemv_device_error().
constexpr int TC_NCW = 16;  // consumer warps
constexpr int TC_THREADS = (TC_NCW + 1) * 32;
constexpr int TC_MAX_NST = 12;
constexpr uint64_t TC_WAIT_NS = 2000000000ull;  // 2 s

static __device__ int g_qgemv_error = 0;

struct TmaGeo {
  int cps;          // chunks (16 words) per stage
  int nblk;         // 32-word blocks per stage (cps / 2)
  int ngs;          // scale groups per stage (box width)
  int nst;          // ring depth
  int wset_bytes;   // bytes of one weight set's packed-word box (16 * nblk * 128)
  int sset_bytes;   // bytes of one scales (or biases) box slot, 1 KB aligned
  int stage_bytes;  // bytes of one stage (all sets)
  int ring_off;     // byte offset of the ring in dynamic shared memory (1 KB aligned)
  int red_off;      // byte offset of the reduction buffer
  int bar_off;      // byte offset of the mbarriers
  int atomic_out;   // split-K partials added atomically into y (in-place residual)
  int row_swz;      // 1: box lines ordered (block, row) with row-dependent swizzle
  int s_swz;        // scale-box swizzle mask: 0 none, 1 (32 B), 3 (64 B), 7 (128 B)
  int pre_stages;   // factored kernel: stages the producer issues before x is staged
  int pf_after;     // factored kernel: L2 prefetch waits until this CTA's last stage has landed
  int acc_off;      // factored kernel: byte offset of the per-tile output accumulators
  int acc_floats;   // factored kernel: their count (tiles of a CTA x 16 rows x M x sets)
  int warp_slots;   // factored kernel: 1 = an fp32 slot per consumer warp and output, summed in
                    // warp order by the epilogue; 0 = one 64-bit fixed-point slot per output
                    // that the warps add into with shared atomics (when the slots do not fit)
};

struct TmaMaps {
  CUtensorMap w[QG_MAX_SEG];
  CUtensorMap s[QG_MAX_SEG];
  CUtensorMap b[QG_MAX_SEG];
};

// Weights are read once per decode step (gigabytes apart), so their L2 lines
// are marked evict-first: streaming them must not push out what is reused
// (activations, KV, and weights prefetched ahead by sc_l2_prefetch).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// tile row read by mma row m (0..15): quarter-warps pair rows 4 apart
__device__ __forceinline__ int tile_row(int m) { return ((m & 7) >> 1) + 4 * (m & 1) + (m & 8); }

// segment of a tile (segments are multiples of 16 rows except the last)
__device__ __forceinline__ int tile_segment(const QGemvParams& p, int n0, int* base) {
  int sidx = 0, b = 0;
#pragma unroll
  for (int s = 0; s < QG_MAX_SEG - 1; ++s)
    if (s + 1 < p.nseg && n0 >= b + p.seg[sidx].rows) { b += p.seg[sidx].rows; ++sidx; }
  *base = b;
  return sidx;
}

template <int BITS, int MT, int EPI, bool NORM, typename XT, typename YT>
__global__ void __launch_bounds__(TC_THREADS, 1)
qgemv_tma_kernel(const QGemvParams p, const TmaGeo geo, const __grid_constant__ TmaMaps maps) {
  using TR = QTraits<BITS>;
  constexpr int NMMA = TR::NMMA;
  constexpr bool DUAL = (EPI == SC_EPI_SWIGLU);
  constexpr int NACC = DUAL ? 2 : 1;
  constexpr int NA = DUAL ? 2 : 4;  // independent accumulators per weight set
  constexpr int RPL = NACC * MT * 4;
  constexpr int NC = TC_NCW * 32;

  extern __shared__ __align__(128) unsigned char smem_tma[];
  __shared__ int s_abort;
  __shared__ float s_rms[16];

  const int M = p.M;
  const int rowlen = M * NMMA * 4 + 8;
  const int split = blockIdx.y;
  const int kc0 = split * p.chunks_per_split;
  const int KW = p.K / TR::PF;
  const int KC = (KW + 15) / 16;
  const int kc1 = min(KC, kc0 + p.chunks_per_split);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // swizzled TMA boxes need 1024-byte aligned shared addresses
  unsigned char* sbase = smem_tma + ((1024 - (smem_u32(smem_tma) & 1023)) & 1023);

  __half* xs = reinterpret_cast<__half*>(sbase);
  unsigned char* ring = sbase + geo.ring_off;
  float* red = reinterpret_cast<float*>(sbase + geo.red_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + geo.bar_off);
  uint64_t* empty = full + TC_MAX_NST;

  if (tid == 0) {
    for (int s = 0; s < geo.nst; ++s) {
      mbar_init(&full[s], 1);  // one expect_tx arrival; completion by the copies' bytes
      mbar_init(&empty[s], TC_NCW);
    }
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == TC_NCW) {
    // The producer streams weights, scales and biases only -- data no kernel
    // of the step writes -- so it starts before the predecessor kernel has
    // finished (no pdl_wait here); the consumers' pdl_wait orders everything
    // that touches activations.
    // ============================ producer ============================
    if (lane == 0) {
      uint32_t it = 0;
      const uint32_t tx = (uint32_t)(NACC * (geo.wset_bytes + 2 * 16 * geo.ngs * 2));
      const uint64_t pol = l2_evict_first_policy();
      for (int tile = blockIdx.x; tile < p.tiles && !s_abort; tile += gridDim.x) {
        const int n0 = tile * 16;
        int sbase_row = 0;
        const int sidx = DUAL ? 0 : tile_segment(p, n0, &sbase_row);
        const int row0 = n0 - sbase_row;
        for (int kcs = kc0; kcs < kc1; kcs += geo.cps) {
          const int s = it % geo.nst;
          const uint32_t ph = (it / geo.nst) & 1;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1, &s_abort, TC_WAIT_NS)) break;
          unsigned char* st = ring + (size_t)s * geo.stage_bytes;
          const int blk0 = kcs / 2;                // 32-word blocks
          const int g0 = kcs * TR::KPC / p.group;  // scale groups
          mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            const int mi = DUAL ? a : sidx;
            unsigned char* wd = st + a * geo.wset_bytes;
            if (geo.row_swz)
              tma_load_3d(wd, &maps.w[mi], 0, row0, blk0, &full[s], pol);
            else
              tma_load_3d(wd, &maps.w[mi], 0, blk0, row0, &full[s], pol);
            unsigned char* sd = st + NACC * geo.wset_bytes + (a * 2) * geo.sset_bytes;
            tma_load_2d(sd, &maps.s[mi], g0, row0, &full[s], pol);
            tma_load_2d(sd + geo.sset_bytes, &maps.b[mi], g0, row0, &full[s], pol);
          }
          ++it;
        }
      }
      if (s_abort) {
        // drain: let every issued stage land before the CTA can exit
        for (uint32_t k = (it > (uint32_t)geo.nst ? it - geo.nst : 0); k < it; ++k) {
          int dummy = 0;
          mbar_wait_bounded(&full[k % geo.nst], (k / geo.nst) & 1, (volatile int*)&dummy, TC_WAIT_NS / 4);
        }
        atomicExch(&g_qgemv_error, 1);
      }
    }
    return;
  }

  // ============================ consumers ============================
  const int g = lane >> 2, t = lane & 3;
  pdl_wait();  // x (and the residual / output buffers) belong to the predecessor until here
  stage_x<BITS, NORM, XT>(p, xs, s_rms, kc0, kc1, tid, NC, 1);

  // Work items of a stage: NACC weight sets x nch chunks; warp w takes items
  // w and w + TC_NCW.  When the stage is full and holds exactly two items per
  // warp (the planned shape), an item's chunk and set are fixed per warp, so
  // its shared-memory offsets are computed once here; the rows g+8 sit at a
  // constant stride from rows g (the swizzle phase repeats every 8 rows).
  // Rows past N and blocks past K arrive zero-filled from TMA (scale = bias =
  // 0 makes w_hat = 0), so the loop needs no bounds tests.
  const int pr0 = tile_row(g);  // tile row of mma row g (mma row g+8 -> pr0 + 8)
  const int lgG = p.lg_group;
  const int w_r8 = geo.row_swz ? 1024 : 8 * geo.nblk * 128;
  const int s_r8 = 16 * geo.ngs;
  int xm[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) xm[mt] = min(mt * 8 + g, M - 1) * NMMA * 4;

  auto woff = [&](int c) -> int {  // packed-word box offset of (chunk c, row pr0, unit t)
    const int u = ((c & 1) << 2) | t;
    if (geo.row_swz) return (c >> 1) * 2048 + pr0 * 128 + ((u ^ (pr0 & 7)) << 4);
    const int l = pr0 * geo.nblk + (c >> 1);
    return l * 128 + ((u ^ (l & 7)) << 4);
  };
  auto soff = [&](int c) -> int {  // scales box offset of (row pr0, group of chunk c / lane t)
    const int gi = ((c * 16 + 4 * t) * TR::PF) >> lgG;
    const int lo = pr0 * geo.ngs * 2 + gi * 2;
    return lo ^ (((lo >> 7) & geo.s_swz) << 4);
  };
  const bool fast_shape = NACC * geo.cps == 2 * TC_NCW;
  int fw[2], fs[2], fx[2];  // per fast-path item: word / scale / x offsets
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = DUAL ? warp : warp + j * TC_NCW;
    const int aset = DUAL ? j : 0;
    fw[j] = aset * geo.wset_bytes + woff(c);
    fs[j] = NACC * geo.wset_bytes + (aset * 2) * geo.sset_bytes + soff(c);
    fx[j] = (c * 4 + t) * rowlen;
  }

  struct Item {
    uint4 w0, w1;
    uint32_t sb0, sb1;
    uint32_t bf[MT][NMMA][2];
  };
  auto load_item = [&](Item& d, const unsigned char* st, const __half* xst, int wo, int so, int xo) {
    d.w0 = *reinterpret_cast<const uint4*>(st + wo);
    d.w1 = *reinterpret_cast<const uint4*>(st + wo + w_r8);
    d.sb0 = (uint32_t)*reinterpret_cast<const uint16_t*>(st + so) |
            ((uint32_t)*reinterpret_cast<const uint16_t*>(st + so + geo.sset_bytes) << 16);
    d.sb1 = (uint32_t)*reinterpret_cast<const uint16_t*>(st + so + s_r8) |
            ((uint32_t)*reinterpret_cast<const uint16_t*>(st + so + s_r8 + geo.sset_bytes) << 16);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint4* src = reinterpret_cast<const uint4*>(xst + xo + xm[mt]);
#pragma unroll
      for (int q = 0; q < NMMA / 2; ++q) {
        const uint4 v = src[q];
        d.bf[mt][2 * q][0] = v.x;
        d.bf[mt][2 * q][1] = v.y;
        d.bf[mt][2 * q + 1][0] = v.z;
        d.bf[mt][2 * q + 1][1] = v.w;
      }
    }
  };
  float acc[NACC][NA][MT][4];
  auto compute_item = [&](const Item& d, int aset) {
    const __half2 s0 = __half2half2(__ushort_as_half((uint16_t)(d.sb0 & 0xffffu)));
    const __half2 b0 = __half2half2(__ushort_as_half((uint16_t)(d.sb0 >> 16)));
    const __half2 s1 = __half2half2(__ushort_as_half((uint16_t)(d.sb1 & 0xffffu)));
    const __half2 b1 = __half2half2(__ushort_as_half((uint16_t)(d.sb1 >> 16)));
    const uint32_t w0[4] = {d.w0.x, d.w0.y, d.w0.z, d.w0.w};
    const uint32_t w1[4] = {d.w1.x, d.w1.y, d.w1.z, d.w1.w};
#pragma unroll
    for (int aa = 0; aa < NACC; ++aa) {
      if (NACC == 2 && aa != aset) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (BITS == 4) {
          __half2 P0[4], P1[4];
          unpack_u4(w0[j], P0);
          unpack_u4(w1[j], P1);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            P0[q] = hfma2_rn(P0[q], s0, b0);
            P1[q] = hfma2_rn(P1[q], s1, b1);
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int i = 2 * j + hh;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
              mma_16816(acc[aa][i % NA][mt], h2_as_u32(P0[2 * hh]), h2_as_u32(P1[2 * hh]),
                        h2_as_u32(P0[2 * hh + 1]), h2_as_u32(P1[2 * hh + 1]), d.bf[mt][i][0], d.bf[mt][i][1]);
          }
        } else {
          __half2 P0[2], P1[2];
          unpack_u8(w0[j], P0);
          unpack_u8(w1[j], P1);
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            P0[q] = hfma2_rn(P0[q], s0, b0);
            P1[q] = hfma2_rn(P1[q], s1, b1);
          }
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            mma_16816(acc[aa][j % NA][mt], h2_as_u32(P0[0]), h2_as_u32(P1[0]), h2_as_u32(P0[1]),
                      h2_as_u32(P1[1]), d.bf[mt][j][0], d.bf[mt][j][1]);
        }
      }
    }
  };

  int s = 0;
  uint32_t ph = 0;
  int rbuf = 0;
  bool aborted = false;
  for (int tile = blockIdx.x; tile < p.tiles && !aborted; tile += gridDim.x) {
    const int n0 = tile * 16;
#pragma unroll
    for (int a = 0; a < NACC; ++a)
#pragma unroll
      for (int q = 0; q < NA; ++q)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[a][q][mt][r] = 0.f;

    for (int kcs = kc0; kcs < kc1; kcs += geo.cps) {
      if (!mbar_wait_bounded(&full[s], ph, &s_abort, TC_WAIT_NS)) { aborted = true; break; }
      const unsigned char* st = ring + (size_t)s * geo.stage_bytes;
      const __half* xst = xs + (kcs - kc0) * 4 * rowlen;
      const int nch = min(kc1 - kcs, geo.cps);
      if (fast_shape && nch == geo.cps) {
        if (MT == 1) {
          // both items in flight before either is computed
          Item da, db;
          load_item(da, st, xst, fw[0], fs[0], fx[0]);
          load_item(db, st, xst, fw[1], fs[1], fx[1]);
          compute_item(da, 0);
          compute_item(db, DUAL ? 1 : 0);
        } else {
          Item da;
          load_item(da, st, xst, fw[0], fs[0], fx[0]);
          compute_item(da, 0);
          load_item(da, st, xst, fw[1], fs[1], fx[1]);
          compute_item(da, DUAL ? 1 : 0);
        }
      } else {
        for (int i = warp; i < NACC * nch; i += TC_NCW) {
          const int aset = (NACC == 2 && i >= nch) ? 1 : 0;
          const int c = i - aset * nch;
          Item da;
          load_item(da, st, xst, aset * geo.wset_bytes + woff(c),
                    NACC * geo.wset_bytes + (aset * 2) * geo.sset_bytes + soff(c), (c * 4 + t) * rowlen);
          compute_item(da, aset);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == geo.nst) {
        s = 0;
        ph ^= 1;
      }
    }
    if (aborted) break;

    // ---- cross-warp reduction and epilogue (consumer warps only) ----
    // red is double-buffered by tile, so one barrier per tile suffices: the
    // next-but-one tile's writes come after every thread passed the next
    // tile's barrier, i.e. after these reads.
    float* rb = red + rbuf * (TC_NCW * 32 * RPL);
    rbuf ^= 1;
#pragma unroll
    for (int a = 0; a < NACC; ++a)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < NA; ++q) v += acc[a][q][mt][r];
          rb[(warp * 32 + lane) * RPL + (a * MT + mt) * 4 + r] = v;
        }
    named_bar_sync(1, NC);
    for (int e = tid; e < 32 * MT * 4; e += NC) {
      const int l = e & 31, rr = e >> 5;
      const int mt = rr >> 2, r = rr & 3;
      const int row = n0 + tile_row((l >> 2) + 8 * (r >> 1));
      const int col = mt * 8 + 2 * (l & 3) + (r & 1);
      if (row >= p.N || col >= p.Mr) continue;
      // the remainder column of a hi / lo pass: same tile row, B column col + Mr
      const int cl = col + p.Mr;
      const int l2 = (l & ~3) | ((cl & 7) >> 1), mt2 = cl >> 3, r2 = (r & 2) | (cl & 1);
      float v[NACC];
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        float sacc = 0.f, slo = 0.f;
#pragma unroll
        for (int w = 0; w < TC_NCW; ++w) sacc += rb[(w * 32 + l) * RPL + (a * MT + mt) * 4 + r];
        if (p.hilo) {
#pragma unroll
          for (int w = 0; w < TC_NCW; ++w) slo += rb[(w * 32 + l2) * RPL + (a * MT + mt2) * 4 + r2];
        }
        v[a] = sacc + slo;
      }
      epilogue<EPI, YT>(p, split, geo.atomic_out != 0, row, col, v);
    }
  }
  if (aborted && lane == 0) atomicExch(&g_qgemv_error, 1);
}

// ---------------------------------------------------------------------------
// Factored decode kernel (M * NGC <= 4, the batch-1 decode case).
//
// Same TMA ring and producer as qgemv_tma_kernel, different arithmetic: the
// weights are never rounded.  Per group,
//     y += scale * sum_k q_k x_k  +  bias * sum_k x_k
// with q_k the exact integer codes.  The A registers hold 1024 + q, or
// 1024 + 16 q for the odd nibbles of a 4-bit word whose x slots then carry
// x / 16 (one AND/OR per pair of codes, no conversion arithmetic); the excess
// 1024 * sum(B) is cancelled by starting the mma accumulator at -1024 * sum(B)
// for that column.  x itself is split into an fp16 high part and an fp16 low part
// (x - hi), carried in otherwise idle columns of the n8 mma tile, so the
// products see x to ~22 bits.  Because the four k-lanes of an mma can hold
// codes of different groups (lane t owns words 4t..4t+3 of a chunk), the B
// tile gives every (batch row m, part, group) its own column: column
// n = (m * 2 + part) * NGC + group, NGC = groups per chunk (1, 2 or 4).
// A lane's B value is x where its words' group matches the column, else 0.
//
// Each consumer warp accumulates its chunks of a tile in registers, reduces
// over its k-lanes, and stores the tile's 16 row sums into its own fp32 slot
// of the tile (no atomics); the CTA's epilogue sums a row's slots in warp
// order after one barrier.  When the slots of all the CTA's tiles do not fit,
// the warps instead add 64-bit fixed-point sums with shared atomics.  No
// CTA-wide barrier sits in the streaming loop.

// 64-bit two's-complement fixed point with 32 fraction bits (|v| < 2^31).
// v * 2^32 is exact in fp32 (a power-of-two scale), so one float -> int64
// conversion rounds exactly as the same product in double would.
__device__ __forceinline__ unsigned long long fx_to_fixed(float v) {
  return (unsigned long long)__float2ll_rn(v * 4294967296.0f);
}
__device__ __forceinline__ float fx_from_fixed(unsigned long long u) {
  return (float)((double)(long long)u * (1.0 / 4294967296.0));
}

// (w & MASK) | 0x64006400 as one three-input logic op: written in C++ the
// compiler splits it in two when the results feed mma operands.
template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or_mag(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(d) : "r"(w), "n"(MASK), "n"(0x64006400u));
  return d;
}

template <int BITS>
__device__ __forceinline__ void unpack_off(uint32_t w, uint32_t (&a)[4]) {
  // fp16 pairs, exact: 4-bit (e0,e4) = 1024 + q, (e1,e5) = 1024 + 16 q, (e2,e6) = 1024 + q,
  // (e3,e7) = 1024 + 16 q -- the x slots of the odd codes hold x / 16; 8-bit (e0,e2) (e1,e3) = 1024 + q
  if (BITS == 4) {
    const uint32_t w8 = w >> 8;
    a[0] = and_or_mag<0x000F000Fu>(w);
    a[1] = and_or_mag<0x00F000F0u>(w);
    a[2] = and_or_mag<0x000F000Fu>(w8);
    a[3] = and_or_mag<0x00F000F0u>(w8);
  } else {
    a[0] = and_or_mag<0x00FF00FFu>(w);
    a[1] = and_or_mag<0x00FF00FFu>(w >> 8);
    a[2] = a[3] = 0u;
  }
}

// Bytes of staged x per chunk: [m][part][q][t] 16-byte B-fragment units, then
// a 64-byte table {xoff(2t), xoff(2t+1), xsum(2t), xsum(2t+1)} per lane t.
__host__ __device__ constexpr int fx_chunk_bytes(int bits, int M) { return M * 2 * (bits == 4 ? 4 : 2) * 64 + 64; }

// 8 consecutive x values of row m from k0 (k0 + 8 <= K), as floats.
template <typename XT>
__device__ __forceinline__ void ld_x8(const QGemvParams& p, int m, int k0, float (&v)[8]) {
  const size_t base = (size_t)m * p.ldx + k0;
  if (p.x_vec) {
    if constexpr (sizeof(XT) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + base);
      const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + base + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      const uint4 a = *reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x) + base);
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(u32_as_h2(w[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = ld_x<XT>(p.x, base + i);
  }
}

// Per-warp x staging for the factored kernel: consumer warp w stages exactly
// the chunks it consumes (w, w + cps, w + 2 cps, ... of the K slice), so it
// needs no CTA barrier before its first stage -- a __syncwarp orders its own
// lanes' writes.  Lanes take (chunk, unit) pairs, UPC units per chunk, so a
// column-group's units are an aligned lane group and its sums reduce by
// shuffles.  With RMSNorm the staged values are x * norm_weight (unscaled):
// the product is linear in x, so the kernel divides its outputs by the row's
// rms at the end instead; this warp's share of sum(x^2) over the whole row
// goes to s_ss[warp][m] and is summed in warp order at the end
// (deterministic).  When the CTA stages the whole row (one K split) that
// share is taken from the values the warp stages anyway (one round trip to
// L2); otherwise from a contiguous K / TC_NCW slice of the row.
constexpr int FXW_PASSES = 4;  // (chunk, unit) passes a warp keeps in registers per batch

template <int BITS, int NGC, bool NORM, typename XT>
__device__ __forceinline__ void stage_x_fx_warp(const QGemvParams& p, unsigned char* xsb, float (*s_ss)[4],
                                                int kc0, int kc1, int cps, int warp, int lane) {
  using TR = QTraits<BITS>;
  constexpr int XQ = TR::NMMA / 2;
  constexpr int UPC = TR::KPC / 8;       // units per chunk
  constexpr int GU = TR::KPC / NGC / 8;  // units of one column-group inside a chunk (>= 4)
  constexpr int CPP = 32 / UPC;          // chunks per pass
  const int M = p.M;
  const int CB = fx_chunk_bytes(BITS, M);
  const int nkc = kc1 - kc0;
  // this warp's chunks: cl = warp + j * cps (the consumer of chunk cl is warp cl % cps), one
  // per stage of a tile; slots past the slice's last chunk (a tile's last stage
  // may be partly empty) are staged as zeros, so their weights add nothing
  const int nj = warp < cps ? (nkc + cps - 1) / cps : 0;
  const int npass = (nj + CPP - 1) / CPP * M;                     // (pass, row) items
  const int jl = lane / UPC, uc = lane % UPC;                      // chunk within a pass, unit
  const bool ss_in_pass = NORM && p.splits == 1;  // the warps' chunks cover the whole row
  float ssm[4] = {0.f, 0.f, 0.f, 0.f};             // this lane's sum(x^2) per batch row
  if (NORM && !ss_in_pass) {
    // sum(x^2) over this warp's contiguous slice of the full row, 8 values per lane per step
    const int per = ((p.K + TC_NCW - 1) / TC_NCW + 7) / 8 * 8;  // 8-aligned slices: vector loads
    const int k_lo = min(p.K, warp * per), k_hi = min(p.K, k_lo + per);
    for (int m = 0; m < M; ++m) {
      float ss = 0.f;
      for (int k0 = k_lo + lane * 8; k0 < k_hi; k0 += 256) {
        float v[8];
        if (k0 + 8 <= k_hi) {
          ld_x8<XT>(p, m, k0, v);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = k0 + i < k_hi ? ld_x<XT>(p.x, (size_t)m * p.ldx + k0 + i) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) s_ss[warp][m] = ss;
    }
  }
  for (int it0 = 0; it0 < npass; it0 += FXW_PASSES) {
    float v[FXW_PASSES][8];
    uint4 nwr[NORM ? FXW_PASSES : 1];
#pragma unroll
    for (int b = 0; b < FXW_PASSES; ++b) {
      const int it = it0 + b;
      const int m = it % M, j = (it / M) * CPP + jl;
      const int cl = warp + j * cps;
      const int k0 = (kc0 + cl) * TR::KPC + uc * 8;
      if (it < npass && j < nj && cl < nkc && k0 < p.K) {
        ld_x8<XT>(p, m, k0, v[b]);
        if (NORM) {
          const uint16_t* nwp = p.norm_w + k0;
          nwr[NORM ? b : 0] = p.x_vec ? *reinterpret_cast<const uint4*>(nwp)
                                      : make_uint4(nwp[0] | ((uint32_t)nwp[1] << 16), nwp[2] | ((uint32_t)nwp[3] << 16),
                                                   nwp[4] | ((uint32_t)nwp[5] << 16), nwp[6] | ((uint32_t)nwp[7] << 16));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[b][i] = 0.f;
        if (NORM) nwr[NORM ? b : 0] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int b = 0; b < FXW_PASSES; ++b) {
      const int it = it0 + b;
      if (it >= npass) break;  // warp-uniform
      const int m = it % M, j = (it / M) * CPP + jl;
      const bool ok = j < nj;
      const int cl = warp + (ok ? j : 0) * cps;
      float x[8];
      if (NORM && ss_in_pass) {
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) sq = fmaf(v[b][i], v[b][i], sq);
#pragma unroll
        for (int mm = 0; mm < 4; ++mm)
          if (mm == m) ssm[mm] += sq;
      }
      if (NORM) {
        const uint32_t nww[4] = {nwr[NORM ? b : 0].x, nwr[NORM ? b : 0].y, nwr[NORM ? b : 0].z, nwr[NORM ? b : 0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(u32_as_h2(nww[i]));
          x[2 * i] = v[b][2 * i] * f.x;
          x[2 * i + 1] = v[b][2 * i + 1] * f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = v[b][i];
      }
      __half hi[8], lo[8];
      float shp[4], slp[4], sxp[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // element pairs (even, odd), converted two at a time
        // odd codes arrive as 16 q: their x slots carry x / 16 (an exact scale)
        const float a = x[2 * i], b = BITS == 4 ? x[2 * i + 1] * 0.0625f : x[2 * i + 1];
        const __half2 hp = __floats2half2_rn(a, b);
        const float2 hf = __half22float2(hp);
        const __half2 lp = __floats2half2_rn(a - hf.x, b - hf.y);
        const float2 lf = __half22float2(lp);
        shp[i] = hf.x + hf.y;
        slp[i] = lf.x + lf.y;
        sxp[i] = x[2 * i] + x[2 * i + 1];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int e = 2 * i + u;
          const int pos = BITS == 4 ? 4 * ((e >> 1) & 1) + 2 * (e & 1) + (e >> 2)
                                    : 4 * (e >> 2) + 2 * (e & 1) + ((e >> 1) & 1);
          hi[pos] = u ? __high2half(hp) : __low2half(hp);
          lo[pos] = u ? __high2half(lp) : __low2half(lp);
        }
      }
      float sh = (shp[0] + shp[1]) + (shp[2] + shp[3]);
      float sl = (slp[0] + slp[1]) + (slp[2] + slp[3]);
      float sx = (sxp[0] + sxp[1]) + (sxp[2] + sxp[3]);
#pragma unroll
      for (int o = 1; o < GU; o <<= 1) {
        sh += __shfl_xor_sync(0xffffffffu, sh, o);
        sl += __shfl_xor_sync(0xffffffffu, sl, o);
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
      }
      if (!ok) continue;
      unsigned char* cb = xsb + (size_t)cl * CB;
      const int t = BITS == 4 ? (uc >> 2) : (uc >> 1);
      const int q = BITS == 4 ? (uc & 3) : (uc & 1);
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const __half* src = part ? lo : hi;
        uint4 o;
        o.x = h2_as_u32(__halves2half2(src[0], src[1]));
        o.y = h2_as_u32(__halves2half2(src[2], src[3]));
        o.z = h2_as_u32(__halves2half2(src[4], src[5]));
        o.w = h2_as_u32(__halves2half2(src[6], src[7]));
        *reinterpret_cast<uint4*>(cb + (((m * 2 + part) * XQ + q) * 4 + t) * 16) = o;
      }
      if (uc % GU == 0) {
        const int grp = uc / GU;
        float* tab = reinterpret_cast<float*>(cb + M * 2 * XQ * 64);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const int col = (m * 2 + part) * NGC + grp;  // < 8
          tab[(col >> 1) * 4 + (col & 1)] = -1024.f * (part ? sl : sh);
          tab[(col >> 1) * 4 + 2 + (col & 1)] = part ? 0.f : sx;
        }
      }
    }
  }
  if (NORM && ss_in_pass) {
#pragma unroll
    for (int mm = 0; mm < 4; ++mm) {
      if (mm >= M) break;  // warp-uniform
      float ss = ssm[mm];
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) s_ss[warp][mm] = ss;
    }
  }
  // columns no (m, part, group) maps to: zero table entries of this warp's chunks
  for (int idx = lane; idx < nj * 8; idx += 32) {
    const int cl = warp + (idx >> 3) * cps, col = idx & 7;
    if (col >= M * 2 * NGC) {
      float* tab = reinterpret_cast<float*>(xsb + (size_t)cl * CB + M * 2 * XQ * 64);
      tab[(col >> 1) * 4 + (col & 1)] = 0.f;
      tab[(col >> 1) * 4 + 2 + (col & 1)] = 0.f;
    }
  }
  __syncwarp();
}

// AR: the epilogue runs the row-parallel all-reduce (p.ar); a template
// parameter, so the other instances carry none of its code.
template <int BITS, int NGC, int EPI, bool NORM, typename XT, typename YT, bool AR = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
qgemv_fx_kernel(const QGemvParams p, const TmaGeo geo, const __grid_constant__ TmaMaps maps) {
  using TR = QTraits<BITS>;
  constexpr int NMMA = TR::NMMA;
  constexpr int XQ = NMMA / 2;
  constexpr bool DUAL = (EPI == SC_EPI_SWIGLU);
  constexpr int NACC = DUAL ? 2 : 1;
  constexpr int NC = TC_NCW * 32;

  extern __shared__ __align__(128) unsigned char smem_tma[];
  __shared__ int s_abort;
  __shared__ float s_part[TC_NCW][4];
  __shared__ __align__(8) uint64_t s_xready;  // consumers have staged x (lets the producer run on)
  __shared__ __align__(16) uint4 s_zero[XQ * 4];  // B fragments of lanes that feed no column

  const int M = p.M;
  const int split = blockIdx.y;
  const int kc0 = split * p.chunks_per_split;
  const int KW = p.K / TR::PF;
  const int KC = (KW + 15) / 16;
  const int kc1 = min(KC, kc0 + p.chunks_per_split);
  const int tid = threadIdx.x;
  // warp index through a shuffle: the compiler then knows it is warp-uniform
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  unsigned char* sbase = smem_tma + ((1024 - (smem_u32(smem_tma) & 1023)) & 1023);
  unsigned char* xsb = sbase;
  unsigned char* ring = sbase + geo.ring_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(sbase + geo.bar_off);
  uint64_t* empty = full + TC_MAX_NST;

  // Per-output accumulators of the CTA's tiles in 64-bit fixed point
  // (2^-32 units): integer atomics make the sum over warps independent of
  // their order, so every run (and every replay) gives the same bits.
  // Per-output partial sums of the CTA's tiles, deterministic either way:
  // warp slots [tile][row][m][set][warp] (fp32, every owning warp writes each
  // of its tiles once), or 64-bit fixed point (2^-32 units) added with integer
  // atomics, whose sum does not depend on the order of the adds.
  unsigned long long* s_acc = reinterpret_cast<unsigned long long*>(sbase + geo.acc_off);
  float* s_slot = reinterpret_cast<float*>(sbase + geo.acc_off);
  if (!geo.warp_slots)
    for (int i = tid; i < geo.acc_floats; i += blockDim.x) s_acc[i] = 0ull;
  if (tid < XQ * 4) s_zero[tid] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    for (int s = 0; s < geo.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 32 * geo.cps);  // every lane of the warps that own a chunk
    }
    mbar_init(&s_xready, TC_NCW);
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == TC_NCW) {
    // producer: weights / scales / biases only, so no pdl_wait (see pdl_wait)
    if (lane == 0) {
      uint32_t it = 0;
      const uint32_t tx = (uint32_t)(NACC * (geo.wset_bytes + 2 * 16 * geo.ngs * 2));
      const uint64_t pol = l2_evict_first_policy();
      for (int tile = blockIdx.x; tile < p.tiles && !s_abort; tile += gridDim.x) {
        const int n0 = tile * 16;
        int sbase_row = 0;
        const int sidx = DUAL ? 0 : tile_segment(p, n0, &sbase_row);
        const int row0 = n0 - sbase_row;
        for (int kcs = kc0; kcs < kc1; kcs += geo.cps) {
          const int s = it % geo.nst;
          const uint32_t ph = (it / geo.nst) & 1;
          // the first pre_stages go out at once (before the predecessor
          // kernel has even finished); the rest wait until x is staged, so
          // the consumers' activation loads do not queue behind a full ring
          if ((int)it == geo.pre_stages && !mbar_wait_bounded(&s_xready, 0, &s_abort, TC_WAIT_NS)) break;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1, &s_abort, TC_WAIT_NS)) break;
          unsigned char* st = ring + (size_t)s * geo.stage_bytes;
          const int blk0 = kcs / 2;
          const int g0 = kcs * TR::KPC / p.group;
          mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            const int mi = DUAL ? a : sidx;
            unsigned char* wd = st + a * geo.wset_bytes;
            if (geo.row_swz)
              tma_load_3d(wd, &maps.w[mi], 0, row0, blk0, &full[s], pol);
            else
              tma_load_3d(wd, &maps.w[mi], 0, blk0, row0, &full[s], pol);
            unsigned char* sd = st + NACC * geo.wset_bytes + (a * 2) * geo.sset_bytes;
            tma_load_2d(sd, &maps.s[mi], g0, row0, &full[s], pol);
            tma_load_2d(sd + geo.sset_bytes, &maps.b[mi], g0, row0, &full[s], pol);
          }
          ++it;
        }
      }
      if (p.pf.count && !s_abort) {
        // The next kernel's weights: once this CTA's own last stage has
        // landed, HBM would otherwise idle through the consumers' drain, the
        // epilogue and the next kernel's start, so pull this CTA's share of
        // them into L2 now (issued earlier they would compete with its own).
        const uint32_t k = it ? it - 1 : 0;
        if (!it || !geo.pf_after ||
            mbar_wait_bounded(&full[k % geo.nst], (k / geo.nst) & 1, &s_abort, TC_WAIT_NS))
          l2_prefetch_share(p.pf, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
      }
      if (s_abort) {
        for (uint32_t k = (it > (uint32_t)geo.nst ? it - geo.nst : 0); k < it; ++k) {
          int dummy = 0;
          mbar_wait_bounded(&full[k % geo.nst], (k / geo.nst) & 1, (volatile int*)&dummy, TC_WAIT_NS / 4);
        }
        atomicExch(&g_qgemv_error, 1);
      }
    }
    return;
  }

  // ============================ consumers ============================
  const int g = lane >> 2, t = lane & 3;
  pdl_wait();
  if (p.stamp && tid == 0) atomicMin(p.stamp, (unsigned long long)globaltimer_ns());
  __shared__ uint32_t s_ep;    // this CTA's epoch of the fused all-reduce
  __shared__ int s_ar_skip;    // the transport already failed: no waits
  if constexpr (AR) {
    if (tid == 0) {
      // the previous fused call (an earlier kernel) is complete: its counter is final
      const P2PArgs& A = *p.ar;
      const uint32_t e = A.ctr[blockIdx.x] + 1;
      A.ctr[blockIdx.x] = e;
      s_ep = e;
      s_ar_skip = *reinterpret_cast<volatile int*>(A.err) != 0;
    }
  }
  // The epilogue's global reads (residual, bias) do not depend on this
  // kernel's results: when every consumer thread owns at most one output of
  // the CTA, issue them now, beside the x loads, so the kernel ends in writes.
  const int n_out = (int)blockIdx.x < p.tiles ? ((p.tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1) * 16 * M : 0;
  const bool pre_epi = !DUAL && p.splits == 1 && !geo.atomic_out && n_out <= NC;
  float pre_bias = 0.f, pre_res = 0.f;
  if (pre_epi && tid < n_out) {
    const int rl = (tid % (16 * M)) / M, mm = tid % M;
    const int row = ((int)blockIdx.x + (tid / (16 * M)) * (int)gridDim.x) * 16 + rl;
    if (row < p.N) {
      if (p.bias) pre_bias = __half2float(__ushort_as_half(p.bias[row]));
      if (EPI == SC_EPI_RESIDUAL) pre_res = p.residual[(size_t)mm * p.ldr + row];
    }
  }
  stage_x_fx_warp<BITS, NGC, NORM, XT>(p, xsb, s_part, kc0, kc1, geo.cps, warp, lane);
  if (lane == 0) mbar_arrive(&s_xready);
  const int CB = fx_chunk_bytes(BITS, M);

  // B-fragment column of this lane and whether its words' group feeds it
  const int bm = g / (2 * NGC), bpart = (g / NGC) & 1, bgrp = g % NGC;
  const bool bact = bm < M && bgrp == ((t * NGC) >> 2);
  const int bx_off = (((bm * 2 + bpart) * XQ) * 4 + t) * 16;
  // C-fragment columns 2t, 2t+1 hold groups grpA and grpA + 1 (the same group when NGC == 1)
  const int grpA = (2 * t) % NGC;

  const int pr0 = tile_row(g);
  const int lgG = p.lg_group;
  const int w_r8 = geo.row_swz ? 1024 : 8 * geo.nblk * 128;
  const int s_r8 = 16 * geo.ngs;
  // Every consumer warp takes chunk `warp` of every stage (cps <= TC_NCW), so
  // all its shared-memory offsets are fixed for the kernel.
  int fo_w, fo_s;
  {
    const int c = warp;
    const int u = ((c & 1) << 2) | t;
    if (geo.row_swz) {
      fo_w = (c >> 1) * 2048 + pr0 * 128 + ((u ^ (pr0 & 7)) << 4);
    } else {
      const int l = pr0 * geo.nblk + (c >> 1);
      fo_w = l * 128 + ((u ^ (l & 7)) << 4);
    }
    const int gi = ((c * TR::KPC) >> lgG) + grpA;
    const int lo = pr0 * geo.ngs * 2 + gi * 2;
    fo_s = lo ^ (((lo >> 7) & geo.s_swz) << 4);
  }
  const int fo_x = warp * CB + bx_off;
  const int fo_t = warp * CB + M * 2 * XQ * 64 + t * 16;

  // Kernel-constant geometry in registers, and this lane's operand addresses
  // in stage 0 of the ring (stage s adds s * stage_bytes).
  const int nst = geo.nst, cps = geo.cps;
  const uint32_t stage_bytes = (uint32_t)geo.stage_bytes;
  const uint32_t wset = (uint32_t)geo.wset_bytes, sset = (uint32_t)geo.sset_bytes;
  const uint32_t ring_w = smem_u32(ring) + fo_w;                        // weight words, set 0
  const uint32_t ring_s = smem_u32(ring) + NACC * wset + fo_s;         // scale word, set 0
  // lanes whose B column is unused read zeros instead of branching
  const uint32_t zero_x = smem_u32(s_zero);

  // A stage's weight words and raw scale / bias words of this lane.  The
  // SwiGLU pair keeps only its words a stage ahead (96 registers): its scales
  // and biases are read from the held slot when they are used.
  constexpr bool PIPE_SB = NACC == 1;
  struct StageRegs {
    uint4 w0[NACC], w1[NACC];
    uint32_t sb[PIPE_SB ? NACC : 1][4];  // scale(row g), scale(row g+8), bias(row g), bias(row g+8)
  };
  auto ld_sb_raw = [&](uint32_t sp) -> uint32_t {
    if (NGC >= 2) return lds_u32(sp);  // groups grpA, grpA + 1
    return lds_u16(sp);
  };
  auto ld_sb4 = [&](uint32_t (&d)[4], uint32_t soff, int a) {  // soff: stage byte offset
    const uint32_t sp = ring_s + soff + (a * 2) * sset;
    d[0] = ld_sb_raw(sp);
    d[1] = ld_sb_raw(sp + s_r8);
    d[2] = ld_sb_raw(sp + sset);
    d[3] = ld_sb_raw(sp + sset + s_r8);
  };
  // A stage holds cps chunks (fewer than TC_NCW for a short K or a narrow
  // scale box): warps past them own no chunk and sit the stream out (their
  // offsets would leave the stage); the empty barriers count only the others.
  const bool has_chunk = warp < cps;
  auto ld_stage = [&](StageRegs& d, uint32_t soff) {
#pragma unroll
    for (int a = 0; a < NACC; ++a) {
      const uint32_t wp = ring_w + soff + a * wset;
      d.w0[a] = lds_v4(wp);
      d.w1[a] = lds_v4(wp + w_r8);
      if (PIPE_SB) ld_sb4(d.sb[PIPE_SB ? a : 0], soff, a);
    }
  };
  // (group grpA, group grpA + 1) of a raw scale / bias word
  auto sb_lo = [](uint32_t r) { return __low2float(u32_as_h2(r)); };
  auto sb_hi = [](uint32_t r) { return NGC >= 2 ? __high2float(u32_as_h2(r)) : __low2float(u32_as_h2(r)); };

  // This CTA's tiles (blockIdx.x, + gridDim.x, ...) and the stages of each.
  // Every stage of a tile is full: the chunk slots past the K slice hold zero
  // x (staged so), which zeroes whatever weights and scales sit there.
  const int my_tiles = (int)blockIdx.x < p.tiles ? (p.tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int kspan = kc1 - kc0;
  const int spt = (kspan + cps - 1) / cps;
  const int nq = has_chunk ? my_tiles * spt : 0;
  int s = 0;
  uint32_t ph = 0;
  bool aborted = false;
  StageRegs cur;
  if (nq > 0) {
    if (mbar_wait_warp(&full[0], 0, &s_abort, TC_WAIT_NS))
      ld_stage(cur, 0u);
    else
      aborted = true;
  }
  float acc[NACC][4];
#pragma unroll
  for (int a = 0; a < NACC; ++a)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[a][r] = 0.f;
  int kst = 0, tl = 0;  // stage within the tile, tile of this CTA
  const uint32_t xbase = smem_u32(xsb);
  // B-fragment and table addresses of this lane in stage 0 of a tile; a lane
  // whose B column is unused reads zeros
  const uint32_t xb0 = bact ? xbase + fo_x : zero_x;
  const uint32_t xstep = bact ? (uint32_t)(cps * CB) : 0u;
  uint32_t xb = xb0, xt = xbase + fo_t;
  const bool warp_slots = geo.warp_slots != 0;
  // One stage: MMAs on `cur`, the next stage's operands into `nxt`.  With one
  // weight set the loop runs two stages per trip with the register sets
  // swapped, so no copies.
  auto stage = [&](int q, StageRegs& cur, StageRegs& nxt) {
    const int s_cur = s;
    // With one weight set every ring read of this stage (words, scales,
    // biases) went into registers during the previous stage: free the slot now.
    if (PIPE_SB) mbar_arrive(&empty[s_cur]);
    // ---- MMAs of the current stage (registers loaded one stage ahead)
    float ca[NACC][4], cz[NACC][4];
    uint32_t bfr[NMMA][2];
#pragma unroll
    for (int qq = 0; qq < XQ; ++qq) {
      const uint4 v = lds_v4(xb + qq * 64);
      bfr[2 * qq][0] = v.x;
      bfr[2 * qq][1] = v.y;
      bfr[2 * qq + 1][0] = v.z;
      bfr[2 * qq + 1][1] = v.w;
    }
    const float4 tb = lds_f4(xt);
#pragma unroll
    for (int a = 0; a < NACC; ++a) {
      const uint32_t r0[4] = {cur.w0[a].x, cur.w0[a].y, cur.w0[a].z, cur.w0[a].w};
      const uint32_t r1[4] = {cur.w1[a].x, cur.w1[a].y, cur.w1[a].z, cur.w1[a].w};
      ca[a][0] = tb.x;
      ca[a][1] = tb.y;
      ca[a][2] = tb.x;
      ca[a][3] = tb.y;
#pragma unroll
      for (int r = 0; r < 4; ++r) cz[a][r] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t A0[4], A1[4];
        unpack_off<BITS>(r0[j], A0);
        unpack_off<BITS>(r1[j], A1);
        if (BITS == 4) {
          mma_16816(ca[a], A0[0], A1[0], A0[1], A1[1], bfr[2 * j][0], bfr[2 * j][1]);
          mma_16816(cz[a], A0[2], A1[2], A0[3], A1[3], bfr[2 * j + 1][0], bfr[2 * j + 1][1]);
        } else if (j & 1) {
          mma_16816(cz[a], A0[0], A1[0], A0[1], A1[1], bfr[j][0], bfr[j][1]);
        } else {
          mma_16816(ca[a], A0[0], A1[0], A0[1], A1[1], bfr[j][0], bfr[j][1]);
        }
      }
    }
    // ---- the next stage's registers load while those MMAs run
    if (++s == nst) {
      s = 0;
      ph ^= 1;
    }
    if (q + 1 < nq) {
      if (mbar_wait_warp(&full[s], ph, &s_abort, TC_WAIT_NS))
        ld_stage(nxt, (uint32_t)s * stage_bytes);
      else
        aborted = true;
    }
    // ---- scales / biases of the current stage
#pragma unroll
    for (int a = 0; a < NACC; ++a) {
      uint32_t sbv[4];
      if (PIPE_SB) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sbv[i] = cur.sb[PIPE_SB ? a : 0][i];
      } else {
        ld_sb4(sbv, (uint32_t)s_cur * stage_bytes, a);
      }
      acc[a][0] = fmaf(sb_lo(sbv[0]), ca[a][0] + cz[a][0], fmaf(sb_lo(sbv[2]), tb.z, acc[a][0]));
      acc[a][1] = fmaf(sb_hi(sbv[0]), ca[a][1] + cz[a][1], fmaf(sb_hi(sbv[2]), tb.w, acc[a][1]));
      acc[a][2] = fmaf(sb_lo(sbv[1]), ca[a][2] + cz[a][2], fmaf(sb_lo(sbv[3]), tb.z, acc[a][2]));
      acc[a][3] = fmaf(sb_hi(sbv[1]), ca[a][3] + cz[a][3], fmaf(sb_hi(sbv[3]), tb.w, acc[a][3]));
    }
    if (!PIPE_SB) mbar_arrive(&empty[s_cur]);  // the scale reads above were the slot's last
    // ---- tile done for this warp: reduce over k-lanes, add into the CTA's tile accumulators
    if (++kst == spt) {
      kst = 0;
      xb = xb0;
      xt = xbase + fo_t;
      const int m = t / NGC;
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        float vg = acc[a][0] + acc[a][1], vg8 = acc[a][2] + acc[a][3];
#pragma unroll
        for (int o = 1; o < NGC; o <<= 1) {
          vg += __shfl_xor_sync(0xffffffffu, vg, o);
          vg8 += __shfl_xor_sync(0xffffffffu, vg8, o);
        }
        if ((t % NGC) == 0 && m < M) {
          if (warp_slots) {
            float* sl = s_slot + (((tl * 16 + pr0) * M + m) * NACC + a) * TC_NCW + warp;
            sl[0] = vg;
            sl[8 * M * NACC * TC_NCW] = vg8;
          } else {
            atomicAdd(&s_acc[((tl * 16 + pr0) * M + m) * NACC + a], fx_to_fixed(vg));
            atomicAdd(&s_acc[((tl * 16 + pr0 + 8) * M + m) * NACC + a], fx_to_fixed(vg8));
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[a][r] = 0.f;
      }
      ++tl;
    } else {
      xb += xstep;
      xt += (uint32_t)(cps * CB);
    }
  };
  StageRegs alt;
  if constexpr (NACC == 1) {
    for (int q = 0; q < nq && !aborted; q += 2) {
      stage(q, cur, alt);
      if (q + 1 < nq && !aborted) stage(q + 1, alt, cur);
    }
  } else {  // the SwiGLU pair has no registers for a second set: one stage per trip
    for (int q = 0; q < nq && !aborted; ++q) {
      stage(q, cur, alt);
      cur = alt;
    }
  }
  if (aborted && lane == 0) atomicExch(&g_qgemv_error, 1);
  // ---- all warps' partial sums are in: the epilogue of every tile of this CTA
  named_bar_sync(1, NC);
  if (s_abort) return;  // a wait gave up: leave the output untouched
  const int total = my_tiles * 16 * M;
  for (int idx = tid; idx < total; idx += NC) {
    const int tli = idx / (16 * M), rem = idx - tli * 16 * M;
    const int rl = rem / M, mm = rem - rl * M;
    const int row = ((int)blockIdx.x + tli * (int)gridDim.x) * 16 + rl;
    float v[2];
    if (geo.warp_slots) {  // warp order: the same bits on every run
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        const float4* sl = reinterpret_cast<const float4*>(s_slot + (idx * NACC + a) * TC_NCW);
        float w16[TC_NCW];
#pragma unroll
        for (int i = 0; i < TC_NCW / 4; ++i) {
          const float4 f = sl[i];
          w16[4 * i] = f.x;
          w16[4 * i + 1] = f.y;
          w16[4 * i + 2] = f.z;
          w16[4 * i + 3] = f.w;
        }
        float sum = w16[0];
#pragma unroll
        for (int w = 1; w < TC_NCW; ++w) sum += w < cps ? w16[w] : 0.f;  // slots of warps without a chunk are unset
        v[a] = sum;
      }
    } else {
#pragma unroll
      for (int a = 0; a < NACC; ++a) v[a] = fx_from_fixed(s_acc[idx * NACC + a]);
    }
    if (NORM) {  // staged x was x * norm_weight: divide by the row's rms (warp partials in warp order)
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < TC_NCW; ++w) ss += s_part[w][mm];
      const float r = sqrtf(ss / (float)p.K + p.eps);
#pragma unroll
      for (int a = 0; a < NACC; ++a) v[a] = v[a] / r;
    }
    if (row >= p.N) continue;
    if constexpr (AR) {
      // this rank's partial (the value the unfused path writes before its
      // all-reduce) to every peer: half line e of region (set, this rank)
      const P2PArgs& A = *p.ar;
      const float part = (v[0] + pre_bias) + pre_res;
      const uint32_t ep = s_ep;
      const size_t e = (size_t)mm * p.N + row;
      for (int k = 1; k < A.world; ++k) {
        const int dst = (A.rank + k) % A.world;  // staggered: ranks do not all hit one peer first
        char* reg = A.data[dst] + (size_t)((ep & 1) * A.world + A.rank) * A.region_bytes;
        st_volatile_v2(reg + e * 8, __float_as_uint(part), ep);
      }
      // the sum over ranks in rank order from zero: the unfused all-reduce's order, so its bits
      bool skip = s_ar_skip != 0;
      uint64_t t0 = 0;
      float acc = 0.f;
      for (int q = 0; q < A.world; ++q) {
        if (q == A.rank) {
          acc += part;
        } else {
          const char* reg = A.data[A.rank] + (size_t)((ep & 1) * A.world + q) * A.region_bytes;
          acc += __uint_as_float(p2p_recv_half(A, reg + e * 8, ep, &skip, &t0));
        }
      }
      reinterpret_cast<float*>(p.y)[(size_t)mm * p.ldy + row] = acc;
      continue;
    }
    if (pre_epi)  // bias / residual already read; same sums, same order as epilogue()
      reinterpret_cast<YT*>(p.y)[(size_t)mm * p.ldy + row] = from_f32<YT>((v[0] + pre_bias) + pre_res);
    else
      epilogue<EPI, YT>(p, split, geo.atomic_out != 0, row, mm, v);
  }
  if (p.stamp) {  // the CTA's last output is written
    named_bar_sync(1, NC);
    if (tid == 0) atomicMax(p.stamp + 1, (unsigned long long)globaltimer_ns());
  }
}

template <int EPI, typename YT>
__global__ void qgemv_splitk_reduce(const QGemvParams p) {
  pdl_trigger();
  pdl_wait();
  // A GEMV CTA whose bounded wait gave up returned without writing its
  // partials: the workspace then holds stale values, so leave y untouched
  // (the error word stays set until sc_qgemv_device_error(1) clears it).
  if (*reinterpret_cast<volatile int*>(&g_qgemv_error)) return;
  const size_t total = (size_t)p.Mr * p.N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int col = (int)(e / p.N), row = (int)(e % p.N);
    float v[2] = {0.f, 0.f};
    const int nacc = (EPI == SC_EPI_SWIGLU) ? 2 : 1;
    for (int a = 0; a < nacc; ++a)
      for (int s = 0; s < p.splits; ++s) v[a] += p.partial[(((size_t)a * p.splits + s) * p.Mr + col) * p.N + row];
    float out;
    if (EPI == SC_EPI_SWIGLU) {
      out = silu_f32(v[0]) * v[1];
    } else {
      out = v[0];
      if (p.bias) out += __half2float(__ushort_as_half(p.bias[row]));
      if (EPI == SC_EPI_RESIDUAL) out += p.residual[(size_t)col * p.ldr + row];
    }
    reinterpret_cast<YT*>(p.y)[(size_t)col * p.ldy + row] = from_f32<YT>(out);
  }
  if (p.stamp) {
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(p.stamp + 1, (unsigned long long)globaltimer_ns());
  }
}

// ------------------------------------------------------------------ host side

struct SplitPlan {
  int splits;
  int chunks_per_split;
  int tiles;
};

static int kpc_of(int bits) { return bits == 4 ? 128 : 64; }
static int nmma_of(int bits) { return bits == 4 ? 8 : 4; }

static size_t xs_bytes(int bits, int M, int nkc) {
  const size_t rowlen = (size_t)M * nmma_of(bits) * 4 + 8;
  return (size_t)nkc * 4 * rowlen * 2;
}

static size_t smem_bytes(int bits, int M, int nkc, int nacc, int MT) {
  return xs_bytes(bits, M, nkc) + (size_t)QG_WARPS * 32 * nacc * MT * 4 * 4;
}

// Direct-load kernel plan (fallback path).
static SplitPlan plan_splits(int M, int K, int N, int bits, int nacc) {
  SplitPlan sp;
  const int KC = (K / (32 / bits) + 15) / 16;
  sp.tiles = (N + 15) / 16;
  const int MT = M > 8 ? 2 : 1;
  int splits = 1;
  while (splits < KC && smem_bytes(bits, M, (KC + splits - 1) / splits, nacc, MT) > (size_t)QG_XS_MAX) ++splits;
  const int want = 2 * sm_count();
  while (sp.tiles * splits < want && (KC + splits) / (splits + 1) >= QG_WARPS) ++splits;
  sp.chunks_per_split = (KC + splits - 1) / splits;
  sp.splits = (KC + sp.chunks_per_split - 1) / sp.chunks_per_split;
  return sp;
}

// ---- TMA pipeline plan
constexpr size_t TC_SMEM_BUDGET = 220 * 1024;
constexpr int TC_SLOT_BUDGET = 64 * 1024;  // factored kernel: per-warp output slots
constexpr size_t TC_XS_BUDGET = 64 * 1024;
constexpr int TC_STAGE_CHUNKS = 32;  // 16 rows x 32 chunks x 64 B = 32 KB of packed words per stage

struct TmaPlan {
  bool ok;
  SplitPlan sp;
  TmaGeo geo;
  size_t smem;
  int grid_x;
};

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Chunk granularity of stages and splits: whole 32-word blocks, and a scale
// box whose width (groups) is a multiple of 8 (16 bytes).
static int tma_unit(int bits, int group) { return std::max(2, 8 * group / kpc_of(bits)); }

// Tuning knobs read once from the environment (0 / unset = built-in choice):
// SC_QGEMV_CPS chunks per stage, SC_QGEMV_NST ring depth, SC_QGEMV_PATH=ldg
// forces the direct-load kernel, SC_QGEMV_FX=0 the batched kernel for decode,
// SC_QGEMM=0 keeps passes of more rows off the tensor-core GEMM,
// SC_QGEMV_WMODE=0/1 the packed-word tensor-map layout (block-major /
// row-swizzled; default: row-swizzled when the driver accepts it).
struct Knobs {
  int cps = 0, nst = 0, ldg = 0, nofx = 0, wmode = -1, pre = -1, pf_after = 1, nok2 = 0;
  Knobs() {
    if (const char* e = getenv("SC_QGEMM")) nok2 = e[0] == '0';
    if (const char* e = getenv("SC_PF_AFTER")) pf_after = atoi(e);
    if (const char* e = getenv("SC_QGEMV_PRE")) pre = atoi(e);
    if (const char* e = getenv("SC_QGEMV_WMODE")) wmode = atoi(e);
    if (const char* e = getenv("SC_QGEMV_FX")) nofx = e[0] == '0';
    if (const char* e = getenv("SC_QGEMV_CPS")) cps = atoi(e);
    if (const char* e = getenv("SC_QGEMV_NST")) nst = atoi(e);
    if (const char* e = getenv("SC_QGEMV_PATH")) ldg = strcmp(e, "ldg") == 0;
  }
};
static const Knobs& knobs() {
  static Knobs k;
  return k;
}

// Shared-memory budget for the staged x slice of the factored kernel (hi/lo
// parts and per-chunk sums: 576 B per 128 values at 4 bits, M = 1).
constexpr size_t TC_XS_BUDGET_FX = 80 * 1024;

static int ngc_of(int bits, int group) { return std::max(1, kpc_of(bits) / group); }

// The factored kernel serves passes whose B tile fits one n8 mma: M * NGC <= 4.
static bool fx_eligible(int M, int bits, int group) { return M * ngc_of(bits, group) <= 4; }

static size_t xs_fx_bytes(int bits, int M, int nkc) { return (size_t)nkc * fx_chunk_bytes(bits, M); }

static TmaPlan plan_tma(int M, int K, int N, int bits, int group, int nacc, int MT, bool fx) {
  TmaPlan tp{};
  tp.ok = false;
  const int KW = K / (32 / bits);
  const int KC = (KW + 15) / 16;
  const int KG = K / group;
  if (KW % 32 || KG % 8) return tp;  // boxes must tile a row exactly; 16-byte scale rows
  const int U = tma_unit(bits, group);
  const int nsm = sm_count();
  SplitPlan sp;
  sp.tiles = (N + 15) / 16;
  int splits = 1;
  auto cps_of = [&](int s) { return round_up((KC + s - 1) / s, U); };
  auto xsb = [&](int nkc) { return fx ? xs_fx_bytes(bits, M, nkc) : xs_bytes(bits, M, nkc); };
  const size_t xs_budget = fx ? TC_XS_BUDGET_FX : TC_XS_BUDGET;
  while (cps_of(splits) > U && xsb(cps_of(splits)) > xs_budget) ++splits;
  // more splits when there are too few tiles for the SMs (keep >= TC_NCW chunks per split)
  while (sp.tiles * splits < nsm && cps_of(splits + 1) >= TC_NCW) ++splits;
  sp.chunks_per_split = cps_of(splits);
  sp.splits = (KC + sp.chunks_per_split - 1) / sp.chunks_per_split;
  TmaGeo geo{};
  // batched kernel: 32 KB of packed words per stage, each consumer warp at
  // most two chunks of it; factored kernel: one chunk per consumer warp
  int cps = knobs().cps > 0 ? knobs().cps : fx ? TC_NCW : TC_STAGE_CHUNKS / nacc;
  cps = std::min(cps, fx ? TC_NCW : 2 * TC_NCW);
  while (cps > U && cps * kpc_of(bits) / group * 2 > 128) cps /= 2;  // scale-box row <= 128 B (swizzle span)
  cps = std::min(cps, sp.chunks_per_split);
  cps = std::max(U, cps / U * U);
  geo.cps = cps;
  geo.nblk = cps / 2;
  geo.ngs = cps * kpc_of(bits) / group;
  {
    const int rowb = geo.ngs * 2;
    geo.s_swz = rowb == 128 ? 7 : rowb == 64 ? 3 : rowb == 32 ? 1 : 0;
  }
  geo.wset_bytes = 16 * geo.nblk * 128;
  geo.sset_bytes = round_up(16 * geo.ngs * 2, 1024);
  geo.stage_bytes = nacc * (geo.wset_bytes + 2 * geo.sset_bytes);
  // the factored kernel stages x for whole stages (a tile's last one zero-padded)
  geo.ring_off = round_up((int)xsb(fx ? round_up(sp.chunks_per_split, cps) : sp.chunks_per_split), 1024);
  const int red_bytes = fx ? 0 : 2 * TC_NCW * 32 * nacc * MT * 4 * 4;  // double-buffered by tile
  tp.grid_x = std::max(1, std::min(sp.tiles, (nsm + sp.splits - 1) / sp.splits));
  // factored kernel: fp32 accumulators for every output of the CTA's tiles
  geo.acc_floats = fx ? ((sp.tiles + tp.grid_x - 1) / tp.grid_x) * 16 * M * nacc : 0;
  // fp32 slots per consumer warp when they fit (no atomics), else 64-bit fixed point
  geo.warp_slots = fx && geo.acc_floats * TC_NCW * 4 <= TC_SLOT_BUDGET;
  const int acc_bytes = round_up(geo.acc_floats * (geo.warp_slots ? TC_NCW * 4 : 8), 16);
  if (acc_bytes > TC_SLOT_BUDGET) return tp;
  const size_t fixed = geo.ring_off + red_bytes + acc_bytes + 2 * TC_MAX_NST * 8 + 1024 /* base alignment */ + 64;
  if (fixed >= TC_SMEM_BUDGET) return tp;
  int nst = (int)std::min<size_t>(TC_MAX_NST, (TC_SMEM_BUDGET - fixed) / geo.stage_bytes);
  if (knobs().nst > 0) nst = std::min(nst, knobs().nst);
  if (nst < 2) return tp;
  geo.nst = nst;
  geo.pre_stages = knobs().pre >= 0 ? std::min(knobs().pre, nst) : nst;
  geo.pf_after = knobs().pf_after;
  geo.red_off = geo.ring_off + nst * geo.stage_bytes;
  geo.acc_off = geo.red_off + red_bytes;
  geo.bar_off = round_up(geo.acc_off + acc_bytes, 16);
  geo.atomic_out = 0;
  geo.row_swz = 1;
  tp.smem = geo.bar_off + 2 * TC_MAX_NST * 8 + 1024;
  tp.sp = sp;
  tp.geo = geo;
  tp.ok = true;
  return tp;
}

// ---- tensor maps (driver entry point fetched through the runtime)
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// mode: 1 = (word, row, block) dims with row-dependent swizzle, 0 = (word, block, row)
static bool encode_wmap(CUtensorMap* m, const uint32_t* wq, int rows, int KW, int nblk, int mode) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3], es[3] = {1, 1, 1};
  if (mode) {
    dims[0] = 32; dims[1] = (cuuint64_t)rows; dims[2] = (cuuint64_t)(KW / 32);
    strides[0] = (cuuint64_t)KW * 4; strides[1] = 128;
    box[0] = 32; box[1] = 16; box[2] = (cuuint32_t)nblk;
  } else {
    dims[0] = 32; dims[1] = (cuuint64_t)(KW / 32); dims[2] = (cuuint64_t)rows;
    strides[0] = 128; strides[1] = (cuuint64_t)KW * 4;
    box[0] = 32; box[1] = (cuuint32_t)nblk; box[2] = 16;
  }
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t*>(wq), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_smap(CUtensorMap* m, const uint16_t* s, int rows, int KG, int ngs, int swz_mask) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)KG, (cuuint64_t)rows}, strides[1] = {(cuuint64_t)KG * 2};
  cuuint32_t box[2] = {(cuuint32_t)ngs, 16}, es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(s), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE,
            swz_mask == 7   ? CU_TENSOR_MAP_SWIZZLE_128B
            : swz_mask == 3 ? CU_TENSOR_MAP_SWIZZLE_64B
            : swz_mask == 1 ? CU_TENSOR_MAP_SWIZZLE_32B
                            : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encode every segment's maps; prefers the row-swizzled layout, falls back to
// the block-major one if the driver rejects non-monotonic strides.
static bool encode_maps(const QGemvParams& p, int bits, int nacc, TmaGeo* geo, TmaMaps* maps) {
  static int mode_ok = knobs().wmode;  // -1 unknown, 1 row-swizzled works, 0 use block-major
  const int KW = p.K / (32 / bits), KG = p.K / p.group;
  const int nmaps = nacc == 2 ? 2 : p.nseg;
  for (int pass = 0; pass < 2; ++pass) {
    const int mode = (mode_ok == 0 || pass == 1) ? 0 : 1;
    bool ok = true;
    for (int s = 0; s < nmaps && ok; ++s) {
      const QSeg& sg = p.seg[s];
      ok = encode_wmap(&maps->w[s], sg.wq, sg.rows, KW, geo->nblk, mode) &&
           encode_smap(&maps->s[s], sg.s, sg.rows, KG, geo->ngs, geo->s_swz) &&
           encode_smap(&maps->b[s], sg.b, sg.rows, KG, geo->ngs, geo->s_swz);
    }
    if (ok) {
      if (mode_ok < 0) mode_ok = mode;
      geo->row_swz = mode;
      return true;
    }
    if (mode == 0) return false;
    mode_ok = 0;
  }
  return false;
}

template <int BITS, int MT, int EPI, bool NORM, typename XT, typename YT>
static int launch_qgemv(QGemvParams& p, const TmaPlan* tp, const TmaMaps* maps, cudaStream_t stream) {
  const int nacc = (EPI == SC_EPI_SWIGLU) ? 2 : 1;
  if (tp) {
    auto kern = qgemv_tma_kernel<BITS, MT, EPI, NORM, XT, YT>;
    static bool configured = false;
    if (!configured) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM_BUDGET);
      configured = true;
    }
    dim3 grid(tp->grid_x, p.splits);
    ::sc::launch(kern, grid, TC_THREADS, tp->smem, stream, p, tp->geo, *maps);
    int st = check_launch("qgemv_tma");
    if (st != SC_OK || p.splits == 1 || tp->geo.atomic_out) return st;
  } else {
    auto kern = qgemv_kernel<BITS, MT, EPI, NORM, XT, YT>;
    const size_t smem = smem_bytes(BITS, p.M, p.chunks_per_split, nacc, MT);
    static bool configured = false;
    if (!configured) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      configured = true;
    }
    int nb = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, QG_THREADS, smem);
    const int slots = std::max(1, std::max(nb, 1) * sm_count() / p.splits);
    const int per_cta = (p.tiles + slots - 1) / slots;
    dim3 grid((p.tiles + per_cta - 1) / per_cta, p.splits);
    ::sc::launch(kern, grid, QG_THREADS, smem, stream, p);
    int st = check_launch("qgemv");
    if (st != SC_OK || p.splits == 1) return st;
  }
  const size_t total = (size_t)p.Mr * p.N;
  const int rb = (int)std::min<size_t>((total + 255) / 256, (size_t)4 * sm_count());
  ::sc::launch(qgemv_splitk_reduce<EPI, YT>, rb, 256, 0, stream, p);
  return check_launch("qgemv_splitk_reduce");
}

template <int BITS, int NGC, int EPI, bool NORM, typename XT, typename YT, bool AR>
static int launch_qgemv_fx_k(QGemvParams& p, const TmaPlan* tp, const TmaMaps* maps, cudaStream_t stream) {
  auto kern = qgemv_fx_kernel<BITS, NGC, EPI, NORM, XT, YT, AR>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM_BUDGET);
    configured = true;
  }
  dim3 grid(tp->grid_x, p.splits);
  ::sc::launch(kern, grid, TC_THREADS, tp->smem, stream, p, tp->geo, *maps);
  int st = check_launch("qgemv_fx");
  if (st != SC_OK || p.splits == 1 || tp->geo.atomic_out) return st;
  const size_t total = (size_t)p.Mr * p.N;
  const int rb = (int)std::min<size_t>((total + 255) / 256, (size_t)4 * sm_count());
  ::sc::launch(qgemv_splitk_reduce<EPI, YT>, rb, 256, 0, stream, p);
  return check_launch("qgemv_splitk_reduce");
}

template <int BITS, int NGC, int EPI, bool NORM, typename XT, typename YT>
static int launch_qgemv_fx(QGemvParams& p, const TmaPlan* tp, const TmaMaps* maps, cudaStream_t stream) {
  // the all-reduce epilogue exists for the shapes the host admits to it:
  // one weight set, no RMSNorm prologue, fp32 output
  if constexpr (EPI != SC_EPI_SWIGLU && !NORM && std::is_same<YT, float>::value) {
    if (p.ar) return launch_qgemv_fx_k<BITS, NGC, EPI, NORM, XT, YT, true>(p, tp, maps, stream);
  }
  if (p.ar) {
    set_error("qlinear_allreduce: no all-reduce epilogue for this kernel instance");
    return SC_ERR_UNSUPPORTED;
  }
  return launch_qgemv_fx_k<BITS, NGC, EPI, NORM, XT, YT, false>(p, tp, maps, stream);
}

template <int BITS, int NGC, int EPI, bool NORM>
static int dispatch_fx_types(QGemvParams& p, const TmaPlan* tp, const TmaMaps* mp, int x_dtype, int y_dtype,
                             cudaStream_t stream) {
  if (x_dtype == SC_F16 && y_dtype == SC_F16) return launch_qgemv_fx<BITS, NGC, EPI, NORM, __half, __half>(p, tp, mp, stream);
  if (x_dtype == SC_F16 && y_dtype == SC_F32) return launch_qgemv_fx<BITS, NGC, EPI, NORM, __half, float>(p, tp, mp, stream);
  if (x_dtype == SC_F32 && y_dtype == SC_F16) return launch_qgemv_fx<BITS, NGC, EPI, NORM, float, __half>(p, tp, mp, stream);
  if (x_dtype == SC_F32 && y_dtype == SC_F32) return launch_qgemv_fx<BITS, NGC, EPI, NORM, float, float>(p, tp, mp, stream);
  set_error("qlinear: unsupported dtype pair x=%d y=%d", x_dtype, y_dtype);
  return SC_ERR_ARG;
}

template <int BITS, int NGC>
static int dispatch_fx(QGemvParams& p, const TmaPlan* tp, const TmaMaps* mp, int epi, int x_dtype, int y_dtype,
                       cudaStream_t stream) {
  const bool n = p.norm_w != nullptr;
  switch (epi) {
    case SC_EPI_STORE:
      return n ? dispatch_fx_types<BITS, NGC, SC_EPI_STORE, true>(p, tp, mp, x_dtype, y_dtype, stream)
               : dispatch_fx_types<BITS, NGC, SC_EPI_STORE, false>(p, tp, mp, x_dtype, y_dtype, stream);
    case SC_EPI_RESIDUAL:
      return n ? dispatch_fx_types<BITS, NGC, SC_EPI_RESIDUAL, true>(p, tp, mp, x_dtype, y_dtype, stream)
               : dispatch_fx_types<BITS, NGC, SC_EPI_RESIDUAL, false>(p, tp, mp, x_dtype, y_dtype, stream);
    case SC_EPI_SWIGLU:
      return n ? dispatch_fx_types<BITS, NGC, SC_EPI_SWIGLU, true>(p, tp, mp, x_dtype, y_dtype, stream)
               : dispatch_fx_types<BITS, NGC, SC_EPI_SWIGLU, false>(p, tp, mp, x_dtype, y_dtype, stream);
  }
  set_error("qlinear: unknown epilogue %d", epi);
  return SC_ERR_ARG;
}

template <int BITS, int MT, int EPI, bool NORM>
static int dispatch_types(QGemvParams& p, const TmaPlan* tp, const TmaMaps* mp, int x_dtype, int y_dtype,
                          cudaStream_t stream) {
  if (x_dtype == SC_F16 && y_dtype == SC_F16) return launch_qgemv<BITS, MT, EPI, NORM, __half, __half>(p, tp, mp, stream);
  if (x_dtype == SC_F16 && y_dtype == SC_F32) return launch_qgemv<BITS, MT, EPI, NORM, __half, float>(p, tp, mp, stream);
  if (x_dtype == SC_F32 && y_dtype == SC_F16) return launch_qgemv<BITS, MT, EPI, NORM, float, __half>(p, tp, mp, stream);
  if (x_dtype == SC_F32 && y_dtype == SC_F32) return launch_qgemv<BITS, MT, EPI, NORM, float, float>(p, tp, mp, stream);
  set_error("qlinear: unsupported dtype pair x=%d y=%d", x_dtype, y_dtype);
  return SC_ERR_ARG;
}

template <int BITS, int MT, int EPI>
static int dispatch_norm(QGemvParams& p, const TmaPlan* tp, const TmaMaps* mp, int x_dtype, int y_dtype,
                         cudaStream_t stream) {
  if (p.norm_w) return dispatch_types<BITS, MT, EPI, true>(p, tp, mp, x_dtype, y_dtype, stream);
  return dispatch_types<BITS, MT, EPI, false>(p, tp, mp, x_dtype, y_dtype, stream);
}

template <int BITS, int MT>
static int dispatch_epi(QGemvParams& p, const TmaPlan* tp, const TmaMaps* mp, int epi, int x_dtype, int y_dtype,
                        cudaStream_t stream) {
  switch (epi) {
    case SC_EPI_STORE: return dispatch_norm<BITS, MT, SC_EPI_STORE>(p, tp, mp, x_dtype, y_dtype, stream);
    case SC_EPI_RESIDUAL: return dispatch_norm<BITS, MT, SC_EPI_RESIDUAL>(p, tp, mp, x_dtype, y_dtype, stream);
    case SC_EPI_SWIGLU: return dispatch_norm<BITS, MT, SC_EPI_SWIGLU>(p, tp, mp, x_dtype, y_dtype, stream);
  }
  set_error("qlinear: unknown epilogue %d", epi);
  return SC_ERR_ARG;
}

// Which kernel a pass uses, and its split plan.  Shared by the launcher and
// the workspace-size query so both always agree.
struct PassPlan {
  bool tma;
  bool fx;  // factored kernel (exact weights); implies tma
  TmaPlan tp;
  SplitPlan sp;
};

static bool aligned(const void* ptr, size_t a) { return ((uintptr_t)ptr % a) == 0; }

static PassPlan plan_pass(int mb, int K, int N, int bits, int group, int nacc, bool tma_ok, bool atomic_ok,
                          bool allow_fx = true) {
  PassPlan pp{};
  const int MT = mb > 8 ? 2 : 1;
  if (tma_ok && !knobs().ldg) {
    pp.fx = allow_fx && fx_eligible(mb, bits, group) && !knobs().nofx;
    pp.tp = plan_tma(mb, K, N, bits, group, nacc, MT, pp.fx);
    if (!pp.tp.ok && pp.fx) {
      pp.fx = false;
      pp.tp = plan_tma(mb, K, N, bits, group, nacc, MT, false);
    }
    if (pp.tp.ok) {
      pp.tma = true;
      pp.sp = pp.tp.sp;
      if (atomic_ok && pp.sp.splits > 1) pp.tp.geo.atomic_out = 1;
      return pp;
    }
  }
  pp.tma = false;
  pp.fx = false;
  pp.sp = plan_splits(mb, K, N, bits, nacc);
  return pp;
}

// mb: rows of x in the pass (partials are kept per row of x, after the hi /
// lo columns of a batched pass were added)
static size_t pass_workspace(const PassPlan& pp, int mb, int N, int nacc) {
  if (pp.sp.splits <= 1 || (pp.tma && pp.tp.geo.atomic_out)) return 0;
  return (size_t)nacc * pp.sp.splits * mb * N * sizeof(float);
}

// One pass over the weights: up to 16 rows of x through the factored decode
// kernel when it is eligible; otherwise up to 8 rows through the batched
// kernel, whose B tile then carries each row twice -- fp16(x) and the fp16
// remainder x - fp16(x) -- so activations keep ~22 bits there too.
struct RowPass {
  int mb;     // rows of x
  bool hilo;  // batched pass with hi / lo rows
  PassPlan pp;
};

static RowPass plan_rows(int rem, int K, int N, int bits, int group, int nacc, bool tma_ok, bool atomic_ok) {
  RowPass r;
  // the factored decode kernel in passes of as many rows as it serves: on
  // B200 a pass of it streams the weights faster than one batched pass over
  // up to 8 rows does (measured: 14336 x 4096, 4-bit g64, 11.5 us per 2-row
  // pass; 23 us for 4 rows and 138 us for 16 rows through the batched kernel)
  const int mfx = 4 / ngc_of(bits, group);
  r.mb = mfx >= 1 && !knobs().nofx ? std::min(mfx, rem) : std::min(16, rem);
  r.pp = plan_pass(r.mb, K, N, bits, group, nacc, tma_ok, atomic_ok);
  r.hilo = false;
  if (!r.pp.fx) {
    r.mb = std::min(8, rem);
    r.hilo = true;
    r.pp = plan_pass(2 * r.mb, K, N, bits, group, nacc, tma_ok, atomic_ok, false);
  }
  return r;
}

static int run_qlinear(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_w, float eps,
                       int nseg, const uint32_t* const* wq, const uint16_t* const* scales,
                       const uint16_t* const* biases, const int* seg_rows, int group, int bits,
                       const uint16_t* bias, int epi, void* y, int y_dtype, int ldy, const float* residual,
                       int ldr, void* ws, size_t ws_bytes, const PrefetchList* pf, cudaStream_t stream,
                       const P2PArgs* ar = nullptr, size_t ar_max_bytes = 0, const P2PArgs* ar_dev = nullptr) {
  SC_REQUIRE(x && y && wq && scales && biases && seg_rows, SC_ERR_ARG, "qlinear: null pointer argument");
  SC_REQUIRE(bits == 4 || bits == 8, SC_ERR_SHAPE, "qlinear: bits must be 4 or 8 (got %d)", bits);
  SC_REQUIRE(group == 32 || group == 64 || group == 128, SC_ERR_SHAPE,
             "qlinear: group_size must be 32, 64 or 128 (got %d)", group);
  SC_REQUIRE(M >= 1 && K >= 1, SC_ERR_SHAPE, "qlinear: M=%d K=%d must be positive", M, K);
  SC_REQUIRE(K % group == 0, SC_ERR_SHAPE, "qlinear: K=%d not a multiple of group_size=%d", K, group);
  SC_REQUIRE(ldx >= K && ldy >= 1, SC_ERR_SHAPE, "qlinear: bad leading dimensions");
  SC_REQUIRE(nseg >= 1 && nseg <= QG_MAX_SEG, SC_ERR_SHAPE, "qlinear: 1..3 weight segments (got %d)", nseg);
  SC_REQUIRE(epi != SC_EPI_RESIDUAL || residual, SC_ERR_ARG, "qlinear: residual epilogue needs residual");
  SC_REQUIRE(epi != SC_EPI_SWIGLU || (nseg == 2 && seg_rows[0] == seg_rows[1]), SC_ERR_SHAPE,
             "qlinear: SwiGLU needs two segments of equal rows");
  SC_REQUIRE(x_dtype == SC_F16 || x_dtype == SC_F32, SC_ERR_ARG, "qlinear: x dtype");
  SC_REQUIRE(y_dtype == SC_F16 || y_dtype == SC_F32, SC_ERR_ARG, "qlinear: y dtype");
  SC_REQUIRE(epi != SC_EPI_SWIGLU || !bias, SC_ERR_UNSUPPORTED, "qlinear: bias with SwiGLU epilogue");

  QGemvParams p{};
  p.stamp = t_next_stamp;
  p.K = K;
  p.ldx = ldx;
  p.norm_w = norm_w;
  p.eps = eps;
  p.nseg = nseg;
  int N = 0;
  bool tma_ok = true;
  for (int s = 0; s < nseg; ++s) {
    SC_REQUIRE(wq[s] && scales[s] && biases[s], SC_ERR_ARG, "qlinear: null weight segment %d", s);
    SC_REQUIRE(seg_rows[s] >= 0, SC_ERR_SHAPE, "qlinear: negative rows");
    p.seg[s] = QSeg{wq[s], scales[s], biases[s], seg_rows[s]};
    N += seg_rows[s];
    // tensor maps need 16-byte bases; a 16-row tile must not straddle two segments
    tma_ok = tma_ok && aligned(wq[s], 16) && aligned(scales[s], 16) && aligned(biases[s], 16) &&
             seg_rows[s] > 0 && (s + 1 == nseg || seg_rows[s] % 16 == 0 || epi == SC_EPI_SWIGLU);
  }
  if (epi == SC_EPI_SWIGLU) N = seg_rows[0];
  SC_REQUIRE(ldy >= N, SC_ERR_SHAPE, "qlinear: ldy=%d < N=%d", ldy, N);
  SC_REQUIRE(epi != SC_EPI_RESIDUAL || ldr >= N, SC_ERR_SHAPE, "qlinear: ldr=%d < N=%d", ldr, N);
  if (N == 0) return SC_OK;
  p.N = N;
  p.group = group;
  p.lg_group = group == 32 ? 5 : group == 64 ? 6 : 7;
  p.bias = bias;
  p.ldy = ldy;
  p.ldr = ldr;
  const int nacc = epi == SC_EPI_SWIGLU ? 2 : 1;
  const size_t xsz = x_dtype == SC_F16 ? 2 : 4;
  const size_t ysz = y_dtype == SC_F16 ? 2 : 4;
  const bool atomic_ok = epi == SC_EPI_RESIDUAL && y_dtype == SC_F32 && (const void*)residual == (const void*)y &&
                         ldr == ldy;

  if (ar) {
    // the all-reduce runs in the epilogue of ONE decode-GEMV pass: the plan
    // (a function of the shape only, so every rank decides alike) must be the
    // factored kernel without split-K, one output per consumer thread
    const RowPass rp = plan_rows(M, K, N, bits, group, nacc, tma_ok, atomic_ok);
    const int max_tiles = rp.pp.tma ? (rp.pp.sp.tiles + rp.pp.tp.grid_x - 1) / rp.pp.tp.grid_x : 0;
    const bool fits = nseg == 1 && epi != SC_EPI_SWIGLU && !norm_w && y_dtype == SC_F32 && ldy == N &&
                      rp.mb == M && !rp.hilo && rp.pp.tma && rp.pp.fx && rp.pp.sp.splits == 1 &&
                      max_tiles * 16 * M <= TC_NCW * 32 && rp.pp.tp.grid_x <= P2P_MAX_CTR &&
                      (size_t)M * N * 4 <= ar_max_bytes;
    SC_REQUIRE(fits, SC_ERR_UNSUPPORTED,
               "qlinear_allreduce: M=%d K=%d N=%d does not run as one unsplit decode-GEMV pass with an fp32 "
               "output of at most %zu bytes (run sc_qlinear_fused + sc_p2p_allreduce)", M, K, N, ar_max_bytes);
    p.ar = ar_dev;
  }

  // More than 16 rows: the tensor-core GEMM (exact weights, x to ~22 bits)
  // when the shape and the workspace allow it; up to 16, decode-GEMV passes.
  if (!ar && M > 16 && !knobs().nok2 && tma_ok &&
      qgemm_eligible(M, K, nseg, seg_rows, epi, bits, group) && ws &&
      ws_bytes >= qgemm_workspace_bytes(M, K, N, epi))
    return run_qgemm(x, x_dtype, M, K, ldx, norm_w, eps, nseg, wq, scales, biases, seg_rows, group, bits, bias, epi,
                     y, y_dtype, ldy, residual, ldr, ws, ws_bytes, stream);
  for (int m0 = 0; m0 < M;) {
    const RowPass rp = plan_rows(M - m0, K, N, bits, group, nacc, tma_ok, atomic_ok);
    const int mb = rp.mb;
    PassPlan pp = rp.pp;
    p.Mr = mb;
    p.hilo = rp.hilo ? 1 : 0;
    p.M = rp.hilo ? 2 * mb : mb;
    p.x = static_cast<const char*>(x) + (size_t)m0 * ldx * xsz;
    p.y = static_cast<char*>(y) + (size_t)m0 * ldy * ysz;
    p.residual = residual ? residual + (size_t)m0 * ldr : nullptr;
    p.pf = (pf && m0 + mb == M) ? *pf : PrefetchList{};  // the last pass carries the prefetch
    p.x_vec = aligned(p.x, 16) && ((size_t)ldx * xsz) % 16 == 0 && (!norm_w || aligned(norm_w, 16));
    TmaMaps maps;
    const TmaPlan* tp = nullptr;
    if (pp.tma && encode_maps(p, bits, nacc, &pp.tp.geo, &maps)) {
      tp = &pp.tp;
    } else if (ar) {
      // every rank must take the same path: refuse rather than fall back alone
      set_error("qlinear_allreduce: tensor maps refused by the driver");
      return SC_ERR_UNSUPPORTED;
    } else if (pp.tma) {
      // tensor maps unavailable: plan this pass for the direct-load kernel
      // (hi / lo rows when they fit its 16-row B tile)
      if (!p.hilo && 2 * mb <= 16) {
        p.hilo = 1;
        p.M = 2 * mb;
      }
      pp = plan_pass(p.M, K, N, bits, group, nacc, false, false, false);
    }
    p.splits = pp.sp.splits;
    p.chunks_per_split = pp.sp.chunks_per_split;
    p.tiles = pp.sp.tiles;
    const size_t need = pass_workspace(pp, mb, N, nacc);
    if (need) {
      SC_REQUIRE(ws && ws_bytes >= need, SC_ERR_WORKSPACE, "qlinear: workspace of %zu bytes needed (got %zu)", need,
                 ws_bytes);
      p.partial = static_cast<float*>(ws);
    } else {
      p.partial = nullptr;
    }
    int st;
    if (tp && pp.fx) {
      const int ngc = ngc_of(bits, group);
      if (bits == 4)
        st = ngc == 1 ? dispatch_fx<4, 1>(p, tp, &maps, epi, x_dtype, y_dtype, stream)
             : ngc == 2 ? dispatch_fx<4, 2>(p, tp, &maps, epi, x_dtype, y_dtype, stream)
                        : dispatch_fx<4, 4>(p, tp, &maps, epi, x_dtype, y_dtype, stream);
      else
        st = ngc == 1 ? dispatch_fx<8, 1>(p, tp, &maps, epi, x_dtype, y_dtype, stream)
                      : dispatch_fx<8, 2>(p, tp, &maps, epi, x_dtype, y_dtype, stream);
    } else if (bits == 4)
      st = p.M > 8 ? dispatch_epi<4, 2>(p, tp, &maps, epi, x_dtype, y_dtype, stream)
                   : dispatch_epi<4, 1>(p, tp, &maps, epi, x_dtype, y_dtype, stream);
    else
      st = p.M > 8 ? dispatch_epi<8, 2>(p, tp, &maps, epi, x_dtype, y_dtype, stream)
                   : dispatch_epi<8, 1>(p, tp, &maps, epi, x_dtype, y_dtype, stream);
    if (st != SC_OK) return st;
    m0 += mb;
  }
  return SC_OK;
}

// Scratch the plain (one weight set, store epilogue) quantized linear needs
// for this exact shape and group: the widest pass over its M split, for the
// tensor-map plan when the weight pointers allow one and for the direct-load
// plan it falls back to when the driver refuses the tensor maps.
size_t qlinear_workspace_need(int M, int K, int N, int group, int bits, bool tma_ok) {
  // shapes sc_qlinear rejects need nothing: it refuses them before any launch
  if (M < 1 || K < 1 || N < 1 || (bits != 4 && bits != 8)) return 0;
  if ((group != 32 && group != 64 && group != 128) || K % group) return 0;
  size_t best = 0;
  for (int m0 = 0; m0 < M;) {
    int step = 16;
    for (int tma = 0; tma < (tma_ok ? 2 : 1); ++tma) {
      const RowPass rp = plan_rows(M - m0, K, N, bits, group, 1, tma != 0, false);
      best = std::max(best, pass_workspace(rp.pp, rp.mb, N, 1));
      // the direct-load plan a pass falls back to when the tensor maps are refused
      const int mv = (rp.hilo || 2 * rp.mb <= 16) ? 2 * rp.mb : rp.mb;
      best = std::max(best, pass_workspace(plan_pass(mv, K, N, bits, group, 1, false, false, false), rp.mb, N, 1));
      step = std::min(step, rp.mb);
    }
    m0 += step;
  }
  return best;
}

}  // namespace sc

extern "C" {

size_t sc_qlinear_workspace_bytes(int M, int K, int N, int bits) {
  if (M < 1 || K < 1 || N < 1 || (bits != 4 && bits != 8)) return 0;
  const int mb = M < 16 ? M : 16;
  size_t best = 0;
  // the tensor-core GEMM (more than 16 rows), SwiGLU worst case
  if (M > 16) best = sc::qgemm_workspace_bytes(M, K, N, SC_EPI_SWIGLU);
  // the widest plan over every pass size, kernel choice and group size
  for (int mm = 1; mm <= mb; ++mm)
    for (int group : {32, 64, 128})
      for (int tma = 0; tma < 2; ++tma) {
        if (K % group) continue;
        const sc::RowPass rp = sc::plan_rows(mm, K, N, bits, group, 2, tma != 0, false);
        best = std::max(best, sc::pass_workspace(rp.pp, rp.mb, N, 2));
        const int mv = 2 * rp.mb <= 16 ? 2 * rp.mb : rp.mb;
        best = std::max(best, sc::pass_workspace(sc::plan_pass(mv, K, N, bits, group, 2, false, false, false), rp.mb,
                                                 N, 2));
      }
  return best;
}

int sc_qgemv_probe_stamps(unsigned long long* pair) {
  sc::t_next_stamp = pair;
  return SC_OK;
}

int sc_qgemv_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sc::g_qgemv_error, sizeof(int));
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(sc::g_qgemv_error, &z, sizeof(int));
  }
  return v;
}

int sc_qlinear(const void* x, int x_dtype, int M, int K, int ldx, const uint32_t* wq, const uint16_t* scales,
               const uint16_t* biases, int N, int group_size, int bits, const uint16_t* bias, void* y,
               int y_dtype, int ldy, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const uint32_t* w[1] = {wq};
  const uint16_t* s[1] = {scales};
  const uint16_t* b[1] = {biases};
  int rows[1] = {N};
  return sc::run_qlinear(x, x_dtype, M, K, ldx, nullptr, 0.f, 1, w, s, b, rows, group_size, bits, bias,
                         SC_EPI_STORE, y, y_dtype, ldy, nullptr, 0, workspace, workspace_bytes, nullptr, stream);
}

int sc_qlinear_fused(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_weight,
                     float norm_eps, int nseg, const uint32_t* const* wq, const uint16_t* const* scales,
                     const uint16_t* const* biases, const int* seg_rows, int group_size, int bits,
                     const uint16_t* bias, int epilogue, void* y, int y_dtype, int ldy, const float* residual,
                     int ldr, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return sc::run_qlinear(x, x_dtype, M, K, ldx, norm_weight, norm_eps, nseg, wq, scales, biases, seg_rows,
                         group_size, bits, bias, epilogue, y, y_dtype, ldy, residual, ldr, workspace,
                         workspace_bytes, nullptr, stream);
}

int sc_qlinear_allreduce(const void* x, int x_dtype, int M, int K, int ldx, const uint32_t* wq,
                         const uint16_t* scales, const uint16_t* biases, int N, int group_size, int bits,
                         const uint16_t* bias, float* y, const float* residual, void* p2p, cudaStream_t stream) {
  sc::P2PArgs a;
  size_t max_bytes = 0;
  const sc::P2PArgs* a_dev = nullptr;
  if (int st = sc::p2p_args_of(p2p, &a, &max_bytes, &a_dev)) return st;
  SC_REQUIRE(a.world >= 2, SC_ERR_ARG, "qlinear_allreduce: transport of %d ranks", a.world);
  const uint32_t* W[1] = {wq};
  const uint16_t* S[1] = {scales};
  const uint16_t* B[1] = {biases};
  const int R[1] = {N};
  return sc::run_qlinear(x, x_dtype, M, K, ldx, nullptr, 0.f, 1, W, S, B, R, group_size, bits, bias,
                         residual ? SC_EPI_RESIDUAL : SC_EPI_STORE, y, SC_F32, N, residual, N, nullptr, 0, nullptr,
                         stream, &a, max_bytes, a_dev);
}

int sc_qlinear_fused_prefetch(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_weight,
                              float norm_eps, int nseg, const uint32_t* const* wq, const uint16_t* const* scales,
                              const uint16_t* const* biases, const int* seg_rows, int group_size, int bits,
                              const uint16_t* bias, int epilogue, void* y, int y_dtype, int ldy,
                              const float* residual, int ldr, void* workspace, size_t workspace_bytes,
                              const void* const* pf_ptrs, const size_t* pf_bytes, int pf_n, size_t pf_max_bytes,
                              cudaStream_t stream) {
  sc::PrefetchList pf;
  if (int st = sc::make_prefetch_list(pf_ptrs, pf_bytes, pf_n, pf_max_bytes, &pf)) return st;
  return sc::run_qlinear(x, x_dtype, M, K, ldx, norm_weight, norm_eps, nseg, wq, scales, biases, seg_rows,
                         group_size, bits, bias, epilogue, y, y_dtype, ldy, residual, ldr, workspace,
                         workspace_bytes, pf.count ? &pf : nullptr, stream);
}

}  // extern "C"
