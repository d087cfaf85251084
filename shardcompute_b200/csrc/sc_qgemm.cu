// K2: group-wise affine 4/8-bit dequant-GEMM on the 5th-generation tensor
// cores (tcgen05 + TMEM), for prefill and batched decode (more rows of x than
// the decode GEMV serves).  Same contract as the quantized linear
// (parallel/quantized_linear.py:168-176, 206-214: mx.quantized_matmul with
// transpose=True), y[M, N] = x[M, K] . (s*q + b)^T, fused epilogues.
//
// Precision.  The reference dequantizes in the activations' precision (fp32
// after the first residual), so the weights must stay exact to ~2^-22: a
// weight w = s*q + b (fp32) is carried as two fp16 parts w_hi = fp16(w),
// w_lo = fp16(w - w_hi), and so is x.  Each 16-deep k step issues three
// kind::f16 MMAs into one fp32 TMEM accumulator: w_hi.x_hi + w_hi.x_lo +
// w_lo.x_hi (w_lo.x_lo is below 2^-22 and dropped).
//
// Tile: 128 weight rows (the MMA's M) x up to 2 x 128 tokens (two MMA N
// tiles, two TMEM accumulators, one dequantized weight tile for both), k
// blocks of 64 (one group at group size 64).  Roles, one CTA per SM, persistent over
// tiles (token tiles fastest, so CTAs working on the same weight rows run
// together and share them in L2):
//   warp 0     TMA producer: the x_hi / x_lo tiles of each k block (2-D maps,
//              128-byte swizzle = the UMMA K-major SW128 layout)
//   warp 1     MMA issuer (one lane) and TMEM owner (alloc / dealloc)
//   warps 2-9  dequant: two threads per weight row r of the tile (r = their
//              TMEM lane: warp w reaches lanes 32*(w%4) .. +31), each taking
//              half of every 64-k block; per k block a thread converts its
//              16 (4-bit) or 32 (8-bit) bytes of codes with their scale /
//              bias (loaded a few k blocks ahead) into w_hi and w_lo in the
//              SW128 layout, fences the async proxy and arrives; after a
//              tile's last k block the same warps are the epilogue
//              (tcgen05.ld of their 32 TMEM lanes, alternate 32-token
//              blocks, then y = acc (+ bias) or residual + acc).
// SwiGLU runs as one GEMM over the stacked [gate; up] rows into a scratch
// [M, 2F], then y = silu(gate) * up row by row.
// Every wait is bounded by %globaltimer; a timeout raises an error word
// (sc_qgemm_device_error), every role stops, copies in flight are drained and
// the TMEM columns are freed before the CTA exits.
#include <string.h>

#include <algorithm>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sc_common.cuh"

namespace sc {

constexpr int QM_TM = 128;                 // weight rows per tile (MMA M)
constexpr int QM_TN = 128;                 // token rows per tile (MMA N, at most)
constexpr int QM_KB = 64;                  // k per block
constexpr int QM_TILE_BYTES = QM_TM * QM_KB * 2;  // one 128 x 64 fp16 operand tile: 16 KB
constexpr int QM_TT = 2;                   // token tiles per work item (one dequantized weight tile feeds both)
constexpr int QM_NST = 2;                  // pipeline stages
// stage: x_hi, x_lo of each token tile, then w_hi, w_lo
constexpr int QM_STAGE_BYTES = (2 * QM_TT + 2) * QM_TILE_BYTES;
constexpr int QM_W_OFF = 2 * QM_TT * QM_TILE_BYTES;
constexpr int QM_THREADS = 10 * 32;       // TMA, MMA, 8 dequant / epilogue warps
constexpr uint64_t QM_WAIT_NS = 2000000000ull;

__device__ int g_qgemm_error = 0;

struct QgemmParams {
  const uint32_t* wq[3];     // weight tensors stacked along N (or gate, up for SwiGLU)
  const uint16_t* sc[3];
  const uint16_t* bi[3];
  int seg_rows[3];
  int nseg;
  int M, K, N;               // N: output columns (sum of the segments' rows)
  int group, lg_group, bits;
  const uint16_t* bias;      // fp16 [N] or null
  int epi;                   // SC_EPI_STORE / SC_EPI_RESIDUAL
  void* y;
  int y_f16;
  int ldy;
  const float* residual;
  int ldr;
  int row_tiles, tok_tiles, tok_groups, kblocks;  // tok_groups: token groups per weight tile
  int ksplit;                // 1, or 2: each work item takes half of the k blocks and adds its result atomically
};

struct QgemmMaps {
  CUtensorMap xhi, xlo;
};

__device__ __forceinline__ uint32_t tmem_alloc_cols(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  return 0;
}
__device__ __forceinline__ void tmem_dealloc_cols(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// UMMA shared-memory descriptor of a K-major operand tile in the 128-byte
// swizzle layout (rows of 64 fp16 = 128 bytes, 8-row atoms of 1 KB): start
// address, leading offset 16 bytes (unused for this layout), stride offset
// 1 KB between 8-row groups, descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: D fp32, A and B fp16, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t umma_idesc_f16(int n) {
  uint32_t d = 0;
  d |= 1u << 4;                      // D format F32
  d |= 0u << 7;                      // A F16
  d |= 0u << 10;                     // B F16
  d |= (uint32_t)(n >> 3) << 17;     // N >> 3
  d |= (uint32_t)(QM_TM >> 4) << 24; // M >> 4
  return d;
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// bounded mbarrier wait of one thread; on giving up raises the CTA abort flag
// and the global error word
__device__ __forceinline__ bool qm_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 31) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > QM_WAIT_NS) {
        *abort = 1;
        atomicExch(&g_qgemm_error, 1);
        return false;
      }
    }
  }
}

// Byte offset of 16-byte chunk c of row r in a SW128 K-major tile.
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// KS: 1, or 2 (each work item takes half of the k blocks; the split is a
// template parameter so the unsplit kernel keeps its constant-folded loops)
template <int BITS, int KS>
__global__ void __launch_bounds__(QM_THREADS, 1) qgemm_tc_kernel(const QgemmParams p,
                                                                 const __grid_constant__ QgemmMaps maps) {
  extern __shared__ __align__(1024) unsigned char qm_smem[];
  __shared__ __align__(8) uint64_t full_x[QM_NST], full_w[QM_NST], empty[QM_NST], acc_full, acc_empty;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;

  unsigned char* base = qm_smem + ((1024 - (smem_u32(qm_smem) & 1023)) & 1023);
  const int warp = __shfl_sync(0xffffffffu, threadIdx.x >> 5, 0), lane = threadIdx.x & 31;
  const int ntiles = p.row_tiles * p.tok_groups * KS;
  // work item `tile`: weight tile rt, token group tg, k half ks (fastest, so both halves run together)
  auto tg_of = [&](int tile) { return (tile / KS) % p.tok_groups; };
  auto rt_of = [&](int tile) { return tile / (KS * p.tok_groups); };
  auto kb_lo = [&](int tile) { return KS == 1 ? 0 : (tile % KS) * (p.kblocks / 2); };
  auto kb_hi = [&](int tile) { return KS == 1 || (tile % KS) == 1 ? p.kblocks : p.kblocks / 2; };
  if (threadIdx.x == 0) {
    for (int s = 0; s < QM_NST; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&full_w[s], 2 * QM_TM);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty, 2 * QM_TM);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_cols(&s_tmem, QM_TT * QM_TN);  // an fp32 accumulator of 128 lanes x 128 columns per token tile
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  pdl_wait();
  volatile int* abort = &s_abort;
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    // ================================ x tiles ================================
    if (lane == 0) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*abort; tile += gridDim.x) {
        const int tt0 = tg_of(tile) * QM_TT;
        const int nsub = min(QM_TT, p.tok_tiles - tt0);
        for (int kb = kb_lo(tile); kb < kb_hi(tile); ++kb, ++it) {
          const int s = it % QM_NST;
          const uint32_t ph = (it / QM_NST) & 1u;
          if (!qm_wait(&empty[s], ph ^ 1u, abort)) break;
          unsigned char* st = base + (size_t)s * QM_STAGE_BYTES;
          mbar_arrive_expect_tx(&full_x[s], (uint32_t)(2 * nsub * QM_TILE_BYTES));
          for (int j = 0; j < nsub; ++j) {
            tma2d(st + 2 * j * QM_TILE_BYTES, &maps.xhi, kb * QM_KB, (tt0 + j) * QM_TN, &full_x[s]);
            tma2d(st + (2 * j + 1) * QM_TILE_BYTES, &maps.xlo, kb * QM_KB, (tt0 + j) * QM_TN, &full_x[s]);
          }
        }
      }
      // drain: every copy issued lands before the CTA may exit
      for (uint32_t k = it > QM_NST ? it - QM_NST : 0; k < it; ++k) {
        int dummy = 0;
        qm_wait(&full_x[k % QM_NST], (k / QM_NST) & 1u, (volatile int*)&dummy);
      }
    }
  } else if (warp == 1) {
    // ================================ MMA issuer ================================
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*abort; tile += gridDim.x, ++tl) {
        const int tt0 = tg_of(tile) * QM_TT;
        const int nsub = min(QM_TT, p.tok_tiles - tt0);
        const int k_first = kb_lo(tile);
        uint32_t idesc[QM_TT];
        for (int j = 0; j < QM_TT; ++j) {
          const int nt = j < nsub ? min(QM_TN, p.M - (tt0 + j) * QM_TN) : 16;
          idesc[j] = umma_idesc_f16((nt + 15) / 16 * 16);  // MMA N: multiple of 16 for M = 128
        }
        // the epilogue has read the previous tile's accumulator
        if (tl > 0 && !qm_wait(&acc_empty, (tl - 1) & 1u, abort)) break;
        tc_fence_after();
        bool ok = true;
        for (int kb = k_first; kb < kb_hi(tile); ++kb, ++it) {
          const int s = it % QM_NST;
          const uint32_t ph = (it / QM_NST) & 1u;
          if (!qm_wait(&full_x[s], ph, abort) || !qm_wait(&full_w[s], ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(base + (size_t)s * QM_STAGE_BYTES);
          const uint32_t wh = st + QM_W_OFF, wl = wh + QM_TILE_BYTES;
#pragma unroll
          for (int kk = 0; kk < QM_KB / 16; ++kk) {
            const uint32_t off = kk * 32;  // 16 fp16 of k inside the 128-byte swizzle atom
            const uint32_t acc = (kb != k_first || kk != 0) ? 1u : 0u;
            for (int j = 0; j < nsub; ++j) {
              const uint32_t xh = st + 2 * j * QM_TILE_BYTES, xl = xh + QM_TILE_BYTES;
              const uint32_t td = tmem + (uint32_t)(j * QM_TN);
              umma_f16(td, umma_desc_sw128(wh + off), umma_desc_sw128(xh + off), idesc[j], acc);
              umma_f16(td, umma_desc_sw128(wh + off), umma_desc_sw128(xl + off), idesc[j], 1u);
              umma_f16(td, umma_desc_sw128(wl + off), umma_desc_sw128(xh + off), idesc[j], 1u);
            }
          }
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        tc_commit(&acc_full);  // the accumulator is complete
      }
      // wait for the last commits before the TMEM can be freed
      if (*abort) {
        for (uint32_t k = it > QM_NST ? it - QM_NST : 0; k < it; ++k) {
          int dummy = 0;
          qm_wait(&empty[k % QM_NST], (k / QM_NST) & 1u, (volatile int*)&dummy);
        }
      }
    }
  } else {
    // ======================= dequant, then epilogue (warps 2-9) =======================
    // Two warps per TMEM lane group: warp w converts half (w - 2) / 4 of every
    // k block (32 k) of row r and, in the epilogue, every other 32-token block.
    const int lane_base = (warp & 3) * 32;    // TMEM lanes this warp may access
    const int r = lane_base + lane;           // tile row of this thread (= its TMEM lane)
    const int half = (warp - 2) >> 2;         // which 32 k of each k block
    constexpr int WPH = QM_KB / 2 * BITS / 32;  // words per half block (4 or 8)
    constexpr int PD = 4;                       // k blocks per load group
    constexpr int NV = PD * WPH / 4;            // uint4 loads per group (4 or 8)
    uint32_t it = 0, tl = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++tl) {
      const int rt = rt_of(tile), tt0 = tg_of(tile) * QM_TT;
      const int k_end = kb_hi(tile);
      // this thread's weight row
      int rr = rt * QM_TM + r, sg = 0;
      const bool inN = rr < p.N;
      while (sg + 1 < p.nseg && rr >= p.seg_rows[sg]) {
        rr -= p.seg_rows[sg];
        ++sg;
      }
      const bool rvalid = inN && rr < p.seg_rows[sg];
      const int KW = p.K * BITS / 32, KG = p.K / p.group;
      const size_t wrow = rvalid ? (size_t)rr : 0;
      const uint32_t* wrow_p = p.wq[sg] + wrow * KW + half * WPH;
      const uint16_t* srow_p = p.sc[sg] + wrow * KG;
      const uint16_t* brow_p = p.bi[sg] + wrow * KG;
      // Codes, scales and biases straight from global memory, one load group
      // (PD k blocks) ahead of the conversion, so a group's latency hides
      // behind the previous group's work.
      uint4 cw[NV], nw[NV];
      uint32_t csb[PD][2], nsb[PD][2];  // per k block: scale | bias << 16 of the half's first and last group
      auto load_group = [&](int kb0, uint4 (&dw)[NV], uint32_t (&dsb)[PD][2]) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int j = (4 * i) / WPH, wi = (4 * i) % WPH;
          const int kb = kb0 + j;
          dw[i] = (rvalid && kb < k_end) ? ldg_stream_v4(wrow_p + (size_t)kb * (2 * WPH) + wi)
                                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < PD; ++j) {
          const int kb = kb0 + j;
          const int k0 = kb * QM_KB + half * (QM_KB / 2);
          const int g0 = k0 >> p.lg_group, g1 = (k0 + QM_KB / 2 - 1) >> p.lg_group;
          const bool v = rvalid && kb < k_end;
          dsb[j][0] = v ? (uint32_t)ldg_u16(srow_p + g0) | ((uint32_t)ldg_u16(brow_p + g0) << 16) : 0u;
          dsb[j][1] = v ? (uint32_t)ldg_u16(srow_p + g1) | ((uint32_t)ldg_u16(brow_p + g1) << 16) : 0u;
        }
      };
      load_group(kb_lo(tile), cw, csb);
      for (int kb0 = kb_lo(tile); kb0 < k_end && ok; kb0 += PD) {
        if (kb0 + PD < k_end) load_group(kb0 + PD, nw, nsb);
#pragma unroll
        for (int jb = 0; jb < PD; ++jb) {
          const int kb = kb0 + jb;
          if (kb >= k_end) break;
          const int s = it % QM_NST;
          const uint32_t ph = (it / QM_NST) & 1u;
          ++it;
          uint32_t w[WPH];
#pragma unroll
          for (int i = 0; i < WPH; ++i) {
            const uint4& q4 = cw[(jb * WPH + i) >> 2];
            const int e = (jb * WPH + i) & 3;
            w[i] = e == 0 ? q4.x : e == 1 ? q4.y : e == 2 ? q4.z : q4.w;
          }
          const int k0 = kb * QM_KB + half * (QM_KB / 2);
          const int g0 = k0 >> p.lg_group;
          const float s0 = __half2float(__ushort_as_half((uint16_t)(csb[jb][0] & 0xffffu)));
          const float b0 = __half2float(__ushort_as_half((uint16_t)(csb[jb][0] >> 16)));
          const float s1 = __half2float(__ushort_as_half((uint16_t)(csb[jb][1] & 0xffffu)));
          const float b1 = __half2float(__ushort_as_half((uint16_t)(csb[jb][1] >> 16)));
          // first k (within the half) of the half's second group, if it has one
          const int split = min(QM_KB / 2, ((g0 + 1) << p.lg_group) - k0);
          ok = __all_sync(0xffffffffu, qm_wait(&empty[s], ph ^ 1u, abort));
          if (!ok) break;
          unsigned char* st = base + (size_t)s * QM_STAGE_BYTES;
          unsigned char* whp = st + QM_W_OFF;
          unsigned char* wlp = whp + QM_TILE_BYTES;
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // 16-byte chunks: 8 k each
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float v[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int k = c * 8 + e * 2 + h;
                uint32_t q;
                if (BITS == 4)
                  q = (w[k >> 3] >> ((k & 7) * 4)) & 15u;
                else
                  q = (w[k >> 2] >> ((k & 3) * 8)) & 255u;
                const bool second = k >= split;
                v[h] = fmaf(second ? s1 : s0, (float)q, second ? b1 : b0);
              }
              const __half2 hh = __floats2half2_rn(v[0], v[1]);
              const float2 hf = __half22float2(hh);
              const __half2 ll = __floats2half2_rn(v[0] - hf.x, v[1] - hf.y);
              hi[e] = h2_as_u32(hh);
              lo[e] = h2_as_u32(ll);
            }
            const int cc = half * 4 + c;
            *reinterpret_cast<uint4*>(whp + sw128(r, cc)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(wlp + sw128(r, cc)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          }
          fence_async_smem();  // generic-proxy writes visible to the tensor cores
          mbar_arrive(&full_w[s]);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) cw[i] = nw[i];
#pragma unroll
        for (int j = 0; j < PD; ++j) {
          csb[j][0] = nsb[j][0];
          csb[j][1] = nsb[j][1];
        }
      }
      if (!ok) break;
      // ---- epilogue: this thread's row, this warp's 32-token blocks of every token tile
      ok = __all_sync(0xffffffffu, qm_wait(&acc_full, tl & 1u, abort));
      if (!ok) break;
      tc_fence_after();
      const int col = rt * QM_TM + r;
      const float bb = (inN && p.bias) ? __half2float(__ushort_as_half(p.bias[col])) : 0.f;
      const int nsub = min(QM_TT, p.tok_tiles - tt0);
      for (int j = 0; j < nsub; ++j) {
        const int tt = tt0 + j;
        const int nt = min(QM_TN, p.M - tt * QM_TN);
        for (int c0 = half * 32; c0 < nt; c0 += 64) {  // warp-uniform: every lane loads (the load is collective)
          float v[32];
          tmem_ld32(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(j * QM_TN + c0), v);
          if (!inN) continue;
#pragma unroll 4
          for (int i = 0; i < 32; ++i) {
            if (c0 + i >= nt) break;
            const int m = tt * QM_TN + c0 + i;
            if (KS > 1) {  // fp32 scratch, zeroed: two halves add in either order to the same bits
              atomicAdd(reinterpret_cast<float*>(p.y) + (size_t)m * p.ldy + col, v[i]);
              continue;
            }
            float o = v[i] + bb;
            if (p.epi == SC_EPI_RESIDUAL) o += p.residual[(size_t)m * p.ldr + col];
            if (p.y_f16)
              reinterpret_cast<__half*>(p.y)[(size_t)m * p.ldy + col] = __float2half_rn(o);
            else
              reinterpret_cast<float*>(p.y)[(size_t)m * p.ldy + col] = o;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty);
    }
  }
  // ---- teardown: the owner frees the TMEM columns once every role is done with them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    tmem_dealloc_cols(tmem, QM_TT * QM_TN);
    tmem_relinquish();
  }
  if (threadIdx.x == 0 && *abort) atomicExch(&g_qgemm_error, 1);
}

// ---------------------------------------------------------------- x split

// x (fp32 or fp16 [M, ldx], optionally RMS-normalised with weight nw) ->
// fp16 high and low parts [M, K] for the GEMM's B operand.
template <typename XT>
__global__ void qgemm_xsplit_kernel(const XT* __restrict__ x, int ldx, int K, const uint16_t* __restrict__ nw,
                                    float eps, __half* __restrict__ xhi, __half* __restrict__ xlo) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const XT* row = x + (size_t)m * ldx;
  __shared__ float s_red[32];
  float rinv = 1.f;
  if (nw) {
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float v = to_f32<XT>(row[k]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (int)(blockDim.x >> 5) ? s_red[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (threadIdx.x == 0) s_red[0] = t;
    }
    __syncthreads();
    rinv = 1.f / sqrtf(s_red[0] / (float)K + eps);
  }
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = to_f32<XT>(row[k]);
    if (nw) v = (v * rinv) * __half2float(__ushort_as_half(nw[k]));
    const __half h = __float2half_rn(v);
    xhi[(size_t)m * K + k] = h;
    xlo[(size_t)m * K + k] = __float2half_rn(v - __half2float(h));
  }
}

// ---------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 qm_encode_fn() {
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

// fp16 [M, K] row-major, box (64 k, 128 rows), 128-byte swizzle
static bool qm_xmap(CUtensorMap* m, const __half* x, int M, int K) {
  auto fn = qm_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M}, strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {QM_KB, QM_TN}, es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether the tensor-core GEMM serves this linear.
bool qgemm_eligible(int M, int K, int nseg, const int* seg_rows, int epi, int bits, int group) {
  if (M < 1 || K % QM_KB || (bits != 4 && bits != 8) || (group != 32 && group != 64 && group != 128)) return false;
  if (K % group) return false;
  if (epi == SC_EPI_SWIGLU && !(nseg == 2 && seg_rows[0] == seg_rows[1])) return false;
  for (int s = 0; s + 1 < nseg; ++s)
    if (seg_rows[s] % QM_TM) return false;  // a 128-row tile must not straddle two tensors
  return true;
}

// y[m, j] = silu(t[m, j]) * t[m, F + j] for the stacked gate|up product t [M, 2F].
template <typename YT>
__global__ void qgemm_swiglu_rows_kernel(const float* __restrict__ t, int M, int F, YT* __restrict__ y, int ldy) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)M * F;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t m = i / F, j = i % F;
    const float g = t[m * 2 * F + j], u = t[m * 2 * F + F + j];
    y[m * ldy + j] = from_f32<YT>(silu_f32(g) * u);
  }
}

size_t qgemm_workspace_bytes(int M, int K, int N, int epi) {
  size_t b = 2 * (size_t)M * K * sizeof(__half) + 512;
  // fp32 scratch: the [gate | up] product (SwiGLU), or the split-k sum
  b += (size_t)M * (epi == SC_EPI_SWIGLU ? 2 * N : N) * sizeof(float) + 256;
  return b;
}

// Split-k finish: y = acc (+ bias) (+ residual), in y's dtype.
template <typename YT>
__global__ void qgemm_finish_kernel(const float* __restrict__ acc, int M, int N, const uint16_t* __restrict__ bias,
                                    const float* residual, int ldr, YT* y, int ldy) {
  pdl_trigger();
  pdl_wait();
  const size_t total = (size_t)M * N;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(e / N), n = (int)(e % N);
    float o = acc[e];
    if (bias) o += __half2float(__ushort_as_half(bias[n]));
    if (residual) o += residual[(size_t)m * ldr + n];
    y[(size_t)m * ldy + n] = from_f32<YT>(o);
  }
}

int run_qgemm(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_w, float eps, int nseg,
              const uint32_t* const* wq, const uint16_t* const* scales, const uint16_t* const* biases,
              const int* seg_rows, int group, int bits, const uint16_t* bias, int epi, void* y, int y_dtype,
              int ldy, const float* residual, int ldr, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const int Nout = epi == SC_EPI_SWIGLU ? seg_rows[0] : [&] {
    int n = 0;
    for (int s = 0; s < nseg; ++s) n += seg_rows[s];
    return n;
  }();
  const size_t need = qgemm_workspace_bytes(M, K, Nout, epi);
  SC_REQUIRE(ws && ws_bytes >= need, SC_ERR_WORKSPACE, "qgemm: workspace of %zu bytes needed (got %zu)", need,
             ws_bytes);
  __half* xhi = reinterpret_cast<__half*>((reinterpret_cast<uintptr_t>(ws) + 255) / 256 * 256);
  __half* xlo = xhi + (size_t)M * K;
  float* tmp = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(xlo + (size_t)M * K) + 255) / 256 * 256);
  // x -> fp16 high / low parts (RMSNorm applied here)
  const int thr = 256;
  if (x_dtype == SC_F32)
    launch(qgemm_xsplit_kernel<float>, dim3(M), dim3(thr), 0, stream, static_cast<const float*>(x), ldx, K, norm_w,
           eps, xhi, xlo);
  else
    launch(qgemm_xsplit_kernel<__half>, dim3(M), dim3(thr), 0, stream, static_cast<const __half*>(x), ldx, K,
           norm_w, eps, xhi, xlo);
  int st = check_launch("qgemm_xsplit");
  if (st != SC_OK) return st;
  QgemmMaps maps;
  SC_REQUIRE(qm_xmap(&maps.xhi, xhi, M, K) && qm_xmap(&maps.xlo, xlo, M, K), SC_ERR_CUDA,
             "qgemm: tensor map of x refused");
  QgemmParams p{};
  int N = 0;
  for (int s = 0; s < nseg; ++s) {
    p.wq[s] = wq[s];
    p.sc[s] = scales[s];
    p.bi[s] = biases[s];
    p.seg_rows[s] = seg_rows[s];
    N += seg_rows[s];
  }
  p.nseg = nseg;
  p.M = M;
  p.K = K;
  p.N = N;
  p.group = group;
  p.lg_group = group == 32 ? 5 : group == 64 ? 6 : 7;
  p.bits = bits;
  p.bias = epi == SC_EPI_SWIGLU ? nullptr : bias;
  p.epi = epi == SC_EPI_SWIGLU ? SC_EPI_STORE : epi;
  p.row_tiles = (N + QM_TM - 1) / QM_TM;
  p.tok_tiles = (M + QM_TN - 1) / QM_TN;
  p.tok_groups = (p.tok_tiles + QM_TT - 1) / QM_TT;
  p.kblocks = K / QM_KB;
  // halves of k as separate work items when twice the tiles still fit one wave of SMs
  p.ksplit = (2 * p.row_tiles * p.tok_groups <= sm_count() && p.kblocks >= 8) ? 2 : 1;
  const bool scratch = epi == SC_EPI_SWIGLU || p.ksplit > 1;
  p.y = scratch ? static_cast<void*>(tmp) : y;
  p.y_f16 = scratch ? 0 : y_dtype == SC_F16;
  p.ldy = scratch ? N : ldy;
  if (p.ksplit > 1) {
    cudaError_t e = cudaMemsetAsync(tmp, 0, (size_t)M * N * sizeof(float), stream);
    SC_REQUIRE(e == cudaSuccess, SC_ERR_CUDA, "qgemm: scratch memset failed (%s)", cudaGetErrorString(e));
  }
  p.residual = residual;
  p.ldr = ldr;
  const int ntiles = p.row_tiles * p.tok_groups * p.ksplit;
  const int grid = std::min(ntiles, sm_count());
  const size_t smem = (size_t)QM_NST * QM_STAGE_BYTES + 1024;
  static bool cfg[2][2] = {};  // shared-memory opt-in, once per instantiation
  auto go = [&](auto kern, int bi, int ki) {
    if (!cfg[bi][ki]) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      cfg[bi][ki] = true;
    }
    launch(kern, dim3(grid), dim3(QM_THREADS), smem, stream, p, maps);
  };
  if (bits == 4)
    p.ksplit == 2 ? go(qgemm_tc_kernel<4, 2>, 0, 1) : go(qgemm_tc_kernel<4, 1>, 0, 0);
  else
    p.ksplit == 2 ? go(qgemm_tc_kernel<8, 2>, 1, 1) : go(qgemm_tc_kernel<8, 1>, 1, 0);
  st = check_launch("qgemm_tc");
  if (st != SC_OK) return st;
  if (epi != SC_EPI_SWIGLU) {
    if (p.ksplit == 1) return SC_OK;
    const int blocks = (int)std::min<size_t>(((size_t)M * N + 255) / 256, (size_t)8 * sm_count());
    const float* res = epi == SC_EPI_RESIDUAL ? residual : nullptr;
    if (y_dtype == SC_F16)
      launch(qgemm_finish_kernel<__half>, dim3(blocks), dim3(256), 0, stream, tmp, M, N, bias, res, ldr,
             static_cast<__half*>(y), ldy);
    else
      launch(qgemm_finish_kernel<float>, dim3(blocks), dim3(256), 0, stream, tmp, M, N, bias, res, ldr,
             static_cast<float*>(y), ldy);
    return check_launch("qgemm_finish");
  }
  const int F = seg_rows[0];
  const int blocks = (int)std::min<size_t>(((size_t)M * F + 255) / 256, (size_t)8 * sm_count());
  if (y_dtype == SC_F16)
    launch(qgemm_swiglu_rows_kernel<__half>, dim3(blocks), dim3(256), 0, stream, tmp, M, F, static_cast<__half*>(y),
           ldy);
  else
    launch(qgemm_swiglu_rows_kernel<float>, dim3(blocks), dim3(256), 0, stream, tmp, M, F, static_cast<float*>(y),
           ldy);
  return check_launch("qgemm_swiglu_rows");
}

}  // namespace sc

extern "C" {

int sc_qgemm_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sc::g_qgemm_error, sizeof(int));
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(sc::g_qgemm_error, &z, sizeof(int));
  }
  return v;
}

size_t sc_qgemm_workspace_bytes(int M, int K, int N, int epilogue) { return sc::qgemm_workspace_bytes(M, K, N, epilogue); }

int sc_qgemm(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_weight, float norm_eps, int nseg,
             const uint32_t* const* wq, const uint16_t* const* scales, const uint16_t* const* biases,
             const int* seg_rows, int group_size, int bits, const uint16_t* bias, int epilogue, void* y, int y_dtype,
             int ldy, const float* residual, int ldr, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(x && y && wq && scales && biases && seg_rows, SC_ERR_ARG, "qgemm: null pointer argument");
  SC_REQUIRE(nseg >= 1 && nseg <= 3, SC_ERR_SHAPE, "qgemm: 1..3 weight segments (got %d)", nseg);
  SC_REQUIRE(qgemm_eligible(M, K, nseg, seg_rows, epilogue, bits, group_size), SC_ERR_UNSUPPORTED,
             "qgemm: shape M=%d K=%d bits=%d group=%d not served by the tensor-core GEMM", M, K, bits, group_size);
  SC_REQUIRE(x_dtype == SC_F16 || x_dtype == SC_F32, SC_ERR_ARG, "qgemm: x dtype");
  SC_REQUIRE(y_dtype == SC_F16 || y_dtype == SC_F32, SC_ERR_ARG, "qgemm: y dtype");
  SC_REQUIRE(epilogue != SC_EPI_RESIDUAL || residual, SC_ERR_ARG, "qgemm: residual epilogue needs residual");
  SC_REQUIRE(epilogue != SC_EPI_SWIGLU || !bias, SC_ERR_UNSUPPORTED, "qgemm: bias with SwiGLU epilogue");
  for (int s = 0; s < nseg; ++s)
    SC_REQUIRE(wq[s] && scales[s] && biases[s] && seg_rows[s] > 0, SC_ERR_ARG, "qgemm: bad weight segment %d", s);
  return run_qgemm(x, x_dtype, M, K, ldx, norm_weight, norm_eps, nseg, wq, scales, biases, seg_rows, group_size,
                   bits, bias, epilogue, y, y_dtype, ldy, residual, ldr, workspace, workspace_bytes, stream);
}

}  // extern "C"
