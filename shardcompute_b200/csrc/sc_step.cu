// Persistent decode step: one launch runs a whole greedy decode token of the
// tensor-parallel quantized Llama (embedding, every layer's q|k|v GEMV,
// attention, o_proj, gate|up, down_proj, the tied LM head and the argmax),
// for batch 1 and 4-bit group-64 weights.  It replaces the ~130 launches per
// token of the per-kernel engine (the reference's per-token forward,
// parallel/transformer.py:516-577, driven by worker/executor.py:267-325).
//
// Why one kernel.  At batch 1 a token is a chain of small dependent GEMVs
// (8-66 MB each at Llama-3-8B TP1, 1-8 MB at TP8).  Launched one by one,
// every GEMV pays a pipeline fill, activation staging in each CTA and an
// epilogue drain while HBM idles.  Here one CTA per SM lives for the whole
// token; its producer warp streams the weights of every GEMV -- and the
// cached keys / values of every attention -- through one shared-memory ring
// without ever waiting on activations, so HBM keeps streaming across op
// boundaries; only the consumer warps wait for their inputs.
//
// Work split (stream-K).  A GEMV's work is the (16-row tile) x (512-k box)
// grid, flattened tile-major; CTA c takes the contiguous range
// [c*T/n, (c+1)*T/n), so every CTA streams the same bytes whatever the
// shape.  A tile cut by a range boundary is a "segment" of each CTA holding
// a piece; segments write partial row sums, and a row's output is the sum of
// its tile's segments in CTA order (deterministic).
//
// Dependencies (no grid barrier).  Outputs are finished per 64-row group:
// the CTA whose segment completes a group (an atomic count) sums the group's
// partials, adds the peers' partials (tensor parallel: pushed over NVLink as
// epoch-tagged 16-byte lines), adds the residual, and writes the NEXT GEMV's
// input already in its B-fragment layout (fp16 high / low parts, per-group
// sums for the exact-weight factorisation, and the per-group sum of squares
// for its RMSNorm); a per-op counter tells the consumers the input is
// complete.  Attention segments merge per kv head the same way: the last
// segment of a head merges the head and stages o_proj's input.  The last CTA
// to finish the LM head writes the token and advances the position.
//
// Numerics follow the per-kernel decode path: weights exact (s * sum q x +
// b * sum x per group), activations carried to ~22 bits, fp32 accumulation,
// fp32 KV cache.  Every wait is bounded (globaltimer); a timeout raises the
// error word and every CTA skips the rest of the step instead of hanging.
#include <string.h>

#include <algorithm>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "sc_common.cuh"

namespace sc {

// ---------------------------------------------------------------- geometry
constexpr int SP_NCW = 12;                     // consumer warps (13 warps x 128 registers fill the register file)
constexpr int SP_NC = SP_NCW * 32;             // consumer threads
constexpr int SP_THREADS = SP_NC + 32;         // + the producer warp
constexpr int SP_KPC = 128;                    // k values per chunk (16 words of 4-bit codes)
constexpr int SP_BOX_CH = 4;                   // chunks per TMA box (two 32-word blocks)
constexpr int SP_BOX_K = SP_BOX_CH * SP_KPC;   // 512 k values per box
constexpr int SP_WBOX = 16 * SP_BOX_CH * 64;   // packed-word bytes of a box: 16 rows x 4 chunks (4 KB)
constexpr int SP_SBOX = 16 * 8 * 2;            // scale (or bias) bytes of a box: 16 rows x 8 groups
constexpr int SP_UNIT = SP_WBOX + 2 * SP_SBOX;   // one unit of a weight image: words, scales, biases (4.5 KB)
constexpr int SP_STAGE_BOXES = 6;              // 24 chunks of one set, or 12 chunk pairs of gate|up
constexpr int SP_STAGE_BYTES = SP_STAGE_BOXES * SP_UNIT;  // 27 KB
constexpr int SP_MAX_NST = 8;
constexpr int SP_WIN = 8;                      // segments in flight per CTA (output slots)
constexpr int SP_MAXT = 4;                     // segments per tile (CTAs a tile may be cut over)
constexpr int SP_CB = 576;                     // staged x bytes per chunk: 512 B fragments + 64 B sums
constexpr int SP_MAX_SEG = 3;                  // weight tensors stacked along N (q | k | v)
constexpr uint64_t SP_WAIT_NS = 2000000000ull;
constexpr int SP_MAX_WORLD = 8;
constexpr size_t SP_ARENA_HDR = 4096;

enum : int { SOP_EMBED = 0, SOP_QKV = 1, SOP_ATTN = 2, SOP_O = 3, SOP_GATEUP = 4, SOP_DOWN = 5, SOP_HEAD = 6 };

// Error codes written to the error word (first one wins).
enum : int { SPE_RING = 2, SPE_PEER = 3, SPE_QKV = 4, SPE_INPUT = 5, SPE_SLOT = 6, SPE_ARGMAX = 7 };

struct StepOp {
  int kind;
  int layer;
  // ---- GEMV
  int nset;                  // 1, or 2 for the gate|up pair (row r of both)
  int nseg;                  // weight tensors stacked along N
  int seg_tiles[SP_MAX_SEG]; // tiles of each tensor
  const unsigned char* img;  // weight image: unit u, set a at (u * nset + a) * SP_UNIT
  int K, kq, tiles;          // reduction length, boxes per row, 16-row tiles
  int rows;                  // valid output rows
  long long total;           // tiles * kq
  const unsigned char* xs;   // staged input (global)
  const float* xss;          // its per-group sums of squares (null: no RMSNorm)
  int xs_bytes;              // staged bytes (kq * 4 chunks)
  int x_ctr, x_need;         // input complete when ctr[x_ctr] reaches (gen+1) * x_need
  float* part;               // segment partials [tiles][SP_MAXT][nset][16]
  int grp_ctr;               // first group counter (QKV: its segment counter; HEAD: its tile counters)
  int seg_need;              // QKV: segments per step (what the attention waits for)
  // ---- conversion of the output into the next GEMV's input
  unsigned char* out_xs;
  float* out_xss;            // null: the next GEMV has no RMSNorm
  const uint16_t* out_norm;  // the next GEMV's RMSNorm weight (null: none)
  int out_ctr;
  float* h;                  // residual stream (row ops, embedding)
  float* trace;              // hidden-state trace row (or null)
  int xchg;                  // exchange index of a tensor-parallel sum (-1: none)
  // ---- attention
  float* kc;                 // this layer's cache [Hkv][Lmax][hd]
  float* vc;
};

struct StepParams {
  const StepOp* ops;
  int nops;
  int* ctr;                  // counters
  int* gen;                  // completed steps (device)
  int* err;                  // error word
  int* info;                 // where the first error was raised: op, CTA, warp, value seen, target
  int* progress;             // [nsm] per CTA: the op its consumers last started (nops: step done)
  unsigned long long* stamps;  // null, or [nsm][nops][4] %globaltimer: op start, input ready, stream done, op done
  int* head_done;
  int* attn_ctr;             // [2 parities][layers][Hkv] segment counts, reset every other step
  unsigned long long* key;   // [2] argmax keys by step parity
  int* tok;                  // token in / out
  int* pos;                  // cache length before this step
  const float* cos_tab;
  const float* sin_tab;
  int max_pos;
  float* logits;             // optional [Vl] (tests)
  const uint32_t* emb_w;     // the vocab-split embedding (its tied weights are the LM head)
  const uint16_t* emb_s;
  const uint16_t* emb_b;
  int vocab_start, vocab_local;
  float* attn_part;          // [layers][Hkv][nsm][G][hd + 4]
  int H, Hq, Hkv, hd, Lmax, nl;
  float eps, scale;
  int xs_alloc;              // shared bytes reserved for staged x (and attention merges)
  int nst;
  int world, rank;
  char* arena[SP_MAX_WORLD]; // every rank's exchange arena as mapped here
  size_t row_region;         // bytes of one (slot, source rank) region of row lines
  size_t key_off;            // offset of the argmax lines
};

// ---------------------------------------------------------------- small helpers

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float ldcg_f(const float* p) { return __ldcg(p); }

__device__ __forceinline__ uint4 ldcg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4_volatile(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint4 ld_v4_volatile(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void raise_err(const StepParams& P, int code) { atomicCAS(P.err, 0, code); }
// The first error also records where: op index, CTA, warp, the value seen and the one waited for.
__device__ __forceinline__ void raise_at(const StepParams& P, int code, int where, int seen, int target) {
  if (atomicCAS(P.err, 0, code) == 0) {
    volatile int* f = P.info;
    f[0] = where;
    f[1] = (int)blockIdx.x;
    f[2] = (int)(threadIdx.x >> 5);
    f[3] = seen;
    f[4] = target;
  }
}
__device__ __forceinline__ bool err_set(const StepParams& P) { return *reinterpret_cast<volatile int*>(P.err) != 0; }

// Spin until ctr reaches target (wrap-safe), giving up after SP_WAIT_NS or
// as soon as any CTA has raised the error word.
__device__ bool wait_ctr(const StepParams& P, const int* ctr, int target, int code, int where) {
  if ((int)(ld_acquire(ctr) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if ((int)(ld_acquire(ctr) - target) >= 0) return true;
    if ((i & 31) == 0) {
      if (err_set(P)) return false;
      if (globaltimer_ns() - t0 > SP_WAIT_NS) {
        raise_at(P, code, where, ld_acquire(ctr), target);
        return false;
      }
    }
  }
}

// One mbarrier wait for a whole warp (the lanes vote), bounded, watching the
// CTA's abort flag and the global error word.
__device__ __forceinline__ bool mbar_wait_all(const StepParams& P, uint64_t* bar, uint32_t parity,
                                              volatile int* abort, int where) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  bool ok = true;
  if (!mbar_try_wait(bar, parity)) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
      if (mbar_try_wait(bar, parity)) break;
      if ((i & 15) == 0) {
        if (*abort || err_set(P)) {
          ok = false;
          break;
        }
        if (globaltimer_ns() - t0 > SP_WAIT_NS) {
          raise_at(P, SPE_RING, where, (int)parity, -1);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// Owner CTA of flat unit u in a range of T units split over n CTAs
// (CTA c holds [c*T/n, (c+1)*T/n)).
__device__ __host__ __forceinline__ int owner_of(long long u, long long T, int n) {
  return (int)(((u + 1) * n - 1) / T);
}
__device__ __host__ __forceinline__ long long range_lo(int c, long long T, int n) { return (long long)c * T / n; }

// CTAs a GEMV's T units (tiles of kq) are split over.  Every CTA of the split
// holds at least one unit, so the CTAs between a tile's first and last owner
// all hold a piece of it (the segment count below relies on that).  Each CTA
// holds at least r = ceil((kq - 1) / (SP_MAXT - 1)) units, so a tile's kq
// units cross at most ceil((kq - 1) / r) + 1 <= SP_MAXT CTAs: small GEMVs on
// many SMs run on fewer CTAs rather than cut a tile into more segments.
__device__ __host__ __forceinline__ int gemv_ctas(long long T, int kq, int n) {
  long long c = std::min<long long>(T, n);
  const long long r = (kq - 1 + SP_MAXT - 2) / (SP_MAXT - 1);
  if (r > 1) c = std::min<long long>(c, std::max<long long>(1, T / r));
  return (int)c;
}

// First CTA holding tile t (units [t*kq, (t+1)*kq)) and the tile's segment count.
__device__ __host__ __forceinline__ int tile_first(int t, int kq, long long T, int n) {
  return owner_of((long long)t * kq, T, n);
}
__device__ __host__ __forceinline__ int tile_nseg(int t, int kq, long long T, int n) {
  return owner_of((long long)(t + 1) * kq - 1, T, n) - tile_first(t, kq, T, n) + 1;
}

// tile row read by mma row m (the permutation keeps the swizzled loads conflict free)
__device__ __forceinline__ int sp_tile_row(int m) { return ((m & 7) >> 1) + 4 * (m & 1) + (m & 8); }

// (w & MASK) | 0x64006400 in one three-input logic op: fp16 pairs 1024 + q (or 1024 + 16 q)
template <uint32_t MASK>
__device__ __forceinline__ uint32_t mag(uint32_t w) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(d) : "r"(w), "n"(MASK), "n"(0x64006400u));
  return d;
}

__device__ __forceinline__ uint64_t evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> shared (16-byte aligned, size a multiple of 16, no
// multicast) with an L2 eviction hint: streamed weights should not push the
// KV cache and the activations out of L2.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                               uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Orderable 64-bit argmax key: the larger value wins, then the lower index
// (the reference argmaxes the gathered logits: ties go to the first index).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

__device__ __forceinline__ unsigned long long warp_max_key(unsigned long long k) {
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
    k = o > k ? o : k;
  }
  return k;
}

// ---------------------------------------------------------------- staged inputs

// Stages 64 values (one quantization group of the next GEMV's input; lane l
// holds values 2l, 2l+1 of the group) in the layout the decode GEMV's B
// fragments read: per 128-k chunk, [part hi/lo][q][t] 16-byte units of fp16
// (the slots of odd codes carry x / 16, matching A = 1024 + 16 q) and a
// 64-byte table of per-column sums: -1024 * sum(part) cancels the code
// offset, sum(x) feeds the bias term.  `w` multiplies x (the next RMSNorm's
// weight; its 1/rms is applied to that GEMV's outputs); xss receives
// sum(x^2) of the unweighted values.
__device__ void stage_group(unsigned char* xs, float* xss, const uint16_t* w, int g, float x0, float x1, int lane) {
  const int k0 = g * 64 + 2 * lane;
  float a = x0, b = x1;
  if (w) {
    const __half2 wp = *reinterpret_cast<const __half2*>(w + k0);
    a = x0 * __low2float(wp);
    b = x1 * __high2float(wp);
  }
  const __half2 hp = __floats2half2_rn(a, b * 0.0625f);
  const float2 hf = __half22float2(hp);
  const __half2 lp = __floats2half2_rn(a - hf.x, b * 0.0625f - hf.y);
  const float2 lf = __half22float2(lp);
  float sh = hf.x + hf.y, sl = lf.x + lf.y, sx = a + b, sq = fmaf(x0, x0, x1 * x1);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    sh += __shfl_xor_sync(0xffffffffu, sh, o);
    sl += __shfl_xor_sync(0xffffffffu, sl, o);
    sx += __shfl_xor_sync(0xffffffffu, sx, o);
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  // lane l: word u = l / 4 of the group, elements e = 2 (l % 4), e + 1.  A
  // 16-byte unit holds the halves [e0 e4 e1 e5 e2 e6 e3 e7], so lane i < 2
  // of a quad pairs its halves with lane i + 2's and writes 8 bytes.
  const uint32_t hw = h2_as_u32(hp), lw = h2_as_u32(lp);
  const uint32_t hw2 = __shfl_down_sync(0xffffffffu, hw, 2);
  const uint32_t lw2 = __shfl_down_sync(0xffffffffu, lw, 2);
  const int i = lane & 3;
  const int cl = (g * 64) / SP_KPC;        // chunk
  const int grp = ((g * 64) % SP_KPC) / 64;  // group within the chunk
  const int u = grp * 8 + (lane >> 2);     // word within the chunk
  const int t = u >> 2, q = u & 3;
  unsigned char* cb = xs + (size_t)cl * SP_CB;
  if (i < 2) {
    const uint32_t w0h = (hw & 0xffffu) | (hw2 << 16), w1h = (hw >> 16) | (hw2 & 0xffff0000u);
    const uint32_t w0l = (lw & 0xffffu) | (lw2 << 16), w1l = (lw >> 16) | (lw2 & 0xffff0000u);
    *reinterpret_cast<uint2*>(cb + ((0 * 4 + q) * 4 + t) * 16 + 8 * i) = make_uint2(w0h, w1h);
    *reinterpret_cast<uint2*>(cb + ((1 * 4 + q) * 4 + t) * 16 + 8 * i) = make_uint2(w0l, w1l);
  }
  if (lane == 0) {
    // B columns: hi part -> column grp, lo part -> column 2 + grp (batch 1, two groups per chunk);
    // lane t of the mma reads {xoff(2t), xoff(2t+1), xsum(2t), xsum(2t+1)} at 16 t
    float* tab = reinterpret_cast<float*>(cb + 512);
    tab[grp] = -1024.f * sh;
    tab[2 + grp] = sx;
    tab[4 + grp] = -1024.f * sl;
    tab[6 + grp] = 0.f;
    if (xss) xss[g] = sq;
  }
}

// Tensor-parallel sum of one 64-value group, in two halves.  push_group
// sends this rank's two values per lane to every peer as one epoch-tagged
// 16-byte line (never waits); recv_group waits for the peers' lines and sums
// all ranks in rank order (false if a wait gave up).  A CTA that completes a
// group in the middle of its stream pushes at once and receives only after
// its stream is done, so no wait on a peer ever holds up a ring that the
// peer may itself be waiting on.
__device__ __forceinline__ uint32_t xchg_epoch(int xchg, int gen) {
  return ((uint32_t)(gen + 1) << 8) | (uint32_t)(xchg & 0xff);
}

__device__ void push_group(const StepParams& P, int xchg, int g, float v0, float v1, int lane, int gen) {
  const uint32_t ep = xchg_epoch(xchg, gen);
  const int slot = xchg & 1;
  const size_t line = (size_t)g * 32 + lane;
  const uint32_t a = __float_as_uint(v0), b = __float_as_uint(v1);
  for (int k = 1; k < P.world; ++k) {
    const int dst = (P.rank + k) % P.world;
    char* base = P.arena[dst] + SP_ARENA_HDR + ((size_t)slot * P.world + P.rank) * P.row_region;
    st_v4_volatile(base + line * 16, a, ep, b, ep);
  }
}

__device__ bool recv_group(const StepParams& P, int xchg, int g, float& v0, float& v1, int lane, int gen) {
  const uint32_t ep = xchg_epoch(xchg, gen);
  const int slot = xchg & 1;
  const size_t line = (size_t)g * 32 + lane;
  float s0 = 0.f, s1 = 0.f;
  bool ok = true;
  for (int r = 0; r < P.world; ++r) {
    float p0 = v0, p1 = v1;
    if (r != P.rank) {
      const char* base = P.arena[P.rank] + SP_ARENA_HDR + ((size_t)slot * P.world + r) * P.row_region;
      uint4 l = ld_v4_volatile(base + line * 16);
      if (ok && (l.y != ep || l.w != ep)) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t i = 1;; ++i) {
          l = ld_v4_volatile(base + line * 16);
          if (l.y == ep && l.w == ep) break;
          if ((i & 31) == 0) {
            if (err_set(P)) {
              ok = false;
              break;
            }
            if (globaltimer_ns() - t0 > SP_WAIT_NS) {
              raise_err(P, SPE_PEER);
              ok = false;
              break;
            }
          }
        }
      }
      p0 = __uint_as_float(l.x);
      p1 = __uint_as_float(l.z);
    }
    s0 = r == 0 ? p0 : s0 + p0;
    s1 = r == 0 ? p1 : s1 + p1;
  }
  v0 = s0;
  v1 = s1;
  return __all_sync(0xffffffffu, ok);
}

__device__ bool xchg_group(const StepParams& P, int xchg, int g, float& v0, float& v1, int lane, int gen) {
  if (P.world == 1) return true;
  push_group(P, xchg, g, v0, v1, lane, gen);
  return recv_group(P, xchg, g, v0, v1, lane, gen);
}

// Output rows (row, row + 1) of set a: the sum of the tile's segment partials in CTA order.
__device__ __forceinline__ void sum_rows(const StepOp& op, int a, int row, int n, float& v0, float& v1) {
  const int t = row >> 4, tr = row & 15;
  const int ns = tile_nseg(t, op.kq, op.total, n);
  float s0 = 0.f, s1 = 0.f;
  for (int j = 0; j < ns; ++j) {
    const float* p = op.part + (((size_t)t * SP_MAXT + j) * op.nset + a) * 16 + tr;
    s0 += ldcg_f(p);
    s1 += ldcg_f(p + 1);
  }
  v0 = s0;
  v1 = s1;
}

// q|k|v output row r: the sum of its tile's segment partials.
__device__ __forceinline__ float qkv_row(const StepOp& qop, int r, int n) {
  const int t = r >> 4;
  const int ns = tile_nseg(t, qop.kq, qop.total, n);
  float a = 0.f;
  for (int j = 0; j < ns; ++j) a += ldcg_f(qop.part + ((size_t)t * SP_MAXT + j) * 16 + (r & 15));
  return a;
}

// Finishing output group g of a GEMV op: the sum of its partials (plus, for
// the row-parallel ops, the peers' partials and the residual), staged as the
// next GEMV's input, then that input's counter.  `received` (row ops at
// tensor parallel): the all-rank sums, already pushed and received.
__device__ void finish_group(const StepParams& P, const StepOp& op, int g, int lane, int n, int gen,
                             const float* received = nullptr) {
  const int row = g * 64 + 2 * lane;
  float v0, v1;
  if (op.kind == SOP_GATEUP) {
    float g0, g1, u0, u1;
    sum_rows(op, 0, row, n, g0, g1);
    sum_rows(op, 1, row, n, u0, u1);
    v0 = silu_f32(g0) * u0;
    v1 = silu_f32(g1) * u1;
  } else {  // O / DOWN: this rank's partial, the peers' partials, the residual
    if (received) {
      v0 = received[0];
      v1 = received[1];
    } else {
      sum_rows(op, 0, row, n, v0, v1);
    }
    const float2 hold = __ldcg(reinterpret_cast<const float2*>(op.h + row));
    v0 = hold.x + v0;
    v1 = hold.y + v1;
    *reinterpret_cast<float2*>(op.h + row) = make_float2(v0, v1);
    if (op.trace) *reinterpret_cast<float2*>(op.trace + row) = make_float2(v0, v1);
  }
  stage_group(op.out_xs, op.out_xss, op.out_norm, g, v0, v1, lane);
  __syncwarp();
  __threadfence();
  if (lane == 0) atomicAdd(P.ctr + op.out_ctr, 1);
}

// ---------------------------------------------------------------- shared state

struct StepShared {
  uint64_t full[SP_MAX_NST];
  uint64_t empty[SP_MAX_NST];
  unsigned long long key;    // this CTA's LM-head candidate
  int abort;
  int gen;
  int pos;
  int cnt[SP_WIN];           // warps that flushed a segment into a slot
  int free_at[SP_WIN];       // first segment allowed into a slot
  float rinv;                // 1 / rms of the current GEMV's input
  int attn_last;             // this CTA completed the current kv head's segments: it merges them
  int ndefer;                // row-op groups completed here, waiting for the peers' partials
  int defer[64];
};

// ---------------------------------------------------------------- GEMV segments

// One CTA's share of a GEMV op: units [lo, hi) (tile rows t_first...), kq
// units per tile row, nC CTAs in the split, the RMSNorm factor of the input.
struct SegCtx {
  long long lo, hi;
  int t_first, kq, nC;
  float rinv;
};

// Warps holding a piece of segment j (chunk p of the CTA's range goes to
// warp p % SP_NCW; the segment's chunks are one contiguous run of them).
__device__ __forceinline__ uint32_t seg_warps(const SegCtx& sc, int j) {
  constexpr uint32_t FULL = (1u << SP_NCW) - 1u;
  const long long tt = sc.t_first + j;
  const long long a = (std::max(sc.lo, tt * sc.kq) - sc.lo) * SP_BOX_CH;
  const long long b = (std::min(sc.hi, (tt + 1) * sc.kq) - sc.lo) * SP_BOX_CH;
  if (b - a >= SP_NCW) return FULL;
  const uint32_t m = ((1u << (int)(b - a)) - 1u) << (int)(a % SP_NCW);
  return (m | (m >> SP_NCW)) & FULL;
}

// Epilogue of segment j, run by the warp that completed it: the warps'
// partials summed in warp order, then the segment's partial to global memory
// (or, for a tile held whole, straight into the LM-head argmax), and, when it
// was the tile group's last segment, the group's finish.  Out of line: it
// runs once per segment and keeps its registers out of the stream loop.
__device__ __noinline__ void seg_epilogue(const StepParams& P, const StepOp& op, StepShared& S,
                                          float (*s_slot)[2][16][SP_NCW], const SegCtx& sc, int j, int c, int gen,
                                          int lane) {
  const int slot = j % SP_WIN;
  const int tile = sc.t_first + j;
  const uint32_t msk = seg_warps(sc, j);
  const int a = lane >> 4, row = lane & 15;
  float v = 0.f;
  if (a < op.nset) {
#pragma unroll
    for (int w = 0; w < SP_NCW; ++w)
      if (msk & (1u << w)) v += s_slot[slot][a][row][w];
    v *= sc.rinv;
  }
  __syncwarp();
  if (lane == 0) {  // the slot is free for segment j + SP_WIN
    S.cnt[slot] = 0;
    __threadfence_block();
    *reinterpret_cast<volatile int*>(&S.free_at[slot]) = j + SP_WIN;
  }
  const int nseg_t = tile_nseg(tile, sc.kq, op.total, sc.nC);
  if (op.kind == SOP_HEAD && nseg_t == 1) {
    // the whole tile is here: logits straight into this CTA's argmax candidate
    unsigned long long k = 0ull;
    const int r = tile * 16 + row;
    if (a == 0 && r < op.rows) {
      if (P.logits) P.logits[r] = v;
      k = argmax_key(v, P.vocab_start + r);
    }
    k = warp_max_key(k);
    if (lane == 0) atomicMax(&S.key, k);
    return;
  }
  const int segslot = c - tile_first(tile, sc.kq, op.total, sc.nC);
  if (a < op.nset) op.part[(((size_t)tile * SP_MAXT + segslot) * op.nset + a) * 16 + row] = v;
  __syncwarp();
  __threadfence();
  if (op.kind == SOP_QKV) {
    if (lane == 0) atomicAdd(P.ctr + op.grp_ctr, 1);
    return;
  }
  if (op.kind == SOP_HEAD) {
    int last = 0;
    if (lane == 0) last = atomicAdd(P.ctr + op.grp_ctr + tile, 1) + 1 - (gen + 1) * nseg_t == 0;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    unsigned long long k = 0ull;
    if (lane < 16) {
      float s = 0.f;
      for (int jj = 0; jj < nseg_t; ++jj) s += ldcg_f(op.part + ((size_t)tile * SP_MAXT + jj) * 16 + lane);
      const int r = tile * 16 + lane;
      if (r < op.rows) {
        if (P.logits) P.logits[r] = s;
        k = argmax_key(s, P.vocab_start + r);
      }
    }
    k = warp_max_key(k);
    if (lane == 0) atomicMax(&S.key, k);
    return;
  }
  // O / DOWN / GATEUP: the group of four tiles
  const int grp = tile >> 2;
  int need = 0;
  for (int tt = grp * 4; tt < grp * 4 + 4; ++tt) need += tile_nseg(tt, sc.kq, op.total, sc.nC);
  int last = 0;
  if (lane == 0) last = atomicAdd(P.ctr + op.grp_ctr + grp, 1) + 1 - (gen + 1) * need == 0;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  if (P.world > 1 && op.kind != SOP_GATEUP) {
    // push this rank's sums now; receive after the stream (see push_group)
    float v0, v1;
    sum_rows(op, 0, grp * 64 + 2 * lane, sc.nC, v0, v1);
    push_group(P, op.xchg, grp, v0, v1, lane, gen);
    if (lane == 0) {
      const int i = atomicAdd(&S.ndefer, 1);
      if (i < 64) S.defer[i] = grp;
      else raise_err(P, SPE_SLOT);
    }
    return;
  }
  finish_group(P, op, grp, lane, sc.nC, gen);
}

// ---------------------------------------------------------------- the kernel

template <int G>
__global__ void __launch_bounds__(SP_THREADS, 1) decode_step_kernel(const __grid_constant__ StepParams P) {
  extern __shared__ __align__(1024) unsigned char sp_smem[];
  __shared__ StepShared S;
  __shared__ __align__(16) uint4 s_zero[16];
  __shared__ float s_slot[SP_WIN][2][16][SP_NCW];
  __shared__ __align__(16) float s_q[G][128];  // rotated queries of one kv head
  __shared__ __align__(16) float s_knew[128], s_vnew[128];

  unsigned char* base = sp_smem + ((1024 - (smem_u32(sp_smem) & 1023)) & 1023);
  unsigned char* xs = base;                 // staged x of the current GEMV (or attention merge scratch)
  unsigned char* ring = base + P.xs_alloc;  // P.nst stages of SP_STAGE_BYTES
  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  const int n = gridDim.x, c = blockIdx.x;

  if (tid == 0) {
    for (int s = 0; s < P.nst; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], SP_NCW);
    }
    S.abort = 0;
    S.gen = *reinterpret_cast<volatile int*>(P.gen);
    S.pos = *reinterpret_cast<volatile int*>(P.pos);
    S.key = 0ull;
    fence_mbar_init();
  }
  if (tid < 16) s_zero[tid] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  const int gen = S.gen;
  const int pos = S.pos;
  const bool pos_ok = pos >= 0 && pos < P.Lmax && pos < P.max_pos;
  const int HD = P.hd;
  const int L = pos_ok ? pos + 1 : 0;         // keys this step attends to
  const long long TA = (long long)P.Hkv * L;  // attention units (head, key)
  const int na = (int)std::min<long long>(n, std::max<long long>(1, (TA + 63) / 64));  // attention CTAs
  const int AK = SP_STAGE_BYTES / (2 * HD * 4);                                       // keys per stage
  if (!pos_ok && tid == 0) raise_err(P, 1);

  if (warp == SP_NCW) {
    // ================================ producer ================================
    if (lane == 0) {
      const uint64_t pol = evict_first();
      uint32_t it = 0;
      bool ok = pos_ok;
      auto acquire = [&](int& s) -> unsigned char* {
        if (*reinterpret_cast<volatile int*>(&S.abort)) return nullptr;
        s = (int)(it % (uint32_t)P.nst);
        const uint32_t ph = (it / (uint32_t)P.nst) & 1u;
        if (!mbar_wait_bounded(&S.empty[s], ph ^ 1u, &S.abort, SP_WAIT_NS)) return nullptr;
        return ring + (size_t)s * SP_STAGE_BYTES;
      };
      for (int oi = 0; oi < P.nops && ok; ++oi) {
        const StepOp& op = P.ops[oi];
        if (op.kind == SOP_EMBED) continue;
        if (op.kind == SOP_ATTN) {
          if (c >= na) continue;
          const long long lo = range_lo(c, TA, na), hi = range_lo(c + 1, TA, na);
          for (long long u = lo; u < hi && ok;) {
            const int h = (int)(u / L);
            const long long seg_end = std::min<long long>(hi, (long long)(h + 1) * L);
            const int k0 = (int)(u - (long long)h * L), k1 = (int)(seg_end - (long long)h * L);
            for (int kt = k0; kt < k1; kt += AK) {
              int s;
              unsigned char* st = acquire(s);
              if (!st) {
                ok = false;
                break;
              }
              // cached keys only: the new one (position pos) comes from this step's q|k|v
              const int nk = std::min(AK, k1 - kt);
              const int nc = std::max(0, std::min(nk, pos - kt));
              const uint32_t bytes = (uint32_t)nc * HD * 4;
              mbar_arrive_expect_tx(&S.full[s], 2 * bytes);
              if (bytes) {
                bulk_load(st, op.kc + ((size_t)h * P.Lmax + kt) * HD, bytes, &S.full[s]);
                bulk_load(st + (size_t)AK * HD * 4, op.vc + ((size_t)h * P.Lmax + kt) * HD, bytes, &S.full[s]);
              }
              ++it;
            }
            u = seg_end;
          }
          continue;
        }
        // GEMV: this CTA's units, SP_STAGE_BOXES / nset per stage
        const int nC = gemv_ctas(op.total, op.kq, n);
        const long long lo = c < nC ? range_lo(c, op.total, nC) : 0, hi = c < nC ? range_lo(c + 1, op.total, nC) : 0;
        // one bulk copy per stage: the CTA's units are contiguous in the op's image
        const int qps = SP_STAGE_BOXES / op.nset;
        const size_t ubytes = (size_t)op.nset * SP_UNIT;
        for (long long u0 = lo; u0 < hi && ok; u0 += qps) {
          int s;
          unsigned char* st = acquire(s);
          if (!st) {
            ok = false;
            break;
          }
          const uint32_t bytes = (uint32_t)(std::min<long long>(qps, hi - u0) * ubytes);
          mbar_arrive_expect_tx(&S.full[s], bytes);
          bulk_load_hint(st, op.img + (size_t)u0 * ubytes, bytes, &S.full[s], pol);
          ++it;
        }
      }
      if (!ok) S.abort = 1;
      // let every copy already issued land before the CTA can exit
      for (uint32_t k = (it > (uint32_t)P.nst ? it - P.nst : 0); k < it; ++k) {
        int dummy = 0;
        mbar_wait_bounded(&S.full[k % P.nst], (k / P.nst) & 1u, (volatile int*)&dummy, SP_WAIT_NS / 4);
      }
    }
    return;
  }

  // ================================ consumers ================================
  const int g = lane >> 2, t = lane & 3;
  const int pr0 = sp_tile_row(g);
  // B-fragment column of this lane (batch 1, two groups per chunk): the hi or
  // lo part of group (g & 1); lanes of other columns read zeros
  const bool bact = g < 4 && (g & 1) == (t >> 1);
  const uint32_t bx_off = (uint32_t)(((((g >> 1) & 1) * 4) * 4 + t) * 16);
  const uint32_t zero_x = smem_u32(s_zero);
  const uint32_t xbase = smem_u32(xs);
  const uint32_t rbase = smem_u32(ring);
  int rs = 0;        // ring slot of the next stage (the producer's sequence, modulo the ring)
  uint32_t rph = 0;  // its mbarrier parity
  auto ring_next = [&]() {
    if (++rs == P.nst) {
      rs = 0;
      rph ^= 1u;
    }
  };
  volatile int* abort = &S.abort;
  if (!pos_ok) *abort = 1;

  auto cbar = [&]() { named_bar_sync(1, SP_NC); };
  // the CTA's abort flag as one decision for the whole warp (before shuffles / votes)
  auto wabort = [&]() -> bool { return __any_sync(0xffffffffu, *abort != 0); };

  auto stamp = [&](int oi, int k) {
    if (P.stamps && tid == 0) P.stamps[((size_t)c * P.nops + oi) * 4 + k] = globaltimer_ns();
  };
  for (int oi = 0; oi < P.nops; ++oi) {
    const StepOp& op = P.ops[oi];
    if (tid == 0) *reinterpret_cast<volatile int*>(P.progress + c) = oi;
    stamp(oi, 0);
    // ---------------------------------------------------------------- embedding
    if (op.kind == SOP_EMBED) {
      const int ng = P.H / 64;
      for (int gg = c + n * warp; gg < ng; gg += n * SP_NCW) {
        if (wabort()) break;
        const int tok = *reinterpret_cast<volatile int*>(P.tok);
        const int lt = tok - P.vocab_start;
        const bool own = lt >= 0 && lt < P.vocab_local;
        float v0 = 0.f, v1 = 0.f;
        const int k = gg * 64 + 2 * lane;
        if (own) {
          const uint32_t w = P.emb_w[(size_t)lt * (P.H / 8) + k / 8];
          const __half s = __ushort_as_half(P.emb_s[(size_t)lt * (P.H / 64) + gg]);
          const __half b = __ushort_as_half(P.emb_b[(size_t)lt * (P.H / 64) + gg]);
          const int sh = (k % 8) * 4;
          const __half q0 = __int2half_rn((int)((w >> sh) & 15u));
          const __half q1 = __int2half_rn((int)((w >> (sh + 4)) & 15u));
          v0 = __half2float(__hfma(q0, s, b));  // s*q + b rounded once, as mx.dequantize
          v1 = __half2float(__hfma(q1, s, b));
        }
        if (!xchg_group(P, op.xchg, gg, v0, v1, lane, gen)) {
          *abort = 1;
          break;
        }
        *reinterpret_cast<float2*>(op.h + k) = make_float2(v0, v1);
        if (op.trace) *reinterpret_cast<float2*>(op.trace + k) = make_float2(v0, v1);
        stage_group(op.out_xs, op.out_xss, op.out_norm, gg, v0, v1, lane);
        __syncwarp();
        __threadfence();
        if (lane == 0) atomicAdd(P.ctr + op.out_ctr, 1);
      }
      stamp(oi, 3);
      continue;
    }

    // ---------------------------------------------------------------- attention
    if (op.kind == SOP_ATTN) {
      if (c >= na) continue;
      const StepOp& qop = P.ops[oi - 1];  // this layer's q|k|v GEMV
      const int nQ = gemv_ctas(qop.total, qop.kq, n);
      const long long lo = range_lo(c, TA, na), hi = range_lo(c + 1, TA, na);
      if (tid == 0 && !*abort && !wait_ctr(P, P.ctr + qop.grp_ctr, (gen + 1) * qop.seg_need, SPE_QKV, oi)) *abort = 1;
      stamp(oi, 1);
      cbar();
      const int LPK = HD / 8, KPW = 32 / LPK;  // lanes per key, keys per warp
      const int sub = lane / LPK, dl = lane % LPK;
      const int d0 = dl * 8;
      int* hctr = P.attn_ctr + ((gen & 1) * P.nl + op.layer) * P.Hkv;
      for (long long u = lo; u < hi;) {
        const int h = (int)(u / L);
        const long long seg_end = std::min<long long>(hi, (long long)(h + 1) * L);
        const int k0 = (int)(u - (long long)h * L), k1 = (int)(seg_end - (long long)h * L);
        const bool has_new = pos >= k0 && pos < k1;
        // rotated queries of the G heads of kv head h, and the new key / value
        if (!*abort) {
          for (int e = tid; e < G * HD / 2; e += SP_NC) {
            const int gq = e / (HD / 2), d = e % (HD / 2);
            const int r = (h * G + gq) * HD + d;
            const float x1 = qkv_row(qop, r, nQ), x2 = qkv_row(qop, r + HD / 2, nQ);
            const float cs = P.cos_tab[(size_t)pos * (HD / 2) + d], sn = P.sin_tab[(size_t)pos * (HD / 2) + d];
            s_q[gq][d] = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(-x2, sn));
            s_q[gq][d + HD / 2] = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
          }
          if (has_new) {
            for (int e = tid; e < HD; e += SP_NC) {
              s_vnew[e] = qkv_row(qop, (P.Hq + P.Hkv + h) * HD + e, nQ);
              if (e < HD / 2) {
                const int rk = (P.Hq + h) * HD + e;
                const float x1 = qkv_row(qop, rk, nQ), x2 = qkv_row(qop, rk + HD / 2, nQ);
                const float cs = P.cos_tab[(size_t)pos * (HD / 2) + e], sn = P.sin_tab[(size_t)pos * (HD / 2) + e];
                s_knew[e] = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(-x2, sn));
                s_knew[e + HD / 2] = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
              }
            }
          }
        }
        cbar();
        if (has_new && !*abort)  // append the new key / value (fp32 cache)
          for (int e = tid; e < HD; e += SP_NC) {
            op.kc[((size_t)h * P.Lmax + pos) * HD + e] = s_knew[e];
            op.vc[((size_t)h * P.Lmax + pos) * HD + e] = s_vnew[e];
          }
        // per lane group (LPK lanes, 8 dims each): online softmax over its keys, for the G heads
        float m[G], l[G], o[G][8];
#pragma unroll
        for (int gq = 0; gq < G; ++gq) {
          m[gq] = -INFINITY;
          l[gq] = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) o[gq][i] = 0.f;
        }
        for (int kt = k0; kt < k1; kt += AK) {
          const int s = rs;
          const uint32_t ph = rph;
          ring_next();
          if (wabort() || !mbar_wait_all(P, &S.full[s], ph, abort, oi)) {
            *abort = 1;
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
            continue;
          }
          const float* tk = reinterpret_cast<const float*>(ring + (size_t)s * SP_STAGE_BYTES);
          const float* tv = tk + (size_t)AK * HD;
          const int nk = std::min(AK, k1 - kt);
          for (int kb = warp * KPW; kb < nk; kb += SP_NCW * KPW) {  // warp-uniform trip count
            const int kk = kb + sub;
            const bool valid = kk < nk;
            const int key = kt + kk;
            // scores of the G heads (K dead afterwards), then the V update
            float p[G], corr[G];
            {
              float4 ka = make_float4(0.f, 0.f, 0.f, 0.f), kb4 = ka;
              if (valid) {
                const float* kp = key == pos ? s_knew : tk + (size_t)kk * HD;
                ka = *reinterpret_cast<const float4*>(kp + d0);
                kb4 = *reinterpret_cast<const float4*>(kp + d0 + 4);
              }
#pragma unroll
              for (int gq = 0; gq < G; ++gq) {
                const float4 qa = *reinterpret_cast<const float4*>(&s_q[gq][d0]);
                const float4 qb = *reinterpret_cast<const float4*>(&s_q[gq][d0 + 4]);
                float dot = qa.x * ka.x;
                dot = fmaf(qa.y, ka.y, dot);
                dot = fmaf(qa.z, ka.z, dot);
                dot = fmaf(qa.w, ka.w, dot);
                dot = fmaf(qb.x, kb4.x, dot);
                dot = fmaf(qb.y, kb4.y, dot);
                dot = fmaf(qb.z, kb4.z, dot);
                dot = fmaf(qb.w, kb4.w, dot);
                for (int off = LPK / 2; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
                const float sc = dot * P.scale;
                const float mn = valid ? fmaxf(m[gq], sc) : m[gq];
                corr[gq] = valid ? expf(m[gq] - mn) : 1.f;
                p[gq] = valid ? expf(sc - mn) : 0.f;
                l[gq] = l[gq] * corr[gq] + p[gq];
                m[gq] = mn;
              }
            }
            if (valid) {
              const float* vp = key == pos ? s_vnew : tv + (size_t)kk * HD;
              const float4 va = *reinterpret_cast<const float4*>(vp + d0);
              const float4 vb = *reinterpret_cast<const float4*>(vp + d0 + 4);
              const float vf[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
              for (int gq = 0; gq < G; ++gq)
#pragma unroll
                for (int i = 0; i < 8; ++i) o[gq][i] = fmaf(p[gq], vf[i], o[gq][i] * corr[gq]);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.empty[s]);
        }
        // merge the lane groups of a warp (xor over the key index), then the warps in order
        for (int off = LPK; off < 32; off <<= 1) {
#pragma unroll
          for (int gq = 0; gq < G; ++gq) {
            const float mo = __shfl_xor_sync(0xffffffffu, m[gq], off);
            const float lo2 = __shfl_xor_sync(0xffffffffu, l[gq], off);
            const float mn = fmaxf(m[gq], mo);
            const float ca = m[gq] == -INFINITY ? 0.f : expf(m[gq] - mn);
            const float cb = mo == -INFINITY ? 0.f : expf(mo - mn);
            l[gq] = l[gq] * ca + lo2 * cb;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float oo = __shfl_xor_sync(0xffffffffu, o[gq][i], off);
              o[gq][i] = o[gq][i] * ca + oo * cb;
            }
            m[gq] = mn;
          }
        }
        float* mscr = reinterpret_cast<float*>(xs);  // [SP_NCW][G][HD + 4]: {m, l, -, -, o[HD]}
        if (sub == 0) {
#pragma unroll
          for (int gq = 0; gq < G; ++gq) {
            float* pw = mscr + ((size_t)warp * G + gq) * (HD + 4);
            if (dl == 0) {
              pw[0] = m[gq];
              pw[1] = l[gq];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) pw[4 + d0 + i] = o[gq][i];
          }
        }
        cbar();
        // this CTA's segment partial of head h
        const int s_first = owner_of((long long)h * L, TA, na);
        const int nsh = owner_of((long long)(h + 1) * L - 1, TA, na) - s_first + 1;
        float* hp = P.attn_part + (((size_t)op.layer * P.Hkv + h) * n) * G * (HD + 4);
        float* pseg = hp + (size_t)(c - s_first) * G * (HD + 4);
        if (!*abort)
          for (int e = tid; e < G * HD; e += SP_NC) {
            const int gq = e / HD, d = e % HD;
            float M = -INFINITY;
            for (int w = 0; w < SP_NCW; ++w) M = fmaxf(M, mscr[((size_t)w * G + gq) * (HD + 4)]);
            float Ls = 0.f, O = 0.f;
            if (M != -INFINITY)
              for (int w = 0; w < SP_NCW; ++w) {
                const float* pw = mscr + ((size_t)w * G + gq) * (HD + 4);
                const float wgt = pw[0] == -INFINITY ? 0.f : expf(pw[0] - M);
                Ls = fmaf(pw[1], wgt, Ls);
                O = fmaf(pw[4 + d], wgt, O);
              }
            float* pp = pseg + (size_t)gq * (HD + 4);
            pp[4 + d] = O;
            if (d == 0) {
              pp[0] = M;
              pp[1] = Ls;
            }
          }
        __threadfence();
        cbar();
        // the last segment of head h merges the head and stages o_proj's input:
        // one warp per 64-value group, the segments' partials loaded 8 at a time
        if (tid == 0) S.attn_last = !*abort && atomicAdd(hctr + h, 1) + 1 == nsh;
        cbar();
        if (S.attn_last) {
          __threadfence();
          for (int grp = warp; grp < G * (HD / 64); grp += SP_NCW) {
            const int gq = grp / (HD / 64), gg = grp % (HD / 64);
            const float* hg = hp + (size_t)gq * (HD + 4);
            const size_t js = (size_t)G * (HD + 4);  // stride between segments
            float M = -INFINITY;
            for (int j = lane; j < nsh; j += 32) M = fmaxf(M, ldcg_f(hg + j * js));
#pragma unroll
            for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
            float Ls = 0.f;
            for (int j = lane; j < nsh; j += 32) {
              const float mj = ldcg_f(hg + j * js);
              Ls += mj == -INFINITY ? 0.f : ldcg_f(hg + j * js + 1) * expf(mj - M);
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, off);
            const int d = gg * 64 + 2 * lane;
            float O0 = 0.f, O1 = 0.f;
            for (int j0 = 0; j0 < nsh; j0 += 8) {
              float mj[8];
              float2 oj[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const int j = std::min(j0 + q, nsh - 1);
                mj[q] = ldcg_f(hg + j * js);
                oj[q] = __ldcg(reinterpret_cast<const float2*>(hg + j * js + 4 + d));
              }
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float wgt = (j0 + q >= nsh || mj[q] == -INFINITY) ? 0.f : expf(mj[q] - M);
                O0 = fmaf(oj[q].x, wgt, O0);
                O1 = fmaf(oj[q].y, wgt, O1);
              }
            }
            const float inv = 1.f / Ls;
            stage_group(op.out_xs, nullptr, nullptr, ((h * G + gq) * HD + gg * 64) / 64, O0 * inv, O1 * inv, lane);
            __syncwarp();
            __threadfence();
            if (lane == 0) atomicAdd(P.ctr + op.out_ctr, 1);
          }
        }
        cbar();
        u = seg_end;
      }
      stamp(oi, 3);
      continue;
    }

    // ---------------------------------------------------------------- GEMV
    const int nC = gemv_ctas(op.total, op.kq, n);
    const long long lo = c < nC ? range_lo(c, op.total, nC) : 0, hi = c < nC ? range_lo(c + 1, op.total, nC) : 0;
    if (lo < hi) {
      // input complete, then staged into shared memory (plain loads: the
      // finishing CTAs wrote it with plain stores, released by their counters)
      if (tid == 0) {
        if (!*abort && !wait_ctr(P, P.ctr + op.x_ctr, (gen + 1) * op.x_need, SPE_INPUT, oi)) *abort = 1;
        stamp(oi, 1);
        for (int i = 0; i < SP_WIN; ++i) {
          S.cnt[i] = 0;
          S.free_at[i] = i;
        }
        S.ndefer = 0;
      }
      cbar();
      if (!wabort()) {
        for (int i = tid; i < op.xs_bytes / 16; i += SP_NC)
          reinterpret_cast<uint4*>(xs)[i] = ldcg_v4(op.xs + (size_t)i * 16);
        if (warp == 0) {
          float rinv = 1.f;
          if (op.xss) {
            float ss = 0.f;
            for (int i = lane; i < op.K / 64; i += 32) ss += ldcg_f(op.xss + i);
#pragma unroll
            for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            rinv = 1.f / sqrtf(ss / (float)op.K + P.eps);
          }
          if (lane == 0) S.rinv = rinv;
        }
      }
      cbar();
      const float rinv = S.rinv;
      const int kq = op.kq;
      const int t_first = (int)(lo / kq);
      const int lo_r = (int)(lo % kq);  // unit of the first chunk within its tile row
      const int nchi = (int)((hi - lo) * SP_BOX_CH);  // chunks of this CTA
      SegCtx sc{lo, hi, t_first, kq, nC, rinv};

      float acc[2][4];
      int cur = -1;  // this warp's current segment (tile - t_first)
      // this warp's partial of segment j into its output slot; the last warp
      // holding a piece of the segment runs the segment epilogue
      auto flush = [&](int j, int nset) {
        const int slot = j % SP_WIN;
        // the slot must have been released by segment j - SP_WIN's epilogue (lane 0 waits)
        int freed = 1;
        if (lane == 0 && *reinterpret_cast<volatile int*>(&S.free_at[slot]) != j) {
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t i = 1; *reinterpret_cast<volatile int*>(&S.free_at[slot]) != j; ++i)
            if ((i & 63) == 0 && (*abort || err_set(P) || globaltimer_ns() - t0 > SP_WAIT_NS)) {
              if (!*abort && !err_set(P)) raise_err(P, SPE_SLOT);
              *abort = 1;
              freed = 0;
              break;
            }
        }
        if (!__shfl_sync(0xffffffffu, freed, 0)) return;
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          if (a >= nset) break;
          float vg = acc[a][0] + acc[a][1], vg8 = acc[a][2] + acc[a][3];
          vg += __shfl_xor_sync(0xffffffffu, vg, 1);  // hi + lo columns (lanes t = 0, 1)
          vg8 += __shfl_xor_sync(0xffffffffu, vg8, 1);
          if (t == 0) {
            s_slot[slot][a][pr0][warp] = vg;
            s_slot[slot][a][pr0 + 8][warp] = vg8;
          }
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          __threadfence_block();
          last = atomicAdd(&S.cnt[slot], 1) + 1 == __popc(seg_warps(sc, j));
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence_block();
          seg_epilogue(P, op, S, s_slot, sc, j, c, gen, lane);
        }
      };

      // per-lane shared-memory offsets of chunk cc of box b
      auto wofs = [&](int b, int cc) -> uint32_t {
        const int uu = ((cc & 1) << 2) | t;
        return (uint32_t)(b * SP_UNIT + (cc >> 1) * 2048 + pr0 * 128 + ((uu ^ (pr0 & 7)) << 4));
      };
      auto sofs = [&](int b, int cc) -> uint32_t { return (uint32_t)(b * SP_UNIT + SP_WBOX + pr0 * 16 + cc * 4); };

      // The stream: NS weight sets; a warp takes chunk slots w (+ SP_NCW for
      // one set) of every stage, loads the ring's part of them into
      // registers, releases the slot, then computes.  Each slot's segment
      // (tile row) and unit within the row advance by a stage's units per
      // stage, tracked incrementally.
      auto run = [&](auto nset_tag) {
        constexpr int NS = decltype(nset_tag)::value;
        constexpr int NK = NS == 1 ? 2 : 1;              // chunk slots per warp per stage
        constexpr int QPS = SP_STAGE_BOXES / NS;         // units per stage
        constexpr int CPS = QPS * SP_BOX_CH;             // chunk slots per stage
        const int nstage = (int)((hi - lo + QPS - 1) / QPS);
        int jk[NK], mk[NK];  // per slot: segment, unit within the tile row
#pragma unroll
        for (int k = 0; k < NK; ++k) {
          const int ub = lo_r + (warp + SP_NCW * k) / SP_BOX_CH;
          jk[k] = ub / kq;
          mk[k] = ub - jk[k] * kq;
        }
        for (int sidx = 0; sidx < nstage; ++sidx) {
          const int s = rs;
          const uint32_t ph = rph;
          ring_next();
          if (wabort() || !mbar_wait_all(P, &S.full[s], ph, abort, oi)) {
            *abort = 1;
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
            continue;
          }
          const uint32_t st = rbase + (uint32_t)s * SP_STAGE_BYTES;
          // the ring's part of this warp's chunks (words, scales, biases) into registers
          uint4 W0[NK][NS], W1[NK][NS];  // words of rows g, g + 8
          uint32_t SB[NK][NS][4];        // scales g, g + 8, biases g, g + 8 (two groups each)
#pragma unroll
          for (int k = 0; k < NK; ++k) {
            const int slotc = warp + SP_NCW * k;
            if (sidx * CPS + slotc < nchi) {
              const int bq = slotc / SP_BOX_CH, cc = slotc % SP_BOX_CH;
#pragma unroll
              for (int a = 0; a < NS; ++a) {
                const int b = bq * NS + a;
                const uint32_t wo = st + wofs(b, cc), so = st + sofs(b, cc);
                W0[k][a] = lds_v4(wo);
                W1[k][a] = lds_v4(wo + 1024);
                SB[k][a][0] = lds_u32(so);
                SB[k][a][1] = lds_u32(so + 128);
                SB[k][a][2] = lds_u32(so + SP_SBOX);
                SB[k][a][3] = lds_u32(so + SP_SBOX + 128);
              }
            }
          }
          // every read of the stage is in registers: hand the slot back to the producer
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.empty[s]);
#pragma unroll
          for (int k = 0; k < NK; ++k) {
            const int slotc = warp + SP_NCW * k;
            if (sidx * CPS + slotc >= nchi) break;
            const int j = jk[k];                                    // segment (tile - t_first)
            const int kc = mk[k] * SP_BOX_CH + (slotc % SP_BOX_CH);  // chunk along K
            if (j != cur) {
              if (cur >= 0) flush(cur, NS);
              cur = j;
#pragma unroll
              for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[a][r] = 0.f;
            }
            // this chunk's B fragments (one 16-byte unit per mma pair) and column sums
            const uint32_t xo = bact ? xbase + (uint32_t)kc * SP_CB + bx_off : zero_x;
            const float4 TB = lds_f4(xbase + (uint32_t)kc * SP_CB + 512 + t * 16);
            float ca[NS][4], cz[NS][4];
#pragma unroll
            for (int a = 0; a < NS; ++a) {
              ca[a][0] = TB.x;
              ca[a][1] = TB.y;
              ca[a][2] = TB.x;
              ca[a][3] = TB.y;
              cz[a][0] = cz[a][1] = cz[a][2] = cz[a][3] = 0.f;
            }
#pragma unroll
            for (int jw = 0; jw < 4; ++jw) {
              const uint4 xb = lds_v4(xo + (bact ? jw * 64 : 0));
#pragma unroll
              for (int a = 0; a < NS; ++a) {
                const uint32_t r0 = jw == 0 ? W0[k][a].x : jw == 1 ? W0[k][a].y : jw == 2 ? W0[k][a].z : W0[k][a].w;
                const uint32_t r1 = jw == 0 ? W1[k][a].x : jw == 1 ? W1[k][a].y : jw == 2 ? W1[k][a].z : W1[k][a].w;
                const uint32_t w8a = r0 >> 8, w8b = r1 >> 8;
                mma_16816(ca[a], mag<0x000F000Fu>(r0), mag<0x000F000Fu>(r1), mag<0x00F000F0u>(r0),
                          mag<0x00F000F0u>(r1), xb.x, xb.y);
                mma_16816(cz[a], mag<0x000F000Fu>(w8a), mag<0x000F000Fu>(w8b), mag<0x00F000F0u>(w8a),
                          mag<0x00F000F0u>(w8b), xb.z, xb.w);
              }
            }
#pragma unroll
            for (int a = 0; a < NS; ++a) {
              const __half2 s0 = u32_as_h2(SB[k][a][0]), s1 = u32_as_h2(SB[k][a][1]);
              const __half2 b0 = u32_as_h2(SB[k][a][2]), b1 = u32_as_h2(SB[k][a][3]);
              acc[a][0] = fmaf(__low2float(s0), ca[a][0] + cz[a][0], fmaf(__low2float(b0), TB.z, acc[a][0]));
              acc[a][1] = fmaf(__high2float(s0), ca[a][1] + cz[a][1], fmaf(__high2float(b0), TB.w, acc[a][1]));
              acc[a][2] = fmaf(__low2float(s1), ca[a][2] + cz[a][2], fmaf(__low2float(b1), TB.z, acc[a][2]));
              acc[a][3] = fmaf(__high2float(s1), ca[a][3] + cz[a][3], fmaf(__high2float(b1), TB.w, acc[a][3]));
            }
          }
#pragma unroll
          for (int k = 0; k < NK; ++k) {
            mk[k] += QPS;
            while (mk[k] >= kq) {
              mk[k] -= kq;
              ++jk[k];
            }
          }
        }
        if (cur >= 0 && !wabort()) flush(cur, NS);
      };
      if (op.nset == 2)
        run(std::integral_constant<int, 2>{});
      else
        run(std::integral_constant<int, 1>{});
      cbar();  // every warp is done with xs and the slots
      stamp(oi, 2);
      // row-op groups completed here: the peers' partials, then the residual and the next input
      const int nd = std::min(S.ndefer, 64);
      for (int i = warp; i < nd && !wabort(); i += SP_NCW) {
        const int grp = S.defer[i];
        float v[2];
        sum_rows(op, 0, grp * 64 + 2 * lane, nC, v[0], v[1]);
        if (!recv_group(P, op.xchg, grp, v[0], v[1], lane, gen)) {
          *abort = 1;
          break;
        }
        finish_group(P, op, grp, lane, nC, gen, v);
      }
    }
    if (op.kind == SOP_HEAD && tid == 0) {
      // this CTA's candidate joins the global argmax; the last CTA publishes the token
      if (!*abort) atomicMax(P.key + (gen & 1), S.key);
      __threadfence();
      const int old = atomicAdd(P.head_done, 1);
      if (old + 1 - (gen + 1) * n == 0) {
        __threadfence();
        unsigned long long k = atomicAdd(P.key + (gen & 1), 0ull);
        if (P.world > 1 && !err_set(P)) {
          const uint32_t ep = ((uint32_t)(gen + 1) << 8) | 0xffu;
          const int slot2 = gen & 1;
          for (int q = 1; q < P.world; ++q) {
            const int dst = (P.rank + q) % P.world;
            char* lb = P.arena[dst] + P.key_off + ((size_t)slot2 * P.world + P.rank) * 16;
            st_v4_volatile(lb, (uint32_t)k, ep, (uint32_t)(k >> 32), ep);
          }
          for (int q = 0; q < P.world; ++q) {
            if (q == P.rank) continue;
            const char* lb = P.arena[P.rank] + P.key_off + ((size_t)slot2 * P.world + q) * 16;
            uint4 l = ld_v4_volatile(lb);
            const uint64_t t0 = globaltimer_ns();
            bool got = true;
            while (l.y != ep || l.w != ep) {
              if (globaltimer_ns() - t0 > SP_WAIT_NS || err_set(P)) {
                raise_err(P, SPE_ARGMAX);
                got = false;
                break;
              }
              l = ld_v4_volatile(lb);
            }
            if (got) {
              const unsigned long long kq2 = ((unsigned long long)l.z << 32) | l.x;
              k = kq2 > k ? kq2 : k;
            }
          }
        }
        if (!err_set(P)) {
          *reinterpret_cast<volatile int*>(P.tok) = key_index(k);
          *reinterpret_cast<volatile int*>(P.pos) = pos + 1;
        }
        // next step's bookkeeping: its argmax slot and attention counters start at zero
        P.key[(gen + 1) & 1] = 0ull;
        int* next_attn = P.attn_ctr + ((gen + 1) & 1) * P.nl * P.Hkv;
        for (int i = 0; i < P.nl * P.Hkv; ++i) next_attn[i] = 0;
        __threadfence();
        atomicAdd(P.gen, 1);
      }
    }
    stamp(oi, 3);
  }
  // (after an error the record keeps the op each CTA gave up in)
  if (tid == 0 && !err_set(P)) *reinterpret_cast<volatile int*>(P.progress + c) = P.nops;
}

// ---------------------------------------------------------------- host side

struct StepLayer {
  const uint16_t* ln1 = nullptr;
  const uint16_t* ln2 = nullptr;
  const uint32_t* w[7] = {};
  const uint16_t* s[7] = {};
  const uint16_t* b[7] = {};
  float* kc = nullptr;
  float* vc = nullptr;
};

struct StepPlan {
  int H, Hq, Hkv, hd, F, Vl, v0, nl, Lmax, world, rank, nsm, device;
  float eps;
  std::vector<StepLayer> layers;
  const uint32_t* emb_w = nullptr;
  const uint16_t* emb_s = nullptr;
  const uint16_t* emb_b = nullptr;
  const uint16_t* fnorm = nullptr;
  int* tok = nullptr;
  int* pos = nullptr;
  const float* cos_tab = nullptr;
  const float* sin_tab = nullptr;
  int max_pos = 0;
  float* trace = nullptr;
  float* logits = nullptr;
  unsigned long long* stamps = nullptr;
  char* arena[SP_MAX_WORLD] = {};
  size_t arena_bytes = 0;
  bool ready = false;
  StepParams P{};
  size_t smem = 0;
  int G = 1;
  int grid = 0;      // CTAs per step: every SM, as far as one CTA fits on each
  int fit[6] = {};   // SMs, CTAs per SM, static smem, dynamic smem, registers, max threads per block
};

// ---------------------------------------------------------------- weight images
//
// Each GEMV op streams its weights from an image written once at finalize:
// unit u (16 rows x 512 k of tile u / kq, block u % kq) of set a sits at
// (u * nset + a) * SP_UNIT, holding the unit's packed words in the order the
// consumers read them from shared memory (two 256-k halves of 16 rows x 128
// bytes, the 16-byte pieces of row r permuted by XOR with r & 7 so the
// fragment loads are bank-conflict free), then its 16 x 8 scales and 16 x 8
// biases.  A CTA's run of units is one contiguous range, so a ring stage is
// one bulk copy.  Rows past the tensor and k past K are zero (a zero scale
// and bias contribute nothing).

struct PackOp {
  const uint32_t* w[SP_MAX_SEG];  // tensors stacked along N (q | k | v), or the gate, up pair
  const uint16_t* s[SP_MAX_SEG];
  const uint16_t* b[SP_MAX_SEG];
  int rows[SP_MAX_SEG];
  int seg_tiles[SP_MAX_SEG];
  int nseg, nset, K, kq, tiles;
  unsigned char* img;
};

__global__ void step_pack_kernel(const PackOp po) {
  constexpr int P16 = SP_UNIT / 16;  // 16-byte pieces per unit
  const long long n16 = (long long)po.tiles * po.kq * po.nset * P16;
  const int KW = po.K / 8, KG = po.K / 64;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x) {
    const long long us = i / P16;
    const int o16 = (int)(i % P16);
    const long long u = us / po.nset;
    const int a = (int)(us % po.nset);
    const int t = (int)(u / po.kq), kb = (int)(u % po.kq);
    int seg = 0, row0 = t * 16;
    while (seg + 1 < po.nseg && row0 >= po.seg_tiles[seg] * 16) {
      row0 -= po.seg_tiles[seg] * 16;
      ++seg;
    }
    const int ti = po.nset == 2 ? a : seg;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (o16 < SP_WBOX / 16) {
      const int zb = o16 >> 7, r = (o16 >> 3) & 15, piece = (o16 & 7) ^ (r & 7);
      const int row = row0 + r, w0 = (kb * 2 + zb) * 32 + piece * 4;
      if (row < po.rows[ti] && w0 < KW) v = *reinterpret_cast<const uint4*>(po.w[ti] + (size_t)row * KW + w0);
    } else {
      const int q = o16 - SP_WBOX / 16, r = q & 15;
      const uint16_t* src = q >= 16 ? po.b[ti] : po.s[ti];
      const int row = row0 + r;
      uint32_t hw[4] = {0u, 0u, 0u, 0u};
      if (row < po.rows[ti])
        for (int g = 0; g < 8; ++g) {
          const int gi = kb * 8 + g;
          if (gi < KG) hw[g >> 1] |= (uint32_t)src[(size_t)row * KG + gi] << (16 * (g & 1));
        }
      v = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
    reinterpret_cast<uint4*>(po.img)[i] = v;
  }
}

static size_t image_bytes(int rows, int K, int nset) {
  return (size_t)((rows + 15) / 16) * ((K + SP_BOX_K - 1) / SP_BOX_K) * nset * SP_UNIT;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
static int kq_of(int K) { return (K + SP_BOX_K - 1) / SP_BOX_K; }
static int staged_bytes(int K) { return kq_of(K) * SP_BOX_CH * SP_CB; }

struct StepLayout {
  size_t ops, ctr, part_qkv, part_o, part_gu, part_down, part_head, attn_part, xs_h, xss_h, xs_o, xs_gu,
      xss_gu, xs_down, h, img, total;
  size_t img_layer;             // weight-image bytes of one layer
  size_t img_off[4], img_head;  // q|k|v, o, gate|up, down within a layer; the head after the layers
  size_t progress;
  int nctr, nops, max_groups;
  int ctr_x, ctr_grp, ctr_head_tile, ctr_attn, ctr_misc;
  int xs_bytes_h, xs_bytes_o, xs_bytes_down;
};

static StepLayout step_layout(const StepPlan& p) {
  StepLayout L{};
  const int nl = p.nl;
  L.nops = 1 + 5 * nl + 1;
  const int qkvN = (p.Hq + 2 * p.Hkv) * p.hd;
  const int G = p.Hq / p.Hkv;
  L.xs_bytes_h = staged_bytes(p.H);
  L.xs_bytes_o = staged_bytes(p.Hq * p.hd);
  L.xs_bytes_down = staged_bytes(p.F);
  L.max_groups = std::max({p.H / 64, p.F / 64, 1});
  L.ctr_x = 0;
  L.ctr_grp = L.nops;
  L.ctr_head_tile = L.ctr_grp + L.nops * L.max_groups;
  L.ctr_attn = L.ctr_head_tile + (p.Vl + 15) / 16;
  L.ctr_misc = (L.ctr_attn + 2 * nl * p.Hkv + 1) / 2 * 2;  // even: the 8-byte keys follow
  L.nctr = L.ctr_misc + 16;  // gen, err, head_done, -, keys[2], -, -, info[8]
  size_t o = 0;
  L.ops = o;
  o = align_up(o + sizeof(StepOp) * L.nops, 128);
  L.ctr = o;
  o = align_up(o + sizeof(int) * L.nctr, 128);
  L.progress = o;
  o = align_up(o + sizeof(int) * p.nsm, 128);
  auto part = [&](int rows, int nset) {
    return align_up(sizeof(float) * (size_t)((rows + 15) / 16) * SP_MAXT * nset * 16, 128);
  };
  L.part_qkv = o;
  o += part(qkvN, 1);
  L.part_o = o;
  o += part(p.H, 1);
  L.part_gu = o;
  o += part(p.F, 2);
  L.part_down = o;
  o += part(p.H, 1);
  L.part_head = o;
  o += part(p.Vl, 1);
  L.attn_part = o;
  o = align_up(o + sizeof(float) * (size_t)nl * p.Hkv * p.nsm * G * (p.hd + 4), 128);
  L.xs_h = o;
  o = align_up(o + L.xs_bytes_h, 128);
  L.xss_h = o;
  o = align_up(o + sizeof(float) * (p.H / 64), 128);
  L.xs_o = o;
  o = align_up(o + L.xs_bytes_o, 128);
  L.xs_gu = o;
  o = align_up(o + L.xs_bytes_h, 128);
  L.xss_gu = o;
  o = align_up(o + sizeof(float) * (p.H / 64), 128);
  L.xs_down = o;
  o = align_up(o + L.xs_bytes_down, 128);
  L.h = o;
  o = align_up(o + sizeof(float) * p.H, 128);
  L.img = o = align_up(o, 1024);
  L.img_off[0] = 0;
  L.img_off[1] = L.img_off[0] + image_bytes(qkvN, p.H, 1);
  L.img_off[2] = L.img_off[1] + image_bytes(p.H, p.Hq * p.hd, 1);
  L.img_off[3] = L.img_off[2] + image_bytes(p.F, p.H, 2);
  L.img_layer = L.img_off[3] + image_bytes(p.H, p.F, 1);
  L.img_head = L.img_layer * nl;
  o += L.img_head + image_bytes(p.Vl, p.H, 1);
  L.total = align_up(o, 128);
  return L;
}

template <int G>
static cudaError_t launch_step(const StepPlan* p, cudaStream_t stream) {
  auto kern = decode_step_kernel<G>;
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p->smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p->grid);
  cfg.blockDim = dim3(SP_THREADS);
  cfg.dynamicSmemBytes = p->smem;
  cfg.stream = stream;
  // Every CTA waits on others: all must be resident at once.  Outside a graph
  // capture the launch is cooperative (the driver refuses it if they cannot
  // all be); inside one it is a plain launch of one CTA per SM, the kernel's
  // shared memory admitting no second CTA, and every wait in it is bounded.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream, &cs);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cs == cudaStreamCaptureStatusNone ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p->P);
}

template <int G>
static size_t step_static_smem() {
  cudaFuncAttributes fa{};
  cudaFuncGetAttributes(&fa, decode_step_kernel<G>);
  return fa.sharedSizeBytes;
}

template <int G>
static void step_fit(size_t dyn, int* blocks, cudaFuncAttributes* fa) {
  cudaFuncSetAttribute(decode_step_kernel<G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  cudaFuncSetAttribute(decode_step_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, decode_step_kernel<G>, SP_THREADS, dyn);
  cudaFuncGetAttributes(fa, decode_step_kernel<G>);
}

static void fit_of(int G, size_t dyn, int* blocks, cudaFuncAttributes* fa) {
  switch (G) {
    case 1: step_fit<1>(dyn, blocks, fa); break;
    case 2: step_fit<2>(dyn, blocks, fa); break;
    case 4: step_fit<4>(dyn, blocks, fa); break;
    default: step_fit<8>(dyn, blocks, fa); break;
  }
}

static size_t static_smem_of(int G) {
  switch (G) {
    case 1: return step_static_smem<1>();
    case 2: return step_static_smem<2>();
    case 4: return step_static_smem<4>();
    default: return step_static_smem<8>();
  }
}

}  // namespace sc

extern "C" {

int sc_step_create(int hidden, int heads, int kv_heads, int head_dim, int ffn, int vocab_local, int vocab_start,
                   int layers, int bits, int group, float eps, int max_seq, int world, int rank, void** step) {
  using namespace sc;
  SC_REQUIRE(step, SC_ERR_ARG, "step_create: null handle pointer");
  *step = nullptr;
  SC_REQUIRE(bits == 4 && group == 64, SC_ERR_UNSUPPORTED,
             "step_create: the persistent decode step covers 4-bit group-64 weights (got %d-bit g%d)", bits, group);
  SC_REQUIRE(hidden > 0 && heads > 0 && kv_heads > 0 && heads % kv_heads == 0 && layers > 0 && max_seq > 0,
             SC_ERR_SHAPE, "step_create: bad model shape");
  SC_REQUIRE(head_dim == 64 || head_dim == 128, SC_ERR_UNSUPPORTED, "step_create: head_dim %d (64 or 128)",
             head_dim);
  const int G = heads / kv_heads;
  SC_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, SC_ERR_UNSUPPORTED, "step_create: GQA group %d (1, 2, 4, 8)", G);
  SC_REQUIRE(hidden % 512 == 0 && ffn % 256 == 0 && ffn >= 512 && (heads * head_dim) % 512 == 0, SC_ERR_UNSUPPORTED,
             "step_create: hidden and heads*head_dim must be multiples of 512, ffn of 256 (>= 512)");
  SC_REQUIRE(vocab_local > 0 && (kv_heads * head_dim) % 16 == 0, SC_ERR_SHAPE, "step_create: bad vocab / kv shape");
  SC_REQUIRE(world >= 1 && world <= SP_MAX_WORLD && rank >= 0 && rank < world, SC_ERR_SHAPE,
             "step_create: rank %d of world %d", rank, world);
  StepPlan* p = new StepPlan();
  p->H = hidden;
  p->Hq = heads;
  p->Hkv = kv_heads;
  p->hd = head_dim;
  p->F = ffn;
  p->Vl = vocab_local;
  p->v0 = vocab_start;
  p->nl = layers;
  p->eps = eps;
  p->Lmax = max_seq;
  p->world = world;
  p->rank = rank;
  p->nsm = sm_count();
  p->G = G;
  cudaGetDevice(&p->device);
  p->layers.resize(layers);
  *step = p;
  return SC_OK;
}

int sc_step_set_layer(void* step, int layer, const uint16_t* ln1, const uint16_t* ln2, const uint32_t* const* wq,
                      const uint16_t* const* scales, const uint16_t* const* biases, float* k_cache, float* v_cache) {
  using namespace sc;
  SC_REQUIRE(step && wq && scales && biases && ln1 && ln2 && k_cache && v_cache, SC_ERR_ARG,
             "step_set_layer: null pointer");
  StepPlan* p = static_cast<StepPlan*>(step);
  SC_REQUIRE(layer >= 0 && layer < p->nl, SC_ERR_SHAPE, "step_set_layer: layer %d of %d", layer, p->nl);
  StepLayer& L = p->layers[layer];
  L.ln1 = ln1;
  L.ln2 = ln2;
  for (int i = 0; i < 7; ++i) {
    SC_REQUIRE(wq[i] && scales[i] && biases[i], SC_ERR_ARG, "step_set_layer: null weight %d", i);
    SC_REQUIRE(((uintptr_t)wq[i] | (uintptr_t)scales[i] | (uintptr_t)biases[i]) % 16 == 0, SC_ERR_ARG,
               "step_set_layer: weight %d not 16-byte aligned", i);
    L.w[i] = wq[i];
    L.s[i] = scales[i];
    L.b[i] = biases[i];
  }
  L.kc = k_cache;
  L.vc = v_cache;
  p->ready = false;
  return SC_OK;
}

int sc_step_set_head(void* step, const uint32_t* embed_wq, const uint16_t* embed_scales,
                     const uint16_t* embed_biases, const uint16_t* final_norm) {
  using namespace sc;
  SC_REQUIRE(step && embed_wq && embed_scales && embed_biases && final_norm, SC_ERR_ARG,
             "step_set_head: null pointer");
  StepPlan* p = static_cast<StepPlan*>(step);
  SC_REQUIRE(((uintptr_t)embed_wq | (uintptr_t)embed_scales | (uintptr_t)embed_biases) % 16 == 0, SC_ERR_ARG,
             "step_set_head: embedding not 16-byte aligned");
  p->emb_w = embed_wq;
  p->emb_s = embed_scales;
  p->emb_b = embed_biases;
  p->fnorm = final_norm;
  p->ready = false;
  return SC_OK;
}

int sc_step_set_io(void* step, int32_t* tok, int32_t* pos, const float* cos_tab, const float* sin_tab, int max_pos,
                   float* trace, float* logits) {
  using namespace sc;
  SC_REQUIRE(step && tok && pos && cos_tab && sin_tab, SC_ERR_ARG, "step_set_io: null pointer");
  StepPlan* p = static_cast<StepPlan*>(step);
  p->tok = tok;
  p->pos = pos;
  p->cos_tab = cos_tab;
  p->sin_tab = sin_tab;
  p->max_pos = max_pos;
  p->trace = trace;
  p->logits = logits;
  p->ready = false;
  return SC_OK;
}

int sc_step_set_timing(void* step, unsigned long long* stamps) {
  using namespace sc;
  SC_REQUIRE(step, SC_ERR_ARG, "step_set_timing: null handle");
  StepPlan* p = static_cast<StepPlan*>(step);
  p->stamps = stamps;
  p->P.stamps = stamps;  // launches after this call (a captured graph keeps what it captured)
  return SC_OK;
}

size_t sc_step_timing_count(void* step) {
  if (!step) return 0;
  const sc::StepPlan* p = static_cast<const sc::StepPlan*>(step);
  return (size_t)p->nsm * (2 + 5 * (size_t)p->nl) * 4;
}

size_t sc_step_arena_bytes(int hidden, int world) {
  return sc::SP_ARENA_HDR + 2 * (size_t)world * (size_t)hidden / 2 * 16 + 2 * (size_t)world * 16;
}

int sc_step_set_peers(void* step, void* const* arenas, size_t arena_bytes) {
  using namespace sc;
  SC_REQUIRE(step && arenas, SC_ERR_ARG, "step_set_peers: null pointer");
  StepPlan* p = static_cast<StepPlan*>(step);
  const size_t need = sc_step_arena_bytes(p->H, p->world);
  SC_REQUIRE(arena_bytes >= need, SC_ERR_WORKSPACE, "step_set_peers: arenas of %zu bytes, %zu needed", arena_bytes,
             need);
  for (int q = 0; q < p->world; ++q) {
    SC_REQUIRE(arenas[q], SC_ERR_ARG, "step_set_peers: null arena of rank %d", q);
    p->arena[q] = static_cast<char*>(arenas[q]);
  }
  p->arena_bytes = arena_bytes;
  p->ready = false;
  return SC_OK;
}

size_t sc_step_workspace_bytes(void* step) {
  if (!step) return 0;
  return sc::step_layout(*static_cast<sc::StepPlan*>(step)).total;
}

int sc_step_finalize(void* step, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(step && workspace, SC_ERR_ARG, "step_finalize: null pointer");
  StepPlan* p = static_cast<StepPlan*>(step);
  p->ready = false;
  const StepLayout L = step_layout(*p);
  SC_REQUIRE(workspace_bytes >= L.total, SC_ERR_WORKSPACE, "step_finalize: workspace of %zu bytes, %zu needed",
             workspace_bytes, L.total);
  SC_REQUIRE(((uintptr_t)workspace % 256) == 0, SC_ERR_ARG, "step_finalize: workspace not 256-byte aligned");
  SC_REQUIRE(p->emb_w && p->tok, SC_ERR_ARG, "step_finalize: head and io not set");
  for (int i = 0; i < p->nl; ++i) SC_REQUIRE(p->layers[i].w[0], SC_ERR_ARG, "step_finalize: layer %d not set", i);
  if (p->world > 1) SC_REQUIRE(p->arena_bytes, SC_ERR_ARG, "step_finalize: tensor parallel needs the peer arenas");
  char* ws = static_cast<char*>(workspace);
  const int n = p->nsm;
  const int H = p->H, hd = p->hd, Hq = p->Hq, Hkv = p->Hkv, F = p->F;
  const int qkvN = (Hq + 2 * Hkv) * hd;
  // everything but the weight images starts at zero (the images are written whole below)
  cudaError_t e = cudaMemsetAsync(ws, 0, L.img, stream);
  SC_REQUIRE(e == cudaSuccess, SC_ERR_CUDA, "step_finalize: memset failed (%s)", cudaGetErrorString(e));
  // ---- weight images
  auto pack = [&](unsigned char* img, int nseg, int nset, const uint32_t* const* w, const uint16_t* const* sc,
                  const uint16_t* const* bi, const int* rws, int K) -> bool {
    PackOp po{};
    po.nseg = nseg;
    po.nset = nset;
    po.K = K;
    po.kq = kq_of(K);
    int total_rows = 0;
    for (int j = 0; j < std::max(nseg, nset); ++j) {
      po.w[j] = w[j];
      po.s[j] = sc[j];
      po.b[j] = bi[j];
      po.rows[j] = rws[j];
      po.seg_tiles[j] = (rws[j] + 15) / 16;
      if (j < nseg) total_rows += po.seg_tiles[j] * 16;
    }
    po.tiles = total_rows / 16;
    po.img = img;
    launch(step_pack_kernel, dim3(4 * n), dim3(256), 0, stream, po);
    return cudaGetLastError() == cudaSuccess;
  };
  bool packed = true;
  for (int i = 0; i < p->nl && packed; ++i) {
    const StepLayer& ly = p->layers[i];
    unsigned char* base = reinterpret_cast<unsigned char*>(ws + L.img + L.img_layer * i);
    const int rq[3] = {Hq * hd, Hkv * hd, Hkv * hd}, ro[1] = {H}, rg[2] = {F, F}, rd[1] = {H};
    packed = pack(base + L.img_off[0], 3, 1, ly.w, ly.s, ly.b, rq, H) &&
             pack(base + L.img_off[1], 1, 1, ly.w + 3, ly.s + 3, ly.b + 3, ro, Hq * hd) &&
             pack(base + L.img_off[2], 1, 2, ly.w + 4, ly.s + 4, ly.b + 4, rg, H) &&
             pack(base + L.img_off[3], 1, 1, ly.w + 6, ly.s + 6, ly.b + 6, rd, F);
  }
  if (packed) {
    const int rv[1] = {p->Vl};
    packed = pack(reinterpret_cast<unsigned char*>(ws + L.img + L.img_head), 1, 1, &p->emb_w, &p->emb_s, &p->emb_b,
                  rv, H);
  }
  SC_REQUIRE(packed, SC_ERR_CUDA, "step_finalize: weight image pack failed");
  // ---- ops
  std::vector<StepOp> ops;
  auto gemv = [&](int kind, int layer, int K, int nrows, int nset) {
    StepOp o{};
    o.kind = kind;
    o.layer = layer;
    o.nset = nset;
    o.nseg = 1;
    o.K = K;
    o.kq = kq_of(K);
    o.rows = nrows;
    o.tiles = (nrows + 15) / 16;
    o.total = (long long)o.tiles * o.kq;
    o.xchg = -1;
    o.xs_bytes = staged_bytes(K);
    return o;
  };
  float* h = reinterpret_cast<float*>(ws + L.h);
  unsigned char* xs_h = reinterpret_cast<unsigned char*>(ws + L.xs_h);
  float* xss_h = reinterpret_cast<float*>(ws + L.xss_h);
  unsigned char* xs_o = reinterpret_cast<unsigned char*>(ws + L.xs_o);
  unsigned char* xs_gu = reinterpret_cast<unsigned char*>(ws + L.xs_gu);
  float* xss_gu = reinterpret_cast<float*>(ws + L.xss_gu);
  unsigned char* xs_down = reinterpret_cast<unsigned char*>(ws + L.xs_down);
  int xchg = 0;
  {
    StepOp eo{};
    eo.kind = SOP_EMBED;
    eo.layer = -1;
    eo.xchg = p->world > 1 ? xchg++ : -1;
    eo.h = h;
    eo.trace = p->trace;
    eo.out_xs = xs_h;
    eo.out_xss = xss_h;
    eo.out_norm = p->layers[0].ln1;
    eo.out_ctr = L.ctr_x + 1;  // the first q|k|v
    ops.push_back(eo);
  }
  for (int i = 0; i < p->nl; ++i) {
    const int oq = (int)ops.size();
    StepOp q = gemv(SOP_QKV, i, H, qkvN, 1);
    q.nseg = 3;
    q.seg_tiles[0] = Hq * hd / 16;
    q.seg_tiles[1] = Hkv * hd / 16;
    q.seg_tiles[2] = Hkv * hd / 16;
    q.img = reinterpret_cast<const unsigned char*>(ws + L.img + L.img_layer * i + L.img_off[0]);
    q.xs = xs_h;
    q.xss = xss_h;
    q.x_ctr = L.ctr_x + oq;
    q.x_need = H / 64;
    q.part = reinterpret_cast<float*>(ws + L.part_qkv);
    q.grp_ctr = L.ctr_grp + oq * L.max_groups;
    for (int tt = 0; tt < q.tiles; ++tt) q.seg_need += tile_nseg(tt, q.kq, q.total, gemv_ctas(q.total, q.kq, n));
    ops.push_back(q);
    StepOp a{};
    a.kind = SOP_ATTN;
    a.layer = i;
    a.kc = p->layers[i].kc;
    a.vc = p->layers[i].vc;
    a.out_xs = xs_o;
    a.out_ctr = L.ctr_x + oq + 2;  // o_proj
    a.xchg = -1;
    ops.push_back(a);
    const int oo = (int)ops.size();
    StepOp o = gemv(SOP_O, i, Hq * hd, H, 1);
    o.img = reinterpret_cast<const unsigned char*>(ws + L.img + L.img_layer * i + L.img_off[1]);
    o.xs = xs_o;
    o.x_ctr = L.ctr_x + oo;
    o.x_need = Hq * hd / 64;
    o.part = reinterpret_cast<float*>(ws + L.part_o);
    o.grp_ctr = L.ctr_grp + oo * L.max_groups;
    o.h = h;
    o.xchg = p->world > 1 ? xchg++ : -1;
    o.out_xs = xs_gu;
    o.out_xss = xss_gu;
    o.out_norm = p->layers[i].ln2;
    o.out_ctr = L.ctr_x + oo + 1;
    ops.push_back(o);
    const int og = (int)ops.size();
    StepOp gu = gemv(SOP_GATEUP, i, H, F, 2);
    gu.img = reinterpret_cast<const unsigned char*>(ws + L.img + L.img_layer * i + L.img_off[2]);
    gu.xs = xs_gu;
    gu.xss = xss_gu;
    gu.x_ctr = L.ctr_x + og;
    gu.x_need = H / 64;
    gu.part = reinterpret_cast<float*>(ws + L.part_gu);
    gu.grp_ctr = L.ctr_grp + og * L.max_groups;
    gu.out_xs = xs_down;
    gu.out_ctr = L.ctr_x + og + 1;
    ops.push_back(gu);
    const int od = (int)ops.size();
    StepOp d = gemv(SOP_DOWN, i, F, H, 1);
    d.img = reinterpret_cast<const unsigned char*>(ws + L.img + L.img_layer * i + L.img_off[3]);
    d.xs = xs_down;
    d.x_ctr = L.ctr_x + od;
    d.x_need = F / 64;
    d.part = reinterpret_cast<float*>(ws + L.part_down);
    d.grp_ctr = L.ctr_grp + od * L.max_groups;
    d.h = h;
    d.trace = p->trace ? p->trace + (size_t)(i + 1) * H : nullptr;
    d.xchg = p->world > 1 ? xchg++ : -1;
    d.out_xs = xs_h;
    d.out_xss = xss_h;
    d.out_norm = i + 1 < p->nl ? p->layers[i + 1].ln1 : p->fnorm;
    d.out_ctr = L.ctr_x + od + 1;  // the next q|k|v, or the head
    ops.push_back(d);
  }
  {
    const int oh = (int)ops.size();
    StepOp ho = gemv(SOP_HEAD, p->nl, H, p->Vl, 1);
    ho.img = reinterpret_cast<const unsigned char*>(ws + L.img + L.img_head);
    ho.xs = xs_h;
    ho.xss = xss_h;
    ho.x_ctr = L.ctr_x + oh;
    ho.x_need = H / 64;
    ho.part = reinterpret_cast<float*>(ws + L.part_head);
    ho.grp_ctr = L.ctr_head_tile;
    ops.push_back(ho);
  }
  SC_REQUIRE((int)ops.size() == L.nops, SC_ERR_ARG, "step_finalize: op count %d != %d", (int)ops.size(), L.nops);
  SC_REQUIRE(xchg <= 255, SC_ERR_UNSUPPORTED, "step_finalize: too many layers for the exchange epochs");
  for (const auto& o : ops) {
    if (o.kind == SOP_EMBED || o.kind == SOP_ATTN) continue;
    for (int tt = 0; tt < o.tiles; ++tt)
      SC_REQUIRE(tile_nseg(tt, o.kq, o.total, gemv_ctas(o.total, o.kq, n)) <= SP_MAXT, SC_ERR_UNSUPPORTED,
                 "step_finalize: a tile of op kind %d spans more than %d CTAs", o.kind, SP_MAXT);
  }
  // ---- shared memory: staged x (or an attention merge), then as many ring stages as fit
  const int G = p->G;
  size_t xs_alloc = std::max({(size_t)L.xs_bytes_h, (size_t)L.xs_bytes_o, (size_t)L.xs_bytes_down,
                              (size_t)SP_NCW * G * (hd + 4) * 4});
  xs_alloc = align_up(xs_alloc, 1024);
  const size_t static_smem = static_smem_of(G);
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, p->device);
  SC_REQUIRE((size_t)optin > static_smem + 1024 + xs_alloc + 2 * SP_STAGE_BYTES, SC_ERR_UNSUPPORTED,
             "step_finalize: %d bytes of shared memory cannot hold the staged input and two stages", optin);
  const size_t budget = (size_t)optin - static_smem - 1024;
  const int nst = (int)std::min<size_t>(SP_MAX_NST, (budget - xs_alloc) / SP_STAGE_BYTES);
  p->smem = xs_alloc + (size_t)nst * SP_STAGE_BYTES + 1024;
  {
    int nb = 0;
    cudaFuncAttributes fa{};
    fit_of(G, p->smem, &nb, &fa);
    p->fit[0] = p->nsm;
    p->fit[1] = nb;
    p->fit[2] = (int)fa.sharedSizeBytes;
    p->fit[3] = (int)p->smem;
    p->fit[4] = fa.numRegs;
    p->fit[5] = fa.maxThreadsPerBlock;
    SC_REQUIRE(nb >= 1 && fa.maxThreadsPerBlock >= SP_THREADS, SC_ERR_UNSUPPORTED,
               "step_finalize: the step kernel does not fit an SM (%d CTAs per SM, %d registers x %d threads, "
               "%zu + %zu bytes of shared memory, at most %d threads per block)",
               nb, fa.numRegs, SP_THREADS, (size_t)fa.sharedSizeBytes, p->smem, fa.maxThreadsPerBlock);
    p->grid = p->nsm;
  }
  // ---- upload
  e = cudaMemcpyAsync(ws + L.ops, ops.data(), sizeof(StepOp) * ops.size(), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  SC_REQUIRE(e == cudaSuccess, SC_ERR_CUDA, "step_finalize: upload failed (%s)", cudaGetErrorString(e));
  StepParams& P = p->P;
  P = StepParams{};
  P.ops = reinterpret_cast<const StepOp*>(ws + L.ops);
  P.nops = L.nops;
  int* ctr = reinterpret_cast<int*>(ws + L.ctr);
  P.ctr = ctr;
  P.attn_ctr = ctr + L.ctr_attn;
  P.gen = ctr + L.ctr_misc + 0;
  P.err = ctr + L.ctr_misc + 1;
  P.info = ctr + L.ctr_misc + 8;
  P.progress = reinterpret_cast<int*>(ws + L.progress);
  P.stamps = p->stamps;
  P.head_done = ctr + L.ctr_misc + 2;
  P.key = reinterpret_cast<unsigned long long*>(ctr + L.ctr_misc + 4);
  P.tok = p->tok;
  P.pos = p->pos;
  P.cos_tab = p->cos_tab;
  P.sin_tab = p->sin_tab;
  P.max_pos = p->max_pos;
  P.logits = p->logits;
  P.emb_w = p->emb_w;
  P.emb_s = p->emb_s;
  P.emb_b = p->emb_b;
  P.vocab_start = p->v0;
  P.vocab_local = p->Vl;
  P.attn_part = reinterpret_cast<float*>(ws + L.attn_part);
  P.H = H;
  P.Hq = Hq;
  P.Hkv = Hkv;
  P.hd = hd;
  P.Lmax = p->Lmax;
  P.nl = p->nl;
  P.eps = p->eps;
  P.scale = 1.f / sqrtf((float)hd);
  P.xs_alloc = (int)xs_alloc;
  P.nst = nst;
  P.world = p->world;
  P.rank = p->rank;
  for (int q = 0; q < p->world; ++q) P.arena[q] = p->arena[q];
  P.row_region = (size_t)H / 2 * 16;
  P.key_off = SP_ARENA_HDR + 2 * (size_t)p->world * P.row_region;
  p->ready = true;
  return SC_OK;
}

int sc_step_run(void* step, cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(step, SC_ERR_ARG, "step_run: null handle");
  StepPlan* p = static_cast<StepPlan*>(step);
  SC_REQUIRE(p->ready, SC_ERR_ARG, "step_run: call sc_step_finalize first");
  cudaError_t e;
  switch (p->G) {
    case 1: e = launch_step<1>(p, stream); break;
    case 2: e = launch_step<2>(p, stream); break;
    case 4: e = launch_step<4>(p, stream); break;
    default: e = launch_step<8>(p, stream); break;
  }
  if (e == cudaErrorCooperativeLaunchTooLarge) {
    cudaGetLastError();
    set_error("step_run: cooperative launch of %d CTAs refused (%d SMs, %d CTAs per SM, %d registers, %d + %d bytes "
              "of shared memory)",
              p->grid, p->fit[0], p->fit[1], p->fit[4], p->fit[2], p->fit[3]);
    return SC_ERR_CUDA;
  }
  note_launch_status(e);
  return check_launch("decode_step");
}

int sc_step_error(void* step, int reset) {
  using namespace sc;
  if (!step) return 0;
  StepPlan* p = static_cast<StepPlan*>(step);
  if (!p->ready) return 0;
  int v = 0;
  cudaMemcpy(&v, p->P.err, sizeof(int), cudaMemcpyDeviceToHost);
  if (reset && v) {
    // a failed step leaves the counters part-way: every count restarts from zero
    const StepLayout L = step_layout(*p);
    cudaMemset(p->P.ctr, 0, sizeof(int) * L.nctr);
  }
  return v;
}

int sc_step_error_info(void* step, int* out, int n) {
  using namespace sc;
  SC_REQUIRE(step && out && n >= 8, SC_ERR_ARG, "step_error_info: null pointer or fewer than 8 ints");
  StepPlan* p = static_cast<StepPlan*>(step);
  SC_REQUIRE(p->ready, SC_ERR_ARG, "step_error_info: call sc_step_finalize first");
  cudaError_t e = cudaMemcpy(out, p->P.info, 8 * sizeof(int), cudaMemcpyDeviceToHost);
  const int np = std::min(n - 8, p->nsm);
  if (e == cudaSuccess && np > 0) e = cudaMemcpy(out + 8, p->P.progress, np * sizeof(int), cudaMemcpyDeviceToHost);
  const int nc = std::min(n - 8 - p->nsm, step_layout(*p).nctr);
  if (e == cudaSuccess && nc > 0) e = cudaMemcpy(out + 8 + p->nsm, p->P.ctr, nc * sizeof(int), cudaMemcpyDeviceToHost);
  SC_REQUIRE(e == cudaSuccess, SC_ERR_CUDA, "step_error_info: copy failed (%s)", cudaGetErrorString(e));
  return SC_OK;
}

int sc_step_fit(void* step, int* out6) {
  using namespace sc;
  SC_REQUIRE(step && out6, SC_ERR_ARG, "step_fit: null pointer");
  const StepPlan* p = static_cast<const StepPlan*>(step);
  for (int i = 0; i < 6; ++i) out6[i] = p->fit[i];
  return SC_OK;
}

int sc_step_destroy(void* step) {
  delete static_cast<sc::StepPlan*>(step);
  return SC_OK;
}

}  // extern "C"
