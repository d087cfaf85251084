// Temperature + top-p sampling over vocab-split logits, with a distributed
// top-p: no rank ever holds the full distribution.  Replaces the sampled
// branch of ParallelExecutor.generate (worker/executor.py:270-306: logits /
// T, softmax, sort, cumsum, keep a token while the mass sorted before it is
// <= top_p, renormalise, draw).
//
// The sort is replaced by a threshold: a token is kept iff the probability
// mass strictly above its own probability is <= top_p, i.e. iff p >= v*, v*
// the smallest probability for which that holds.  v* is found by a 4-level
// radix select on the fp32 bits of p (non-negative floats order like their
// bits): per level each rank builds a 256-bin histogram of probability mass
// over the keys that share the bits fixed so far, the ranks sum their
// histograms, and the lowest non-empty bin whose mass-above stays <= top_p
// fixes the next 8 bits.  The draw then walks the kept tokens in vocabulary
// order (ranks in order, then indices): the first token whose cumulative
// kept mass exceeds u * (total kept mass), u a uniform per row.
//
// Phases per row (a CTA of SM_THREADS per row); between them a tensor-parallel
// caller combines the ranks' values (max / sum / gather, see the entry
// point); one rank alone runs every phase in one launch.
#include <algorithm>

#include "sc_common.cuh"

namespace sc {

constexpr int SM_THREADS = 1024;
constexpr int SM_WARPS = SM_THREADS / 32;
constexpr int SM_BINS = 256;

// Per-row state (floats, field-major [ST_N][B]): the values the phases exchange.
enum : int {
  ST_MAX = 0,     // max of logits / T (this rank's, then the global one)
  ST_Z = 1,       // sum of exp(logit / T - max)
  ST_A = 2,       // mass strictly above the keys that match the prefix
  ST_PREFIX = 3,  // key bits fixed so far (int bits)
  ST_KEPT = 4,    // this rank's kept mass
  ST_BASE = 5,    // kept mass of the ranks before this one
  ST_TOTAL = 6,   // total kept mass
  ST_TOKEN = 7,   // 1 + the drawn token on the rank that owns it, else 0
  ST_N = 8
};

__device__ __forceinline__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (warp == 0) {
    t = lane < SM_WARPS ? sh[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}

__device__ __forceinline__ float block_max(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < SM_WARPS ? sh[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (lane == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}

struct SampleArgs {
  const float* logits;
  int B;                 // rows
  int V, ld;             // this rank's vocab slice
  float invT, top_p;
  float* st;             // [ST_N][B]: each field contiguous over the rows
  float* hist;           // [B][SM_BINS]
  const float* u;        // [B] uniforms in [0, 1)
  int vocab_start;       // global id of this slice's first token
};

__device__ __forceinline__ float prob_of(const SampleArgs& a, const float* row, int i, float gmax, float rz) {
  return expf(row[i] * a.invT - gmax) * rz;
}

// phase 0: this rank's max of logits / T
__device__ void ph_max(const SampleArgs& a, int b, float* sh) {
  const float* row = a.logits + (size_t)b * a.ld;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < a.V; i += SM_THREADS) m = fmaxf(m, row[i] * a.invT);
  m = block_max(m, sh);
  if (threadIdx.x == 0) a.st[ST_MAX * a.B + b] = m;
}

// phase 1: this rank's sum of exp (global max in ST_MAX)
__device__ void ph_sum(const SampleArgs& a, int b, float* sh) {
  const float* row = a.logits + (size_t)b * a.ld;
  const float gmax = a.st[ST_MAX * a.B + b];
  float z = 0.f;
  for (int i = threadIdx.x; i < a.V; i += SM_THREADS) z += expf(row[i] * a.invT - gmax);
  z = block_sum(z, sh);
  if (threadIdx.x == 0) {
    a.st[ST_Z * a.B + b] = z;
    a.st[ST_A * a.B + b] = 0.f;
    a.st[ST_PREFIX * a.B + b] = __int_as_float(0);
  }
}

// phase 2 (per level): this rank's histogram of mass over the next 8 key bits
__device__ void ph_hist(const SampleArgs& a, int b, int level, float* sh, float (*wh)[SM_BINS]) {
  const float* row = a.logits + (size_t)b * a.ld;
  const float gmax = a.st[ST_MAX * a.B + b], rz = 1.f / a.st[ST_Z * a.B + b];
  const uint32_t prefix = (uint32_t)__float_as_int(a.st[ST_PREFIX * a.B + b]);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < SM_WARPS * SM_BINS; i += SM_THREADS) (&wh[0][0])[i] = 0.f;
  __syncthreads();
  const int sh_hi = 32 - 8 * level, sh_bin = 24 - 8 * level;
  for (int i = threadIdx.x; i < a.V; i += SM_THREADS) {
    const float p = prob_of(a, row, i, gmax, rz);
    const uint32_t key = __float_as_uint(p);
    if (level == 0 || (key >> sh_hi) == prefix) atomicAdd(&wh[warp][(key >> sh_bin) & 255u], p);
  }
  __syncthreads();
  // the warps' histograms summed in warp order
  for (int bin = threadIdx.x; bin < SM_BINS; bin += SM_THREADS) {
    float s = 0.f;
    for (int w = 0; w < SM_WARPS; ++w) s += wh[w][bin];
    a.hist[(size_t)b * SM_BINS + bin] = s;
  }
  (void)lane;
  (void)sh;
}

// phase 3 (per level, after the ranks' histograms were summed): fix 8 more bits
__device__ void ph_select(const SampleArgs& a, int b) {
  if (threadIdx.x != 0) return;
  const float* h = a.hist + (size_t)b * SM_BINS;
  float C = a.st[ST_A * a.B + b];
  int pick = -1;
  float A_pick = C;
  for (int bin = SM_BINS - 1; bin >= 0; --bin) {
    if (C > a.top_p) break;  // every lower bin has at least this much above it
    if (h[bin] > 0.f) {
      pick = bin;
      A_pick = C;
    }
    C += h[bin];
  }
  if (pick < 0) {  // nothing fits (top_p below the largest mass): keep the top bin
    for (int bin = SM_BINS - 1; bin >= 0; --bin)
      if (h[bin] > 0.f) {
        pick = bin;
        break;
      }
    A_pick = a.st[ST_A * a.B + b];
    if (pick < 0) pick = 0;
  }
  const uint32_t prefix = (uint32_t)__float_as_int(a.st[ST_PREFIX * a.B + b]);
  a.st[ST_PREFIX * a.B + b] = __int_as_float((int)((prefix << 8) | (uint32_t)pick));
  a.st[ST_A * a.B + b] = A_pick;
}

// phase 4: this rank's kept mass (keys >= the boundary key)
__device__ void ph_kept(const SampleArgs& a, int b, float* sh) {
  const float* row = a.logits + (size_t)b * a.ld;
  const float gmax = a.st[ST_MAX * a.B + b], rz = 1.f / a.st[ST_Z * a.B + b];
  const uint32_t vkey = (uint32_t)__float_as_int(a.st[ST_PREFIX * a.B + b]);
  float k = 0.f;
  for (int i = threadIdx.x; i < a.V; i += SM_THREADS) {
    const float p = prob_of(a, row, i, gmax, rz);
    if (__float_as_uint(p) >= vkey) k += p;
  }
  k = block_sum(k, sh);
  if (threadIdx.x == 0) a.st[ST_KEPT * a.B + b] = k;
}

// phase 5 (ST_BASE / ST_TOTAL set): the draw, if it falls in this rank's slice
__device__ void ph_pick(const SampleArgs& a, int b, float* sh, float* scan) {
  const float* row = a.logits + (size_t)b * a.ld;
  const float gmax = a.st[ST_MAX * a.B + b], rz = 1.f / a.st[ST_Z * a.B + b];
  const uint32_t vkey = (uint32_t)__float_as_int(a.st[ST_PREFIX * a.B + b]);
  const float base = a.st[ST_BASE * a.B + b], total = a.st[ST_TOTAL * a.B + b];
  const float kept = a.st[ST_KEPT * a.B + b];
  // the ranks' intervals [base, base + kept) tile [0, total) exactly (every rank
  // sums the same masses in rank order), so a target below total has one owner
  const float target = fminf(a.u[b] * total, __uint_as_float(__float_as_uint(total) - 1u));
  constexpr int NONE = 0x7fffffff;  // atomicMin below: "no crossing yet" must be the largest int
  __shared__ int s_tok;
  if (threadIdx.x == 0) s_tok = NONE;
  __syncthreads();
  const bool mine = kept > 0.f && target >= base && target < base + kept;
  if (mine) {
    // blocked prefix sum over the slice, SM_THREADS consecutive values per round
    float run = base;
    for (int i0 = 0; i0 < a.V && s_tok == NONE; i0 += SM_THREADS) {
      const int i = i0 + threadIdx.x;
      float p = 0.f;
      if (i < a.V) {
        p = prob_of(a, row, i, gmax, rz);
        if (__float_as_uint(p) < vkey) p = 0.f;
      }
      // inclusive scan in the block (warp shuffles, then the warp sums in order)
      float v = p;
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (lane == 31) scan[warp] = v;
      __syncthreads();
      if (warp == 0) {
        float w = lane < SM_WARPS ? scan[lane] : 0.f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float t = __shfl_up_sync(0xffffffffu, w, o);
          if (lane >= o) w += t;
        }
        if (lane < SM_WARPS) scan[lane] = w;
      }
      __syncthreads();
      const float cum = run + (warp ? scan[warp - 1] : 0.f) + v;
      if (p > 0.f && cum > target) atomicMin(&s_tok, i);  // the first crossing index (lowest i)
      __syncthreads();
      run += scan[SM_WARPS - 1];
      __syncthreads();
    }
    if (threadIdx.x == 0 && s_tok == NONE) {
      // rounding left the target past the last kept token of this slice: take that token
      for (int i = a.V - 1; i >= 0; --i)
        if (__float_as_uint(prob_of(a, row, i, gmax, rz)) >= vkey) {
          s_tok = i;
          break;
        }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0)
    a.st[ST_TOKEN * a.B + b] = mine && s_tok != NONE ? (float)(a.vocab_start + s_tok + 1) : 0.f;
  (void)sh;
}

__global__ void __launch_bounds__(SM_THREADS) sample_phase_kernel(const SampleArgs a, int phase, int level) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sh[33];
  __shared__ float wh[SM_WARPS][SM_BINS];
  __shared__ float scan[SM_WARPS];
  const int b = blockIdx.x;
  switch (phase) {
    case 0: ph_max(a, b, sh); break;
    case 1: ph_sum(a, b, sh); break;
    case 2: ph_hist(a, b, level, sh, wh); break;
    case 3: ph_select(a, b); break;
    case 4: ph_kept(a, b, sh); break;
    case 5: ph_pick(a, b, sh, scan); break;
  }
}

// One rank: every phase in one launch.
__global__ void __launch_bounds__(SM_THREADS) sample_fused_kernel(const SampleArgs a, int32_t* tok) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sh[33];
  __shared__ float wh[SM_WARPS][SM_BINS];
  __shared__ float scan[SM_WARPS];
  const int b = blockIdx.x;
  ph_max(a, b, sh);
  __syncthreads();
  ph_sum(a, b, sh);
  __syncthreads();
  for (int level = 0; level < 4; ++level) {
    ph_hist(a, b, level, sh, wh);
    __syncthreads();
    ph_select(a, b);
    __syncthreads();
  }
  ph_kept(a, b, sh);
  __syncthreads();
  if (threadIdx.x == 0) {
    a.st[ST_BASE * a.B + b] = 0.f;
    a.st[ST_TOTAL * a.B + b] = a.st[ST_KEPT * a.B + b];
  }
  __syncthreads();
  ph_pick(a, b, sh, scan);
  __syncthreads();
  if (threadIdx.x == 0) {
    const int t = (int)a.st[ST_TOKEN * a.B + b] - 1;
    if (t >= 0) tok[b] = t;
  }
}

// Tensor-parallel glue on the device (st field-major [ST_N][B]): ST_MAX from
// the gathered maxima, ST_BASE / ST_TOTAL from the gathered kept masses
// (gathered: [world][B]), and the token from ST_TOKEN once the ranks' values
// were summed (exactly one rank holds 1 + token; the token is left as it was
// if none does).
__global__ void sample_combine_kernel(float* st, const float* gathered, int B, int world, int rank, int what,
                                      int32_t* tok) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (what == 0) {
    float m = -INFINITY;
    for (int r = 0; r < world; ++r) m = fmaxf(m, gathered[(size_t)r * B + b]);
    st[ST_MAX * B + b] = m;
  } else if (what == 1) {
    float base = 0.f, total = 0.f;
    for (int r = 0; r < world; ++r) {
      const float k = gathered[(size_t)r * B + b];
      if (r < rank) base += k;
      total += k;
    }
    st[ST_BASE * B + b] = base;
    st[ST_TOTAL * B + b] = total;
  } else {
    const int t = (int)st[ST_TOKEN * B + b] - 1;
    if (t >= 0) tok[b] = t;
  }
}

// Uniforms in [0, 1) for the draws: SplitMix64 (Steele, Lea and Flood's
// splittable generator; the 64-bit finaliser of Vigna's reference version)
// applied to seed + (counter * B + row) * golden-ratio increment.  The
// counter lives on the device and advances by one per call, so a captured
// graph draws fresh uniforms on every replay, identically on every rank.
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void sample_uniforms_kernel(uint64_t seed, unsigned long long* counter, int B, float* u) {
  pdl_wait();
  pdl_trigger();
  const unsigned long long c = *counter;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const uint64_t z = splitmix64(seed + (c * (uint64_t)B + (uint64_t)b) * 0x9E3779B97F4A7C15ull);
    const float f = (float)((double)(z >> 11) * (1.0 / 9007199254740992.0));
    u[b] = f < 1.f ? f : 0.99999994f;
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = c + 1;
}

}  // namespace sc

extern "C" {

int sc_sample_uniforms(uint64_t seed, unsigned long long* counter, int B, float* u, cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(counter && u && B > 0, SC_ERR_ARG, "sample_uniforms: bad arguments");
  launch(sample_uniforms_kernel, dim3(1), dim3(256), 0, stream, seed, counter, B, u);
  return check_launch("sample_uniforms");
}

size_t sc_sample_workspace_bytes(int B) { return (size_t)B * (sc::ST_N + sc::SM_BINS) * sizeof(float); }

// One rank holding the whole vocabulary: tok[b] = the draw of row b.
int sc_sample_topp(const float* logits, int B, int V, int ld, float temperature, float top_p, const float* u,
                   int vocab_start, int32_t* tok, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(logits && u && tok && workspace, SC_ERR_ARG, "sample_topp: null pointer");
  SC_REQUIRE(B > 0 && V > 0 && ld >= V, SC_ERR_SHAPE, "sample_topp: bad shape");
  SC_REQUIRE(temperature > 0.f && top_p > 0.f, SC_ERR_ARG,
             "sample_topp: temperature and top_p must be positive (temperature 0 is the greedy argmax)");
  SC_REQUIRE(workspace_bytes >= sc_sample_workspace_bytes(B), SC_ERR_WORKSPACE, "sample_topp: workspace too small");
  SampleArgs a{logits, B, V, ld, 1.f / temperature, top_p, static_cast<float*>(workspace),
               static_cast<float*>(workspace) + (size_t)B * ST_N, u, vocab_start};
  launch(sample_fused_kernel, dim3(B), dim3(SM_THREADS), 0, stream, a, tok);
  return check_launch("sample_topp");
}

// One phase of the distributed sampler on this rank's vocab slice (phase 0
// max, 1 exp-sum, 2 histogram of `level`, 3 select of `level`, 4 kept mass,
// 5 pick).  The caller combines across ranks: after 0, gather ST_MAX and run
// sc_sample_combine(what 0); after 1, sum ST_Z; after each 2, sum the
// histograms; after 4, gather ST_KEPT and run sc_sample_combine(what 1);
// after 5, sum ST_TOKEN and run sc_sample_combine(what 2).
int sc_sample_phase(const float* logits, int B, int V, int ld, float temperature, float top_p, const float* u,
                    int vocab_start, int phase, int level, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(logits && workspace, SC_ERR_ARG, "sample_phase: null pointer");
  SC_REQUIRE(phase >= 0 && phase <= 5 && level >= 0 && level < 4, SC_ERR_ARG, "sample_phase: bad phase");
  SC_REQUIRE(phase != 5 || u, SC_ERR_ARG, "sample_phase: the pick needs the uniforms");
  SC_REQUIRE(workspace_bytes >= sc_sample_workspace_bytes(B), SC_ERR_WORKSPACE, "sample_phase: workspace too small");
  SampleArgs a{logits, B, V, ld, 1.f / temperature, top_p, static_cast<float*>(workspace),
               static_cast<float*>(workspace) + (size_t)B * ST_N, u, vocab_start};
  launch(sample_phase_kernel, dim3(B), dim3(SM_THREADS), 0, stream, a, phase, level);
  return check_launch("sample_phase");
}

int sc_sample_combine(void* workspace, const float* gathered, int B, int world, int rank, int what, int32_t* tok,
                      cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(workspace && (what == 2 ? tok != nullptr : gathered != nullptr), SC_ERR_ARG, "sample_combine: null");
  launch(sample_combine_kernel, dim3((B + 127) / 128), dim3(128), 0, stream, static_cast<float*>(workspace), gathered,
         B, world, rank, what, tok);
  return check_launch("sample_combine");
}

}  // extern "C"
