// K5 / K7 and the ABI plumbing: RMSNorm, SiLU*mul, add, greedy argmax over
// vocab-split logits, status strings and the thread-local error message.
#include <atomic>
#include <stdarg.h>
#include <stdio.h>
#include <climits>

#include <algorithm>

#include "sc_common.cuh"

namespace sc {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// Kernels enqueued by this library (each successful check follows exactly one launch).
static std::atomic<unsigned long long> g_launches{0};

static thread_local cudaError_t g_launch_status = cudaSuccess;

void note_launch_status(cudaError_t e) {
  if (e != cudaSuccess && g_launch_status == cudaSuccess) g_launch_status = e;
}

int check_launch(const char* what, cudaError_t launch_status) {
  const cudaError_t last = cudaGetLastError();  // also clears a sticky launch error
  const cudaError_t noted = g_launch_status;
  g_launch_status = cudaSuccess;
  const cudaError_t e = launch_status != cudaSuccess ? launch_status : (noted != cudaSuccess ? noted : last);
  if (e != cudaSuccess) {
    set_error("%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
    return SC_ERR_CUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SC_OK;
}

int check_launch(const char* what) { return check_launch(what, cudaSuccess); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("SC_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename T>
__device__ __forceinline__ float ldf(const void* p, size_t i) {
  return to_f32<T>(reinterpret_cast<const T*>(p)[i]);
}

// One CTA per row: y = x / sqrt(mean(x^2) + eps) * w
template <typename XT, typename YT>
__global__ void rmsnorm_kernel(const void* __restrict__ x, int H, const uint16_t* __restrict__ w, float eps,
                               void* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = ldf<XT>(x, (size_t)row * H + i);
    ss = fmaf(v, v, ss);
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rms = sqrtf(red[0] / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = ldf<XT>(x, (size_t)row * H + i);
    reinterpret_cast<YT*>(y)[(size_t)row * H + i] =
        from_f32<YT>((v / rms) * __half2float(__ushort_as_half(w[i])));
  }
}

template <typename IT, typename OT>
__global__ void silu_mul_kernel(const void* __restrict__ g, const void* __restrict__ u, size_t n, void* __restrict__ o) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<OT*>(o)[i] = from_f32<OT>(silu_f32(ldf<IT>(g, i)) * ldf<IT>(u, i));
}

template <typename AT, typename BT, typename YT>
__global__ void add_kernel(const void* __restrict__ a, const void* __restrict__ b, size_t n, void* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<YT*>(y)[i] = from_f32<YT>(ldf<AT>(a, i) + ldf<BT>(b, i));
}

// (value, index) ordering: larger value wins, lower index breaks ties.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

constexpr int AM_THREADS = 256;
constexpr int AM_CHUNK = 4096;

__global__ void argmax_partial_kernel(const float* __restrict__ logits, int N, int ldl, float* __restrict__ pv,
                                      int* __restrict__ pi, int nchunks) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x, row = blockIdx.y;
  const int beg = c * AM_CHUNK, end = min(N, beg + AM_CHUNK);
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int i = beg + threadIdx.x; i < end; i += AM_THREADS) {
    const float v = logits[(size_t)row * ldl + i];
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[AM_THREADS / 32];
  __shared__ int si[AM_THREADS / 32];
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < AM_THREADS / 32; ++w)
      if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    pv[(size_t)row * nchunks + c] = bv;
    pi[(size_t)row * nchunks + c] = bi;
  }
}

__global__ void argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int nchunks,
                                    int offset, float* __restrict__ val, int32_t* __restrict__ idx) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int c = threadIdx.x; c < nchunks; c += 32) {
    const float v = pv[(size_t)row * nchunks + c];
    const int i = pi[(size_t)row * nchunks + c];
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (threadIdx.x == 0) {
    val[row] = bv;
    idx[row] = bi == INT_MAX ? -1 : bi + offset;
  }
}

__global__ void argmax_merge_kernel(const float* __restrict__ vals, const int32_t* __restrict__ idxs, int M, int world,
                                    int32_t* __restrict__ tok, int32_t* __restrict__ pos, int adv) {
  pdl_trigger();
  pdl_wait();
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int r = 0; r < world; ++r) {
      const float v = vals[(size_t)r * M + m];
      const int i = idxs[(size_t)r * M + m];
      if (i >= 0 && better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    tok[m] = bi == INT_MAX ? 0 : bi;
  }
  if (pos && threadIdx.x == 0) *pos += adv;
}

template <typename A, typename B>
static int add_dispatch_y(const void* a, const void* b, size_t n, void* y, int yd, cudaStream_t st) {
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 8 * (size_t)sm_count());
  if (yd == SC_F16) ::sc::launch(add_kernel<A, B, __half>, blocks, 256, 0, st, a, b, n, y);
  else ::sc::launch(add_kernel<A, B, float>, blocks, 256, 0, st, a, b, n, y);
  return check_launch("add");
}

}  // namespace sc

extern "C" {

int sc_abi_version(void) { return SC_ABI_VERSION; }

const char* sc_status_name(int status) {
  switch (status) {
    case SC_OK: return "SC_OK";
    case SC_ERR_SHAPE: return "SC_ERR_SHAPE";
    case SC_ERR_CUDA: return "SC_ERR_CUDA";
    case SC_ERR_NCCL: return "SC_ERR_NCCL";
    case SC_ERR_TIMEOUT: return "SC_ERR_TIMEOUT";
    case SC_ERR_ARG: return "SC_ERR_ARG";
    case SC_ERR_UNSUPPORTED: return "SC_ERR_UNSUPPORTED";
    case SC_ERR_WORKSPACE: return "SC_ERR_WORKSPACE";
  }
  return "SC_ERR_UNKNOWN";
}

const char* sc_last_error(void) { return sc::g_err; }

unsigned long long sc_launch_count(void) { return sc::g_launches.load(std::memory_order_relaxed); }

int sc_rmsnorm(const void* x, int x_dtype, int M, int H, const uint16_t* w, float eps, void* y, int y_dtype,
               cudaStream_t stream) {
  SC_REQUIRE(H > 0, SC_ERR_SHAPE, "rmsnorm: H must be positive");
  if (M <= 0) return SC_OK;
  SC_REQUIRE(x && w && y, SC_ERR_ARG, "rmsnorm: null pointer");
  const int threads = std::min(1024, std::max(32, (H + 31) / 32 * 32 / 4));
  if (x_dtype == SC_F32 && y_dtype == SC_F32) ::sc::launch(sc::rmsnorm_kernel<float, float>, M, threads, 0, stream, x, H, w, eps, y);
  else if (x_dtype == SC_F32 && y_dtype == SC_F16) ::sc::launch(sc::rmsnorm_kernel<float, __half>, M, threads, 0, stream, x, H, w, eps, y);
  else if (x_dtype == SC_F16 && y_dtype == SC_F32) ::sc::launch(sc::rmsnorm_kernel<__half, float>, M, threads, 0, stream, x, H, w, eps, y);
  else if (x_dtype == SC_F16 && y_dtype == SC_F16) ::sc::launch(sc::rmsnorm_kernel<__half, __half>, M, threads, 0, stream, x, H, w, eps, y);
  else SC_REQUIRE(false, SC_ERR_ARG, "rmsnorm: dtype");
  return sc::check_launch("rmsnorm");
}

int sc_silu_mul(const void* gate, const void* up, int in_dtype, size_t n, void* out, int out_dtype,
                cudaStream_t stream) {
  if (n == 0) return SC_OK;
  SC_REQUIRE(gate && up && out, SC_ERR_ARG, "silu_mul: null pointer");
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 8 * (size_t)sc::sm_count());
  if (in_dtype == SC_F32 && out_dtype == SC_F32) ::sc::launch(sc::silu_mul_kernel<float, float>, blocks, 256, 0, stream, gate, up, n, out);
  else if (in_dtype == SC_F32 && out_dtype == SC_F16) ::sc::launch(sc::silu_mul_kernel<float, __half>, blocks, 256, 0, stream, gate, up, n, out);
  else if (in_dtype == SC_F16 && out_dtype == SC_F32) ::sc::launch(sc::silu_mul_kernel<__half, float>, blocks, 256, 0, stream, gate, up, n, out);
  else if (in_dtype == SC_F16 && out_dtype == SC_F16) ::sc::launch(sc::silu_mul_kernel<__half, __half>, blocks, 256, 0, stream, gate, up, n, out);
  else SC_REQUIRE(false, SC_ERR_ARG, "silu_mul: dtype");
  return sc::check_launch("silu_mul");
}

int sc_add(const void* a, int a_dtype, const void* b, int b_dtype, size_t n, void* y, int y_dtype,
           cudaStream_t stream) {
  if (n == 0) return SC_OK;
  SC_REQUIRE(a && b && y, SC_ERR_ARG, "add: null pointer");
  SC_REQUIRE((a_dtype == SC_F16 || a_dtype == SC_F32) && (b_dtype == SC_F16 || b_dtype == SC_F32) &&
                 (y_dtype == SC_F16 || y_dtype == SC_F32),
             SC_ERR_ARG, "add: dtype");
  if (a_dtype == SC_F32 && b_dtype == SC_F32) return sc::add_dispatch_y<float, float>(a, b, n, y, y_dtype, stream);
  if (a_dtype == SC_F32 && b_dtype == SC_F16) return sc::add_dispatch_y<float, __half>(a, b, n, y, y_dtype, stream);
  if (a_dtype == SC_F16 && b_dtype == SC_F32) return sc::add_dispatch_y<__half, float>(a, b, n, y, y_dtype, stream);
  return sc::add_dispatch_y<__half, __half>(a, b, n, y, y_dtype, stream);
}

size_t sc_argmax_workspace_bytes(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  const size_t nch = (N + sc::AM_CHUNK - 1) / sc::AM_CHUNK;
  return (size_t)M * nch * (sizeof(float) + sizeof(int));
}

int sc_argmax(const float* logits, int M, int N, int ldl, int index_offset, float* val, int32_t* idx,
              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  SC_REQUIRE(N > 0 && ldl >= N, SC_ERR_SHAPE, "argmax: bad N/ldl");
  if (M <= 0) return SC_OK;
  SC_REQUIRE(logits && val && idx, SC_ERR_ARG, "argmax: null pointer");
  const size_t need = sc_argmax_workspace_bytes(M, N);
  SC_REQUIRE(workspace && workspace_bytes >= need, SC_ERR_WORKSPACE, "argmax: workspace of %zu bytes needed", need);
  const int nch = (N + sc::AM_CHUNK - 1) / sc::AM_CHUNK;
  float* pv = (float*)workspace;
  int* pi = (int*)(pv + (size_t)M * nch);
  ::sc::launch(sc::argmax_partial_kernel, dim3(nch, M), sc::AM_THREADS, 0, stream, logits, N, ldl, pv, pi, nch);
  int st = sc::check_launch("argmax_partial");
  if (st != SC_OK) return st;
  ::sc::launch(sc::argmax_final_kernel, M, 32, 0, stream, pv, pi, nch, index_offset, val, idx);
  return sc::check_launch("argmax_final");
}

int sc_argmax_merge(const float* vals, const int32_t* idxs, int M, int world, int32_t* token_out, int32_t* pos,
                    int pos_advance, cudaStream_t stream) {
  SC_REQUIRE(world >= 1, SC_ERR_SHAPE, "argmax_merge: world must be >= 1");
  if (M <= 0) return SC_OK;
  SC_REQUIRE(vals && idxs && token_out, SC_ERR_ARG, "argmax_merge: null pointer");
  ::sc::launch(sc::argmax_merge_kernel, 1, 256, 0, stream, vals, idxs, M, world, token_out, pos, pos_advance);
  return sc::check_launch("argmax_merge");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// L2 prefetch of upcoming weights.  Launched right after a GEMV, this kernel
// starts while that GEMV runs (programmatic dependent launch), issues
// fire-and-forget cp.async.bulk.prefetch.L2 requests for the next GEMV's
// weights so HBM stays busy through the GEMV's tail, the kernels in between
// and the next launch, and then waits for its predecessor before exiting so
// stream order is kept for everything after it.
namespace sc {

__global__ void l2_prefetch_kernel(const PrefetchList L) {
  pdl_trigger();
  l2_prefetch_share(L, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
  pdl_wait();
}

int make_prefetch_list(const void* const* ptrs, const size_t* bytes, int n, size_t max_bytes, PrefetchList* L) {
  SC_REQUIRE(n >= 0 && n <= PF_MAX_REGIONS, SC_ERR_ARG, "l2 prefetch: 0..%d regions (got %d)", PF_MAX_REGIONS, n);
  SC_REQUIRE(n == 0 || (ptrs && bytes), SC_ERR_ARG, "l2 prefetch: null region list");
  *L = PrefetchList{};
  size_t budget = max_bytes ? max_bytes : (size_t)-1;
  for (int r = 0; r < n && budget; ++r) {
    const uintptr_t a = (uintptr_t)ptrs[r];
    if (!a || bytes[r] < 16) continue;
    const uintptr_t a16 = (a + 15) & ~(uintptr_t)15;  // bulk prefetch wants 16-byte aligned starts
    size_t len = bytes[r] - (a16 - a);
    len = std::min(len & ~(size_t)15, budget);
    if (!len) continue;
    L->p[L->count] = reinterpret_cast<const unsigned char*>(a16);
    L->n[L->count] = len;
    ++L->count;
    budget -= len;
  }
  return SC_OK;
}

}  // namespace sc

extern "C" int sc_l2_prefetch(const void* const* ptrs, const size_t* bytes, int n, size_t max_bytes,
                              cudaStream_t stream) {
  sc::PrefetchList L;
  if (int st = sc::make_prefetch_list(ptrs, bytes, n, max_bytes, &L)) return st;
  if (L.count == 0) return SC_OK;
  ::sc::launch(sc::l2_prefetch_kernel, 8, 128, 0, stream, L);
  return sc::check_launch("l2_prefetch");
}
