// Shared helpers of the sm_100a kernels: status handling, fp16 packing and
// the inline-PTX wrappers the kernels use (mbarrier, bulk/tensor copies,
// mma.sync).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <utility>
#include <stdio.h>

#include "../../include/sc_b200.h"

namespace sc {

// Thread-local error message, read back through sc_last_error().
void set_error(const char* fmt, ...);

// Returns SC_OK or SC_ERR_CUDA (with the launch error recorded).
int check_launch(const char* what);
int check_launch(const char* what, cudaError_t launch_status);

// Programmatic dependent launch.  Every kernel of this library is launched
// with programmatic stream serialisation, so it may be scheduled while its
// predecessor in the stream is still running (hiding the launch gap and the
// predecessor's tail).  Each kernel therefore (1) executes pdl_wait() in
// every CTA before it reads anything a predecessor writes or writes anything
// a predecessor reads -- griddepcontrol.wait returns once every prerequisite
// grid has completed and its memory is visible -- and (2) signals
// pdl_trigger() as soon as its own CTAs are all resident, letting the next
// kernel's CTAs take SMs as they free up.  Only reads of data no kernel of the
// step writes (weights, scales, biases) may precede pdl_wait().  Without the
// launch attribute both instructions are no-ops.  SC_PDL=0 disables it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();
// Split-K scratch of sc_qlinear for this exact shape and group (one weight
// set, store epilogue); tma_ok: the weight pointers are 16-byte aligned.
size_t qlinear_workspace_need(int M, int K, int N, int group, int bits, bool tma_ok);
// The tensor-core dequant-GEMM (sc_qgemm.cu): eligibility, scratch, launch.
bool qgemm_eligible(int M, int K, int nseg, const int* seg_rows, int epi, int bits, int group);
size_t qgemm_workspace_bytes(int M, int K, int N, int epi);
int run_qgemm(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_w, float eps, int nseg,
              const uint32_t* const* wq, const uint16_t* const* scales, const uint16_t* const* biases,
              const int* seg_rows, int group, int bits, const uint16_t* bias, int epi, void* y, int y_dtype,
              int ldy, const float* residual, int ldr, void* ws, size_t ws_bytes, cudaStream_t stream);
// Records a failed launch for the next check_launch() on this thread.
void note_launch_status(cudaError_t e);

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  note_launch_status(e);
  return e;
}

#define SC_REQUIRE(cond, code, ...)          \
  do {                                       \
    if (!(cond)) {                           \
      ::sc::set_error(__VA_ARGS__);          \
      return (code);                         \
    }                                        \
  } while (0)

// ---------------------------------------------------------------- L2 prefetch

// Up to PF_MAX_REGIONS device byte ranges to pull into L2 (16-byte aligned
// starts, lengths multiples of 16), cut into PF_CHUNK-byte bulk prefetches.
constexpr int PF_MAX_REGIONS = 12;
constexpr unsigned PF_CHUNK = 32u << 10;

struct PrefetchList {
  const unsigned char* p[PF_MAX_REGIONS];
  unsigned long long n[PF_MAX_REGIONS];
  int count;
};

// Builds a list from caller regions: starts rounded up to 16 bytes, lengths
// down to 16, at most max_bytes in total (0 = no cap), regions in order.
int make_prefetch_list(const void* const* ptrs, const size_t* bytes, int n, size_t max_bytes, PrefetchList* L);

// Issues this participant's share of the list's chunks (chunk c of the whole
// list goes to participant c % nparts).  Fire and forget: nothing waits for
// the data, and a prefetch is only a hint to the memory system.
__device__ __forceinline__ void l2_prefetch_share(const PrefetchList& L, uint32_t part, uint32_t nparts) {
  unsigned long long c0 = 0;  // first list-wide chunk index of region r
#pragma unroll
  for (int r = 0; r < PF_MAX_REGIONS; ++r) {
    if (r >= L.count) break;
    const unsigned long long n = L.n[r];
    const unsigned long long nch = (n + PF_CHUNK - 1) / PF_CHUNK;
    for (unsigned long long c = (part + nparts - c0 % nparts) % nparts; c < nch; c += nparts) {
      const unsigned long long off = c * PF_CHUNK;
      const unsigned long long rem = n - off;
      const uint32_t sz = (uint32_t)(rem < PF_CHUNK ? rem : PF_CHUNK);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(L.p[r] + off), "r"(sz) : "memory");
    }
    c0 += nch;
  }
}

inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ---------------------------------------------------------------- fp16 bits

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ __half2 hfma2_rn(__half2 a, __half2 b, __half2 c) {
  // fma.rn.f16x2: a*b+c computed exactly, rounded once.
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(h2_as_u32(a)), "r"(h2_as_u32(b)), "r"(h2_as_u32(c)));
  return u32_as_h2(d);
}

// 4-bit codes of one word -> four half2 (q_p, q_{p+4}), p = 0..3, exact.
// (w & 0x000F000F) | 0x64006400 is the fp16 pair (1024 + q0, 1024 + q4); the
// 0x00F0 masks give 1024 + 16*q, undone by an exact fma with 1/16 and -64.
__device__ __forceinline__ void unpack_u4(uint32_t w, __half2 (&p)[4]) {
  const uint32_t MAG = 0x64006400u;
  uint32_t w8 = w >> 8;
  uint32_t t0 = (w & 0x000F000Fu) | MAG;
  uint32_t t1 = (w & 0x00F000F0u) | MAG;
  uint32_t t2 = (w8 & 0x000F000Fu) | MAG;
  uint32_t t3 = (w8 & 0x00F000F0u) | MAG;
  const __half2 k1024 = u32_as_h2(0x64006400u);  // 1024
  const __half2 k16th = u32_as_h2(0x2C002C00u);  // 1/16
  const __half2 km64 = u32_as_h2(0xD400D400u);   // -64
  p[0] = __hsub2(u32_as_h2(t0), k1024);
  p[1] = hfma2_rn(u32_as_h2(t1), k16th, km64);
  p[2] = __hsub2(u32_as_h2(t2), k1024);
  p[3] = hfma2_rn(u32_as_h2(t3), k16th, km64);
}

// 8-bit codes of one word -> two half2 (q0, q2), (q1, q3), exact.
__device__ __forceinline__ void unpack_u8(uint32_t w, __half2 (&p)[2]) {
  const uint32_t MAG = 0x64006400u;
  const __half2 k1024 = u32_as_h2(0x64006400u);
  p[0] = __hsub2(u32_as_h2((w & 0x00FF00FFu) | MAG), k1024);
  p[1] = __hsub2(u32_as_h2(((w >> 8) & 0x00FF00FFu) | MAG), k1024);
}

// ---------------------------------------------------------------- memory

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// ---------------------------------------------------------------- async copy / mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory loads by 32-bit shared-window address (no generic-to-shared
// conversion per access).
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(tx) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread is parked by the
// hardware until the phase completes (or the hint, in ns, runs out) instead of
// re-polling the barrier, which would take shared-memory issue slots from the
// warps and the TMA writes that do the work.
constexpr uint32_t MBAR_SUSPEND_NS = 20000;

// Non-blocking probe of a phase (no suspension): for waits whose wake-up
// latency matters more than the issue slots a spin takes.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(MBAR_SUSPEND_NS)
      : "memory");
  return ok != 0;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`
// (both addresses and the size multiples of 16 bytes; no multicast).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits that cannot hang the GPU: give up after `limit_ns` (or as soon as
// another warp of the CTA gave up), raise *abort and report false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort = 1;
        return false;
      }
    }
  }
}

// The same wait for a whole warp (every lane passes the same barrier and
// parity): the result is a vote, identical on all lanes, so the caller's
// branches on it stay warp-uniform.  The first poll is the fast path.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                               uint64_t limit_ns) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort, limit_ns));
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- tensor core

// D(16x8, fp32) += A(16x16, fp16 row) * B(16x8, fp16 col)
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  // a pure register op: not volatile, so the compiler may schedule it freely
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- misc

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + expf(-x)); }

}  // namespace sc
