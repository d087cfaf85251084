// sc_qlinear_noalloc: the quantized linear with its split-K scratch in a
// fixed, statically allocated device array instead of a caller workspace.
//
// Some callers have no device allocator to hand, or must not touch one on
// the call path: a thin C / FFI binding that links only this library and
// the CUDA runtime (no torch, no caching allocator), or a serving loop whose
// HBM is already fully reserved for weights and the KV cache, where a
// failed or stalling allocation mid-request is worse than a clear refusal.
// This entry point allocates nothing; it runs the same kernels as
// sc_qlinear with the scratch below.
//
// Limits and rules:
//   * the scratch holds NOALLOC_SCRATCH_BYTES (4 MiB); a shape whose split-K
//     plan (for its own group size) needs more is refused with
//     SC_ERR_WORKSPACE before anything is launched;
//   * nothing in the scratch has to start at zero: the split-K partials are
//     each written once before the reduce kernel reads them, so no clearing
//     is done;
//   * the first call on a device looks up the scratch's device address
//     (cudaGetSymbolAddress) and caches it; make that first call before any
//     stream capture;
//   * there is one scratch per device: calls that overlap in time on the
//     same device (other streams, other host threads) race on it.
#include <mutex>

#include "sc_common.cuh"

namespace sc {

constexpr size_t NOALLOC_SCRATCH_BYTES = 4u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

static void* g_noalloc_addr[64];
static std::mutex g_noalloc_mu;

static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  SC_REQUIRE(e == cudaSuccess, SC_ERR_CUDA, "qlinear_noalloc: cudaGetDevice failed (%s)", cudaGetErrorString(e));
  SC_REQUIRE(dev >= 0 && dev < 64, SC_ERR_ARG, "qlinear_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    SC_REQUIRE(e == cudaSuccess && p, SC_ERR_CUDA, "qlinear_noalloc: cudaGetSymbolAddress failed (%s)",
               cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return SC_OK;
}

}  // namespace sc

extern "C" {

int sc_qlinear_noalloc(const void* x, int x_dtype, int M, int K, int ldx, const uint32_t* wq,
                       const uint16_t* scales, const uint16_t* biases, int N, int group_size, int bits,
                       const uint16_t* bias, void* y, int y_dtype, int ldy, cudaStream_t stream) {
  // the real plan of this shape and group (what sc_qlinear would ask for), so
  // no shape that fits is refused; computed before anything is launched
  const bool tma_ok = ((uintptr_t)wq % 16 == 0) && ((uintptr_t)scales % 16 == 0) && ((uintptr_t)biases % 16 == 0);
  const size_t need = sc::qlinear_workspace_need(M, K, N, group_size, bits, tma_ok);
  SC_REQUIRE(need <= sc::NOALLOC_SCRATCH_BYTES, SC_ERR_WORKSPACE,
             "qlinear_noalloc: shape M=%d K=%d N=%d bits=%d may need %zu bytes of scratch; the static scratch "
             "holds %zu (use sc_qlinear with a caller workspace)",
             M, K, N, bits, need, sc::NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int st = sc::noalloc_scratch(&scratch);
  if (st != SC_OK) return st;
  return sc_qlinear(x, x_dtype, M, K, ldx, wq, scales, biases, N, group_size, bits, bias, y, y_dtype, ldy, scratch,
                    sc::NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
