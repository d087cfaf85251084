// Peer-memory transport pieces shared by the one-shot collectives
// (sc_p2p.cu) and the decode GEMV whose epilogue runs the row-parallel
// all-reduce itself (sc_qgemv.cu): the kernel-side view of a transport, the
// 16-byte "LL" line stores / loads and the bounded poll of an 8-byte
// {word, epoch} half line.  The protocol is described in sc_p2p.cu.
#pragma once

#include "sc_common.cuh"

namespace sc {

constexpr int P2P_MAX_WORLD = 8;
constexpr size_t P2P_HDR = 4096;   // per-block counters (up to 512), error word at 2048, P2PArgs at 3072
constexpr size_t P2P_ERR_OFF = 2048;
constexpr size_t P2P_ARGS_OFF = 3072;  // a device copy of the transport's P2PArgs, written when it is opened
constexpr int P2P_MAX_CTR = (int)(P2P_ERR_OFF / 4);

// A transport as its kernels see it.
struct P2PArgs {
  char* data[P2P_MAX_WORLD];  // LL regions of every rank's arena as mapped here
  uint32_t* ctr;              // this rank's per-block call counters
  int* err;                   // this rank's error word (device)
  int* host_err;              // host-mapped copy
  size_t region_bytes;
  uint64_t timeout_ns;
  int world, rank;
};

static_assert(sizeof(P2PArgs) <= P2P_HDR - P2P_ARGS_OFF, "P2PArgs must fit the arena header");

// The kernel-side view of a transport made by sc_p2p_create / sc_p2p_open,
// its largest message and the device copy of that view (in the arena's
// header); an error status for a null handle, a peer not mapped or another
// current device.
int p2p_args_of(void* p2p, P2PArgs* out, size_t* max_bytes, const P2PArgs** dev_args);

__device__ __forceinline__ void st_volatile_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_volatile_v2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ uint2 ld_volatile_v2(const void* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// Raise the transport's sticky error word and its host-mapped copy.
__device__ __forceinline__ void p2p_raise(const P2PArgs& a) {
  atomicExch(a.err, 1);
  *reinterpret_cast<volatile int*>(a.host_err) = 1;
  __threadfence_system();
}

// Polls the 8-byte half line {word, epoch} at p until it carries `ep`; gives
// up after the transport's timeout (counted from *t0, set on the first miss),
// raising the error word and setting *skip (later polls return at once).
__device__ __forceinline__ uint32_t p2p_recv_half(const P2PArgs& a, const void* p, uint32_t ep, bool* skip,
                                                  uint64_t* t0) {
  uint2 v = ld_volatile_v2(p);
  if (v.y == ep || *skip) return v.x;
  if (*t0 == 0) *t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    v = ld_volatile_v2(p);
    if (v.y == ep) return v.x;
    if ((i & 127) == 0 &&
        (*reinterpret_cast<volatile int*>(a.err) != 0 || globaltimer_ns() - *t0 > a.timeout_ns)) {
      p2p_raise(a);
      *skip = true;
      return v.x;
    }
  }
}

}  // namespace sc
