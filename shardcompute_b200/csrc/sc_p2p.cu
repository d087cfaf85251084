// One-shot all-reduce and all-gather over NVLink peer memory, for the small
// per-token messages of tensor-parallel decode (a [B, hidden] fp32 partial
// after every row-parallel linear, the per-rank argmax pair after the LM
// head).  They replace the reference's TCP ring collectives
// (collectives/all_reduce.py:58-193, collectives/all_gather.py:54-162) where
// NCCL's ring / tree kernels are latency-bound: a 16 KB NCCL all-reduce costs
// ~22 us inside a CUDA graph on two B200s, one of these a few us.
//
// Transport.  Every rank owns one device arena (cudaMalloc, exported with
// cudaIpcGetMemHandle and mapped by every peer with cudaIpcOpenMemHandle).
// A message travels as "LL" lines of 16 bytes, {word0, epoch, word1, epoch}:
// the sender writes each line with one 16-byte volatile store straight into
// the receiver's arena, and the receiver polls the line until both epoch
// fields equal the current call's epoch.  An 8-byte half-line {word, epoch}
// is written atomically, so a matching epoch proves its payload word arrived;
// no fence or separate flag round trip is needed.
//
// Epochs.  Every call runs the same fixed grid (P2P_CTAS blocks); block c
// keeps its own call counter in the arena header and uses epoch = counter + 1.
// All ranks make the same sequence of calls, so block c of every rank agrees
// on the epoch.  Regions are double-buffered by epoch parity: a sender at
// call n writes buffer set n&1, which the receiver last read at call n-2;
// the sender only reaches call n after receiving the receiver's call n-1
// lines, which the receiver sends only after its call n-2 kernel completed
// (every kernel of the library waits on its predecessor with griddepcontrol
// before touching data).
//
// Failure.  Every poll is bounded (globaltimer, default 2 s).  A block that
// gives up raises the arena's error word and a host-mapped copy of it, and
// every later call skips its waits; sc_p2p_status reads the host copy without
// touching the GPU.  The results of the failed and all later calls are
// undefined; the host tears the transport down (sc_p2p_destroy) and falls
// back to NCCL or aborts.
#include <string.h>

#include "sc_p2p.cuh"

namespace sc {

constexpr int P2P_CTAS = 16;       // fixed grid: every call runs the same blocks
constexpr int P2P_THREADS = 256;

struct P2P {
  int world, rank, device;
  size_t max_bytes;     // largest payload per rank per call
  size_t region_bytes;  // LL bytes of one (buffer set, source rank) region
  char* arena;          // own arena: header + 2 x world regions
  char* peer[P2P_MAX_WORLD];
  bool mapped[P2P_MAX_WORLD];  // peer[q] came from cudaIpcOpenMemHandle
  int* host_err;               // host-mapped error word
  int* host_err_dev;           // its device address
  uint64_t timeout_ns;
};

// Payload word `wi` of a message of `count` elements of T (zero past the end).
template <typename T>
__device__ __forceinline__ uint32_t payload_word(const T* src, size_t count, size_t wi) {
  if constexpr (sizeof(T) == 4) {
    return wi < count ? reinterpret_cast<const uint32_t*>(src)[wi] : 0u;
  } else {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
    const size_t e = 2 * wi;
    const uint32_t lo = e < count ? s[e] : 0u;
    const uint32_t hi = e + 1 < count ? s[e + 1] : 0u;
    return lo | (hi << 16);
  }
}

// Block prologue shared by both collectives: wait for the predecessor, take
// this block's epoch, read the sticky error word.
__device__ __forceinline__ uint32_t p2p_begin(const P2PArgs& a, bool* skip) {
  __shared__ uint32_t s_ep;
  __shared__ int s_err;
  pdl_wait();
  if (threadIdx.x == 0) {
    const uint32_t e = a.ctr[blockIdx.x] + 1;
    a.ctr[blockIdx.x] = e;
    s_ep = e;
    s_err = *reinterpret_cast<volatile int*>(a.err);
  }
  __syncthreads();
  pdl_trigger();
  *skip = s_err != 0;
  return s_ep;
}

// Lines [l0, l1) of this block.
__device__ __forceinline__ void p2p_block_lines(size_t lines, size_t* l0, size_t* l1) {
  const size_t per = (lines + gridDim.x - 1) / gridDim.x;
  *l0 = min(lines, (size_t)blockIdx.x * per);
  *l1 = min(lines, *l0 + per);
}

__device__ __forceinline__ uint4* p2p_line(const P2PArgs& a, int arena_rank, int set, int src, size_t l) {
  return reinterpret_cast<uint4*>(a.data[arena_rank] + (size_t)(set * a.world + src) * a.region_bytes) + l;
}

// Sends lines [l0, l1) of `src` to every peer's region (set, rank).
template <typename T>
__device__ __forceinline__ void p2p_push(const P2PArgs& a, const T* src, size_t count, size_t l0, size_t l1,
                                         int set, uint32_t ep) {
  for (size_t l = l0 + threadIdx.x; l < l1; l += blockDim.x) {
    const uint32_t w0 = payload_word(src, count, 2 * l), w1 = payload_word(src, count, 2 * l + 1);
    for (int k = 1; k < a.world; ++k) {
      const int dst = (a.rank + k) % a.world;  // staggered so ranks do not all hit one peer first
      st_volatile_v4(p2p_line(a, dst, set, a.rank, l), w0, ep, w1, ep);
    }
  }
}

// Polls one line of this rank's region (set, src) until it carries epoch `ep`
// (or the wait gives up: error raised, *skip set, whatever is there returned).
__device__ __forceinline__ uint4 p2p_recv_line(const P2PArgs& a, int set, int src, size_t l, uint32_t ep,
                                               bool* skip, uint64_t* t0) {
  const uint4* p = p2p_line(a, a.rank, set, src, l);
  uint4 v = ld_volatile_v4(p);
  if ((v.y == ep && v.w == ep) || *skip) return v;
  if (*t0 == 0) *t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    v = ld_volatile_v4(p);
    if (v.y == ep && v.w == ep) return v;
    if ((i & 127) == 0) {
      if (*reinterpret_cast<volatile int*>(a.err) != 0 || globaltimer_ns() - *t0 > a.timeout_ns) {
        p2p_raise(a);
        *skip = true;
        return v;
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ void add_word(float* acc, uint32_t w) {
  if constexpr (sizeof(T) == 4) {
    acc[0] += __uint_as_float(w);
  } else {
    const __half2 h = u32_as_h2(w);
    acc[0] += __low2float(h);
    acc[1] += __high2float(h);
  }
}

template <typename T>
__device__ __forceinline__ void store_elems(T* dst, size_t count, size_t e0, const float* v, int n) {
  for (int i = 0; i < n; ++i) {
    if (e0 + i < count) {
      if constexpr (sizeof(T) == 4) {
        dst[e0 + i] = v[i];
      } else {
        dst[e0 + i] = __float2half_rn(v[i]);
      }
    }
  }
}

// recv = sum over ranks (in rank order, fp32 accumulation) of send.
// recv may alias send: every thread reads and writes only its own lines.
template <typename T>
__global__ void __launch_bounds__(P2P_THREADS) p2p_allreduce_kernel(const __grid_constant__ P2PArgs a, const T* send, T* recv,
                                                                    size_t count) {
  bool skip;
  const uint32_t ep = p2p_begin(a, &skip);
  const int set = ep & 1;
  constexpr int EPW = 4 / sizeof(T);  // elements per payload word
  const size_t words = (count + EPW - 1) / EPW, lines = (words + 1) / 2;
  size_t l0, l1;
  p2p_block_lines(lines, &l0, &l1);
  p2p_push(a, send, count, l0, l1, set, ep);
  uint64_t t0 = 0;
  for (size_t l = l0 + threadIdx.x; l < l1; l += blockDim.x) {
    float acc[2 * EPW];
#pragma unroll
    for (int i = 0; i < 2 * EPW; ++i) acc[i] = 0.f;
    for (int q = 0; q < a.world; ++q) {
      uint32_t w0, w1;
      if (q == a.rank) {
        w0 = payload_word(send, count, 2 * l);
        w1 = payload_word(send, count, 2 * l + 1);
      } else {
        const uint4 v = p2p_recv_line(a, set, q, l, ep, &skip, &t0);
        w0 = v.x;
        w1 = v.z;
      }
      add_word<T>(acc, w0);
      add_word<T>(acc + EPW, w1);
    }
    store_elems(recv, count, 2 * l * EPW, acc, 2 * EPW);
  }
}

// recv[q * count + i] = send_q[i] for every rank q (4-byte elements).
__global__ void __launch_bounds__(P2P_THREADS) p2p_allgather_kernel(const __grid_constant__ P2PArgs a, const uint32_t* send,
                                                                    uint32_t* recv, size_t count) {
  bool skip;
  const uint32_t ep = p2p_begin(a, &skip);
  const int set = ep & 1;
  const size_t lines = (count + 1) / 2;
  size_t l0, l1;
  p2p_block_lines(lines, &l0, &l1);
  p2p_push(a, send, count, l0, l1, set, ep);
  uint64_t t0 = 0;
  for (size_t l = l0 + threadIdx.x; l < l1; l += blockDim.x) {
    for (int q = 0; q < a.world; ++q) {
      uint32_t w0, w1;
      if (q == a.rank) {
        w0 = payload_word(send, count, 2 * l);
        w1 = payload_word(send, count, 2 * l + 1);
      } else {
        const uint4 v = p2p_recv_line(a, set, q, l, ep, &skip, &t0);
        w0 = v.x;
        w1 = v.z;
      }
      uint32_t* dst = recv + (size_t)q * count;
      dst[2 * l] = w0;
      if (2 * l + 1 < count) dst[2 * l + 1] = w1;
    }
  }
}

static P2PArgs p2p_args(const P2P* h) {
  P2PArgs a = {};
  for (int q = 0; q < h->world; ++q) a.data[q] = h->peer[q] + P2P_HDR;
  a.ctr = reinterpret_cast<uint32_t*>(h->arena);
  a.err = reinterpret_cast<int*>(h->arena + P2P_ERR_OFF);
  a.host_err = h->host_err_dev;
  a.region_bytes = h->region_bytes;
  a.timeout_ns = h->timeout_ns;
  a.world = h->world;
  a.rank = h->rank;
  return a;
}

static int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SC_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return SC_ERR_CUDA;
}

static int p2p_check_device(const P2P* h) {
  int dev = -1;
  cudaGetDevice(&dev);
  SC_REQUIRE(dev == h->device, SC_ERR_ARG, "p2p: current device %d, transport created on %d", dev, h->device);
  return SC_OK;
}

// Writes the transport's kernel-side view into its arena header (for kernels
// that take it by address) once every peer is mapped.
static int p2p_publish(const P2P* h) {
  for (int q = 0; q < h->world; ++q)
    if (!h->peer[q]) return SC_OK;
  const P2PArgs a = p2p_args(h);
  return cuda_status(cudaMemcpy(h->arena + P2P_ARGS_OFF, &a, sizeof(a), cudaMemcpyHostToDevice),
                     "p2p: publishing the transport's arguments");
}

int p2p_args_of(void* p2p, P2PArgs* out, size_t* max_bytes, const P2PArgs** dev_args) {
  SC_REQUIRE(p2p && out, SC_ERR_ARG, "p2p: null transport");
  const P2P* h = static_cast<const P2P*>(p2p);
  for (int q = 0; q < h->world; ++q) SC_REQUIRE(h->peer[q], SC_ERR_ARG, "p2p: rank %d not mapped", q);
  if (int st = p2p_check_device(h)) return st;
  *out = p2p_args(h);
  if (max_bytes) *max_bytes = h->max_bytes;
  if (dev_args) *dev_args = reinterpret_cast<const P2PArgs*>(h->arena + P2P_ARGS_OFF);
  return SC_OK;
}

}  // namespace sc

extern "C" {

size_t sc_p2p_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int sc_p2p_create(int world, int rank, size_t max_bytes, void** p2p_out, void* handle_out, size_t handle_bytes) {
  using namespace sc;
  SC_REQUIRE(p2p_out && handle_out, SC_ERR_ARG, "p2p_create: null pointer");
  SC_REQUIRE(world >= 2 && world <= P2P_MAX_WORLD && rank >= 0 && rank < world, SC_ERR_SHAPE,
             "p2p_create: rank %d of world %d (2..%d ranks)", rank, world, P2P_MAX_WORLD);
  SC_REQUIRE(max_bytes >= 8 && max_bytes <= ((size_t)256 << 20), SC_ERR_SHAPE,
             "p2p_create: max_bytes %zu outside [8, 256 MiB]", max_bytes);
  SC_REQUIRE(handle_bytes >= sizeof(cudaIpcMemHandle_t), SC_ERR_ARG, "p2p_create: handle buffer of %zu bytes < %zu",
             handle_bytes, sizeof(cudaIpcMemHandle_t));
  P2P* h = new P2P();
  h->world = world;
  h->rank = rank;
  cudaGetDevice(&h->device);
  h->max_bytes = max_bytes;
  h->region_bytes = ((max_bytes + 7) / 8 * 16 + 255) / 256 * 256;  // 16-byte line per 8 payload bytes
  h->timeout_ns = 2000000000ull;
  const size_t bytes = P2P_HDR + 2 * (size_t)world * h->region_bytes;
  int st = cuda_status(cudaMalloc(&h->arena, bytes), "p2p_create: cudaMalloc");
  if (st == SC_OK) st = cuda_status(cudaMemset(h->arena, 0, bytes), "p2p_create: cudaMemset");
  if (st == SC_OK)
    st = cuda_status(cudaHostAlloc(reinterpret_cast<void**>(&h->host_err), sizeof(int), cudaHostAllocMapped),
                     "p2p_create: cudaHostAlloc");
  if (st == SC_OK) {
    *h->host_err = 0;
    st = cuda_status(cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->host_err_dev), h->host_err, 0),
                     "p2p_create: cudaHostGetDevicePointer");
  }
  cudaIpcMemHandle_t ipc;
  if (st == SC_OK) st = cuda_status(cudaIpcGetMemHandle(&ipc, h->arena), "p2p_create: cudaIpcGetMemHandle");
  if (st == SC_OK) st = cuda_status(cudaDeviceSynchronize(), "p2p_create: synchronize");
  if (st != SC_OK) {
    if (h->arena) cudaFree(h->arena);
    if (h->host_err) cudaFreeHost(h->host_err);
    delete h;
    return st;
  }
  for (int q = 0; q < P2P_MAX_WORLD; ++q) h->peer[q] = nullptr;
  h->peer[rank] = h->arena;
  memcpy(handle_out, &ipc, sizeof(ipc));
  *p2p_out = h;
  return SC_OK;
}

// Every rank's arena as mapped in this process (bases[world]) and the arena
// size, for a kernel that lays out its own lines in a transport it owns.
int sc_p2p_arenas(void* p2p, void** bases, size_t* arena_bytes) {
  using namespace sc;
  SC_REQUIRE(p2p && bases && arena_bytes, SC_ERR_ARG, "p2p_arenas: null pointer");
  P2P* h = static_cast<P2P*>(p2p);
  for (int q = 0; q < h->world; ++q) {
    SC_REQUIRE(h->peer[q], SC_ERR_ARG, "p2p_arenas: rank %d's arena is not mapped (call sc_p2p_open first)", q);
    bases[q] = h->peer[q];
  }
  *arena_bytes = P2P_HDR + 2 * (size_t)h->world * h->region_bytes;
  return SC_OK;
}

int sc_p2p_open(void* p2p, const void* handles, size_t handle_bytes) {
  using namespace sc;
  SC_REQUIRE(p2p && handles, SC_ERR_ARG, "p2p_open: null pointer");
  P2P* h = static_cast<P2P*>(p2p);
  SC_REQUIRE(handle_bytes >= sizeof(cudaIpcMemHandle_t), SC_ERR_ARG, "p2p_open: handle stride %zu < %zu",
             handle_bytes, sizeof(cudaIpcMemHandle_t));
  if (int st = p2p_check_device(h)) return st;
  for (int q = 0; q < h->world; ++q) {
    if (q == h->rank || h->peer[q]) continue;
    cudaIpcMemHandle_t ipc;
    memcpy(&ipc, static_cast<const char*>(handles) + (size_t)q * handle_bytes, sizeof(ipc));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("p2p_open: cudaIpcOpenMemHandle of rank %d: %s", q, cudaGetErrorString(e));
      return SC_ERR_CUDA;
    }
    h->peer[q] = static_cast<char*>(ptr);
    h->mapped[q] = true;
  }
  return p2p_publish(h);
}

int sc_p2p_open_loopback(void* p2p) {
  using namespace sc;
  SC_REQUIRE(p2p, SC_ERR_ARG, "p2p_open_loopback: null pointer");
  P2P* h = static_cast<P2P*>(p2p);
  for (int q = 0; q < h->world; ++q)
    if (!h->peer[q]) h->peer[q] = h->arena;
  return p2p_publish(h);
}

int sc_p2p_set_timeout(void* p2p, uint64_t timeout_ns) {
  using namespace sc;
  SC_REQUIRE(p2p, SC_ERR_ARG, "p2p_set_timeout: null pointer");
  SC_REQUIRE(timeout_ns >= 1000000ull && timeout_ns <= 60000000000ull, SC_ERR_ARG,
             "p2p_set_timeout: %llu ns outside [1 ms, 60 s]", (unsigned long long)timeout_ns);
  static_cast<P2P*>(p2p)->timeout_ns = timeout_ns;
  return p2p_publish(static_cast<P2P*>(p2p));
}

int sc_p2p_status(void* p2p, int* timed_out) {
  using namespace sc;
  SC_REQUIRE(p2p && timed_out, SC_ERR_ARG, "p2p_status: null pointer");
  *timed_out = *reinterpret_cast<volatile int*>(static_cast<P2P*>(p2p)->host_err);
  return SC_OK;
}

int sc_p2p_destroy(void* p2p) {
  using namespace sc;
  if (!p2p) return SC_OK;
  P2P* h = static_cast<P2P*>(p2p);
  int st = SC_OK;
  for (int q = 0; q < h->world; ++q) {
    if (h->mapped[q]) {
      const int s = cuda_status(cudaIpcCloseMemHandle(h->peer[q]), "p2p_destroy: cudaIpcCloseMemHandle");
      if (st == SC_OK) st = s;
    }
  }
  const int s1 = cuda_status(cudaFree(h->arena), "p2p_destroy: cudaFree");
  const int s2 = cuda_status(cudaFreeHost(h->host_err), "p2p_destroy: cudaFreeHost");
  if (st == SC_OK) st = s1 != SC_OK ? s1 : s2;
  delete h;
  return st;
}

int sc_p2p_allreduce(const void* send, void* recv, size_t count, int dtype, void* p2p, cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(p2p && send && recv, SC_ERR_ARG, "p2p_allreduce: null pointer");
  const P2P* h = static_cast<const P2P*>(p2p);
  SC_REQUIRE(dtype == SC_F32 || dtype == SC_F16, SC_ERR_UNSUPPORTED, "p2p_allreduce: dtype %d (f16 / f32 only)",
             dtype);
  for (int q = 0; q < h->world; ++q) SC_REQUIRE(h->peer[q], SC_ERR_ARG, "p2p_allreduce: rank %d not mapped", q);
  const size_t esz = dtype == SC_F32 ? 4 : 2;
  SC_REQUIRE(count * esz <= h->max_bytes, SC_ERR_SHAPE, "p2p_allreduce: %zu bytes > transport limit %zu",
             count * esz, h->max_bytes);
  SC_REQUIRE(((uintptr_t)send | (uintptr_t)recv) % esz == 0, SC_ERR_ARG, "p2p_allreduce: misaligned buffers");
  if (int st = p2p_check_device(h)) return st;
  if (count == 0) return SC_OK;
  const P2PArgs a = p2p_args(h);
  if (dtype == SC_F32)
    launch(p2p_allreduce_kernel<float>, dim3(P2P_CTAS), dim3(P2P_THREADS), 0, stream, a,
           static_cast<const float*>(send), static_cast<float*>(recv), count);
  else
    launch(p2p_allreduce_kernel<__half>, dim3(P2P_CTAS), dim3(P2P_THREADS), 0, stream, a,
           static_cast<const __half*>(send), static_cast<__half*>(recv), count);
  return check_launch("p2p_allreduce");
}

int sc_p2p_allgather(const void* send, void* recv, size_t count_per_rank, int dtype, void* p2p,
                     cudaStream_t stream) {
  using namespace sc;
  SC_REQUIRE(p2p && send && recv, SC_ERR_ARG, "p2p_allgather: null pointer");
  const P2P* h = static_cast<const P2P*>(p2p);
  SC_REQUIRE(dtype == SC_F32 || dtype == SC_I32, SC_ERR_UNSUPPORTED,
             "p2p_allgather: dtype %d (4-byte types only)", dtype);
  for (int q = 0; q < h->world; ++q) SC_REQUIRE(h->peer[q], SC_ERR_ARG, "p2p_allgather: rank %d not mapped", q);
  SC_REQUIRE(count_per_rank * 4 <= h->max_bytes, SC_ERR_SHAPE, "p2p_allgather: %zu bytes > transport limit %zu",
             count_per_rank * 4, h->max_bytes);
  SC_REQUIRE(((uintptr_t)send | (uintptr_t)recv) % 4 == 0, SC_ERR_ARG, "p2p_allgather: misaligned buffers");
  if (int st = p2p_check_device(h)) return st;
  if (count_per_rank == 0) return SC_OK;
  launch(p2p_allgather_kernel, dim3(P2P_CTAS), dim3(P2P_THREADS), 0, stream, p2p_args(h),
         static_cast<const uint32_t*>(send), static_cast<uint32_t*>(recv), count_per_rank);
  return check_launch("p2p_allgather");
}

}  // extern "C"
