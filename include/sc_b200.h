/*
 * sc_b200.h -- C ABI of libsc_b200.so, the sm_100a kernels behind the
 * tensor-parallel quantized decode path of shardcompute.
 *
 * Conventions
 *   - Every entry point is extern "C", returns an int status (SC_OK = 0),
 *     takes device pointers + sizes + a cudaStream_t, and keeps no reference
 *     to any buffer after it returns.  Calls enqueue work on `stream` and do
 *     not synchronise; they are safe to capture in a CUDA graph.
 *   - Buffers are caller-owned.  Entry points that need scratch take a
 *     `workspace` pointer and size; the matching *_workspace_bytes() query
 *     gives the size.  Nothing here allocates device memory, except the
 *     peer-memory transport's arena (sc_p2p_create / sc_p2p_destroy) and the
 *     static scratch of sc_qlinear_noalloc.
 *   - fp16 tensors are passed as uint16_t*; dtype codes are SC_F16 / SC_F32.
 *   - The weight format is MLX's group-wise affine format that the reference
 *     stores in its shards: wq uint32 [rows, K*bits/32] with element j of a
 *     word at bits [bits*j, bits*(j+1)); scales/biases fp16 [rows, K/group];
 *     dequant w = scale*q + bias.
 *   - sc_last_error() returns a thread-local message for the last failure.
 *
 * Reference interfaces replaced (paths inside Aarjav0210/shardcompute):
 *   see the comment above each declaration.
 */
#ifndef SC_B200_H
#define SC_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_ABI_VERSION 1

enum sc_status {
  SC_OK = 0,
  SC_ERR_SHAPE = 1,       /* maps to ValueError in the Python layer */
  SC_ERR_CUDA = 2,        /* RuntimeError */
  SC_ERR_NCCL = 3,        /* RuntimeError */
  SC_ERR_TIMEOUT = 4,     /* TimeoutError */
  SC_ERR_ARG = 5,         /* ValueError (null pointer, bad enum) */
  SC_ERR_UNSUPPORTED = 6, /* NotImplementedError */
  SC_ERR_WORKSPACE = 7    /* ValueError: workspace too small */
};

enum sc_dtype { SC_F16 = 0, SC_F32 = 1, SC_I32 = 2, SC_U8 = 3 };  /* SC_U8: raw bytes (send / recv / broadcast) */

/* Epilogues of the fused quantized linear. */
enum sc_epilogue {
  SC_EPI_STORE = 0,    /* y = x.W^T (+ bias)                              */
  SC_EPI_RESIDUAL = 1, /* y = residual + x.W^T (+ bias); y may alias it   */
  SC_EPI_SWIGLU = 2    /* two segments: y = silu(x.W0^T) * (x.W1^T)       */
};

enum sc_reduce_op { SC_OP_SUM = 0, SC_OP_MAX = 1, SC_OP_MIN = 2, SC_OP_AVG = 3 };

int sc_abi_version(void);
const char* sc_status_name(int status);
const char* sc_last_error(void);
/* Number of kernels this library has enqueued in this process (a kernel
 * inside a captured CUDA graph counts once, at capture).  Instrumentation
 * for benchmarks; no counterpart in the reference. */
unsigned long long sc_launch_count(void);

/* ------------------------------------------------------------------ K1 --
 * Quantized linear: y[M, N] = x[M, K] . dequant(wq, scales, biases)^T + bias
 * Replaces the mx.quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size, bits) calls of
 *   parallel/quantized_linear.py:168-176  QuantizedColumnParallelLinear.forward
 *   parallel/quantized_linear.py:206-214  QuantizedColumnParallelLinear.forward_sync
 *   parallel/quantized_linear.py:435-443  QuantizedRowParallelLinear.forward (partial)
 *   parallel/quantized_linear.py:472-480  QuantizedRowParallelLinear.forward_partial
 * and the tied LM head matmul of parallel/transformer.py:565-569.
 *   x: fp16 or fp32 [M, ldx]; bias: fp16 [N] or NULL; y: fp16 or fp32 [M, ldy].
 *   bits in {4, 8}; group_size in {32, 64, 128}; K % group_size == 0.
 *   Any M >= 1.  Up to 16 rows run passes of the decode GEMV (exact
 *   weights; 4 rows per pass, 2 at 4-bit group 64, 1 at group 32); more
 *   rows run the tcgen05 tensor-core GEMM (sc_qgemm) when K % 64 == 0 and
 *   the workspace holds its scratch, else GEMV passes.
 *   sc_qlinear_workspace_bytes covers every case.
 */
size_t sc_qlinear_workspace_bytes(int M, int K, int N, int bits);
int sc_qlinear(const void* x, int x_dtype, int M, int K, int ldx,
               const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
               int N, int group_size, int bits, const uint16_t* bias,
               void* y, int y_dtype, int ldy,
               void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* K2: the tensor-core dequant-GEMM behind sc_qlinear for more than 16 rows
 * of x (prefill, batched decode past batch 16): tcgen05.mma kind::f16 with fp32 accumulators in
 * TMEM; weights carried exactly as fp16 high + low parts, x likewise.  Same
 * arguments and epilogues as sc_qlinear_fused.  Replaces the prefill-shaped
 * mx.quantized_matmul calls (parallel/quantized_linear.py:168-176, 206-214,
 * parallel/transformer.py:639).  K % 64 == 0; stacked weight segments a
 * multiple of 128 rows (the last excepted).  Scratch: x's two fp16 parts and,
 * for SwiGLU, the [M, 2N] gate|up product. */
size_t sc_qgemm_workspace_bytes(int M, int K, int N, int epilogue);
int sc_qgemm(const void* x, int x_dtype, int M, int K, int ldx, const uint16_t* norm_weight, float norm_eps,
             int nseg, const uint32_t* const* wq, const uint16_t* const* scales, const uint16_t* const* biases,
             const int* seg_rows, int group_size, int bits, const uint16_t* bias, int epilogue, void* y,
             int y_dtype, int ldy, const float* residual, int ldr, void* workspace, size_t workspace_bytes,
             cudaStream_t stream);
/* Device error word of the tensor-core GEMM: nonzero after a bounded wait
 * gave up (the output is then undefined).  reset != 0 clears it. */
int sc_qgemm_device_error(int reset);

/* sc_qlinear without a caller workspace: its split-K scratch is a fixed
 * 4 MiB array the library allocates statically on each device.  No
 * counterpart in the reference.  For callers that cannot allocate on the
 * call path (an FFI binding with no device allocator of its own; a serving
 * loop whose HBM is fully reserved).  Shapes whose split-K plan (for
 * their own group size) needs more than 4 MiB are refused with
 * SC_ERR_WORKSPACE before any launch.  The first call on a device looks the
 * scratch up; make it before any stream capture.  One scratch per device:
 * calls overlapping in time on one device race. */
int sc_qlinear_noalloc(const void* x, int x_dtype, int M, int K, int ldx,
                       const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                       int N, int group_size, int bits, const uint16_t* bias,
                       void* y, int y_dtype, int ldy, cudaStream_t stream);

/* Device-side error word of the quantized-linear kernels: nonzero after a
 * kernel gave up on a bounded wait (it then stops without touching the
 * output; while the word is set, split-K passes leave y untouched too).
 * Synchronises with the device; reset != 0 clears it.  No reference
 * counterpart (the reference has no device code). */
int sc_qgemv_device_error(int reset);
/* In-step timing of the decode GEMV: the sc_qlinear* launches this host
 * thread makes after this call carry `pair` (two uint64 in device memory,
 * preset to {UINT64_MAX, 0}); the decode kernel atomically lowers pair[0] to
 * the %globaltimer (ns) at which its first consumer passed the dependency
 * wait and raises pair[1] to its last CTA's exit (or its split-K reduce's).
 * No event is recorded, so programmatic dependent launch stays on.  NULL
 * stops it. */
int sc_qgemv_probe_stamps(unsigned long long* pair);

/* Fused form used by the decode engine (no reference counterpart as one
 * call; it fuses the reference's RMSNorm -> q/k/v or gate/up linears ->
 * SiLU*mul, and linear -> residual add, parallel/transformer.py:240-252,
 * parallel/mlp.py:239-245).
 *   norm_weight: fp16 [K] or NULL; when set, each x row is RMS-normalised
 *     (x / sqrt(mean(x^2) + eps) * w) before the product.
 *   nseg segments (1..3) share x; for SC_EPI_STORE / SC_EPI_RESIDUAL their
 *   rows are concatenated along N (y has sum(seg_rows) columns); for
 *   SC_EPI_SWIGLU nseg must be 2 with equal rows and y = silu(y0) * y1.
 *   residual: fp32 [M, ldr] (SC_EPI_RESIDUAL only). */
int sc_qlinear_fused(const void* x, int x_dtype, int M, int K, int ldx,
                     const uint16_t* norm_weight, float norm_eps,
                     int nseg, const uint32_t* const* wq, const uint16_t* const* scales,
                     const uint16_t* const* biases, const int* seg_rows,
                     int group_size, int bits, const uint16_t* bias, int epilogue,
                     void* y, int y_dtype, int ldy, const float* residual, int ldr,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* sc_qlinear_fused that also pulls the NEXT kernel's weights into L2: up to
 * 12 regions (pf_ptrs / pf_bytes, at most pf_max_bytes in total, 0 = no
 * cap; starts rounded up and lengths down to 16 bytes).  The decode kernel
 * (M <= 4 rows) issues them from each CTA's copy engine as soon as that CTA's
 * own last weight tile has landed, so HBM keeps streaming through the
 * consumers' drain, the kernel boundary and the next kernel's start; other
 * passes ignore the list.  A hint only: results do not depend on it.  No
 * reference counterpart (the reference streams weights through MLX). */
int sc_qlinear_fused_prefetch(const void* x, int x_dtype, int M, int K, int ldx,
                              const uint16_t* norm_weight, float norm_eps,
                              int nseg, const uint32_t* const* wq, const uint16_t* const* scales,
                              const uint16_t* const* biases, const int* seg_rows,
                              int group_size, int bits, const uint16_t* bias, int epilogue,
                              void* y, int y_dtype, int ldy, const float* residual, int ldr,
                              void* workspace, size_t workspace_bytes,
                              const void* const* pf_ptrs, const size_t* pf_bytes, int pf_n,
                              size_t pf_max_bytes, cudaStream_t stream);

/* Row-parallel quantized linear with its all-reduce in the GEMV epilogue:
 * y[M, N] (fp32, ldy = N) = the sum over the transport's ranks, in rank
 * order from zero, of each rank's x.W_r^T (+ bias) (+ residual where it is
 * passed: rank 0 in tensor-parallel decode) -- the bits sc_qlinear_fused
 * followed by sc_p2p_allreduce gives, on every rank.  Each CTA pushes its
 * outputs to every peer as {value, epoch} half lines over NVLink and sums
 * its rows from the ranks' lines, so no all-reduce launch follows.  y may
 * alias residual.  Replaces QuantizedRowParallelLinear.forward's quantized
 * matmul + all_reduce (parallel/quantized_linear.py:419-455, the all-reduce
 * at 446-447).  p2p: a transport (sc_p2p_create + sc_p2p_open) reserved for
 * these calls -- their per-CTA epochs live in its header -- whose max_bytes
 * holds M * N * 4; every rank makes the same sequence of calls.  Returns
 * SC_ERR_UNSUPPORTED before any launch when the shape does not run as one
 * unsplit decode-GEMV pass with one output per consumer thread (batch 1-2
 * at 4-bit g64, up to 4 at 8-bit); the caller then runs sc_qlinear_fused
 * and sc_p2p_allreduce.  Polls are bounded like sc_p2p_allreduce's (the
 * transport's error word, sc_p2p_status). */
int sc_qlinear_allreduce(const void* x, int x_dtype, int M, int K, int ldx, const uint32_t* wq,
                         const uint16_t* scales, const uint16_t* biases, int N, int group_size, int bits,
                         const uint16_t* bias, float* y, const float* residual, void* p2p,
                         cudaStream_t stream);

/* Prefetch up to 12 device regions into L2 (at most max_bytes in total, 0 =
 * no cap) without waiting for them.  The decode step issues it right after a
 * GEMV for the next GEMV's weights, so HBM keeps streaming through kernel
 * boundaries and the attention kernels in between.  Region starts are
 * rounded up to 16 bytes.  No reference counterpart (the reference streams
 * weights through MLX with no prefetch). */
int sc_l2_prefetch(const void* const* ptrs, const size_t* bytes, int n, size_t max_bytes,
                   cudaStream_t stream);

/* ------------------------------------------------------------------ K3 --
 * Vocab-split embedding gather.  Replaces QuantizedParallelEmbedding.forward
 * before its all-reduce (parallel/embedding.py:322-356): local = id - v0,
 * rows with id outside [v0, v1) are zero, others are dequantized exactly
 * (fp16 of scale*q + bias, one rounding).  The table holds v1 - v0 rows.
 * out: fp16 or fp32 [n, H]. */
int sc_embed_gather_q(const int32_t* ids, int n, const uint32_t* wq, const uint16_t* scales,
                      const uint16_t* biases, int vocab_start, int vocab_end, int H,
                      int group_size, int bits, void* out, int out_dtype, cudaStream_t stream);
/* fp16-table variant of the same masked gather (vocab-split fp16 table). */
int sc_embed_gather_f16(const int32_t* ids, int n, const uint16_t* table, int vocab_start,
                        int vocab_end, int H, void* out, int out_dtype, cudaStream_t stream);

/* mx.dequantize of a whole table (QuantizedParallelEmbedding.dequantize_weight,
 * parallel/embedding.py:369-379): out fp16 [rows, K]. */
int sc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                  int rows, int K, int group_size, int bits, uint16_t* out, cudaStream_t stream);
/* Group-wise affine quantization (the mx.quantize calls of
 * parallel/quantized_linear.py:116,353 and parallel/embedding.py:303):
 * per group bias = min, scale = (max - min) / (2^bits - 1), both rounded to
 * fp16, q = clamp(rint((w - bias) / scale)).  w: fp16 [rows, K]. */
int sc_quantize(const uint16_t* w, int rows, int K, int group_size, int bits,
                uint32_t* wq, uint16_t* scales, uint16_t* biases, cudaStream_t stream);

/* ------------------------------------------------------------------ K4 --
 * RoPE + KV append.  Replaces RoPE.__call__ and the KV concatenation of
 * ParallelAttention.forward (parallel/attention.py:421-433).
 *   qkv: fp32 [B*S, (Hq + 2*Hkv) * hd], per token the q heads, then k, then v.
 *   *pos (device int32): cache length before this call; token s of every
 *   sequence goes to position *pos + s (all sequences share one length).
 *   Positions at or past Lmax / max_pos are not written.
 *   cos_tab/sin_tab: fp32 [max_pos, hd/2].
 *   q_out: fp32 [B*S, Hq*hd]; k_cache/v_cache: fp32 [B, Hkv, Lmax, hd] (fp32 as the
 *   reference's cache is: RoPE's fp32 tables promote k, and v follows the fp32 hidden state). */
int sc_rope_append(const float* qkv, int B, int S, int Hq, int Hkv, int hd,
                   const int32_t* pos, const float* cos_tab, const float* sin_tab, int max_pos,
                   float* q_out, float* k_cache, float* v_cache, int Lmax,
                   cudaStream_t stream);

/* Split-KV GQA flash-decode over the preallocated cache.  Replaces
 * parallel/attention.py:436-466 (GQA repeat, q.k^T*scale, causal mask,
 * softmax, @v).  Query s of sequence b sees keys [0, min(*pos + s, Lmax-1)].
 *   q: fp32 [B*S, Hq*hd]; out: fp16 or fp32 [B*S, Hq*hd]; splits 1..64. */
size_t sc_flash_decode_workspace_bytes(int B, int S, int Hq, int hd, int splits);
int sc_flash_decode(const float* q, const float* k_cache, const float* v_cache,
                    const int32_t* pos, int B, int S, int Hq, int Hkv, int hd, int Lmax,
                    float scale, int splits, void* out, int out_dtype,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Fused decode attention for one new token per sequence (S = 1): RoPE of
 * q and of the new k at position *pos, append of k and v to the cache, and
 * split-KV attention over positions [0, *pos] with the splits merged by the
 * last CTA of each (sequence, kv head) -- the work of sc_rope_append +
 * sc_flash_decode (parallel/attention.py:421-466) in one launch.
 *   qkv: fp32 [B, (Hq + 2*Hkv) * hd]; caches fp32 [B, Hkv, Lmax, hd];
 *   out: fp16 or fp32 [B, Hq*hd]; splits 1..64; workspace:
 *   sc_attn_decode_workspace_bytes;
 *   tickets: int32 [B*Hkv], zero before the first call and left zero by
 *   every call (the split merge counts arrivals in it). */
size_t sc_attn_decode_workspace_bytes(int B, int Hq, int hd, int splits);
/* Device-side error word of sc_attn_decode: nonzero after a CTA gave up
 * waiting for its K/V tiles (bounded wait; its output is then undefined).
 * Synchronises with the device; reset != 0 clears it.  No reference
 * counterpart. */
int sc_attn_device_error(int reset);
int sc_attn_decode(const float* qkv, int B, int Hq, int Hkv, int hd, const int32_t* pos,
                   const float* cos_tab, const float* sin_tab, int max_pos,
                   float* k_cache, float* v_cache, int Lmax, float scale, int splits,
                   void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                   int32_t* tickets, cudaStream_t stream);

/* ------------------------------------------------------------------ K5 --
 * RMSNorm (parallel/transformer.py:46-61): y = x / sqrt(mean(x^2)+eps) * w. */
int sc_rmsnorm(const void* x, int x_dtype, int M, int H, const uint16_t* w, float eps,
               void* y, int y_dtype, cudaStream_t stream);
/* silu(gate) * up (parallel/mlp.py:161-162,245). */
int sc_silu_mul(const void* gate, const void* up, int in_dtype, size_t n, void* out,
                int out_dtype, cudaStream_t stream);
/* y = a + b elementwise (residual adds, parallel/transformer.py:246,252). */
int sc_add(const void* a, int a_dtype, const void* b, int b_dtype, size_t n, void* y,
           int y_dtype, cudaStream_t stream);

/* ------------------------------------------------------------------ K7 --
 * Greedy token (worker/executor.py:276-278) over vocab-split logits.
 * sc_argmax: per row of logits fp32 [M, ldl] (N columns) the max value and
 * its lowest index, plus index_offset, into val[M] / idx[M].
 * sc_argmax_merge: picks, per row, the best of `world` (val, idx) candidates
 * laid out [world, M] (largest value, lowest index on ties) and writes the
 * token to token_out[M]; when pos != NULL it also adds pos_advance to *pos. */
size_t sc_argmax_workspace_bytes(int M, int N);
int sc_argmax(const float* logits, int M, int N, int ldl, int index_offset,
              float* val, int32_t* idx, void* workspace, size_t workspace_bytes,
              cudaStream_t stream);
int sc_argmax_merge(const float* vals, const int32_t* idxs, int M, int world,
                    int32_t* token_out, int32_t* pos, int pos_advance, cudaStream_t stream);

/* ------------------------------------------------------------ collectives --
 * NCCL over NVLink in place of the TCP ring collectives of
 * collectives/all_reduce.py:58-193 and collectives/all_gather.py:54-162
 * (Communicator.all_reduce / all_gather / broadcast,
 * collectives/communicator.py:259-507).  `comm` is an opaque handle. */
int sc_comm_unique_id(void* uid_out, size_t uid_bytes);
int sc_comm_init(const void* uid, size_t uid_bytes, int world, int rank, void** comm_out);
int sc_comm_destroy(void* comm);
int sc_comm_abort(void* comm);
/* Non-blocking health check: *async_error = NCCL's asynchronous error code. */
int sc_comm_poll(void* comm, int* async_error);
int sc_allreduce(const void* send, void* recv, size_t count, int dtype, int op, void* comm,
                 cudaStream_t stream);
int sc_allgather(const void* send, void* recv, size_t count_per_rank, int dtype, void* comm,
                 cudaStream_t stream);
int sc_broadcast(const void* send, void* recv, size_t count, int dtype, int root, void* comm,
                 cudaStream_t stream);
/* Point-to-point (Communicator.send / recv, collectives/communicator.py:520-561,
 * and the pipeline stage transfers of worker/executor.py:376-479): a rank's
 * sc_send to `peer` matches that peer's sc_recv of the same count and dtype. */
int sc_send(const void* buf, size_t count, int dtype, int peer, void* comm, cudaStream_t stream);
int sc_recv(void* buf, size_t count, int dtype, int peer, void* comm, cudaStream_t stream);

/* ------------------------------------------------------ NVLink peer memory --
 * One-shot all-reduce / all-gather through peer memory for the small
 * per-token messages of decode (same reference interfaces as above:
 * collectives/all_reduce.py:58-193, collectives/all_gather.py:54-162); the
 * Python Communicator uses them instead of NCCL for messages up to max_bytes.
 * Each rank owns an IPC-exported device arena (the one allocation of this
 * library, made by sc_p2p_create and freed by sc_p2p_destroy).  Setup:
 * sc_p2p_create on every rank -> exchange the handle bytes (host store) ->
 * sc_p2p_open with all ranks' handles in rank order (own entry ignored) ->
 * host barrier before the first call.  Every rank must make the same
 * sequence of calls (same counts), like any collective, and must not
 * destroy its transport while a peer may still send (host barrier first).
 * Waits are bounded (sc_p2p_set_timeout, default 2 s); after a timeout
 * sc_p2p_status reports 1 (read from host memory, no GPU call) and results
 * are undefined until the transport is recreated.  All-reduce: sum in rank
 * order with fp32 accumulation, f16 / f32, recv may alias send.  All-gather:
 * recv[q * count + i] = rank q's send[i], 4-byte dtypes (f32 / i32). */
size_t sc_p2p_handle_bytes(void);
int sc_p2p_create(int world, int rank, size_t max_bytes, void** p2p_out, void* handle_out,
                  size_t handle_bytes);
int sc_p2p_open(void* p2p, const void* handles, size_t handle_bytes);
/* Maps every unmapped rank onto this process's own arena: nothing but this
 * process writes it, so a call waits for peers that never send.  Used to
 * test the bounded wait on one GPU. */
int sc_p2p_open_loopback(void* p2p);
int sc_p2p_set_timeout(void* p2p, uint64_t timeout_ns);
int sc_p2p_status(void* p2p, int* timed_out);
int sc_p2p_destroy(void* p2p);
int sc_p2p_allreduce(const void* send, void* recv, size_t count, int dtype, void* p2p,
                     cudaStream_t stream);
int sc_p2p_allgather(const void* send, void* recv, size_t count_per_rank, int dtype, void* p2p,
                     cudaStream_t stream);

/* ------------------------------------------------------------------ K7b --
 * Temperature + top-p sampling over vocab-split logits (worker/executor.py:
 * 270-306): logits / T, softmax, keep a token while the probability mass
 * above it is <= top_p, renormalise, draw with a uniform u per row (inverse
 * CDF over the kept tokens in vocabulary order).  A threshold found by a
 * 4-level radix select on the probabilities' bits replaces the sort, so
 * tensor-parallel ranks never gather the logits.
 *   sc_sample_topp: one rank holding the whole vocabulary (one launch).
 *   sc_sample_phase / sc_sample_combine: the same on each rank's vocab slice;
 *     between phases the caller exchanges the fields of the field-major state
 *     [8][B] at the start of the workspace (phase 0 -> all-gather field 0 and
 *     combine what=0; 1 -> all-reduce-sum field 1; every phase 2 (levels
 *     0..3) -> all-reduce-sum the [B][256] histograms that follow the state,
 *     then phase 3 of that level; 4 -> all-gather field 4 and combine what=1;
 *     5 -> all-reduce-sum field 7 and combine what=2, which writes tok).
 *   sc_sample_uniforms: B uniforms from (seed, a device counter advanced by
 *     one per call), the same on every rank. */
size_t sc_sample_workspace_bytes(int B);
int sc_sample_topp(const float* logits, int B, int V, int ld, float temperature, float top_p, const float* u,
                   int vocab_start, int32_t* tok, void* workspace, size_t workspace_bytes, cudaStream_t stream);
int sc_sample_phase(const float* logits, int B, int V, int ld, float temperature, float top_p, const float* u,
                    int vocab_start, int phase, int level, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream);
int sc_sample_combine(void* workspace, const float* gathered, int B, int world, int rank, int what, int32_t* tok,
                      cudaStream_t stream);
int sc_sample_uniforms(uint64_t seed, unsigned long long* counter, int B, float* u, cudaStream_t stream);

/* ----------------------------------------------------- persistent decode step --
 * One launch per greedy decode token of the tensor-parallel quantized Llama at
 * batch 1 (4-bit, group 64): the embedding gather, every layer's RMSNorm ->
 * q|k|v -> RoPE + KV append + attention -> o_proj + residual -> RMSNorm ->
 * gate|up + SiLU*mul -> down_proj + residual, the final RMSNorm, the tied LM
 * head and the greedy argmax.  Replaces, as one kernel, the per-token call
 * chain of ParallelTransformer.forward (parallel/transformer.py:516-577)
 * driven by ParallelExecutor.generate's greedy loop
 * (worker/executor.py:267-325); its collectives (the row-parallel all-reduces,
 * parallel/quantized_linear.py:446-447, parallel/mlp.py:252; the embedding
 * all-reduce, parallel/embedding.py:358; the logits all-gather before the
 * argmax, parallel/transformer.py:570-573) run inside the kernel over NVLink
 * peer memory.
 *
 * Setup (not on the hot path): sc_step_create; sc_step_set_layer for every
 * layer (wq / scales / biases: the 7 linears q, k, v, o, gate, up, down in the
 * MLX layout, 16-byte aligned; caches fp32 [Hkv, max_seq, head_dim]);
 * sc_step_set_head (the vocab-split embedding, whose weights are the tied LM
 * head, and the final norm); sc_step_set_io (tok: int32 [1], the token to
 * embed, overwritten with the sampled one; pos: int32 [1], the cache length,
 * advanced by one; cos/sin fp32 [max_pos, head_dim/2]; trace: fp32
 * [layers+1, hidden] or NULL, receives the hidden state after the embedding
 * and every layer; logits: fp32 [vocab_local] or NULL); with world > 1,
 * sc_step_set_peers (every rank's exchange arena as mapped here, at least
 * sc_step_arena_bytes each, zero on creation); then sc_step_finalize with a
 * caller workspace of sc_step_workspace_bytes (256-byte aligned; the plan,
 * tensor maps and counters live there and must stay untouched).
 * sc_step_run enqueues one step (one kernel, one CTA per SM, every CTA
 * resident; capturable in a CUDA graph).  A wait that runs out (2 s) raises
 * the error word, read by sc_step_error (reset != 0 restarts the counters).
 * No reference counterpart as one call (the reference runs the same math as
 * per-layer MLX ops and TCP collectives). */
int sc_step_create(int hidden, int heads, int kv_heads, int head_dim, int ffn, int vocab_local, int vocab_start,
                   int layers, int bits, int group, float eps, int max_seq, int world, int rank, void** step);
int sc_step_set_layer(void* step, int layer, const uint16_t* ln1, const uint16_t* ln2,
                      const uint32_t* const* wq, const uint16_t* const* scales, const uint16_t* const* biases,
                      float* k_cache, float* v_cache);
int sc_step_set_head(void* step, const uint32_t* embed_wq, const uint16_t* embed_scales,
                     const uint16_t* embed_biases, const uint16_t* final_norm);
int sc_step_set_io(void* step, int32_t* tok, int32_t* pos, const float* cos_tab, const float* sin_tab,
                   int max_pos, float* trace, float* logits);
size_t sc_step_arena_bytes(int hidden, int world);
int sc_step_set_peers(void* step, void* const* arenas, size_t arena_bytes);
size_t sc_step_workspace_bytes(void* step);
int sc_step_finalize(void* step, void* workspace, size_t workspace_bytes, cudaStream_t stream);
int sc_step_run(void* step, cudaStream_t stream);
int sc_step_error(void* step, int reset);
/* Where the first error was raised: out[0] op index, out[1] CTA, out[2] warp,
 * out[3] the counter value seen, out[4] the target, then (n > 8) the op each
 * CTA's consumers last started (the op count: step finished), one int per SM,
 * then the step's dependency counters (input counts per op first). */
int sc_step_error_info(void* step, int* out, int n);
/* Optional per-op timing of later launches: stamps holds
 * sc_step_timing_count(step) = SMs x ops x 4 uint64 %globaltimer values (ns)
 * per CTA and op: op start, input ready, weight stream done, op done (0:
 * not reached).  nullptr turns it off. */
int sc_step_set_timing(void* step, unsigned long long* stamps);
size_t sc_step_timing_count(void* step);
/* After finalize: {SMs, CTAs per SM, static shared bytes, dynamic shared
 * bytes, registers per thread, max threads per block} of the step kernel. */
int sc_step_fit(void* step, int* out6);
int sc_step_destroy(void* step);

/* Every rank's arena of a peer-memory transport as mapped in this process
 * (bases[world]) and the arena size, for a kernel that lays out its own lines
 * in a transport it owns (the persistent decode step).  No reference
 * counterpart. */
int sc_p2p_arenas(void* p2p, void** bases, size_t* arena_bytes);

#ifdef __cplusplus
}
#endif
#endif /* SC_B200_H */
