/*
 * ravel_b200.h -- C ABI of the B200 (sm_100a) implementation of RAVEL's exact
 * event-memory operator.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * handle (cudaStream_t passed as void*), never allocates or frees, never
 * synchronises the host, and returns a status code (RAVEL_OK == 0).  The
 * caller owns every buffer: outputs, the "tape" that carries the sorted event
 * order from a forward call to its backward call, and per-call scratch.
 * Sizes of the tape and scratch come from ravel_tape_bytes() and
 * ravel_scratch_bytes().  Work is enqueued on `stream`; the entry points that
 * take their tape and scratch from the caller may be captured in a CUDA graph.
 *
 * Layouts (all C-contiguous, element strides only):
 *   addresses     [B, T, C]         int32 or int64  (addr_dtype)
 *   write_mask    [B, T]            uint8 0/1 or NULL (NULL: every step writes)
 *   payloads      [B, T, C, D]      float32 / bfloat16 / float16 / float64
 *   latest values [B, T, C, k, D]   payload dtype;  mask [B, T, C, k] uint8
 *   sums          [B, T, C, D]      payload dtype;  mask [B, T, C]    uint8
 *   cache values  [B, C, A, D]      payload dtype;  filled [B, C, A]  uint8
 * A "stream" is one (b, c) pair; streams never interact.
 *
 * Semantics are those of the reference's ravel_lm/ravel_memory.py (paths
 * relative to the ravel-lm project); each declaration cites the function it
 * replaces.  Prefill addresses are reduced with a floor modulo of A after the
 * reference's integer-width conversion; decode addresses are clamped to
 * [0, A-1].
 */
#ifndef RAVEL_B200_H
#define RAVEL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define RAVEL_OK 0
#define RAVEL_ERR_INVALID_ARG 1   /* bad shape, dtype, k <= 0, A <= 0, null pointer */
#define RAVEL_ERR_WORKSPACE 2     /* tape or scratch smaller than required */
#define RAVEL_ERR_CUDA 3          /* a CUDA launch or runtime call failed */
#define RAVEL_ERR_UNSUPPORTED 4   /* sizes beyond the supported range */
#define RAVEL_ERR_DEVICE 5        /* a kernel flagged an error (ravel_device_error) */

/* ---- dtype codes ------------------------------------------------------- */
#define RAVEL_F32 0
#define RAVEL_BF16 1
#define RAVEL_F16 2
#define RAVEL_F64 3
#define RAVEL_I32 0
#define RAVEL_I64 1

/* ---- tape flags -------------------------------------------------------- */
/* reads use their own addresses (read_addresses given and not the write tensor) */
#define RAVEL_TAPE_GENERAL_READS 1
/* a write_mask is given */
#define RAVEL_TAPE_WRITE_MASK 2

/* ---- device-side error bits (ravel_device_error) ------------------------ */
/* A wait on another block (a scan's look-back, the fused GEMM's pipeline
 * barriers) hit its poll limit and gave up instead of hanging.  Sizes,
 * pointers, alignment and workspace are checked on the host before any launch,
 * so kernels carry no other error bit. */
#define RAVEL_DEVERR_SPIN 1

/* Bytes of the tape written by a forward call and read by its backward call. */
size_t ravel_tape_bytes(int64_t B, int64_t T, int64_t C, int64_t A, int tape_flags);

/* Bytes of per-call scratch sufficient for every entry point at these sizes
 * and this payload dtype. */
size_t ravel_scratch_bytes(int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, int64_t k,
                           int dtype, int tape_flags);

/*
 * Sort the write events of every stream by (address, time) and, for general
 * reads, find each read's latest earlier write.  Replaces the key build, mask
 * compaction, torch.sort and searchsorted of ravel_lm/ravel_memory.py:126-159
 * (and :200-216, :231-235 of causal_sum_lookup).
 * raddr == NULL or raddr == waddr: reads alias writes.
 */
int ravel_tape_build(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask,
                     int64_t B, int64_t T, int64_t C, int64_t A, int tape_flags,
                     void* tape, size_t tape_bytes, void* scratch, size_t scratch_bytes,
                     void* stream);

/*
 * Latest-k gather from a built tape: values[b,t,c,j] = payload of the j-th
 * latest write with the same (b, c, address) strictly before t, else
 * candidate*0; mask = validity.  Replaces ravel_lm/ravel_memory.py:160-176.
 * raddr is needed whenever tape_flags is nonzero (reads that differ from the
 * writes, or a write mask): the read addresses, or the write addresses when
 * reads alias writes.  With tape_flags == 0 it may be NULL.
 */
int ravel_latestk_fwd_tape(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                           const void* payload, int dtype, int64_t B, int64_t T, int64_t C,
                           int64_t D, int64_t A, int64_t k, void* out_vals, uint8_t* out_mask,
                           void* stream);

/*
 * causal_last_k_lookup forward (ravel_lm/ravel_memory.py:52-176):
 * ravel_tape_build + ravel_latestk_fwd_tape.  The tape is kept for the backward.
 */
int ravel_latestk_fwd(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask,
                      const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                      int64_t A, int64_t k, void* out_vals, uint8_t* out_mask,
                      void* tape, size_t tape_bytes, void* scratch, size_t scratch_bytes,
                      void* stream);

/*
 * Gradient of the latest-k values w.r.t. payloads (the autograd of
 * index_select + mask multiply at ravel_lm/ravel_memory.py:173-175):
 * grad_payload[src] = sum of grad_vals over the valid slots that read src.
 * grad_payload [B,T,C,D] is fully overwritten.  Deterministic for every row
 * shape: a gather, no atomics (one lane per 16-byte vector when a row is 2^m
 * <= 32 vectors, else one warp per write over the row's elements).
 */
int ravel_latestk_bwd(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                      const void* grad_vals, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                      int64_t A, int64_t k, void* grad_payload, void* scratch, size_t scratch_bytes,
                      void* stream);

/*
 * ravel_latestk_bwd that adds its gradient to grad_payload instead of
 * overwriting it (grad_payload += d values / d payloads, one rounding per
 * element for 16-bit payloads).  Replaces autograd's sum of the latest-k and
 * segmented-sum payload gradients when both lookups of a memory layer read the
 * same payload tensor (ravel_lm/model.py:367-384): the sum's gradient is
 * written first, this call adds the latest-k gradient to it in place.
 */
int ravel_latestk_bwd_accumulate(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                                 const void* grad_vals, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                                 int64_t A, int64_t k, void* grad_payload, void* scratch, size_t scratch_bytes,
                                 void* stream);

/*
 * Segmented-sum lookup from a built tape: sums[b,t,c] = sum of payloads of
 * writes with the same (b, c, address) strictly before t (float32
 * accumulation, float64 for float64 payloads); mask = at least one such write.
 * Replaces ravel_lm/ravel_memory.py:216-241.
 */
int ravel_segsum_fwd_tape(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                          const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                          int64_t A, void* out_sums, uint8_t* out_mask, void* scratch,
                          size_t scratch_bytes, void* stream);

/* causal_sum_lookup forward (ravel_lm/ravel_memory.py:179-241). */
int ravel_segsum_fwd(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask,
                     const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                     int64_t A, void* out_sums, uint8_t* out_mask, void* tape, size_t tape_bytes,
                     void* scratch, size_t scratch_bytes, void* stream);

/*
 * Gradient of the sums w.r.t. payloads (autograd of ravel_lm/ravel_memory.py:
 * 217-240): each write receives the sum of grad_sums over later reads of its
 * (b, c, address).  grad_payload [B,T,C,D] is fully overwritten.
 */
int ravel_segsum_bwd(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                     const void* grad_sums, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                     int64_t A, void* grad_payload, void* scratch, size_t scratch_bytes,
                     void* stream);

/*
 * Decode cache read (RavelLayerCache.read, ravel_lm/ravel_memory.py:271-281):
 * out_vals[b,c] = values[b,c,clamp(addr)] * filled, out_mask[b,c] = filled.
 */
int ravel_cache_read(const void* values, const uint8_t* filled, const void* addr, int addr_dtype,
                     int dtype, int64_t B, int64_t C, int64_t A, int64_t D, void* out_vals,
                     uint8_t* out_mask, void* stream);

/*
 * Decode cache write (RavelLayerCache.write, ravel_lm/ravel_memory.py:283-292):
 * values[b,c,clamp(addr)] = payload[b,c]; filled[...] = 1.  In place.
 */
int ravel_cache_write(void* values, uint8_t* filled, const void* addr, int addr_dtype,
                      const void* payload, int dtype, int64_t B, int64_t C, int64_t A, int64_t D,
                      void* stream);

/*
 * One decode step of a memory layer in one launch: the read of
 * RavelMemoryLayer.step (ravel_lm/model.py:421) followed by its write (:424),
 * for every (b, c).  The read sees the cache as it was before this step.
 */
int ravel_cache_step(void* values, uint8_t* filled, const void* raddr, const void* waddr,
                     int addr_dtype, const void* payload, int dtype, int64_t B, int64_t C,
                     int64_t A, int64_t D, void* out_vals, uint8_t* out_mask, void* stream);

/*
 * Bulk prefill of the decode cache.  Replaces the token-by-token prefill of
 * ravel_lm/model.py:600-602, whose memory layers write the cache once per
 * position (RavelMemoryLayer.step, :424, i.e. RavelLayerCache.write,
 * ravel_lm/ravel_memory.py:283-292).  The result equals ravel_cache_write of
 * (addr[:, t], payload[:, t]) for t = 0 .. T-1 in order: for every (b, c) and
 * clamped address, the latest t that writes it wins and its filled flag is set;
 * entries no position writes keep their contents.  addr [B, T, C], payload
 * [B, T, C, D] in the cache's dtype.  One per-stream sort plus one copy kernel;
 * scratch of ravel_cache_prefill_scratch_bytes(B, T, C, A) bytes holds the sort.
 */
size_t ravel_cache_prefill_scratch_bytes(int64_t B, int64_t T, int64_t C, int64_t A);
int ravel_cache_prefill(void* values, uint8_t* filled, const void* addr, int addr_dtype,
                        const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t A,
                        int64_t D, void* scratch, size_t scratch_bytes, void* stream);

/*
 * causal_sum_lookup forward for callers that cannot allocate device memory.
 * No counterpart in the reference: it exists for hosts that may not call
 * cudaMalloc or a caching allocator on this path -- plugin interfaces whose
 * enqueue step must not allocate, or foreign-language callers with no CUDA
 * allocator of their own.  Same
 * arguments and results as ravel_segsum_fwd, minus tape and scratch: both live
 * in one file-scope device array of RAVEL_NOALLOC_SCRATCH_BYTES that every GPU
 * loading this library holds until the process exits.  Returns
 * RAVEL_ERR_WORKSPACE, launching nothing, when ravel_tape_bytes() +
 * ravel_scratch_bytes() of the call exceed that size.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture.  All calls
 * share the array, so calls that overlap on the GPU (other streams, other host
 * threads) race; serialise them.  No backward: the tape is not kept.
 */
#define RAVEL_NOALLOC_SCRATCH_BYTES (32u << 20)
int ravel_segsum_fwd_noalloc(const void* waddr, const void* raddr, int addr_dtype,
                             const uint8_t* wmask, const void* payload, int dtype, int64_t B,
                             int64_t T, int64_t C, int64_t D, int64_t A, void* out_sums,
                             uint8_t* out_mask, void* stream);

/*
 * Literal address families of a memory layer (literal_addresses_from_tokens,
 * ravel_lm/model.py:195-231): out[b, t, j] for j < n_heads, int64, from token
 * ids [B, T] (int64), each family modulo A (floor), previous tokens before the
 * start taken as bos_token_id.  Bit for bit the reference's values.
 */
int ravel_literal_addresses(const int64_t* tokens, int64_t B, int64_t T, int n_heads, int64_t bos_token_id,
                            int64_t A, int64_t* out, void* stream);

/*
 * ravel_tape_build for a memory layer, straight from its token ids: head c <
 * n_literal takes literal address family c of the tokens (as
 * ravel_literal_addresses computes it), head c >= n_literal the learned address
 * learned_write[b, t, c - n_literal] (reads: learned_read) -- the concatenation
 * of ravel_lm/model.py:347-349 followed by the sort of
 * ravel_lm/ravel_memory.py:126-159, with the literal hashing done in the sort's
 * key build and no [B, T, C] address tensor materialised.  learned_* are
 * [B, T, C - n_literal] int32/int64 (learned_dtype); NULL when C == n_literal.
 * When tape_flags != 0, read_addr_out [B, T, C] int32 receives every read's
 * folded address; pass it as raddr (RAVEL_I32) to the lookup entry points that
 * use this tape.  A must be below 2^31.
 */
int ravel_tape_build_tokens(const int64_t* tokens, int n_literal, int64_t bos_token_id, const void* learned_write,
                            const void* learned_read, int learned_dtype, const uint8_t* wmask, int64_t B, int64_t T,
                            int64_t C, int64_t A, int tape_flags, int32_t* read_addr_out, void* tape,
                            size_t tape_bytes, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Latest-k source table from a built tape: src[(b*T + t)*C + c][j] = the flat
 * payload row ((b*T + t')*C + c) of read (b, t, c)'s j-th latest earlier write,
 * -1 for an invalid slot (the rows ravel_lm/ravel_memory.py:173-174 gathers).
 * src is [B*T*C, k] int32.  raddr as for ravel_latestk_fwd_tape.
 */
int ravel_latestk_sources(const void* tape, int tape_flags, const void* raddr, int addr_dtype, int64_t B, int64_t T,
                          int64_t C, int64_t A, int64_t k, int32_t* src, void* stream);

/*
 * A memory layer's read-out, fused: out[n] = A[n] * W^T with the read rows
 * A[n] = [payload[src[n, c, j]] for c < C, j < k (zero for -1) | sums[n, c] for
 * c < C] -- torch.cat of the latest-k values and sums (ravel_lm/model.py:383-385)
 * followed by fast_linear (:386) -- without A ever being written: a tcgen05
 * kernel (kind::tf32: TF32 inputs, float32 accumulation) gathers every A tile
 * into shared memory.  payload [B*T*C, D], sums [B*T, C, D] or NULL (no sum
 * read), weight [N, K] with K = C*k*D (+ C*D), all float32, D a multiple of 4,
 * 16-byte aligned.  With x and gate ([B*T, N]) the output is the gate residual
 * x + sigmoid(gate) * (A * W^T) (ravel_lm/model.py:388), and pre (optional)
 * receives A * W^T itself.
 */
int ravel_gather_gemm(const float* payload, const int32_t* src, const float* sums, int64_t B, int64_t T, int64_t C,
                      int64_t D, int64_t k, const float* weight, int64_t N, const float* x, const float* gate,
                      float* out, float* pre, void* stream);

/* The read rows A of ravel_gather_gemm written out ([B*T, K] float32), for its backward. */
int ravel_gather_rows(const float* payload, const int32_t* src, const float* sums, int64_t B, int64_t T, int64_t C,
                      int64_t D, int64_t k, float* rows, void* stream);

/*
 * Gate residual of a memory layer, out = x + sigmoid(gate) * fused, elementwise
 * over n elements of float32 or bfloat16 (gate_residual,
 * ravel_lm/triton_block.py:383-387, called at ravel_lm/model.py:388).  Same
 * arithmetic and rounding as the reference's torch ops (sigmoid, mul, add), so
 * results are equal bit for bit.  Other dtypes: RAVEL_ERR_UNSUPPORTED.
 */
int ravel_gate_residual_fwd(const void* x, const void* gate, const void* fused, void* out, int64_t n, int dtype,
                            void* stream);

/*
 * Its backward (the autograd of the same ops): grad_gate = ((grad_out * fused)
 * * (1 - s)) * s, grad_fused = grad_out * s with s = sigmoid(gate); the
 * gradient of x is grad_out itself.
 */
int ravel_gate_residual_bwd(const void* gate, const void* fused, const void* grad_out, void* grad_gate,
                            void* grad_fused, int64_t n, int dtype, void* stream);

/*
 * RMSNorm over the last dimension: y = x * rsqrt(mean(x^2) + eps) * weight for
 * M rows of K elements (rms_norm, ravel_lm/triton_block.py:320-323, the
 * RMSNorm of ravel_lm/model.py:31-39), float32 or bfloat16 with float32 math.
 * rstd [M] (float32) is kept for the backward.  K <= 4096.
 */
int ravel_rms_norm_fwd(const void* x, const void* weight, float eps, void* y, float* rstd, int64_t M, int64_t K,
                       int dtype, void* stream);

/* Scratch bytes of ravel_rms_norm_bwd (per-block partial weight gradients). */
size_t ravel_rms_norm_scratch_bytes(int64_t M, int64_t K);

/*
 * RMSNorm backward: grad_x [M, K] and grad_weight [K] (deterministic: no
 * atomics, a fixed summation order for a given M).
 */
int ravel_rms_norm_bwd(const void* x, const void* weight, const void* grad_y, const float* rstd, void* grad_x,
                       void* grad_weight, int64_t M, int64_t K, int dtype, void* scratch, size_t scratch_bytes,
                       void* stream);

/*
 * Poll limit of every wait on another block, on the current device (default
 * 2^22 polls, about a second of waiting; 1 .. 2^28).  A copy to device memory:
 * call it between steps, not while a stream is being captured.
 */
int ravel_set_wait_limit(uint32_t polls);

/*
 * Self-test of the bounded wait: one warp waits on *flag (a device word) with
 * the wait the scans use.  Given a word nothing sets, the wait gives up after
 * the poll limit, RAVEL_DEVERR_SPIN appears in ravel_device_error, and the
 * context stays usable.
 */
int ravel_wait_selftest(const uint32_t* flag, void* stream);

/* Copy the device error word (RAVEL_DEVERR_* bits) of the current device into
 * *out after the work queued on `stream`; synchronises that stream. */
int ravel_device_error(int* out, void* stream);

/* Reset the device error word of the current device. */
int ravel_clear_device_error(void* stream);

/* Number of kernels this library has launched in this process (all devices). */
uint64_t ravel_kernel_launches(void);

/* ---- per-entry GPU timing (instrumentation; no reference counterpart) ---
 * ravel_timing_start(n) creates n pairs of CUDA events on the current device
 * and turns timing on, discarding earlier records.  While it is on, every
 * compute entry point above records one pair on its stream around the work it
 * enqueues (none while the stream is being captured into a graph; calls past
 * the n-th are not recorded).  ravel_timing_stop() turns it off and keeps the
 * records; ravel_timing_count() is how many were made;
 * ravel_timing_read(i, &entry, &ms) waits for record i's end event and returns
 * the entry point's name (a static string) and the milliseconds between the
 * pair.  Call start/stop while no entry point runs on another thread. */
int ravel_timing_start(int64_t max_records);
int ravel_timing_stop(void);
int64_t ravel_timing_count(void);
int ravel_timing_read(int64_t i, const char** entry, float* ms);

/* Human-readable name of a status code. */
const char* ravel_status_string(int status);

/* Library version string. */
const char* ravel_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RAVEL_B200_H */
