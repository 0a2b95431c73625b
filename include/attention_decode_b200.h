/*
 * attention_decode_b200.h -- C ABI of the B200 (sm_100a) BF16 split-K
 * attention-decode library (libattention_decode_b200.so).
 *
 * Operation (single query token per sequence, GQA):
 *     O[b, hq, 0, :] = softmax(Q[b, hq, 0, :] . K[b, hq / G, :L_b, :]^T / sqrt(D))
 *                      . V[b, hq / G, :L_b, :]
 * with G = Hq / Hkv, every tensor BF16 and contiguous (BHSD layout), FP32
 * softmax and accumulation.  L_b = S for every sequence unless a `seqlens`
 * array is given.
 *
 * The library replaces the reference's CUDA extension entry point
 *     at::Tensor attention_decode_cuda(q, k, v)      csrc/decode.cu:223-258
 * bound to Python as `forward`                       csrc/binding.cpp:3-8
 * with plain pointers, sizes and a caller-supplied stream and workspace, so
 * any FFI (ctypes, cgo, JNI, N-API) can bind it.  No decode function
 * allocates device memory, synchronises the host or keeps per-call state (the
 * exchange set-up functions at the end are the only ones that allocate or map
 * memory): every call is
 * stream-ordered and may be captured in a CUDA graph, and concurrent calls on
 * different streams are independent as long as their workspaces differ.
 *
 * Workspace: the first `header_bytes` of a workspace hold the scheduler state
 * of one call.  It must be zero when a call starts, and every call that
 * completes leaves it zero again.  Pass ADB_FLAG_HEADER_ZEROED when that is
 * known to hold (a workspace zeroed once and then reused only by calls that
 * are ordered on one stream); without the flag the library zeroes the header
 * with one cudaMemsetAsync on the call's stream.  Calls that may run
 * concurrently must use different workspaces.
 *
 * Error convention: every function returns an adb_status; on failure a
 * message is kept in thread-local storage (adb_last_error).  Argument errors
 * are detected on the host before any launch, mirroring the TORCH_CHECKs at
 * csrc/decode.cu:225-244.
 */
#ifndef ATTENTION_DECODE_B200_H
#define ATTENTION_DECODE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ADB_API __attribute__((visibility("default")))
#else
#define ADB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Flags of adb_decode / adb_decode_partial. */
#define ADB_FLAG_HEADER_ZEROED 1u /* the workspace header is already zero */

typedef enum adb_status {
  ADB_OK = 0,
  ADB_ERR_INVALID_ARGUMENT = 1, /* sizes, null pointers, contract violations */
  ADB_ERR_UNSUPPORTED = 2,      /* head_dim not in {64,128}, group not in {1,4,8} */
  ADB_ERR_DEVICE = 3,           /* device is not compute capability 10.x      */
  ADB_ERR_WORKSPACE = 4,        /* workspace missing, too small or misaligned  */
  ADB_ERR_CUDA = 5              /* CUDA runtime error during set-up or launch  */
} adb_status;

/* Library version string, e.g. "attention_decode_b200 0.1.0 sm_100a". */
ADB_API const char* adb_version(void);

/* Message of the last failing call on this thread ("" if none). */
ADB_API const char* adb_last_error(void);

/* Checks that `device` is a compute-capability 10.x GPU that this build can
 * run on.  Replaces the per-call capability gate at csrc/decode.cu:243-244
 * (which required 12.0). */
ADB_API int adb_check_device(int device);

/* Bytes of device workspace adb_decode / adb_decode_partial need for this
 * problem on `device` (depends on the device's SM count), and the size of its
 * leading scheduler header (may be NULL).  `has_seqlens` is non-zero when a
 * per-sequence length array will be passed.  Replaces the reference's
 * internal `at::empty({heads, splits, D + 2})` partial buffer
 * (csrc/decode.cu:205). */
ADB_API int adb_decode_workspace_size(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                      int64_t kv_len, int64_t head_dim, int has_seqlens,
                                      int device, size_t* bytes, size_t* header_bytes);

/* Full decode into a BF16 output [batch, q_heads, 1, head_dim].
 *   q        [batch, q_heads, 1, head_dim]       bf16, contiguous
 *   k, v     [batch, kv_heads, kv_len, head_dim] bf16, contiguous
 *   seqlens  NULL, or int32 [batch] on the device: sequence b uses its first
 *            seqlens[b] tokens (values are clamped to [0, kv_len]; a length
 *            of 0 gives an all-zero output row, as the FP32 oracle does)
 *   out      [batch, q_heads, 1, head_dim]       bf16
 *   workspace at least adb_decode_workspace_size() bytes, 256-byte aligned
 *   flags    ADB_FLAG_HEADER_ZEROED or 0 (see "Workspace" above)
 *   stream   cudaStream_t (NULL = legacy default stream)
 * The whole decode is one kernel launch (plus the header memset when the flag
 * is not given), launched with programmatic stream serialisation so that it
 * can start while the previous kernel in the stream drains. 
 * Replaces attention_decode_cuda (csrc/decode.cu:223-258) and its launch path
 * decode_bf16_mma + merge_splits (csrc/decode.cu:70-211).  K/V pointers that
 * are not 16-byte aligned are accepted (slower fallback path), matching the
 * reference's unaligned dispatch (csrc/decode.cu:212-220). */
ADB_API int adb_decode(const void* q, const void* k, const void* v, const int32_t* seqlens,
                       void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                       int64_t kv_len, int64_t head_dim, void* workspace,
                       size_t workspace_bytes, unsigned flags, int device, void* stream);

/* Decode over an FP8 (e4m3, OCP "fn" encoding) K/V cache (no reference
 * counterpart: the reference reads BF16 only).  k, v: [batch, kv_heads,
 * kv_len, 128] e4m3 bytes, contiguous, 16-byte aligned; the values they
 * stand for are k * k_scale and v * v_scale (per-tensor scales, positive and
 * finite).  The result is the BF16 decode of those values (FP32 softmax and
 * accumulation, Q rounded to FP16 for the tensor-core products), so it
 * streams half the bytes of the BF16 path.  head_dim 128 only.  Other
 * arguments as adb_decode (seqlens optional); workspace from
 * adb_decode_workspace_size. */
ADB_API int adb_decode_fp8(const void* q, const void* k, const void* v, const int32_t* seqlens,
                           void* out, int64_t batch, int64_t q_heads, int64_t kv_heads,
                           int64_t kv_len, int64_t head_dim, float k_scale, float v_scale,
                           void* workspace, size_t workspace_bytes, unsigned flags, int device,
                           void* stream);

/* One decode step of a serving loop with the new token appended (no
 * reference counterpart: the reference decodes a cache that already holds
 * every token).  Sequence b has seqlens[b] tokens cached in k_cache /
 * v_cache [batch, kv_heads, kv_capacity, head_dim] (bf16, contiguous); the
 * step's new token is k_new / v_new [batch, kv_heads, 1, head_dim].  The
 * output is attention over the seqlens[b] cached tokens and the new one --
 * what adb_decode computes after the token is written at position
 * seqlens[b] and the length raised by one -- and the kernel also writes the
 * new token into the cache at position seqlens[b], replacing the separate
 * append launch of a decode loop.  seqlens is not modified (raise it on the
 * stream after the call).  A sequence whose cache is full (seqlens[b] >=
 * kv_capacity) gets attention over kv_capacity cached tokens and the new
 * one, no write, and bit 8 of the device error word (adb_read_error_flag).
 * Workspace as adb_decode with kv_len = kv_capacity and has_seqlens = 1. */
#define ADB_ERROR_FLAG_APPEND_FULL 8
ADB_API int adb_decode_append(const void* q, const void* k_new, const void* v_new, void* k_cache,
                              void* v_cache, const int32_t* seqlens, void* out, int64_t batch,
                              int64_t q_heads, int64_t kv_heads, int64_t kv_capacity,
                              int64_t head_dim, void* workspace, size_t workspace_bytes,
                              unsigned flags, int device, void* stream);

/* Layouts of a paged K/V cache (adb_decode_paged). */
#define ADB_PAGED_HND 0 /* [num_blocks][kv_heads][page_size][head_dim] */
#define ADB_PAGED_NHD 1 /* [num_blocks][page_size][kv_heads][head_dim] */

/* Decode over a paged K/V cache (no reference counterpart: the reference
 * takes contiguous [B, Hkv, S, D] tensors only; this is the layout a serving
 * engine's KV cache uses).  k_cache / v_cache are pools of num_blocks pages
 * of page_size tokens each (bf16, 16-byte aligned, layout HND or NHD);
 * page j of sequence b is block_table[b * block_table_stride + j] (int32 on
 * the device), and sequence b uses its first seqlens[b] tokens (int32 on the
 * device, clamped to [0, max_blocks_per_seq * page_size]).  page_size is a
 * power of two from 8 to 2^20.  Only the pages that hold a sequence's tokens
 * are read; block-table entries past a sequence's last page are never used.
 * Size the workspace with adb_decode_workspace_size(batch, q_heads,
 * kv_heads, max_blocks_per_seq * page_size, head_dim, 1, ...).  Output,
 * flags, workspace and stream as adb_decode. */
ADB_API int adb_decode_paged(const void* q, const void* k_cache, const void* v_cache,
                             const int32_t* block_table, int64_t block_table_stride,
                             const int32_t* seqlens, void* out, int64_t batch, int64_t q_heads,
                             int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                             int64_t page_size, int64_t max_blocks_per_seq, int layout,
                             void* workspace, size_t workspace_bytes, unsigned flags, int device,
                             void* stream);

/* Size of the fixed device array that adb_decode_no_alloc uses as its
 * workspace (8 MiB, held by every GPU that loads the library). */
#define ADB_NO_ALLOC_WORKSPACE_BYTES (8u << 20)

/* Decode exactly like adb_decode, but without any workspace argument and
 * without allocating device memory: the scratch is a fixed array of
 * ADB_NO_ALLOC_WORKSPACE_BYTES inside the library.  It has no counterpart in
 * the reference, whose entry point always allocates its partial buffer.
 *
 * It is meant for callers that cannot allocate device memory themselves:
 * hosts binding the C ABI from another language whose device memory is owned
 * by a different allocator, and serving loops that must not enter
 * cudaMalloc/cudaFree (which synchronise the device) or run under a fixed
 * memory budget.  The caller still passes Q, K, V, seqlens and the output.
 *
 * Limits and behaviour:
 *  - problems whose scratch would exceed ADB_NO_ALLOC_WORKSPACE_BYTES are
 *    rejected with ADB_ERR_WORKSPACE.  No work stealing is used here, so the
 *    scratch is exactly: a header of 8*ctas + 8 + 8*batch*kv_heads bytes,
 *    then slots = ctas + batch*kv_heads segment states of group*head_dim
 *    and group*2 floats, each of the three parts rounded up to 256 bytes,
 *    where ctas = min(SM count, batch*kv_heads*ceil(kv_len/tile)) and tile
 *    is 128 tokens (64 when that product is below twice the SM count).
 *    About (148 + batch*kv_heads) * group * (head_dim + 2) * 4 bytes on a
 *    B200; adb_decode_workspace_size gives an upper bound (it also counts
 *    the slots work stealing may use);
 *  - the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current and keeps it; make that
 *    first call before any stream capture.  The kept address is invalid
 *    after cudaDeviceReset (or any teardown of the device's primary
 *    context): do not call this entry point again in that process;
 *  - every call uses the same array, and its scheduler header is cleared with
 *    one cudaMemsetAsync on `stream` before the kernel, so calls that overlap
 *    on the GPU (different streams, or different host threads) race and
 *    corrupt each other's results: order them on one stream or use
 *    adb_decode;
 *  - no cudaMalloc, cudaFree or other allocating call is made. */
ADB_API int adb_decode_no_alloc(const void* q, const void* k, const void* v,
                                const int32_t* seqlens, void* out, int64_t batch,
                                int64_t q_heads, int64_t kv_heads, int64_t kv_len,
                                int64_t head_dim, int device, void* stream);

/* Partial decode for sequence sharding: instead of the normalised output it
 * writes, per query-head row r = b * q_heads + hq,
 *   acc[r, 0:head_dim]  unnormalised sum_t exp(s_t - m) * V_t   (fp32)
 *   ml[r, 0] = m        max logit s_t = q.k_t / sqrt(D) (natural units)
 *   ml[r, 1] = l        sum_t exp(s_t - m)
 * over this call's KV.  An empty sequence gives acc = 0, m = -inf, l = 0.
 * The state layout is the reference's split partial (acc[D], m, l)
 * (csrc/decode.cu:127-129,160), kept as two arrays. */
ADB_API int adb_decode_partial(const void* q, const void* k, const void* v,
                               const int32_t* seqlens, float* acc, float* ml,
                               int64_t batch, int64_t q_heads, int64_t kv_heads,
                               int64_t kv_len, int64_t head_dim, void* workspace,
                               size_t workspace_bytes, unsigned flags, int device,
                               void* stream);

/* Merges `parts` partial states per row into BF16 output rows:
 *   M = max_r m_r,  O = sum_r e^(m_r - M) acc_r / sum_r e^(m_r - M) l_r.
 * Part r's arrays start at acc + r * acc_part_stride and
 * ml + r * ml_part_stride (floats; rows are contiguous inside a part), so an
 * all-gathered buffer of packed [acc | ml] blocks can be merged in place.
 * Rows whose every part is empty (l = 0) become zeros.
 * Replaces merge_splits (csrc/decode.cu:169-184) for the cross-GPU merge. */
ADB_API int adb_combine(const float* acc, int64_t acc_part_stride, const float* ml,
                        int64_t ml_part_stride, int64_t parts, int64_t rows,
                        int64_t head_dim, void* out, int device, void* stream);

/* ---- Sequence sharding over NVLink peer memory (no reference counterpart:
 * the reference is single-GPU; this replaces an NCCL all_gather of the
 * partial states followed by adb_combine).
 *
 * Each of `world` ranks (one process per GPU, world <= 8) allocates one
 * exchange buffer of adb_exchange_size() bytes with adb_exchange_alloc (zeroed),
 * shares its adb_ipc_handle() with the other ranks through any host channel,
 * and maps theirs with adb_ipc_open; exchange[r] is then rank r's buffer as
 * seen from this process (its own buffer at exchange[rank]).  A step is
 *   adb_decode_exchange(...)   partial decode of this rank's token shard; the
 *                              kernel stores its states straight into every
 *                              rank's buffer over NVLink and raises a flag
 *   adb_exchange_merge(...)    waits (bounded) for every rank's flag, then
 *                              merges the `world` states per row into BF16
 * both on one stream; every rank makes the same sequence of calls.  Nothing
 * synchronises the host, so a step can be captured in a CUDA graph.  The
 * buffers hold two calls' states (by call parity), so ranks may drift apart
 * by one call without a barrier.  If a peer's states do not arrive within
 * `timeout_us`, the merge writes zero rows and sets bit 4 of the device error
 * word (adb_read_error_flag).  Buffers must stay mapped until every rank has
 * finished its last step. */
#define ADB_IPC_HANDLE_BYTES 64
#define ADB_ERROR_FLAG_PEER_TIMEOUT 4

ADB_API int adb_exchange_size(int64_t rows, int64_t head_dim, int world, size_t* bytes);
ADB_API int adb_exchange_alloc(size_t bytes, int device, void** buffer);
ADB_API int adb_exchange_free(void* buffer, int device);
ADB_API int adb_ipc_handle(void* buffer, int device, unsigned char* handle);
ADB_API int adb_ipc_open(const unsigned char* handle, int device, void** buffer);
ADB_API int adb_ipc_close(void* buffer, int device);

/* Partial decode (as adb_decode_partial) whose states go to slot `rank` of
 * every rank's exchange buffer.  `exchange` holds `world` device pointers. */
ADB_API int adb_decode_exchange(const void* q, const void* k, const void* v,
                                const int32_t* seqlens, int64_t batch, int64_t q_heads,
                                int64_t kv_heads, int64_t kv_len, int64_t head_dim,
                                void* const* exchange, int world, int rank, void* workspace,
                                size_t workspace_bytes, unsigned flags, int device,
                                void* stream);

/* Merge step on this rank's own buffer: out [rows, head_dim] BF16 with
 * rows = batch * q_heads.  One kernel, launched with programmatic stream
 * serialisation behind the decode. */
ADB_API int adb_exchange_merge(const void* exchange, int world, int64_t rows, int64_t head_dim,
                               void* out, int64_t timeout_us, int device, void* stream);

/* adb_decode_exchange and adb_exchange_merge in ONE launch: after this rank's
 * states are published, the kernel's first CTAs wait (bounded by
 * `timeout_us`) for every rank's flag of the call and merge the rows into
 * `out` [batch * q_heads, head_dim] BF16, with no second kernel and no grid
 * boundary between the exchange and the merge.  Only for ranks that run on
 * DISTINCT GPUs: each rank's kernel waits for the others' kernels, so two
 * ranks sharing a GPU must use the two-call form.  Same errors and timeout
 * behaviour as the pair it replaces. */
ADB_API int adb_decode_exchange_merged(const void* q, const void* k, const void* v,
                                       const int32_t* seqlens, int64_t batch, int64_t q_heads,
                                       int64_t kv_heads, int64_t kv_len, int64_t head_dim,
                                       void* const* exchange, int world, int rank, void* out,
                                       int64_t timeout_us, void* workspace, size_t workspace_bytes,
                                       unsigned flags, int device, void* stream);

/* Reads (and optionally clears) the sticky device error word that kernels
 * set when a bounded wait gives up; 0 means no kernel has reported an
 * error on `device`.  Synchronous (a device-to-host copy); for diagnostics. */
ADB_API int adb_read_error_flag(int device, int* flag, int reset);

/* Diagnostics (no reference counterpart: the reference has no instrumentation).
 * adb_launch_count: kernels this process has launched through the library.
 * adb_timing_enable: on the calling thread, record a CUDA event pair around
 *   every partial (streaming) kernel launched from then on.
 * adb_timing_read: wait for the recorded events, return the summed duration
 *   in milliseconds and the number of timed launches, and forget them. */
ADB_API int adb_launch_count(int64_t* launches);
ADB_API int adb_timing_enable(int enable);
ADB_API int adb_timing_read(double* total_ms, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* ATTENTION_DECODE_B200_H */
