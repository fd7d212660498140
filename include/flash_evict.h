/*
 * flash_evict.h -- C ABI of the B200 (sm_100a) evict() prefill path.
 *
 * The reference (anishesg/flash-evict-prefill) is a Python package whose hot
 * path is one Triton kernel plus PyTorch selection ops.  Each entry point below
 * replaces one piece of that path; the Python package `flash_evict` (same
 * module path and signatures as the reference) binds them with ctypes.
 *
 * Conventions
 *  - All pointers are device pointers unless stated otherwise; sizes are
 *    element counts; strides are in elements.
 *  - Q is [batch, q_heads, tokens, channels], K and V are
 *    [batch, kv_heads, tokens, channels], each with arbitrary strides as long
 *    as the channel stride is 1, the other strides are multiples of 8 elements
 *    (16 bytes) and the base pointer is 16-byte aligned (the TMA rules).
 *  - dtype: FE_DTYPE_F16 or FE_DTYPE_BF16.  Q, K, V and the output share it.
 *  - channels (head dimension): 1..256.  Up to 128 the attention is one
 *    launch; 129..256 run as two launches on the stream, one per 128-channel
 *    half of V and the output.
 *  - `stream` is a cudaStream_t passed as void*; every launch is asynchronous
 *    on it and no entry point synchronizes the host.
 *  - Return value: FE_STATUS_OK or an error code; fe_last_error() gives the
 *    message for the calling thread.
 *  - Errors of kernels that ran after their call returned: every device-side
 *    wait is bounded (fe_set_watchdog_ns); a kernel that gives up records
 *    FE_STATUS_TIMEOUT (a gather kernel records FE_STATUS_BAD_INDEX) in the
 *    device status word and, once the library has attached it, in a word of
 *    mapped pinned host memory for that device.  Every compute entry point
 *    reads that host word on entry without synchronizing: a code found there
 *    is returned as the call's error (the call launches nothing) and cleared.
 *    The first compute call on a device in a CUDA context attaches the word
 *    (one pinned host allocation per process, and a one-thread kernel on the
 *    caller's stream); calls made while the stream is being captured do not
 *    attach.  Outputs of a kernel that gave up hold NaN where it could mark
 *    them (attention rows and their statistics, importance, SnapKV scores).
 *    fe_device_status() is the synchronous check.
 *  - A "query block" is FE_QUERY_BLOCK consecutive query rows.  Passing
 *    query_blocks == NULL processes all rows; otherwise only the listed block
 *    indices (device int32 array) are processed, which is how a rank of a
 *    query-sharded job restricts the work to its own rows.
 */
#ifndef FLASH_EVICT_B200_H
#define FLASH_EVICT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FE_API __attribute__((visibility("default")))
#else
#define FE_API
#endif

#define FE_STATUS_OK 0
#define FE_STATUS_INVALID 1     /* bad argument (shape, stride, value)          */
#define FE_STATUS_UNSUPPORTED 2 /* valid request outside what the kernels do    */
#define FE_STATUS_CUDA 3        /* a CUDA runtime/driver call failed            */
#define FE_STATUS_TIMEOUT 4     /* a device wait exceeded the watchdog limit    */
#define FE_STATUS_BAD_INDEX 5   /* a gather index was outside [0, tokens)       */

#define FE_DTYPE_F16 0
#define FE_DTYPE_BF16 1

#define FE_QUERY_BLOCK 256

/* Attention forward (traversal 1).
 * Replaces the first KV traversal of `_prefill` (flash_evict/prefill.py:23-60)
 * and the output allocation/launch of `prefill` (flash_evict/prefill.py:102-137).
 * Writes out = softmax(scale * Q K^T [causal]) V as a contiguous
 * [batch, q_heads, tokens, channels] tensor of `dtype`, and the final softmax
 * statistics of each query row to row_stats[(b*q_heads+h)*tokens+q] =
 * {m, l} (FP32; m in log2 units of scale*log2(e)*logit, l the row sum of
 * exp2(logit*scale*log2e - m)).  Deterministic: the same inputs give the same
 * bits whether or not scores are computed afterwards. */
FE_API int fe_attention_fwd(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                     const void* v, const int64_t* v_strides, void* out, float* row_stats, int64_t batch,
                     int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels, int dtype,
                     int causal, float scale, const int32_t* query_blocks, int64_t num_query_blocks,
                     void* stream);

/* Exact importance by replay (traversal 2), one store per KV token.
 * Replaces the replay loop and atomics of `_prefill`
 * (flash_evict/prefill.py:61-83) and the zero-fill of the score buffer
 * (flash_evict/prefill.py:129):
 *   importance[b,hkv,k] = ||V[b,hkv,k]||_1 (if value_weighted)
 *       * sum_{g, q} w_q * softmax(QK^T)[b, hkv*G+g, q, k]
 *   w_q = exp(recency_decay * (q - (tokens-1))) * [q >= tokens - W],
 *   W = min(tokens, observation_window or tokens).
 * row_stats must come from fe_attention_fwd on the same inputs.  Each output
 * element is written exactly once in a fixed order (no atomics, bitwise
 * reproducible).  Rows whose FP32 weight underflows (< 2^-126) are skipped.
 * With query_blocks != NULL the sum runs over the listed query blocks only
 * (a partial sum, to be all-reduced across ranks). */
FE_API int fe_replay_scores(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                     const void* v, const int64_t* v_strides, const float* row_stats, float* importance,
                     int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels,
                     int dtype, int causal, float scale, float recency_decay, int64_t observation_window,
                     int value_weighted, const int32_t* query_blocks, int64_t num_query_blocks, void* stream);

/* First query row the replay scores for these arguments: the start of the
 * observation window, raised past rows whose FP32 weight
 * exp(-recency_decay * (tokens-1-q)) is below 2^-127 (skipped exactly).  A
 * query-sharded caller exchanges the row statistics of rows >= this one.
 * Host-only. */
FE_API int64_t fe_replay_first_scored_row(int64_t tokens, float recency_decay, int64_t observation_window);

/* fe_replay_scores restricted to the key tiles [key_tile_begin, key_tile_end)
 * (128 keys each): only importance[b, hkv, 128*key_tile_begin ..
 * 128*key_tile_end) is written, summed over all scored query rows (or the
 * listed query blocks).  A query-sharded job uses it to split the replay
 * evenly by keys across ranks when the scored rows are concentrated in a few
 * query blocks (recency decay, observation window): each rank needs the row
 * statistics of every scored row, and the ranks' key ranges are then
 * combined.  No counterpart in the reference (single GPU). */
FE_API int fe_replay_scores_range(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                  const void* v, const int64_t* v_strides, const float* row_stats,
                                  float* importance, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                  int64_t tokens, int64_t channels, int dtype, int causal, float scale,
                                  float recency_decay, int64_t observation_window, int value_weighted,
                                  const int32_t* query_blocks, int64_t num_query_blocks, int64_t key_tile_begin,
                                  int64_t key_tile_end, void* stream);
/* Token selection.  Replaces `select_tokens` (flash_evict/prefill.py:140-170).
 * importance: contiguous FP32 [rows, tokens].  For each row: the past region
 * is the first tokens-recent scores; if pool_kernel > 1 and budget > recent it
 * is average-pooled (stride 1, zero padding pool_kernel/2, divisor
 * pool_kernel); the budget-recent largest pooled scores are kept (ties: larger
 * value first, then lower index; NaN counts as largest) together with the last
 * `recent` tokens.  indices: int64 [rows, budget], ascending.  mask: uint8
 * [rows, tokens]; with mask_evict != 0 an element is 1 when the token is
 * evicted (the reference's ~keep), else 1 when kept.  Any length: past
 * regions up to 786432 tokens are held in shared memory, longer ones are
 * re-read from `importance` on every radix pass (same result). */
FE_API int fe_select_tokens(const float* importance, int64_t rows, int64_t tokens, int64_t budget, int64_t recent,
                     int64_t pool_kernel, int64_t* indices, uint8_t* mask, int mask_evict, void* stream);

/* The whole evict() path in one call (attention, replay, selection).
 * Replaces `evict` (flash_evict/prefill.py:173-180).  row_stats is caller
 * workspace of 2*batch*q_heads*tokens floats.  mask is the eviction mask
 * (1 = evict). */
FE_API int fe_evict(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, const void* v,
             const int64_t* v_strides, void* out, float* importance, int64_t* indices, uint8_t* mask,
             float* row_stats, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens,
             int64_t channels, int dtype, int causal, float scale, float recency_decay,
             int64_t observation_window, int value_weighted, int64_t budget, int64_t recent,
             int64_t pool_kernel, void* stream);

/* KV compaction gather.  Replaces `gather_tokens(x, indices)` from the
 * adapters' kv_distill dependency, applied to K and V after selection
 * (flash_evict/kv_distill_adapter.py:38-39, flash_evict/streaming_adapter.py:86,
 * flash_evict/quality_adapter.py:109-110; README.md:31 gives its meaning as
 * x.gather(2, indices[..., None].expand(-1, -1, -1, channels))):
 *   k_out[b,h,j,:] = k[b,h,indices[b,h,j],:]   (and the same for v).
 * k, v: [batch, heads, tokens, channels] with element strides (channel
 * stride 1, other strides >= 0), elem_bytes bytes per element (1, 2, 4, 8);
 * v and v_out may both be NULL to gather K only.  indices: contiguous int64
 * [batch, heads, budget], any order.  k_out, v_out: contiguous
 * [batch, heads, budget, channels].  An index outside [0, tokens) does not
 * fault: its destination row is zero-filled and FE_STATUS_BAD_INDEX is raised
 * in the device status word (fe_device_status). */
FE_API int fe_gather_tokens(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                            const int64_t* indices, void* k_out, void* v_out, int64_t batch, int64_t heads,
                            int64_t tokens, int64_t budget, int64_t channels, int64_t elem_bytes, void* stream);
/* fe_select_tokens and fe_gather_tokens in one launch: rows = batch*heads of
 * importance are selected exactly as by fe_select_tokens, and each CTA of the
 * selection copies the K/V rows of the indices it produced into k_out/v_out
 * (layouts as in fe_gather_tokens).  Replaces the compress step of the
 * adapters, `select_tokens` followed by two `gather_tokens`
 * (flash_evict/kv_distill_adapter.py:35-39). */
FE_API int fe_select_gather(const float* importance, int64_t batch, int64_t heads, int64_t tokens, int64_t budget,
                            int64_t recent, int64_t pool_kernel, int64_t* indices, uint8_t* mask, int mask_evict,
                            const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                            void* k_out, void* v_out, int64_t channels, int64_t elem_bytes, void* stream);
/* Several selection policies in one launch: policy i selects budgets[i] tokens
 * of importance[i] (contiguous FP32 [batch*heads, tokens]) with recents[i]
 * reserved and pool_kernels[i] pooling, exactly as fe_select_tokens would,
 * writing indices[i] ([batch*heads, budgets[i]]) and masks[i].  With k != NULL
 * each policy also compacts K (and V, if not NULL) into k_outs[i] / v_outs[i]
 * as fe_select_gather does.  Replaces the per-method selection loop of the
 * paired multi-policy controller (flash_evict/quality_adapter.py:95-111,
 * choose_indices at :39-51): methods sharing one prefill differ only in
 * budget, reserved suffix and score tensor.  1 <= npolicies <= 8; the arrays
 * (budgets, recents, pool_kernels, and the pointer arrays) are host memory. */
FE_API int fe_select_multi(const float* const* importance, int64_t batch, int64_t heads, int64_t tokens,
                           int npolicies, const int64_t* budgets, const int64_t* recents,
                           const int64_t* pool_kernels, int64_t* const* indices, uint8_t* const* masks,
                           int mask_evict, const void* k, const int64_t* k_strides, const void* v,
                           const int64_t* v_strides, void* const* k_outs, void* const* v_outs, int64_t channels,
                           int64_t elem_bytes, void* stream);
/* fe_evict followed by the compaction of K and V into k_out/v_out
 * ([batch, kv_heads, budget, channels], dtype of the inputs), the selection
 * and the gather sharing one launch.  README.md:27-31 (evict, then gather). */
FE_API int fe_evict_compact(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                            const void* v, const int64_t* v_strides, void* out, float* importance, int64_t* indices,
                            uint8_t* mask, void* k_out, void* v_out, float* row_stats, int64_t batch,
                            int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels, int dtype,
                            int causal, float scale, float recency_decay, int64_t observation_window,
                            int value_weighted, int64_t budget, int64_t recent, int64_t pool_kernel, void* stream);
/* SnapKV observation-window scores, the reference's comparison baseline.
 * Replaces `snap_scores` (flash_evict/baselines.py:12-26): with
 * w = min(window, tokens), for the last w query rows of every query head
 *   p = softmax(round(Q_w K^T) * scale, causal)   (FP32)
 * where round() is the rounding of the FP32 dot products to `dtype` that the
 * reference's native-dtype matmul performs; p is summed over the w rows and
 * averaged over the G = q_heads/kv_heads query heads of each KV head:
 * scores: FP32 [batch, kv_heads, tokens], contiguous.  Two launches (split
 * row statistics, then a key-stationary scoring pass); the w x tokens matrix
 * is never stored.  workspace: at least fe_snap_workspace_floats(...) floats,
 * 8-byte aligned, contents irrelevant.  Q/K layout rules as for
 * fe_attention_fwd; channels <= 256. */
FE_API int64_t fe_snap_workspace_floats(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens,
                                        int64_t window);
FE_API int fe_snap_scores(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                          float* scores, float* workspace, int64_t workspace_floats, int64_t batch, int64_t q_heads,
                          int64_t kv_heads, int64_t tokens, int64_t channels, int dtype, float scale, int64_t window,
                          void* stream);
/* evict() without any device allocation: like fe_evict, but the row-statistics
 * scratch lives in a fixed array inside this library instead of a
 * caller-provided workspace.  No counterpart in the reference (which always
 * allocates through PyTorch); it exists for callers that cannot allocate
 * device memory when they evict -- custom pools that own all GPU memory,
 * engines that forbid cudaMalloc on the serving path, plain C/FFI hosts.
 *  - Limit: batch*q_heads*tokens <= 4194304 (the array is 32 MiB and is
 *    reserved on every GPU that loads the library until process exit);
 *    larger requests return FE_STATUS_UNSUPPORTED with a message.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress); make that first call before any stream capture.
 *  - All calls on a device share the one array: calls that can overlap on the
 *    GPU (different streams, no ordering between them) race on it.  Nothing
 *    in it has to start zeroed: the attention kernel writes every row the
 *    replay reads earlier on the same stream -- valid statistics, or NaN if
 *    that kernel gave up on a wait (watchdog), so an aborted call yields NaN
 *    importance, never the previous call's statistics.
 *  - A timeout of an earlier call's kernel is returned as this call's error
 *    when the host status word is attached; this entry point never attaches
 *    it (that allocates pinned host memory), so make one call of another
 *    entry point on the device first, or poll fe_device_status().
 *  - Calls no cudaMalloc, cudaFree or allocating library routine. */
FE_API int fe_evict_noalloc(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                            const void* v, const int64_t* v_strides, void* out, float* importance,
                            int64_t* indices, uint8_t* mask, int64_t batch, int64_t q_heads, int64_t kv_heads,
                            int64_t tokens, int64_t channels, int dtype, int causal, float scale,
                            float recency_decay, int64_t observation_window, int value_weighted, int64_t budget,
                            int64_t recent, int64_t pool_kernel, void* stream);

/* Read (and optionally clear) the device status word of `device`: the largest
 * FE_STATUS_* code any kernel raised since the last clear.  Synchronizes that
 * device; clearing also clears the device's host status word. */
FE_API int fe_device_status(int device, int clear, int* status_out);

/* Watchdog limit for every device-side wait, in nanoseconds (default 2e9). */
FE_API void fe_set_watchdog_ns(int64_t ns);

/* Launch a kernel whose bounded wait can never be satisfied, with the given
 * limit; it raises FE_STATUS_TIMEOUT and returns cleanly.  Used by tests to
 * exercise the timeout path without hanging a GPU.  Attaches the host status
 * word of the current device (it does not report an earlier pending code). */
FE_API int fe_watchdog_selftest(int64_t timeout_ns, void* stream);

/* Evaluate the kernels' two exp2 implementations elementwise: out_poly = the
 * packed FP32x2 FMA-pipe polynomial (Cody-Waite reduction + degree-4 minimax,
 * used for a share of the replay's exponentials; arguments below -125 give
 * 2^-125 * p(0), about 2.35e-38), out_mufu = the hardware ex2.approx.
 * Diagnostic for tests; no counterpart in the reference (Triton's exp2). */
FE_API int fe_selftest_exp2(const float* in, float* out_poly, float* out_mufu, int64_t n, void* stream);

/* Message describing the last error returned on the calling thread. */
FE_API const char* fe_last_error(void);

/* ABI version of this library. */
FE_API int fe_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_EVICT_B200_H */
