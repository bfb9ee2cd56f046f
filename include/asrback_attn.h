/*
 * asrback_attn.h: C ABI of the B200 (sm_100a) attention kernels that replace
 * the attention calls on asrback's decode and encoder hot path.
 *
 * Every entry point takes plain device pointers, element strides (in
 * elements, not bytes), sizes and a CUDA stream, launches its kernels on that
 * stream and returns at once: nothing here synchronizes, allocates device
 * memory or reads device memory back, so every call can be recorded in a CUDA
 * graph. Each call returns ASRBACK_OK or an error code; asrback_last_error()
 * then holds a one-line message for the calling thread.
 *
 * Faults found on the device (a row position outside the cache) cannot be
 * returned by a launch. The kernels skip that row, write zeros for it and set
 * a bit in the caller's `status` word (device memory, int32), which the caller
 * may read after the stream has finished.
 *
 * Reference call sites (paths inside the asrback project):
 *   - asrback_whisper_self_attention_step  replaces the fixed-shape step branch
 *     of DecoderLayer.forward, src/asrback/models/whisper.py:222-237
 *     (scatter_ of the step's key/value at each row's position, then
 *     MultiHeadAttention.attend with the step mask of whisper.py:262-264);
 *   - asrback_whisper_cross_attention_step replaces the cross-attention call
 *     whisper.py:239-240 (attend over the window's encoder keys, no mask);
 *   - asrback_whisper_self_attention_prefix and
 *     asrback_whisper_cross_attention_prefix replace the same two calls in
 *     DecoderLayer.forward's eager branch (whisper.py:228-236, 239-240) as
 *     the prompt pass (_prefill, whisper.py:847-849) and language detection
 *     (_detect_languages, whisper.py:979-981) use it: P tokens per window at
 *     positions 0..P-1, length == P, causal self-attention;
 *   - asrback_qwen3_attention_step replaces TextAttention.step between
 *     qkv_proj and o_proj, src/asrback/models/qwen3_asr.py:392-432, with
 *     _project (qwen3_asr.py:366-372: per-head RMSNorm of q and k, rotate-half
 *     RoPE) and the cache write (qwen3_asr.py:409-411) fused in;
 *   - asrback_whisper_encoder_attention replaces the unmasked SDPA call of
 *     MultiHeadAttention.forward, whisper.py:108-110 (via attend, :102-104),
 *     in the encoder layers (whisper.py:123-125);
 *   - asrback_varlen_attention replaces attend(q, k, v, segments, causal),
 *     src/asrback/models/qwen3_asr.py:152-181 (torch varlen_attn with equal
 *     query/key segments), called by TextAttention.prefill (qwen3_asr.py:
 *     374-390, causal) and AudioAttention.forward (qwen3_asr.py:214-219,
 *     non-causal windows);
 *   - asrback_whisper_cross_kv_projection replaces set_encoder_output's work
 *     per decoder layer (whisper.py:313-319): k_proj / v_proj of the encoder
 *     states (project_key_value, whisper.py:88-91) written into the
 *     cross-attention cache without the copy pass;
 *   - asrback_greedy_step replaces what a greedy step does after the decoder:
 *     the logits (whisper.py:337-342, qwen3_asr.py:1189 lm_head), _choose
 *     without sampling (whisper.py:962-975 with the suppress mask,
 *     qwen3_asr.py:1203-1213) and the decode-state update of _step
 *     (whisper.py:951-960, qwen3_asr.py:1190-1201).
 */
#ifndef ASRBACK_ATTN_H_
#define ASRBACK_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ASRBACK_API __attribute__((visibility("default")))
#else
#define ASRBACK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (the reference runs bfloat16 on CUDA, float32 on CPU). */
#define ASRBACK_BF16 0
#define ASRBACK_F32 1

/* Return codes. */
#define ASRBACK_OK 0
#define ASRBACK_ERR_ARGUMENT 1 /* a size, stride, alignment or pointer is invalid */
#define ASRBACK_ERR_CUDA 2     /* a CUDA call failed (launch, attribute, ...) */
#define ASRBACK_ERR_WORKSPACE 3 /* the workspace is smaller than needed */

/* Bits of the device-side status word. */
#define ASRBACK_STATUS_POSITION 1 /* a row's position was < 0 or >= cache length */
#define ASRBACK_STATUS_TIMEOUT 2  /* a bounded wait inside a kernel gave up */
#define ASRBACK_STATUS_SEGMENT 4  /* a segment of cu_seqlens lay outside the tensor or
                                     exceeded max_length (asrback_varlen_attention) */

/* Version of this ABI: (major << 16) | minor. */
ASRBACK_API int asrback_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
ASRBACK_API const char* asrback_last_error(void);

/* Number of SMs of the current device (for callers sizing their work). */
ASRBACK_API int asrback_device_sm_count(void);

/*
 * Bytes of workspace the decode entry points need for `batch` rows with
 * `heads` query heads of `head_dim` over at most `max_keys` keys per row
 * (cache view length). The workspace holds per-row completion counters and the
 * partial results of split rows. It must be zero-filled before its first use;
 * every call leaves its counters at zero again, so one workspace serves any
 * number of calls in stream order. Calls that run concurrently on different
 * streams need separate workspaces.
 */
ASRBACK_API size_t asrback_decode_workspace_bytes(int batch, int heads, int head_dim, int max_keys);

/*
 * Whisper decoder self-attention for one step (one query per row).
 *
 * query       (batch, heads, head_dim)  at query[b*q_stride_batch + h*q_stride_head + d]
 * key, value  (batch, heads, head_dim)  the step's new key/value, strides kv_stride_*
 * key_cache,  (batch, heads, cache_length, head_dim) at
 * value_cache   [b*cache_stride_batch + h*cache_stride_head + p*head_dim + d]
 *             (rows of one head contiguous: the layout of DecoderCache,
 *              whisper.py:156-196, possibly narrowed to a KV bucket)
 * positions   (batch,) int64, device: row b writes its key/value at
 *             positions[b] and attends to keys 0..positions[b]
 * out         (batch, heads, head_dim) at out[b*out_stride_batch + h*out_stride_head + d]
 * scale       softmax scale (1/sqrt(head_dim) in the reference)
 * head_dim    64 (Whisper); dtype ASRBACK_BF16 or ASRBACK_F32; all tensors
 *             share the dtype; pointers 16-byte aligned.
 */
ASRBACK_API int asrback_whisper_self_attention_step(
    int dtype, int batch, int heads, int head_dim, int cache_length,
    const void* query, int64_t q_stride_batch, int64_t q_stride_head,
    const void* key, const void* value, int64_t kv_stride_batch, int64_t kv_stride_head,
    void* key_cache, void* value_cache, int64_t cache_stride_batch, int64_t cache_stride_head,
    const int64_t* positions,
    void* out, int64_t out_stride_batch, int64_t out_stride_head,
    float scale, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Whisper decoder cross-attention for one step: every row attends, without a
 * mask, to all `length` encoder keys of its window. Layouts as above
 * (caches (batch, heads, length, head_dim), rows of one head contiguous).
 */
ASRBACK_API int asrback_whisper_cross_attention_step(
    int dtype, int batch, int heads, int head_dim, int length,
    const void* query, int64_t q_stride_batch, int64_t q_stride_head,
    const void* key_cache, const void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head,
    void* out, int64_t out_stride_batch, int64_t out_stride_head,
    float scale, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Whisper decoder self-attention for a prompt pass: `tokens` (P) query tokens
 * per window, token t attending causally to cache keys 0..t. This is the
 * eager branch of DecoderLayer.forward (whisper.py:228-236) with length == P
 * and positions 0..P-1, the only form its callers use: the caller has already
 * written the pass's keys/values into the cache at positions 0..P-1
 * (index_copy_, whisper.py:231-232); this call reads them and writes nothing
 * to the cache.
 *
 * query       (windows*tokens, heads, head_dim): window w's token t at row
 *             r = w*tokens + t, query[r*q_stride_token + h*q_stride_head + d]
 * key_cache,  (windows, heads, cache_length, head_dim) as for the step, with
 * value_cache   cache_length >= tokens
 * out         (windows*tokens, heads, head_dim), strides out_stride_*
 * workspace   asrback_whisper_prefix_workspace_bytes(windows, tokens, heads,
 *             head_dim, length) bytes (covers both prompt-pass calls)
 * windows*tokens <= 65535; other conditions as for the step.
 */
/*
 * Workspace bytes that asrback_whisper_self_attention_prefix (over `tokens`
 * cache positions) and asrback_whisper_cross_attention_prefix (over `length`
 * encoder keys) need for `windows` windows of `tokens` tokens: the larger of
 * the two. Host-only; 0 for non-positive sizes.
 */
ASRBACK_API size_t asrback_whisper_prefix_workspace_bytes(int windows, int tokens, int heads,
                                                          int head_dim, int length);

ASRBACK_API int asrback_whisper_self_attention_prefix(
    int dtype, int windows, int tokens, int heads, int head_dim, int cache_length,
    const void* query, int64_t q_stride_token, int64_t q_stride_head,
    const void* key_cache, const void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head,
    void* out, int64_t out_stride_token, int64_t out_stride_head,
    float scale, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Whisper decoder cross-attention for a prompt pass (whisper.py:239-240 in
 * the eager branch): each of a window's `tokens` query rows attends, without
 * a mask, to all `length` encoder keys of that window. Query and output rows
 * as in asrback_whisper_self_attention_prefix, caches as in
 * asrback_whisper_cross_attention_step; workspace
 * asrback_whisper_prefix_workspace_bytes(windows, tokens, heads, head_dim,
 * length). In bf16 with at most 128 tokens the call runs on the tensor cores
 * (a window's tokens are one query tile per head; no workspace used); past
 * 128 tokens each CTA takes 4 tokens of a window, so that every key staged in
 * shared memory serves all 4 queries; in float32 a CTA takes one token.
 */
ASRBACK_API int asrback_whisper_cross_attention_prefix(
    int dtype, int windows, int tokens, int heads, int head_dim, int length,
    const void* query, int64_t q_stride_token, int64_t q_stride_head,
    const void* key_cache, const void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head,
    void* out, int64_t out_stride_token, int64_t out_stride_head,
    float scale, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * The cross-attention step above, for callers that cannot allocate device
 * memory: no counterpart in the reference (which always runs inside PyTorch
 * and its caching allocator). A host that binds this C ABI from another
 * language may have no device allocator to hand out a workspace, and a serving
 * loop must not call cudaMalloc per request, since it synchronizes the device
 * and stalls every other stream. This entry point takes no workspace and
 * allocates nothing: its split-KV scratch is a 1 MiB file-scope device array
 * (per device that loads the library, held until exit) that covers up to 4096
 * split (row, head) units; larger splits are rejected with
 * ASRBACK_ERR_ARGUMENT. Same arguments and results as
 * asrback_whisper_cross_attention_step otherwise.
 *
 * The first call on a device looks up the array's device address (with that
 * device current) and should come before any stream capture. All calls share
 * the one array and clear its counters on their stream first, so calls that
 * overlap on the GPU (different streams, no ordering) race and must not be
 * issued.
 */
ASRBACK_API int asrback_whisper_cross_attention_step_noalloc(
    int dtype, int batch, int heads, int head_dim, int length,
    const void* query, int64_t q_stride_batch, int64_t q_stride_head,
    const void* key_cache, const void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head,
    void* out, int64_t out_stride_batch, int64_t out_stride_head,
    float scale, int32_t* status, void* stream);

/*
 * Qwen3 decoder attention for one step, between qkv_proj and o_proj.
 *
 * qkv          (batch, (heads + 2*kv_heads)*head_dim) at qkv[b*qkv_stride_batch + j]:
 *              q | k | v as qkv_proj writes them (qwen3_asr.py:366-369)
 * q_norm_weight, k_norm_weight  (head_dim,) RMSNorm weights, eps their epsilon
 * cos, sin     RoPE tables (table_length, head_dim), row stride table_stride;
 *              row positions[b] is used (qwen3_asr.py:507)
 * positions    (batch,) int64, device
 * key_cache,   (batch, cache_length, kv_heads, head_dim) at
 * value_cache    [b*cache_stride_batch + p*kv_heads*head_dim + h*head_dim + d]
 *              (KVCache, qwen3_asr.py:333-347, possibly narrowed to a bucket)
 * out          (batch, heads*head_dim) at out[b*out_stride_batch + h*head_dim + d]
 * Query head h reads key/value head h / (heads / kv_heads). head_dim 128,
 * kv_heads 8, heads 8 or 16 (grouped-query factor 1 or 2).
 */
ASRBACK_API int asrback_qwen3_attention_step(
    int dtype, int batch, int heads, int kv_heads, int head_dim, int cache_length,
    const void* qkv, int64_t qkv_stride_batch,
    const void* q_norm_weight, const void* k_norm_weight, float eps,
    const void* cos, const void* sin, int64_t table_stride, int table_length,
    const int64_t* positions,
    void* key_cache, void* value_cache, int64_t cache_stride_batch,
    void* out, int64_t out_stride_batch,
    float scale, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Whisper encoder self-attention (non-causal) over `length` frames.
 *
 * q, k, v, out  (batch, heads, length, head_dim) at
 *               [b*stride_batch + h*stride_head + s*stride_seq + d]; the four
 *               tensors share the strides (the reference's transposed views
 *               of (batch, length, heads*head_dim) projections have
 *               stride_seq = heads*head_dim, stride_head = head_dim).
 * head_dim 64, dtype ASRBACK_BF16; 16-byte aligned rows.
 */
ASRBACK_API int asrback_whisper_encoder_attention(
    int dtype, int batch, int heads, int head_dim, int length,
    const void* q, const void* k, const void* v, void* out,
    int64_t stride_batch, int64_t stride_head, int64_t stride_seq,
    float scale, int32_t* status, void* stream);

/*
 * Attention within segments of packed tokens: asrback's attend(q, k, v,
 * segments, causal) (qwen3_asr.py:152-181), i.e. varlen_attn(q, k, v,
 * cu_seqlens, cu_seqlens, max_length, max_length, window_size=(-1, 0) if
 * causal else (-1, -1), enable_gqa) with the same segments for queries and
 * keys.
 *
 * q, out        (tokens, heads, head_dim) at [t*stride_token + h*stride_head + d];
 * key, value    (tokens, kv_heads, head_dim), each with its own strides (the
 *               reference hands attend a rotated, contiguous key and the value
 *               as a view of the fused projection);
 *               query head h reads key/value head h / (heads / kv_heads);
 * cu_seqlens    device int32, segments + 1 entries: segment s is tokens
 *               cu_seqlens[s] .. cu_seqlens[s+1]-1 (the reference's
 *               Segments.starts); every segment at most max_length tokens;
 * causal        nonzero: token i of a segment attends to tokens 0..i of it.
 * head_dim 64 or 128; dtype ASRBACK_BF16 (tensor cores) or ASRBACK_F32.
 * A segment outside [0, tokens) or longer than max_length is skipped (its
 * output rows are not written) and sets ASRBACK_STATUS_SEGMENT.
 */
ASRBACK_API int asrback_varlen_attention(
    int dtype, int tokens, int heads, int kv_heads, int head_dim,
    const void* q, int64_t q_stride_token, int64_t q_stride_head,
    const void* key, int64_t k_stride_token, int64_t k_stride_head,
    const void* value, int64_t v_stride_token, int64_t v_stride_head,
    const int32_t* cu_seqlens, int segments, int max_length, int causal,
    void* out, int64_t out_stride_token, int64_t out_stride_head,
    float scale, int32_t* status, void* stream);

/*
 * Cross-attention keys and values of one Whisper decoder layer, written into
 * the cache layout:
 *   keys[b][h][t][d]   = sum_k x[b][t][k] * k_weight[h*64 + d][k]
 *   values[b][h][t][d] = sum_k x[b][t][k] * v_weight[h*64 + d][k] + v_bias[h*64 + d]
 * for b < batch, t < tokens, heads = width / 64, d < 64.
 * x            (batch, tokens, width) at [b*x_stride_batch + t*x_stride_token + k]
 *              (the encoder output);
 * k_weight, v_weight (width, width) rows at w_stride (nn.Linear weights:
 *              out_features x in_features); v_bias (width,) or null;
 * keys, values (batch, heads, length >= tokens, 64) cache views at
 *              [b*c_stride_batch + h*c_stride_head + t*c_stride_token + d]
 *              (cross_keys[layer, :batch] / cross_values[layer, :batch]).
 * width a multiple of 128. dtype ASRBACK_BF16 (tensor cores; fp32 sums, the
 * bias added in fp32, one rounding to bf16 as nn.Linear returns it) or
 * ASRBACK_F32.
 */
ASRBACK_API int asrback_whisper_cross_kv_projection(
    int dtype, int batch, int tokens, int width,
    const void* x, int64_t x_stride_batch, int64_t x_stride_token,
    const void* k_weight, const void* v_weight, int64_t w_stride, const void* v_bias,
    void* keys, void* values,
    int64_t c_stride_batch, int64_t c_stride_head, int64_t c_stride_token,
    int32_t* status, void* stream);

/*
 * Workspace of asrback_greedy_step for up to `batch` rows: a header of ticket
 * counters (zero before the first call; every call leaves them zero) and the
 * per-CTA and per-group partials. 16-byte aligned; reusable by consecutive
 * calls on one stream.
 */
ASRBACK_API size_t asrback_greedy_step_workspace_bytes(int batch);

/*
 * One greedy step after the decoder, for `batch` rows:
 *   logits[b][v] = hidden[b] . weight[v]  (bf16: fp32 sums rounded to bf16,
 *                  as the reference's bf16 matmul returns them; f32: fp32);
 *   suppressed tokens (suppress[v] != 0, or suppress null: none) get -inf;
 *   token[b]   = first index of the row's maximum (torch argmax);
 *   logprob[b] = log_softmax(logits[b])[token[b]] = -ln(sum_v exp(x - max)).
 * hidden (batch, hidden_dim) rows at hidden_stride; weight (vocab, hidden_dim)
 * rows at weight_stride (Whisper's tied embedding, Qwen3's lm_head.weight).
 * out_token (int64) / out_logprob (float), if given, receive token / logprob.
 * If `tokens` is given, the decode state is updated as _step does (int64
 * tokens at tokens[b * tokens_stride], position, end; uint8 finished; float
 * sum_logprobs; int64 generated (batch, generated_cols) at generated_stride):
 *   a finished row keeps its token and position; an active row advances;
 *   sum_logprobs[b] += logprob (active rows); generated[b][position] = token;
 *   finished[b] |= token in eos_ids[0..n_eos) or position >= end[b].
 * eos_ids is a HOST array (at most 8), copied into the launch.
 * dtype ASRBACK_BF16: batch <= 128, hidden_dim and strides multiples of 8;
 * ASRBACK_F32: batch <= 64, batch * hidden_dim * 4 <= 200 KB.
 * A position outside [0, generated_cols) skips the write and sets
 * ASRBACK_STATUS_POSITION.
 */
ASRBACK_API int asrback_greedy_step(
    int dtype, int batch, int vocab, int hidden_dim,
    const void* hidden, int64_t hidden_stride,
    const void* weight, int64_t weight_stride,
    const uint8_t* suppress,
    int64_t* out_token, float* out_logprob,
    int64_t* tokens, int64_t tokens_stride, int64_t* position, const int64_t* end,
    uint8_t* finished, float* sum_logprobs,
    int64_t* generated, int64_t generated_stride, int64_t generated_cols,
    const int64_t* eos_ids, int n_eos,
    void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Self-test of the kernels' bounded waits: one CTA waits on an mbarrier that
 * nothing completes, gives up after budget_ns (at most 1 s) of %globaltimer,
 * sets ASRBACK_STATUS_TIMEOUT in `status` and exits; the context stays usable.
 * Lets a host check the timeout path on its own GPU without faulting it.
 */
ASRBACK_API int asrback_selftest_bounded_wait(int64_t budget_ns, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ASRBACK_ATTN_H_ */
