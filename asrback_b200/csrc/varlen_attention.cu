// Attention within the segments of packed (tokens, heads, head_dim) tensors:
// asrback's `attend(q, k, v, segments, causal)` (qwen3_asr.py:152-181), i.e.
// torch's varlen_attn with equal query and key segments, window (-1, 0) when
// causal, grouped-query heads. bfloat16 runs on the tensor cores
// (varlen_attention_tc.cu); float32 (the reference's CPU dtype, for the 1e-4
// parity check) runs here: one thread per query row, keys and values staged
// through shared memory, online softmax in fp32.
#include "capi_internal.h"
#include "common.cuh"

namespace asrback {

int varlen_attention_tc(int tokens, int heads, int kv_heads, int head_dim, const void* q,
                        int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                        int64_t k_head, const void* v, int64_t v_tok, int64_t v_head,
                        const int32_t* cu, int segments,
                        int max_length, int causal, void* out, int64_t o_tok, int64_t o_head,
                        float scale, int32_t* status, cudaStream_t stream);

namespace {

constexpr int kRowsS = 64;  // query rows per CTA (one per thread)
constexpr int kKeysS = 32;  // keys per shared-memory tile

struct SimtParams {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  int64_t q_tok, q_head, k_tok, k_head, v_tok, v_head, o_tok, o_head;
  const int32_t* cu;
  int tokens;
  int max_length;
  int group;
  int causal;
  float scale_log2;
  int32_t* status;
};

template <int D>
__global__ void __launch_bounds__(kRowsS) varlen_attention_simt(const __grid_constant__ SimtParams p) {
  __shared__ float ks[kKeysS][D];
  __shared__ float vs[kKeysS][D];
  const int seg = blockIdx.z, h = blockIdx.y;
  const int start = p.cu[seg];
  const int len = p.cu[seg + 1] - start;
  if (start < 0 || len < 0 || start + len > p.tokens || len > p.max_length) {
    if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0 && p.status)
      atomicOr(p.status, ASRBACK_STATUS_SEGMENT);
    return;
  }
  const int first_row = blockIdx.x * kRowsS;
  if (first_row >= len) return;
  const int row = first_row + threadIdx.x;
  const int kvh = h / p.group;
  const bool valid = row < len;
  const int limit = p.causal ? min(len, row + 1) : len;
  const int block_limit = p.causal ? min(len, first_row + kRowsS) : len;
  float qr[D], o[D];
  const float* q = p.q + static_cast<int64_t>(start + row) * p.q_tok + h * p.q_head;
#pragma unroll
  for (int d = 0; d < D; ++d) {
    qr[d] = valid ? q[d] * p.scale_log2 : 0.f;
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < block_limit; k0 += kKeysS) {
    const int n = min(kKeysS, block_limit - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < kKeysS * D; i += kRowsS) {
      const int r = i / D, d = i % D;
      const int64_t tok = start + k0 + r;
      ks[r][d] = r < n ? p.k[tok * p.k_tok + kvh * p.k_head + d] : 0.f;
      vs[r][d] = r < n ? p.v[tok * p.v_tok + kvh * p.v_head + d] : 0.f;
    }
    __syncthreads();
    float s[kKeysS];
    float mt = m;
#pragma unroll 4
    for (int r = 0; r < kKeysS; ++r) {
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) dot = fmaf(qr[d], ks[r][d], dot);
      s[r] = k0 + r < limit ? dot : -INFINITY;
      mt = fmaxf(mt, s[r]);
    }
    if (mt == -INFINITY) continue;  // nothing this row may read in this tile
    const float alpha = fast_exp2(m - mt);
    l *= alpha;
#pragma unroll
    for (int d = 0; d < D; ++d) o[d] *= alpha;
#pragma unroll 4
    for (int r = 0; r < kKeysS; ++r) {
      const float pr = fast_exp2(s[r] - mt);
      l += pr;
#pragma unroll
      for (int d = 0; d < D; ++d) o[d] = fmaf(pr, vs[r][d], o[d]);
    }
    m = mt;
  }
  if (!valid) return;
  float* out = p.out + static_cast<int64_t>(start + row) * p.o_tok + h * p.o_head;
  const float inv = 1.f / l;
#pragma unroll
  for (int d = 0; d < D; ++d) out[d] = o[d] * inv;
}

}  // namespace

}  // namespace asrback

using namespace asrback;

extern "C" int asrback_varlen_attention(int dtype, int tokens, int heads, int kv_heads,
                                        int head_dim, const void* q, int64_t q_stride_token,
                                        int64_t q_stride_head, const void* key,
                                        int64_t k_stride_token, int64_t k_stride_head,
                                        const void* value, int64_t v_stride_token,
                                        int64_t v_stride_head, const int32_t* cu_seqlens, int segments, int max_length,
                                        int causal, void* out, int64_t out_stride_token,
                                        int64_t out_stride_head, float scale, int32_t* status,
                                        void* stream) {
  if (dtype != ASRBACK_BF16 && dtype != ASRBACK_F32)
    return fail(ASRBACK_ERR_ARGUMENT, "dtype must be ASRBACK_BF16 or ASRBACK_F32, got %d", dtype);
  if (head_dim != 64 && head_dim != 128)
    return fail(ASRBACK_ERR_ARGUMENT, "head_dim must be 64 or 128, got %d", head_dim);
  if (tokens < 1 || heads < 1 || kv_heads < 1 || segments < 1 || max_length < 1 ||
      heads > 65535 || segments > 65535)
    return fail(ASRBACK_ERR_ARGUMENT,
                "tokens, heads, kv_heads, segments and max_length must be positive (got %d, %d, "
                "%d, %d, %d)",
                tokens, heads, kv_heads, segments, max_length);
  if (heads % kv_heads != 0)
    return fail(ASRBACK_ERR_ARGUMENT, "heads (%d) must be a multiple of kv_heads (%d)", heads,
                kv_heads);
  if (!q || !key || !value || !out || !cu_seqlens)
    return fail(ASRBACK_ERR_ARGUMENT, "null tensor pointer");
  if (!aligned16(q) || !aligned16(key) || !aligned16(value) || !aligned16(out))
    return fail(ASRBACK_ERR_ARGUMENT, "tensor pointers must be 16-byte aligned");
  const int64_t elem = dtype == ASRBACK_BF16 ? 2 : 4;
  for (int64_t s : {q_stride_token, q_stride_head, k_stride_token, k_stride_head, v_stride_token,
                    v_stride_head, out_stride_token, out_stride_head})
    if (s <= 0 || (s * elem) % 16 != 0)
      return fail(ASRBACK_ERR_ARGUMENT, "strides must be positive multiples of 16 bytes");
  if (q_stride_head < head_dim || k_stride_head < head_dim || v_stride_head < head_dim ||
      out_stride_head < head_dim || q_stride_token < (int64_t)heads * head_dim ||
      k_stride_token < (int64_t)kv_heads * head_dim || v_stride_token < (int64_t)kv_heads * head_dim ||
      out_stride_token < (int64_t)heads * head_dim)
    return fail(ASRBACK_ERR_ARGUMENT, "strides do not hold (tokens, heads, head_dim) rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == ASRBACK_BF16) {
    if (int rc = varlen_attention_tc(tokens, heads, kv_heads, head_dim, q, q_stride_token,
                                     q_stride_head, key, k_stride_token, k_stride_head, value,
                                     v_stride_token, v_stride_head, cu_seqlens, segments, max_length, causal, out,
                                     out_stride_token, out_stride_head, scale, status, s))
      return rc;
    return ok();
  }
  SimtParams p{static_cast<const float*>(q), static_cast<const float*>(key),
               static_cast<const float*>(value), static_cast<float*>(out), q_stride_token,
               q_stride_head, k_stride_token, k_stride_head, v_stride_token, v_stride_head,
               out_stride_token, out_stride_head,
               cu_seqlens, tokens, max_length, heads / kv_heads, causal ? 1 : 0,
               scale * 1.4426950408889634f, status};
  dim3 grid((max_length + kRowsS - 1) / kRowsS, heads, segments);
  if (head_dim == 128)
    varlen_attention_simt<128><<<grid, kRowsS, 0, s>>>(p);
  else
    varlen_attention_simt<64><<<grid, kRowsS, 0, s>>>(p);
  if (int rc = check_cuda(cudaGetLastError(), "varlen attention launch")) return rc;
  return ok();
}
