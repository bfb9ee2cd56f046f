// Whisper encoder self-attention (non-causal), MultiHeadAttention.forward at
// whisper.py:108-110 calling F.scaled_dot_product_attention unmasked.
//
// bfloat16 runs on the tensor cores (encoder_attention_tc.cu). float32 (the
// reference's CPU dtype, used for the 1e-4 parity check) runs here on the
// SIMT path: one thread per query row, the block's keys and values staged in
// shared memory, online softmax in fp32.
#include "capi_internal.h"
#include "common.cuh"

namespace asrback {

namespace {

constexpr int kRows = 64;   // query rows per CTA (one per thread)
constexpr int kKeys = 64;   // keys per shared-memory tile
constexpr int kDim = 64;

struct EncoderParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t sb, sh, ss;
  int length;
  int heads;
  float scale_log2;
};

template <typename T>
__device__ __forceinline__ float to_f(T x) {
  return static_cast<float>(x);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__global__ void __launch_bounds__(kRows) encoder_attention_simt(const __grid_constant__ EncoderParams p) {
  __shared__ float ks[kKeys][kDim];
  __shared__ float vs[kKeys][kDim];
  const int b = blockIdx.z, h = blockIdx.y;
  const int row = blockIdx.x * kRows + threadIdx.x;
  const int64_t base = b * p.sb + h * p.sh;
  const T* q = static_cast<const T*>(p.q) + base;
  const T* k = static_cast<const T*>(p.k) + base;
  const T* v = static_cast<const T*>(p.v) + base;
  float qr[kDim], o[kDim];
  const bool valid = row < p.length;
#pragma unroll
  for (int d = 0; d < kDim; ++d) {
    qr[d] = valid ? to_f(q[row * p.ss + d]) * p.scale_log2 : 0.f;
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < p.length; k0 += kKeys) {
    const int n = min(kKeys, p.length - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < kKeys * kDim; i += kRows) {
      const int r = i / kDim, d = i % kDim;
      ks[r][d] = r < n ? to_f(k[(k0 + r) * p.ss + d]) : 0.f;
      vs[r][d] = r < n ? to_f(v[(k0 + r) * p.ss + d]) : 0.f;
    }
    __syncthreads();
    float s[kKeys];
    float mt = m;
#pragma unroll 4
    for (int r = 0; r < kKeys; ++r) {
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < kDim; ++d) dot = fmaf(qr[d], ks[r][d], dot);
      s[r] = r < n ? dot : -INFINITY;
      mt = fmaxf(mt, s[r]);
    }
    const float alpha = fast_exp2(m - mt);
    l *= alpha;
#pragma unroll
    for (int d = 0; d < kDim; ++d) o[d] *= alpha;
#pragma unroll 4
    for (int r = 0; r < kKeys; ++r) {
      const float pr = fast_exp2(s[r] - mt);
      l += pr;
#pragma unroll
      for (int d = 0; d < kDim; ++d) o[d] = fmaf(pr, vs[r][d], o[d]);
    }
    m = mt;
  }
  if (!valid) return;
  T* out = static_cast<T*>(p.out) + base + row * p.ss;
  const float inv = 1.f / l;
#pragma unroll
  for (int d = 0; d < kDim; ++d) out[d] = T(o[d] * inv);
}

}  // namespace

int encoder_attention_tc(int batch, int heads, int length, const void* q, const void* k,
                         const void* v, void* out, int64_t sb, int64_t sh, int64_t ss, float scale,
                         int32_t* status, cudaStream_t stream);

}  // namespace asrback

using namespace asrback;

extern "C" int asrback_whisper_encoder_attention(int dtype, int batch, int heads, int head_dim,
                                                 int length, const void* q, const void* k,
                                                 const void* v, void* out, int64_t stride_batch,
                                                 int64_t stride_head, int64_t stride_seq,
                                                 float scale, int32_t* status, void* stream) {
  (void)status;
  if (dtype != ASRBACK_BF16 && dtype != ASRBACK_F32)
    return fail(ASRBACK_ERR_ARGUMENT, "dtype must be ASRBACK_BF16 or ASRBACK_F32, got %d", dtype);
  if (head_dim != kDim)
    return fail(ASRBACK_ERR_ARGUMENT, "head_dim must be 64 (Whisper), got %d", head_dim);
  if (batch < 1 || heads < 1 || length < 1 || batch > 65535 || heads > 65535)
    return fail(ASRBACK_ERR_ARGUMENT, "batch, heads and length must be positive");
  if (!q || !k || !v || !out) return fail(ASRBACK_ERR_ARGUMENT, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(ASRBACK_ERR_ARGUMENT, "tensor pointers must be 16-byte aligned");
  const int64_t elem = dtype == ASRBACK_BF16 ? 2 : 4;
  for (int64_t s : {stride_batch, stride_head, stride_seq})
    if (s <= 0 || (s * elem) % 16 != 0)
      return fail(ASRBACK_ERR_ARGUMENT, "strides must be positive multiples of 16 bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == ASRBACK_BF16) {
    // Tensor cores (tcgen05, TMEM accumulators): encoder_attention_tc.cu.
    if (int rc = encoder_attention_tc(batch, heads, length, q, k, v, out, stride_batch,
                                      stride_head, stride_seq, scale, status, s))
      return rc;
    return ok();
  }
  EncoderParams p{q, k, v, out, stride_batch, stride_head, stride_seq, length, heads,
                  scale * 1.4426950408889634f};
  dim3 grid((length + kRows - 1) / kRows, heads, batch);
  encoder_attention_simt<float><<<grid, kRows, 0, s>>>(p);
  if (int rc = check_cuda(cudaGetLastError(), "encoder attention launch")) return rc;
  return ok();
}
