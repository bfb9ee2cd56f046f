// Cross-attention key/value projection straight into the Whisper decoder's
// cache layout: for one decoder layer and windows b < batch,
//   keys[b][h][t][d]   = sum_k x[b][t][k] * Wk[h*64 + d][k]
//   values[b][h][t][d] = sum_k x[b][t][k] * Wv[h*64 + d][k] + bv[h*64 + d]
// Replaces set_encoder_output (whisper.py:313-319): per layer,
// encoder_attn.project_key_value (k_proj without bias, v_proj with bias,
// whisper.py:88-91), _split_heads, and the copy into cross_keys /
// cross_values[index, :batch]. The copy pass is gone: the GEMM's epilogue
// writes each head's rows where the cache keeps them.
//
// bf16 on the tensor cores. A tile is 128 tokens of one window (M) x kN
// output features (N: kN / 64 heads of either K or V) x the width in
// 64-element chunks (K). Persistent CTAs take tiles window by window, the
// feature tiles fastest, so that the CTAs running together share the
// window's rows and every CTA shares the weights in L2. Warp 0 streams the
// chunks (TMA: a 3-D map over the windows' rows, tokens past the window read
// as zeros; 2-D maps over the weights) through a 4-stage ring; warp 1 issues
// tcgen05.mma into two TMEM accumulators (both warps run their loops
// warp-wide and issue from an elected lane); warps 4-7 (thread = token) add the
// bias, round to bf16 and store each head's 32 rows per warp as 4 KB of
// contiguous cache, staged through shared memory. float32 runs a SIMT tiled
// GEMM with the same output layout.
#include <algorithm>

#include "capi_internal.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace asrback {
namespace {

using namespace tc;

constexpr int kHeadDim = 64;
constexpr int kRows = 128;  // tokens per tile (= TMEM lanes)
constexpr int kChunk = 64;  // width elements per K chunk (128 bytes of bf16)

struct ProjParams {
  const __nv_bfloat16* bias_v;  // (width,), or null
  void* out_k;
  void* out_v;
  int64_t o_sb, o_sh, o_st;  // cache strides (elements); d is contiguous
  int batch, tokens, width;
  int tiles_m, tiles_n;
  int32_t* status;
};

template <int kN>
struct ProjShape {
  static constexpr int kABytes = kRows * 128;  // 128 tokens x 64 bf16
  static constexpr int kBBytes = kN * 128;     // kN features x 64 bf16
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = kN == 256 ? 4 : 6;
  static constexpr int kOffStage = kStages * kStageBytes;  // epilogue staging, 4 warps x 4 KB
  static constexpr int kOffBar = kOffStage + 4 * 32 * 128;
  static constexpr int kNumBars = 2 * kStages + 4;  // full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int kOffSlot = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffSlot + 16 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory exceeds a CTA's 227 KB");
};

template <int kN>
__global__ void __launch_bounds__(256, 1)
    cross_kv_projection_tc(const __grid_constant__ CUtensorMap map_x,
                           const __grid_constant__ CUtensorMap map_wk,
                           const __grid_constant__ CUtensorMap map_wv,
                           const __grid_constant__ ProjParams p) {
  using Sh = ProjShape<kN>;
  constexpr int S = Sh::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Sh::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sh::kOffSlot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.batch * p.tiles_m * p.tiles_n;
  const int chunks = (p.width + kChunk - 1) / kChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  bool timed_out = false;

  // Tile index -> window, token tile, feature tile (feature tiles fastest).
  auto tile_coords = [&](int index, int& b, int& t0, int& n0) {
    n0 = (index % p.tiles_n) * kN;
    t0 = ((index / p.tiles_n) % p.tiles_m) * kRows;
    b = index / (p.tiles_n * p.tiles_m);
  };

  // The TMA and MMA warps run their loops warp-wide (waits by every lane, the
  // loop state warp-uniform) and issue from one elected lane.
  auto wait_warp = [](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
  };
  // One lane per warp, elected once: a tcgen05.commit tracks the MMAs of its
  // own thread, so the MMA warp's issues and commits all come from it.
  const bool leader = elect_one();
  if (warp == 0) {
    if (leader) {
      prefetch_tensormap(&map_x);
      prefetch_tensormap(&map_wk);
      prefetch_tensormap(&map_wv);
    }
    __syncwarp();
    const uint64_t keep = l2_evict_last_policy();
    int g = 0;
    bool ok = true;
    for (int index = blockIdx.x; index < tiles && ok; index += gridDim.x) {
      int b, t0, n0;
      tile_coords(index, b, t0, n0);
      const bool is_v = n0 >= p.width;
      const CUtensorMap* map_w = is_v ? &map_wv : &map_wk;
      const int row0 = is_v ? n0 - p.width : n0;
      for (int kc = 0; kc < chunks; ++kc, ++g) {
        const int s = g % S;
        if (g >= S) ok = wait_warp(&empty[s], ((g / S) - 1) & 1);
        if (!ok) break;
        if (leader) {
          uint8_t* stage = smem + s * Sh::kStageBytes;
          mbar_arrive_expect_tx(&full[s], Sh::kStageBytes);
          tma_load_3d(stage, &map_x, kc * kChunk, t0, b, &full[s]);
          tma_load_2d_hint(stage + Sh::kABytes, map_w, kc * kChunk, row0, &full[s], keep);
        }
        __syncwarp();
      }
    }
    timed_out = !ok;
  } else if (warp == 1) {
    constexpr uint32_t kIdesc = idesc_bf16(kRows, kN, false);
    const uint64_t a_desc = sw128_desc(smem_addr(smem), 16, 1024);
    const uint64_t b_desc = sw128_desc(smem_addr(smem + Sh::kABytes), 16, 1024);
    constexpr uint64_t kStage = Sh::kStageBytes >> 4;
    int g = 0, lt = 0;
    bool ok = true;
    for (int index = blockIdx.x; index < tiles && ok; index += gridDim.x, ++lt) {
      const int a = lt & 1;
      if (lt >= 2) ok = wait_warp(&acc_empty[a], ((lt >> 1) - 1) & 1);
      tc_fence_after();
      for (int kc = 0; kc < chunks && ok; ++kc, ++g) {
        const int s = g % S;
        ok = wait_warp(&full[s], (g / S) & 1);
        if (!ok) break;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int k = 0; k < kChunk / 16; ++k)
            mma_ss(tmem + a * kN, a_desc + s * kStage + 2 * k, b_desc + s * kStage + 2 * k, kIdesc,
                   kc > 0 || k > 0);
          mma_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok) {
        if (leader) mma_commit(&acc_full[a]);
        __syncwarp();
      }
    }
    timed_out = !ok;
  } else if (warp >= 4) {
    // Thread = token row of the tile (= TMEM lane).
    const int quarter = warp & 3;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* stage = smem + Sh::kOffStage + quarter * 32 * 128;
    bool ok = true;
    int lt = 0;
    for (int index = blockIdx.x; index < tiles; index += gridDim.x, ++lt) {
      const int a = lt & 1;
      // Warp-uniform, since the TMEM reads below are warp-wide.
      ok = __all_sync(0xffffffffu, ok && mbar_spin_bounded(&acc_full[a], (lt >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      int b, t0, n0;
      tile_coords(index, b, t0, n0);
      const bool is_v = n0 >= p.width;
      const int f0 = is_v ? n0 - p.width : n0;  // first feature of the tile within K or V
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(is_v ? p.out_v : p.out_k) + b * p.o_sb;
      const int row0 = t0 + quarter * 32;  // the warp's first token
#pragma unroll 1
      for (int hh = 0; hh < kN / kHeadDim; ++hh) {
        float x[64];
        tmem_ld32(tmem + lane_bits + a * kN + hh * kHeadDim, x);
        tmem_ld32(tmem + lane_bits + a * kN + hh * kHeadDim + 32, x + 32);
        if (is_v && p.bias_v) {
          const __nv_bfloat16* bias = p.bias_v + f0 + hh * kHeadDim;
#pragma unroll
          for (int i = 0; i < 64; ++i) x[i] += __bfloat162float(bias[i]);
        }
        // Row `lane` of the warp's 32 into the staging rows (16-byte chunk c
        // at c ^ (row & 7): eight rows' chunks in distinct banks), then each
        // store instruction writes four rows' 128 contiguous bytes.
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 u;
          u.x = bf16x2(x[8 * c], x[8 * c + 1]);
          u.y = bf16x2(x[8 * c + 2], x[8 * c + 3]);
          u.z = bf16x2(x[8 * c + 4], x[8 * c + 5]);
          u.w = bf16x2(x[8 * c + 6], x[8 * c + 7]);
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) = u;
        }
        __syncwarp();
        __nv_bfloat16* head = out + static_cast<int64_t>(f0 / kHeadDim + hh) * p.o_sh;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3), c = lane & 7;
          if (row0 + r < p.tokens) {
            const uint4 u =
                *reinterpret_cast<const uint4*>(stage + r * 128 + ((c ^ (r & 7)) << 4));
            *reinterpret_cast<uint4*>(head + static_cast<int64_t>(row0 + r) * p.o_st + 8 * c) = u;
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    if (!ok) timed_out = true;
  }
  if (timed_out && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kN);
  }
}

// ------------------------------------------------------------ float32, SIMT

constexpr int kSimtTile = 64;  // 64 tokens x 64 features (one head) per CTA
constexpr int kSimtK = 16;

__global__ void __launch_bounds__(256)
    cross_kv_projection_simt(const float* __restrict__ x, int64_t x_sb, int64_t x_st,
                             const float* __restrict__ wk, const float* __restrict__ wv,
                             int64_t w_stride, const float* __restrict__ bias_v,
                             const __grid_constant__ ProjParams p) {
  __shared__ float xs[kSimtK][kSimtTile + 1];
  __shared__ float ws[kSimtK][kSimtTile + 1];
  griddep_wait();
  griddep_launch_dependents();
  const int t0 = blockIdx.x * kSimtTile;
  const int head = blockIdx.y % (p.width / kHeadDim);
  const bool is_v = blockIdx.y >= p.width / kHeadDim;
  const int b = blockIdx.z;
  const float* w = (is_v ? wv : wk) + static_cast<int64_t>(head) * kHeadDim * w_stride;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 4 x 4 outputs each
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.width; k0 += kSimtK) {
    for (int i = threadIdx.x; i < kSimtK * kSimtTile; i += 256) {
      const int kk = i % kSimtK, r = i / kSimtK;
      const int t = t0 + r;
      xs[kk][r] = (t < p.tokens && k0 + kk < p.width) ? x[b * x_sb + t * x_st + k0 + kk] : 0.f;
      ws[kk][r] = (k0 + kk < p.width) ? w[static_cast<int64_t>(r) * w_stride + k0 + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtK; ++kk)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xs[kk][ty * 4 + i], ws[kk][tx * 4 + j], acc[i][j]);
    __syncthreads();
  }
  float* out = static_cast<float*>(is_v ? p.out_v : p.out_k) + b * p.o_sb + head * p.o_sh;
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= p.tokens) continue;
    for (int j = 0; j < 4; ++j) {
      const int d = tx * 4 + j;
      const float bias = is_v && bias_v ? bias_v[head * kHeadDim + d] : 0.f;
      out[static_cast<int64_t>(t) * p.o_st + d] = acc[i][j] + bias;
    }
  }
}

int encode_map(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
               const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  int rc = ASRBACK_OK;
  auto encode = tensor_map_encoder(&rc);
  if (!encode) return rc;
  cuuint32_t elem_strides[3] = {1, 1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                        strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(ASRBACK_ERR_ARGUMENT, "cuTensorMapEncodeTiled rejected the layout (error %d)",
                (int)res);
  return ASRBACK_OK;
}

template <int kN>
int launch_tc(int batch, int tokens, int width, const void* x, int64_t x_sb, int64_t x_st,
              const void* wk, const void* wv, int64_t w_stride, ProjParams p, cudaStream_t stream) {
  using Sh = ProjShape<kN>;
  CUtensorMap mx, mk, mv;
  {
    cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)tokens, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)x_st * 2, (cuuint64_t)x_sb * 2};
    cuuint32_t box[3] = {kChunk, kRows, 1};
    if (int rc = encode_map(&mx, 3, x, dims, strides, box)) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)width};
    cuuint64_t strides[1] = {(cuuint64_t)w_stride * 2};
    cuuint32_t box[2] = {kChunk, kN};
    if (int rc = encode_map(&mk, 2, wk, dims, strides, box)) return rc;
    if (int rc = encode_map(&mv, 2, wv, dims, strides, box)) return rc;
  }
  p.tiles_m = (tokens + kRows - 1) / kRows;
  p.tiles_n = 2 * width / kN;
  auto kernel = cross_kv_projection_tc<kN>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 Sh::kSmemBytes),
                            "cudaFuncSetAttribute(cross kv projection)"))
      return rc;
    prepared_device = device;
  }
  const int tiles = batch * p.tiles_m * p.tiles_n;
  const int ctas = std::min(tiles, sm_count());
  return launch_pdl(kernel, dim3(ctas), dim3(256), Sh::kSmemBytes, stream,
                    "cross kv projection (tensor core) launch", mx, mk, mv, p);
}

}  // namespace
}  // namespace asrback

using namespace asrback;

extern "C" int asrback_whisper_cross_kv_projection(
    int dtype, int batch, int tokens, int width, const void* x, int64_t x_stride_batch,
    int64_t x_stride_token, const void* k_weight, const void* v_weight, int64_t w_stride,
    const void* v_bias, void* keys, void* values, int64_t c_stride_batch, int64_t c_stride_head,
    int64_t c_stride_token, int32_t* status, void* stream) {
  if (dtype != ASRBACK_BF16 && dtype != ASRBACK_F32)
    return fail(ASRBACK_ERR_ARGUMENT, "dtype must be ASRBACK_BF16 or ASRBACK_F32, got %d", dtype);
  if (batch < 1 || tokens < 1 || batch > 65535)
    return fail(ASRBACK_ERR_ARGUMENT, "batch (%d) and tokens (%d) must be positive", batch, tokens);
  if (width < kHeadDim || width % 128 != 0)
    return fail(ASRBACK_ERR_ARGUMENT, "width must be a positive multiple of 128, got %d", width);
  if (!x || !k_weight || !v_weight || !keys || !values)
    return fail(ASRBACK_ERR_ARGUMENT, "null tensor pointer");
  if (x_stride_token < width || x_stride_batch < (int64_t)tokens * x_stride_token ||
      w_stride < width)
    return fail(ASRBACK_ERR_ARGUMENT, "x must be (batch, tokens, width) rows, weights (width, width)");
  if (c_stride_token < kHeadDim || c_stride_head < (int64_t)tokens * c_stride_token ||
      c_stride_batch < (int64_t)(width / kHeadDim) * c_stride_head)
    return fail(ASRBACK_ERR_ARGUMENT,
                "the caches must be (batch, heads, length >= tokens, 64) views with contiguous rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProjParams p{};
  p.out_k = keys;
  p.out_v = values;
  p.o_sb = c_stride_batch;
  p.o_sh = c_stride_head;
  p.o_st = c_stride_token;
  p.batch = batch;
  p.tokens = tokens;
  p.width = width;
  p.status = status;
  if (dtype == ASRBACK_BF16) {
    if (!aligned16(x) || !aligned16(k_weight) || !aligned16(v_weight) || !aligned16(keys) ||
        !aligned16(values) || x_stride_token % 8 || x_stride_batch % 8 || w_stride % 8 ||
        c_stride_token % 8 || c_stride_head % 8 || c_stride_batch % 8)
      return fail(ASRBACK_ERR_ARGUMENT, "bf16 tensors and strides must be 16-byte aligned");
    p.bias_v = static_cast<const __nv_bfloat16*>(v_bias);
    const int rc = width % 256 == 0
                       ? launch_tc<256>(batch, tokens, width, x, x_stride_batch, x_stride_token,
                                        k_weight, v_weight, w_stride, p, s)
                       : launch_tc<128>(batch, tokens, width, x, x_stride_batch, x_stride_token,
                                        k_weight, v_weight, w_stride, p, s);
    return rc ? rc : ok();
  }
  dim3 grid((tokens + kSimtTile - 1) / kSimtTile, 2 * (width / kHeadDim), batch);
  if (int rc = launch_pdl(cross_kv_projection_simt, grid, dim3(256), 0, s,
                          "cross kv projection (f32) launch", static_cast<const float*>(x),
                          x_stride_batch, x_stride_token, static_cast<const float*>(k_weight),
                          static_cast<const float*>(v_weight), w_stride,
                          static_cast<const float*>(v_bias), p))
    return rc;
  return ok();
}
