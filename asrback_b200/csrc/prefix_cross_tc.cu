// Whisper prompt-pass cross-attention (bf16, head_dim 64) on the 5th-generation
// tensor cores: the P tokens of a window's prompt pass (language detection,
// P = 1, or the prompt of _prefill) attend over the window's encoder keys.
//
// Replaces the cross-attention call of DecoderLayer.forward's eager branch
// with length == P (whisper.py:239-240 via attend :102-104), as the
// CUDA-core decode kernel's prefix mode does, for P <= 128. There every
// staged key row serves the P queries through shuffle-reduced dot products and
// the launch is bound by that arithmetic; here a (window, head) item is one
// 128-row query tile holding the P tokens (the other rows zero) against the
// window's key tiles, so the scores and P V run on the tensor cores and the
// launch is bound by reading the keys and values once.
//
// The structure follows the encoder kernel with one query tile per item:
//   warp 0      TMA: each item's P query rows (3-D map over the prompt rows)
//               into one of two Q buffers whose other rows stay zero, and the
//               window's K/V tiles of 128 keys into a 4-stage ring that runs on
//               across items (4-D maps over the cache's (window, head,
//               position, 64) layout; rows past the window read as zeros);
//   warp 1      allocates TMEM and issues the MMAs (warp-wide loop, one
//               elected lane): S(J) = Q K(J)^T into S buffer J & 1, then, per
//               key tile J, O (+)= P(J) V(J) and S(J + 2) into the buffer that
//               P(J) V has read (the tensor core runs one thread's MMAs in
//               order), so S(J + 1) is computed while the softmax of J runs;
//   warps 4-7   softmax and output of query rows 32q .. 32q + 31 (thread =
//               TMEM lane = row); only the ceil(P / 32) warps that hold prompt
//               rows run, and the barriers they feed count them alone.
// Key tiles are numbered J over all of a CTA's items. TMEM: S buffers [0,128)
// and [128,256) (P written over their first 64 columns), O [256,320).
// The running max is rescaled lazily (by more than 8 in log2 units, once the
// previous P V is done), as in the encoder kernel.
#include "tcgen05.cuh"

namespace asrback {

namespace {

using namespace tc;

constexpr int kRows = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKeys = 128;  // keys per tile
constexpr int kDim = 64;
constexpr int kStages = 4;
constexpr int kTileBytes = kRows * kDim * 2;  // 16 KB: a Q, K or V tile
constexpr int kThreads = 8 * 32;              // warps 0-3 control (2, 3 idle), 4-7 softmax
constexpr int kTmemCols = 512;                // 320 used; allocations are powers of two
constexpr int kColO = 256;
constexpr float kRescaleThreshold = 8.0f;

constexpr int kOffQ = 0;  // two Q buffers
constexpr int kOffK = 2 * kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
// Small-prompt softmax staging: [16][128] float scores, [16][64] bf16 pairs.
constexpr int kOffStage = kOffV + kStages * kTileBytes;
constexpr int kOffBar = kOffStage + 16 * kKeys * 4 + 16 * (kKeys / 2) * 4;
// barriers: q_full[2], q_empty[2], kv_full[S], kv_empty[S], s_full[2],
// p_full[2], o_full, o_final, o_free
constexpr int kNumBars = 2 + 2 + 2 * kStages + 2 + 2 + 3;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack

struct PrefixParams {
  void* out;
  int64_t o_st, o_sh;  // output strides (elements): prompt row, head
  int tokens;          // P, the prompt rows per window (1..128)
  int length;          // keys per window
  int heads;
  int items;           // windows * heads
  int softmax_warps;   // ceil(P / 32)
  float scale_log2;
  int32_t* status;
};

// kPad > 0: prompts of at most kPad (a power of two up to 16) rows, whose
// softmax shares each row's work out over 32 / kPad lanes; 0: a row per lane.
template <int kPad>
__global__ void __launch_bounds__(kThreads, 1)
    prefix_cross_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                           const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v,
                           const __grid_constant__ PrefixParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;  // [Q buffer]
  uint64_t* q_empty = q_full + 2;
  uint64_t* kv_full = q_empty + 2;  // K and V of a ring slot
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [S buffer]
  uint64_t* p_full = s_full + 2;          // [S buffer]
  uint64_t* o_full = p_full + 2;
  uint64_t* o_final = o_full + 1;
  uint64_t* o_free = o_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_k = (p.length + kKeys - 1) / kKeys;
  const int n_items = p.items > (int)blockIdx.x
                          ? (p.items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                          : 0;
  const int total = n_items * n_k;
  auto item_index = [&](int li) { return (int)blockIdx.x + li * (int)gridDim.x; };

  // The Q buffers' rows past the prompt stay zero: TMA writes rows < P only.
  for (int i = threadIdx.x; i < 2 * kTileBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem + kOffQ)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async();  // the generic-proxy zeros before the tensor core's reads
  if (threadIdx.x == 0) {
    for (int q = 0; q < 2; ++q) {
      mbar_init(&q_full[q], 1);
      mbar_init(&q_empty[q], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], p.softmax_warps);  // one arrival per running softmax warp
    }
    mbar_init(o_full, 1);
    mbar_init(o_final, 1);
    mbar_init(o_free, p.softmax_warps);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  bool timed_out = false;

  auto wait_warp = [](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
  };
  // One lane per warp, elected once: a tcgen05.commit tracks the MMAs of its
  // own thread, so the MMA warp's issues and commits all come from it.
  const bool leader = elect_one();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (leader) {
      prefetch_tensormap(&map_q);
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
    }
    __syncwarp();
    bool ok = true;
    int g = 0;  // key tiles loaded (= J)
    for (int li = 0; li < n_items && ok; ++li) {
      const int index = item_index(li);
      const int h = index % p.heads, w = index / p.heads;
      const int qb = li & 1;
      if (li >= 2) ok = wait_warp(&q_empty[qb], ((li >> 1) - 1) & 1);
      if (!ok) break;
      if (leader) {
        mbar_arrive_expect_tx(&q_full[qb], static_cast<uint32_t>(p.tokens * kDim * 2));
        tma_load_3d(smem + kOffQ + qb * kTileBytes, &map_q, 0, h, w * p.tokens, &q_full[qb]);
      }
      __syncwarp();
      for (int j = 0; j < n_k; ++j, ++g) {
        const int s = g % kStages;
        if (g >= kStages) ok = wait_warp(&kv_empty[s], ((g / kStages) - 1) & 1);
        if (!ok) break;
        if (leader) {
          mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
          tma_load_4d(smem + kOffK + s * kTileBytes, &map_k, 0, h, j * kKeys, w, &kv_full[s]);
          tma_load_4d(smem + kOffV + s * kTileBytes, &map_v, 0, h, j * kKeys, w, &kv_full[s]);
        }
        __syncwarp();
      }
    }
    timed_out = !ok;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (total > 0) {
      constexpr uint32_t kIdescQK = idesc_bf16(kRows, kKeys, false);
      constexpr uint32_t kIdescPV = idesc_bf16(kRows, kDim, true);
      const uint64_t q_desc = sw128_desc(smem_addr(smem + kOffQ), 16, 1024);
      const uint64_t k_desc = sw128_desc(smem_addr(smem + kOffK), 16, 1024);
      const uint64_t v_desc = sw128_desc(smem_addr(smem + kOffV), kTileBytes, 1024);
      constexpr uint64_t kStepK = 32 >> 4, kStepV = 2048 >> 4, kTile = kTileBytes >> 4;
      bool ok = true;
      // Key tile X's position: item li (Q buffer li & 1), tile j in it, ring
      // slot s and lap; stepped without branches.
      struct Pos {
        int li, j, s, lap;
      };
      auto advance = [&](Pos c) {
        c.j = c.j + 1 == n_k ? 0 : c.j + 1;
        c.li += c.j == 0 ? 1 : 0;
        c.s = c.s + 1 == kStages ? 0 : c.s + 1;
        c.lap += c.s == 0 ? 1 : 0;
        return c;
      };
      // S(X) into buffer `buf`: waits for the K/V tile (one barrier for both;
      // P V of the tile comes later in this stream) and, first of an item, for
      // its Q. After the item's last S the Q buffer is free.
      auto qk = [&](const Pos& c, int buf) {
        const int qb = c.li & 1;
        if (c.j == 0) ok = ok && wait_warp(&q_full[qb], (c.li >> 1) & 1);
        ok = ok && wait_warp(&kv_full[c.s], c.lap & 1);
        if (!ok) return;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int k = 0; k < kDim / 16; ++k)
            mma_ss(tmem + 128 * buf, q_desc + qb * kTile + k * kStepK,
                   k_desc + c.s * kTile + k * kStepK, kIdescQK, k > 0);
          mma_commit(&s_full[buf]);
          if (c.j == n_k - 1) mma_commit(&q_empty[qb]);
        }
        __syncwarp();
      };
      Pos c0{0, 0, 0, 0};
      Pos c2 = advance(advance(c0));
      qk(c0, 0);
      if (total > 1) qk(advance(c0), 1);
      for (int J = 0; J < total && ok; ++J) {
        const int buf = J & 1;
        // O (+)= P(J) V(J) once the softmax has written P(J) (an item's first
        // also once the previous item's output has been read out of O).
        ok = ok && wait_warp(&p_full[buf], (J >> 1) & 1);
        if (c0.j == 0 && c0.li > 0) ok = ok && wait_warp(o_free, (c0.li - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int k = 0; k < kKeys / 16; ++k)
            mma_ts(tmem + kColO, tmem + 128 * buf + k * 8, v_desc + c0.s * kTile + k * kStepV,
                   kIdescPV, (c0.j > 0 || k > 0));
          mma_commit(c0.j + 1 < n_k ? o_full : o_final);
          if (J + kStages < total) mma_commit(&kv_empty[c0.s]);
        }
        __syncwarp();
        if (J + 2 < total) qk(c2, buf);
        c0 = advance(c0);
        c2 = advance(c2);
      }
      timed_out = !ok;
    }
  } else if (warp >= 4 && warp - 4 < p.softmax_warps) {
    // ---------------- softmax and output (one query row per thread) ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // prompt row of this thread (zeros past P)
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_bits + kColO;
    float* s_rows = reinterpret_cast<float*>(smem + kOffStage);  // [kPad][128] scores
    uint32_t* p_rows = reinterpret_cast<uint32_t*>(smem + kOffStage + 16 * kKeys * 4);
    bool ok = true;
    for (int li = 0; li < n_items && ok; ++li) {
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n_k && ok; ++j) {
        const int J = li * n_k + j;
        const int buf = J & 1;
        const uint32_t tS = tmem + lane_bits + 128 * buf;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[buf], (J >> 1) & 1));
        if (!ok) break;
        tc_fence_after();
        const int valid = min(kKeys, p.length - j * kKeys);
        float v[kKeys];
        tmem_ld128(tS, v);
        if constexpr (kPad > 0) {
          // Small prompt: each row's 128 scores go through shared memory to
          // its G lanes, C columns each, so the exponentials are shared out.
          // Row r is held by lanes r * G .. r * G + G - 1 (its max, sum and
          // running state replicated in them); lane t < kPad holds TMEM row t.
          constexpr int G = 32 / kPad, C = kKeys / G;
          const int r = lane / G, part = lane % G;
          if (lane < kPad) {
#pragma unroll
            for (int i = 0; i < kKeys; i += 4)
              *reinterpret_cast<float4*>(s_rows + lane * kKeys + i) =
                  make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          }
          __syncwarp();
          float x[C];
#pragma unroll
          for (int i = 0; i < C; i += 4) {
            const float4 f = *reinterpret_cast<const float4*>(s_rows + r * kKeys + part * C + i);
            x[i] = part * C + i < valid ? f.x : -INFINITY;
            x[i + 1] = part * C + i + 1 < valid ? f.y : -INFINITY;
            x[i + 2] = part * C + i + 2 < valid ? f.z : -INFINITY;
            x[i + 3] = part * C + i + 3 < valid ? f.w : -INFINITY;
          }
          float mx = x[0];
#pragma unroll
          for (int i = 1; i < C; ++i) mx = fmaxf(mx, x[i]);
#pragma unroll
          for (int off = G / 2; off >= 1; off >>= 1)
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          const float m_tile = mx * p.scale_log2;
          const bool move = m_tile > m_used + kRescaleThreshold;
          if (__any_sync(0xffffffffu, move)) {
            const float m_new = move ? m_tile : m_used;
            if (j > 0) {
              ok = __all_sync(0xffffffffu,
                              mbar_wait_bounded(o_full, (li * (n_k - 1) + j - 1) & 1));
              if (!ok) break;
              tc_fence_after();
              const float alpha_row = move ? fast_exp2(m_used - m_new) : 1.f;
              // TMEM row t's factor, from the first lane of row t's group.
              const float a = __shfl_sync(0xffffffffu, alpha_row, lane < kPad ? lane * G : lane);
              const float alpha = lane < kPad ? a : 1.f;
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                float o[16];
                tmem_ld16(tO + 16 * c, o);
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= alpha;
                tmem_st16f(tO + 16 * c, o);
              }
              tmem_wait_st();
              l *= alpha_row;
            }
            m_used = m_new;
          }
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < C; i += 2) {
            const float p0 = fast_exp2(fmaf(x[i], p.scale_log2, -m_used));
            const float p1 = fast_exp2(fmaf(x[i + 1], p.scale_log2, -m_used));
            sum += p0 + p1;
            p_rows[r * (kKeys / 2) + (part * C + i) / 2] = bf16x2(p0, p1);
          }
#pragma unroll
          for (int off = G / 2; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
          l += sum;
          __syncwarp();
          // TMEM row t takes row t's P (rows past kPad: zeros).
          uint32_t packed[32];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const uint4 u = lane < kPad ? *reinterpret_cast<const uint4*>(
                                                p_rows + lane * (kKeys / 2) + 32 * half + i)
                                          : make_uint4(0u, 0u, 0u, 0u);
              packed[i] = u.x;
              packed[i + 1] = u.y;
              packed[i + 2] = u.z;
              packed[i + 3] = u.w;
            }
            tmem_st32u(tS + 32 * half, packed);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[buf]);
        } else {
          if (valid < kKeys) {
  #pragma unroll
            for (int i = 0; i < kKeys; ++i)
              if (i >= valid) v[i] = -INFINITY;
          }
          float acc[8];
  #pragma unroll
          for (int a = 0; a < 8; ++a) acc[a] = fmaxf(v[a], v[8 + a]);
  #pragma unroll
          for (int i = 16; i < kKeys; i += 16)
  #pragma unroll
            for (int a = 0; a < 8; ++a) acc[a] = fmax3(acc[a], v[i + a], v[i + 8 + a]);
          const float mx = fmaxf(fmax3(acc[0], acc[1], acc[2]),
                                 fmax3(fmax3(acc[3], acc[4], acc[5]), acc[6], acc[7]));
          const float m_tile = mx * p.scale_log2;
          const bool move = m_tile > m_used + kRescaleThreshold;
          if (__any_sync(0xffffffffu, move)) {
            const float m_new = move ? m_tile : m_used;
            if (j > 0) {
              // O must be idle: P(J-1) V done (the S just read was issued after
              // P(J-2) V, not after P(J-1) V).
              ok = __all_sync(0xffffffffu, mbar_wait_bounded(o_full, (li * (n_k - 1) + j - 1) & 1));
              if (!ok) break;
              tc_fence_after();
              const float alpha = move ? fast_exp2(m_used - m_new) : 1.f;
  #pragma unroll
              for (int c = 0; c < 4; ++c) {
                float o[16];
                tmem_ld16(tO + 16 * c, o);
  #pragma unroll
                for (int i = 0; i < 16; ++i) o[i] *= alpha;
                tmem_st16f(tO + 16 * c, o);
              }
              tmem_wait_st();
              l *= alpha;
            }
            m_used = m_new;
          }
          const uint64_t scale2 = pack2(p.scale_log2, p.scale_log2);
          const uint64_t neg_m2 = pack2(-m_used, -m_used);
          uint64_t sum2[4];
  #pragma unroll
          for (int a = 0; a < 4; ++a) sum2[a] = pack2(0.f, 0.f);
  #pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t packed[32];
  #pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = 64 * half + 2 * i;
              float x0, x1;
              unpack2(ffma2(pack2(v[col], v[col + 1]), scale2, neg_m2), x0, x1);
              const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
              sum2[i & 3] = fadd2(sum2[i & 3], pack2(p0, p1));
              packed[i] = bf16x2(p0, p1);
            }
            tmem_st32u(tS + 32 * half, packed);
          }
          float lo0, hi0;
          unpack2(fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3])), lo0, hi0);
          l += lo0 + hi0;
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[buf]);
        }
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(o_final, li & 1));
      if (!ok) break;
      tc_fence_after();
      const int index = item_index(li);
      const int h = index % p.heads, w = index / p.heads;
      // Small prompt: row t's sum is held by the lanes of its group.
      const float l_row =
          kPad > 0 ? __shfl_sync(0xffffffffu, l, lane < kPad ? lane * (32 / (kPad > 0 ? kPad : 1))
                                                              : lane)
                   : l;
      const float inv = 1.f / l_row;
      const int64_t off = row < p.tokens ? static_cast<int64_t>(w * p.tokens + row) * p.o_st +
                                               static_cast<int64_t>(h) * p.o_sh
                                         : 0;
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + off;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(tO + 32 * c, o);
        if (row < p.tokens) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u;
            u.x = bf16x2(o[i] * inv, o[i + 1] * inv);
            u.y = bf16x2(o[i + 2] * inv, o[i + 3] * inv);
            u.z = bf16x2(o[i + 4] * inv, o[i + 5] * inv);
            u.w = bf16x2(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4*>(out + 32 * c + i) = u;
          }
        }
      }
      // O has been read: the next item's first P V may overwrite it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
    }
    timed_out = !ok;
  }
  if (timed_out && p.status && lane == 0) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- host side ----

// The prompt rows as a 3-D map {d, head, row} (row = window * P + token), box
// 64 x 1 x P; the cache as a 4-D map {d, head, position, window}, box
// 64 x 1 x 128 x 1. 128-byte swizzle; reads past an extent are zeros.
int make_maps(CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv, const void* q, int rows,
              int heads, int tokens, int64_t q_st, int64_t q_sh, const void* k, const void* v,
              int windows, int length, int64_t c_sb, int64_t c_sh) {
  int rc = ASRBACK_OK;
  auto encode = tensor_map_encoder(&rc);
  if (!encode) return rc;
  const cuuint32_t ones[4] = {1, 1, 1, 1};
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)heads, (cuuint64_t)rows};
    cuuint64_t strides[2] = {(cuuint64_t)q_sh * 2, (cuuint64_t)q_st * 2};
    cuuint32_t box[3] = {kDim, 1, (cuuint32_t)tokens};
    CUresult res = encode(mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims,
                          strides, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (res != CUDA_SUCCESS)
      return fail(ASRBACK_ERR_ARGUMENT,
                  "cuTensorMapEncodeTiled rejected the prompt rows (error %d): strides (%lld, %lld)",
                  (int)res, (long long)q_st, (long long)q_sh);
  }
  cuuint64_t dims[4] = {(cuuint64_t)kDim, (cuuint64_t)heads, (cuuint64_t)length,
                        (cuuint64_t)windows};
  cuuint64_t strides[3] = {(cuuint64_t)c_sh * 2, (cuuint64_t)kDim * 2, (cuuint64_t)c_sb * 2};
  cuuint32_t box[4] = {kDim, 1, kKeys, 1};
  for (CUtensorMap* m : {mk, mv}) {
    const void* base = m == mk ? k : v;
    CUresult res = encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                          strides, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (res != CUDA_SUCCESS)
      return fail(ASRBACK_ERR_ARGUMENT,
                  "cuTensorMapEncodeTiled rejected the cache (error %d): strides (%lld, %lld)",
                  (int)res, (long long)c_sb, (long long)c_sh);
  }
  return ASRBACK_OK;
}

template <int kPad>
int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
           const PrefixParams& p, cudaStream_t stream) {
  auto kernel = prefix_cross_tc_kernel<kPad>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
            "cudaFuncSetAttribute(prompt-pass cross attention)"))
      return rc;
    prepared_device = device;
  }
  // Persistent: one CTA per SM (512 TMEM columns each), at most one per item.
  const int ctas = p.items < sm_count() ? p.items : sm_count();
  return launch_pdl(kernel, dim3(ctas), dim3(kThreads), kSmemBytes, stream,
                    "prompt-pass cross attention (tensor core) launch", mq, mk, mv, p);
}

}  // namespace

// Launches the tensor-core prompt-pass cross-attention; arguments already
// validated by the caller (bf16, head_dim 64, 16-byte aligned pointers and
// strides, 1 <= tokens <= 128).
int whisper_cross_prefix_tc(int windows, int tokens, int heads, int length, const void* q,
                            int64_t q_st, int64_t q_sh, const void* k, const void* v,
                            int64_t c_sb, int64_t c_sh, void* out, int64_t o_st, int64_t o_sh,
                            float scale, int32_t* status, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  if (int rc = make_maps(&mq, &mk, &mv, q, windows * tokens, heads, tokens, q_st, q_sh, k, v,
                         windows, length, c_sb, c_sh))
    return rc;
  PrefixParams p{out,     o_st,  o_sh, tokens, length, heads, windows * heads,
                 (tokens + 31) / 32, scale * 1.4426950408889634f, status};
  // Prompts of up to 16 rows share each row's softmax out over the warp.
  if (tokens <= 1) return launch<1>(mq, mk, mv, p, stream);
  if (tokens <= 2) return launch<2>(mq, mk, mv, p, stream);
  if (tokens <= 4) return launch<4>(mq, mk, mv, p, stream);
  if (tokens <= 8) return launch<8>(mq, mk, mv, p, stream);
  if (tokens <= 16) return launch<16>(mq, mk, mv, p, stream);
  return launch<0>(mq, mk, mv, p, stream);
}

}  // namespace asrback
