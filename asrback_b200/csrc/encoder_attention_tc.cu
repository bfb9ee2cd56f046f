// Whisper encoder self-attention (non-causal, head_dim 64, bf16) on the
// 5th-generation tensor cores: tcgen05.mma with accumulators in tensor memory.
//
// Replaces F.scaled_dot_product_attention in MultiHeadAttention.forward
// (whisper.py:108-110, via attend :102-104) for the encoder layers.
//
// One CTA owns one (window b, head h) and two 128-row query tiles. Warp roles:
//   warp 0      TMA producer: both Q tiles once, then K/V tiles of 128 keys
//               into a STAGES-deep ring (4-D tensor maps over the projections'
//               (batch, length, heads, 64) layout, 128-byte swizzle; rows past
//               the window read as zeros);
//   warp 1      allocates the 512 TMEM columns; one lane issues every MMA:
//               S_t = Q_t K^T (SS: both operands from shared memory) and
//               O_t += P_t V (TS: P from TMEM, V from shared memory);
//   warps 4-7   softmax of query tile 0 (thread = TMEM lane = query row);
//   warps 8-11  softmax of query tile 1.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384)
//               P0 [384,448) P1 [448,512) (P as packed bf16 pairs).
// The two softmax groups ping-pong: while one turns S into P, the tensor core
// computes the other's S or P V. The running max is rescaled lazily: P uses a
// stale max m until a tile's max exceeds it by more than 8 (log2 units), and
// only then are O (in TMEM) and the row sum rescaled, so P stays <= 2^8.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace asrback {

namespace {

constexpr int kRows = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKeys = 128;  // keys per tile
constexpr int kDim = 64;
constexpr int kStages = 4;
constexpr int kTileBytes = kRows * kDim * 2;  // 16 KB, one Q, K or V tile
constexpr int kThreads = 12 * 32;
constexpr int kTmemCols = 512;
// TMEM column of S, O and P for query tile t.
__host__ __device__ constexpr int col_s(int t) { return 128 * t; }
__host__ __device__ constexpr int col_o(int t) { return 256 + 64 * t; }
__host__ __device__ constexpr int col_p(int t) { return 384 + 64 * t; }
// Lazy rescale threshold (log2 units): P <= 2^8 between rescales.
constexpr float kRescaleThreshold = 8.0f;

constexpr int kOffQ = 0;
constexpr int kOffK = 2 * kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffBar = kOffV + kStages * kTileBytes;
// barriers: q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], o_full[2]
constexpr int kNumBars = 1 + 3 * kStages + 6;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack

struct TcParams {
  void* out;
  int64_t sb, sh, ss;  // output strides (elements)
  int length;
  int q_pairs;
  float scale_log2;
  int32_t* status;
};

// ---- PTX wrappers (tcgen05, TMA tensor loads) ----

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(slot)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T (both K-major or as the descriptors say).
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem].
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05 op this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (tcgen05 format:
// start >> 4 at [0,14), LBO >> 4 at [16,30), SBO >> 4 at [32,46), version 1
// at [46,48), layout type 2 = SWIZZLE_128B at [61,64)).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: D f32, A and B bf16, A K-major, B K-major
// or MN-major, N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__global__ void __launch_bounds__(kThreads, 1)
    encoder_attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                                const __grid_constant__ CUtensorMap map_k,
                                const __grid_constant__ CUtensorMap map_v,
                                const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n_k = (p.length + kKeys - 1) / kKeys;
  const uint64_t deadline = global_timer_ns() + kWaitBudgetNs;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);  // one arrival per softmax warp
      mbar_init(&o_full[t], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool timed_out = false;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&map_q);
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      tma_load_4d(smem + kOffQ, &map_q, 0, h, (2 * pair) * kRows, b, q_full);
      tma_load_4d(smem + kOffQ + kTileBytes, &map_q, 0, h, (2 * pair + 1) * kRows, b, q_full);
      for (int j = 0; j < n_k; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, deadline)) {
          timed_out = true;
          break;
        }
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_4d(smem + kOffK + s * kTileBytes, &map_k, 0, h, j * kKeys, b, &k_full[s]);
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_4d(smem + kOffV + s * kTileBytes, &map_v, 0, h, j * kKeys, b, &v_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdescQK = idesc_bf16(kRows, kKeys, false);
      constexpr uint32_t kIdescPV = idesc_bf16(kRows, kDim, true);
      const uint32_t q_addr = smem_addr(smem + kOffQ);
      const uint32_t k_addr = smem_addr(smem + kOffK);
      const uint32_t v_addr = smem_addr(smem + kOffV);
      auto issue_qk = [&](int t, int s) {
        // K = 64 in four steps of 16 elements (32 bytes inside the swizzled row).
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k) {
          const uint64_t a = sw128_desc(q_addr + t * kTileBytes + k * 32, 16, 1024);
          const uint64_t bd = sw128_desc(k_addr + s * kTileBytes + k * 32, 16, 1024);
          mma_ss(tmem + col_s(t), a, bd, kIdescQK, k > 0);
        }
      };
      auto issue_pv = [&](int t, int s, bool accumulate) {
        // K = 128 keys in eight steps of 16: P advances 8 TMEM columns (bf16
        // pairs), V two 8-row swizzle atoms (2048 bytes).
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          const uint64_t bd = sw128_desc(v_addr + s * kTileBytes + k * 2048, kTileBytes, 1024);
          mma_ts(tmem + col_o(t), tmem + col_p(t) + k * 8, bd, kIdescPV, (accumulate || k > 0));
        }
      };
      bool ok = mbar_wait(q_full, 0, deadline);
      for (int j = 0; j < n_k && ok; ++j) {
        const int s = j % kStages;
        ok = mbar_wait(&k_full[s], (j / kStages) & 1, deadline);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t) {
          if (j > 0) {
            ok = mbar_wait(&p_full[t], (j - 1) & 1, deadline);
            if (!ok) break;
            tc_fence_after();
          }
          issue_qk(t, s);
          mma_commit(&s_full[t]);
          if (j > 0) {
            const int sp = (j - 1) % kStages;
            if (t == 0) {
              ok = mbar_wait(&v_full[sp], ((j - 1) / kStages) & 1, deadline);
              if (!ok) break;
            }
            issue_pv(t, sp, j - 1 > 0);
            mma_commit(&o_full[t]);
          }
        }
        if (ok && j > 0 && (j - 1) + kStages < n_k) mma_commit(&kv_empty[(j - 1) % kStages]);
      }
      if (ok) {
        const int sp = (n_k - 1) % kStages;
        ok = mbar_wait(&v_full[sp], ((n_k - 1) / kStages) & 1, deadline);
        for (int t = 0; t < 2 && ok; ++t) {
          ok = mbar_wait(&p_full[t], (n_k - 1) & 1, deadline);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, sp, n_k - 1 > 0);
          mma_commit(&o_full[t]);
        }
      }
      timed_out = !ok;
    }
  } else if (warp >= 4) {
    // ---------------- softmax (one query row per thread) ----------------
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_bits + col_s(t);
    const uint32_t tO = tmem + lane_bits + col_o(t);
    const uint32_t tP = tmem + lane_bits + col_p(t);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_k && ok; ++j) {
      ok = mbar_wait(&s_full[t], j & 1, deadline);
      if (!ok) break;
      tc_fence_after();
      const int valid = min(kKeys, p.length - j * kKeys);
      float v[32];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tS + 32 * c, v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (32 * c + i < valid) mx = fmaxf(mx, v[i]);
      }
      const float m_tile = mx * p.scale_log2;
      bool o_ready = j == 0;  // P/O of the previous tile no longer in use
      if (m_tile > m_used + kRescaleThreshold) {
        if (j > 0) {
          ok = mbar_wait(&o_full[t], (j - 1) & 1, deadline);
          if (!ok) break;
          tc_fence_after();
          o_ready = true;
          const float alpha = fast_exp2(m_used - m_tile);
          float o[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32(tO + 32 * c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + 32 * c, o);
          }
          tmem_wait_st();
          l *= alpha;
        }
        m_used = m_tile;
      }
      if (!o_ready) {
        ok = mbar_wait(&o_full[t], (j - 1) & 1, deadline);
        if (!ok) break;
        tc_fence_after();
      }
      const float neg_m = -m_used;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tS + 32 * c, v);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int col = 32 * c + 2 * i;
          const float p0 = col < valid ? fast_exp2(fmaf(v[2 * i], p.scale_log2, neg_m)) : 0.f;
          const float p1 = col + 1 < valid ? fast_exp2(fmaf(v[2 * i + 1], p.scale_log2, neg_m)) : 0.f;
          const __nv_bfloat162 pair2 = __floats2bfloat162_rn(p0, p1);
          l += p0 + p1;
          packed[i] = *reinterpret_cast<const uint32_t*>(&pair2);
        }
        tmem_st16(tP + 16 * c, packed);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok) ok = mbar_wait(&o_full[t], (n_k - 1) & 1, deadline);
    timed_out = !ok;
    if (ok) {
      tc_fence_after();
      const int row = (2 * pair + t) * kRows + row_in_tile;
      const float inv = 1.f / l;
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + b * p.sb + h * p.sh +
                           static_cast<int64_t>(row) * p.ss;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(tO + 32 * c, o);
        if (row < p.length) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u;
            uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              __nv_bfloat162 h2 = __floats2bfloat162_rn(o[i + 2 * k] * inv, o[i + 2 * k + 1] * inv);
              w[k] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(out + 32 * c + i) = u;
          }
        }
      }
    }
  }
  if (timed_out && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- host side ----

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder(int* rc) {
  static std::mutex lock;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> guard(lock);
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult query;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &query);
    if (err != cudaSuccess || query != cudaDriverEntryPointSuccess || ptr == nullptr) {
      *rc = fail(ASRBACK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
      return nullptr;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// (batch, length, heads, 64) bf16 view with the given element strides as a
// 4-D tensor map {d, head, position, batch}; 64 x 1 x 128 x 1 boxes, 128-byte
// swizzle, zero fill past the window.
int make_map(CUtensorMap* map, const void* base, int batch, int heads, int length, int64_t sb,
             int64_t sh, int64_t ss) {
  int rc = ASRBACK_OK;
  auto encode = tensor_map_encoder(&rc);
  if (!encode) return rc;
  cuuint64_t dims[4] = {(cuuint64_t)kDim, (cuuint64_t)heads, (cuuint64_t)length, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)ss * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {kDim, 1, kRows, 1};
  cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                        strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(ASRBACK_ERR_ARGUMENT,
                "cuTensorMapEncodeTiled rejected the layout (error %d): strides (%lld, %lld, %lld)",
                (int)res, (long long)sb, (long long)sh, (long long)ss);
  return ASRBACK_OK;
}

}  // namespace

// Launches the tensor-core encoder attention; arguments already validated
// (bf16, head_dim 64, 16-byte aligned rows and strides).
int encoder_attention_tc(int batch, int heads, int length, const void* q, const void* k,
                         const void* v, void* out, int64_t sb, int64_t sh, int64_t ss, float scale,
                         int32_t* status, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(&mq, q, batch, heads, length, sb, sh, ss)) return rc;
  if (int rc = make_map(&mk, k, batch, heads, length, sb, sh, ss)) return rc;
  if (int rc = make_map(&mv, v, batch, heads, length, sb, sh, ss)) return rc;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(cudaFuncSetAttribute(encoder_attention_tc_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kSmemBytes),
                            "cudaFuncSetAttribute(encoder attention)"))
      return rc;
    prepared_device = device;
  }
  TcParams p{out, sb, sh, ss, length, (length + 2 * kRows - 1) / (2 * kRows),
             scale * 1.4426950408889634f, status};
  dim3 grid(p.q_pairs, heads, batch);
  encoder_attention_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(mq, mk, mv, p);
  return check_cuda(cudaGetLastError(), "encoder attention (tensor core) launch");
}

}  // namespace asrback
