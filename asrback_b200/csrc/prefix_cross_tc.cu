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
// Two items run at once, one per slot x = 0, 1 (a CTA's items 2i and 2i + 1;
// with an odd count the last runs alone), each slot with its own Q buffer, S
// buffer, O accumulator and softmax warps, so that one slot's softmax runs
// while the other's is waiting for its scores. Roles:
//   warp 0      TMA: each item's P query rows (3-D map over the prompt rows)
//               into its slot's Q buffer, whose other rows stay zero, and the
//               pair's K/V tiles of 128 keys, the two slots' tiles alternating,
//               into a 5-stage ring (4-D maps over the cache's (window, head,
//               position, 64) layout; rows past the window read as zeros);
//   warp 1      allocates TMEM and issues the MMAs (warp-wide loop, one
//               elected lane), in the ring's order: per key tile of a slot,
//               O_x (+)= P_x V then that slot's next S_x = Q_x K^T into the
//               buffer P_x V has read (the tensor core runs one thread's MMAs
//               in order);
//   warps 4-7   softmax and output of slot 0, warps 8-11 of slot 1: query rows
//               32q .. 32q + 31 (thread = TMEM lane = row); only the
//               ceil(P / 32) warps of a slot that hold prompt rows run, and the
//               barriers they feed count them alone; prompts of up to 8 rows
//               share each row out over four lanes (16-lane TMEM loads and
//               stores). For prompts of up to 64 rows slot 1's rows start at
//               row 32 or 64 of its tile, so that the two slots' softmax warps
//               run on different sub-partitions.
// Split items (up to 64 rows over an even number of key tiles): the two slots
// run the two halves of one item's keys (its rows in one Q buffer twice, the
// two Q buffers alternating by item), and the warps of each warpgroup on the
// other slot's lane quarters (idle otherwise: warps 8.. for slot 0, 4 + s..
// for slot 1, s = the softmax warps per slot) take the epilogue: slot 1's half
// goes through shared memory to slot 0's epilogue warps, which merge it with
// slot 0's and write the output, while the softmax warps run the next item
// into the slot's other O buffer.
// TMEM: slot x's S at [256x, 256x + 128) (P written over its first 64
// columns), its O at [256x + 128, 256x + 192) and, for split items of odd
// pair index, [256x + 192, 256x + 256).
// The running max is rescaled lazily (by more than 8 in log2 units, once the
// previous P V is done), as in the encoder kernel.
#include "tcgen05.cuh"

namespace asrback {

namespace {

using namespace tc;

constexpr int kRows = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKeys = 128;  // keys per tile
constexpr int kDim = 64;
constexpr int kStages = 5;
constexpr int kTileBytes = kRows * kDim * 2;  // 16 KB: a Q, K or V tile
constexpr int kThreads = 12 * 32;  // warps 0-3 control (2, 3 idle), 4-11 softmax and epilogue
constexpr int kTmemCols = 512;     // per slot: S 128 + two O buffers of 64
__host__ __device__ constexpr int col_s(int x) { return 256 * x; }
__host__ __device__ constexpr int col_o(int x) { return 256 * x + 128; }  // + 64: split's 2nd
constexpr float kRescaleThreshold = 8.0f;
// Registers per thread: 168 at launch (384 x 168 = 64512); the control
// warpgroup keeps 56, the two softmax warpgroups take 224.
constexpr int kLaunchRegs = 168;
constexpr int kControlRegs = 56;
constexpr int kSoftmaxRegs = 224;
static_assert(128 * kControlRegs + 256 * kSoftmaxRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch's register pool");

constexpr int kOffQ = 0;  // two Q buffers: one per slot, or (split items) per item parity
constexpr int kOffK = 2 * kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
// Split items (prompts of up to kSplitRows rows): slot 1 hands its half's
// output rows (unnormalised O, rows padded to 68 floats so that eight rows'
// 16-byte stores hit distinct banks) and each row's (max, sum) to slot 0.
constexpr int kSplitRows = 64;
constexpr int kXchStride = 68;
constexpr int kOffXchO = kOffV + kStages * kTileBytes;
constexpr int kOffXchML = kOffXchO + kSplitRows * kXchStride * 4;
// Split items: each slot's softmax hands its rows' (max, sum) to the epilogue
// warps, per O buffer: [slot][buffer][kSplitRows] float2.
constexpr int kOffML = kOffXchML + kSplitRows * 8;
constexpr int kOffBar = kOffML + 2 * 2 * kSplitRows * 8;
// barriers: q_full[2], q_empty[2], kv_full[S], kv_empty[S], per slot s_full,
// p_full, o_full, per (slot, O buffer) o_final, o_free, ml_full, ml_empty,
// then xch_full, xch_empty
constexpr int kNumBars = 2 + 2 + 2 * kStages + 3 * 2 + 4 * 4 + 2;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");

struct PrefixParams {
  void* out;
  int64_t o_st, o_sh;  // output strides (elements): prompt row, head
  int tokens;          // P, the prompt rows per window (1..128)
  int length;          // keys per window
  int heads;
  int items;           // windows * heads
  int softmax_warps;   // per slot: ceil(P / 32)
  int row1;            // first query-tile row of slot 1's prompt (0, 32 or 64)
  int split;           // 1: each item's key tiles in two halves, one per slot
  float scale_log2;
  int32_t* status;
};

// kSmall: prompts of at most 8 rows, each row's softmax shared out over four
// lanes; otherwise a row per lane.
template <bool kSmall>
__global__ void __launch_bounds__(kThreads, 1)
    prefix_cross_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                           const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v,
                           const __grid_constant__ PrefixParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;  // [slot]
  uint64_t* q_empty = q_full + 2;
  uint64_t* kv_full = q_empty + 2;  // K and V of a ring slot
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [slot]
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_final = o_full + 2;  // [2 * slot + O buffer]
  uint64_t* o_free = o_final + 4;
  uint64_t* ml_full = o_free + 4;
  uint64_t* ml_empty = ml_full + 4;
  uint64_t* xch_full = ml_empty + 4;
  uint64_t* xch_empty = xch_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.items > (int)blockIdx.x
                          ? (p.items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                          : 0;
  // A unit is an item (window, head) or, split, one half of its key tiles:
  // unit u of this CTA runs in slot u & 1 as part of pair u / 2.
  const int n_tiles = (p.length + kKeys - 1) / kKeys;  // key tiles per item
  const int n_k = p.split ? (n_tiles + 1) / 2 : n_tiles;  // key tiles per unit
  const int n_units = p.split ? 2 * n_items : n_items;
  const int n_pairs = (n_units + 1) / 2;
  const int total = n_units * n_k;  // key tiles over all units
  auto item_index = [&](int u) {
    return (int)blockIdx.x + (p.split ? u >> 1 : u) * (int)gridDim.x;
  };
  // First key tile of unit u (the second half of a split item starts at n_k).
  auto first_tile = [&](int u) { return p.split ? (u & 1) * n_k : 0; };
  // Units of pair i: 2i (slot 0) and 2i + 1 (slot 1, when there is one).
  auto pair_size = [&](int i) { return 2 * i + 1 < n_units ? 2 : 1; };
  // Ring index of key tile j of pair i's slot x: the two slots' tiles alternate.
  auto ring_index = [&](int i, int j, int x) {
    return 2 * n_k * i + (pair_size(i) == 2 ? 2 * j + x : j);
  };

  // The Q buffers' rows past the prompt stay zero: TMA writes rows < P only.
  for (int i = threadIdx.x; i < 2 * kTileBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem + kOffQ)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async();  // the generic-proxy zeros before the tensor core's reads
  if (threadIdx.x == 0) {
    for (int x = 0; x < 2; ++x) {
      mbar_init(&q_full[x], 1);
      mbar_init(&q_empty[x], 1);
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], p.softmax_warps);  // one arrival per running softmax warp
      mbar_init(&o_full[x], 1);
    }
    for (int e = 0; e < 4; ++e) {
      mbar_init(&o_final[e], 1);
      // Split items: the slot's epilogue warps free O (as many as it has
      // softmax warps); otherwise each softmax warp.
      mbar_init(&o_free[e], p.softmax_warps);
      mbar_init(&ml_full[e], p.softmax_warps);
      mbar_init(&ml_empty[e], p.softmax_warps);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(xch_full, p.softmax_warps);
    mbar_init(xch_empty, p.softmax_warps);
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

  // Each warpgroup leaves through its own branch (status, fences, one
  // CTA-wide named barrier, the TMEM release): a register budget is fixed per
  // branch, so the branches never rejoin.
  if (warp < 4) {
    reg_release<kControlRegs>();
    // One lane per warp, elected once: a tcgen05.commit tracks the MMAs of
    // its own thread, so the MMA warp's issues and commits all come from it.
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
      int g = 0;  // key tiles loaded, in ring order
      for (int i = 0; i < n_pairs && ok; ++i) {
        const int ps = pair_size(i);
        if (p.split) {
          // Both slots run the same item: buffer i & 1 takes its rows twice
          // (at row 0 for slot 0, at row1 for slot 1), free once the item
          // two pairs back has issued its last S, long before this pair's
          // keys are due.
          const int b = i & 1;
          if (i >= 2) ok = wait_warp(&q_empty[b], ((i >> 1) - 1) & 1);
          if (!ok) break;
          const int index = item_index(2 * i);
          const int h = index % p.heads, w = index / p.heads;
          if (leader) {
            mbar_arrive_expect_tx(&q_full[b], static_cast<uint32_t>(2 * p.tokens * kDim * 2));
            tma_load_3d(smem + kOffQ + b * kTileBytes, &map_q, 0, h, w * p.tokens, &q_full[b]);
            tma_load_3d(smem + kOffQ + b * kTileBytes + p.row1 * 128, &map_q, 0, h, w * p.tokens,
                        &q_full[b]);
          }
          __syncwarp();
        }
        for (int x = 0; x < ps && ok && !p.split; ++x) {
          // Slot x's Q buffer is free once its previous item has issued its
          // last S.
          if (i >= 1) ok = wait_warp(&q_empty[x], (i - 1) & 1);
          if (!ok) break;
          const int index = item_index(2 * i + x);
          const int h = index % p.heads, w = index / p.heads;
          if (leader) {
            mbar_arrive_expect_tx(&q_full[x], static_cast<uint32_t>(p.tokens * kDim * 2));
            tma_load_3d(smem + kOffQ + x * kTileBytes + x * p.row1 * 128, &map_q, 0, h,
                        w * p.tokens, &q_full[x]);
          }
          __syncwarp();
        }
        for (int j = 0; j < n_k && ok; ++j) {
          for (int x = 0; x < ps; ++x, ++g) {
            const int s = g % kStages;
            if (g >= kStages) ok = wait_warp(&kv_empty[s], ((g / kStages) - 1) & 1);
            if (!ok) break;
            const int index = item_index(2 * i + x);
            const int h = index % p.heads, w = index / p.heads;
            const int key = (first_tile(2 * i + x) + j) * kKeys;
            if (leader) {
              mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
              tma_load_4d(smem + kOffK + s * kTileBytes, &map_k, 0, h, key, w, &kv_full[s]);
              tma_load_4d(smem + kOffV + s * kTileBytes, &map_v, 0, h, key, w, &kv_full[s]);
            }
            __syncwarp();
          }
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
        // S_x of key tile j of pair i: waits for the K/V tile (one barrier
        // for both; the tile's P V comes later in this stream) and, first of an
        // item, for its Q. After the item's last S its Q buffer is free (split:
        // the pair's buffer i & 1 after slot 1's last S; otherwise slot x's).
        auto qk = [&](int i, int j, int x) {
          const int g = ring_index(i, j, x), s = g % kStages;
          const int b = p.split ? i & 1 : x;
          if (j == 0) ok = ok && wait_warp(&q_full[b], (p.split ? i >> 1 : i) & 1);
          ok = ok && wait_warp(&kv_full[s], (g / kStages) & 1);
          if (!ok) return;
          tc_fence_after();
          if (leader) {
#pragma unroll
            for (int k = 0; k < kDim / 16; ++k)
              mma_ss(tmem + col_s(x), q_desc + b * kTile + k * kStepK,
                     k_desc + s * kTile + k * kStepK, kIdescQK, k > 0);
            mma_commit(&s_full[x]);
            if (j == n_k - 1 && (!p.split || x == 1)) mma_commit(&q_empty[b]);
          }
          __syncwarp();
        };
        for (int x = 0; x < pair_size(0); ++x) qk(0, 0, x);
        for (int i = 0; i < n_pairs && ok; ++i) {
          const int ps = pair_size(i);
          for (int j = 0; j < n_k && ok; ++j) {
            for (int x = 0; x < ps && ok; ++x) {
              // O_x (+)= P_x V once the softmax has written P_x (an item's
              // first also once the slot's previous output has been read).
              const int t = i * n_k + j;  // slot x's key tiles so far
              // Split items alternate between the slot's two O buffers, so an
              // item's first P V waits for the epilogue of the item two back.
              const int ob = p.split ? i & 1 : 0;
              ok = ok && wait_warp(&p_full[x], t & 1);
              if (j == 0 && i >= (p.split ? 2 : 1))
                ok = ok && wait_warp(&o_free[2 * x + ob], (p.split ? (i >> 1) - 1 : i - 1) & 1);
              if (!ok) break;
              tc_fence_after();
              const int g = ring_index(i, j, x), s = g % kStages;
              if (leader) {
#pragma unroll
                for (int k = 0; k < kKeys / 16; ++k)
                  mma_ts(tmem + col_o(x) + 64 * ob, tmem + col_s(x) + k * 8,
                         v_desc + s * kTile + k * kStepV, kIdescPV, (j > 0 || k > 0));
                mma_commit(j + 1 < n_k ? &o_full[x] : &o_final[2 * x + ob]);
                if (g + kStages < total) mma_commit(&kv_empty[s]);
              }
              __syncwarp();
              // Slot x's next S, into the buffer this P V has read.
              if (j + 1 < n_k) {
                qk(i, j + 1, x);
              } else if (2 * (i + 1) + x < n_units) {
                qk(i + 1, 0, x);
              }
            }
          }
        }
        timed_out = !ok;
      }
    }
    if (timed_out && p.status && lane == 0) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
    tc_fence_before();
    named_sync(1, kThreads);
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
  } else {
    reg_acquire<kSoftmaxRegs>();
    // ---------------- softmax, epilogue and output ----------------
    const int slot = (warp - 4) >> 2;
    const int quarter = warp & 3;
    // Slot 1's prompt rows start at row1 of its tile (a lane quarter of
    // their own for prompts up to 64 rows, so that the two slots' softmax
    // warps run on different sub-partitions).
    const int q0 = slot * p.row1 / 32;
    bool ok = true;
    float* xch_o = reinterpret_cast<float*>(smem + kOffXchO);
    float2* xch_ml = reinterpret_cast<float2*>(smem + kOffXchML);
    float2* ml = reinterpret_cast<float2*>(smem + kOffML);
    // Split items: a warpgroup's warps on the other slot's row quarters are
    // that slot's epilogue warps (es: the slot a warp finishes; its rows
    // start at erow0).
    const int sw = p.softmax_warps;
    int es = -1, erow0 = 0;
    if (p.split) {
      if (slot == 1 && quarter < sw) {
        es = 0;
        erow0 = quarter * 32;
      } else if (slot == 0 && quarter >= sw && quarter < 2 * sw) {
        es = 1;
        erow0 = (quarter - sw) * 32;
      }
    }
    if (es >= 0) {
      // ---------------- split items: epilogue ----------------
      // Per item: the O buffer once the last P V is done and the softmax has
      // handed over each row's (max, sum). Slot 1's half goes through shared
      // memory to slot 0's epilogue warps, which fold it into slot 0's half
      // and write the output. The softmax warps meanwhile run the next item
      // into the slot's other O buffer.
      const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
      const int row = erow0 + lane;
      const bool live = row < p.tokens;
      for (int it = 0; ok && 2 * it + es < n_units; ++it) {
        const int e = 2 * es + (it & 1);
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&o_final[e], (it >> 1) & 1));
        ok = ok && __all_sync(0xffffffffu, mbar_wait_bounded(&ml_full[e], (it >> 1) & 1));
        if (!ok) break;
        tc_fence_after();
        const float2 mine = live ? ml[kSplitRows * e + row] : make_float2(0.f, 0.f);
        float o[64];
        tmem_ld32(tmem + lane_bits + col_o(es) + 64 * (it & 1), o);
        tmem_ld32(tmem + lane_bits + col_o(es) + 64 * (it & 1) + 32, o + 32);
        if (es == 1) {
          // Second half: rows' unnormalised O and (max, sum) to slot 0's
          // epilogue warps once they have read the previous item's.
          if (it > 0) ok = __all_sync(0xffffffffu, mbar_wait_bounded(xch_empty, (it - 1) & 1));
          if (!ok) break;
          if (live) {
#pragma unroll
            for (int i = 0; i < 64; i += 4)
              *reinterpret_cast<float4*>(xch_o + row * kXchStride + i) =
                  make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
            xch_ml[row] = mine;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(xch_full);
            mbar_arrive(&ml_empty[e]);
            mbar_arrive(&o_free[e]);
          }
          continue;
        }
        // First half: fold the second half's rows in and write the output.
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(xch_full, it & 1));
        if (!ok) break;
        if (live) {
          const float2 other = xch_ml[row];
          const float m = fmaxf(mine.x, other.x);
          const float a0 = fast_exp2(mine.x - m), a1 = fast_exp2(other.x - m);
          const float inv = 1.f / (mine.y * a0 + other.y * a1);
          const float b0 = a0 * inv, b1 = a1 * inv;
          const int index = item_index(2 * it);
          const int h = index % p.heads, w = index / p.heads;
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) +
                               static_cast<int64_t>(w * p.tokens + row) * p.o_st +
                               static_cast<int64_t>(h) * p.o_sh;
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
            const float4 f0 = *reinterpret_cast<const float4*>(xch_o + row * kXchStride + i);
            const float4 f1 = *reinterpret_cast<const float4*>(xch_o + row * kXchStride + i + 4);
            uint4 u;
            u.x = bf16x2(o[i] * b0 + f0.x * b1, o[i + 1] * b0 + f0.y * b1);
            u.y = bf16x2(o[i + 2] * b0 + f0.z * b1, o[i + 3] * b0 + f0.w * b1);
            u.z = bf16x2(o[i + 4] * b0 + f1.x * b1, o[i + 5] * b0 + f1.y * b1);
            u.w = bf16x2(o[i + 6] * b0 + f1.z * b1, o[i + 7] * b0 + f1.w * b1);
            *reinterpret_cast<uint4*>(out + i) = u;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(xch_empty);
          mbar_arrive(&ml_empty[e]);
          mbar_arrive(&o_free[e]);
        }
      }
    } else if (quarter >= q0 && quarter < q0 + p.softmax_warps) {
      const int row = (quarter - q0) * 32 + lane;  // prompt row of this thread (zeros past P)
      const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
      const uint32_t tS = tmem + lane_bits + col_s(slot);
      for (int it = 0; ok && 2 * it + slot < n_units; ++it) {
        const int tile0 = first_tile(2 * it + slot);
        const int ob = p.split ? it & 1 : 0;  // O buffer of this item
        const uint32_t tO = tmem + lane_bits + col_o(slot) + 64 * ob;
        float m_used = -INFINITY, l = 0.f;
        for (int j = 0; j < n_k && ok; ++j) {
          const int t = it * n_k + j;  // this slot's key tiles so far
          ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[slot], t & 1));
          if (!ok) break;
          tc_fence_after();
          const int valid = min(kKeys, p.length - (tile0 + j) * kKeys);
          if constexpr (kSmall) {
            // Prompts of up to 8 rows: a 16x256b load hands row t's 128 scores
            // to lanes 4t .. 4t + 3, 32 columns each (8k + c and 8k + c + 1,
            // c = 2 (lane % 4)), which is also the 16x128b store's layout of
            // the packed P words; the lanes of rows past P write zero P.
            const int c = 2 * (lane & 3);
            const bool live = (lane >> 2) < p.tokens;
            uint32_t r[64];
            tmem_ld_16x256b_x16(tS, r);
            float x[32];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              x[2 * k] = 8 * k + c < valid ? __uint_as_float(r[4 * k]) : -INFINITY;
              x[2 * k + 1] = 8 * k + c + 1 < valid ? __uint_as_float(r[4 * k + 1]) : -INFINITY;
            }
            float mx = fmaxf(x[0], x[1]);
#pragma unroll
            for (int i = 2; i < 32; i += 2) mx = fmax3(mx, x[i], x[i + 1]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_tile = mx * p.scale_log2;
            const bool move = live && m_tile > m_used + kRescaleThreshold;
            if (__any_sync(0xffffffffu, move)) {
              const float m_new = move ? m_tile : m_used;
              if (j > 0) {
                ok = __all_sync(0xffffffffu,
                                mbar_wait_bounded(&o_full[slot], (it * (n_k - 1) + j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const float alpha_row = move ? fast_exp2(m_used - m_new) : 1.f;
                // TMEM row t's factor, from the first lane of row t's group.
                const float a = __shfl_sync(0xffffffffu, alpha_row, lane < 8 ? 4 * lane : lane);
                const float alpha = lane < 8 ? a : 1.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  float o[16];
                  tmem_ld16(tO + 16 * q, o);
#pragma unroll
                  for (int i = 0; i < 16; ++i) o[i] *= alpha;
                  tmem_st16f(tO + 16 * q, o);
                }
                tmem_wait_st();
                l *= alpha_row;
              }
              m_used = m_new;
            }
            float sum = 0.f;
            uint32_t packed[32];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const float p0 = fast_exp2(fmaf(x[2 * k], p.scale_log2, -m_used));
              const float p1 = fast_exp2(fmaf(x[2 * k + 1], p.scale_log2, -m_used));
              sum += p0 + p1;
              packed[2 * k] = live ? bf16x2(p0, p1) : 0u;
              packed[2 * k + 1] = 0u;  // rows 8.. of the quarter
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            l += sum;
            tmem_st_16x128b_x16(tS, packed);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[slot]);
          } else {
            float v[kKeys];
            tmem_ld128(tS, v);
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
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(&o_full[slot], (it * (n_k - 1) + j - 1) & 1));
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
            if (lane == 0) mbar_arrive(&p_full[slot]);
          }
        }
        if (!ok) break;
        // Small prompt: row t's max and sum are held by lanes 4t .. 4t + 3.
        const float l_row = kSmall ? __shfl_sync(0xffffffffu, l, lane < 8 ? 4 * lane : lane) : l;
        if (p.split) {
          // The epilogue warps take over: each row's (max, sum) for this O
          // buffer, once they have read those of the item two back.
          const float m_row =
              kSmall ? __shfl_sync(0xffffffffu, m_used, lane < 8 ? 4 * lane : lane) : m_used;
          const int e = 2 * slot + ob;
          if (it >= 2)
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(&ml_empty[e], ((it >> 1) - 1) & 1));
          if (!ok) break;
          if (!kSmall || lane < 8) ml[kSplitRows * e + row] = make_float2(m_row, l_row);
          __syncwarp();
          if (lane == 0) mbar_arrive(&ml_full[e]);
          continue;
        }
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&o_final[2 * slot], it & 1));
        if (!ok) break;
        tc_fence_after();
        const int index = item_index(2 * it + slot);
        const int h = index % p.heads, w = index / p.heads;
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
        if (lane == 0) mbar_arrive(&o_free[2 * slot]);
      }
    }
    timed_out = !ok;
    if (timed_out && p.status && lane == 0) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
    tc_fence_before();
    named_sync(1, kThreads);
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

template <bool kSmall>
int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
           const PrefixParams& p, cudaStream_t stream) {
  auto kernel = prefix_cross_tc_kernel<kSmall>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
            "cudaFuncSetAttribute(prompt-pass cross attention)"))
      return rc;
    if (int rc = check_launch_registers(kernel, kLaunchRegs, "prompt-pass cross attention"))
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
  const int softmax_warps = (tokens + 31) / 32;
  // Prompts of up to kSplitRows rows over an even number (2 or more) of key
  // tiles run each item as two halves, one per slot, merged in the CTA.
  const int n_tiles = (length + kKeys - 1) / kKeys;
  const int split = tokens <= kSplitRows && n_tiles >= 2 && n_tiles % 2 == 0 ? 1 : 0;
  PrefixParams p{out,
                 o_st,
                 o_sh,
                 tokens,
                 length,
                 heads,
                 windows * heads,
                 softmax_warps,
                 softmax_warps <= 2 ? 32 * softmax_warps : 0,
                 split,
                 scale * 1.4426950408889634f,
                 status};
  // Prompts of up to 8 rows share each row's softmax out over four lanes.
  return tokens <= 8 ? launch<true>(mq, mk, mv, p, stream) : launch<false>(mq, mk, mv, p, stream);
}

}  // namespace asrback
