// Attention within the segments of packed (tokens, heads, head_dim) tensors on
// the 5th-generation tensor cores (tcgen05, accumulators in tensor memory),
// bf16, head_dim 64 or 128, causal or not, grouped-query heads.
//
// Replaces asrback's `attend(q, k, v, segments, causal)` (qwen3_asr.py:152-181):
//   - Qwen3 prompt prefill, TextAttention.prefill (qwen3_asr.py:374-390):
//     causal, 16 query heads over 8 key/value heads, head_dim 128;
//   - Qwen3 audio encoder, AudioAttention.forward (qwen3_asr.py:214-219):
//     non-causal windows.
// Segment s holds the tokens cu[s] .. cu[s+1]-1 (the reference's `starts`).
//
// Work item: one (segment, query head) and two adjacent 128-row query tiles
// of the segment, which share every key/value tile they read. The kernel is
// persistent: one CTA per SM takes items blockIdx.x, + gridDim.x, ... Roles:
//   warp 0      TMA: both Q tiles, then K/V tiles of 128 keys of the query
//               head's key/value head into a STAGES-deep ring. A tile is
//               head_dim / 64 column blocks of 128 bytes (128-byte swizzle);
//               rows past the segment belong to the next one and are masked,
//               rows past the tensor read as zeros. The next item's Q loads
//               once the current item's last S is done;
//   warp 1      allocates the 512 TMEM columns and issues every MMA (the
//               loop runs warp-wide, an elected lane issues): S = Q K^T (SS)
//               and O += P V (TS: P from TMEM);
//   warp 2      the item list: 32 lanes look up 32 of the CTA's items at a
//               time (the segment bounds are global loads) and publish the
//               valid ones, in order, into an 8-entry shared-memory ring
//               that the other roles read;
//   warps 4-11  softmax of query tile 0 and 1 (thread = TMEM lane = row), and
//               the epilogue: O / l as bf16, staged per warp in shared memory
//               so that each store instruction writes whole 128-byte rows.
// TMEM of query tile t: S_t [256t, 256t+128), the softmax writing P_t (packed
// bf16 pairs) over its first 64 columns, and O_t [256t+128, 256t+128+D).
// Per key tile j the MMA warp issues P_t(j-1) V, then S_t(j) into the same
// columns (the tensor core runs one thread's MMAs in order), so S_t(j)'s
// completion also means O_t is idle: the lazy rescale (P uses a stale max
// until a tile's max exceeds it by more than 8 in log2 units) needs no wait.
// The next item's first P V waits until the current item's epilogue has read
// O_t. Causal: query row r reads keys 0..r of its segment, so a query tile
// stops at the key tile of its own rows and only that diagonal tile is masked.
//
// Single-tile mode (every segment at most 128 tokens, e.g. the audio windows):
// an item is one (segment, query head), one query tile and one key tile. Item
// k uses Q buffer, TMEM S/O columns and softmax warpgroup k & 1 (those of
// query tile t = k & 1 above), and the MMA warp issues S(k + 1) before
// P(k) V(k), so item k+1's S runs under item k's softmax and item k's
// epilogue under item k+1's softmax.
#include <algorithm>

#include "tcgen05.cuh"

namespace asrback {

namespace {

using namespace tc;

constexpr int kRows = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKeys = 128;  // keys per tile
constexpr int kThreads = 12 * 32;
// Registers per thread: 168 at launch (384 x 168 = 64512); the warpgroup of
// the TMA, MMA and item-list warps keeps 72, the two softmax warpgroups take
// 208 (128 x 72 + 256 x 208 = 62464), so neither spills: a key tile's 128
// scores and the row state stay in registers.
constexpr int kLaunchRegs = 168;
constexpr int kControlRegs = 72;
constexpr int kSoftmaxRegs = 208;
static_assert(128 * kControlRegs + 256 * kSoftmaxRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch's register pool");
constexpr int kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;
constexpr int kItemSlots = 8;        // entries of the shared-memory item ring
constexpr int kItemReaders = 2 + 8;  // TMA warp, MMA warp, 8 softmax warps
constexpr int kStageRowBytes = 128;  // epilogue staging: 64 bf16 columns per row
constexpr int kStageWarpBytes = 32 * kStageRowBytes;

// One work item: a (segment, query head, pair of adjacent 128-row query tiles).
struct Item {
  int start, len;    // the segment's first token and length
  int h, kvh;        // query head, its key/value head
  int first_row[2];  // first row of each query tile within the segment
  int n_k[2];        // key tiles each query tile reads (0: the tile is absent)
  int n_max;         // 0: no work (a skipped item, or the end of the list)
};

template <int D>
struct VarlenShape {
  static constexpr int kAtoms = D / 64;           // 128-byte column blocks per row
  static constexpr int kAtomBytes = kRows * 128;  // one column block of a tile
  static constexpr int kTileBytes = kAtoms * kAtomBytes;
  static constexpr int kStages = D == 128 ? 2 : 4;
  static constexpr int kOffQ = 0;  // two Q tiles
  static constexpr int kOffK = 2 * kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffStage = kOffV + kStages * kTileBytes;  // 8 warps x 32 rows
  static constexpr int kOffBar = kOffStage + 8 * kStageWarpBytes;
  // barriers: q_full[2], q_empty[2], kv_full[S], kv_empty[S], s_full[2],
  // p_full[2], o_full[2], o_free[2], item_full[R], item_empty[R]
  static constexpr int kNumBars = 2 + 2 + 2 * kStages + 2 + 2 + 2 + 2 + 2 * kItemSlots;
  static constexpr int kOffItems = kOffBar + kNumBars * 8;
  static constexpr int kOffTmemSlot = kOffItems + kItemSlots * static_cast<int>(sizeof(Item));
  static constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory exceeds a CTA's 227 KB");
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
};

struct VarlenParams {
  void* out;
  int64_t os_tok, os_head;  // output strides (elements)
  const int32_t* cu;        // segment starts, segments + 1 entries
  int segments;
  int heads;
  int pairs;                // query-tile pairs per segment at max_length
  int tokens;
  int max_length;
  int group;                // query heads per key/value head
  int causal;
  float scale_log2;
  int32_t* status;
};

// Items are numbered head fastest (the query heads of one key/value head run
// together), then segment, then pair. With the pair slowest, the CTAs' strided
// shares each hold every pair index in proportion: under the causal mask a
// later pair costs more, and a CTA count that is a multiple of the pairs per
// segment would otherwise hand each CTA pairs of one cost only.
__device__ __forceinline__ Item item_at(const VarlenParams& p, int index) {
  Item it;
  it.h = index % p.heads;
  const int seg = (index / p.heads) % p.segments;
  const int pair = index / (p.heads * p.segments);
  it.start = p.cu[seg];
  it.len = p.cu[seg + 1] - it.start;
  it.kvh = it.h / p.group;
  it.n_k[0] = it.n_k[1] = it.n_max = 0;
  it.first_row[0] = it.first_row[1] = 0;
  // A segment outside the tensor or longer than the launch covers is skipped
  // (its output rows untouched) and reported once; nothing is read or written
  // out of bounds.
  if (it.start < 0 || it.len < 0 || it.start + it.len > p.tokens || it.len > p.max_length) {
    if (pair == 0 && it.h == 0 && p.status) atomicOr(p.status, ASRBACK_STATUS_SEGMENT);
    return it;
  }
  if (pair * 2 * kRows >= it.len) return it;  // the segment is shorter
  const int n_seg = (it.len + kKeys - 1) / kKeys;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    it.first_row[t] = (2 * pair + t) * kRows;
    it.n_k[t] = it.first_row[t] >= it.len
                    ? 0
                    : (p.causal ? min(n_seg, it.first_row[t] / kKeys + 1) : n_seg);
  }
  it.n_max = max(it.n_k[0], it.n_k[1]);
  return it;
}

template <int D, bool kSingle>
__global__ void __launch_bounds__(kThreads, 1)
    varlen_attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                               const __grid_constant__ CUtensorMap map_k,
                               const __grid_constant__ CUtensorMap map_v,
                               const __grid_constant__ VarlenParams p) {
  using Sh = VarlenShape<D>;
  constexpr int S = Sh::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Sh::kOffBar);
  uint64_t* q_full = bars;  // [2]: per Q buffer (pair mode: [0] only)
  uint64_t* q_empty = q_full + 2;
  uint64_t* kv_full = q_empty + 2;  // K and V of a ring slot, one barrier
  uint64_t* kv_empty = kv_full + S;
  uint64_t* s_full = kv_empty + S;  // [2]: per query tile (single-tile mode: per item parity)
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_free = o_full + 2;
  uint64_t* item_full = o_free + 2;
  uint64_t* item_empty = item_full + kItemSlots;
  Item* ring = reinterpret_cast<Item*>(smem + Sh::kOffItems);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sh::kOffTmemSlot);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // TMEM columns of query tile t's S and O.
  auto s_col = [](int t) { return 256 * t; };
  auto o_col = [](int t) { return 256 * t + 128; };

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);  // one arrival per softmax warp
      mbar_init(&o_full[t], 1);
      mbar_init(&o_free[t], 4);
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int e = 0; e < kItemSlots; ++e) {
      mbar_init(&item_full[e], 1);
      mbar_init(&item_empty[e], kItemReaders);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool timed_out = false;

  // Entry n of the CTA's item list, read by a whole warp; false if the wait
  // ran out. Every reader warp releases every entry, the end-of-list entry
  // (n_max 0) included.
  auto read_item = [&](int n, Item& it) {
    const int e = n % kItemSlots;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&item_full[e], (n / kItemSlots) & 1)))
      return false;
    it = ring[e];
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[e]);
    return true;
  };

  // Waits of a role run warp-wide: every lane polls, the warp agrees.
  auto wait_warp = [](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
  };

  // Each warpgroup leaves through its own branch (status, fences, one
  // CTA-wide named barrier, the TMEM release): a register budget is fixed per
  // branch, so the branches never rejoin.
  if (warp < 4) {
  reg_release<kControlRegs>();
  // One lane per warp, elected once: a tcgen05.commit tracks the MMAs of its
  // own thread, so the MMA warp's issues and commits all come from it.
  const bool leader = elect_one();
  // The TMA and MMA warps run their loops warp-wide (the loop state stays
  // warp-uniform) and issue from one elected lane.
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (leader) {
      prefetch_tensormap(&map_q);
      prefetch_tensormap(&map_k);
      prefetch_tensormap(&map_v);
    }
    __syncwarp();
    int g = 0;  // K/V tiles loaded, over all items
    auto load_kv = [&](const Item& it, int j) {
      const int s = g % S;
      if (g >= S && !wait_warp(&kv_empty[s], ((g / S) - 1) & 1)) return false;
      if (leader) {
        mbar_arrive_expect_tx(&kv_full[s], 2 * Sh::kTileBytes);
#pragma unroll
        for (int a = 0; a < Sh::kAtoms; ++a)
          tma_load_3d(smem + Sh::kOffK + s * Sh::kTileBytes + a * Sh::kAtomBytes, &map_k,
                      64 * a, it.kvh, it.start + j * kKeys, &kv_full[s]);
#pragma unroll
        for (int a = 0; a < Sh::kAtoms; ++a)
          tma_load_3d(smem + Sh::kOffV + s * Sh::kTileBytes + a * Sh::kAtomBytes, &map_v,
                      64 * a, it.kvh, it.start + j * kKeys, &kv_full[s]);
      }
      __syncwarp();
      ++g;
      return true;
    };
    for (int n = 0;; ++n) {
      Item it;
      if (!read_item(n, it)) {
        timed_out = true;
        break;
      }
      if (it.n_max == 0) break;
      if constexpr (kSingle) {
        // Item n: Q into buffer n & 1 once item n-2's S is done, then its
        // one key/value tile.
        const int b = n & 1;
        if (n >= 2 && !wait_warp(&q_empty[b], ((n >> 1) - 1) & 1)) {
          timed_out = true;
          break;
        }
        if (leader) {
          mbar_arrive_expect_tx(&q_full[b], Sh::kTileBytes);
#pragma unroll
          for (int a = 0; a < Sh::kAtoms; ++a)
            tma_load_3d(smem + Sh::kOffQ + b * Sh::kTileBytes + a * Sh::kAtomBytes, &map_q,
                        64 * a, it.h, it.start, &q_full[b]);
        }
        __syncwarp();
        if (!load_kv(it, 0)) {
          timed_out = true;
          break;
        }
      } else {
        // Q of the previous item is in use until its last S is done.
        if (n > 0 && !wait_warp(q_empty, (n - 1) & 1)) {
          timed_out = true;
          break;
        }
        const int q_tiles = it.n_k[1] > 0 ? 2 : 1;
        if (leader) {
          mbar_arrive_expect_tx(q_full, q_tiles * Sh::kTileBytes);
          for (int t = 0; t < q_tiles; ++t)
#pragma unroll
            for (int a = 0; a < Sh::kAtoms; ++a)
              tma_load_3d(smem + Sh::kOffQ + t * Sh::kTileBytes + a * Sh::kAtomBytes, &map_q,
                          64 * a, it.h, it.start + it.first_row[t], q_full);
        }
        __syncwarp();
        for (int j = 0; j < it.n_max && !timed_out; ++j) timed_out = !load_kv(it, j);
        if (timed_out) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t kIdescQK = idesc_bf16(kRows, kKeys, false);
    // P V in one MMA per 16 keys over all head_dim columns: V is an MN-major
    // operand whose 64-column blocks lie kAtomBytes apart (the descriptor's
    // leading byte offset), so N = head_dim spans them.
    constexpr uint32_t kIdescPV = idesc_bf16(kRows, D, true);
    // Descriptors are built once and stepped by adds of address >> 4:
    // 32 bytes per 16 elements along K inside a 128-byte block, one block
    // (kAtomBytes) per 64 elements, 2048 bytes per 16 rows of V.
    const uint64_t q_desc = sw128_desc(smem_addr(smem + Sh::kOffQ), 16, 1024);
    const uint64_t k_desc = sw128_desc(smem_addr(smem + Sh::kOffK), 16, 1024);
    const uint64_t v_desc = sw128_desc(smem_addr(smem + Sh::kOffV), Sh::kAtomBytes, 1024);
    constexpr uint64_t kTile = Sh::kTileBytes >> 4, kAtom = Sh::kAtomBytes >> 4;
    // S_t = Q buffer t . K tile of ring slot s (called by the elected lane).
    auto issue_qk = [&](int t, int s) {
      // K = head_dim in steps of 16: four per 128-byte block.
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint64_t off = (k / 4) * kAtom + (k % 4) * (32 >> 4);
        mma_ss(tmem + s_col(t), q_desc + t * kTile + off, k_desc + s * kTile + off, kIdescQK,
               k > 0);
      }
    };
    // O_t (+)= P_t . V tile of ring slot s (called by the elected lane).
    auto issue_pv = [&](int t, int s, bool accumulate) {
      // K = 128 keys in steps of 16: P advances 8 TMEM columns (bf16 pairs),
      // V 16 rows (2048 bytes) within each of its column blocks.
#pragma unroll
      for (int k = 0; k < kKeys / 16; ++k)
        mma_ts(tmem + o_col(t), tmem + s_col(t) + k * 8, v_desc + s * kTile + k * (2048 >> 4),
               kIdescPV, accumulate || k > 0);
    };
    bool ok = true;
    if constexpr (kSingle) {
      // Before P(k) V(k), S is issued for items up to k + 1: S(m)
      // overwrites P(m - 2), whose P V is already issued. P V(k) overwrites
      // O_{k & 1} once item k-2's epilogue has read it. S(k) waited for its
      // K/V slot (one barrier for both), so P V(k) reads V without a wait.
      int k_s = 0;  // items whose S is issued
      bool more = true;
      for (int k = 0; ok; ++k) {
        while (more && k_s < k + 2) {
          Item it;
          ok = read_item(k_s, it);
          if (!ok) break;
          if (it.n_max == 0) {
            more = false;
            break;
          }
          const int t = k_s & 1;
          ok = wait_warp(&q_full[t], (k_s >> 1) & 1) &&
               wait_warp(&kv_full[k_s % S], (k_s / S) & 1);
          if (!ok) break;
          tc_fence_after();
          if (leader) {
            issue_qk(t, k_s % S);
            mma_commit(&s_full[t]);
            mma_commit(&q_empty[t]);
          }
          __syncwarp();
          ++k_s;
        }
        if (!ok || k >= k_s) break;
        const int t = k & 1;
        ok = wait_warp(&p_full[t], (k >> 1) & 1);
        if (ok && k >= 2) ok = wait_warp(&o_free[t], ((k >> 1) - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          issue_pv(t, k % S, false);
          mma_commit(&o_full[t]);
          mma_commit(&kv_empty[k % S]);
        }
        __syncwarp();
      }
    } else {
      int base = 0;            // global index of the item's first K/V tile
      int p_seen[2] = {0, 0};  // p_full completions consumed, per query tile
      int o_done[2] = {0, 0};  // items whose O_t is final (o_full commits)
      for (int n = 0; ok; ++n) {
        Item it;
        ok = read_item(n, it);
        if (!ok || it.n_max == 0) break;
        ok = wait_warp(q_full, n & 1);
        // Step j: for each query tile still reading keys, P_t(j-1) V(j-1)
        // once its softmax has written P_t(j-1) (the first of an item also
        // once the previous item's epilogue has read O_t), then S_t(j) over
        // the same columns (or, after its last key tile, the commit that
        // O_t is final). After the item's last S its Q buffer is released.
        // The wait for K/V tile j (one barrier for both) comes before S(j),
        // so P V(j) at step j + 1 reads V without another wait.
        for (int j = 0; j <= it.n_max && ok; ++j) {
          const int g = base + j;
          if (j < it.n_max) ok = wait_warp(&kv_full[g % S], (g / S) & 1);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (it.n_k[t] == 0 || j > it.n_k[t]) continue;
            if (j > 0) {
              ok = wait_warp(&p_full[t], p_seen[t] & 1);
              ++p_seen[t];
              if (ok && j == 1 && o_done[t] > 0) ok = wait_warp(&o_free[t], (o_done[t] - 1) & 1);
              if (!ok) break;
              tc_fence_after();
              if (leader) issue_pv(t, (g - 1) % S, j > 1);
              __syncwarp();
            }
            if (leader) {
              if (j < it.n_k[t]) {
                issue_qk(t, g % S);
                mma_commit(&s_full[t]);
              } else {
                mma_commit(&o_full[t]);
              }
            }
            __syncwarp();
            if (j >= it.n_k[t]) ++o_done[t];
          }
          if (!ok) break;
          if (leader) {
            if (j == it.n_max - 1) mma_commit(q_empty);
            if (j > 0) mma_commit(&kv_empty[(g - 1) % S]);
          }
          __syncwarp();
        }
        base += it.n_max;
      }
    }
    timed_out = !ok;
  } else if (warp == 2) {
    // ---------------- item list ----------------
    // Lane i looks up item base + i * gridDim.x; the valid ones are published
    // in order, at most kItemSlots per round so that no lane waits on an
    // entry another lane of this warp has yet to write.
    const int items = p.segments * p.heads * p.pairs;
    int n = 0;  // entries published
    for (int base = blockIdx.x; base < items && !timed_out; base += 32 * gridDim.x) {
      const int index = base + lane * gridDim.x;
      Item it;
      if (index < items) {
        it = item_at(p, index);
      } else {
        it.n_max = 0;
      }
      const uint32_t valid = __ballot_sync(0xffffffffu, it.n_max > 0);
      const int rank = __popc(valid & ((1u << lane) - 1u));
      for (int round = 0; round < __popc(valid); round += kItemSlots) {
        if (it.n_max > 0 && rank >= round && rank < round + kItemSlots) {
          const int m = n + rank;
          const int e = m % kItemSlots;
          if (m >= kItemSlots && !mbar_wait_bounded(&item_empty[e], ((m / kItemSlots) - 1) & 1)) {
            timed_out = true;
          } else {
            ring[e] = it;
            mbar_arrive(&item_full[e]);
          }
        }
        if (__any_sync(0xffffffffu, timed_out)) {
          timed_out = true;
          break;
        }
      }
      n += __popc(valid);
    }
    // The end of the list.
    if (!timed_out && lane == 0) {
      const int e = n % kItemSlots;
      if (n >= kItemSlots && !mbar_wait_bounded(&item_empty[e], ((n / kItemSlots) - 1) & 1)) {
        timed_out = true;
      } else {
        ring[e].n_max = 0;
        mbar_arrive(&item_full[e]);
      }
    }
  }
  if (timed_out && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
  tc_fence_before();
  named_sync(1, kThreads);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  } else {
    reg_acquire<kSoftmaxRegs>();
    // ---------------- softmax and epilogue (one query row per thread) ----------------
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_bits + s_col(t);
    const uint32_t tO = tmem + lane_bits + o_col(t);
    uint8_t* stage = smem + Sh::kOffStage + (warp - 4) * kStageWarpBytes;
    bool ok = true;
    int s_seen = 0, o_seen = 0;  // s_full[t] / o_full[t] completions consumed

    // Output rows of this warp for the item whose O_t is final: O / l as bf16. Each lane writes its row into the staging rows
    // (16-byte chunk c at position c ^ (row & 7), so that eight rows' chunks
    // fall in distinct banks); then each store instruction writes four rows'
    // 128 contiguous bytes.
    auto epilogue = [&](int start, int len, int h, int first_row, float l) {
      ok = __all_sync(0xffffffffu, mbar_spin_bounded(&o_full[t], o_seen & 1));
      ++o_seen;
      if (!ok) return;
      tc_fence_after();
      const float inv = 1.f / l;
      const int row0 = first_row + quarter * 32;  // the warp's first row in the segment
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) +
                           static_cast<int64_t>(start + row0) * p.os_tok + h * p.os_head;
#pragma unroll
      for (int half = 0; half < D / 64; ++half) {
        float o[64];
        tmem_ld64(tO + 64 * half, o);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 u;
          u.x = bf16x2(o[8 * c] * inv, o[8 * c + 1] * inv);
          u.y = bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          u.z = bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          u.w = bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(stage + lane * kStageRowBytes + ((c ^ (lane & 7)) << 4)) = u;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3), c = lane & 7;
          if (row0 + r < len) {
            const uint4 u =
                *reinterpret_cast<const uint4*>(stage + r * kStageRowBytes + ((c ^ (r & 7)) << 4));
            *reinterpret_cast<uint4*>(out + r * p.os_tok + 64 * half + 8 * c) = u;
          }
        }
        __syncwarp();
      }
      // O_t has been read: the next item's P V may overwrite it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[t]);
    };

    for (int n = 0; ok; ++n) {
      Item it;
      ok = read_item(n, it);
      if (!ok || it.n_max == 0) break;
      if (kSingle ? ((n & 1) != t) : it.n_k[t] == 0) continue;
      const int tile = kSingle ? 0 : t;
      const int row = it.first_row[tile] + quarter * 32 + lane;  // within the segment
      // Keys this row may read: its segment, and (causal) up to itself.
      const int limit = p.causal ? min(it.len, row + 1) : it.len;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_k[tile] && ok; ++j) {
        ok = __all_sync(0xffffffffu, mbar_spin_bounded(&s_full[t], s_seen & 1));
        ++s_seen;
        if (!ok) break;
        tc_fence_after();
        const int valid = limit - j * kKeys;
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
        // Rows whose tile max passes the used max by more than the threshold
        // move it; the warp rescales O together (tcgen05.ld/st are
        // warp-wide), the other rows with alpha = 1.
        const bool move = m_tile > m_used + kRescaleThreshold;
        if (__any_sync(0xffffffffu, move)) {
          const float m_new = move ? m_tile : m_used;
          if (j > 0) {
            // O_t is idle: P_t(j-1) V was issued before S_t(j), which is done.
            const float alpha = move ? fast_exp2(m_used - m_new) : 1.f;
#pragma unroll
            for (int c = 0; c < D / 16; ++c) {
              float o[16];
              tmem_ld16(tO + 16 * c, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] *= alpha;
              tmem_st16f(tO + 16 * c, o);
            }
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
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      epilogue(it.start, it.len, it.h, it.first_row[tile], l);
    }
    timed_out = !ok;
    if (timed_out && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
    tc_fence_before();
    named_sync(1, kThreads);
  }
}

// (tokens, heads, head_dim) bf16 view with the given element strides as a
// 3-D tensor map {d, head, token}; 64 x 1 x 128 boxes (one 128-byte column
// block of 128 rows), 128-byte swizzle, zero fill past the tensor.
int make_map_3d(CUtensorMap* map, const void* base, int tokens, int heads, int head_dim,
                int64_t s_tok, int64_t s_head) {
  int rc = ASRBACK_OK;
  auto encode = tensor_map_encoder(&rc);
  if (!encode) return rc;
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)s_head * 2, (cuuint64_t)s_tok * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kRows};
  cuuint32_t elem_strides[3] = {1, 1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(ASRBACK_ERR_ARGUMENT,
                "cuTensorMapEncodeTiled rejected the layout (error %d): strides (%lld, %lld)",
                (int)res, (long long)s_tok, (long long)s_head);
  return ASRBACK_OK;
}

template <int D, bool kSingle>
int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
           const VarlenParams& p, cudaStream_t stream) {
  using Sh = VarlenShape<D>;
  auto kernel = varlen_attention_tc_kernel<D, kSingle>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmemBytes),
            "cudaFuncSetAttribute(varlen attention)"))
      return rc;
    if (int rc = check_launch_registers(kernel, kLaunchRegs, "varlen attention")) return rc;
    prepared_device = device;
  }
  // Persistent: one CTA per SM (512 TMEM columns each), at most one per item.
  const long long items = (long long)p.segments * p.heads * p.pairs;
  const int ctas = static_cast<int>(std::min<long long>(items, sm_count()));
  kernel<<<ctas, kThreads, Sh::kSmemBytes, stream>>>(mq, mk, mv, p);
  return check_cuda(cudaGetLastError(), "varlen attention (tensor core) launch");
}

}  // namespace

// Launches the tensor-core varlen attention; arguments already validated
// (bf16, head_dim 64 or 128, 16-byte aligned pointers and strides).
int varlen_attention_tc(int tokens, int heads, int kv_heads, int head_dim, const void* q,
                        int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                        int64_t k_head, const void* v, int64_t v_tok, int64_t v_head,
                        const int32_t* cu, int segments,
                        int max_length, int causal, void* out, int64_t o_tok, int64_t o_head,
                        float scale, int32_t* status, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  if (int rc = make_map_3d(&mq, q, tokens, heads, head_dim, q_tok, q_head)) return rc;
  if (int rc = make_map_3d(&mk, k, tokens, kv_heads, head_dim, k_tok, k_head)) return rc;
  if (int rc = make_map_3d(&mv, v, tokens, kv_heads, head_dim, v_tok, v_head)) return rc;
  VarlenParams p{out,
                 o_tok,
                 o_head,
                 cu,
                 segments,
                 heads,
                 (max_length + 2 * kRows - 1) / (2 * kRows),
                 tokens,
                 max_length,
                 heads / kv_heads,
                 causal ? 1 : 0,
                 scale * 1.4426950408889634f,
                 status};
  // Segments of at most one query tile run two items per CTA at a time.
  const bool single = max_length <= kRows;
  if (head_dim == 128)
    return single ? launch<128, true>(mq, mk, mv, p, stream)
                  : launch<128, false>(mq, mk, mv, p, stream);
  return single ? launch<64, true>(mq, mk, mv, p, stream) : launch<64, false>(mq, mk, mv, p, stream);
}

}  // namespace asrback
