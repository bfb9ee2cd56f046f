// Whisper encoder self-attention (non-causal, head_dim 64, bf16) on the
// 5th-generation tensor cores: tcgen05.mma with accumulators in tensor memory.
//
// Replaces F.scaled_dot_product_attention in MultiHeadAttention.forward
// (whisper.py:108-110, via attend :102-104) for the encoder layers.
//
// A work item is one (window b, head h) and two 128-row query tiles; the
// kernel is persistent (one CTA per SM takes items blockIdx.x, + gridDim.x,
// ..., the pair index fastest so that CTAs running together share each
// (window, head)'s keys and values in L2). Warp roles:
//   warp 0      TMA producer: each item's two Q tiles into one of two Q
//               buffers (once the item two before has issued its last S), and
//               its K/V tiles of 128 keys into a STAGES-deep ring that runs on
//               across items (4-D tensor maps over the projections' (batch,
//               length, heads, 64) layout, 128-byte swizzle; rows past the
//               window read as zeros);
//   warp 1      allocates the 512 TMEM columns and issues every MMA (the
//               loop runs warp-wide, an elected lane issues):
//               S = Q_t K^T (SS: both operands from shared memory) and
//               O_t += P V (TS: P from TMEM, V from shared memory);
//   warps 4-7   softmax of query tile 0 (thread = TMEM lane = query row);
//   warps 8-11  softmax of query tile 1.
// TMEM columns: three S buffers [0,128) [128,256) [256,384), O0 [384,448),
// O1 [448,512). Key tiles are numbered J over all of a CTA's items (item i,
// tile j: J = i * n_k + j). The k-th S (tile t, k = 2J + t) goes to buffer
// k % 3; its softmax writes P (packed bf16 pairs) over the buffer's first 64
// columns, and the next S into that buffer is issued right after that P V
// (the tensor core runs one thread's MMAs in order). So S_1(J+1) follows
// P_0(J) V and S_0(J+2) follows P_1(J) V: each tile's next S is computed
// while the other tile's softmax runs, and a softmax goes from one key tile
// to the next without waiting for the tensor core, across item boundaries
// too; an item's first P V into O_t waits only until the previous item's
// epilogue has read O_t.
// Barriers that can run ahead of their waiters come in copies so that no
// waiter ever sees one complete twice: one S barrier per buffer, two P
// barriers per tile (alternating), and O's last P V commits to a barrier of
// its own.
// The running max is rescaled lazily: P uses a stale max m until a tile's max
// exceeds it by more than 8 (log2 units), and only then are O (in TMEM, once
// its previous P V is done) and the row sum rescaled, so P stays <= 2^8.
#include "tcgen05.cuh"

namespace asrback {

namespace {

using namespace tc;

constexpr int kRows = 128;  // query rows per tile (= TMEM lanes)
constexpr int kKeys = 128;  // keys per tile
constexpr int kDim = 64;
constexpr int kStages = 4;
constexpr int kTileBytes = kRows * kDim * 2;  // 16 KB, one Q, K or V tile
// warp 0 TMA, warp 1 MMA (and TMEM owner), warps 2-3 idle, warps 4-11 softmax.
constexpr int kThreads = 12 * 32;
// Registers per thread: the launch gives every thread 168 (384 x 168 = 64512);
// the TMA/MMA warpgroup keeps 56 and the two softmax warpgroups take 224
// (128 x 56 + 256 x 224 = 64512), enough for a key tile's 128 scores, its 64
// packed P words and the row state without spilling.
constexpr int kLaunchRegs = 168;
constexpr int kControlRegs = 56;
constexpr int kSoftmaxRegs = 224;
static_assert(128 * kControlRegs + 256 * kSoftmaxRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch's register pool");
constexpr int kTmemCols = 512;
// TMEM column of S, O and P for query tile t.
// Three S buffers of 128 columns rotate over the two query tiles: the k-th
// S (k = 2j + t) goes to buffer k % 3, and P overwrites the first 64 columns
// of its own S buffer.
__host__ __device__ constexpr int col_buf(int b) { return 128 * b; }
__host__ __device__ constexpr int buf_of(int t, int j) { return (2 * j + t) % 3; }
__host__ __device__ constexpr int col_o(int t) { return 384 + 64 * t; }
// Lazy rescale threshold (log2 units): P <= 2^8 between rescales.
constexpr float kRescaleThreshold = 8.0f;

constexpr int kOffQ = 0;  // two Q buffers of two tiles
constexpr int kOffK = 4 * kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffBar = kOffV + kStages * kTileBytes;
// barriers: q_full[2], q_empty[2] (per Q buffer), kv_full[S], kv_empty[S],
// s_full[3] (one per S buffer), p_full[2][2] (per tile, alternating),
// o_full[2], o_final[2], o_free[2]
constexpr int kNumBars = 2 + 2 + 2 * kStages + 3 + 4 + 2 + 2 + 2;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack

struct TcParams {
  void* out;
  int64_t sb, sh, ss;  // output strides (elements)
  int length;
  int q_pairs;
  int heads;
  int items;  // q_pairs * heads * batch
  float scale_log2;
  int32_t* status;
};

// exp2 of two floats on the FMA pipe, to take load off the SFU: 2^x =
// 2^round(x) * q(f), f = x - round(x) in [-1/2, 1/2], q a cubic fitted here
// for least maximum relative error over that interval (7.5e-5 in float32
// Horner form, below the 2^-9 of the bf16 P it feeds). round(x) comes from
// adding 1.5 * 2^23, whose low mantissa bits then hold it; shifted into the
// exponent field it scales q. Arguments are clamped at -126 (the results there
// are ~1e-38, i.e. zero for P).
constexpr float kPolyC0 = 0.99992805719375610f;
constexpr float kPolyC1 = 0.69326096773147583f;
constexpr float kPolyC2 = 0.24261114001274109f;
constexpr float kPolyC3 = 0.05517166852951050f;
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ void exp2_pair_fma(float x0, float x1, float& e0, float& e1) {
  const uint64_t xx = pack2(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t yy = fadd2(xx, pack2(kRoundMagic, kRoundMagic));
  const uint64_t rr = fadd2(yy, pack2(-kRoundMagic, -kRoundMagic));
  const uint64_t ff = ffma2(rr, pack2(-1.f, -1.f), xx);
  uint64_t pp = ffma2(pack2(kPolyC3, kPolyC3), ff, pack2(kPolyC2, kPolyC2));
  pp = ffma2(pp, ff, pack2(kPolyC1, kPolyC1));
  pp = ffma2(pp, ff, pack2(kPolyC0, kPolyC0));
  float y0, y1, q0, q1;
  unpack2(yy, y0, y1);
  unpack2(pp, q0, q1);
  e0 = __int_as_float(__float_as_int(q0) + (__float_as_int(y0) << 23));
  e1 = __int_as_float(__float_as_int(q1) + (__float_as_int(y1) << 23));
}

// One pair in kPolyEvery takes the FMA-pipe exp2 (0: none). With the MMA
// issue loop warp-wide the SFU is the busiest unit of the softmax; moving a
// quarter of the pairs to the FMA pipe took a layer over 32 windows from 465
// to 442 us on B200 (one in 3: 446, one in 6: 442, one in 8: 443, one in 16:
// 449).
#ifndef ASRBACK_ENCODER_POLY_EVERY
#define ASRBACK_ENCODER_POLY_EVERY 4
#endif
constexpr int kPolyEvery = ASRBACK_ENCODER_POLY_EVERY;

__global__ void __launch_bounds__(kThreads, 1)
    encoder_attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                                const __grid_constant__ CUtensorMap map_k,
                                const __grid_constant__ CUtensorMap map_v,
                                const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;  // [Q buffer]
  uint64_t* q_empty = q_full + 2;
  uint64_t* kv_full = q_empty + 2;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [buffer]
  uint64_t* p_full = s_full + 3;          // [2 * t + (J & 1)]
  uint64_t* o_full = p_full + 4;
  uint64_t* o_final = o_full + 2;
  uint64_t* o_free = o_final + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_k = (p.length + kKeys - 1) / kKeys;
  // This CTA's items: blockIdx.x, + gridDim.x, ...
  const int n_items = p.items > (int)blockIdx.x
                          ? (p.items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                          : 0;
  const int total = n_items * n_k;  // key tiles over all items
  auto item_index = [&](int li) { return (int)blockIdx.x + li * (int)gridDim.x; };

  if (threadIdx.x == 0) {
    for (int q = 0; q < 2; ++q) {
      mbar_init(&q_full[q], 1);
      mbar_init(&q_empty[q], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 3; ++b) mbar_init(&s_full[b], 1);
    for (int t = 0; t < 4; ++t) mbar_init(&p_full[t], 4);  // one arrival per softmax warp
    for (int t = 0; t < 2; ++t) {
      mbar_init(&o_full[t], 1);
      mbar_init(&o_final[t], 1);
      mbar_init(&o_free[t], 4);
    }
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

  // Each warpgroup leaves through its own branch (status, fences, one
  // CTA-wide named barrier, the TMEM release): a register budget is fixed per
  // branch, so the branches never rejoin.
  if (warp < 4) {
    reg_release<kControlRegs>();
    // One lane per warp, elected once: a tcgen05.commit tracks the MMAs of
    // its own thread, so the MMA warp's issues and commits all come from it.
    const bool leader = elect_one();
    // Both control warps run their loops warp-wide (waits by every lane, so
    // the loop state stays warp-uniform) and issue from one elected lane.
    auto wait_warp = [](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
    };
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
        const int pair = index % p.q_pairs, h = (index / p.q_pairs) % p.heads;
        const int b = index / (p.q_pairs * p.heads);
        const int qb = li & 1;
        if (li >= 2) ok = wait_warp(&q_empty[qb], ((li >> 1) - 1) & 1);
        if (!ok) break;
        if (leader) {
          uint8_t* qdst = smem + kOffQ + qb * 2 * kTileBytes;
          mbar_arrive_expect_tx(&q_full[qb], 2 * kTileBytes);
          tma_load_4d(qdst, &map_q, 0, h, (2 * pair) * kRows, b, &q_full[qb]);
          tma_load_4d(qdst + kTileBytes, &map_q, 0, h, (2 * pair + 1) * kRows, b, &q_full[qb]);
        }
        __syncwarp();
        for (int j = 0; j < n_k; ++j, ++g) {
          const int s = g % kStages;
          if (g >= kStages) ok = wait_warp(&kv_empty[s], ((g / kStages) - 1) & 1);
          if (!ok) break;
          if (leader) {
            // K and V of a key tile complete one barrier: the first MMA that
            // reads the tile (its S of query tile 0) waits once for both.
            mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
            tma_load_4d(smem + kOffK + s * kTileBytes, &map_k, 0, h, j * kKeys, b, &kv_full[s]);
            tma_load_4d(smem + kOffV + s * kTileBytes, &map_v, 0, h, j * kKeys, b, &kv_full[s]);
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
        // Descriptors are built once; a step moves the start-address field
        // (address >> 4): 32 bytes along K inside a swizzled row (Q, K), two
        // 8-row swizzle atoms of V (2048 bytes), one tile (kTileBytes). The
        // tensor core takes few MMAs ahead, so the instructions between two
        // MMAs are kept to adds and the waits that are needed.
        const uint64_t q_desc = sw128_desc(smem_addr(smem + kOffQ), 16, 1024);
        const uint64_t k_desc = sw128_desc(smem_addr(smem + kOffK), 16, 1024);
        const uint64_t v_desc = sw128_desc(smem_addr(smem + kOffV), kTileBytes, 1024);
        constexpr uint64_t kStepK = 32 >> 4, kStepV = 2048 >> 4, kTile = kTileBytes >> 4;
        bool ok = true;
        // Position of key tile X in the sequence: item li (Q buffer li & 1), tile
        // j within it, ring slot s, ring lap, S buffer of tile 0. Kept as running
        // counters (one per tile stream below) so the loop divides nothing.
        struct Cursor {
          int X, li, j, s, lap, buf0;
          __device__ void next(int n_k) {
            ++X;
            if (++j == n_k) {
              j = 0;
              ++li;
            }
            if (++s == kStages) {
              s = 0;
              ++lap;
            }
            buf0 = buf0 == 0 ? 2 : buf0 - 1;  // (2X) % 3 steps by 2 mod 3
          }
        };
        // S_t(X): query tile t of item li against key tile X. In issue order
        // S_0(X) comes first of the MMAs that read key tile X (then S_1(X),
        // P_0 V, P_1 V), so it alone waits for the tile; an item's first S also
        // waits for its Q. After the item's last S (t = 1, j == n_k - 1) the Q
        // buffer is free.
        auto issue_qk = [&](int t, const Cursor& c) {
          const int qb = c.li & 1;
          if (t == 0) {
            if (c.j == 0) ok = ok && wait_warp(&q_full[qb], (c.li >> 1) & 1);
            ok = ok && wait_warp(&kv_full[c.s], c.lap & 1);
          }
          if (!ok) return;
          tc_fence_after();
          const int s = c.s;
          const int buf = t == 0 ? c.buf0 : (c.buf0 == 2 ? 0 : c.buf0 + 1);
          if (leader) {
            // K = 64 in four steps of 16 elements.
#pragma unroll
            for (int k = 0; k < kDim / 16; ++k)
              mma_ss(tmem + col_buf(buf), q_desc + (2 * qb + t) * kTile + k * kStepK,
                     k_desc + s * kTile + k * kStepK, kIdescQK, k > 0);
            mma_commit(&s_full[buf]);
            if (t == 1 && c.j == n_k - 1) mma_commit(&q_empty[qb]);
          }
          __syncwarp();
        };
        // O_t (+)= P_t(J) V(J); an item's first one waits until the previous
        // item's epilogue has read O_t; the item's last one commits o_final.
        auto issue_pv = [&](int t, const Cursor& c) {
          const int J = c.X, li = c.li, j = c.j, s = c.s;
          ok = ok && wait_warp(&p_full[2 * t + (J & 1)], (J >> 1) & 1);
          if (j == 0 && li > 0) ok = ok && wait_warp(&o_free[t], (li - 1) & 1);
          if (!ok) return;
          tc_fence_after();
          const int buf = t == 0 ? c.buf0 : (c.buf0 == 2 ? 0 : c.buf0 + 1);
          if (leader) {
            // K = 128 keys in eight steps of 16: P advances 8 TMEM columns
            // (bf16 pairs), V two 8-row swizzle atoms.
#pragma unroll
            for (int k = 0; k < kKeys / 16; ++k)
              mma_ts(tmem + col_o(t), tmem + col_buf(buf) + k * 8, v_desc + s * kTile + k * kStepV,
                     kIdescPV, (j > 0 || k > 0));
            mma_commit(j + 1 < n_k ? &o_full[t] : &o_final[t]);
          }
          __syncwarp();
        };
        // Three cursors: the P V tile J, and the S tiles J + 1 and J + 2.
        Cursor c0{0, 0, 0, 0, 0, 0};
        Cursor c1 = c0, c2 = c0;
        issue_qk(0, c0);
        issue_qk(1, c0);
        c1.next(n_k);
        c2.next(n_k);
        c2.next(n_k);
        if (total > 1) issue_qk(0, c1);
        for (int J = 0; J < total && ok; ++J) {
          issue_pv(0, c0);
          if (ok && J + 1 < total) issue_qk(1, c1);
          if (ok) issue_pv(1, c0);
          if (ok && J + 2 < total) issue_qk(0, c2);
          if (ok && J + kStages < total) {
            if (leader) mma_commit(&kv_empty[c0.s]);
            __syncwarp();
          }
          c0.next(n_k);
          c1.next(n_k);
          c2.next(n_k);
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
    // ---------------- softmax and epilogue (one query row per thread) ----------------
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_bits = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_bits + col_o(t);
    bool ok = true;
    for (int li = 0; li < n_items && ok; ++li) {
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n_k && ok; ++j) {
        const int J = li * n_k + j;
        // This tile's S is the k-th (k = 2J + t): buffer k % 3, the
        // (k / 3)-th completion of that buffer's barrier.
        const int buf = buf_of(t, J);
        const uint32_t tS = tmem + lane_bits + col_buf(buf);
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[buf], ((2 * J + t) / 3) & 1));
        if (!ok) break;
        tc_fence_after();
        const int valid = min(kKeys, p.length - j * kKeys);
        float v[kKeys];
        tmem_ld128(tS, v);
        if (valid < kKeys) {
          // Keys past the window (the ragged last tile) take no weight.
#pragma unroll
          for (int i = 0; i < kKeys; ++i)
            if (i >= valid) v[i] = -INFINITY;
        }
        // Row max as eight short independent chains.
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
            // O_t must be idle: P_t(j-1) V done. (P_t(j-2) V is: S_t(j), just
            // completed, was issued after it.)
            ok = __all_sync(0xffffffffu,
                            mbar_wait_bounded(&o_full[t], (li * (n_k - 1) + j - 1) & 1));
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
            float x0, x1, p0, p1;
            unpack2(ffma2(pack2(v[col], v[col + 1]), scale2, neg_m2), x0, x1);
            if (kPolyEvery > 0 && (i % (kPolyEvery > 0 ? kPolyEvery : 1)) == kPolyEvery - 1) {
              exp2_pair_fma(x0, x1, p0, p1);
            } else {
              p0 = fast_exp2(x0);
              p1 = fast_exp2(x1);
            }
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
        if (lane == 0) mbar_arrive(&p_full[2 * t + (J & 1)]);
      }
      if (!ok) break;
      // O_t is final after P_t(n_k - 1) V, whose commit has a barrier of its own.
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&o_final[t], li & 1));
      if (!ok) break;
      tc_fence_after();
      const int index = item_index(li);
      const int pair = index % p.q_pairs, h = (index / p.q_pairs) % p.heads;
      const int b = index / (p.q_pairs * p.heads);
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
            u.x = bf16x2(o[i] * inv, o[i + 1] * inv);
            u.y = bf16x2(o[i + 2] * inv, o[i + 3] * inv);
            u.z = bf16x2(o[i + 4] * inv, o[i + 5] * inv);
            u.w = bf16x2(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4*>(out + 32 * c + i) = u;
          }
        }
      }
      // O_t has been read: the next item's first P V may overwrite it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[t]);
    }
    timed_out = !ok;
    if (timed_out && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
    tc_fence_before();
    named_sync(1, kThreads);
  }
}

// ---- host side ----

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
    if (int rc = check_launch_registers(encoder_attention_tc_kernel, kLaunchRegs,
                                        "encoder attention"))
      return rc;
    prepared_device = device;
  }
  const int q_pairs = (length + 2 * kRows - 1) / (2 * kRows);
  TcParams p{out, sb, sh, ss, length, q_pairs, heads, q_pairs * heads * batch,
             scale * 1.4426950408889634f, status};
  // Persistent: one CTA per SM (512 TMEM columns each), at most one per item.
  const int ctas = p.items < sm_count() ? p.items : sm_count();
  return launch_pdl(encoder_attention_tc_kernel, dim3(ctas), dim3(kThreads), kSmemBytes, stream,
                    "encoder attention (tensor core) launch", mq, mk, mv, p);
}

}  // namespace asrback
