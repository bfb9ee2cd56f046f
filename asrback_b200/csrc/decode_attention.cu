// Split-KV decode attention for one query token per row, sm_100a.
//
// One template serves the three decode call sites of asrback:
//   kWhisperSelf  - DecoderLayer.forward step branch (whisper.py:222-237):
//                   the step's key/value are written at positions[b] and the
//                   row attends to keys 0..positions[b];
//   kWhisperCross - the cross-attention call (whisper.py:239-240): all keys;
//   kQwen3        - TextAttention.step (qwen3_asr.py:392-432): q/k RMSNorm and
//                   rotate-half RoPE (qwen3_asr.py:366-372) in the prologue,
//                   the key/value write (:409-411), then grouped-query
//                   attention, query head h reading key/value head h / QPK.
// The Whisper modes also serve the eager prompt pass (whisper.py:228-240 with
// length == P, from _prefill and _detect_languages): each of a window's P
// tokens is a query row of its own that reads the window's cache row; self
// attention then reads keys 0..t for token t and writes nothing (the caller
// has already written the pass's keys/values).
//
// Work split. A CTA owns one row b, one group of G key/value heads and one
// chunk of key positions (a "split"). Its keys stream through shared memory
// in tiles of TP positions x G heads x D, each tile one contiguous block of
// the cache moved by the TMA engine (cp.async.bulk) into a STAGES-deep ring
// guarded by mbarriers; one producer warp issues the copies, the consumer
// warps compute. Only the positions a row has written are read (positions[b]
// is read on the device, so the launch shape depends only on the cache view).
//
// Compute. LPK = D/8 lanes share a key row, each lane holding eight elements
// (16 bytes of bf16); a warp covers KPW = 32/LPK keys per pass. Scores are
// reduced with xor-shuffles inside the LPK lanes and folded into an online
// softmax (base-2, the scale pre-multiplied by log2 e) once per tile. The key
// at the row's own position (the one this step writes) is taken from
// registers, so the cache write and the tile reads never overlap.
//
// Splits. The grid has num_splits CTAs per (row, group); a row uses as many
// as its own key count fills at `chunk` keys or more apiece and cuts its keys
// evenly between them (whole tiles), so the CTAs of a launch carry similar
// byte counts whatever the rows' lengths. A row's splits each leave (m, l, o)
// partials in the workspace; the last CTA of the row to finish (an atomic
// counter, re-armed to zero by that CTA) merges them and writes the output.
// A row with a single active split writes its output directly.
#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace asrback {

enum DecodeMode { kWhisperSelf = 0, kWhisperCross = 1, kQwen3 = 2 };

constexpr int kMaxSplits = 64;

// prefix_cross_tc.cu: the tensor-core prompt-pass cross-attention.
int whisper_cross_prefix_tc(int windows, int tokens, int heads, int length, const void* q,
                            int64_t q_st, int64_t q_sh, const void* k, const void* v,
                            int64_t c_sb, int64_t c_sh, void* out, int64_t o_st, int64_t o_sh,
                            float scale, int32_t* status, cudaStream_t stream);

struct DecodeParams {
  // query (Whisper): element (b, h, d) at q[b*q_sb + h*q_sh + d]
  const void* q;
  int64_t q_sb, q_sh;
  // the step's new key/value (Whisper self): (b, h, d) at [b*kn_sb + h*kn_sh + d]
  const void* k_new;
  const void* v_new;
  int64_t kn_sb, kn_sh;
  // caches: element (b, kv head h, position p, d) at [b*c_sb + h*c_sh + p*c_sp + d]
  void* k_cache;
  void* v_cache;
  int64_t c_sb, c_sh, c_sp;
  const int64_t* positions;  // (batch,) or null for a fixed key count
  // Prefix calls (Whisper eager branch), tokens_per_row > 0: query row r is
  // token t = r % tokens_per_row of cache row r / tokens_per_row. Self
  // attention then reads the cache's keys 0..t (all of them written before
  // the launch) and writes none; positions and k_new/v_new are unused.
  // Zero: one query row per cache row (the step calls).
  int tokens_per_row;
  int length;                // cross: key count; self/Qwen3: cache view length
  void* out;                 // (b, q head h, d) at out[b*o_sb + h*o_sh + d]
  int64_t o_sb, o_sh;
  float scale_log2;          // softmax scale * log2(e)
  int groups;                // key/value head groups (grid.y)
  int chunk;                 // key positions per split
  int num_splits;            // grid.x
  // Qwen3 split clusters: a row's num_splits CTAs (2..C::CLUSTER_MAX) are
  // launched as one thread-block cluster along x, and splits 1.. hand their
  // partial states to split 0 through split 0's shared memory. 0: off.
  int cluster_splits;
  float* partial;            // workspace partials
  int* counters;             // workspace counters, one per (row, group)
  int32_t* status;           // device status word (may be null)
  // Qwen3 prologue
  const void* qkv;
  int64_t qkv_sb;
  const void* q_norm_w;
  const void* k_norm_w;
  float eps;
  const void* cos;
  const void* sin;
  int64_t table_s;
  int q_heads;
  int kv_heads;
};

template <typename T_, int D_, int G_, int QPK_, int WPH_, int TP_, int STAGES_, int MODE_>
struct DecodeConfig {
  using T = T_;
  static constexpr int D = D_, G = G_, QPK = QPK_, WPH = WPH_, TP = TP_, STAGES = STAGES_;
  static constexpr int MODE = MODE_;
  static constexpr int LPK = D / 8;
  static constexpr int KPW = 32 / LPK;
  static constexpr int NP = TP / (WPH * KPW);
  static constexpr int CWARPS = G * WPH;
  static constexpr int CTHREADS = CWARPS * 32;
  static constexpr int THREADS = CTHREADS + 32;
  static constexpr int QH = G * QPK;
  static constexpr int ROW_BYTES = G * D * (int)sizeof(T);
  static constexpr int TILE_BYTES = TP * ROW_BYTES;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = STAGES * TILE_BYTES;
  static constexpr int RING_BYTES = 2 * STAGES * TILE_BYTES;
  // The cross-warp merge slots and the split-merge weights are used only once
  // the ring has drained, so they share its shared memory when they fit.
  static constexpr int MERGE_FLOATS = CWARPS * QPK * (D + 2);
  // Split merge: per (query head, split) the weight and the row sum.
  static constexpr int SCRATCH_BYTES = MERGE_FLOATS * 4 + 2 * QH * kMaxSplits * 4;
  static constexpr bool SCRATCH_IN_RING = SCRATCH_BYTES <= RING_BYTES;
  static constexpr int OFF_MERGE = SCRATCH_IN_RING ? 0 : RING_BYTES;
  static constexpr int OFF_WEIGHTS = OFF_MERGE + MERGE_FLOATS * 4;
  static constexpr int OFF_BAR =
      ((SCRATCH_IN_RING ? RING_BYTES : RING_BYTES + SCRATCH_BYTES) + 15) / 16 * 16;
  // Split cluster (Qwen3): a ready flag per split, then splits 1..'s partial
  // states, [CLUSTER_MAX - 1][QH][D + 2], in split 0's shared memory. As
  // many splits as fit in 227 KB, at most 4 (the cluster sizes used).
  static constexpr int OFF_XFLAG = OFF_BAR + 2 * STAGES * 8 + 16;
  static constexpr int OFF_XFER = OFF_XFLAG + 64;
  static constexpr int XSLOT_BYTES = QH * (D + 2) * 4;
  static constexpr int CLUSTER_FIT = 1 + (227 * 1024 - OFF_XFER - 1024) / XSLOT_BYTES;
  static constexpr int CLUSTER_MAX = MODE != 2 ? 0 : CLUSTER_FIT > 4 ? 4 : CLUSTER_FIT;
  static constexpr int XFER_BYTES = MODE == 2 ? 64 + (CLUSTER_MAX - 1) * XSLOT_BYTES : 0;
  static constexpr int SMEM = OFF_BAR + 2 * STAGES * 8 + 16 + XFER_BYTES;
  // CTAs per SM that shared memory (228 KB, 1 KB reserved per CTA) and the
  // 2048-thread limit allow; registers are budgeted to match.
  static constexpr int BY_SMEM = (228 * 1024) / (SMEM + 1024);
  static constexpr int BY_THREADS = 2048 / THREADS;
  static constexpr int MIN_BLOCKS =
      (BY_SMEM < BY_THREADS ? BY_SMEM : BY_THREADS) < 1 ? 1
                                                        : (BY_SMEM < BY_THREADS ? BY_SMEM : BY_THREADS);
  static_assert(NP >= 1 && NP * WPH * KPW == TP, "tile must split evenly over warps");
  static_assert(LPK >= 1 && LPK <= 32 && (32 % LPK) == 0, "head_dim must be 8..256");
  static_assert(TILE_BYTES % 16 == 0, "bulk copies move 16-byte multiples");
};

template <int LPK>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int off = LPK / 2; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// Per-head RMSNorm then rotate-half RoPE of one head row held as lane slices
// (LPK = D/8 lanes per row). Rounds like the reference's elementwise ops in T:
// F.rms_norm rounds x * rsqrt(mean(x^2) + eps) * w once; the rotation rounds
// x*cos, rotated*sin and their sum (each torch op rounds its result).
// The weight, cos and sin slices come in already loaded (w, cs, sn).
template <typename T, int D>
__device__ __forceinline__ void norm_rope(float* x, const float* w, const float* cs,
                                          const float* sn, float eps, int c) {
  using S = Slice<T, D>;
  constexpr int LPK = D / 8;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss = fmaf(x[j], x[j], ss);
  ss = group_sum<LPK>(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  float y[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = S::round(__fmul_rn(__fmul_rn(x[j], r), w[j]));
  float partner[8];
  bool first_half[8];
  if constexpr (sizeof(T) == 2) {
    // Element 8c+j pairs with 8c+j +- D/2, held by lane c ^ (LPK/2).
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      partner[j] = __shfl_xor_sync(0xffffffffu, y[j], LPK / 2);
      first_half[j] = c < LPK / 2;
    }
  } else {
    // f32 slices hold 4c+j and D/2+4c+j in the same lane.
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      partner[j] = y[j ^ 4];
      first_half[j] = j < 4;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float rotated = first_half[j] ? -partner[j] : partner[j];
    const float a = S::round(__fmul_rn(y[j], cs[j]));
    const float b = S::round(__fmul_rn(rotated, sn[j]));
    x[j] = S::round(__fadd_rn(a, b));
  }
}

// Folds state (m2, l2, o2) into (m, l, o); m in log2 units, -inf = empty.
__device__ __forceinline__ void merge_state(float& m, float& l, float* o, float m2, float l2,
                                            const float* o2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  const float a = fast_exp2(m - mm);
  const float b = fast_exp2(m2 - mm);
  l = l * a + l2 * b;
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = o[j] * a + o2[j] * b;
  m = mm;
}

template <class C>
__global__ void __launch_bounds__(C::THREADS, C::MIN_BLOCKS)
    decode_attention_kernel(const __grid_constant__ DecodeParams p) {
  using T = typename C::T;
  constexpr int D = C::D, G = C::G, QPK = C::QPK, WPH = C::WPH, TP = C::TP;
  constexpr int STAGES = C::STAGES, MODE = C::MODE;
  using S = Slice<T, D>;
  constexpr int LPK = C::LPK, KPW = C::KPW, NP = C::NP, QH = C::QH;
  extern __shared__ __align__(128) uint8_t smem[];

  const int split = blockIdx.x;
  const int grp = blockIdx.y;
  const int b = blockIdx.z;  // query row (grouped prefix: token group)
  const bool prefix = p.tokens_per_row > 0;
  // Grouped prefix (Whisper prompt pass with QPK > 1): blockIdx.z is a group
  // of QPK consecutive tokens of one window, so every staged key serves QPK
  // queries. Query row qrow0 + qi is token tok0 + qi, present while below
  // tokens_per_row; absent ones compute on zeros and write nothing. Causal
  // self-attention reads keys 0 .. the group's last token and masks key k
  // for token tok0 + qi < k.
  constexpr bool kGrouped = MODE != kQwen3 && QPK > 1;
  static_assert(!kGrouped || G == 1, "token groups serve the Whisper prompt pass only");
  constexpr bool kCausalGroup = kGrouped && MODE == kWhisperSelf;
  int cb = b, tok0 = 0;  // cache row, first token
  int64_t qrow0 = b;
  if constexpr (kGrouped) {
    const int groups = (p.tokens_per_row + QPK - 1) / QPK;
    cb = b / groups;
    tok0 = (b % groups) * QPK;
    qrow0 = (int64_t)cb * p.tokens_per_row + tok0;
  } else if (prefix) {
    cb = b / p.tokens_per_row;
  }
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Launched with programmatic stream serialization: the CTA may be resident
  // before the previous kernel of the stream has finished, so it reads no
  // input (positions, caches, queries, workspace) before that kernel is done;
  // then the next launch may begin to be scheduled.
  // A split cluster's ready flags are cleared, and the cluster meets, before
  // anything can return: then any split may set its flag in split 0.
  uint32_t* xflag = reinterpret_cast<uint32_t*>(smem + C::OFF_XFLAG);
  // In a split cluster every thread also meets the cluster's exit barrier
  // exactly once before it returns: split 0's threads wait there, the others
  // only arrive. So split 0 stays resident until no other split can store
  // into its shared memory, even when its bounded wait for a flag gave up.
  const bool in_cluster = MODE == kQwen3 && p.cluster_splits != 0;
  if constexpr (MODE == kQwen3) {
    if (p.cluster_splits) {
      if (threadIdx.x < 8) xflag[threadIdx.x] = 0u;
      cluster_sync();
    }
  }

  griddep_wait();
  griddep_launch_dependents();

  // Qwen3: the consumer warps' inputs that do not depend on the row's
  // position (query, the step's own key/value, the norm weights) are loaded
  // first, together, so that their latencies overlap the position read, the
  // barrier set-up and each other. (The Whisper modes load their query and
  // key where they use them: hoisted, their launches took 1-3 % longer.)
  const int g = warp / WPH;   // head within the group
  const int wh = warp % WPH;  // warp within the head
  const int ks = lane / LPK;  // key slot within a warp pass
  const int c = lane % LPK;   // slice of the row
  const int kv_head = grp * G + g;
  float q[QPK][8];
  float own_k[8], own_v[8], wq[8], wk[8];
  if constexpr (MODE == kQwen3) {
    if (warp < C::CWARPS) {
      const T* row = static_cast<const T*>(p.qkv) + b * p.qkv_sb;
#pragma unroll
      for (int qi = 0; qi < QPK; ++qi) S::load_global_nc(row + (kv_head * QPK + qi) * D, c, q[qi]);
      S::load_global_nc(row + (p.q_heads + kv_head) * D, c, own_k);
      S::load_global_nc(row + (p.q_heads + p.kv_heads + kv_head) * D, c, own_v);
      S::load_global_nc(static_cast<const T*>(p.q_norm_w), c, wq);
      S::load_global_nc(static_cast<const T*>(p.k_norm_w), c, wk);
    }
  }

  // Keys of this row: n_cached read from the cache, plus (self/Qwen3 steps)
  // the step's own key at index `pos`.
  int pos = 0, n_cached, n_total;
  if constexpr (MODE == kWhisperCross) {
    n_cached = n_total = p.length;
  } else if (MODE == kWhisperSelf && prefix) {
    n_cached = n_total = kGrouped ? min(tok0 + QPK, p.tokens_per_row) : b % p.tokens_per_row + 1;
  } else {
    const int64_t given = p.positions[b];
    if (given < 0 || given >= p.length) {
      if (split == 0) {
        T* out = static_cast<T*>(p.out) + b * p.o_sb;
        for (int i = threadIdx.x; i < QH * D; i += C::THREADS) {
          const int h = grp * QH + i / D;
          out[h * p.o_sh + i % D] = T(0.f);
        }
        if (threadIdx.x == 0 && p.status) atomicOr(p.status, ASRBACK_STATUS_POSITION);
      }
      if (in_cluster) cluster_exit_arrive();
      return;
    }
    pos = static_cast<int>(given);
    n_cached = pos;
    n_total = pos + 1;
  }
  // This row's splits: at most p.num_splits, each at least p.chunk keys (but
  // one), the row's keys cut evenly into whole tiles, none left empty.
  int active = min(p.num_splits, (n_total + p.chunk - 1) / p.chunk);
  const int per = ((n_total + active - 1) / active + TP - 1) / TP * TP;
  active = (n_total + per - 1) / per;
  if (split >= active) {
    if (in_cluster) cluster_exit_arrive();
    return;
  }
  const int k0 = split * per;
  const int k1 = min(k0 + per, n_cached);
  const int n_tiles = k1 > k0 ? (k1 - k0 + TP - 1) / TP : 0;
  const bool has_own_key = MODE != kWhisperCross && !prefix && split == active - 1;
  const uint64_t deadline = global_timer_ns() + kWaitBudgetNs;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + STAGES;
  int* last_flag = reinterpret_cast<int*>(empty + STAGES);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::CWARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int64_t head0 = (int64_t)grp * G;
  const T* kbase = static_cast<const T*>(p.k_cache) + cb * p.c_sb + head0 * p.c_sh;
  const T* vbase = static_cast<const T*>(p.v_cache) + cb * p.c_sb + head0 * p.c_sh;

  if (warp == C::CWARPS) {
    // Producer warp. When a tile's rows are contiguous in the cache (each
    // position holds exactly this group's heads: Whisper, or Qwen3 with every
    // key/value head in one group), lane 0 moves it with one bulk copy per
    // tensor; otherwise each lane copies one position's slice of the group.
    const bool contiguous = p.c_sp == (int64_t)G * D;
    const uint64_t policy = l2_evict_first_policy();
    for (int t = 0; t < n_tiles; ++t) {
      const int s = t % STAGES;
      int ready = 1;
      if (t >= STAGES && lane == 0) ready = mbar_wait(&empty[s], ((t / STAGES) - 1) & 1, deadline);
      if (!__shfl_sync(0xffffffffu, ready, 0)) {
        if (lane == 0 && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
        break;
      }
      const int first = k0 + t * TP;
      const int rows = min(TP, k1 - first);
      if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(2 * rows * C::ROW_BYTES));
      __syncwarp();
      uint8_t* kdst = smem + C::OFF_K + s * C::TILE_BYTES;
      uint8_t* vdst = smem + C::OFF_V + s * C::TILE_BYTES;
      if (contiguous) {
        if (lane == 0) {
          const uint32_t bytes = static_cast<uint32_t>(rows * C::ROW_BYTES);
          bulk_g2s(kdst, kbase + first * p.c_sp, bytes, &full[s], policy);
          bulk_g2s(vdst, vbase + first * p.c_sp, bytes, &full[s], policy);
        }
      } else {
        for (int r = lane; r < rows; r += 32) {
          const int64_t off = (int64_t)(first + r) * p.c_sp;
          bulk_g2s(kdst + r * C::ROW_BYTES, kbase + off, C::ROW_BYTES, &full[s], policy);
          bulk_g2s(vdst + r * C::ROW_BYTES, vbase + off, C::ROW_BYTES, &full[s], policy);
        }
      }
    }
    if (in_cluster) cluster_exit_arrive();
    return;
  }

  // ---------------- consumers ----------------
  const bool owner = wh == 0 && ks == 0;  // lanes that hold the row's own key state

  float m[QPK], l[QPK], o[QPK][8];
#pragma unroll
  for (int qi = 0; qi < QPK; ++qi) {
    m[qi] = -INFINITY;
    l[qi] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[qi][j] = 0.f;
  }

  if constexpr (MODE == kQwen3) {
    float cs[8], sn[8];
    S::load_global_nc(static_cast<const T*>(p.cos) + pos * p.table_s, c, cs);
    S::load_global_nc(static_cast<const T*>(p.sin) + pos * p.table_s, c, sn);
#pragma unroll
    for (int qi = 0; qi < QPK; ++qi) norm_rope<T, D>(q[qi], wq, cs, sn, p.eps, c);
    if (has_own_key) norm_rope<T, D>(own_k, wk, cs, sn, p.eps, c);
  } else if constexpr (kGrouped) {
#pragma unroll
    for (int qi = 0; qi < QPK; ++qi) {
      if (tok0 + qi < p.tokens_per_row) {
        S::load_global_nc(static_cast<const T*>(p.q) + (qrow0 + qi) * p.q_sb +
                              (int64_t)kv_head * p.q_sh, c, q[qi]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) q[qi][j] = 0.f;
      }
    }
  } else {
    const T* qrow = static_cast<const T*>(p.q) + b * p.q_sb + (int64_t)kv_head * p.q_sh;
    S::load_global_nc(qrow, c, q[0]);
    if constexpr (MODE == kWhisperSelf) {
      if (has_own_key) {
        const int64_t off = b * p.kn_sb + (int64_t)kv_head * p.kn_sh;
        S::load_global_nc(static_cast<const T*>(p.k_new) + off, c, own_k);
        S::load_global_nc(static_cast<const T*>(p.v_new) + off, c, own_v);
      }
    }
  }
#pragma unroll
  for (int qi = 0; qi < QPK; ++qi)
#pragma unroll
    for (int j = 0; j < 8; ++j) q[qi][j] *= p.scale_log2;

  if constexpr (MODE != kWhisperCross) {
    if (has_own_key) {
      if (owner) {
        const int64_t off = cb * p.c_sb + (int64_t)kv_head * p.c_sh + (int64_t)pos * p.c_sp;
        S::store(static_cast<T*>(p.k_cache) + off, c, own_k);
        S::store(static_cast<T*>(p.v_cache) + off, c, own_v);
      }
#pragma unroll
      for (int qi = 0; qi < QPK; ++qi) {
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf(q[qi][j], own_k[j], dot);
        dot = group_sum<LPK>(dot);
        if (owner) {
          m[qi] = dot;
          l[qi] = 1.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) o[qi][j] = own_v[j];
        }
      }
    }
  }

  // Main loop over this split's tiles.
  bool timed_out = false;
  for (int t = 0; t < n_tiles; ++t) {
    const int s = t % STAGES;
    if (!mbar_wait(&full[s], (t / STAGES) & 1, deadline)) {
      timed_out = true;
      break;
    }
    const int rows = min(TP, k1 - (k0 + t * TP));
    const T* ktile = reinterpret_cast<const T*>(smem + C::OFF_K + s * C::TILE_BYTES);
    const T* vtile = reinterpret_cast<const T*>(smem + C::OFF_V + s * C::TILE_BYTES);
    float sc[QPK][NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      // Grouped causal prompt pass (a few keys per group): a pass wholly past
      // the tile's keys is skipped by the whole CTA, its scores masked. (In
      // the decode steps the same skip made the launches 3 % slower.)
      if constexpr (kCausalGroup) {
        if (i * (WPH * KPW) >= rows) {
#pragma unroll
          for (int qi = 0; qi < QPK; ++qi) sc[qi][i] = -INFINITY;
          continue;
        }
      }
      const int kt = wh * KPW + ks + i * (WPH * KPW);
      float kv[8];
      if (kt < rows) {
        S::load(ktile + (kt * G + g) * D, c, kv);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) kv[j] = 0.f;
      }
#pragma unroll
      for (int qi = 0; qi < QPK; ++qi) {
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf(q[qi][j], kv[j], dot);
        dot = group_sum<LPK>(dot);
        const bool seen = !kCausalGroup || k0 + t * TP + kt <= tok0 + qi;
        sc[qi][i] = kt < rows && seen ? dot : -INFINITY;
      }
    }
    float pr[QPK][NP];
#pragma unroll
    for (int qi = 0; qi < QPK; ++qi) {
      float mt = m[qi];
#pragma unroll
      for (int i = 0; i < NP; ++i) mt = fmaxf(mt, sc[qi][i]);
      const float base = mt == -INFINITY ? 0.f : mt;
      const float alpha = fast_exp2(m[qi] - base);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        pr[qi][i] = fast_exp2(sc[qi][i] - base);
        sum += pr[qi][i];
      }
      l[qi] = l[qi] * alpha + sum;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[qi][j] *= alpha;
      m[qi] = mt;
    }
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int kt = wh * KPW + ks + i * (WPH * KPW);
      if (kt < rows) {
        float vv[8];
        S::load(vtile + (kt * G + g) * D, c, vv);
#pragma unroll
        for (int qi = 0; qi < QPK; ++qi)
#pragma unroll
          for (int j = 0; j < 8; ++j) o[qi][j] = fmaf(pr[qi][i], vv[j], o[qi][j]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (timed_out && lane == 0 && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);

  // Merge the KPW key slots of the warp (lanes c, c+LPK, ...).
#pragma unroll
  for (int off = LPK; off < 32; off <<= 1) {
#pragma unroll
    for (int qi = 0; qi < QPK; ++qi) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m[qi], off);
      const float l2 = __shfl_xor_sync(0xffffffffu, l[qi], off);
      float o2[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o2[j] = __shfl_xor_sync(0xffffffffu, o[qi][j], off);
      merge_state(m[qi], l[qi], o[qi], m2, l2, o2);
    }
  }

  // Merge the WPH warps of each head through shared memory.
  if constexpr (WPH > 1) {
    float* merge = reinterpret_cast<float*>(smem + C::OFF_MERGE);
    // The slots may share the ring: every warp must be done with its tiles.
    if constexpr (C::SCRATCH_IN_RING) named_sync(1, C::CTHREADS);
    if (ks == 0) {
#pragma unroll
      for (int qi = 0; qi < QPK; ++qi) {
        float* slot = merge + (warp * QPK + qi) * (D + 2);
#pragma unroll
        for (int j = 0; j < 8; ++j) slot[S::elem(c, j)] = o[qi][j];
        if (c == 0) {
          slot[D] = m[qi];
          slot[D + 1] = l[qi];
        }
      }
    }
    named_sync(1, C::CTHREADS);
    if (wh == 0) {
      for (int w2 = 1; w2 < WPH; ++w2) {
#pragma unroll
        for (int qi = 0; qi < QPK; ++qi) {
          const float* slot = merge + ((g * WPH + w2) * QPK + qi) * (D + 2);
          float o2[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o2[j] = slot[S::elem(c, j)];
          merge_state(m[qi], l[qi], o[qi], slot[D], slot[D + 1], o2);
        }
      }
    }
  }

  T* out_row = static_cast<T*>(p.out) + b * p.o_sb;
  if (active == 1) {
    if (owner) {
#pragma unroll
      for (int qi = 0; qi < QPK; ++qi) {
        const float inv = 1.f / l[qi];
        float r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = o[qi][j] * inv;
        if constexpr (kGrouped) {
          if (tok0 + qi < p.tokens_per_row)
            S::store(static_cast<T*>(p.out) + (qrow0 + qi) * p.o_sb + (int64_t)kv_head * p.o_sh, c,
                     r);
        } else {
          S::store(out_row + (int64_t)(kv_head * QPK + qi) * p.o_sh, c, r);
        }
      }
    }
    if (in_cluster) cluster_exit_arrive();
    return;
  }

  // A split cluster: splits 1.. write their states into split 0's shared
  // memory and set their ready flags there (release); split 0 waits for the
  // flags of the row's active splits (acquire), folds the states into its own
  // and writes the output. No workspace, counter or global round trip. A
  // split past the row's active ones has already returned without touching
  // split 0, and split 0 stays until every active split has set its flag.
  if constexpr (MODE == kQwen3) {
    if (p.cluster_splits) {
      float* xfer = reinterpret_cast<float*>(smem + C::OFF_XFER);
      if (split > 0) {
        if (owner) {
#pragma unroll
          for (int qi = 0; qi < QPK; ++qi) {
            const uint32_t slot = cluster_map(
                smem_addr(xfer + ((split - 1) * QH + g * QPK + qi) * (D + 2)), 0);
#pragma unroll
            for (int j = 0; j < 8; ++j) st_cluster_f32(slot + 4 * S::elem(c, j), o[qi][j]);
            if (c == 0) {
              st_cluster_f32(slot + 4 * D, m[qi]);
              st_cluster_f32(slot + 4 * (D + 1), l[qi]);
            }
          }
          fence_cluster();
        }
        named_sync(1, C::CTHREADS);
        if (threadIdx.x == 0) st_release_cluster_u32(cluster_map(smem_addr(xflag + split), 0), 1u);
        cluster_exit_arrive();
        return;
      }
      if (owner) {
        // Two budgets: a split may itself have waited out one on its tiles.
        bool got = true;
        for (int s2 = 1; s2 < active && got; ++s2) {
          got = false;
          for (int attempt = 0; attempt < 2 && !got; ++attempt) {
            const uint64_t until = global_timer_ns() + kWaitBudgetNs;
            while (!(got = ld_acquire_cluster_u32(xflag + s2) != 0u) &&
                   global_timer_ns() < until) {
            }
          }
        }
        if (!got && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
#pragma unroll
        for (int qi = 0; qi < QPK; ++qi) {
          for (int s2 = 1; s2 < active && got; ++s2) {
            const float* slot = xfer + ((s2 - 1) * QH + g * QPK + qi) * (D + 2);
            float o2[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o2[j] = slot[S::elem(c, j)];
            merge_state(m[qi], l[qi], o[qi], slot[D], slot[D + 1], o2);
          }
          const float inv = 1.f / l[qi];
          float r[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) r[j] = o[qi][j] * inv;
          S::store(out_row + (int64_t)(kv_head * QPK + qi) * p.o_sh, c, r);
        }
      }
      cluster_exit_wait();
      return;
    }
  }

  // Several splits: publish this split's partial state, then the last CTA of
  // the (row, group) to arrive merges all of them.
  const int unit = b * p.groups + grp;
  float* part = p.partial + (size_t)unit * p.num_splits * QH * (D + 2);
  if (owner) {
#pragma unroll
    for (int qi = 0; qi < QPK; ++qi) {
      float* slot = part + ((size_t)split * QH + g * QPK + qi) * (D + 2);
#pragma unroll
      for (int j = 0; j < 8; ++j) slot[S::elem(c, j)] = o[qi][j];
      if (c == 0) {
        slot[D] = m[qi];
        slot[D + 1] = l[qi];
      }
    }
  }
  __threadfence();
  named_sync(1, C::CTHREADS);
  if (threadIdx.x == 0) {
    const int previous = atomicAdd(&p.counters[unit], 1);
    *last_flag = previous == active - 1;
  }
  named_sync(1, C::CTHREADS);
  if (!*last_flag) return;
  __threadfence();

  // The merge reads every split's (m, l) per head at once, one pair per
  // thread, into shared memory; then one thread per head forms the weights;
  // then each output element sums its splits with four loads in flight.
  float* weights = reinterpret_cast<float*>(smem + C::OFF_WEIGHTS);  // [QH][kMaxSplits]
  float* sums = weights + QH * kMaxSplits;                             // [QH][kMaxSplits]
  for (int i = threadIdx.x; i < QH * active; i += C::CTHREADS) {
    const int h = i / active, s = i - h * active;
    const float* slot = part + ((size_t)s * QH + h) * (D + 2);
    weights[h * kMaxSplits + s] = __ldcg(slot + D);
    sums[h * kMaxSplits + s] = __ldcg(slot + D + 1);
  }
  named_sync(1, C::CTHREADS);
  for (int h = threadIdx.x; h < QH; h += C::CTHREADS) {
    float* w = weights + h * kMaxSplits;
    const float* ls = sums + h * kMaxSplits;
    float mx = -INFINITY;
    for (int s = 0; s < active; ++s) mx = fmaxf(mx, w[s]);
    float den = 0.f;
    for (int s = 0; s < active; ++s) {
      const float e = w[s] == -INFINITY ? 0.f : fast_exp2(w[s] - mx);
      w[s] = e;
      den += e * ls[s];
    }
    const float inv = 1.f / den;
    for (int s = 0; s < active; ++s) w[s] *= inv;
  }
  named_sync(1, C::CTHREADS);
  const size_t split_step = (size_t)QH * (D + 2);
  for (int i = threadIdx.x; i < QH * D; i += C::CTHREADS) {
    const int h = i / D, d = i % D;
    const float* w = weights + h * kMaxSplits;
    const float* col = part + (size_t)h * (D + 2) + d;
    float acc = 0.f;
    int s = 0;
    for (; s + 4 <= active; s += 4) {
      const float v0 = __ldcg(col + (s + 0) * split_step);
      const float v1 = __ldcg(col + (s + 1) * split_step);
      const float v2 = __ldcg(col + (s + 2) * split_step);
      const float v3 = __ldcg(col + (s + 3) * split_step);
      acc = fmaf(w[s], v0, acc);
      acc = fmaf(w[s + 1], v1, acc);
      acc = fmaf(w[s + 2], v2, acc);
      acc = fmaf(w[s + 3], v3, acc);
    }
    for (; s < active; ++s) acc = fmaf(w[s], __ldcg(col + s * split_step), acc);
    if constexpr (kGrouped) {
      if (tok0 + h < p.tokens_per_row)
        static_cast<T*>(p.out)[(qrow0 + h) * p.o_sb + (int64_t)grp * p.o_sh + d] = T(acc);
    } else {
      out_row[(int64_t)(grp * QH + h) * p.o_sh + d] = T(acc);
    }
  }
  if (threadIdx.x == 0) p.counters[unit] = 0;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

// Workspace layout, the same for every entry point so that one zero-filled
// workspace serves them all: a fixed region of kCounterCap counters (one per
// (row, group) unit of a split call, zero between calls), then the partials of
// the current call. Calls that do not split use no workspace.
constexpr int kCounterCap = 16384;
constexpr size_t kCounterBytes = kCounterCap * sizeof(int);

size_t workspace_bytes_for(int units, int qh_per_unit, int head_dim, int splits) {
  if (splits <= 1) return 0;
  return kCounterBytes + (size_t)units * splits * qh_per_unit * (head_dim + 2) * sizeof(float);
}

// Points the call's counters and partials into `workspace` after checking it.
int bind_workspace(DecodeParams& p, int units, int qh_per_unit, int head_dim, void* workspace,
                   size_t have) {
  if (p.num_splits <= 1) return ASRBACK_OK;
  if (units > kCounterCap)
    return fail(ASRBACK_ERR_ARGUMENT, "%d split units exceed the workspace's %d counters", units,
                kCounterCap);
  const size_t need = workspace_bytes_for(units, qh_per_unit, head_dim, p.num_splits);
  if (need > have || workspace == nullptr)
    return fail(ASRBACK_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu needed", have,
                need);
  p.counters = static_cast<int*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  return ASRBACK_OK;
}

// Optional override of the keys per split (tuning sweeps; unset or 0 = the
// heuristic). Read at every call so that one process can sweep it.
int chunk_override() {
  const char* env = std::getenv("ASRBACK_SPLIT_CHUNK");
  return env ? std::atoi(env) : 0;
}

// Splits for `units` independent (row, group) units of at most `max_keys`
// keys: as many CTAs per unit as fill the GPU's resident slots once
// (`ctas_per_sm` per SM; a second partial wave would leave the first wave's
// SMs idle at the end), at most one per tile and kMaxSplits. `chunk` is the
// fewest keys a split takes (whole tiles, at least `granule_tiles`); the
// kernel cuts each row's own keys evenly between the splits it uses.
void choose_split(int units, int max_keys, int tile, int granule_tiles, int ctas_per_sm,
                  int* chunk, int* splits) {
  const int tiles = (max_keys + tile - 1) / tile;
  int want = 1;
  int chunk_tiles = granule_tiles;
  const int override_keys = chunk_override();
  if (override_keys > 0) {
    chunk_tiles = (override_keys + tile - 1) / tile;
    want = (tiles + chunk_tiles - 1) / chunk_tiles;
  } else {
    want = sm_count() * ctas_per_sm / units;
  }
  want = want < 1 ? 1 : want;
  want = want > tiles ? tiles : want;
  want = want > kMaxSplits ? kMaxSplits : want;
  chunk_tiles = chunk_tiles < 1 ? 1 : chunk_tiles;
  *chunk = chunk_tiles * tile;
  *splits = want;
}

// Kernel shape per call site and dtype: warps per key/value head, key
// positions per tile, ring stages. A tile is 16 KB (bf16 Whisper) or 32 KB
// (Qwen3) of keys, as much of values. The defaults come from sweeps on B200;
// a build may override them with -D for new sweeps.
#ifndef ASRBACK_SHAPE_WHISPER_SELF_BF16
#define ASRBACK_SHAPE_WHISPER_SELF_BF16 4, 64, 2
#endif
#ifndef ASRBACK_SHAPE_WHISPER_CROSS_BF16
#define ASRBACK_SHAPE_WHISPER_CROSS_BF16 8, 128, 2
#endif
#ifndef ASRBACK_SHAPE_WHISPER_F32
#define ASRBACK_SHAPE_WHISPER_F32 4, 32, 4
#endif
// Prompt-pass cross-attention with kPrefixTokens tokens per CTA.
#ifndef ASRBACK_SHAPE_WHISPER_PREFIX_BF16
#define ASRBACK_SHAPE_WHISPER_PREFIX_BF16 4, 64, 4
#endif
// Prompt-pass causal self-attention with kPrefixTokens tokens per CTA (keys:
// the prompt so far, a few tiles at most).
#ifndef ASRBACK_SHAPE_WHISPER_SELF_PREFIX_BF16
#define ASRBACK_SHAPE_WHISPER_SELF_PREFIX_BF16 1, 64, 2
#endif
constexpr int kPrefixTokens = 4;
// Qwen3: key/value heads per CTA (a divisor of 8), then the shape.
#ifndef ASRBACK_QWEN3_GROUP
#define ASRBACK_QWEN3_GROUP 8
#endif
// Three stages (192 KB of ring, one CTA per SM, as the grid holds at most one
// wave): batch 64 26.6 -> 25.2 us per launch; 32 and 16 rows unchanged.
#ifndef ASRBACK_SHAPE_QWEN3_BF16
#define ASRBACK_SHAPE_QWEN3_BF16 2, 16, 3
#endif
#ifndef ASRBACK_SHAPE_QWEN3_F32
#define ASRBACK_SHAPE_QWEN3_F32 1, 8, 3
#endif

using bf16 = __nv_bfloat16;
using WhisperSelfBf16 = DecodeConfig<bf16, 64, 1, 1, ASRBACK_SHAPE_WHISPER_SELF_BF16, kWhisperSelf>;
using WhisperSelfF32 = DecodeConfig<float, 64, 1, 1, ASRBACK_SHAPE_WHISPER_F32, kWhisperSelf>;
using WhisperCrossBf16 = DecodeConfig<bf16, 64, 1, 1, ASRBACK_SHAPE_WHISPER_CROSS_BF16, kWhisperCross>;
using WhisperCrossF32 = DecodeConfig<float, 64, 1, 1, ASRBACK_SHAPE_WHISPER_F32, kWhisperCross>;
using WhisperCrossPrefixBf16 =
    DecodeConfig<bf16, 64, 1, kPrefixTokens, ASRBACK_SHAPE_WHISPER_PREFIX_BF16, kWhisperCross>;
using WhisperSelfPrefixBf16 =
    DecodeConfig<bf16, 64, 1, kPrefixTokens, ASRBACK_SHAPE_WHISPER_SELF_PREFIX_BF16, kWhisperSelf>;
template <int QPK>
using Qwen3Bf16 = DecodeConfig<bf16, 128, ASRBACK_QWEN3_GROUP, QPK, ASRBACK_SHAPE_QWEN3_BF16, kQwen3>;
template <int QPK>
using Qwen3F32 = DecodeConfig<float, 128, ASRBACK_QWEN3_GROUP, QPK, ASRBACK_SHAPE_QWEN3_F32, kQwen3>;

// Splits `units` (row, group) units of at most p.length keys for config C.
// A Qwen3 split takes at least 64 positions (four 16-position tiles), so
// that a short row is not cut into splits whose merge costs more than their
// streaming saves.
template <class C>
constexpr int split_granule_tiles() {
  return C::MODE == kQwen3 ? (64 + C::TP - 1) / C::TP : 1;
}

// Splits for units that all hold `keys` keys (the grouped prompt pass): the
// launch takes ceil(units * s / resident) waves of CTAs that each stream 1/s
// of a unit's keys, plus a merge once the unit is split (counted as 1/10 of a
// unit's streaming). The s <= 8 with the least total is taken, the smallest on
// ties; the keys are cut into whole tiles.
void choose_split_waves(int units, int keys, int tile, int ctas_per_sm, int* chunk, int* splits) {
  const int64_t resident = (int64_t)sm_count() * ctas_per_sm;
  const int tiles = (keys + tile - 1) / tile;
  int best = 1;
  double best_cost = 0.0;
  for (int s = 1; s <= 8 && s <= tiles; ++s) {
    const int64_t waves = ((int64_t)units * s + resident - 1) / resident;
    const double cost = (double)waves / s + (s > 1 ? 0.1 : 0.0);
    if (s == 1 || cost < best_cost - 1e-9) {
      best = s;
      best_cost = cost;
    }
  }
  *splits = best;
  *chunk = (tiles + best - 1) / best * tile;
}

template <class C>
void split_for(DecodeParams& p, int units) {
  choose_split(units, p.length, C::TP, split_granule_tiles<C>(), C::MIN_BLOCKS, &p.chunk,
               &p.num_splits);
}

// Workspace bytes config C needs for `units` units of `qh` query heads.
template <class C>
size_t workspace_for(int units, int qh, int max_keys) {
  int chunk, splits;
  choose_split(units, max_keys, C::TP, split_granule_tiles<C>(), C::MIN_BLOCKS, &chunk, &splits);
  return workspace_bytes_for(units, qh, C::D, splits);
}

template <class C>
int launch(const DecodeParams& p, int batch, cudaStream_t stream) {
  auto kernel = decode_attention_kernel<C>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
            "cudaFuncSetAttribute(max dynamic shared memory)"))
      return rc;
    prepared_device = device;
  }
  return launch_pdl(kernel, dim3(p.num_splits, p.groups, batch), dim3(C::THREADS), C::SMEM, stream,
                    "decode attention launch", p);
}

// Splits, binds the workspace and launches config C.
template <class C>
int run(DecodeParams& p, int batch, int units, int qh_per_unit, void* workspace, size_t bytes,
        cudaStream_t stream) {
  split_for<C>(p, units);
  if (int rc = bind_workspace(p, units, qh_per_unit, C::D, workspace, bytes)) return rc;
  return launch<C>(p, batch, stream);
}

// Split clusters are on unless ASRBACK_SPLIT_PAIR=0 (A/B timing); read at
// every call so that one process can compare both.
bool pair_enabled() {
  const char* env = std::getenv("ASRBACK_SPLIT_PAIR");
  return !(env && env[0] == '0');
}

// Sets config C's dynamic shared-memory limit once per device.
template <class C>
int prepare_smem(int* device_out) {
  auto kernel = decode_attention_kernel<C>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
            "cudaFuncSetAttribute(max dynamic shared memory)"))
      return rc;
    prepared_device = device;
  }
  *device_out = device;
  return ASRBACK_OK;
}

// How many clusters of `size` CTAs of config C the device runs at once
// (cached per device and size; 0 if it cannot run one).
template <class C>
int active_clusters(int size) {
  static thread_local int cached_device = -1;
  static thread_local int cache[9];
  int device = 0;
  if (prepare_smem<C>(&device) != ASRBACK_OK) return 0;
  if (cached_device != device) {
    for (int& n : cache) n = -1;
    cached_device = device;
  }
  if (cache[size] < 0) {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(size, 1, 1);
    config.blockDim = dim3(C::THREADS);
    config.dynamicSmemBytes = C::SMEM;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = size;
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, decode_attention_kernel<C>, &config) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    cache[size] = n;
  }
  return cache[size];
}

// Launches config C with each row's splits as one cluster along x.
template <class C>
int launch_cluster(const DecodeParams& p, int batch, cudaStream_t stream) {
  int device = 0;
  if (int rc = prepare_smem<C>(&device)) return rc;
  return launch_pdl_cluster(decode_attention_kernel<C>, dim3(p.num_splits, p.groups, batch),
                            dim3(C::THREADS), C::SMEM, p.num_splits, stream,
                            "decode attention launch (split clusters)", p);
}

// Qwen3: one unit per (row, group of C::G key/value heads). When the
// heuristic cuts rows in 2 or 4 splits and all the clusters fit on the
// device at once, a row's splits run as one cluster (no workspace);
// otherwise, or with clusters off, the splits merge through the workspace.
// (Measured on B200, 28-layer graphs: clusters of 2 and 4 splits were
// faster than the workspace merge, 26.4 against 28.2 us at 64 rows and 18.9
// against 19.8 at 32; clusters of 3 and 8 slower, 25.4 against 23.4 at 48
// rows and 17.9 against 17.6 at 16.)
template <class C>
int run_qwen3(DecodeParams& p, int batch, void* workspace, size_t bytes, cudaStream_t stream) {
  static_assert(8 % C::G == 0, "key/value head groups must divide 8");
  p.groups = p.kv_heads / C::G;
  const int units = batch * p.groups;
  split_for<C>(p, units);
  if ((p.num_splits == 2 || p.num_splits == 4) && p.num_splits <= C::CLUSTER_MAX &&
      pair_enabled() && active_clusters<C>(p.num_splits) >= units) {
    p.cluster_splits = p.num_splits;
    return launch_cluster<C>(p, batch, stream);
  }
  if (int rc = bind_workspace(p, units, C::QH, C::D, workspace, bytes)) return rc;
  return launch<C>(p, batch, stream);
}

int check_dtype(int dtype) {
  if (dtype != ASRBACK_BF16 && dtype != ASRBACK_F32)
    return fail(ASRBACK_ERR_ARGUMENT, "dtype must be ASRBACK_BF16 or ASRBACK_F32, got %d", dtype);
  return ASRBACK_OK;
}

int check_strides_aligned(int dtype, std::initializer_list<int64_t> strides) {
  const int64_t elem = dtype == ASRBACK_BF16 ? 2 : 4;
  for (int64_t s : strides)
    if (s < 0 || (s * elem) % 16 != 0)
      return fail(ASRBACK_ERR_ARGUMENT, "every stride must be a non-negative multiple of 16 bytes");
  return ASRBACK_OK;
}

// The tensor-core prompt-pass cross-attention (prefix_cross_tc.cu), used for
// bf16 prompt passes of at most 128 tokens unless ASRBACK_PREFIX_TC=0 (A/B
// timing; read at every call so that one process can compare both).
constexpr int kPrefixTcMaxTokens = 128;
bool prefix_tc_enabled() {
  const char* env = std::getenv("ASRBACK_PREFIX_TC");
  return !(env && env[0] == '0');
}

int whisper_common(int dtype, int batch, int heads, int head_dim, int length, const void* query,
                   int64_t q_sb, int64_t q_sh, const void* kc, const void* vc, int64_t c_sb,
                   int64_t c_sh, const void* out, int64_t o_sb, int64_t o_sh) {
  if (int rc = check_dtype(dtype)) return rc;
  if (head_dim != 64)
    return fail(ASRBACK_ERR_ARGUMENT, "head_dim must be 64 (Whisper), got %d", head_dim);
  if (batch < 1 || heads < 1 || length < 1 || batch > 65535 || heads > 65535)
    return fail(ASRBACK_ERR_ARGUMENT, "batch, heads and length must be positive (got %d, %d, %d)",
                batch, heads, length);
  if (!query || !kc || !vc || !out) return fail(ASRBACK_ERR_ARGUMENT, "null tensor pointer");
  if (!aligned16(query) || !aligned16(kc) || !aligned16(vc) || !aligned16(out))
    return fail(ASRBACK_ERR_ARGUMENT, "tensor pointers must be 16-byte aligned");
  if (c_sh < (int64_t)length * head_dim || c_sb < (int64_t)heads * c_sh)
    return fail(ASRBACK_ERR_ARGUMENT,
                "cache strides (%lld, %lld) do not hold (heads=%d, length=%d, head_dim=%d) rows",
                (long long)c_sb, (long long)c_sh, heads, length, head_dim);
  return check_strides_aligned(dtype, {q_sb, q_sh, c_sb, c_sh, o_sb, o_sh});
}

}  // namespace

// Workspace bytes of the two prompt-pass calls for these sizes (the largest).
size_t prefix_workspace_bytes(int windows, int tokens, int heads, int head_dim, int length) {
  if (windows < 1 || tokens < 1 || heads < 1 || head_dim < 1 || length < 1) return 0;
  const int units = windows * tokens * heads;
  size_t need = 0;
  for (size_t n : {workspace_for<WhisperSelfBf16>(units, 1, tokens),
                   workspace_for<WhisperSelfF32>(units, 1, tokens),
                   workspace_for<WhisperCrossBf16>(units, 1, length),
                   workspace_for<WhisperCrossF32>(units, 1, length)})
    need = n > need ? n : need;
  if (tokens >= kPrefixTokens) {
    const int grouped = windows * ((tokens + kPrefixTokens - 1) / kPrefixTokens) * heads;
    const size_t self = workspace_for<WhisperSelfPrefixBf16>(grouped, kPrefixTokens, tokens);
    need = self > need ? self : need;
    int chunk, splits;
    choose_split_waves(grouped, length, WhisperCrossPrefixBf16::TP,
                       WhisperCrossPrefixBf16::MIN_BLOCKS, &chunk, &splits);
    const size_t n = workspace_bytes_for(grouped, kPrefixTokens, 64, splits);
    need = n > need ? n : need;
  }
  return need;
}

size_t decode_workspace_bytes(int batch, int heads, int head_dim, int max_keys) {
  if (batch < 1 || heads < 1 || head_dim < 1 || max_keys < 1) return 0;
  // Whisper: one unit per (row, head); Qwen3: one per row, all heads. The
  // largest need of any configuration that a call with these sizes may use.
  const int units = batch * heads;
  size_t need = 0;
  for (size_t n : {workspace_for<WhisperSelfBf16>(units, 1, max_keys),
                   workspace_for<WhisperSelfF32>(units, 1, max_keys),
                   workspace_for<WhisperCrossBf16>(units, 1, max_keys),
                   workspace_for<WhisperCrossF32>(units, 1, max_keys),
                   workspace_for<Qwen3Bf16<2>>(batch * (8 / Qwen3Bf16<2>::G), Qwen3Bf16<2>::QH, max_keys),
                   workspace_for<Qwen3F32<2>>(batch * (8 / Qwen3F32<2>::G), Qwen3F32<2>::QH, max_keys)})
    need = n > need ? n : need;
  return need;
}

}  // namespace asrback

using namespace asrback;

extern "C" {

size_t asrback_decode_workspace_bytes(int batch, int heads, int head_dim, int max_keys) {
  return decode_workspace_bytes(batch, heads, head_dim, max_keys);
}

size_t asrback_whisper_prefix_workspace_bytes(int windows, int tokens, int heads, int head_dim,
                                              int length) {
  return prefix_workspace_bytes(windows, tokens, heads, head_dim, length);
}

int asrback_whisper_self_attention_step(
    int dtype, int batch, int heads, int head_dim, int cache_length, const void* query,
    int64_t q_stride_batch, int64_t q_stride_head, const void* key, const void* value,
    int64_t kv_stride_batch, int64_t kv_stride_head, void* key_cache, void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head, const int64_t* positions, void* out,
    int64_t out_stride_batch, int64_t out_stride_head, float scale, void* workspace,
    size_t workspace_bytes, int32_t* status, void* stream) {
  if (int rc = whisper_common(dtype, batch, heads, head_dim, cache_length, query, q_stride_batch,
                              q_stride_head, key_cache, value_cache, cache_stride_batch,
                              cache_stride_head, out, out_stride_batch, out_stride_head))
    return rc;
  if (!key || !value || !positions || !aligned16(key) || !aligned16(value))
    return fail(ASRBACK_ERR_ARGUMENT, "key, value and positions must be non-null, 16-byte aligned");
  if (int rc = check_strides_aligned(dtype, {kv_stride_batch, kv_stride_head})) return rc;
  DecodeParams p{};
  p.q = query;
  p.q_sb = q_stride_batch;
  p.q_sh = q_stride_head;
  p.k_new = key;
  p.v_new = value;
  p.kn_sb = kv_stride_batch;
  p.kn_sh = kv_stride_head;
  p.k_cache = key_cache;
  p.v_cache = value_cache;
  p.c_sb = cache_stride_batch;
  p.c_sh = cache_stride_head;
  p.c_sp = head_dim;
  p.positions = positions;
  p.length = cache_length;
  p.out = out;
  p.o_sb = out_stride_batch;
  p.o_sh = out_stride_head;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.groups = heads;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int units = batch * heads;
  int rc = dtype == ASRBACK_BF16
               ? run<WhisperSelfBf16>(p, batch, units, 1, workspace, workspace_bytes, s)
               : run<WhisperSelfF32>(p, batch, units, 1, workspace, workspace_bytes, s);
  return rc ? rc : ok();
}

int asrback_whisper_self_attention_prefix(
    int dtype, int windows, int tokens, int heads, int head_dim, int cache_length,
    const void* query, int64_t q_stride_token, int64_t q_stride_head, const void* key_cache,
    const void* value_cache, int64_t cache_stride_batch, int64_t cache_stride_head, void* out,
    int64_t out_stride_token, int64_t out_stride_head, float scale, void* workspace,
    size_t workspace_bytes, int32_t* status, void* stream) {
  if (windows < 1 || tokens < 1 || (int64_t)windows * tokens > 65535)
    return fail(ASRBACK_ERR_ARGUMENT, "windows (%d) x tokens (%d) must be in [1, 65535]", windows,
                tokens);
  if (tokens > cache_length)
    return fail(ASRBACK_ERR_ARGUMENT, "tokens (%d) exceed the cache length (%d)", tokens,
                cache_length);
  if (int rc = whisper_common(dtype, windows, heads, head_dim, cache_length, query, q_stride_token,
                              q_stride_head, key_cache, value_cache, cache_stride_batch,
                              cache_stride_head, out, out_stride_token, out_stride_head))
    return rc;
  DecodeParams p{};
  p.q = query;
  p.q_sb = q_stride_token;
  p.q_sh = q_stride_head;
  p.k_cache = const_cast<void*>(key_cache);
  p.v_cache = const_cast<void*>(value_cache);
  p.c_sb = cache_stride_batch;
  p.c_sh = cache_stride_head;
  p.c_sp = head_dim;
  p.tokens_per_row = tokens;
  p.length = tokens;
  p.out = out;
  p.o_sb = out_stride_token;
  p.o_sh = out_stride_head;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.groups = heads;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (dtype == ASRBACK_BF16 && tokens >= kPrefixTokens) {
    // kPrefixTokens tokens of a window per CTA: a quarter of the CTAs, each
    // staged key serving the group's tokens that see it.
    const int rows = windows * ((tokens + kPrefixTokens - 1) / kPrefixTokens);
    rc = run<WhisperSelfPrefixBf16>(p, rows, rows * heads, kPrefixTokens, workspace,
                                    workspace_bytes, s);
  } else {
    const int rows = windows * tokens;
    const int units = rows * heads;
    rc = dtype == ASRBACK_BF16
             ? run<WhisperSelfBf16>(p, rows, units, 1, workspace, workspace_bytes, s)
             : run<WhisperSelfF32>(p, rows, units, 1, workspace, workspace_bytes, s);
  }
  return rc ? rc : ok();
}

int asrback_whisper_cross_attention_prefix(
    int dtype, int windows, int tokens, int heads, int head_dim, int length, const void* query,
    int64_t q_stride_token, int64_t q_stride_head, const void* key_cache, const void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head, void* out, int64_t out_stride_token,
    int64_t out_stride_head, float scale, void* workspace, size_t workspace_bytes,
    int32_t* status, void* stream) {
  if (windows < 1 || tokens < 1 || (int64_t)windows * tokens > 65535)
    return fail(ASRBACK_ERR_ARGUMENT, "windows (%d) x tokens (%d) must be in [1, 65535]", windows,
                tokens);
  if (int rc = whisper_common(dtype, windows, heads, head_dim, length, query, q_stride_token,
                              q_stride_head, key_cache, value_cache, cache_stride_batch,
                              cache_stride_head, out, out_stride_token, out_stride_head))
    return rc;
  DecodeParams p{};
  p.q = query;
  p.q_sb = q_stride_token;
  p.q_sh = q_stride_head;
  p.k_cache = const_cast<void*>(key_cache);
  p.v_cache = const_cast<void*>(value_cache);
  p.c_sb = cache_stride_batch;
  p.c_sh = cache_stride_head;
  p.c_sp = head_dim;
  p.tokens_per_row = tokens;
  p.length = length;
  p.out = out;
  p.o_sb = out_stride_token;
  p.o_sh = out_stride_head;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.groups = heads;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (dtype == ASRBACK_BF16 && tokens <= kPrefixTcMaxTokens && prefix_tc_enabled()) {
    rc = whisper_cross_prefix_tc(windows, tokens, heads, length, query, q_stride_token,
                                 q_stride_head, key_cache, value_cache, cache_stride_batch,
                                 cache_stride_head, out, out_stride_token, out_stride_head, scale,
                                 status, s);
  } else if (dtype == ASRBACK_BF16 && tokens >= kPrefixTokens) {
    // kPrefixTokens tokens of a window per CTA: each staged key serves them all.
    using C = WhisperCrossPrefixBf16;
    const int rows = windows * ((tokens + kPrefixTokens - 1) / kPrefixTokens);
    const int units = rows * heads;
    choose_split_waves(units, length, C::TP, C::MIN_BLOCKS, &p.chunk, &p.num_splits);
    rc = bind_workspace(p, units, kPrefixTokens, C::D, workspace, workspace_bytes);
    if (!rc) rc = launch<C>(p, rows, s);
  } else {
    const int rows = windows * tokens;
    const int units = rows * heads;
    rc = dtype == ASRBACK_BF16
             ? run<WhisperCrossBf16>(p, rows, units, 1, workspace, workspace_bytes, s)
             : run<WhisperCrossF32>(p, rows, units, 1, workspace, workspace_bytes, s);
  }
  return rc ? rc : ok();
}

int asrback_whisper_cross_attention_step(int dtype, int batch, int heads, int head_dim, int length,
                                         const void* query, int64_t q_stride_batch,
                                         int64_t q_stride_head, const void* key_cache,
                                         const void* value_cache, int64_t cache_stride_batch,
                                         int64_t cache_stride_head, void* out,
                                         int64_t out_stride_batch, int64_t out_stride_head,
                                         float scale, void* workspace, size_t workspace_bytes,
                                         int32_t* status, void* stream) {
  if (int rc = whisper_common(dtype, batch, heads, head_dim, length, query, q_stride_batch,
                              q_stride_head, key_cache, value_cache, cache_stride_batch,
                              cache_stride_head, out, out_stride_batch, out_stride_head))
    return rc;
  DecodeParams p{};
  p.q = query;
  p.q_sb = q_stride_batch;
  p.q_sh = q_stride_head;
  p.k_cache = const_cast<void*>(key_cache);
  p.v_cache = const_cast<void*>(value_cache);
  p.c_sb = cache_stride_batch;
  p.c_sh = cache_stride_head;
  p.c_sp = head_dim;
  p.length = length;
  p.out = out;
  p.o_sb = out_stride_batch;
  p.o_sh = out_stride_head;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.groups = heads;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int units = batch * heads;
  int rc = dtype == ASRBACK_BF16
               ? run<WhisperCrossBf16>(p, batch, units, 1, workspace, workspace_bytes, s)
               : run<WhisperCrossF32>(p, batch, units, 1, workspace, workspace_bytes, s);
  return rc ? rc : ok();
}

int asrback_qwen3_attention_step(int dtype, int batch, int heads, int kv_heads, int head_dim,
                                 int cache_length, const void* qkv, int64_t qkv_stride_batch,
                                 const void* q_norm_weight, const void* k_norm_weight, float eps,
                                 const void* cos, const void* sin, int64_t table_stride,
                                 int table_length, const int64_t* positions, void* key_cache,
                                 void* value_cache, int64_t cache_stride_batch, void* out,
                                 int64_t out_stride_batch, float scale, void* workspace,
                                 size_t workspace_bytes, int32_t* status, void* stream) {
  if (int rc = check_dtype(dtype)) return rc;
  if (head_dim != 128 || kv_heads != 8 || (heads != 8 && heads != 16))
    return fail(ASRBACK_ERR_ARGUMENT,
                "Qwen3 attention supports head_dim 128, 8 key/value heads and 8 or 16 query heads "
                "(got %d, %d, %d)",
                head_dim, kv_heads, heads);
  if (batch < 1 || batch > 65535 || cache_length < 1)
    return fail(ASRBACK_ERR_ARGUMENT, "batch and cache_length must be positive");
  if (table_length < cache_length)
    return fail(ASRBACK_ERR_ARGUMENT, "RoPE tables have %d rows, fewer than the cache's %d",
                table_length, cache_length);
  if (!qkv || !q_norm_weight || !k_norm_weight || !cos || !sin || !positions || !key_cache ||
      !value_cache || !out)
    return fail(ASRBACK_ERR_ARGUMENT, "null tensor pointer");
  for (const void* ptr : {qkv, q_norm_weight, k_norm_weight, cos, sin, (const void*)key_cache,
                          (const void*)value_cache, (const void*)out})
    if (!aligned16(ptr)) return fail(ASRBACK_ERR_ARGUMENT, "tensor pointers must be 16-byte aligned");
  if (cache_stride_batch < (int64_t)cache_length * kv_heads * head_dim)
    return fail(ASRBACK_ERR_ARGUMENT, "cache batch stride %lld is smaller than a row (%lld)",
                (long long)cache_stride_batch, (long long)cache_length * kv_heads * head_dim);
  if (qkv_stride_batch < (int64_t)(heads + 2 * kv_heads) * head_dim ||
      out_stride_batch < (int64_t)heads * head_dim || table_stride < head_dim)
    return fail(ASRBACK_ERR_ARGUMENT, "qkv, out or table row stride is smaller than a row");
  if (int rc = check_strides_aligned(dtype, {qkv_stride_batch, cache_stride_batch, out_stride_batch,
                                             table_stride}))
    return rc;
  DecodeParams p{};
  p.qkv = qkv;
  p.qkv_sb = qkv_stride_batch;
  p.q_norm_w = q_norm_weight;
  p.k_norm_w = k_norm_weight;
  p.eps = eps;
  p.cos = cos;
  p.sin = sin;
  p.table_s = table_stride;
  p.q_heads = heads;
  p.kv_heads = kv_heads;
  p.k_cache = key_cache;
  p.v_cache = value_cache;
  p.c_sb = cache_stride_batch;
  p.c_sh = head_dim;
  p.c_sp = (int64_t)kv_heads * head_dim;
  p.positions = positions;
  p.length = cache_length;
  p.out = out;
  p.o_sb = out_stride_batch;
  p.o_sh = head_dim;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == ASRBACK_BF16;
  int rc;
  if (heads == 16)
    rc = bf ? run_qwen3<Qwen3Bf16<2>>(p, batch, workspace, workspace_bytes, s)
            : run_qwen3<Qwen3F32<2>>(p, batch, workspace, workspace_bytes, s);
  else
    rc = bf ? run_qwen3<Qwen3Bf16<1>>(p, batch, workspace, workspace_bytes, s)
            : run_qwen3<Qwen3F32<1>>(p, batch, workspace, workspace_bytes, s);
  return rc ? rc : ok();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Cross-attention step that allocates nothing
// ---------------------------------------------------------------------------
//
// Some callers cannot hand this library a workspace: a host that binds the C
// ABI from another language (Go, Java, Rust) often has no device allocator of
// its own, and a serving loop must not call cudaMalloc per request because it
// synchronizes the whole device and stalls every other stream of the process.
// For them this entry point keeps its split-KV scratch (completion counters,
// then partial results) in a file-scope device array instead.

namespace asrback {
namespace {

// 1 MiB per device that loads the library, held until the process exits:
// room for kNoallocCounters split (row, head) units and their partials. The
// split heuristic needs at most ~0.5 MiB for any batch of Whisper heads.
constexpr int kNoallocCounters = 4096;
constexpr size_t kNoallocScratchBytes = size_t(1) << 20;
constexpr size_t kNoallocCounterBytes = kNoallocCounters * sizeof(int);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// Device address of g_noalloc_scratch on the current device. The lookup runs
// once per device (with that device current) and is cached; on a host, the
// name g_noalloc_scratch is only a stand-in for the device symbol, never an
// address a kernel may be given.
int noalloc_scratch(void** out) {
  static std::mutex lock;
  static void* addresses[64] = {nullptr};
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (device < 0 || device >= 64) return fail(ASRBACK_ERR_ARGUMENT, "device %d out of range", device);
  std::lock_guard<std::mutex> guard(lock);
  if (addresses[device] == nullptr) {
    void* ptr = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&ptr, g_noalloc_scratch),
                            "cudaGetSymbolAddress(no-allocation scratch)"))
      return rc;
    addresses[device] = ptr;
  }
  *out = addresses[device];
  return ASRBACK_OK;
}

}  // namespace
}  // namespace asrback

extern "C" int asrback_whisper_cross_attention_step_noalloc(
    int dtype, int batch, int heads, int head_dim, int length, const void* query,
    int64_t q_stride_batch, int64_t q_stride_head, const void* key_cache, const void* value_cache,
    int64_t cache_stride_batch, int64_t cache_stride_head, void* out, int64_t out_stride_batch,
    int64_t out_stride_head, float scale, int32_t* status, void* stream) {
  if (int rc = whisper_common(dtype, batch, heads, head_dim, length, query, q_stride_batch,
                              q_stride_head, key_cache, value_cache, cache_stride_batch,
                              cache_stride_head, out, out_stride_batch, out_stride_head))
    return rc;
  // Set-up on the first call on each device: the scratch's device address.
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  DecodeParams p{};
  p.q = query;
  p.q_sb = q_stride_batch;
  p.q_sh = q_stride_head;
  p.k_cache = const_cast<void*>(key_cache);
  p.v_cache = const_cast<void*>(value_cache);
  p.c_sb = cache_stride_batch;
  p.c_sh = cache_stride_head;
  p.c_sp = head_dim;
  p.length = length;
  p.out = out;
  p.o_sb = out_stride_batch;
  p.o_sh = out_stride_head;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.groups = heads;
  p.status = status;
  if (dtype == ASRBACK_BF16)
    split_for<WhisperCrossBf16>(p, batch * heads);
  else
    split_for<WhisperCrossF32>(p, batch * heads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.num_splits > 1) {
    const int units = batch * heads;
    const size_t partial_bytes =
        (size_t)units * p.num_splits * (head_dim + 2) * sizeof(float);
    if (units > kNoallocCounters || partial_bytes > kNoallocScratchBytes - kNoallocCounterBytes)
      return fail(ASRBACK_ERR_ARGUMENT,
                  "this call splits %d (row, head) units %d ways and needs %zu bytes of scratch; "
                  "the no-allocation entry point holds %d units and %zu bytes (use "
                  "asrback_whisper_cross_attention_step with a workspace instead)",
                  units, p.num_splits, partial_bytes + kNoallocCounterBytes, kNoallocCounters,
                  kNoallocScratchBytes);
    // The array keeps the previous call's contents: the counters must start at zero.
    if (int rc = check_cuda(cudaMemsetAsync(scratch, 0, units * sizeof(int), s),
                            "cudaMemsetAsync(no-allocation counters)"))
      return rc;
    p.counters = static_cast<int*>(scratch);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(scratch) + kNoallocCounterBytes);
  }
  int rc = dtype == ASRBACK_BF16 ? launch<WhisperCrossBf16>(p, batch, s)
                                 : launch<WhisperCrossF32>(p, batch, s);
  return rc ? rc : ok();
}
