// Greedy step epilogue: logits = weight . hidden^T, the greedy `_choose`
// (argmax, log_softmax at the argmax) and the decode-state update, in one
// launch. Replaces, for steps without sampling (temperatures None):
//   - whisper.py:949-960 (Transcriber._step after decode: `logits`
//     whisper.py:337-342 with the tied embedding, `_choose` :962-975 with the
//     suppress mask, the state update);
//   - qwen3_asr.py:1189-1201 (`_lm_head`, `_choose` :1203-1213, the state
//     update with several EOS ids).
//
// bf16 (the GPU path): logits on the tensor cores. A tile is 128 vocabulary
// rows (M) x the batch rows (N = 64 or 128, rows past the batch read as
// zeros) x the hidden width in 64-element chunks (K), accumulated in TMEM.
// Warp 0 streams the weight (TMA, evict-first: it is read once) and the
// hidden rows (evict-last: every CTA re-reads them) through a shared-memory
// ring; warp 1 issues the MMAs into two TMEM accumulators; warps 4-7 take a
// finished accumulator (thread = vocabulary row), round each logit to bf16 as
// the reference's bf16 matmul output is, apply the suppress mask, transpose
// the tile through shared memory and fold each batch column into a running
// (max, first argmax, sum of exp(x - max)). The dominant cost is reading the
// weight once: an HBM-bound GEMV-like GEMM.
// float32: one warp per vocabulary row (SIMT), the same running reduction.
//
// Each CTA writes its per-row partials; the last CTA to finish (a ticket
// counter in the workspace, left at zero afterwards) merges them in CTA
// order and applies the state update:
//   token = first index of the maximum; logprob = -ln(sum exp(x - max));
//   finished rows keep token and position; active rows advance;
//   sum_logprobs += logprob (active rows); generated[row, position] = token;
//   finished |= token in eos_ids | position >= end.
#include <algorithm>

#include "capi_internal.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace asrback {
namespace {

using namespace tc;

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kVocabTile = 128;  // vocabulary rows per tile (= TMEM lanes)
constexpr int kChunk = 64;       // hidden elements per K chunk (128 bytes of bf16)
constexpr int kMaxEos = 8;
constexpr int kNoIndex = 0x7fffffff;
constexpr int kSimtWarps = 8;
constexpr int kSimtMaxBatch = 64;
// Workspace: a 256-byte header of tickets (the final one, then one per group
// of CTAs in the tensor-core kernel), then the partials: one per (CTA, row),
// then (tensor-core kernel) one per (group, row).
constexpr int kWorkspaceHeader = 256;

struct Partial {
  float m;  // largest logit seen
  float s;  // sum of exp(x - m)
  int idx;  // first index holding m
  int pad;
};

// Running (max, first argmax, sum of exp(x - max)) of a logit stream.
struct Running {
  float m, s;
  int idx;
  __device__ __forceinline__ void init() {
    m = -INFINITY;
    s = 0.f;
    idx = kNoIndex;
  }
  // Logit x at index i; indices arrive in increasing order.
  __device__ __forceinline__ void push(float x, int i) {
    if (x > m) {
      s = s * fast_exp2((m - x) * kLog2e) + 1.f;
      m = x;
      idx = i;
    } else if (x > -INFINITY) {
      s += fast_exp2((x - m) * kLog2e);
    }
  }
  // Another stream's summary (any index order; ties go to the lower index).
  __device__ __forceinline__ void merge(float m2, float s2, int i2) {
    if (m2 == -INFINITY) return;
    if (m2 > m || (m2 == m && i2 < idx)) {
      s = s * fast_exp2((m - m2) * kLog2e) + s2;
      m = m2;
      idx = i2;
    } else {
      s += s2 * fast_exp2((m2 - m) * kLog2e);
    }
  }
};

struct StepParams {
  int batch;
  int vocab;
  const uint8_t* suppress;  // vocab flags (nonzero: never chosen), or null
  Partial* partials;        // [gridDim.x][batch]
  unsigned* ticket;
  int64_t* out_token;       // (batch,), or null
  float* out_logprob;       // (batch,), or null
  // Decode state; tokens null: no update.
  int64_t* tokens;
  int64_t tokens_stride;
  int64_t* position;
  const int64_t* end;
  uint8_t* finished;
  float* sum_logprobs;
  int64_t* generated;
  int64_t generated_stride;
  int64_t generated_cols;
  int n_eos;
  int64_t eos[kMaxEos];
  int32_t* status;
};

// Takes this CTA's ticket (one thread, after the CTA's partials are written
// and fenced); true for the last CTA to finish, which also resets the counter
// for the next launch (every CTA of this one has drawn its ticket).
__device__ __forceinline__ bool take_ticket(const StepParams& p) {
  const bool last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
  if (last) *p.ticket = 0u;
  return last;
}

// The tensor-core kernel merges in two levels. Its CTAs form groups of
// kGroupCtas; each group counts on its own ticket (p.ticket[1 + group]),
// which its last CTA resets. True for that last CTA.
constexpr int kGroupCtas = 16;
__device__ __forceinline__ bool take_group_ticket(const StepParams& p) {
  const int group = blockIdx.x / kGroupCtas;
  const int size = min(kGroupCtas, (int)gridDim.x - group * kGroupCtas);
  unsigned* counter = p.ticket + 1 + group;
  const bool last = atomicAdd(counter, 1u) == static_cast<unsigned>(size - 1);
  if (last) *counter = 0u;
  return last;
}

// Lanes per row in a merge over `nthreads` threads: R (a power of two, at
// most 32, adjacent lanes) share a row.
__device__ __forceinline__ int lanes_per_row(int batch, int nthreads) {
  int R = 32;
  while (R > 1 && R * batch > nthreads) R >>= 1;
  return R;
}

// Row b's summary over the partials src[c * batch + b], c < parts: each of the
// row's R lanes (j = its index) merges every R-th one, loading 20 at a time so
// that the loads overlap, then the R combine through shuffles. Every lane of
// the warp takes part (rows past the batch merge nothing).
__device__ __forceinline__ Running merge_row(const Partial* src, int parts, int batch, int b, int j,
                                             int R) {
  constexpr int kUnroll = 20;
  Running r;
  r.init();
  if (b < batch) {
    for (int c0 = j; c0 < parts; c0 += kUnroll * R) {
      float4 q[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * R;
        q[u] = c < parts ? __ldcg(reinterpret_cast<const float4*>(src + c * batch + b))
                         : make_float4(-INFINITY, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) r.merge(q[u].x, q[u].y, __float_as_int(q[u].z));
    }
  }
  for (int o = 1; o < R; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, r.m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, r.s, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, r.idx, o);
    r.merge(m2, s2, i2);
  }
  return r;
}

// Merges `parts` partials per row from src into one per row in dst (a group
// of CTAs' partials into the group's). All `nthreads` threads call it.
__device__ void merge_rows(const Partial* src, int parts, Partial* dst, int batch, int tid,
                           int nthreads) {
  const int R = lanes_per_row(batch, nthreads);
  const int j = tid % R;
  for (int base = 0; base < batch; base += nthreads / R) {
    const int b = base + tid / R;
    const Running r = merge_row(src, parts, batch, b, j, R);
    if (b < batch && j == 0) dst[b] = Partial{r.m, r.s, r.idx, 0};
  }
}

// The last merge: `parts` partials per row from src, then each row's token,
// log-probability and decode-state update. All `nthreads` (a multiple of 32)
// threads of the CTA call it. The thread that updates a row loads the row's
// decode state first, so that those loads overlap the partials'.
__device__ void finish_rows(const StepParams& p, const Partial* src, int parts, int tid,
                            int nthreads) {
  const int R = lanes_per_row(p.batch, nthreads);
  const int rows_per_pass = nthreads / R;
  const int j = tid % R;
  for (int base = 0; base < p.batch; base += rows_per_pass) {
    const int b = base + tid / R;
    const bool updates = b < p.batch && j == 0 && p.tokens;
    bool done = false;
    int64_t position = 0, end = 0, old_token = 0;
    float sum = 0.f;
    if (updates) {
      done = p.finished[b] != 0;
      position = p.position[b];
      end = p.end[b];
      old_token = p.tokens[b * p.tokens_stride];
      sum = p.sum_logprobs[b];
    }
    const Running r = merge_row(src, parts, p.batch, b, j, R);
    if (b >= p.batch || j != 0) continue;
    // torch's argmax of a row that is all -inf is its first index.
    const int64_t token = r.idx == kNoIndex ? 0 : r.idx;
    const float logprob = r.m == -INFINITY ? __int_as_float(0x7fc00000) : -logf(r.s);
    if (p.out_token) p.out_token[b] = token;
    if (p.out_logprob) p.out_logprob[b] = logprob;
    if (updates) {
      const int64_t pos = position + (done ? 0 : 1);
      const int64_t tok = done ? old_token : token;
      if (!done) p.sum_logprobs[b] = sum + logprob;
      bool eos = false;
      for (int e = 0; e < p.n_eos; ++e) eos |= tok == p.eos[e];
      if (pos >= 0 && pos < p.generated_cols) {
        p.generated[b * p.generated_stride + pos] = tok;
      } else if (p.status) {
        atomicOr(p.status, ASRBACK_STATUS_POSITION);
      }
      p.finished[b] = done || eos || pos >= end;
      p.position[b] = pos;
      p.tokens[b * p.tokens_stride] = tok;
    }
  }
}

// ------------------------------------------------------------ bf16, tcgen05

template <int kN>
struct TcShape {
  static constexpr int kWBytes = kVocabTile * 128;  // 128 rows x 64 bf16
  static constexpr int kHBytes = kN * 128;          // kN rows x 64 bf16
  static constexpr int kStageBytes = kWBytes + kHBytes;
  static constexpr int kStages = kN == 64 ? 7 : 4;
  static constexpr int kOffT = kStages * kStageBytes;  // logits tile, [128][kN + 1] f32
  static constexpr int kOffRed = kOffT + kVocabTile * (kN + 1) * 4;
  static constexpr int kOffBar = kOffRed + kVocabTile * static_cast<int>(sizeof(Partial));
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;  // TMEM slot, last-CTA flag
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory exceeds a CTA's 227 KB");
};

template <int kN>
__global__ void __launch_bounds__(256, 1)
    greedy_step_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                          const __grid_constant__ CUtensorMap map_h, const int hidden_dim,
                          const __grid_constant__ StepParams p) {
  using Sh = TcShape<kN>;
  constexpr int S = Sh::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Sh::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Sh::kOffMisc);
  int* last_flag = reinterpret_cast<int*>(smem + Sh::kOffMisc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.vocab + kVocabTile - 1) / kVocabTile;
  const int chunks = (hidden_dim + kChunk - 1) / kChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool timed_out = false;

  // The TMA and MMA warps run their loops warp-wide (waits by every lane, the
  // loop state warp-uniform) and issue from one elected lane.
  auto wait_warp = [](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
  };
  // One lane per warp, elected once: a tcgen05.commit tracks the MMAs of its
  // own thread, so the MMA warp's issues and commits all come from it.
  const bool leader = elect_one();
  if (warp == 0) {
    // ---------------- TMA: weight tile and hidden rows per K chunk ----------------
    if (leader) {
      prefetch_tensormap(&map_w);
      prefetch_tensormap(&map_h);
    }
    __syncwarp();
    const uint64_t stream = l2_evict_first_policy();
    const uint64_t keep = l2_evict_last_policy();
    int g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      for (int kc = 0; kc < chunks; ++kc, ++g) {
        const int s = g % S;
        if (g >= S) ok = wait_warp(&empty[s], ((g / S) - 1) & 1);
        if (!ok) break;
        if (leader) {
          uint8_t* stage = smem + s * Sh::kStageBytes;
          mbar_arrive_expect_tx(&full[s], Sh::kStageBytes);
          tma_load_2d_hint(stage, &map_w, kc * kChunk, tile * kVocabTile, &full[s], stream);
          tma_load_2d_hint(stage + Sh::kWBytes, &map_h, kc * kChunk, 0, &full[s], keep);
        }
        __syncwarp();
      }
    }
    timed_out = !ok;
  } else if (warp == 1) {
    // ---------------- MMA: D[vocab row][batch row] in TMEM ----------------
    constexpr uint32_t kIdesc = idesc_bf16(kVocabTile, kN, false);
    const uint64_t w_desc = sw128_desc(smem_addr(smem), 16, 1024);
    const uint64_t h_desc = sw128_desc(smem_addr(smem + Sh::kWBytes), 16, 1024);
    constexpr uint64_t kStage = Sh::kStageBytes >> 4;
    int g = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++lt) {
      const int a = lt & 1;
      if (lt >= 2) ok = wait_warp(&acc_empty[a], ((lt >> 1) - 1) & 1);
      tc_fence_after();
      for (int kc = 0; kc < chunks && ok; ++kc, ++g) {
        const int s = g % S;
        ok = wait_warp(&full[s], (g / S) & 1);
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          // K = 64 in steps of 16: 32 bytes along the 128-byte swizzled row.
#pragma unroll
          for (int k = 0; k < kChunk / 16; ++k)
            mma_ss(tmem + a * kN, w_desc + s * kStage + 2 * k, h_desc + s * kStage + 2 * k, kIdesc,
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
    // ---------------- epilogue: bf16 logits, mask, column reductions ----------------
    const int tid = threadIdx.x - 128;  // = TMEM lane = vocabulary row within the tile
    const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float* tile_t = reinterpret_cast<float*>(smem + Sh::kOffT);
    Partial* red = reinterpret_cast<Partial*>(smem + Sh::kOffRed);
    constexpr int kParts = kVocabTile / kN;  // threads per batch column
    constexpr int kRowsPer = kVocabTile / kParts;
    const int col = tid % kN, part = tid / kN;
    Running run;
    run.init();
    bool ok = true;
    int lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int a = lt & 1;
      // Warp-uniform, since the TMEM reads below are warp-wide.
      ok = __all_sync(0xffffffffu, ok && mbar_spin_bounded(&acc_full[a], (lt >> 1) & 1));
      if (ok) {
        tc_fence_after();
        const int v = tile * kVocabTile + tid;
        const bool keep = v < p.vocab && !(p.suppress && p.suppress[v]);
#pragma unroll
        for (int h = 0; h < kN / 32; ++h) {
          float x[32];
          tmem_ld32(tmem + lane_bits + a * kN + 32 * h, x);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            tile_t[tid * (kN + 1) + 32 * h + i] =
                keep ? __bfloat162float(__float2bfloat16_rn(x[i])) : -INFINITY;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);
      }
      // Every thread takes every named barrier, whatever its `ok`, so that a
      // timed-out wait cannot leave the others at a barrier.
      named_sync(1, 128);
      Running loc;
      loc.init();
      if (ok) {
        for (int r = part * kRowsPer; r < (part + 1) * kRowsPer; ++r)
          loc.push(tile_t[r * (kN + 1) + col], tile * kVocabTile + r);
      }
      if (kParts > 1 && part > 0) red[tid] = Partial{loc.m, loc.s, loc.idx, 0};
      named_sync(1, 128);
      if (part == 0) {
        run.merge(loc.m, loc.s, loc.idx);
        for (int q = 1; q < kParts; ++q) {
          const Partial o = red[q * kN + col];
          run.merge(o.m, o.s, o.idx);
        }
      }
      named_sync(1, 128);  // the tile buffer is free again
    }
    if (!ok) timed_out = true;
    if (part == 0 && col < p.batch)
      p.partials[blockIdx.x * p.batch + col] = Partial{run.m, run.s, run.idx, 0};
    __threadfence();
    named_sync(1, 128);
    if (tid == 0) *last_flag = take_group_ticket(p);
  }
  if (timed_out && p.status) atomicOr(p.status, ASRBACK_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kN);
  }
  // Two-level merge: the last CTA of each group of kGroupCtas merges the
  // group's partials into one per row; the last group to finish merges those
  // and updates the state.
  if (*last_flag) {
    __threadfence();
    const int group = blockIdx.x / kGroupCtas;
    const int first = group * kGroupCtas;
    const int groups = (gridDim.x + kGroupCtas - 1) / kGroupCtas;
    Partial* group_partials = p.partials + gridDim.x * p.batch;
    merge_rows(p.partials + first * p.batch, min(kGroupCtas, (int)gridDim.x - first),
               group_partials + group * p.batch, p.batch, threadIdx.x, blockDim.x);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const bool last = atomicAdd(p.ticket, 1u) == static_cast<unsigned>(groups - 1);
      if (last) *p.ticket = 0u;
      *last_flag = last;
    }
    __syncthreads();
    if (*last_flag) {
      __threadfence();
      finish_rows(p, group_partials, groups, threadIdx.x, blockDim.x);
    }
  }
}

// ------------------------------------------------------------ float32, SIMT

__global__ void __launch_bounds__(kSimtWarps * 32)
    greedy_step_simt_kernel(const float* __restrict__ weight, int64_t w_stride,
                            const float* __restrict__ hidden, int64_t h_stride, int hidden_dim,
                            const __grid_constant__ StepParams p) {
  extern __shared__ float hs[];  // [batch][hidden_dim]
  __shared__ Partial red[kSimtWarps][kSimtMaxBatch];
  __shared__ int last_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < p.batch * hidden_dim; i += blockDim.x)
    hs[i] = hidden[(i / hidden_dim) * h_stride + i % hidden_dim];
  __syncthreads();
  Running run[2];  // columns lane and lane + 32
  run[0].init();
  run[1].init();
  for (int v = blockIdx.x * kSimtWarps + warp; v < p.vocab; v += gridDim.x * kSimtWarps) {
    float acc[kSimtMaxBatch];
#pragma unroll
    for (int b = 0; b < kSimtMaxBatch; ++b) acc[b] = 0.f;
    const float* row = weight + static_cast<int64_t>(v) * w_stride;
    for (int k = lane; k < hidden_dim; k += 32) {
      const float w = row[k];
#pragma unroll
      for (int b = 0; b < kSimtMaxBatch; ++b)
        if (b < p.batch) acc[b] = fmaf(w, hs[b * hidden_dim + k], acc[b]);
    }
    const bool masked = p.suppress && p.suppress[v];
#pragma unroll
    for (int b = 0; b < kSimtMaxBatch; ++b) {
      if (b >= p.batch) break;
      float x = acc[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == (b & 31)) run[b >> 5].push(masked ? -INFINITY : x, v);
    }
  }
  for (int h = 0; h < 2; ++h) {
    const int b = lane + 32 * h;
    if (b < p.batch) red[warp][b] = Partial{run[h].m, run[h].s, run[h].idx, 0};
  }
  __syncthreads();
  if (threadIdx.x < p.batch) {
    Running r;
    r.init();
    for (int w = 0; w < kSimtWarps; ++w) {
      const Partial q = red[w][threadIdx.x];
      r.merge(q.m, q.s, q.idx);
    }
    p.partials[blockIdx.x * p.batch + threadIdx.x] = Partial{r.m, r.s, r.idx, 0};
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_flag = take_ticket(p);
  __syncthreads();
  if (last_flag) {
    __threadfence();
    finish_rows(p, p.partials, gridDim.x, threadIdx.x, blockDim.x);
  }
}

int make_map_2d(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t stride,
                uint32_t box_rows) {
  int rc = ASRBACK_OK;
  auto encode = tensor_map_encoder(&rc);
  if (!encode) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kChunk, box_rows};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(ASRBACK_ERR_ARGUMENT, "cuTensorMapEncodeTiled rejected the layout (error %d)",
                (int)res);
  return ASRBACK_OK;
}

template <int kN>
int launch_tc(const void* hidden, int64_t h_stride, const void* weight, int64_t w_stride,
              int hidden_dim, const StepParams& p, cudaStream_t stream) {
  using Sh = TcShape<kN>;
  CUtensorMap mw, mh;
  if (int rc = make_map_2d(&mw, weight, hidden_dim, p.vocab, w_stride, kVocabTile)) return rc;
  if (int rc = make_map_2d(&mh, hidden, hidden_dim, p.batch, h_stride, kN)) return rc;
  auto kernel = greedy_step_tc_kernel<kN>;
  static thread_local int prepared_device = -1;
  int device = 0;
  if (int rc = check_cuda(cudaGetDevice(&device), "cudaGetDevice")) return rc;
  if (prepared_device != device) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 Sh::kSmemBytes),
                            "cudaFuncSetAttribute(greedy step)"))
      return rc;
    prepared_device = device;
  }
  const int tiles = (p.vocab + kVocabTile - 1) / kVocabTile;
  const int ctas = std::min(tiles, sm_count());
  // One ticket per group of CTAs after the first in the workspace header.
  if (1 + (ctas + kGroupCtas - 1) / kGroupCtas > kWorkspaceHeader / (int)sizeof(unsigned))
    return fail(ASRBACK_ERR_ARGUMENT, "%d CTAs need more group tickets than the workspace holds",
                ctas);
  kernel<<<ctas, 256, Sh::kSmemBytes, stream>>>(mw, mh, hidden_dim, p);
  return check_cuda(cudaGetLastError(), "greedy step (tensor core) launch");
}

}  // namespace
}  // namespace asrback

using namespace asrback;

extern "C" size_t asrback_greedy_step_workspace_bytes(int batch) {
  if (batch < 1) return 0;
  return kWorkspaceHeader + static_cast<size_t>(2 * sm_count()) * batch * sizeof(Partial);
}

extern "C" int asrback_greedy_step(int dtype, int batch, int vocab, int hidden_dim,
                                   const void* hidden, int64_t hidden_stride, const void* weight,
                                   int64_t weight_stride, const uint8_t* suppress,
                                   int64_t* out_token, float* out_logprob, int64_t* tokens,
                                   int64_t tokens_stride, int64_t* position, const int64_t* end,
                                   uint8_t* finished, float* sum_logprobs, int64_t* generated,
                                   int64_t generated_stride, int64_t generated_cols,
                                   const int64_t* eos_ids, int n_eos, void* workspace,
                                   size_t workspace_bytes, int32_t* status, void* stream) {
  if (dtype != ASRBACK_BF16 && dtype != ASRBACK_F32)
    return fail(ASRBACK_ERR_ARGUMENT, "dtype must be ASRBACK_BF16 or ASRBACK_F32, got %d", dtype);
  const int max_batch = dtype == ASRBACK_BF16 ? 128 : kSimtMaxBatch;
  if (batch < 1 || batch > max_batch)
    return fail(ASRBACK_ERR_ARGUMENT, "batch must be in [1, %d], got %d", max_batch, batch);
  if (vocab < 1 || hidden_dim < 1)
    return fail(ASRBACK_ERR_ARGUMENT, "vocab and hidden_dim must be positive (got %d, %d)", vocab,
                hidden_dim);
  if (!hidden || !weight) return fail(ASRBACK_ERR_ARGUMENT, "null hidden or weight pointer");
  if (hidden_stride < hidden_dim || weight_stride < hidden_dim)
    return fail(ASRBACK_ERR_ARGUMENT, "row strides must be at least hidden_dim");
  if (dtype == ASRBACK_BF16) {
    if (hidden_dim % 8 != 0 || hidden_stride % 8 != 0 || weight_stride % 8 != 0 ||
        !aligned16(hidden) || !aligned16(weight))
      return fail(ASRBACK_ERR_ARGUMENT,
                  "bf16 rows must start on 16-byte boundaries: hidden_dim and strides multiples "
                  "of 8, pointers 16-byte aligned");
  } else if (static_cast<size_t>(batch) * hidden_dim * 4 > 200 * 1024) {
    return fail(ASRBACK_ERR_ARGUMENT, "float32: batch x hidden_dim must fit 200 KB of shared memory");
  }
  if (n_eos < 0 || n_eos > kMaxEos || (n_eos > 0 && !eos_ids))
    return fail(ASRBACK_ERR_ARGUMENT, "n_eos must be in [0, %d] with eos_ids given", kMaxEos);
  if (tokens && (!position || !end || !finished || !sum_logprobs || !generated ||
                 generated_cols < 1 || tokens_stride < 1 || generated_stride < generated_cols))
    return fail(ASRBACK_ERR_ARGUMENT, "state update needs position, end, finished, sum_logprobs "
                                      "and generated (generated_stride >= generated_cols >= 1)");
  if (!workspace) return fail(ASRBACK_ERR_ARGUMENT, "null workspace");
  if (workspace_bytes < asrback_greedy_step_workspace_bytes(batch))
    return fail(ASRBACK_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", workspace_bytes,
                asrback_greedy_step_workspace_bytes(batch));
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return fail(ASRBACK_ERR_ARGUMENT, "workspace must be 16-byte aligned");

  StepParams p{};
  p.batch = batch;
  p.vocab = vocab;
  p.suppress = suppress;
  p.ticket = static_cast<unsigned*>(workspace);
  p.partials = reinterpret_cast<Partial*>(static_cast<uint8_t*>(workspace) + kWorkspaceHeader);
  p.out_token = out_token;
  p.out_logprob = out_logprob;
  p.tokens = tokens;
  p.tokens_stride = tokens_stride;
  p.position = position;
  p.end = end;
  p.finished = finished;
  p.sum_logprobs = sum_logprobs;
  p.generated = generated;
  p.generated_stride = generated_stride;
  p.generated_cols = generated_cols;
  p.n_eos = n_eos;
  for (int e = 0; e < n_eos; ++e) p.eos[e] = eos_ids[e];
  p.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == ASRBACK_BF16) {
    const int rc = batch <= 64 ? launch_tc<64>(hidden, hidden_stride, weight, weight_stride,
                                               hidden_dim, p, s)
                               : launch_tc<128>(hidden, hidden_stride, weight, weight_stride,
                                                hidden_dim, p, s);
    return rc ? rc : ok();
  }
  const int ctas = std::min((vocab + kSimtWarps - 1) / kSimtWarps, 2 * sm_count());
  const size_t smem = static_cast<size_t>(batch) * hidden_dim * 4;
  if (int rc = check_cuda(cudaFuncSetAttribute(greedy_step_simt_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem)),
                          "cudaFuncSetAttribute(greedy step f32)"))
    return rc;
  greedy_step_simt_kernel<<<ctas, kSimtWarps * 32, smem, s>>>(
      static_cast<const float*>(weight), weight_stride, static_cast<const float*>(hidden),
      hidden_stride, hidden_dim, p);
  if (int rc = check_cuda(cudaGetLastError(), "greedy step (f32) launch")) return rc;
  return ok();
}
