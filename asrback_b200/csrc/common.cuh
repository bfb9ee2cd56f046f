// Device helpers shared by the asrback sm_100a kernels: mbarrier and bulk-copy
// (TMA engine) wrappers in inline PTX, bounded waits, programmatic dependent
// launch, packed f32x2 arithmetic, and bf16/f32 vector unpacking. Host helpers
// for the C ABI's error reporting live in capi.cu.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/asrback_attn.h"

namespace asrback {

// A wait inside a kernel gives up this long after the kernel's CTA started
// (nanoseconds of %globaltimer). No healthy wait comes near it; it only keeps a
// broken copy from hanging the GPU.
constexpr uint64_t kWaitBudgetNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking test: has the phase with `parity` completed?
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// ---- thread-block clusters: a split pair's partial crosses in shared memory ----

// Every thread of every CTA of the cluster arrives, then waits for all.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The cluster's exit barrier: a thread that will not touch another CTA's
// shared memory again arrives (release: its remote stores come first) and may
// then return without waiting.
__device__ __forceinline__ void cluster_exit_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}

// The exit barrier for a CTA whose shared memory others write: arrive, then
// wait until every thread of the cluster has arrived, so that no remote store
// can land after this CTA has returned.
__device__ __forceinline__ void cluster_exit_wait() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// This CTA's shared-memory address `addr` as seen in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void fence_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}

// Arrives, with release at cluster scope, on a barrier in another CTA of the
// cluster (address from cluster_map).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
               : "memory");
}

// Stores `v` with release at cluster scope into another CTA's shared memory
// (address from cluster_map): the writes before it are visible to a reader
// that acquires the value.
__device__ __forceinline__ void st_release_cluster_u32(uint32_t remote, uint32_t v) {
  asm volatile("st.release.cluster.shared::cluster.u32 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
}

// Loads this CTA's shared-memory word with acquire at cluster scope.
__device__ __forceinline__ uint32_t ld_acquire_cluster_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cluster.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
  return v;
}

// try_wait with acquire at cluster scope (the arrival came from another CTA).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with `parity` to complete, or until `deadline`
// (%globaltimer ns) has passed. Returns false on a timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline) {
  if (mbar_try_wait(bar, parity)) return true;
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0 && global_timer_ns() > deadline) return false;
  }
}

// As mbar_wait, with a budget of kWaitBudgetNs counted from the wait's own
// first slow poll: a wait that is already satisfied, or soon is, reads no
// timer (a %globaltimer read costs more than a satisfied try_wait).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t deadline = 0;
  for (uint32_t spins = 1;; ++spins) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spins & 63u) == 0) {
      const uint64_t now = global_timer_ns();
      if (deadline == 0) {
        deadline = now + kWaitBudgetNs;
      } else if (now > deadline) {
        return false;
      }
    }
  }
}

// As mbar_wait_bounded, polling with the non-suspending test (a hand-off
// between warps of one CTA, where a suspended waiter wakes late).
__device__ __forceinline__ bool mbar_spin_bounded(uint64_t* bar, uint32_t parity) {
  uint64_t deadline = 0;
  for (uint32_t spins = 1;; ++spins) {
    if (mbar_test(bar, parity)) return true;
    if ((spins & 255u) == 0) {
      const uint64_t now = global_timer_ns();
      if (deadline == 0) {
        deadline = now + kWaitBudgetNs;
      } else if (now > deadline) {
        return false;
      }
    }
  }
}

// As mbar_wait, polling with the non-suspending test (for hand-offs between
// warps of one CTA, where a suspended waiter would add wake-up latency).
__device__ __forceinline__ bool mbar_spin(uint64_t* bar, uint32_t parity, uint64_t deadline) {
  uint32_t spins = 0;
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if ((++spins & 255u) == 0 && global_timer_ns() > deadline) return false;
  }
}

// Programmatic dependent launch (a kernel launched with programmatic stream
// serialization may start before the previous kernel in its stream ends).
// griddep_wait blocks until that kernel has completed and its writes are
// visible; griddep_launch_dependents lets the next such kernel start once
// every CTA of this grid has issued it (or exited). Both are no-ops for a
// kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// L2 policy for data read once per step (the KV stream): evict first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// L2 policy for data every CTA re-reads (a small operand): evict last.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Bulk copy (TMA engine, untiled) of `bytes` from global to this CTA's shared
// memory, completing `bytes` of transaction count on `bar`. Both addresses
// 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Packed f32 pairs (low element first) and Blackwell's paired f32 FMA / add
// / multiply.
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Named barrier among `threads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// Eight-element lane slices. A lane owns eight elements of a head_dim row:
//   bf16: elements 8c .. 8c+7 (one 16-byte vector);
//   f32:  elements 4c .. 4c+3 and D/2+4c .. D/2+4c+3 (two 16-byte vectors),
// so that the LPK = D/8 lanes of one row read it as contiguous 128-byte
// phases either way.
// ---------------------------------------------------------------------------
template <typename T, int D>
struct Slice;

template <int D>
struct Slice<__nv_bfloat16, D> {
  __device__ __forceinline__ static int elem(int c, int j) { return 8 * c + j; }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  // Loads the lane's slice of a row starting at `row` (global or shared).
  __device__ __forceinline__ static void load(const __nv_bfloat16* row, int c, float* f) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + 8 * c);
    unpack(u, f);
  }
  __device__ __forceinline__ static void load_global_nc(const __nv_bfloat16* row, int c, float* f) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + 8 * c));
    unpack(u, f);
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* row, int c, const float* f) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(row + 8 * c) = u;
  }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <int D>
struct Slice<float, D> {
  __device__ __forceinline__ static int elem(int c, int j) {
    return j < 4 ? 4 * c + j : D / 2 + 4 * c + (j - 4);
  }
  __device__ __forceinline__ static void load(const float* row, int c, float* f) {
    const float4 a = *reinterpret_cast<const float4*>(row + 4 * c);
    const float4 b = *reinterpret_cast<const float4*>(row + D / 2 + 4 * c);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ __forceinline__ static void load_global_nc(const float* row, int c, float* f) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(row + 4 * c));
    const float4 b = __ldg(reinterpret_cast<const float4*>(row + D / 2 + 4 * c));
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ __forceinline__ static void store(float* row, int c, const float* f) {
    *reinterpret_cast<float4*>(row + 4 * c) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(row + D / 2 + 4 * c) = make_float4(f[4], f[5], f[6], f[7]);
  }
  __device__ __forceinline__ static float round(float x) { return x; }
};

// exp2 on the SFU (ex2.approx, relative error ~2^-22); exp2(-inf) = 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace asrback
