// C ABI plumbing: per-thread error messages, ABI version, device queries.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/asrback_attn.h"
#include "capi_internal.h"
#include "common.cuh"

namespace asrback {

namespace {
thread_local char g_last_error[512] = "";
}

int fail(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return code;
}

int ok() {
  g_last_error[0] = '\0';
  return ASRBACK_OK;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return ASRBACK_OK;
  return fail(ASRBACK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int sm_count() {
  static std::mutex lock;
  static int counts[64] = {0};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> guard(lock);
  if (counts[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    counts[device] = n;
  }
  return counts[device];
}

namespace {

// Waits on an mbarrier that nothing arrives at, with the same bounded wait the
// attention kernels use, given up after `budget_ns`: the wait must return
// false, and the kernel reports ASRBACK_STATUS_TIMEOUT and exits normally.
__global__ void bounded_wait_selftest(uint64_t budget_ns, int32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const uint64_t deadline = global_timer_ns() + budget_ns;
  if (!mbar_wait(&bar, 0, deadline)) atomicOr(status, ASRBACK_STATUS_TIMEOUT);
}

}  // namespace

}  // namespace asrback

extern "C" {

int asrback_selftest_bounded_wait(int64_t budget_ns, int32_t* status, void* stream) {
  using namespace asrback;
  if (budget_ns <= 0 || budget_ns > 1000000000LL || status == nullptr)
    return fail(ASRBACK_ERR_ARGUMENT, "budget_ns must be in (0, 1e9] and status non-null");
  bounded_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(budget_ns), status);
  if (int rc = check_cuda(cudaGetLastError(), "bounded wait self-test launch")) return rc;
  return ok();
}


int asrback_abi_version(void) { return (1 << 16) | 3; }

const char* asrback_last_error(void) { return asrback::g_last_error; }

int asrback_device_sm_count(void) { return asrback::sm_count(); }

}  // extern "C"
