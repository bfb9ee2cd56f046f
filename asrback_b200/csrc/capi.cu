// C ABI plumbing: per-thread error messages, ABI version, device queries.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/asrback_attn.h"
#include "capi_internal.h"

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

}  // namespace asrback

extern "C" {

int asrback_abi_version(void) { return (1 << 16) | 1; }

const char* asrback_last_error(void) { return asrback::g_last_error; }

int asrback_device_sm_count(void) { return asrback::sm_count(); }

}  // extern "C"
