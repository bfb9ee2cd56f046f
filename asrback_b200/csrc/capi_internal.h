// Host-side helpers shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace asrback {

// Records a printf-style message as this thread's last error; returns `code`.
int fail(int code, const char* fmt, ...);
// Clears this thread's last error; returns ASRBACK_OK.
int ok();
// SM count of the current device (cached per device).
int sm_count();
// Checks a CUDA result; on failure records it and returns ASRBACK_ERR_CUDA.
int check_cuda(cudaError_t err, const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace asrback
