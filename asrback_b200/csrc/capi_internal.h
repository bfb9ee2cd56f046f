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

// Programmatic dependent launch is on unless a build sets ASRBACK_PDL to 0.
#ifndef ASRBACK_PDL
#define ASRBACK_PDL 1
#endif

// Launches `kernel` with programmatic stream serialization: its CTAs may be
// scheduled while the previous kernel of the stream finishes, so the kernel
// must call griddep_wait() before it reads any input. Returns an ABI code.
template <typename... Params, typename... Args>
int launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               const char* what, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = ASRBACK_PDL ? 1 : 0;
  return check_cuda(cudaLaunchKernelEx(&config, kernel, static_cast<Args&&>(args)...), what);
}

// As launch_pdl, with the grid's CTAs in clusters of `cluster_x` along x.
template <typename... Params, typename... Args>
int launch_pdl_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       unsigned cluster_x, cudaStream_t stream, const char* what, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[2];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = cluster_x;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[1].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = ASRBACK_PDL ? 2 : 1;
  return check_cuda(cudaLaunchKernelEx(&config, kernel, static_cast<Args&&>(args)...), what);
}

}  // namespace asrback
