// sd_internal.h -- host-side helpers shared by the translation units of the library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "../../include/specdec_b200.h"

namespace sd {

// Records a printf-style message for specdec_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Checks cudaGetLastError() after a launch; counts `n` launches on success.
int after_launch(const char* what, int n = 1);
// SM count of the current device (cached per device).
int device_sm_count();

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Launch with programmatic stream serialization: the kernel may start while the work
// before it on the stream drains, so it must execute griddepcontrol.wait before it
// reads anything that work writes (the kernels launched this way do so first thing).
template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(SPECDEC_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return after_launch(what);
}

}  // namespace sd
