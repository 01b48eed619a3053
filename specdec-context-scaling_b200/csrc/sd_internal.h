// sd_internal.h -- host-side helpers shared by the translation units of the library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sd {

// Records a printf-style message for specdec_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Checks cudaGetLastError() after a launch; counts `n` launches on success.
int after_launch(const char* what, int n = 1);
// SM count of the current device (cached per device).
int device_sm_count();

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace sd
