// The per-device error word.  Kernels OR a kErr* bit into it when a bounded
// wait expires; the host reads it with dgxm_device_error().  The library is
// built as one translation unit, so this single definition is shared by every
// kernel without relocatable device code.
#pragma once

namespace dgxm {

__device__ int g_device_error = 0;

__device__ __forceinline__ void report_device_error(int bits) { atomicOr(&g_device_error, bits); }

}  // namespace dgxm
