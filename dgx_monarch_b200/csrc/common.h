// Host-side helpers shared by the C-ABI translation units: status plumbing,
// a per-thread error message, CUDA error capture and TMA descriptor encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/dgxm_sp.h"

namespace dgxm {

// Set the calling thread's last error message and return `code`.
int fail(int code, const char* fmt, ...);

// Map a CUDA runtime error to DGXM_ERR_CUDA with a message.
int cuda_fail(cudaError_t e, const char* what);

#define DGXM_CUDA_TRY(expr)                                  \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return ::dgxm::cuda_fail(_e, #expr); \
  } while (0)

// Raise `kern`'s dynamic shared-memory limit to `bytes` on the current device,
// once per device: `done` keeps one bit per device ordinal below 64 (others
// are set on every call).  Safe to call from several host threads.
template <typename Kernel>
cudaError_t set_smem_limit_once(Kernel kern, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? uint64_t(1) << dev : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Encode a 4-D tiled tensor map over a (batch, row, head, col) tensor whose
// innermost dimension `cols` is contiguous.  Strides are in elements.
// box = {box_cols, 1, box_rows, 1}, 128-byte swizzle, zero fill out of bounds.
int encode_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elt_bytes,
                  int64_t cols, int64_t heads, int64_t rows, int64_t batch, int64_t s_head,
                  int64_t s_row, int64_t s_batch, int box_cols, int box_rows);

// Stores into a per-device error word written by kernels whose bounded waits
// expired (bit flags, see kErr* below).
constexpr int kErrProducerTimeout = 1;
constexpr int kErrMmaTimeout = 2;
constexpr int kErrSoftmaxTimeout = 4;
constexpr int kErrEpilogueTimeout = 8;
constexpr int kErrPeerTimeout = 16;

}  // namespace dgxm
