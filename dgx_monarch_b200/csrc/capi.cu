// Status plumbing, tensor-map encoding and the device error word for the C ABI.
#include <string.h>

#include "common.h"
#include "device_error.cuh"

namespace dgxm {

static thread_local char g_msg[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DGXM_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e),
              cudaGetErrorString(e));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  }
  return fn;
}

int encode_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elt_bytes,
                  int64_t cols, int64_t heads, int64_t rows, int64_t batch, int64_t s_head,
                  int64_t s_row, int64_t s_batch, int box_cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(DGXM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(DGXM_ERR_INVALID, "tensor base address %p is not 16-byte aligned", base);
  // A size-1 dimension's stride is never used to address memory; give it a
  // legal value so callers may pass any stride there.
  if (heads == 1) s_head = cols;
  if (batch == 1) s_batch = rows * s_row;
  const int64_t bs[3] = {s_head * elt_bytes, s_row * elt_bytes, s_batch * elt_bytes};
  for (int i = 0; i < 3; ++i) {
    if (bs[i] <= 0 || bs[i] % 16 != 0 || bs[i] >= (int64_t(1) << 40))
      return fail(DGXM_ERR_INVALID,
                  "tensor stride %lld bytes (dim %d) must be a positive multiple of 16",
                  (long long)bs[i], i + 1);
  }
  cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)heads, (cuuint64_t)rows,
                        (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)bs[0], (cuuint64_t)bs[1], (cuuint64_t)bs[2]};
  cuuint32_t box[4] = {(cuuint32_t)box_cols, 1u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DGXM_ERR_INVALID, "cuTensorMapEncodeTiled returned %d", (int)r);
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int dgxm_abi_version(void) { return 2; }

extern "C" const char* dgxm_last_error_message(void) { return dgxm::g_msg; }

extern "C" int dgxm_device_error(int clear) {
  int value = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return -dgxm::cuda_fail(e, "cudaDeviceSynchronize");
  e = cudaMemcpyFromSymbol(&value, dgxm::g_device_error, sizeof(int));
  if (e != cudaSuccess) return -dgxm::cuda_fail(e, "cudaMemcpyFromSymbol");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(dgxm::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return -dgxm::cuda_fail(e, "cudaMemcpyToSymbol");
  }
  return value;
}

// A strided copy between host and device memory (or within either): `height`
// rows of `width` bytes, row pitches `dpitch` / `spitch`.  One copy-engine
// transfer; the head-group slices of a (B, L, H, D) tensor are such copies.
extern "C" int dgxm_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width,
                            int64_t height, void* stream) {
  using namespace dgxm;
  if (width < 0 || height < 0 || dpitch < width || spitch < width)
    return fail(DGXM_ERR_INVALID, "2-D copy of %lld x %lld bytes with pitches %lld / %lld", (long long)height,
                (long long)width, (long long)dpitch, (long long)spitch);
  if (width == 0 || height == 0) return DGXM_OK;
  if (dst == nullptr || src == nullptr) return fail(DGXM_ERR_INVALID, "NULL 2-D copy pointer");
  DGXM_CUDA_TRY(cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch),
                                  static_cast<size_t>(width), static_cast<size_t>(height), cudaMemcpyDefault,
                                  static_cast<cudaStream_t>(stream)));
  return DGXM_OK;
}
