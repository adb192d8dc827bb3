// The classifier-free-guidance combine of the dual-model CFG split
// (actor/dual_model_cfg.py:75-94): after the cfg group's all-gather, both
// ranks hold (cond, uncond) and combine them with comfy's default
//   uncond + (cond - uncond) * cfg
// Each operation rounds to the prediction dtype as torch's three elementwise
// ops do (the difference, the product with the scalar taken as fp32, the
// sum), with no fused multiply-add, so the result is bit-identical to the
// unfused torch expression on the device.

namespace dgxm {

struct CfgCombineParams {
  const void* cond;
  const void* uncond;
  void* out;
  int64_t n;
  float cfg;
  int dtype;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__device__ __forceinline__ T combine_one(T c, T u, float cfg) {
  const T d = from_f<T>(__fsub_rn(to_f(c), to_f(u)));
  const T m = from_f<T>(__fmul_rn(to_f(d), cfg));
  return from_f<T>(__fadd_rn(to_f(u), to_f(m)));
}

template <typename T>
__global__ void __launch_bounds__(256) cfg_combine_kernel(const __grid_constant__ CfgCombineParams p) {
  constexpr int kVec = 16 / sizeof(T);
  const int64_t nvec = p.n / kVec;
  const uint4* c4 = static_cast<const uint4*>(p.cond);
  const uint4* u4 = static_cast<const uint4*>(p.uncond);
  uint4* o4 = static_cast<uint4*>(p.out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 cv = c4[i], uv = u4[i];
    uint4 ov;
    const T* c = reinterpret_cast<const T*>(&cv);
    const T* u = reinterpret_cast<const T*>(&uv);
    T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int j = 0; j < kVec; ++j) o[j] = combine_one<T>(c[j], u[j], p.cfg);
    o4[i] = ov;
  }
  // The tail that does not fill a 16-byte vector.
  for (int64_t i = nvec * kVec + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < p.n; i += stride)
    static_cast<T*>(p.out)[i] = combine_one<T>(static_cast<const T*>(p.cond)[i],
                                               static_cast<const T*>(p.uncond)[i], p.cfg);
}

}  // namespace dgxm

extern "C" int dgxm_cfg_combine(const void* cond, const void* uncond, int64_t n, int32_t dtype,
                                double cfg_scale, void* out, void* stream) {
  using namespace dgxm;
  if (n < 0) return fail(DGXM_ERR_INVALID, "negative element count");
  if (dtype != DGXM_DTYPE_F32 && dtype != DGXM_DTYPE_BF16 && dtype != DGXM_DTYPE_F16)
    return fail(DGXM_ERR_UNSUPPORTED, "prediction dtype %d is not supported", dtype);
  if (n == 0) return DGXM_OK;
  if (cond == nullptr || uncond == nullptr || out == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL cond, uncond or output");
  if ((reinterpret_cast<uintptr_t>(cond) | reinterpret_cast<uintptr_t>(uncond) |
       reinterpret_cast<uintptr_t>(out)) % 16)
    return fail(DGXM_ERR_INVALID, "cond, uncond and out must be 16-byte aligned");
  CfgCombineParams p;
  p.cond = cond;
  p.uncond = uncond;
  p.out = out;
  p.n = n;
  p.cfg = static_cast<float>(cfg_scale);
  p.dtype = dtype;
  const int eb = elt_bytes(dtype);
  const int grid = grid_for((n * eb + 15) / 16, 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DGXM_DTYPE_F32: cfg_combine_kernel<float><<<grid, 256, 0, st>>>(p); break;
    case DGXM_DTYPE_BF16: cfg_combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p); break;
    case DGXM_DTYPE_F16: cfg_combine_kernel<__half><<<grid, 256, 0, st>>>(p); break;
    default: return fail(DGXM_ERR_UNSUPPORTED, "prediction dtype %d is not supported", dtype);
  }
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}
