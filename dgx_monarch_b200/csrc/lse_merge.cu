// Log-sum-exp merge of partial attention results over disjoint key blocks.
//
// For every (batch, row, head):
//   lse = log(sum_i exp(lse_i))
//   out = sum_i exp(lse_i - lse) * out_i
// computed in fp32.  This is the combine step of ring attention: each ring
// step attends the local queries to one rotating key/value block and leaves
// (out_i, lse_i); the merge folds them into the exact full-axis result.
//
// HBM-bound: one warp per (batch, row, head) row of head_dim = 128 values;
// each lane owns four consecutive values, so every part's row is read with one
// fully coalesced 256-byte (bf16 / fp16) or 512-byte (fp32) warp access.  The common
// part counts (the ring degrees) are compiled in, so all of a row's loads are
// in flight at once.
#include "common.h"
#include "ptx.cuh"

namespace dgxm {

constexpr int kMaxMergeParts = 16;

struct MergeParams {
  const void* out[kMaxMergeParts];
  const float* lse[kMaxMergeParts];
  void* dst;
  float* dst_lse;
  int n;
  int batch, rows, heads;
};

// Element types of the parts and the output: DGXM_DTYPE_BF16, _F16 or _F32.
template <int T>
__device__ __forceinline__ float4 load_part(const void* base, int64_t elem) {
  if constexpr (T == DGXM_DTYPE_F32) {
    return *reinterpret_cast<const float4*>(static_cast<const float*>(base) + elem);
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + elem);
    float2 a, c;
    if constexpr (T == DGXM_DTYPE_F16) {
      a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      c = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    } else {
      a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
      c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
    }
    return make_float4(a.x, a.y, c.x, c.y);
  }
}

// NP > 0 fixes the part count at compile time: every part's row and LSE is
// loaded before the first is used, so a warp keeps NP loads in flight
// instead of one (NP == 0 loops over p.n parts).
template <int PART, int OUT, int NP>
__global__ void __launch_bounds__(256) lse_merge_kernel(const __grid_constant__ MergeParams p) {
  constexpr int kSlots = NP > 0 ? NP : 1;
  const int warps_per_block = blockDim.x >> 5;
  const int64_t total = static_cast<int64_t>(p.batch) * p.rows * p.heads;
  const int lane = threadIdx.x & 31;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
       item < total; item += static_cast<int64_t>(gridDim.x) * warps_per_block) {
    // item enumerates (b, row, h) with h fastest, matching the (B, L, H, D) rows.
    const int h = static_cast<int>(item % p.heads);
    const int64_t br = item / p.heads;
    const int row = static_cast<int>(br % p.rows);
    const int b = static_cast<int>(br / p.rows);
    const int64_t lse_idx = (static_cast<int64_t>(b) * p.heads + h) * p.rows + row;
    const int64_t elem = item * 128 + lane * 4;
    float mx = -INFINITY, wsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (NP > 0) {
      float li[kSlots];
      float4 xv[kSlots];
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        li[i] = p.lse[i][lse_idx];
        xv[i] = load_part<PART>(p.out[i], elem);
      }
#pragma unroll
      for (int i = 0; i < NP; ++i) mx = fmaxf(mx, li[i]);
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        // A part with lse = -inf saw no keys for this row and carries no weight.
        const float w = (li[i] == -INFINITY) ? 0.f : __expf(li[i] - mx);
        wsum += w;
        acc.x = fmaf(w, xv[i].x, acc.x);
        acc.y = fmaf(w, xv[i].y, acc.y);
        acc.z = fmaf(w, xv[i].z, acc.z);
        acc.w = fmaf(w, xv[i].w, acc.w);
      }
    } else {
      for (int i = 0; i < p.n; ++i) mx = fmaxf(mx, p.lse[i][lse_idx]);
      for (int i = 0; i < p.n; ++i) {
        const float li = p.lse[i][lse_idx];
        const float w = (li == -INFINITY) ? 0.f : __expf(li - mx);
        wsum += w;
        const float4 x = load_part<PART>(p.out[i], elem);
        acc.x = fmaf(w, x.x, acc.x);
        acc.y = fmaf(w, x.y, acc.y);
        acc.z = fmaf(w, x.z, acc.z);
        acc.w = fmaf(w, x.w, acc.w);
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    if constexpr (OUT == DGXM_DTYPE_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(p.dst) + elem) =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    } else {
      constexpr bool kF16 = OUT == DGXM_DTYPE_F16;
      uint2 w;
      w.x = pack16<kF16>(acc.x * inv, acc.y * inv);
      w.y = pack16<kF16>(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.dst) + elem) = w;
    }
    if (lane == 0 && p.dst_lse != nullptr)
      p.dst_lse[lse_idx] = wsum > 0.f ? mx + __logf(wsum) : -INFINITY;
  }
}

template <int PART, int OUT>
static void launch_merge(const MergeParams& prm, int blocks, cudaStream_t st) {
  switch (prm.n) {
    case 1: lse_merge_kernel<PART, OUT, 1><<<blocks, 256, 0, st>>>(prm); break;
    case 2: lse_merge_kernel<PART, OUT, 2><<<blocks, 256, 0, st>>>(prm); break;
    case 3: lse_merge_kernel<PART, OUT, 3><<<blocks, 256, 0, st>>>(prm); break;
    case 4: lse_merge_kernel<PART, OUT, 4><<<blocks, 256, 0, st>>>(prm); break;
    case 8: lse_merge_kernel<PART, OUT, 8><<<blocks, 256, 0, st>>>(prm); break;
    default: lse_merge_kernel<PART, OUT, 0><<<blocks, 256, 0, st>>>(prm); break;
  }
}

}  // namespace dgxm

extern "C" int dgxm_lse_merge(int32_t batch, int32_t rows, int32_t heads, int32_t head_dim,
                              int32_t n_parts, const void* const* parts_out, int32_t part_dtype,
                              const float* const* parts_lse, void* out, int32_t out_dtype,
                              float* lse_out, void* stream) {
  using namespace dgxm;
  if (batch < 0 || rows < 0 || heads <= 0)
    return fail(DGXM_ERR_INVALID, "merge extents must be non-negative (heads positive)");
  if (head_dim != 128)
    return fail(DGXM_ERR_UNSUPPORTED, "merge head_dim %d is not supported (128)", head_dim);
  if (n_parts < 1 || n_parts > kMaxMergeParts)
    return fail(DGXM_ERR_INVALID, "merge takes 1..%d parts, got %d", kMaxMergeParts, n_parts);
  auto float_type = [](int t) {
    return t == DGXM_DTYPE_F32 || t == DGXM_DTYPE_BF16 || t == DGXM_DTYPE_F16;
  };
  if (!float_type(part_dtype))
    return fail(DGXM_ERR_UNSUPPORTED, "merge part dtype %d is not supported", part_dtype);
  if (!float_type(out_dtype))
    return fail(DGXM_ERR_UNSUPPORTED, "merge output dtype %d is not supported", out_dtype);
  // 16-bit parts merge into fp32 or their own 16-bit format.
  const bool mixed16 = part_dtype != DGXM_DTYPE_F32 && out_dtype != DGXM_DTYPE_F32 &&
                       part_dtype != out_dtype;
  if (mixed16)
    return fail(DGXM_ERR_UNSUPPORTED, "merge of %s parts into a %s output is not supported",
                part_dtype == DGXM_DTYPE_F16 ? "f16" : "bf16", out_dtype == DGXM_DTYPE_F16 ? "f16" : "bf16");
  if (parts_out == nullptr || parts_lse == nullptr)
    return fail(DGXM_ERR_INVALID, "merge part arrays must be non-NULL");
  // Nothing to merge: empty tensors may carry NULL data pointers.
  if (batch == 0 || rows == 0) return DGXM_OK;
  if (out == nullptr) return fail(DGXM_ERR_INVALID, "merge output must be non-NULL");
  MergeParams prm;
  memset(&prm, 0, sizeof(prm));
  for (int i = 0; i < n_parts; ++i) {
    if (parts_out[i] == nullptr || parts_lse[i] == nullptr)
      return fail(DGXM_ERR_INVALID, "merge part %d is NULL", i);
    if (reinterpret_cast<uintptr_t>(parts_out[i]) % 16 != 0)
      return fail(DGXM_ERR_INVALID, "merge part %d is not 16-byte aligned", i);
    prm.out[i] = parts_out[i];
    prm.lse[i] = parts_lse[i];
  }
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return fail(DGXM_ERR_INVALID, "merge output is not 16-byte aligned");
  prm.dst = out;
  prm.dst_lse = lse_out;
  prm.n = n_parts;
  prm.batch = batch;
  prm.rows = rows;
  prm.heads = heads;
  int dev = 0, sms = 148;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  DGXM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t items = static_cast<int64_t>(batch) * rows * heads;
  const int64_t want = (items + 7) / 8;
  const int blocks = static_cast<int>(want < int64_t(sms) * 16 ? want : int64_t(sms) * 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Ring steps hand fp32 parts; 16-bit parts come from callers that merge
  // blocks they attended themselves.
  constexpr int F32 = DGXM_DTYPE_F32, BF = DGXM_DTYPE_BF16, H = DGXM_DTYPE_F16;
  if (part_dtype == F32) {
    if (out_dtype == F32) launch_merge<F32, F32>(prm, blocks, st);
    else if (out_dtype == BF) launch_merge<F32, BF>(prm, blocks, st);
    else launch_merge<F32, H>(prm, blocks, st);
  } else if (part_dtype == BF) {
    if (out_dtype == F32) launch_merge<BF, F32>(prm, blocks, st);
    else launch_merge<BF, BF>(prm, blocks, st);
  } else {
    if (out_dtype == F32) launch_merge<H, F32>(prm, blocks, st);
    else launch_merge<H, H>(prm, blocks, st);
  }
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}
