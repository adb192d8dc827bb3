// QKV projection fused with the Ulysses prologue: one persistent tcgen05
// GEMM whose epilogue applies the Linear bias, per-head Q/K RMSNorm and RoPE
// and stores every head row straight into the receive tensor of the rank that
// owns the head (NVLink peer stores) -- the compute step and the
// sequence->head all-to-all in one kernel.
//
// It replaces, for the Flux/Krea2 joint blocks, the QKV Linear, the QKNorm
// and RoPE the block runs before the attention seam, and the
// SeqAllToAll4D(2, 1) scatter (adapters/usp_full_axis.py:27-29); the Wan
// variant with a norm over the whole hidden size keeps the separate prologue
// kernel (a row's norm spans 40 head tiles).
//
// Roles (10 warps): warp 0 issues TMA loads of x and W tiles into a 4-stage
// ring, warp 1 issues the MMAs (one thread), warps 2-5 and 6-9 run the
// epilogue of the tile's first and second head with one thread per output
// row.  Tiles are 128 tokens x 256 output features, i.e. two heads of q, k or
// v (M128 N256 MMAs), so the per-head norm and the RoPE pairs never leave a
// thread, and a K step reads 48 KB for 4 MFLOP where 128-wide tiles read
// 32 KB for 2.  Two TMEM accumulators of 256 columns alternate so the
// epilogue of one tile overlaps the MMAs of the next.
//
// Rounding follows the separate ops it fuses: the Linear output is rounded
// to bf16 (bias added in fp32 first), the norm output is bf16(x * rsqrt) then
// bf16(n * w), RoPE rotates in fp32 and rounds once more.
#include "common.h"
#include "ptx.cuh"

namespace dgxm {

constexpr int kQkvStages = 4;
constexpr int kQkvThreads = 10 * 32;
constexpr int kQkvTile = 128;                    // tokens per tile, and features per head
constexpr int kQkvTileN = 256;                   // features per tile: two heads
constexpr int kQkvBk = 64;                       // K per stage (one 128-byte swizzle atom)
constexpr int kQkvTileBytes = kQkvTile * 128;    // the x tile per stage: 16 KB
constexpr int kQkvWBytes = kQkvTileN * 128;      // the W tile per stage: 32 KB
constexpr int kQkvStageBytes = kQkvTileBytes + kQkvWBytes;
constexpr int kQkvSmemBytes = 1024 + kQkvStages * kQkvStageBytes + 512;

struct __align__(64) QkvGemmParams {
  CUtensorMap tmap_x;  // dims (K, 1, M, 1), box (64, 1, 128, 1)
  CUtensorMap tmap_w;  // dims (K, 1, N, 1), box (64, 1, 256, 1)
  int m, k_tiles, heads, n_tiles, m_tiles;
  const __nv_bfloat16* bias;     // N entries or NULL
  const __nv_bfloat16* norm_w[2];
  int norm_head;                 // per-head RMSNorm on q and k
  float eps;
  const float* rope;             // (seq_local, 64, 2) cos/sin by local row, or NULL
  char* dst[3][DGXM_MAX_WORLD];  // (S, heads/world, 128) bf16 receive tensors
  int world, rank, seq_local, row0, seg0;
};

struct QkvBars {
  static constexpr int kFull = 0;
  static constexpr int kEmpty = kFull + kQkvStages;
  static constexpr int kAccFull = kEmpty + kQkvStages;  // 2
  static constexpr int kAccEmpty = kAccFull + 2;        // 2
  static constexpr int kDrain = kAccEmpty + 2;
  static constexpr int kCount = kDrain + 1;
};

__device__ __forceinline__ int64_t qkv_gathered_row(int r, int l, int seq_local, int world, int seg0) {
  if (seg0 == 0) return static_cast<int64_t>(r) * seq_local + l;
  if (l < seg0) return static_cast<int64_t>(r) * seg0 + l;
  return static_cast<int64_t>(world) * seg0 + static_cast<int64_t>(r) * (seq_local - seg0) + (l - seg0);
}

__global__ void __launch_bounds__(kQkvThreads, 1) qkv_gemm_prologue_kernel(const __grid_constant__ QkvGemmParams p) {
  using B = QkvBars;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  uint8_t* ctrl = smem + kQkvStages * kQkvStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ctrl);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + B::kCount * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQkvStages; ++s) {
      mbar_init(bar(B::kFull + s), 1);
      mbar_init(bar(B::kEmpty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(B::kAccFull + a), 1);
      mbar_init(bar(B::kAccEmpty + a), 256);  // every epilogue thread
    }
    mbar_init(bar(B::kDrain), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_x);
    tma_prefetch_desc(&p.tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 2 * kQkvTileN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
        for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
          const int s = it % kQkvStages;
          if (!mbar_wait(bar(B::kEmpty + s), ((it / kQkvStages) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t dst = base + s * kQkvStageBytes;
          mbar_expect_tx(bar(B::kFull + s), kQkvStageBytes);
          tma_load_4d(dst, &p.tmap_x, bar(B::kFull + s), kt * kQkvBk, 0, mt * kQkvTile, 0);
          tma_load_4d(dst + kQkvTileBytes, &p.tmap_w, bar(B::kFull + s), kt * kQkvBk, 0, nt * kQkvTileN, 0);
        }
      }
      if (!ok) {
        report_device_error(kErrProducerTimeout);
        *abort_flag = 1;
        // Let the loads already issued land before the CTA can exit.
        const int first = it > kQkvStages ? it - kQkvStages : 0;
        for (int i = first; i < it; ++i) mbar_wait(bar(B::kFull + i % kQkvStages), (i / kQkvStages) & 1, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_make(kQkvTile, kQkvTileN, 1u, false);
      int it = 0, u = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++u) {
        const int a = u & 1;
        if (!(ok = mbar_wait(bar(B::kAccEmpty + a), ((u >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t acc = tmem + a * kQkvTileN;
        for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
          const int s = it % kQkvStages;
          if (!(ok = mbar_wait(bar(B::kFull + s), (it / kQkvStages) & 1, abort_flag))) break;
          tc_fence_after();
          const uint32_t sa = base + s * kQkvStageBytes;
#pragma unroll
          for (int kk = 0; kk < kQkvBk / 16; ++kk) {
            const uint64_t da = sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t db = sdesc_sw128(sa + kQkvTileBytes + kk * 32, 16, 1024);
            umma_f16_ss(acc, da, db, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar(B::kEmpty + s));
        }
        if (ok) umma_commit(bar(B::kAccFull + a));
      }
      if (!ok) {
        report_device_error(kErrMmaTimeout);
        *abort_flag = 1;
      }
      // Every MMA issued has completed before TMEM is released.
      umma_commit(bar(B::kDrain));
      mbar_wait(bar(B::kDrain), 0, nullptr);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                      // TMEM lane quarter of this warp
    const int hs = (warp - 2) >> 2;              // which of the tile's two heads (warps 2-5, 6-9)
    const int row = q * 32 + lane;               // row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int hl = p.heads / p.world;
    int u = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++u) {
      const int a = u & 1;
      const bool got = __all_sync(0xffffffffu, mbar_wait(bar(B::kAccFull + a), (u >> 1) & 1, abort_flag));
      if (!got) {
        report_device_error(kErrEpilogueTimeout);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int mt = tile / p.n_tiles, nt = tile % p.n_tiles;
      // This warp group's head of the tile (q, k and v each span a whole
      // number of tiles, the head count being even).
      {
        const int gh = nt * (kQkvTileN / kQkvTile) + hs;  // head over q | k | v
        const int which = gh / p.heads;            // 0 q, 1 k, 2 v
        const int head = gh - which * p.heads;
        // Linear output: fp32 accumulator + bias, rounded to bf16, kept packed.
        uint32_t y[64];
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + a * kQkvTileN + hs * kQkvTile + c * 32, r);
          tmem_wait_ld();
          reg_fence32(r);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float v0 = __uint_as_float(r[2 * i]), v1 = __uint_as_float(r[2 * i + 1]);
            if (p.bias != nullptr) {
              const int n = gh * kQkvTile + c * 32 + 2 * i;
              v0 += __bfloat162float(p.bias[n]);
              v1 += __bfloat162float(p.bias[n + 1]);
            }
            const uint32_t packed = pack_bf16x2(v0, v1);
            y[c * 16 + i] = packed;
            const float b0 = __uint_as_float(packed << 16), b1 = __uint_as_float(packed & 0xFFFF0000u);
            ss = fmaf(b0, b0, ss);
            ss = fmaf(b1, b1, ss);
          }
        }
        // This warp's half of the accumulator is in registers; once both
        // halves are, the MMA may refill it.
        tc_fence_before();
        mbar_arrive(bar(B::kAccEmpty + a));
        const int m = mt * kQkvTile + row;
        if (m < p.m) {
          const int l = p.row0 + m;                // local row in this rank's joint order
          const int64_t grow = qkv_gathered_row(p.rank, l, p.seq_local, p.world, p.seg0);
          const int owner = head / hl, hh = head - owner * hl;
          uint4* dst = reinterpret_cast<uint4*>(p.dst[which][owner] + (grow * hl + hh) * 256);
          if (which < 2 && (p.norm_head || p.rope != nullptr)) {
            const float sc = rsqrtf(ss / 128.f + p.eps);
            const __nv_bfloat16* w = p.norm_w[which];
            const float* rope_row = p.rope == nullptr ? nullptr : p.rope + static_cast<int64_t>(l) * 128;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              float x0 = __uint_as_float(y[i] << 16), x1 = __uint_as_float(y[i] & 0xFFFF0000u);
              if (p.norm_head) {
                x0 = __bfloat162float(__float2bfloat16(x0 * sc));
                x1 = __bfloat162float(__float2bfloat16(x1 * sc));
                if (w != nullptr) {
                  x0 = __bfloat162float(__float2bfloat16(x0 * __bfloat162float(w[2 * i])));
                  x1 = __bfloat162float(__float2bfloat16(x1 * __bfloat162float(w[2 * i + 1])));
                }
              }
              if (rope_row != nullptr) {
                const float cs = rope_row[2 * i], sn = rope_row[2 * i + 1];
                const float r0 = fmaf(-sn, x1, cs * x0);
                const float r1 = fmaf(cs, x1, sn * x0);
                x0 = r0;
                x1 = r1;
              }
              y[i] = pack_bf16x2(x0, x1);
            }
          }
#pragma unroll
          for (int v = 0; v < 16; ++v) dst[v] = make_uint4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kQkvTileN);
  }
}

}  // namespace dgxm

extern "C" int dgxm_qkv_gemm_prologue_scatter(const dgxm_qkv_gemm_desc* d, const void* x,
                                              const void* w_qkv, const void* bias,
                                              const void* norm_q_w, const void* norm_k_w,
                                              const float* rope, void* const* dst, void* stream) {
  using namespace dgxm;
  if (d == nullptr || x == nullptr || w_qkv == nullptr || dst == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL descriptor, input, weight or destination");
  if (d->world < 1 || d->world > DGXM_MAX_WORLD || d->rank < 0 || d->rank >= d->world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", d->rank, d->world);
  if (d->heads <= 0 || d->heads % d->world)
    return fail(DGXM_ERR_INVALID, "%d heads are not divisible by the Ulysses degree %d", d->heads, d->world);
  if (d->heads % (kQkvTileN / kQkvTile))
    return fail(DGXM_ERR_UNSUPPORTED, "the fused QKV kernel takes an even head count (two heads per tile), got %d",
                d->heads);
  if (d->m < 0 || d->k <= 0 || d->k % 8 || d->x_row_stride % 8 || d->x_row_stride < d->k)
    return fail(DGXM_ERR_INVALID, "m %d / k %d / row stride %lld: k and the stride must be multiples of 8",
                d->m, d->k, (long long)d->x_row_stride);
  if (d->seq_local <= 0 || d->row0 < 0 || d->row0 + d->m > d->seq_local || d->seg0 < 0 || d->seg0 >= d->seq_local)
    return fail(DGXM_ERR_INVALID, "rows [%d, %d) do not fit the %d local rows (seg0 %d)", d->row0,
                d->row0 + d->m, d->seq_local, d->seg0);
  if (d->norm_mode != DGXM_NORM_NONE && d->norm_mode != DGXM_NORM_HEAD)
    return fail(DGXM_ERR_UNSUPPORTED, "the fused QKV kernel applies per-head norms only (mode %d)", d->norm_mode);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_qkv)) % 16)
    return fail(DGXM_ERR_INVALID, "x and w_qkv must be 16-byte aligned");
  for (int i = 0; i < 3 * d->world; ++i)
    if (dst[i] == nullptr || reinterpret_cast<uintptr_t>(dst[i]) % 16)
      return fail(DGXM_ERR_INVALID, "destination %d is NULL or not 16-byte aligned", i);
  if (d->m == 0) return DGXM_OK;
  QkvGemmParams p;
  memset(&p, 0, sizeof(p));
  const int64_t n = 3LL * d->heads * 128;
  int rc;
  if ((rc = encode_map_4d(&p.tmap_x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d->k, 1, d->m, 1, d->k,
                          d->x_row_stride, d->x_row_stride * d->m, kQkvBk, kQkvTile)))
    return rc;
  if ((rc = encode_map_4d(&p.tmap_w, w_qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d->k, 1, n, 1, d->k, d->k,
                          d->k * n, kQkvBk, kQkvTileN)))
    return rc;
  p.m = d->m;
  p.k_tiles = (d->k + kQkvBk - 1) / kQkvBk;
  p.heads = d->heads;
  p.n_tiles = 3 * d->heads * kQkvTile / kQkvTileN;
  p.m_tiles = (d->m + kQkvTile - 1) / kQkvTile;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.norm_w[0] = static_cast<const __nv_bfloat16*>(norm_q_w);
  p.norm_w[1] = static_cast<const __nv_bfloat16*>(norm_k_w);
  p.norm_head = d->norm_mode == DGXM_NORM_HEAD;
  p.eps = d->eps;
  p.rope = rope;
  for (int t = 0; t < 3; ++t)
    for (int r = 0; r < d->world; ++r) p.dst[t][r] = static_cast<char*>(dst[t * d->world + r]);
  p.world = d->world;
  p.rank = d->rank;
  p.seq_local = d->seq_local;
  p.row0 = d->row0;
  p.seg0 = d->seg0;
  int dev = 0, sms = 148;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  DGXM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  static std::atomic<uint64_t> configured{0};  // bit per device
  DGXM_CUDA_TRY(set_smem_limit_once(qkv_gemm_prologue_kernel, kQkvSmemBytes, configured));
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < sms ? tiles : sms;
  qkv_gemm_prologue_kernel<<<grid, kQkvThreads, kQkvSmemBytes, static_cast<cudaStream_t>(stream)>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}
