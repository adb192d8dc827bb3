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
// The kernel runs as clusters of two CTAs, one tcgen05 pair on the two SMs of
// a TPC.  A pair tile is 256 tokens x 256 output features (two heads of q, k
// or v): each CTA loads its own 128 token rows of x and its own 128 rows of W
// (one head), and the even CTA issues M256 N256 MMAs that read both CTAs'
// operands and leave each CTA's 128 token rows x 256 features in its own
// TMEM.  A K step costs each SM 32 KB of operand loads for 512 MMA clocks,
// where a one-CTA 128 x 256 tile loads 48 KB for the same clocks.
//
// Roles per CTA (10 warps): warp 0 issues this CTA's TMA loads into a 5-stage
// ring (their completion counted on the even CTA's barrier), warp 1 of the
// even CTA issues the MMAs (one thread), warps 2-5 and 6-9 run the epilogue of
// the tile's first and second head, one thread per token row.  Two TMEM
// accumulators of 256 columns alternate so the epilogue of one tile overlaps
// the MMAs of the next.  The epilogue stages each warp's 32 finished head rows
// in shared memory and stores them two whole 256-byte rows per instruction.
//
// Rounding follows the separate ops it fuses: the Linear output is rounded
// to bf16 (bias added in fp32 first), the norm output is bf16(x * rsqrt) then
// bf16(n * w), RoPE rotates in fp32 and rounds once more.
#include "common.h"
#include "ptx.cuh"

namespace dgxm {

constexpr int kQkvStages = 5;
constexpr int kQkvThreads = 10 * 32;
constexpr int kQkvTile = 128;                        // token rows per CTA, and features per head
constexpr int kQkvPairM = 2 * kQkvTile;              // token rows per pair tile
constexpr int kQkvTileN = 256;                       // features per tile: two heads
constexpr int kQkvBk = 64;                           // K per stage (one 128-byte swizzle atom)
constexpr int kQkvHalfBytes = kQkvTile * 128;        // 128 rows x 64 bf16: 16 KB
constexpr int kQkvStageBytes = 2 * kQkvHalfBytes;    // this CTA's x rows and W rows
constexpr int kQkvPairStageBytes = 2 * kQkvStageBytes;
constexpr int kQkvStagingBytes = 8 * 32 * 256;       // per epilogue warp: 32 head rows
constexpr int kQkvSmemBytes = 1024 + kQkvStages * kQkvStageBytes + kQkvStagingBytes + 512;

// One token stream's projection: its rows, weight, bias and QKNorm weights.
struct __align__(64) QkvProblem {
  CUtensorMap tmap_x;  // dims (K, 1, M, 1), box (64, 1, 128, 1)
  CUtensorMap tmap_w;  // dims (K, 1, N, 1), box (64, 1, 128, 1)
  const __nv_bfloat16* bias;     // N entries or NULL
  const __nv_bfloat16* norm_w[2];
  int m, m_tiles, tiles, row0;   // rows, pair-tile rows, pair tiles, local row of the first row
};

// Up to two streams (a joint block's text and image) in one launch: their
// pair tiles are numbered one stream after the other.  The streams share the
// input width, the heads, the RoPE table and the receive tensors.
struct __align__(64) QkvGemmParams {
  QkvProblem prob[2];
  int n_prob, k_tiles, heads, n_tiles;
  int norm_head;                 // per-head RMSNorm on q and k
  float eps;
  const float* rope;             // (seq_local, 64, 2) cos/sin by local row, or NULL
  char* dst[3][DGXM_MAX_WORLD];  // (S, heads/world, 128) bf16 receive tensors
  int world, rank, seq_local, seg0;
};

// The stream of pair tile `tile` and the tile's index within it.
__device__ __forceinline__ const QkvProblem& qkv_problem(const QkvGemmParams& p, int tile, int& local) {
  if (tile < p.prob[0].tiles) {
    local = tile;
    return p.prob[0];
  }
  local = tile - p.prob[0].tiles;
  return p.prob[1];
}

// Barriers of each CTA.  The even CTA's Full and AccEmpty count for the pair;
// Empty and AccFull are signalled in both CTAs by the even CTA's commits.
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

// Pair tiles run in groups of kQkvGroupM token-tile rows, feature tiles
// outermost within a group, so the pairs resident at one time share a few x
// panels and a few W panels (about 13 + 14 MB at the C2 width) instead of
// sweeping all of W for every two token-tile rows.
constexpr int kQkvGroupM = 8;

__device__ __forceinline__ void qkv_tile_coords(int tile, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int per_group = kQkvGroupM * n_tiles;
  const int g = tile / per_group, r = tile - g * per_group;
  const int rows = min(kQkvGroupM, m_tiles - g * kQkvGroupM);  // token-tile rows in this group
  mt = g * kQkvGroupM + r % rows;
  nt = r / rows;
}

// One half of a warp's 32 RoPE rows (pairs 32h .. 32h + 31 of each row: 256
// contiguous bytes) into its staging rows, two rows per instruction; 16-byte
// chunk c of row r goes to chunk c ^ (r & 15), as the output rows do.
__device__ __forceinline__ void qkv_stage_rope(const float* rope, const QkvProblem& pr, uint8_t* stage_rows,
                                               int m0, int lane, int h) {
  const int cc = lane & 15;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int rr = 2 * j + (lane >> 4);
    const int mr = m0 + rr;
    if (mr < pr.m)
      cp_async16(smem_u32(stage_rows + rr * 256 + ((cc ^ (rr & 15)) << 4)),
                 rope + static_cast<int64_t>(pr.row0 + mr) * 128 + h * 64 + cc * 4);
  }
}

__global__ void __launch_bounds__(kQkvThreads, 1) qkv_gemm_prologue_kernel(const __grid_constant__ QkvGemmParams p) {
  using B = QkvBars;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  uint8_t* staging = smem + kQkvStages * kQkvStageBytes;
  uint8_t* ctrl = staging + kQkvStagingBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ctrl);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + B::kCount * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();     // 0: issues the pair's MMAs
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int tiles = p.prob[0].tiles + (p.n_prob > 1 ? p.prob[1].tiles : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQkvStages; ++s) {
      mbar_init(bar(B::kFull + s), 1);
      mbar_init(bar(B::kEmpty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(B::kAccFull + a), 1);
      mbar_init(bar(B::kAccEmpty + a), 16);  // every epilogue warp of both CTAs
    }
    mbar_init(bar(B::kDrain), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < p.n_prob; ++i) {
      tma_prefetch_desc(&p.prob[i].tmap_x);
      tma_prefetch_desc(&p.prob[i].tmap_w);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 2 * kQkvTileN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += pairs) {
        int lt, mt, nt;
        const QkvProblem& pr = qkv_problem(p, tile, lt);
        qkv_tile_coords(lt, pr.m_tiles, p.n_tiles, mt, nt);
        for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
          const int s = it % kQkvStages;
          if (!mbar_wait(bar(B::kEmpty + s), ((it / kQkvStages) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t dst = base + s * kQkvStageBytes;
          const uint32_t full = mapa_shared(bar(B::kFull + s), 0);
          if (cta == 0) mbar_expect_tx(bar(B::kFull + s), kQkvPairStageBytes);
          tma_load_4d_pair(dst, &pr.tmap_x, full, kt * kQkvBk, 0, mt * kQkvPairM + cta * kQkvTile, 0);
          tma_load_4d_pair(dst + kQkvHalfBytes, &pr.tmap_w, full, kt * kQkvBk, 0,
                           nt * kQkvTileN + cta * kQkvTile, 0);
        }
      }
      if (!ok) {
        report_device_error(kErrProducerTimeout);
        *abort_flag = 1;
        // Let the loads already issued land before the pair can exit (both
        // CTAs' loads report on the even CTA's barriers).
        if (cta == 0) {
          const int first = it > kQkvStages ? it - kQkvStages : 0;
          for (int i = first; i < it; ++i) mbar_wait(bar(B::kFull + i % kQkvStages), (i / kQkvStages) & 1, nullptr);
        } else {
          for (int i = 0; i < 50; ++i) __nanosleep(1000);  // the odd CTA cannot test those barriers
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && cta == 0) {
      constexpr uint32_t idesc = idesc_make(kQkvPairM, kQkvTileN, 1u, false);
      int it = 0, u = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < tiles; tile += pairs, ++u) {
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
            const uint64_t db = sdesc_sw128(sa + kQkvHalfBytes + kk * 32, 16, 1024);
            umma_f16_ss_pair(acc, da, db, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair_to(bar(B::kEmpty + s), 0x3);
        }
        if (ok) umma_commit_pair_to(bar(B::kAccFull + a), 0x3);
      }
      if (!ok) {
        report_device_error(kErrMmaTimeout);
        *abort_flag = 1;
      }
      // Every MMA issued has completed before either CTA releases its TMEM.
      umma_commit_pair_to(bar(B::kDrain), 0x1);
      mbar_wait(bar(B::kDrain), 0, nullptr);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                      // TMEM lane quarter of this warp
    const int hs = (warp - 2) >> 2;              // which of the tile's two heads (warps 2-5, 6-9)
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc_empty = mapa_shared(bar(B::kAccEmpty), 0);
    uint8_t* stage_rows = staging + (warp - 2) * (32 * 256);
    const int hl = p.heads / p.world;
    int u = 0;
    for (int tile = pair; tile < tiles; tile += pairs, ++u) {
      const int a = u & 1;
      int lt, mt, nt;
      const QkvProblem& pr = qkv_problem(p, tile, lt);
      qkv_tile_coords(lt, pr.m_tiles, p.n_tiles, mt, nt);
      // This warp group's head of the tile (q, k and v each span a whole
      // number of tiles, the head count being even).
      const int gh = nt * (kQkvTileN / kQkvTile) + hs;  // head over q | k | v
      const int which = gh / p.heads;                  // 0 q, 1 k, 2 v
      const int head = gh - which * p.heads;
      const int m0 = mt * kQkvPairM + static_cast<int>(cta) * kQkvTile + q * 32;  // this warp's first row
      const bool rope = which < 2 && p.rope != nullptr;
      // The first half of the warp's 32 RoPE rows is fetched while the MMAs run.
      if (rope) qkv_stage_rope(p.rope, pr, stage_rows, m0, lane, 0);
      const bool got = __all_sync(0xffffffffu, mbar_wait(bar(B::kAccFull + a), (u >> 1) & 1, abort_flag));
      if (!got) {
        cp_async_wait_all();
        report_device_error(kErrEpilogueTimeout);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
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
          if (pr.bias != nullptr) {
            const int n = gh * kQkvTile + c * 32 + 2 * i;
            v0 += __bfloat162float(pr.bias[n]);
            v1 += __bfloat162float(pr.bias[n + 1]);
          }
          const uint32_t packed = pack_bf16x2(v0, v1);
          y[c * 16 + i] = packed;
          const float b0 = __uint_as_float(packed << 16), b1 = __uint_as_float(packed & 0xFFFF0000u);
          ss = fmaf(b0, b0, ss);
          ss = fmaf(b1, b1, ss);
        }
      }
      // This warp's rows of the accumulator are in registers; once every
      // epilogue warp of both CTAs has arrived, the MMAs may refill it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty + a * 8);
      if (which < 2 && p.norm_head) {
        const float sc = rsqrtf(ss / 128.f + p.eps);
        const __nv_bfloat16* w = pr.norm_w[which];
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          float x0 = __uint_as_float(y[i] << 16), x1 = __uint_as_float(y[i] & 0xFFFF0000u);
          x0 = __bfloat162float(__float2bfloat16(x0 * sc));
          x1 = __bfloat162float(__float2bfloat16(x1 * sc));
          if (w != nullptr) {
            x0 = __bfloat162float(__float2bfloat16(x0 * __bfloat162float(w[2 * i])));
            x1 = __bfloat162float(__float2bfloat16(x1 * __bfloat162float(w[2 * i + 1])));
          }
          y[i] = pack_bf16x2(x0, x1);
        }
      }
      if (rope) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1) qkv_stage_rope(p.rope, pr, stage_rows, m0, lane, 1);
          cp_async_wait_all();
          __syncwarp();
          // Row `lane`'s pairs 32h + 2c and 32h + 2c + 1: (cos, sin, cos, sin).
          const float4* mine = reinterpret_cast<const float4*>(stage_rows + lane * 256);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float4 t = mine[c ^ (lane & 15)];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int i = 32 * h + 2 * c + e;
              const float cs = e ? t.z : t.x, sn = e ? t.w : t.y;
              const float x0 = __uint_as_float(y[i] << 16), x1 = __uint_as_float(y[i] & 0xFFFF0000u);
              y[i] = pack_bf16x2(fmaf(-sn, x1, cs * x0), fmaf(cs, x1, sn * x0));
            }
          }
          __syncwarp();
        }
      }
      // Stage the warp's 32 rows (16-byte chunk c of row r at chunk c ^ (r & 15),
      // so that both the row-wise writes and the chunk-wise reads below are free
      // of bank conflicts), then store two whole rows per instruction.
      uint4* mine = reinterpret_cast<uint4*>(stage_rows + lane * 256);
#pragma unroll
      for (int c = 0; c < 16; ++c)
        mine[c ^ (lane & 15)] = make_uint4(y[4 * c], y[4 * c + 1], y[4 * c + 2], y[4 * c + 3]);
      __syncwarp();
      const int owner = head / hl, hh = head - owner * hl;
      char* const dst_base = p.dst[which][owner];
      const int cc = lane & 15;
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int rr = 2 * j + (lane >> 4);
        const int mr = m0 + rr;
        if (mr < pr.m) {
          const uint4 v = reinterpret_cast<const uint4*>(stage_rows + rr * 256)[cc ^ (rr & 15)];
          const int64_t grow = qkv_gathered_row(p.rank, pr.row0 + mr, p.seq_local, p.world, p.seg0);
          reinterpret_cast<uint4*>(dst_base + (grow * hl + hh) * 256)[cc] = v;
        }
      }
      __syncwarp();
    }
  }
  tc_fence_before();
  cluster_sync();  // the pair's MMAs drained and every TMEM read done in both CTAs
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * kQkvTileN);
  }
}

}  // namespace dgxm

namespace dgxm {

// Check and launch the grouped projection of n (1 or 2) streams.
static int qkv_launch(const dgxm_qkv_gemm_desc* d, int n, const dgxm_qkv_stream* st, const float* rope,
                      void* const* dst, void* stream) {
  if (d == nullptr || st == nullptr || dst == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL descriptor, streams or destination");
  if (n < 1 || n > 2) return fail(DGXM_ERR_INVALID, "%d streams (1 or 2)", n);
  if (d->world < 1 || d->world > DGXM_MAX_WORLD || d->rank < 0 || d->rank >= d->world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", d->rank, d->world);
  if (d->heads <= 0 || d->heads % d->world)
    return fail(DGXM_ERR_INVALID, "%d heads are not divisible by the Ulysses degree %d", d->heads, d->world);
  if (d->heads % (kQkvTileN / kQkvTile))
    return fail(DGXM_ERR_UNSUPPORTED, "the fused QKV kernel takes an even head count (two heads per tile), got %d",
                d->heads);
  if (d->k <= 0 || d->k % 8)
    return fail(DGXM_ERR_INVALID, "k %d must be a positive multiple of 8", d->k);
  if (d->seq_local <= 0 || d->seg0 < 0 || d->seg0 >= d->seq_local)
    return fail(DGXM_ERR_INVALID, "seg0 %d does not split the %d local rows", d->seg0, d->seq_local);
  if (d->norm_mode != DGXM_NORM_NONE && d->norm_mode != DGXM_NORM_HEAD)
    return fail(DGXM_ERR_UNSUPPORTED, "the fused QKV kernel applies per-head norms only (mode %d)", d->norm_mode);
  if (reinterpret_cast<uintptr_t>(rope) % 16) return fail(DGXM_ERR_INVALID, "rope must be 16-byte aligned");
  for (int i = 0; i < n; ++i) {
    const dgxm_qkv_stream& s = st[i];
    if (s.m == 0) continue;  // an empty stream may pass NULL pointers
    if (s.x == nullptr || s.w_qkv == nullptr)
      return fail(DGXM_ERR_INVALID, "stream %d: NULL input or weight", i);
    if (s.m < 0 || s.x_row_stride % 8 || s.x_row_stride < d->k)
      return fail(DGXM_ERR_INVALID, "stream %d: m %d / row stride %lld (a multiple of 8, at least k %d)", i, s.m,
                  (long long)s.x_row_stride, d->k);
    if (s.row0 < 0 || s.row0 + s.m > d->seq_local)
      return fail(DGXM_ERR_INVALID, "stream %d: rows [%d, %d) do not fit the %d local rows", i, s.row0,
                  s.row0 + s.m, d->seq_local);
    if ((reinterpret_cast<uintptr_t>(s.x) | reinterpret_cast<uintptr_t>(s.w_qkv)) % 16)
      return fail(DGXM_ERR_INVALID, "stream %d: x and w_qkv must be 16-byte aligned", i);
  }
  for (int i = 0; i < 3 * d->world; ++i)
    if (dst[i] == nullptr || reinterpret_cast<uintptr_t>(dst[i]) % 16)
      return fail(DGXM_ERR_INVALID, "destination %d is NULL or not 16-byte aligned", i);
  QkvGemmParams p;
  memset(&p, 0, sizeof(p));
  const int64_t nw = 3LL * d->heads * 128;
  p.k_tiles = (d->k + kQkvBk - 1) / kQkvBk;
  p.heads = d->heads;
  p.n_tiles = 3 * d->heads * kQkvTile / kQkvTileN;
  int tiles = 0;
  for (int i = 0; i < n; ++i) {
    const dgxm_qkv_stream& s = st[i];
    if (s.m == 0) continue;  // no rows, no tiles
    QkvProblem& pr = p.prob[p.n_prob++];
    int rc;
    if ((rc = encode_map_4d(&pr.tmap_x, s.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d->k, 1, s.m, 1, d->k,
                            s.x_row_stride, s.x_row_stride * s.m, kQkvBk, kQkvTile)))
      return rc;
    if ((rc = encode_map_4d(&pr.tmap_w, s.w_qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d->k, 1, nw, 1, d->k, d->k,
                            d->k * nw, kQkvBk, kQkvTile)))
      return rc;
    pr.bias = static_cast<const __nv_bfloat16*>(s.bias);
    pr.norm_w[0] = static_cast<const __nv_bfloat16*>(s.norm_q_w);
    pr.norm_w[1] = static_cast<const __nv_bfloat16*>(s.norm_k_w);
    pr.m = s.m;
    pr.m_tiles = (s.m + kQkvPairM - 1) / kQkvPairM;
    pr.tiles = pr.m_tiles * p.n_tiles;
    pr.row0 = s.row0;
    tiles += pr.tiles;
  }
  if (tiles == 0) return DGXM_OK;
  p.norm_head = d->norm_mode == DGXM_NORM_HEAD;
  p.eps = d->eps;
  p.rope = rope;
  for (int t = 0; t < 3; ++t)
    for (int r = 0; r < d->world; ++r) p.dst[t][r] = static_cast<char*>(dst[t * d->world + r]);
  p.world = d->world;
  p.rank = d->rank;
  p.seq_local = d->seq_local;
  p.seg0 = d->seg0;
  int dev = 0;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  static std::atomic<uint64_t> configured{0};  // bit per device
  DGXM_CUDA_TRY(set_smem_limit_once(qkv_gemm_prologue_kernel, kQkvSmemBytes, configured));
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kQkvThreads);
  cfg.dynamicSmemBytes = kQkvSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Pairs resident at once (one per TPC when nothing else runs), cached per device.
  static std::atomic<int> max_pairs[64];
  int pairs = dev < 64 ? max_pairs[dev].load() : 0;
  if (pairs <= 0) {
    cfg.gridDim = dim3(2);
    DGXM_CUDA_TRY(cudaOccupancyMaxActiveClusters(&pairs, qkv_gemm_prologue_kernel, &cfg));
    if (pairs <= 0) return fail(DGXM_ERR_CUDA, "no CTA pair of the fused QKV kernel fits on device %d", dev);
    if (dev < 64) max_pairs[dev].store(pairs);
  }
  cfg.gridDim = dim3(2 * (tiles < pairs ? tiles : pairs));
  DGXM_CUDA_TRY(cudaLaunchKernelEx(&cfg, qkv_gemm_prologue_kernel, p));
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int dgxm_qkv_gemm_prologue_scatter(const dgxm_qkv_gemm_desc* d, const void* x,
                                              const void* w_qkv, const void* bias,
                                              const void* norm_q_w, const void* norm_k_w,
                                              const float* rope, void* const* dst, void* stream) {
  using namespace dgxm;
  if (d == nullptr || x == nullptr || w_qkv == nullptr || dst == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL descriptor, input, weight or destination");
  if (d->m < 0 || d->k <= 0 || d->k % 8 || d->x_row_stride % 8 || d->x_row_stride < d->k)
    return fail(DGXM_ERR_INVALID, "m %d / k %d / row stride %lld: k and the stride must be multiples of 8",
                d->m, d->k, (long long)d->x_row_stride);
  if (d->seq_local <= 0 || d->row0 < 0 || d->row0 + d->m > d->seq_local || d->seg0 < 0 || d->seg0 >= d->seq_local)
    return fail(DGXM_ERR_INVALID, "rows [%d, %d) do not fit the %d local rows (seg0 %d)", d->row0,
                d->row0 + d->m, d->seq_local, d->seg0);
  dgxm_qkv_stream s;
  s.x = x;
  s.w_qkv = w_qkv;
  s.bias = bias;
  s.norm_q_w = norm_q_w;
  s.norm_k_w = norm_k_w;
  s.x_row_stride = d->x_row_stride;
  s.m = d->m;
  s.row0 = d->row0;
  return qkv_launch(d, 1, &s, rope, dst, stream);
}

extern "C" int dgxm_qkv_gemm_prologue_scatter_streams(const dgxm_qkv_gemm_desc* d, int32_t n_streams,
                                                      const dgxm_qkv_stream* streams, const float* rope,
                                                      void* const* dst, void* stream) {
  return dgxm::qkv_launch(d, n_streams, streams, rope, dst, stream);
}
