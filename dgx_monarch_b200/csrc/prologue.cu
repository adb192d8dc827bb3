// Fused Ulysses prologue and FP8 quantisation.
//
// Q/K RMSNorm and multi-axis RoPE applied to a rank's rows while they are
// scattered head-slice by head-slice into the peers' receive tensors -- the
// sequence->head all-to-all of dgxm_ulysses_scatter with the per-token math
// the family forwards run just before the attention seam folded in.  V is
// moved unchanged.  Two kernels:
//   qkv_prologue_scatter_kernel  one block per token row, for the Wan
//                                norm_q/norm_k over the whole hidden size
//                                (adapters/wan_family.py:70-73);
//   qkv_prologue_head_kernel     one half-warp per head row, for the
//                                Flux/Krea2 per-head QKNorm or no norm.
//
// Rounding follows the separate ops it fuses: the norm's output is rounded
// to bf16 (the module's output dtype), RoPE then rotates that in fp32 and
// rounds once more.
//
// quantize kernels: per-head absmax (fp32) and e4m3 values x / (amax / 448),
// the FP8 inputs of the attention's kind::f8f6f4 path.
#include "common.h"
#include "ptx.cuh"

namespace dgxm {

struct PrologueParams {
  const char* src[3];
  int64_t s_sb[3], s_sl[3], s_sh[3];  // bytes
  char* dst[3][DGXM_MAX_WORLD];
  const __nv_bfloat16* norm_w[2];     // q, k weights (may be NULL)
  const float* rope;                  // (rows, D/2, 2) cos/sin per local row, or NULL
  int64_t rope_sb;                    // elements between batch items (0: shared)
  int norm_mode;                      // DGXM_NORM_*
  float eps;
  int world, rank, batch, seq_local, heads, seg0;
};

__device__ __forceinline__ int64_t gathered_row_p(int r, int l, int seq_local, int world, int seg0) {
  if (seg0 == 0) return static_cast<int64_t>(r) * seq_local + l;
  if (l < seg0) return static_cast<int64_t>(r) * seg0 + l;
  return static_cast<int64_t>(world) * seg0 + static_cast<int64_t>(r) * (seq_local - seg0) + (l - seg0);
}

constexpr int kPrologueThreads = 256;
constexpr int kPrologueMaxHidden = 6144;  // H * D of one row (static shared memory bound)

__global__ void __launch_bounds__(kPrologueThreads) qkv_prologue_scatter_kernel(const __grid_constant__ PrologueParams p) {
  __shared__ float buf[kPrologueMaxHidden];
  __shared__ __align__(16) __nv_bfloat16 obuf[kPrologueMaxHidden];
  __shared__ float red[kPrologueThreads / 32];
  __shared__ float row_scale;
  const int hid = p.heads * 128;
  const int hl = p.heads / p.world;
  const int64_t seq_full = static_cast<int64_t>(p.seq_local) * p.world;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t item = blockIdx.x; item < static_cast<int64_t>(p.batch) * p.seq_local; item += gridDim.x) {
    const int b = static_cast<int>(item / p.seq_local);
    const int l = static_cast<int>(item - static_cast<int64_t>(b) * p.seq_local);
    const int64_t grow = static_cast<int64_t>(b) * seq_full + gathered_row_p(p.rank, l, p.seq_local, p.world, p.seg0);
    for (int t = 0; t < 3; ++t) {
      const char* row = p.src[t] + b * p.s_sb[t] + static_cast<int64_t>(l) * p.s_sl[t];
      const bool math = t < 2 && (p.norm_mode != DGXM_NORM_NONE || p.rope != nullptr);
      if (math) {
        // Load the row (all heads) as fp32.
        for (int v = threadIdx.x; v < hid / 8; v += blockDim.x) {
          const int h = v / 16, part = v % 16;
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row + h * p.s_sh[t]) + part);
          const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(pr[i]);
            buf[v * 8 + 2 * i] = f.x;
            buf[v * 8 + 2 * i + 1] = f.y;
          }
        }
        __syncthreads();
        if (p.norm_mode == DGXM_NORM_HIDDEN) {
          float ss = 0.f;
          for (int i = threadIdx.x; i < hid; i += blockDim.x) ss = fmaf(buf[i], buf[i], ss);
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          if (lane == 0) red[warp] = ss;
          __syncthreads();
          if (threadIdx.x == 0) {
            float tot = 0.f;
            for (int w = 0; w < kPrologueThreads / 32; ++w) tot += red[w];
            row_scale = rsqrtf(tot / hid + p.eps);
          }
          __syncthreads();
        }
        const __nv_bfloat16* w = p.norm_w[t];
        const float* rope_row = p.rope == nullptr ? nullptr : p.rope + b * p.rope_sb + static_cast<int64_t>(l) * 128;
        for (int pr = threadIdx.x; pr < hid / 2; pr += blockDim.x) {
          const int e = 2 * pr;
          float x0 = buf[e], x1 = buf[e + 1];
          if (p.norm_mode == DGXM_NORM_HIDDEN) {
            const float sc = row_scale;
            // the norm module's output: bf16(x * rsqrt(mean + eps)) * weight, rounded
            const int wi = e;
            float n0 = __bfloat162float(__float2bfloat16(x0 * sc));
            float n1 = __bfloat162float(__float2bfloat16(x1 * sc));
            if (w != nullptr) {
              n0 = __bfloat162float(__float2bfloat16(n0 * __bfloat162float(w[wi])));
              n1 = __bfloat162float(__float2bfloat16(n1 * __bfloat162float(w[wi + 1])));
            }
            x0 = n0;
            x1 = n1;
          }
          if (rope_row != nullptr) {
            const int i = (e % 128) / 2;
            const float c = rope_row[2 * i], s = rope_row[2 * i + 1];
            const float y0 = fmaf(-s, x1, c * x0);
            const float y1 = fmaf(c, x1, s * x0);
            x0 = y0;
            x1 = y1;
          }
          reinterpret_cast<__nv_bfloat162*>(obuf)[pr] = __floats2bfloat162_rn(x0, x1);
        }
        __syncthreads();
        for (int v = threadIdx.x; v < hid / 8; v += blockDim.x) {
          const int h = v / 16, part = v % 16;
          const int r = h / hl, hh = h - r * hl;
          char* dst = p.dst[t][r] + (grow * hl + hh) * 256;
          reinterpret_cast<uint4*>(dst)[part] = reinterpret_cast<const uint4*>(obuf)[v];
        }
        __syncthreads();
      } else {
        for (int v = threadIdx.x; v < hid / 8; v += blockDim.x) {
          const int h = v / 16, part = v % 16;
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(row + h * p.s_sh[t]) + part);
          const int r = h / hl, hh = h - r * hl;
          char* dst = p.dst[t][r] + (grow * hl + hh) * 256;
          reinterpret_cast<uint4*>(dst)[part] = raw;
        }
      }
    }
  }
}

// Per-head norm (or none): each half-warp owns one (tensor, head) row of a
// token -- sub-lane s holds values [8s, 8s + 8), four RoPE pairs -- so a warp
// reads and writes two 256-byte head rows per access, and every half-warp has
// two rows in flight before it uses either.  The head's sum of squares is the
// sub-lane sums reduced over the half-warp; no block barrier is needed.
__device__ __forceinline__ uint4 prologue_head_math(const PrologueParams& p, uint4 raw, int t, int sub,
                                                   const float* rope_row) {
  float x[8];
  const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(pr[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
  // The reduction runs on every lane whatever row it holds (the norm mode is
  // uniform over the kernel), so a warp whose halves hold a k row and a v row
  // still meets every shuffle.
  float ss = 0.f;
  if (p.norm_mode == DGXM_NORM_HEAD) {
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  if (t == 2 || (p.norm_mode != DGXM_NORM_HEAD && rope_row == nullptr)) return raw;
  if (p.norm_mode == DGXM_NORM_HEAD) {
    const float sc = rsqrtf(ss / 128.f + p.eps);
    const __nv_bfloat16* w = p.norm_w[t];
    uint4 wv = make_uint4(0u, 0u, 0u, 0u);
    if (w != nullptr) wv = __ldg(reinterpret_cast<const uint4*>(w) + sub);  // this lane's 8 weights
    const __nv_bfloat16* wl = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float n = __bfloat162float(__float2bfloat16(x[i] * sc));
      if (w != nullptr) n = __bfloat162float(__float2bfloat16(n * __bfloat162float(wl[i])));
      x[i] = n;
    }
  }
  if (rope_row != nullptr) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float4 cs = __ldg(reinterpret_cast<const float4*>(rope_row) + 2 * sub + q);
      float* y = x + 4 * q;
      const float y0 = fmaf(-cs.y, y[1], cs.x * y[0]), y1 = fmaf(cs.x, y[1], cs.y * y[0]);
      const float y2 = fmaf(-cs.w, y[3], cs.z * y[2]), y3 = fmaf(cs.z, y[3], cs.w * y[2]);
      y[0] = y0; y[1] = y1; y[2] = y2; y[3] = y3;
    }
  }
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    o[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return out;
}

__global__ void __launch_bounds__(256) qkv_prologue_head_kernel(const __grid_constant__ PrologueParams p) {
  const int hl = p.heads / p.world;
  const int items = 3 * p.heads;  // (tensor, head) rows of one token
  const int lane = threadIdx.x & 31, sub = lane & 15;
  const int worker = threadIdx.x >> 4, workers = blockDim.x >> 4;  // half-warps
  const int64_t seq_full = static_cast<int64_t>(p.seq_local) * p.world;
  for (int64_t token = blockIdx.x; token < static_cast<int64_t>(p.batch) * p.seq_local; token += gridDim.x) {
    const int b = static_cast<int>(token / p.seq_local);
    const int l = static_cast<int>(token - static_cast<int64_t>(b) * p.seq_local);
    const int64_t grow = static_cast<int64_t>(b) * seq_full + gathered_row_p(p.rank, l, p.seq_local, p.world, p.seg0);
    const float* rope_row = p.rope == nullptr ? nullptr : p.rope + b * p.rope_sb + static_cast<int64_t>(l) * 128;
    // Both half-warps of a warp run the same trip count, so the shuffles of
    // the norm always see full warps.
    const int rounds = (items + 2 * workers - 1) / (2 * workers);
    for (int k = 0; k < rounds; ++k) {
      const int i0 = worker + 2 * workers * k, i1 = i0 + workers;
      const bool v0 = i0 < items, v1 = i1 < items;
      const int c0 = v0 ? i0 : 0, c1 = v1 ? i1 : 0;
      const int t0 = c0 / p.heads, h0 = c0 - t0 * p.heads;
      const int t1 = c1 / p.heads, h1 = c1 - t1 * p.heads;
      const uint4 r0 = __ldg(reinterpret_cast<const uint4*>(p.src[t0] + b * p.s_sb[t0] + static_cast<int64_t>(l) * p.s_sl[t0] +
                                                            h0 * p.s_sh[t0]) + sub);
      const uint4 r1 = __ldg(reinterpret_cast<const uint4*>(p.src[t1] + b * p.s_sb[t1] + static_cast<int64_t>(l) * p.s_sl[t1] +
                                                            h1 * p.s_sh[t1]) + sub);
      const uint4 o0 = prologue_head_math(p, r0, t0, sub, t0 < 2 ? rope_row : nullptr);
      const uint4 o1 = prologue_head_math(p, r1, t1, sub, t1 < 2 ? rope_row : nullptr);
      if (v0) {
        const int own = h0 / hl;
        reinterpret_cast<uint4*>(p.dst[t0][own] + (grow * hl + (h0 - own * hl)) * 256)[sub] = o0;
      }
      if (v1) {
        const int own = h1 / hl;
        reinterpret_cast<uint4*>(p.dst[t1][own] + (grow * hl + (h1 - own * hl)) * 256)[sub] = o1;
      }
    }
  }
}

// ---------------------------------------------------------------- FP8
struct QuantParams {
  const char* x;
  int64_t sb, sl, sh;  // bytes
  uint8_t* out;        // contiguous (B, L, H, D) e4m3
  float* amax;         // per head: accumulated absmax, then rewritten as descale
  const uint32_t* keep;  // optional row keep bits (bit l % 32 of word l / 32); cleared rows skip the absmax
  int64_t keep_sb;       // words between batch rows of `keep` (0: one mask for every batch row)
  int batch, rows, heads;
};

// Up to three tensors (q, k, v) quantised by the same launches: blockIdx.y
// picks the tensor, so one call fills the GPU with all three.
constexpr int kMaxQuantItems = 3;
struct QuantBatch {
  QuantParams t[kMaxQuantItems];
  int n;
};

// Per-head absmax.  Thread (h, part) of a block owns 16 bytes of head h in
// every row the block visits, keeps a running max in a register, reduces it
// over the head's 16 lanes with shuffles, and issues one atomicMax per head
// per block -- not one per 16 bytes, which would serialise on 'heads'
// addresses.  Non-negative floats order like their bit patterns.
__global__ void __launch_bounds__(1024) absmax_kernel(const __grid_constant__ QuantBatch pb) {
  const QuantParams& p = pb.t[blockIdx.y];
  const int slot = threadIdx.x;         // h * 16 + part
  const int h = slot / 16, part = slot % 16;
  float m = 0.f;
  if (h < p.heads) {
    const int64_t rows = static_cast<int64_t>(p.batch) * p.rows;
    for (int64_t br = blockIdx.x; br < rows; br += gridDim.x) {
      const int b = static_cast<int>(br / p.rows);
      const int l = static_cast<int>(br - static_cast<int64_t>(b) * p.rows);
      // A pad row the attention will exclude does not set its head's scale:
      // the scale is the one the real rows alone would give.
      if (p.keep != nullptr && !((__ldg(p.keep + b * p.keep_sb + (l >> 5)) >> (l & 31)) & 1u)) continue;
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p.x + b * p.sb + l * p.sl + h * p.sh) + part);
      const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(pr[k]);
        m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  // The 16 lanes of one head are 16 consecutive lanes of a warp.
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (part == 0 && h < p.heads) atomicMax(reinterpret_cast<unsigned int*>(p.amax) + h, __float_as_uint(m));
}

// Blocks stride over (batch, row); threads over the row's (head, 16-byte
// part) vectors, so the index math is a shift and a mask per vector.
__global__ void __launch_bounds__(256) quantize_e4m3_kernel(const __grid_constant__ QuantBatch pb) {
  const QuantParams& p = pb.t[blockIdx.y];
  const int per_row = p.heads * 16;
  for (int64_t row = blockIdx.x; row < static_cast<int64_t>(p.batch) * p.rows; row += gridDim.x) {
    const int b = static_cast<int>(row / p.rows);
    const int l = static_cast<int>(row - static_cast<int64_t>(b) * p.rows);
    for (int v = threadIdx.x; v < per_row; v += blockDim.x) {
    const int h = v >> 4, part = v & 15;
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p.x + b * p.sb + l * p.sl + h * p.sh) + part);
    const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float amax = fmaxf(p.amax[h], 1e-12f);
    const float scale = amax / 448.f;
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float2 a = __bfloat1622float2(pr[2 * k]);
      const float2 c = __bfloat1622float2(pr[2 * k + 1]);
      w[k] = pack_e4m3x4(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale), __fdiv_rn(c.x, scale),
                         __fdiv_rn(c.y, scale));
    }
    const int64_t o = (row * p.heads + h) * 128 + part * 8;
    *reinterpret_cast<uint2*>(p.out + o) = make_uint2(w[0], w[1]);
    }
  }
}

__global__ void descale_kernel(const __grid_constant__ QuantBatch pb) {
  const QuantParams& p = pb.t[blockIdx.y];
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h < p.heads) p.amax[h] = fmaxf(p.amax[h], 1e-12f) / 448.f;
}

}  // namespace dgxm

extern "C" int dgxm_qkv_prologue_scatter(const dgxm_prologue_desc* d, const void* const* src,
                                         const void* norm_q_w, const void* norm_k_w,
                                         const float* rope, void* const* dst, void* stream) {
  using namespace dgxm;
  if (d == nullptr || src == nullptr || dst == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL prologue argument");
  if (d->world < 1 || d->world > DGXM_MAX_WORLD || d->rank < 0 || d->rank >= d->world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", d->rank, d->world);
  if (d->head_dim != 128) return fail(DGXM_ERR_UNSUPPORTED, "prologue head_dim must be 128");
  if (d->heads <= 0 || d->heads % d->world || d->heads * 128 > kPrologueMaxHidden)
    return fail(DGXM_ERR_INVALID, "%d heads: not divisible by %d or above %d hidden", d->heads,
                d->world, kPrologueMaxHidden);
  if (d->norm_mode < DGXM_NORM_NONE || d->norm_mode > DGXM_NORM_HEAD)
    return fail(DGXM_ERR_INVALID, "unknown norm mode %d", d->norm_mode);
  if (d->seg0 < 0 || d->seg0 >= d->seq_local)
    return fail(DGXM_ERR_INVALID, "joint segment of %d rows does not split %d local rows", d->seg0,
                d->seq_local);
  if (d->batch <= 0 || d->seq_local <= 0) return DGXM_OK;
  PrologueParams p;
  memset(&p, 0, sizeof(p));
  for (int t = 0; t < 3; ++t) {
    if (src[t] == nullptr || reinterpret_cast<uintptr_t>(src[t]) % 16)
      return fail(DGXM_ERR_INVALID, "source %d is NULL or misaligned", t);
    p.src[t] = static_cast<const char*>(src[t]);
    p.s_sb[t] = d->src_stride[t][0] * 2;
    p.s_sl[t] = d->src_stride[t][1] * 2;
    p.s_sh[t] = d->src_stride[t][2] * 2;
    if (p.s_sb[t] % 16 || p.s_sl[t] % 16 || p.s_sh[t] % 16)
      return fail(DGXM_ERR_INVALID, "source %d strides are not 16-byte multiples", t);
    for (int r = 0; r < d->world; ++r) {
      void* q = dst[t * d->world + r];
      if (q == nullptr || reinterpret_cast<uintptr_t>(q) % 16)
        return fail(DGXM_ERR_INVALID, "destination %d of tensor %d is NULL or misaligned", r, t);
      p.dst[t][r] = static_cast<char*>(q);
    }
  }
  if (d->norm_mode != DGXM_NORM_NONE && (norm_q_w == nullptr) != (norm_k_w == nullptr))
    return fail(DGXM_ERR_INVALID, "give both norm weights or neither");
  if ((reinterpret_cast<uintptr_t>(norm_q_w) | reinterpret_cast<uintptr_t>(norm_k_w)) % 16)
    return fail(DGXM_ERR_INVALID, "norm weights must be 16-byte aligned");
  p.norm_w[0] = static_cast<const __nv_bfloat16*>(norm_q_w);
  p.norm_w[1] = static_cast<const __nv_bfloat16*>(norm_k_w);
  p.rope = rope;
  p.rope_sb = d->rope_batch_stride;
  p.norm_mode = d->norm_mode;
  p.eps = d->eps;
  p.world = d->world;
  p.rank = d->rank;
  p.batch = d->batch;
  p.seq_local = d->seq_local;
  p.heads = d->heads;
  p.seg0 = d->seg0;
  int dev = 0, sms = 148;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  DGXM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t rows = static_cast<int64_t>(d->batch) * d->seq_local;
  if (d->norm_mode != DGXM_NORM_HIDDEN) {
    // Per-head norm or none: nothing couples the heads of a row.
    const int blocks = static_cast<int>(rows < int64_t(sms) * 16 ? rows : int64_t(sms) * 16);
    qkv_prologue_head_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    DGXM_CUDA_TRY(cudaGetLastError());
    return DGXM_OK;
  }
  const int blocks = static_cast<int>(rows < int64_t(sms) * 8 ? rows : int64_t(sms) * 8);
  qkv_prologue_scatter_kernel<<<blocks, kPrologueThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

namespace dgxm {
// Checks of one quantisation item; fills its kernel parameters.
static int quant_item(const dgxm_quant_item& it, QuantParams* p) {
  if (it.x == nullptr || it.out == nullptr || it.descale == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL quantisation argument");
  if (it.head_dim != 128) return fail(DGXM_ERR_UNSUPPORTED, "quantisation head_dim must be 128");
  if (it.batch < 0 || it.rows < 0 || it.heads <= 0) return fail(DGXM_ERR_INVALID, "bad extents");
  if (it.heads > 64)
    return fail(DGXM_ERR_UNSUPPORTED, "quantisation supports up to 64 heads, got %d", it.heads);
  if (reinterpret_cast<uintptr_t>(it.x) % 16 || reinterpret_cast<uintptr_t>(it.out) % 16 ||
      (it.stride[0] * 2) % 16 || (it.stride[1] * 2) % 16 || (it.stride[2] * 2) % 16)
    return fail(DGXM_ERR_INVALID, "quantisation tensors must be 16-byte aligned");
  if (it.keep_batch_stride < 0) return fail(DGXM_ERR_INVALID, "negative keep-bit batch stride");
  p->x = static_cast<const char*>(it.x);
  p->sb = it.stride[0] * 2;
  p->sl = it.stride[1] * 2;
  p->sh = it.stride[2] * 2;
  p->out = static_cast<uint8_t*>(it.out);
  p->amax = it.descale;
  p->keep = it.keep;
  p->keep_sb = it.keep_batch_stride;
  p->batch = it.batch;
  p->rows = it.rows;
  p->heads = it.heads;
  return DGXM_OK;
}

// Every item is checked before anything is launched; then one memset per
// descale vector and three launches cover all items.
static int quantize_e4m3_batch(int32_t n, const dgxm_quant_item* items, void* stream) {
  if (items == nullptr || n < 1 || n > kMaxQuantItems)
    return fail(DGXM_ERR_INVALID, "quantisation batches take 1 to %d items, got %d", kMaxQuantItems, n);
  QuantBatch pb;
  memset(&pb, 0, sizeof(pb));
  int64_t max_rows = 0;
  int max_heads = 1;
  for (int i = 0; i < n; ++i) {
    if (int rc = quant_item(items[i], &pb.t[i])) return rc;
    max_rows = std::max<int64_t>(max_rows, static_cast<int64_t>(items[i].batch) * items[i].rows);
    max_heads = std::max(max_heads, static_cast<int>(items[i].heads));
  }
  pb.n = n;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i)
    DGXM_CUDA_TRY(cudaMemsetAsync(items[i].descale, 0, sizeof(float) * items[i].heads, st));
  if (max_rows == 0) return DGXM_OK;
  int dev = 0, sms = 148;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  DGXM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  // Blocks beyond an item's rows find no work in their stride loop.
  const int amax_blocks = static_cast<int>(std::min<int64_t>(max_rows, int64_t(sms) * 4));
  const int amax_threads = (max_heads * 16 + 31) / 32 * 32;
  absmax_kernel<<<dim3(amax_blocks, n), amax_threads, 0, st>>>(pb);
  const int qblocks = static_cast<int>(std::min<int64_t>(max_rows, int64_t(sms) * 8));
  quantize_e4m3_kernel<<<dim3(qblocks, n), 256, 0, st>>>(pb);
  descale_kernel<<<dim3(1, n), 64, 0, st>>>(pb);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}
}  // namespace dgxm

extern "C" int dgxm_quantize_e4m3_per_head(int32_t batch, int32_t rows, int32_t heads,
                                           int32_t head_dim, const void* x, const int64_t* stride,
                                           void* out, float* descale, void* stream) {
  if (stride == nullptr) return dgxm::fail(DGXM_ERR_INVALID, "NULL quantisation argument");
  dgxm_quant_item it{batch, rows, heads, head_dim, x, {stride[0], stride[1], stride[2]},
                     nullptr, 0, out, descale};
  return dgxm::quantize_e4m3_batch(1, &it, stream);
}

extern "C" int dgxm_quantize_e4m3_per_head_masked(int32_t batch, int32_t rows, int32_t heads,
                                                  int32_t head_dim, const void* x,
                                                  const int64_t* stride, const uint32_t* keep,
                                                  int64_t keep_batch_stride, void* out,
                                                  float* descale, void* stream) {
  if (keep == nullptr) return dgxm::fail(DGXM_ERR_INVALID, "NULL keep bits");
  if (stride == nullptr) return dgxm::fail(DGXM_ERR_INVALID, "NULL quantisation argument");
  dgxm_quant_item it{batch, rows, heads, head_dim, x, {stride[0], stride[1], stride[2]},
                     keep, keep_batch_stride, out, descale};
  return dgxm::quantize_e4m3_batch(1, &it, stream);
}

extern "C" int dgxm_quantize_e4m3_per_head_batch(int32_t n, const dgxm_quant_item* items,
                                                 void* stream) {
  return dgxm::quantize_e4m3_batch(n, items, stream);
}
