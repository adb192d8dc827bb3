// Non-causal attention forward for sm_100a (B200): tcgen05 MMAs with TMEM
// accumulators, TMA-staged Q/K/V tiles, warp-specialised online softmax.
//
// One CTA owns 256 query rows of one (batch, head): two 128-row Q tiles that
// ping-pong on the tensor core.  While the softmax warpgroup of tile 0 turns
// S0 = Q0 K_j^T into probabilities, the tensor core computes P1 V_{j-1} and
// S1 = Q1 K_j^T, and vice versa, so the exponentials overlap the MMAs.
//
// Warp roles (18 warps, 576 threads):
//   warps 0-7   softmax + output correction + epilogue for Q tile 0: two
//               threads per row, warps 0-3 own key columns 0-63 of the
//               tile's rows, warps 4-7 columns 64-127
//   warps 8-15  the same for Q tile 1
//   warp  16    TMA producer (Q once, then K_j / V_j through a stage ring)
//   warp  17    TMEM allocator and single-thread MMA issuer
//
// Tensor memory (512 columns x 128 lanes x 32 bit):
//   [  0,128) S0 (fp32 logits); P0 overwrites its first columns (bf16 pairs
//             or e4m3 quads) once the softmax has read S0
//   [128,256) S1 / P1
//   [256,384) O0 (fp32 output accumulator)
//   [384,512) O1
//
// Shared memory: Q tiles (2 x 128 rows x 128 cols) then a ring of K/V stages,
// every tile stored as 128-byte rows with the 128-byte swizzle that both TMA
// and the MMA shared-memory descriptors use.
//
// The math follows the per-block contract of the reference's ring processor
// (adapters/cudnn_ring_attention.py:61-89): out = softmax(scale * Q K^T) V and
// the fp32 natural-log LSE of the scaled logits, per (batch, head, row).
#include "common.h"
#include "device_error.cuh"
#include "ptx.cuh"

// Softmax instruction choices (all compute the same function):
//   DGXM_SM_MAX3      three-input max for the row reduction
//   DGXM_SM_POLY_MOD  every N-th pair of exponentials on the FMA pipe
//                     (exp2_poly2) instead of MUFU; 0 (the default) runs
//                     every exponential on MUFU.  With P released in 4
//                     chunks the MUFU-only loop is the fastest: the per-block
//                     period at 75,600 keys is 3749 clocks against 3802 (1/16
//                     on the FMA pipe), 3839 (1/8) and 4002 (1/4).
#ifndef DGXM_SM_MAX3
#define DGXM_SM_MAX3 1
#endif
#ifndef DGXM_SM_POLY_MOD
#define DGXM_SM_POLY_MOD 0
#endif
#ifndef DGXM_SM_PAIR_BARRIER
#define DGXM_SM_PAIR_BARRIER 1  // exchange row halves over a 64-thread barrier per warp pair
#endif
#ifndef DGXM_SM_WARP_ARRIVE
#define DGXM_SM_WARP_ARRIVE 1  // one P-release arrival per softmax warp (0: one per thread)
#endif
#ifndef DGXM_SM_THR_BF16
#define DGXM_SM_THR_BF16 8.0f  // stale-max threshold of the bf16 kernel (log2 units)
#endif
// P is released to the tensor core in 1, 2 or 4 chunks per block (at most 2
// for e4m3), chosen per call (DGXM_ATTN_P_CHUNKS in the descriptor flags;
// this default when the flags leave it 0).  With more than one, each softmax
// thread stores and signals a chunk of its probabilities as soon as they are
// computed, and the MMA issuer starts the P.V steps of that chunk while the
// rest is still in the exponential loop: the softmax -> P.V dependency that
// bounds the block time shrinks by the later chunks' share of the loop.
#ifndef DGXM_SM_P_CHUNKS
#define DGXM_SM_P_CHUNKS 4
#endif

namespace dgxm {

constexpr int kSoftmaxWarps = 16;  // 2 tiles x 2 column halves x 4 lane quarters
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;        // allocates TMEM and issues every MMA (one thread)
constexpr int kAttnThreads = 18 * 32;
constexpr int kCtrlXmaxOffset = 1024;  // row-max / row-sum exchange area inside the control block
constexpr int kTileRows = 128;   // rows per Q tile and per K/V tile
constexpr int kHeadDim = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// HD: the head dimension, 128 or (16-bit inputs) 64.
template <bool FP8, bool F16 = false, int HD = kHeadDim>
struct AttnCfg {
  static_assert(HD == 128 || (HD == 64 && !FP8), "head dimension 128, or 64 for 16-bit inputs");
  static constexpr int kEltBytes = FP8 ? 1 : 2;
  static constexpr int kBoxCols = 128 / kEltBytes;          // elements in one 128-byte row
  static constexpr int kBoxes = HD / kBoxCols;              // 128-byte column blocks per tile
  static constexpr int kBoxBytes = kTileRows * 128;         // 16 KB
  static constexpr int kTileBytes = kBoxes * kBoxBytes;     // one 128-row tile
  static constexpr int kStages = (FP8 || HD == 64) ? 8 : 4;
  static constexpr int kMmaK = FP8 ? 32 : 16;               // K extent of one MMA
  static constexpr int kKSteps = HD / kMmaK;                // MMAs per Q K^T product
  static constexpr int kPCols = kTileRows * kEltBytes / 4;  // TMEM columns holding P
  // Stale-max threshold (log2 units) below which the running max is kept and
  // O is not rescaled; P values then stay below 2^kThr.
  static constexpr float kThr = FP8 ? 4.0f : DGXM_SM_THR_BF16;
  // e4m3 probabilities are stored scaled by 2^4 so typical values sit in the
  // normal range; the epilogue divides the factor back out.
  static constexpr float kPScale = FP8 ? 16.0f : 1.0f;
  static constexpr float kPScaleLog2 = FP8 ? 4.0f : 0.0f;
  // Operand format: e4m3 (kind::f8f6f4) 0; under kind::f16, f16 0 and bf16 1.
  // P takes the inputs' 16-bit format, so A and B of P.V always match.
  static constexpr uint32_t kFmt = FP8 ? 0u : (F16 ? 0u : 1u);
  static constexpr uint32_t kIdescQK = idesc_make(128, 128, kFmt, false);
  static constexpr uint32_t kIdescPV = idesc_make(128, HD, kFmt, true);
  // CTA-pair products: M256, each CTA holding 128 of the rows.
  static constexpr uint32_t kIdescQK2 = idesc_make(256, 128, kFmt, false);
  static constexpr uint32_t kIdescPV2 = idesc_make(256, HD, kFmt, true);
  static constexpr int kSmemBytes = 1024 /*align slack*/ + 2 * kTileBytes + kStages * kTileBytes +
                                    1024 /*barriers + slots*/ + 12 * 128 * 4 /*row exchange*/;
};

// P chunks of a kernel built for NCH: e4m3 blocks hold whole 32-key MMA
// steps per column half only up to two chunks.
template <bool FP8, int NCH>
__host__ __device__ constexpr int p_chunks() {
  static_assert(NCH == 1 || NCH == 2 || NCH == 4, "P chunks: 1, 2 or 4");
  return (FP8 && NCH > 2) ? 2 : NCH;
}

struct __align__(64) AttnParams {
  CUtensorMap tmap_q;  // dims (D, H, L, B), box (128 bytes, 1, 128, 1)
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  void* o;
  float* lse;
  const float* q_descale;
  const float* k_descale;
  const float* v_descale;
  int64_t o_sb, o_sl, o_sh;
  int64_t lse_sb, lse_sh, lse_sl;
  int q_len, kv_len, q_heads, kv_heads;
  int n_kv_tiles;
  float scale_log2;
  int flags;
  // Fused inverse all-to-all: when o_rows > 0, query row i goes to
  // o_peer[i / o_rows] at row i % o_rows and head o_head_off + h.
  void* o_peer[DGXM_MAX_WORLD];
  int o_rows;
  int o_head_off;
  int o_world;
  int o_seg0;  // joint order of the gathered axis (0 = rank-major)
  // Replicated text: o_txt rows before (o_txt_front) or after the o_img_rows
  // image rows; a text row goes to every rank's o_txt_peer tensor.
  int o_txt, o_txt_front, o_img_rows;
  int64_t o_txt_sb;
  void* o_txt_peer[DGXM_MAX_WORLD];
  // Extras (the EXTRA kernel variant only): keep bits over keys (0 excludes
  // the key) and over query rows (0 writes a zero output row), and additive
  // biases for query-row groups, added to the scaled logits.
  const uint32_t* kmask;
  int64_t kmask_sb;  // words
  int kmask_words;
  const uint32_t* qmask;
  int64_t qmask_sb;
  int n_bias;
  int bias_q0[DGXM_MAX_BIAS_GROUPS], bias_q1[DGXM_MAX_BIAS_GROUPS];
  const float* bias[DGXM_MAX_BIAS_GROUPS];
  int64_t bias_sb[DGXM_MAX_BIAS_GROUPS], bias_sh[DGXM_MAX_BIAS_GROUPS], bias_sq[DGXM_MAX_BIAS_GROUPS];
  int bias_len[DGXM_MAX_BIAS_GROUPS];
  float inv_scale;
};

// Barrier slots inside the control block.
template <int kStages, int kPChunks>
struct Bars {
  static constexpr int kQ = 0;
  static constexpr int kKvFull = 1;
  static constexpr int kKvEmpty = kKvFull + kStages;
  static constexpr int kSFull = kKvEmpty + kStages;  // 2
  static constexpr int kPFull = kSFull + 2;          // 2 tiles x kPChunks, tile-major
  static constexpr int kOFull = kPFull + 2 * kPChunks;  // 2
  static constexpr int kPvDone = kOFull + 2;         // 2
  static constexpr int kDrain = kPvDone + 2;
  static constexpr int kCount = kDrain + 1;
};

// Shared-memory descriptors split into a low word (start address in 16-byte
// units | leading byte offset) and a constant high word (stride byte offset,
// sm100 version, 128-byte swizzle).  The MMA issuer keeps one low word per
// tile and adds compile-time offsets, so each MMA costs one integer add per
// operand: the issuing thread shares its SM sub-partition with softmax warps
// and must not spend its issue slots on descriptor arithmetic.
__host__ __device__ constexpr uint32_t sdesc_hi(uint32_t sbo_bytes) {
  return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);
}

__device__ __forceinline__ uint32_t sdesc_lo(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}

__device__ __forceinline__ uint64_t sdesc_join(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}

// S = Q K^T: both operands K-major, one 128-byte swizzle atom per 64 (bf16)
// or 128 (e4m3) head-dim columns.  q_lo / k_lo are the tiles' low words.
template <bool FP8, bool F16, int HD>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_lo, uint32_t k_lo) {
  using C = AttnCfg<FP8, F16, HD>;
  constexpr uint32_t hi = sdesc_hi(1024);
#pragma unroll
  for (int kk = 0; kk < C::kKSteps; ++kk) {
    const uint32_t byte = kk * 32;  // each MMA consumes 32 bytes of the head dimension
    const uint32_t off = ((byte / 128) * C::kBoxBytes + (byte % 128)) >> 4;
    const uint64_t a = sdesc_join(q_lo + off, hi);
    const uint64_t b = sdesc_join(k_lo + off, hi);
    if constexpr (FP8)
      umma_f8_ss(d_tmem, a, b, C::kIdescQK, kk > 0 ? 1u : 0u);
    else
      umma_f16_ss(d_tmem, a, b, C::kIdescQK, kk > 0 ? 1u : 0u);
  }
}

// The CTA-pair S = Q K^T: each CTA holds its own Q tile and 64 of the
// block's 128 keys (64-row boxes, kBoxBytes / 2 apart), and the even CTA's
// M256 N128 products write both CTAs' S tiles.
template <bool F16, int HD>
__device__ __forceinline__ void issue_qk_pair(uint32_t d_tmem, uint32_t q_lo, uint32_t k_lo) {
  using C = AttnCfg<false, F16, HD>;
  constexpr uint32_t hi = sdesc_hi(1024);
#pragma unroll
  for (int kk = 0; kk < C::kKSteps; ++kk) {
    const uint32_t byte = kk * 32;
    const uint32_t off_q = ((byte / 128) * C::kBoxBytes + (byte % 128)) >> 4;
    const uint32_t off_k = ((byte / 128) * (C::kBoxBytes / 2) + (byte % 128)) >> 4;
    umma_f16_ss_pair(d_tmem, sdesc_join(q_lo + off_q, hi), sdesc_join(k_lo + off_k, hi), C::kIdescQK2,
                     kk > 0 ? 1u : 0u);
  }
}

template <bool FP8, bool F16, int HD, bool PAIR>
__device__ __forceinline__ void issue_qk_any(uint32_t d_tmem, uint32_t q_lo, uint32_t k_lo) {
  if constexpr (PAIR)
    issue_qk_pair<F16, HD>(d_tmem, q_lo, k_lo);
  else
    issue_qk<FP8, F16, HD>(d_tmem, q_lo, k_lo);
}

// O += P V: P from tensor memory, V MN-major (head_dim along the 128-byte
// rows, keys down the rows; the second 128-byte column block of bf16 sits
// kBoxBytes further, the leading byte offset).
template <bool FP8, bool F16, int HD>
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_lo,
                                         bool accumulate) {
  using C = AttnCfg<FP8, F16, HD>;
  constexpr uint32_t hi = sdesc_hi(1024);
#pragma unroll
  for (int kk = 0; kk < C::kKSteps; ++kk) {
    const uint64_t b = sdesc_join(v_lo + ((kk * C::kMmaK * 128) >> 4), hi);
    const uint32_t a = p_tmem + kk * (C::kMmaK * C::kEltBytes / 4);
    const uint32_t acc = (accumulate || kk > 0) ? 1u : 0u;
    if constexpr (FP8)
      umma_f8_ts(d_tmem, a, b, C::kIdescPV, acc);
    else
      umma_f16_ts(d_tmem, a, b, C::kIdescPV, acc);
  }
}

// The P V steps of one P chunk: the keys [64 c + ch K, 64 c + (ch + 1) K) of
// both column halves c, K = 64 / kPChunks -- the probabilities one chunk of
// every softmax thread has stored.  The first step of chunk 0 starts the
// accumulation when `accumulate` is false.
// PAIR: the CTA-pair product, each CTA's P in its own TMEM and 64 of the head
// dimensions of V (one 128-byte column block of all 128 keys) in its own
// shared memory.
template <bool FP8, bool F16, int HD, int kPChunks, bool PAIR = false>
__device__ __forceinline__ void issue_pv_chunk(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_lo,
                                               bool accumulate, int ch) {
  using C = AttnCfg<FP8, F16, HD>;
  constexpr uint32_t hi = sdesc_hi(1024);
  constexpr int kKeys = 64 / kPChunks;         // keys of one column half in one chunk
  constexpr int kSteps = kKeys / C::kMmaK;     // MMAs per column half per chunk
  static_assert(kSteps >= 1 && kKeys % C::kMmaK == 0, "a chunk holds whole MMA K steps");
#pragma unroll
  for (int c = 0; c < 2; ++c) {
#pragma unroll
    for (int q = 0; q < kSteps; ++q) {
      const int kk = (c * 64 + ch * kKeys) / C::kMmaK + q;
      const uint64_t b = sdesc_join(v_lo + ((kk * C::kMmaK * 128) >> 4), hi);
      const uint32_t a = p_tmem + kk * (C::kMmaK * C::kEltBytes / 4);
      const uint32_t acc = (accumulate || ch > 0 || c > 0 || q > 0) ? 1u : 0u;
      if constexpr (PAIR)
        umma_f16_ts_pair(d_tmem, a, b, C::kIdescPV2, acc);
      else if constexpr (FP8)
        umma_f8_ts(d_tmem, a, b, C::kIdescPV, acc);
      else
        umma_f16_ts(d_tmem, a, b, C::kIdescPV, acc);
    }
  }
}

// O += P V of one tile, chunk by chunk as the softmax releases P: each chunk
// waits for its own barrier.  Returns false when a wait gave up.
template <bool FP8, bool F16, int HD, int kPChunks, int kBarPFull, bool PAIR = false>
__device__ __forceinline__ bool issue_pv_chunks(uint64_t* bars, uint32_t d_tmem, uint32_t p_tmem,
                                                uint32_t v_lo, bool accumulate, int parity,
                                                volatile int* abort_flag) {
#pragma unroll
  for (int ch = 0; ch < kPChunks; ++ch) {
    if (!mbar_wait(smem_u32(&bars[kBarPFull + ch]), parity, abort_flag)) return false;
    tc_fence_after();
    issue_pv_chunk<FP8, F16, HD, kPChunks, PAIR>(d_tmem, p_tmem, v_lo, accumulate, ch);
  }
  return true;
}

// Release one P chunk of a softmax warp.  Every thread has waited for its
// own TMEM stores and fenced them; the warp then meets, and one arrival per
// warp (or per thread) goes to the chunk's barrier.  Fewer arrivals mean
// fewer shared-memory atomics on the barrier the MMA issuer is testing.
__device__ __forceinline__ void release_p(uint32_t b, int lane) {
  if (DGXM_SM_WARP_ARRIVE) {
    __syncwarp();
    if (lane == 0) mbar_arrive(b);
  } else {
    mbar_arrive(b);
  }
}

// The CTA-pair release: one arrival per warp of either CTA on the even CTA's
// chunk barrier (a shared::cluster address).  The arrival is relaxed: what it
// hands over is P in this CTA's TMEM, whose stores every thread of the warp
// has completed (tcgen05.wait::st) and fenced (tcgen05.fence::before_thread_
// sync) before the warp meets, and the issuer orders its products after its
// wait with tcgen05.fence::after_thread_sync; the issuer reads nothing the
// softmax writes through generic memory.  A release at cluster scope would
// make every softmax warp wait for its earlier shared-memory traffic to
// become visible to the peer SM at each of the 8 hand-offs per block: that
// measured 740 against 1188 TFLOP/s at 75,600 keys.
__device__ __forceinline__ void release_p_pair(uint32_t leader_bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster_relaxed(leader_bar);
}

// Commit of the MMA issuer: to this CTA's barrier, or for a CTA pair to the
// barrier at the same offset in both CTAs.
template <bool PAIR>
__device__ __forceinline__ void attn_commit(uint32_t bar) {
  if constexpr (PAIR)
    umma_commit_pair_to(bar, 0x3);
  else
    umma_commit(bar);
}

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, int bits) {
  report_device_error(bits);
  *abort_flag = 1;
}

// K/V ring stages of a CTA-pair kernel (16 KB each: half a block of K or V);
// 8 holds the same bytes as the single-CTA ring.
#ifndef DGXM_PAIR_STAGES
#define DGXM_PAIR_STAGES 8
#endif
constexpr int kPairStages = DGXM_PAIR_STAGES;

// Dynamic shared memory of a kernel variant: a pair's ring of kPairStages
// half-tile stages in place of the single-CTA ring.
template <bool FP8, bool F16, int HD, bool PAIR>
__host__ __device__ constexpr int attn_smem_bytes() {
  using C = AttnCfg<FP8, F16, HD>;
  return PAIR ? C::kSmemBytes - C::kStages * C::kTileBytes + kPairStages * (C::kTileBytes / 2) : C::kSmemBytes;
}

// F16: 16-bit inputs (and P) are fp16 instead of bf16; a 16-bit output is
// then fp16 too.
//
// PAIR: the kernel runs as clusters of two CTAs on the two SMs of a TPC, one
// tcgen05 pair.  Each CTA keeps its two Q tiles, its S, P and O in its own
// TMEM and its own softmax; a K/V stage holds half of a block (K: 64 of the
// 128 keys; V: 64 of the head dimensions of all keys), so each SM loads half
// the K/V bytes.  The even CTA issues M256 products over both CTAs' operands
// -- half the MMAs per FLOP of one CTA -- and its commits signal both CTAs;
// the loads of both CTAs and the P releases of both CTAs' softmax warps are
// counted on the even CTA's barriers.
template <bool FP8, bool OUT_F32, bool EXTRA, int NCH, bool F16, int HD, bool PAIR>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_fwd_kernel(const __grid_constant__ AttnParams p) {
  using C = AttnCfg<FP8, F16, HD>;
  constexpr int kPChunks = p_chunks<FP8, NCH>();
  static_assert(!PAIR || (!FP8 && HD == kHeadDim && kPChunks > 1 && DGXM_SM_WARP_ARRIVE),
                "CTA pairs: 16-bit inputs, head dim 128, chunked P release, one arrival per warp");
  constexpr int kStageBytes = PAIR ? C::kTileBytes / 2 : C::kTileBytes;
  constexpr int kStages = PAIR ? kPairStages : C::kStages;
  static_assert(attn_smem_bytes<FP8, F16, HD, PAIR>() <= 227 * 1024, "shared memory of one CTA");
  using B = Bars<kStages, kPChunks>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t sQ = base;
  const uint32_t sKV = base + 2 * C::kTileBytes;
  uint8_t* ctrl = smem + 2 * C::kTileBytes + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ctrl);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ctrl + B::kCount * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar(B::kQ), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B::kKvFull + s), 1);
      mbar_init(bar(B::kKvEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B::kSFull + t), 1);
      for (int ch = 0; ch < kPChunks; ++ch)
        mbar_init(bar(B::kPFull + t * kPChunks + ch), PAIR ? 16 : (DGXM_SM_WARP_ARRIVE ? 8 : 256));
      mbar_init(bar(B::kOFull + t), 1);
      mbar_init(bar(B::kPvDone + t), 1);
    }
    mbar_init(bar(B::kDrain), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&p.tmap_q);
    tma_prefetch_desc(&p.tmap_k);
    tma_prefetch_desc(&p.tmap_v);
  }
  if (warp == kMmaWarp) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t cta = PAIR ? cluster_ctarank() : 0u;  // 0 issues a pair's MMAs

  const int qtile = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (p.q_heads / p.kv_heads);
  const int row0 = qtile * 2 * kTileRows;
  const int nkv = p.n_kv_tiles;
  const bool safe_order = (p.flags & DGXM_ATTN_SAFE_ORDER) != 0;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued_count = 0;  // loads issued into the K/V ring so far
      bool ok = true;
      const uint64_t keep = l2_policy_evict_last();   // K/V are re-read by every Q tile
      const uint64_t once = l2_policy_evict_first();  // Q is read by this CTA only
      if constexpr (PAIR) {
        // Both CTAs' loads count on the even CTA's barriers.
        if (cta == 0) mbar_expect_tx(bar(B::kQ), 4 * C::kTileBytes);
        const uint32_t qbar = mapa_shared(bar(B::kQ), 0);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < C::kBoxes; ++c)
            tma_load_4d_pair_hint(sQ + t * C::kTileBytes + c * C::kBoxBytes, &p.tmap_q, qbar,
                                  c * C::kBoxCols, h, row0 + t * kTileRows, b, once);
      } else {
        mbar_expect_tx(bar(B::kQ), 2 * C::kTileBytes);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < C::kBoxes; ++c)
            tma_load_4d_hint(sQ + t * C::kTileBytes + c * C::kBoxBytes, &p.tmap_q, bar(B::kQ),
                             c * C::kBoxCols, h, row0 + t * kTileRows, b, once);
      }
      for (int idx = 0; idx < 2 * nkv; ++idx) {
        const int s = idx % kStages;
        const int ph = (idx / kStages) & 1;
        if (!mbar_wait(bar(B::kKvEmpty + s), ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        if constexpr (PAIR) {
          // K: this CTA's 64 keys of the block, both 128-byte column blocks
          // (tmap_k has 64-row boxes); V: this CTA's 128-byte column block of
          // all 128 keys.
          if (cta == 0) mbar_expect_tx(bar(B::kKvFull + s), 2 * kStageBytes);
          const uint32_t fbar = mapa_shared(bar(B::kKvFull + s), 0);
          const uint32_t dst = sKV + s * kStageBytes;
          if (idx & 1) {
            tma_load_4d_pair_hint(dst, &p.tmap_v, fbar, static_cast<int>(cta) * C::kBoxCols, hk,
                                  (idx >> 1) * kTileRows, b, keep);
          } else {
            for (int c = 0; c < C::kBoxes; ++c)
              tma_load_4d_pair_hint(dst + c * (C::kBoxBytes / 2), &p.tmap_k, fbar, c * C::kBoxCols, hk,
                                    (idx >> 1) * kTileRows + static_cast<int>(cta) * (kTileRows / 2), b,
                                    keep);
          }
        } else {
          mbar_expect_tx(bar(B::kKvFull + s), C::kTileBytes);
          const void* map = (idx & 1) ? static_cast<const void*>(&p.tmap_v)
                                      : static_cast<const void*>(&p.tmap_k);
          for (int c = 0; c < C::kBoxes; ++c)
            tma_load_4d_hint(sKV + s * C::kTileBytes + c * C::kBoxBytes, map,
                             bar(B::kKvFull + s), c * C::kBoxCols, hk, (idx >> 1) * kTileRows, b,
                             keep);
        }
        issued_count = idx + 1;
      }
      if (!ok) {
        raise_abort(abort_flag, kErrProducerTimeout);
        // Let the copies already in flight land before the CTA can exit (a
        // pair's loads all report on the even CTA's barriers, which the odd
        // CTA cannot test: it gives its own copies a fixed 50 us instead).
        if (cta == 0) {
          mbar_wait(bar(B::kQ), 0, nullptr);
          const int first = issued_count > kStages ? issued_count - kStages : 0;
          for (int idx = first; idx < issued_count; ++idx)
            mbar_wait(bar(B::kKvFull + idx % kStages), (idx / kStages) & 1, nullptr);
        } else {
          for (int i = 0; i < 50; ++i) __nanosleep(1000);
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // One thread issues both tiles' products in the order
    //   S0_j = Q0 K_j^T, O1 += P1_{j-1} V_{j-1}, S1_j = Q1 K_j^T, O0 += P0_j V_j
    // so each softmax group's exponentials overlap the other tile's two
    // products.  P_t sits in S_t's tensor memory, so S_t of the next block is
    // issued only after the P_t V that reads it (tcgen05 operations of one
    // thread execute in issue order; DGXM_ATTN_SAFE_ORDER drains instead).
    if (lane == 0 && cta == 0) {
      const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
      const uint32_t q0_lo = sdesc_lo(sQ, 16), q1_lo = sdesc_lo(sQ + C::kTileBytes, 16);
      const uint32_t kv_lo_k = sdesc_lo(sKV, 16);             // stage 0, K-major view
      const uint32_t kv_lo_v = sdesc_lo(sKV, C::kBoxBytes);   // stage 0, MN-major view
      constexpr uint32_t kStageLo = kStageBytes >> 4;        // low-word step per stage
      bool ok = mbar_wait(bar(B::kQ), 0, abort_flag);
      tc_fence_after();
      for (int j = 0; ok && j < nkv; ++j) {
        const int ki = 2 * j;
        const int ks = ki % kStages;
        if (!(ok = mbar_wait(bar(B::kKvFull + ks), (ki / kStages) & 1, abort_flag))) break;
        tc_fence_after();
        // S0 = Q0 K_j^T
        if (safe_order && j > 0) {
          if (!(ok = mbar_wait(bar(B::kPvDone + 0), (j - 1) & 1, abort_flag))) break;
          tc_fence_after();
        }
        issue_qk_any<FP8, F16, HD, PAIR>(tS0, q0_lo, kv_lo_k + ks * kStageLo);
        attn_commit<PAIR>(bar(B::kSFull + 0));
        // O1 += P1 V_{j-1}
        if (j > 0) {
          const int vs = (2 * j - 1) % kStages;
          if constexpr (kPChunks > 1) {
            if (!(ok = issue_pv_chunks<FP8, F16, HD, kPChunks, B::kPFull + kPChunks, PAIR>(
                      bars, tO1, tS1, kv_lo_v + vs * kStageLo, j - 1 > 0, (j - 1) & 1, abort_flag)))
              break;
          } else {
            if (!(ok = mbar_wait(bar(B::kPFull + 1), (j - 1) & 1, abort_flag))) break;
            tc_fence_after();
            issue_pv<FP8, F16, HD>(tO1, tS1, kv_lo_v + vs * kStageLo, j - 1 > 0);
          }
          attn_commit<PAIR>(bar(B::kKvEmpty + vs));
          if (safe_order) {
            attn_commit<PAIR>(bar(B::kPvDone + 1));
            if (!(ok = mbar_wait(bar(B::kPvDone + 1), (j - 1) & 1, abort_flag))) break;
            tc_fence_after();
          }
        }
        // S1 = Q1 K_j^T
        issue_qk_any<FP8, F16, HD, PAIR>(tS1, q1_lo, kv_lo_k + ks * kStageLo);
        attn_commit<PAIR>(bar(B::kSFull + 1));
        attn_commit<PAIR>(bar(B::kKvEmpty + ks));
        // O0 += P0 V_j
        const int vi = 2 * j + 1;
        const int vs = vi % kStages;
        if (!(ok = mbar_wait(bar(B::kKvFull + vs), (vi / kStages) & 1, abort_flag))) break;
        if constexpr (kPChunks > 1) {
          if (!(ok = issue_pv_chunks<FP8, F16, HD, kPChunks, B::kPFull, PAIR>(bars, tO0, tS0, kv_lo_v + vs * kStageLo, j > 0,
                                                     j & 1, abort_flag)))
            break;
        } else {
          if (!(ok = mbar_wait(bar(B::kPFull + 0), j & 1, abort_flag))) break;
          tc_fence_after();
          issue_pv<FP8, F16, HD>(tO0, tS0, kv_lo_v + vs * kStageLo, j > 0);
        }
        if (safe_order) attn_commit<PAIR>(bar(B::kPvDone + 0));
        if (j == nkv - 1) attn_commit<PAIR>(bar(B::kOFull + 0));
      }
      if (ok) {
        // O1 += P1 V_{n-1}
        const int vs = (2 * nkv - 1) % kStages;
        if constexpr (kPChunks > 1) {
          ok = issue_pv_chunks<FP8, F16, HD, kPChunks, B::kPFull + kPChunks, PAIR>(bars, tO1, tS1, kv_lo_v + vs * kStageLo,
                                                            nkv - 1 > 0, (nkv - 1) & 1, abort_flag);
        } else {
          ok = mbar_wait(bar(B::kPFull + 1), (nkv - 1) & 1, abort_flag);
          if (ok) {
            tc_fence_after();
            issue_pv<FP8, F16, HD>(tO1, tS1, kv_lo_v + vs * kStageLo, nkv - 1 > 0);
          }
        }
        if (ok) {
          attn_commit<PAIR>(bar(B::kKvEmpty + vs));
          attn_commit<PAIR>(bar(B::kOFull + 1));
        }
      }
      if (!ok) {
        raise_abort(abort_flag, kErrMmaTimeout);
        // Wait for the MMAs already issued before TMEM is released.
        if constexpr (PAIR)
          umma_commit_pair_to(bar(B::kDrain), 0x1);
        else
          umma_commit(bar(B::kDrain));
        mbar_wait(bar(B::kDrain), 0, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    // Two threads per query row: warps 4c..4c+3 of a tile's group own the
    // key columns [64c, 64c+64) of every row of their TMEM lane quarter.
    // The halves exchange row maxima through shared memory behind a named
    // barrier, so both apply the same running max; each keeps a partial row
    // sum and rescales / writes its own half of the output columns.
    const int t = warp / 8;          // Q tile of this group
    const int c = (warp / 4) & 1;    // column half
    const int sub = warp & 3;        // TMEM lane quarter this warp may access
    const int r = sub * 32 + lane;   // row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    // The two threads of a row sit in warps sub and sub + 4 of the group; they
    // meet on a barrier of their own warp pair, or of the whole group.
    const int xbar_id = DGXM_SM_PAIR_BARRIER ? 1 + t * 4 + sub : 1 + t;
    const int xbar_threads = DGXM_SM_PAIR_BARRIER ? 64 : 256;
    const uint32_t tS = tmem + lane_off + t * 128 + c * 64;
    const uint32_t tP = tmem + lane_off + t * 128 + c * (C::kPCols / 2);
    const uint32_t tO = tmem + lane_off + 256 + t * 128 + c * (HD / 2);  // this half's output columns
    float* xmax = reinterpret_cast<float*>(ctrl + kCtrlXmaxOffset);  // [2 parity][2 tile][2 half][128]
    const uint32_t pfull_leader = PAIR ? mapa_shared(bar(B::kPFull), 0) : 0u;  // the even CTA's chunk barriers
    float sl2 = p.scale_log2;
    if constexpr (FP8) sl2 *= p.q_descale[h] * p.k_descale[hk];
    float m_run = -INFINITY;  // running max of the scaled logits, log2 units
    float l_run = 0.f;        // this half's running sum of exp2(s * sl2 - m_run)
    // EXTRA: this row's bias group (if any).  A bias is in logit units and is
    // added to the raw dot products before they are scaled: divided by the
    // softmax scale, and for e4m3 inputs also by the q and k descales the raw
    // products leave out.
    const float* bias_row = nullptr;
    int bias_len = 0;
    float bias_mul = p.inv_scale;
    if constexpr (FP8 && EXTRA) bias_mul /= p.q_descale[h] * p.k_descale[hk];
    if constexpr (EXTRA) {
      const int qrow = row0 + t * kTileRows + r;
      for (int g = 0; g < p.n_bias; ++g) {
        if (qrow >= p.bias_q0[g] && qrow < p.bias_q1[g] && p.bias[g] != nullptr) {
          bias_row = p.bias[g] + static_cast<int64_t>(b) * p.bias_sb[g] +
                     static_cast<int64_t>(h) * p.bias_sh[g] +
                     static_cast<int64_t>(qrow - p.bias_q0[g]) * p.bias_sq[g];
          bias_len = p.bias_len[g];
        }
      }
    }
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const bool got = __all_sync(0xffffffffu, mbar_wait(bar(B::kSFull + t), j & 1, abort_flag));
      if (!got) raise_abort(abort_flag, kErrSoftmaxTimeout);
      uint32_t sr[2][32];
      if (got) {
        tc_fence_after();
        tmem_ld32(tS, sr[0]);
        tmem_ld32(tS + 32, sr[1]);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) sr[0][i] = sr[1][i] = 0u;
      }
      reg_fence32(sr[0]);
      reg_fence32(sr[1]);
      float s[64];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
        for (int i = 0; i < 32; ++i) s[h2 * 32 + i] = __uint_as_float(sr[h2][i]);
      const int valid = p.kv_len - j * kTileRows - c * 64;
      if constexpr (EXTRA) {
        const int key0 = j * kTileRows + c * 64;
        if (bias_row != nullptr) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (key0 + i < bias_len) s[i] += __ldg(bias_row + key0 + i) * bias_mul;
        }
        if (p.kmask != nullptr) {
          const uint32_t* km = p.kmask + static_cast<int64_t>(b) * p.kmask_sb;
          const int w = key0 >> 5;
          const uint32_t m0 = w < p.kmask_words ? __ldg(km + w) : 0u;
          const uint32_t m1 = w + 1 < p.kmask_words ? __ldg(km + w + 1) : 0u;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (!((m0 >> i) & 1u)) s[i] = -INFINITY;
            if (!((m1 >> i) & 1u)) s[32 + i] = -INFINITY;
          }
        }
      }
      if (valid < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= valid) s[i] = -INFINITY;
      }
#if DGXM_SM_MAX3
      float mx0 = fmax3(s[0], s[1], s[2]), mx1 = fmax3(s[3], s[4], s[5]);
      float mx2 = fmax3(s[6], s[7], s[8]), mx3 = fmax3(s[9], s[10], s[11]);
#pragma unroll
      for (int i = 12; i < 60; i += 8) {
        mx0 = fmax3(mx0, s[i], s[i + 1]);
        mx1 = fmax3(mx1, s[i + 2], s[i + 3]);
        mx2 = fmax3(mx2, s[i + 4], s[i + 5]);
        mx3 = fmax3(mx3, s[i + 6], s[i + 7]);
      }
      const float half_max = fmaxf(fmax3(mx0, mx1, fmax3(s[60], s[61], s[62])), fmax3(mx2, mx3, s[63]));
#else
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int i = 4; i < 64; i += 4) {
        mx0 = fmaxf(mx0, s[i]);
        mx1 = fmaxf(mx1, s[i + 1]);
        mx2 = fmaxf(mx2, s[i + 2]);
        mx3 = fmaxf(mx3, s[i + 3]);
      }
      const float half_max = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
#endif
      // Exchange with the other half of the row.  Double-buffered by
      // iteration parity: a buffer is rewritten two barriers after it was read.
      float* xm = xmax + ((j & 1) * 4 + t * 2) * 128;
      xm[c * 128 + r] = half_max;
      // Every warp of the group arrives here exactly once per iteration, and
      // all of them take the same stop decision, so the barrier counts of
      // later iterations can never mismatch.
      if (named_barrier_or(xbar_id, xbar_threads, !got || *abort_flag != 0)) {
        ok = false;
        break;
      }
      const float row_max = fmaxf(half_max, xm[(c ^ 1) * 128 + r]);
      const float m_cand = fmaxf(m_run, row_max * sl2);
      // Both halves of a row see the same maximum, so their warp votes agree.
      const bool grow = m_cand > m_run + C::kThr;
      float alpha = 1.f;
      bool rescale = false;
      if (__any_sync(0xffffffffu, grow)) {
        // 0 on the first block (m_run = -inf).  With extras a row can see
        // only excluded keys while another row of the warp grows; its
        // m_run = m_cand = -inf, and -inf - -inf must give 1, not NaN.
        alpha = ex2_approx((EXTRA && m_cand == -INFINITY) ? 0.f : m_run - m_cand);
        m_run = m_cand;
        rescale = j > 0;
      }
      l_run *= alpha;
      // p = 2^(s * sl2 - m) (times kPScale for e4m3, folded into the exponent).
      // A row whose keys so far were all excluded keeps m = -inf and p = 0.
      const float bias = -(EXTRA && m_run == -INFINITY ? 0.f : m_run) + C::kPScaleLog2;
      if constexpr (kPChunks > 1) {
        const uint64_t sl2x2 = pk2(sl2, sl2), biasx2 = pk2(bias, bias);
        uint64_t sum_a = pk2(0.f, 0.f), sum_b = pk2(0.f, 0.f);
        constexpr int kPairs = 32 / kPChunks;  // exponential pairs per chunk
#pragma unroll
        for (int ch = 0; ch < kPChunks; ++ch) {
          uint32_t pk[kPairs];
#pragma unroll
          for (int q = 0; q < kPairs; ++q) {
            const int i = ch * kPairs + q;
            uint64_t x = ffma2(pk2(s[2 * i], s[2 * i + 1]), sl2x2, biasx2);
            float p0, p1;
            if (DGXM_SM_POLY_MOD > 0 && (i % (DGXM_SM_POLY_MOD > 0 ? DGXM_SM_POLY_MOD : 1)) == 0) {
              x = exp2_poly2(x);
              upk2(x, p0, p1);
            } else {
              upk2(x, p0, p1);
              p0 = ex2_approx(p0);
              p1 = ex2_approx(p1);
              x = pk2(p0, p1);
            }
            if (i & 1) sum_b = fadd2(sum_b, x); else sum_a = fadd2(sum_a, x);
            if constexpr (FP8) {
              s[2 * i] = p0;
              s[2 * i + 1] = p1;
            } else {
              pk[q] = pack16<F16>(p0, p1);
            }
          }
          if constexpr (FP8) {
            // 2 kPairs keys of this chunk, four per column.
            uint32_t q8[kPairs / 2];
#pragma unroll
            for (int k = 0; k < kPairs / 2; ++k) {
              const int e = 2 * ch * kPairs + 4 * k;
              q8[k] = pack_e4m3x4(s[e], s[e + 1], s[e + 2], s[e + 3]);
            }
            tmem_st_n<kPairs / 2>(tP + ch * (kPairs / 2), q8);
          } else {
            tmem_st_n<kPairs>(tP + ch * kPairs, pk);
          }
          if (ch == 0 && rescale) {
            // O is rescaled before the first chunk is released, since the
            // P V of this block starts with that chunk.  O_t is quiescent
            // here: the commit behind this S_t also covered the previous
            // P_t V product.  Eight columns at a time, because the later
            // chunks' logits are still held in registers.
#pragma unroll
            for (int h8 = 0; h8 < HD / 16; ++h8) {
              uint32_t o[8];
              tmem_ld8(tO + h8 * 8, o);
              tmem_wait_ld();
              reg_fence8(o);
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st8(tO + h8 * 8, o);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          if constexpr (PAIR)
            release_p_pair(pfull_leader + (t * kPChunks + ch) * 8, lane);
          else
            release_p(bar(B::kPFull + t * kPChunks + ch), lane);
        }
        float a0, a1, b0, b1;
        upk2(sum_a, a0, a1);
        upk2(sum_b, b0, b1);
        l_run += ((a0 + a1) + (b0 + b1)) * (1.0f / C::kPScale);
      } else {
        const uint64_t sl2x2 = pk2(sl2, sl2), biasx2 = pk2(bias, bias);
        uint64_t sum_a = pk2(0.f, 0.f), sum_b = pk2(0.f, 0.f);
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          uint64_t x = ffma2(pk2(s[2 * i], s[2 * i + 1]), sl2x2, biasx2);
          float p0, p1;
          if (DGXM_SM_POLY_MOD > 0 && (i % (DGXM_SM_POLY_MOD > 0 ? DGXM_SM_POLY_MOD : 1)) == 0) {
            x = exp2_poly2(x);
            upk2(x, p0, p1);
          } else {
            upk2(x, p0, p1);
            p0 = ex2_approx(p0);
            p1 = ex2_approx(p1);
            x = pk2(p0, p1);
          }
          if (i & 1) sum_b = fadd2(sum_b, x); else sum_a = fadd2(sum_a, x);
          if constexpr (FP8) {
            s[2 * i] = p0;
            s[2 * i + 1] = p1;
          } else {
            pk[i] = pack16<F16>(p0, p1);
          }
        }
        {
          float a0, a1, b0, b1;
          upk2(sum_a, a0, a1);
          upk2(sum_b, b0, b1);
          l_run += ((a0 + a1) + (b0 + b1)) * (1.0f / C::kPScale);
        }
        if constexpr (FP8) {
          uint32_t q8[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            q8[i] = pack_e4m3x4(s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
          tmem_st16(tP, q8);
        } else {
          tmem_st32(tP, pk);
        }
        if (rescale) {
          // O_t is quiescent here: the commit behind this S_t also covered the
          // previous P_t V product.
#pragma unroll
          for (int h2 = 0; h2 < HD / 64; ++h2) {
            uint32_t o[32];
            tmem_ld32(tO + h2 * 32, o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + h2 * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        release_p(bar(B::kPFull + t), lane);
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B::kOFull + t), 0, abort_flag));
    // Combine the two halves' row sums (all threads of the group take part,
    // so the barrier is reached even when a wait above gave up).
    float* lsum = xmax + (8 + t * 2) * 128;
    lsum[c * 128 + r] = l_run;
    named_barrier_sync(xbar_id, xbar_threads);
    const float l_row = l_run + lsum[(c ^ 1) * 128 + r];
    if (!ok) {
      raise_abort(abort_flag, kErrSoftmaxTimeout);
    } else {
      tc_fence_after();
      const int grow = row0 + t * kTileRows + r;
      const bool row_ok = grow < p.q_len;
      float inv = 1.f / (l_row * C::kPScale);
      if constexpr (FP8) inv *= p.v_descale[hk];
      bool row_empty = false;
      if constexpr (EXTRA) {
        bool row_dropped = false;
        if (p.qmask != nullptr && row_ok) {
          const uint32_t wq = __ldg(p.qmask + static_cast<int64_t>(b) * p.qmask_sb + (grow >> 5));
          row_dropped = !((wq >> (grow & 31)) & 1u);
        }
        // A dropped row, or one that saw no key at all (its maximum never
        // left -inf; the exp2 polynomial floors excluded keys at 2^-125, so
        // the sum alone cannot tell), is written as zeros with LSE -inf.
        row_empty = row_dropped || m_run == -INFINITY || !(l_row > 0.f);
        if (row_empty) inv = 0.f;
      }
      void* obase = p.o;
      int orow_idx = grow;
      int ohead = h;
      int64_t osb = p.o_sb;
      int n_dst = 1;  // a replicated text row is stored to every rank
      if (p.o_rows > 0) {
        int peer = 0, lrow = 0;
        bool txt = false;
        if (row_ok) {
          int g = grow;
          if (p.o_txt > 0) {
            if (p.o_txt_front) {
              txt = g < p.o_txt;
              if (!txt) g -= p.o_txt;
            } else {
              txt = g >= p.o_img_rows;
              if (txt) g -= p.o_img_rows;
            }
          }
          if (txt) {
            n_dst = p.o_world;
            lrow = g;
          } else if (p.o_seg0 == 0) {
            peer = g / p.o_rows;
            lrow = g - peer * p.o_rows;
          } else if (g < p.o_world * p.o_seg0) {
            peer = g / p.o_seg0;
            lrow = g - peer * p.o_seg0;
          } else {
            const int seg1 = p.o_rows - p.o_seg0;
            const int t2 = g - p.o_world * p.o_seg0;
            peer = t2 / seg1;
            lrow = p.o_seg0 + (t2 - peer * seg1);
          }
        }
        obase = txt ? p.o_txt_peer[0] : p.o_peer[peer];
        osb = txt ? p.o_txt_sb : p.o_sb;
        orow_idx = lrow;
        ohead = p.o_head_off + h;
      }
      const int64_t ooff = (static_cast<int64_t>(b) * osb + static_cast<int64_t>(orow_idx) * p.o_sl +
                            static_cast<int64_t>(ohead) * p.o_sh) *
                               (OUT_F32 ? 4 : 2) +
                           c * (HD / 2) * (OUT_F32 ? 4 : 2);
#pragma unroll
      for (int h2 = 0; h2 < HD / 64; ++h2) {
        uint32_t o[32];
        tmem_ld32(tO + h2 * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
        if (row_ok) {
          if constexpr (OUT_F32) {
            float4 f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              f[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                 __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
            for (int dd = 0; dd < n_dst; ++dd) {
              float4* dst = reinterpret_cast<float4*>(
                  static_cast<char*>(dd == 0 ? obase : p.o_txt_peer[dd]) + ooff + h2 * 128);
#pragma unroll
              for (int i = 0; i < 8; ++i) dst[i] = f[i];
            }
          } else {
            uint4 w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              w[i].x = pack16<F16>(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
              w[i].y = pack16<F16>(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
              w[i].z = pack16<F16>(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
              w[i].w = pack16<F16>(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
            }
            for (int dd = 0; dd < n_dst; ++dd) {
              uint4* dst = reinterpret_cast<uint4*>(
                  static_cast<char*>(dd == 0 ? obase : p.o_txt_peer[dd]) + ooff + h2 * 64);
#pragma unroll
              for (int i = 0; i < 4; ++i) dst[i] = w[i];
            }
          }
        }
      }
      if (c == 0 && row_ok && p.lse != nullptr) {
        p.lse[static_cast<int64_t>(b) * p.lse_sb + static_cast<int64_t>(h) * p.lse_sh +
              static_cast<int64_t>(grow) * p.lse_sl] =
            row_empty ? -INFINITY : (m_run + log2f(l_row)) * kLn2;
      }
    }
  }
  if constexpr (PAIR) {
    tc_fence_before();
    cluster_sync();  // the pair's products complete and every TMEM read done in both CTAs
    if (warp == kMmaWarp) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, 512);
    }
  } else {
    __syncthreads();
    if (warp == kMmaWarp) {
      tc_fence_after();
      tmem_dealloc(tmem, 512);
    }
  }
}

template <bool FP8, bool OUT_F32, bool EXTRA, int NCH, bool F16 = false, int HD = kHeadDim, bool PAIR = false>
static int launch_attn(const AttnParams& prm, dim3 grid, cudaStream_t stream) {
  using C = AttnCfg<FP8, F16, HD>;
  static std::atomic<uint64_t> configured{0};  // one bit per device ordinal
  auto kern = attn_fwd_kernel<FP8, OUT_F32, EXTRA, NCH, F16, HD, PAIR>;
  constexpr int kSmem = attn_smem_bytes<FP8, F16, HD, PAIR>();
  DGXM_CUDA_TRY(set_smem_limit_once(kern, kSmem, configured));
  if constexpr (PAIR) {
    // Clusters of two along the Q tiles (the grid's x extent is even).
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    DGXM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, prm));
  } else {
    kern<<<grid, kAttnThreads, kSmem, stream>>>(prm);
    DGXM_CUDA_TRY(cudaGetLastError());
  }
  return DGXM_OK;
}

static bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace dgxm

namespace dgxm {

// Whether the current device can hold a cluster of two attention CTAs (both
// SMs of one TPC free for a 576-thread CTA with about 200 KB of shared
// memory), asked once per device.  Where it cannot -- a partition without
// whole TPCs, say -- 16-bit attention runs on single CTAs.
static bool pair_fits() {
  static std::atomic<int> state[64];  // 0 not asked, 1 fits, 2 does not
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (dev < 64) {
    const int known = state[dev].load(std::memory_order_acquire);
    if (known != 0) return known == 1;
  }
  auto kern = attn_fwd_kernel<false, false, false, DGXM_SM_P_CHUNKS, false, kHeadDim, true>;
  static std::atomic<uint64_t> configured{0};
  bool fits = false;
  constexpr int kSmem = attn_smem_bytes<false, false, kHeadDim, true>();
  if (set_smem_limit_once(kern, kSmem, configured) == cudaSuccess) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    fits = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0;
  }
  if (!fits) cudaGetLastError();  // a failed query leaves no error for the next call
  if (dev < 64) state[dev].store(fits ? 1 : 2, std::memory_order_release);
  return fits;
}

// Whether a call runs the CTA-pair kernel: built for 16-bit inputs at head
// dim 128 with the chunked P release, not turned off by DGXM_ATTN_ONE_CTA,
// and the device holds a pair.
static bool attn_uses_pair(const dgxm_attn_desc* d) {
  const int nch = (d->flags & DGXM_ATTN_P_CHUNKS_MASK) >> DGXM_ATTN_P_CHUNKS_SHIFT;
  return (d->flags & DGXM_ATTN_ONE_CTA) == 0 && d->in_dtype != DGXM_DTYPE_E4M3 &&
         d->head_dim == kHeadDim && nch != 1 && pair_fits();
}

// Validate the descriptor and fill the kernel parameters (everything but
// the output routing, which the caller sets).
static int prepare_attn(const dgxm_attn_desc* d, const void* q, const void* k, const void* v,
                        const float* q_descale, const float* k_descale, const float* v_descale,
                        void* o, float* lse, AttnParams* out_prm, dim3* out_grid, bool* skip) {
  if (d == nullptr) return fail(DGXM_ERR_INVALID, "attention descriptor is NULL");
  if (d->batch < 0 || d->q_len < 0 || d->kv_len < 0 || d->q_heads <= 0 || d->kv_heads <= 0)
    return fail(DGXM_ERR_INVALID, "negative or zero attention extent (batch=%d q_len=%d kv_len=%d "
                "q_heads=%d kv_heads=%d)", d->batch, d->q_len, d->kv_len, d->q_heads, d->kv_heads);
  if (d->head_dim != kHeadDim && !(d->head_dim == 64 && d->in_dtype != DGXM_DTYPE_E4M3))
    return fail(DGXM_ERR_UNSUPPORTED,
                "head_dim %d is not supported (this build runs 128, and 64 for 16-bit inputs)",
                d->head_dim);
  if (d->q_heads % d->kv_heads != 0)
    return fail(DGXM_ERR_INVALID, "query heads (%d) must be divisible by key/value heads (%d)",
                d->q_heads, d->kv_heads);
  *skip = false;
  if (d->batch == 0 || d->q_len == 0) {
    *skip = true;
    return DGXM_OK;
  }
  if (d->kv_len == 0)
    return fail(DGXM_ERR_INVALID, "attention over an empty key axis has no defined output");
  if (d->batch > 65535 || d->q_heads > 65535)
    return fail(DGXM_ERR_UNSUPPORTED, "batch %d or heads %d exceed the launch grid", d->batch,
                d->q_heads);
  const bool fp8 = d->in_dtype == DGXM_DTYPE_E4M3;
  const bool f16 = d->in_dtype == DGXM_DTYPE_F16;
  if (!fp8 && !f16 && d->in_dtype != DGXM_DTYPE_BF16)
    return fail(DGXM_ERR_UNSUPPORTED, "input dtype %d is not supported (bf16, f16 or e4m3)",
                d->in_dtype);
  // A 16-bit output takes the inputs' 16-bit format (bf16 for e4m3 inputs).
  const bool out_f32 = d->out_dtype == DGXM_DTYPE_F32;
  const int out16 = f16 ? DGXM_DTYPE_F16 : DGXM_DTYPE_BF16;
  if (!out_f32 && d->out_dtype != out16)
    return fail(DGXM_ERR_UNSUPPORTED,
                "output dtype %d is not supported for input dtype %d (f32, or %s)", d->out_dtype,
                d->in_dtype, f16 ? "f16" : "bf16");
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return fail(DGXM_ERR_INVALID, "q, k, v and o must be non-NULL");
  if (fp8 && (q_descale == nullptr || k_descale == nullptr || v_descale == nullptr))
    return fail(DGXM_ERR_INVALID, "e4m3 attention needs q, k and v descale arrays");
  const int out_bytes = out_f32 ? 4 : 2;
  if (!aligned16(o) || (d->o_stride[1] * out_bytes) % 16 != 0 ||
      (d->o_stride[2] * out_bytes) % 16 != 0 || (d->o_stride[0] * out_bytes) % 16 != 0)
    return fail(DGXM_ERR_INVALID, "output base and strides must be 16-byte aligned");

  AttnParams& prm = *out_prm;
  memset(&prm, 0, sizeof(prm));
  const CUtensorMapDataType dt = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                : (f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  const int eb = fp8 ? 1 : 2;
  const int box_cols = 128 / eb;
  int rc;
  if ((rc = encode_map_4d(&prm.tmap_q, q, dt, eb, d->head_dim, d->q_heads, d->q_len, d->batch,
                          d->q_stride[2], d->q_stride[1], d->q_stride[0], box_cols, kTileRows)))
    return rc;
  // A CTA pair loads K in 64-key halves.
  const bool pair = attn_uses_pair(d);
  if ((rc = encode_map_4d(&prm.tmap_k, k, dt, eb, d->head_dim, d->kv_heads, d->kv_len, d->batch,
                          d->k_stride[2], d->k_stride[1], d->k_stride[0], box_cols,
                          pair ? kTileRows / 2 : kTileRows)))
    return rc;
  if ((rc = encode_map_4d(&prm.tmap_v, v, dt, eb, d->head_dim, d->kv_heads, d->kv_len, d->batch,
                          d->v_stride[2], d->v_stride[1], d->v_stride[0], box_cols, kTileRows)))
    return rc;
  prm.o = o;
  prm.lse = lse;
  prm.q_descale = q_descale;
  prm.k_descale = k_descale;
  prm.v_descale = v_descale;
  prm.o_sb = d->o_stride[0];
  prm.o_sl = d->o_stride[1];
  prm.o_sh = d->o_stride[2];
  prm.lse_sb = d->lse_stride[0];
  prm.lse_sh = d->lse_stride[1];
  prm.lse_sl = d->lse_stride[2];
  prm.q_len = d->q_len;
  prm.kv_len = d->kv_len;
  prm.q_heads = d->q_heads;
  prm.kv_heads = d->kv_heads;
  prm.n_kv_tiles = (d->kv_len + kTileRows - 1) / kTileRows;
  const float scale = d->softmax_scale > 0.f ? d->softmax_scale : 1.0f / sqrtf((float)d->head_dim);
  prm.scale_log2 = scale * kLog2e;
  prm.flags = d->flags;

  const unsigned qtiles = (d->q_len + 2 * kTileRows - 1) / (2 * kTileRows);
  *out_grid = dim3(pair ? (qtiles + 1) & ~1u : qtiles, d->q_heads, d->batch);
  return DGXM_OK;
}

// Instantiations: bf16 inputs release P in 4 chunks (the default) or 1; e4m3
// in 2 (4 runs as 2) or 1; fp16 runs the default.  2 chunks select 4 for bf16.
template <bool EXTRA, int NCH>
static int dispatch_attn_n(const dgxm_attn_desc* d, const AttnParams& prm, dim3 grid, cudaStream_t st) {
  const bool fp8 = d->in_dtype == DGXM_DTYPE_E4M3;
  const bool out_f32 = d->out_dtype == DGXM_DTYPE_F32;
  constexpr int kFp8Chunks = p_chunks<true, NCH>();  // 4 runs as 2: one instantiation
  if (fp8)
    return out_f32 ? launch_attn<true, true, EXTRA, kFp8Chunks>(prm, grid, st)
                   : launch_attn<true, false, EXTRA, kFp8Chunks>(prm, grid, st);
  return out_f32 ? launch_attn<false, true, EXTRA, NCH>(prm, grid, st)
                 : launch_attn<false, false, EXTRA, NCH>(prm, grid, st);
}

template <bool EXTRA>
static int dispatch_attn_t(const dgxm_attn_desc* d, const AttnParams& prm, dim3 grid, cudaStream_t st) {
  int nch = (d->flags & DGXM_ATTN_P_CHUNKS_MASK) >> DGXM_ATTN_P_CHUNKS_SHIFT;
  if (nch != 0 && nch != 1 && nch != 2 && nch != 4)
    return fail(DGXM_ERR_INVALID, "%d P chunks per block (1, 2 or 4)", nch);
  if (d->head_dim == 64) {
    // Head dimension 64 (16-bit inputs): the library's default release of P.
    const bool f32 = d->out_dtype == DGXM_DTYPE_F32;
    if (d->in_dtype == DGXM_DTYPE_F16)
      return f32 ? launch_attn<false, true, EXTRA, DGXM_SM_P_CHUNKS, true, 64>(prm, grid, st)
                 : launch_attn<false, false, EXTRA, DGXM_SM_P_CHUNKS, true, 64>(prm, grid, st);
    return f32 ? launch_attn<false, true, EXTRA, DGXM_SM_P_CHUNKS, false, 64>(prm, grid, st)
               : launch_attn<false, false, EXTRA, DGXM_SM_P_CHUNKS, false, 64>(prm, grid, st);
  }
  if (attn_uses_pair(d)) {
    const bool f32 = d->out_dtype == DGXM_DTYPE_F32;
    if (d->in_dtype == DGXM_DTYPE_F16)
      return f32 ? launch_attn<false, true, EXTRA, DGXM_SM_P_CHUNKS, true, kHeadDim, true>(prm, grid, st)
                 : launch_attn<false, false, EXTRA, DGXM_SM_P_CHUNKS, true, kHeadDim, true>(prm, grid, st);
    return f32 ? launch_attn<false, true, EXTRA, DGXM_SM_P_CHUNKS, false, kHeadDim, true>(prm, grid, st)
               : launch_attn<false, false, EXTRA, DGXM_SM_P_CHUNKS, false, kHeadDim, true>(prm, grid, st);
  }
  if (d->in_dtype == DGXM_DTYPE_F16) {
    // fp16 inputs run the library's default release of P.
    if (d->out_dtype == DGXM_DTYPE_F32)
      return launch_attn<false, true, EXTRA, DGXM_SM_P_CHUNKS, true>(prm, grid, st);
    return launch_attn<false, false, EXTRA, DGXM_SM_P_CHUNKS, true>(prm, grid, st);
  }
  if (nch == 1) return dispatch_attn_n<EXTRA, 1>(d, prm, grid, st);
  return dispatch_attn_n<EXTRA, DGXM_SM_P_CHUNKS>(d, prm, grid, st);
}

static int dispatch_attn(const dgxm_attn_desc* d, const AttnParams& prm, dim3 grid, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool extra = prm.kmask != nullptr || prm.qmask != nullptr || prm.n_bias > 0;
  return extra ? dispatch_attn_t<true>(d, prm, grid, st) : dispatch_attn_t<false>(d, prm, grid, st);
}

// Fill the output routing of the fused inverse all-to-all.
static int set_route(const dgxm_attn_desc* d, const dgxm_attn_route* rt, AttnParams* prm) {
  if (rt->world < 1 || rt->world > DGXM_MAX_WORLD || rt->rank < 0 || rt->rank >= rt->world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", rt->rank, rt->world);
  if (rt->txt_rows < 0 || (rt->txt_front != 0 && rt->txt_front != 1))
    return fail(DGXM_ERR_INVALID, "text rows %d / front flag %d out of range", rt->txt_rows,
                rt->txt_front);
  if (rt->txt_rows > 0 && rt->seg0 != 0)
    return fail(DGXM_ERR_INVALID, "replicated text needs the rank-major image order (seg0 = 0)");
  if (rt->seq_local <= 0 ||
      static_cast<int64_t>(rt->seq_local) * rt->world + rt->txt_rows != d->q_len)
    return fail(DGXM_ERR_INVALID, "seq_local %d x world %d + %d text rows does not cover q_len %d",
                rt->seq_local, rt->world, rt->txt_rows, d->q_len);
  if (rt->seg0 < 0 || rt->seg0 >= rt->seq_local)
    return fail(DGXM_ERR_INVALID, "joint segment of %d rows does not split %d local rows", rt->seg0,
                rt->seq_local);
  for (int r = 0; r < rt->world; ++r) {
    if (rt->o_peers[r] == nullptr || reinterpret_cast<uintptr_t>(rt->o_peers[r]) % 16)
      return fail(DGXM_ERR_INVALID, "output peer %d is NULL or not 16-byte aligned", r);
    prm->o_peer[r] = rt->o_peers[r];
    if (rt->txt_rows > 0) {
      if (rt->txt_peers[r] == nullptr || reinterpret_cast<uintptr_t>(rt->txt_peers[r]) % 16)
        return fail(DGXM_ERR_INVALID, "text output peer %d is NULL or not 16-byte aligned", r);
      prm->o_txt_peer[r] = rt->txt_peers[r];
    }
  }
  prm->o_rows = rt->seq_local;
  prm->o_head_off = rt->rank * d->q_heads;
  prm->o_world = rt->world;
  prm->o_seg0 = rt->seg0;
  prm->o_txt = rt->txt_rows;
  prm->o_txt_front = rt->txt_front;
  prm->o_img_rows = rt->seq_local * rt->world;
  prm->o_txt_sb = static_cast<int64_t>(rt->txt_rows) * d->o_stride[1];
  return DGXM_OK;
}

// Fill the keep masks and query-group biases.
static int set_extras(const dgxm_attn_desc* d, const dgxm_attn_extras* ex, AttnParams* prm) {
  prm->kmask = ex->key_keep;
  prm->kmask_sb = ex->key_keep_batch_stride;
  prm->kmask_words = (d->kv_len + 31) / 32;
  prm->qmask = ex->query_keep;
  prm->qmask_sb = ex->query_keep_batch_stride;
  if (ex->n_bias_groups < 0 || ex->n_bias_groups > DGXM_MAX_BIAS_GROUPS)
    return fail(DGXM_ERR_INVALID, "%d bias groups (at most %d)", ex->n_bias_groups,
                DGXM_MAX_BIAS_GROUPS);
  prm->n_bias = ex->n_bias_groups;
  for (int g = 0; g < ex->n_bias_groups; ++g) {
    if (ex->bias_row_begin[g] < 0 || ex->bias_row_end[g] < ex->bias_row_begin[g] ||
        ex->bias_row_end[g] > d->q_len)
      return fail(DGXM_ERR_INVALID, "bias group %d rows [%d, %d) outside [0, %d)", g,
                  ex->bias_row_begin[g], ex->bias_row_end[g], d->q_len);
    if (ex->bias_keys[g] < 0 || ex->bias_keys[g] > d->kv_len)
      return fail(DGXM_ERR_INVALID, "bias group %d declares %d keys over %d", g, ex->bias_keys[g],
                  d->kv_len);
    prm->bias_q0[g] = ex->bias_row_begin[g];
    prm->bias_q1[g] = ex->bias_row_end[g];
    prm->bias[g] = ex->bias[g];
    prm->bias_sb[g] = ex->bias_stride[g][0];
    prm->bias_sh[g] = ex->bias_stride[g][1];
    prm->bias_sq[g] = ex->bias_stride[g][2];
    prm->bias_len[g] = ex->bias_keys[g];
  }
  const float scale = d->softmax_scale > 0.f ? d->softmax_scale : 1.0f / sqrtf((float)d->head_dim);
  prm->inv_scale = 1.0f / scale;
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int dgxm_attn_fwd(const dgxm_attn_desc* d, const void* q, const void* k, const void* v,
                             const float* q_descale, const float* k_descale,
                             const float* v_descale, void* o, float* lse, void* stream) {
  using namespace dgxm;
  AttnParams prm;
  dim3 grid;
  bool skip = false;
  int rc = prepare_attn(d, q, k, v, q_descale, k_descale, v_descale, o, lse, &prm, &grid, &skip);
  if (rc != DGXM_OK || skip) return rc;
  return dispatch_attn(d, prm, grid, stream);
}

extern "C" int dgxm_attn_fwd_routed(const dgxm_attn_desc* d, const void* q, const void* k,
                                    const void* v, const float* q_descale, const float* k_descale,
                                    const float* v_descale, void* const* o_peers, int32_t world,
                                    int32_t rank, int32_t seq_local, int32_t seg0, float* lse,
                                    void* stream) {
  using namespace dgxm;
  if (o_peers == nullptr) return fail(DGXM_ERR_INVALID, "o_peers is NULL");
  if (world < 1 || world > DGXM_MAX_WORLD || rank < 0 || rank >= world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", rank, world);
  if (d == nullptr) return fail(DGXM_ERR_INVALID, "attention descriptor is NULL");
  if (seq_local <= 0 || static_cast<int64_t>(seq_local) * world != d->q_len)
    return fail(DGXM_ERR_INVALID, "seq_local %d x world %d does not cover q_len %d", seq_local,
                world, d->q_len);
  for (int r = 0; r < world; ++r)
    if (o_peers[r] == nullptr || reinterpret_cast<uintptr_t>(o_peers[r]) % 16)
      return fail(DGXM_ERR_INVALID, "output peer %d is NULL or not 16-byte aligned", r);
  AttnParams prm;
  dim3 grid;
  bool skip = false;
  int rc = prepare_attn(d, q, k, v, q_descale, k_descale, v_descale, o_peers[0], lse, &prm,
                        &grid, &skip);
  if (rc != DGXM_OK || skip) return rc;
  dgxm_attn_route rt;
  memset(&rt, 0, sizeof(rt));
  for (int r = 0; r < world; ++r) rt.o_peers[r] = o_peers[r];
  rt.world = world;
  rt.rank = rank;
  rt.seq_local = seq_local;
  rt.seg0 = seg0;
  if ((rc = set_route(d, &rt, &prm))) return rc;
  return dispatch_attn(d, prm, grid, stream);
}

extern "C" int dgxm_attn_fwd_ext(const dgxm_attn_desc* d, const dgxm_attn_extras* extras,
                                 const dgxm_attn_route* route, const void* q, const void* k,
                                 const void* v, const float* q_descale, const float* k_descale,
                                 const float* v_descale, void* o, float* lse, void* stream) {
  using namespace dgxm;
  if (d == nullptr) return fail(DGXM_ERR_INVALID, "attention descriptor is NULL");
  void* o0 = o;
  if (route != nullptr) {
    if (route->world < 1 || route->world > DGXM_MAX_WORLD)
      return fail(DGXM_ERR_INVALID, "route world %d out of range", route->world);
    o0 = route->o_peers[0];
  }
  AttnParams prm;
  dim3 grid;
  bool skip = false;
  int rc = prepare_attn(d, q, k, v, q_descale, k_descale, v_descale, o0, lse, &prm, &grid, &skip);
  if (rc != DGXM_OK || skip) return rc;
  if (route != nullptr && (rc = set_route(d, route, &prm))) return rc;
  if (extras != nullptr && (rc = set_extras(d, extras, &prm))) return rc;
  return dispatch_attn(d, prm, grid, stream);
}
