/*
 * dgxm_sp.h -- C ABI of the B200 sequence-parallel attention path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*), returns an int status (DGXM_OK == 0), never aborts the
 * process, and waits on the device only for a bounded time.  A failed call
 * leaves a human-readable reason in dgxm_last_error_message() for the calling
 * thread.  Nothing here allocates device memory except dgxm_comm_create and
 * the ring entry point (which owns its rotation buffers through the comm
 * handle).
 *
 * The reference (dgx-monarch) is pure Python; these functions replace the
 * third-party library calls its attention seam makes.  Each declaration names
 * the reference call site it stands in for (paths within the dgx-monarch
 * source tree).
 */
#ifndef DGXM_SP_H
#define DGXM_SP_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define DGXM_OK 0
#define DGXM_ERR_INVALID 1     /* bad argument: shape, stride, alignment, dtype */
#define DGXM_ERR_UNSUPPORTED 2 /* well-formed request this build does not run   */
#define DGXM_ERR_CUDA 3        /* a CUDA runtime or driver call failed          */
#define DGXM_ERR_TIMEOUT 4     /* a bounded device wait expired                 */
#define DGXM_ERR_STATE 5       /* handle misuse (closed, wrong generation)      */

/* ------------------------------------------------------------ dtypes */
#define DGXM_DTYPE_BF16 0
#define DGXM_DTYPE_F16 1
#define DGXM_DTYPE_E4M3 2
#define DGXM_DTYPE_F32 3

/* ------------------------------------------------------------ attention flags */
/* Drain each P.V product before the next Q.K^T product reuses its tensor
 * memory columns (slower; kept as a cross-check of the fast ordering). */
#define DGXM_ATTN_SAFE_ORDER 1

/* Version of this ABI; bumped on any incompatible change. */
int dgxm_abi_version(void);

/* Message describing the last failed call made on this thread ("" if none). */
const char* dgxm_last_error_message(void);

/* Read (and optionally clear) the device-side error word that bounded waits
 * set when they expire.  Synchronises the current device.  Returns 0 when no
 * kernel has reported a problem. */
int dgxm_device_error(int clear);

/* ------------------------------------------------------------ attention */
/*
 * Non-causal attention forward over (batch, row, head, head_dim) tensors, the
 * layout the reference's ring processors use.  head_dim must be contiguous.
 * Strides are in elements.  lse (may be NULL) receives the natural-log
 * log-sum-exp of the scaled logits as fp32 shaped by lse_stride.
 */
typedef struct dgxm_attn_desc {
  int32_t batch;
  int32_t q_len;
  int32_t kv_len;
  int32_t q_heads;
  int32_t kv_heads;   /* q_heads % kv_heads == 0 (grouped-query attention) */
  int32_t head_dim;   /* 128 */
  int32_t in_dtype;   /* DGXM_DTYPE_BF16 or DGXM_DTYPE_E4M3 */
  int32_t out_dtype;  /* DGXM_DTYPE_BF16 or DGXM_DTYPE_F32 */
  int64_t q_stride[3];   /* batch, row, head */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t lse_stride[3]; /* batch, head, row */
  float softmax_scale;   /* <= 0 selects 1/sqrt(head_dim) */
  int32_t flags;         /* DGXM_ATTN_* */
} dgxm_attn_desc;

/*
 * Replaces the block attention the reference reaches through
 *   adapters/cudnn_ring_attention.py:66-89   (TorchCudnnRingProcessor.__call__,
 *                                             returns out (B,L,H,D) + fp32 lse (B,H,L)),
 *   adapters/wan_ring_full_context.py:160-167 (aten._scaled_dot_product_flash_attention),
 *   adapters/usp_full_axis.py:17-24          (usp_attn.ring_attn_fn at ring world 1).
 * For DGXM_DTYPE_E4M3 inputs, q_descale holds one fp32 factor per query head
 * and k_descale / v_descale one per key/value head; they are ignored for bf16.
 */
int dgxm_attn_fwd(const dgxm_attn_desc* desc, const void* q, const void* k, const void* v,
                  const float* q_descale, const float* k_descale, const float* v_descale,
                  void* o, float* lse, void* stream);

/* ------------------------------------------------------------ LSE merge */
/*
 * Merge n_parts partial attention results over disjoint key blocks:
 *   lse = log(sum_i exp(lse_i)),  out = sum_i exp(lse_i - lse) * out_i
 * in fp32.  parts_out[i] is (batch, rows, heads, head_dim) of part_dtype
 * (BF16 or F32), contiguous; parts_lse[i] is fp32 (batch, heads, rows),
 * contiguous.  out is written in out_dtype (BF16 or F32) with the same
 * layout; lse_out (may be NULL) is fp32 (batch, heads, rows).
 * parts_out / parts_lse are HOST arrays of device pointers, n_parts <= 16.
 *
 * Replaces the ring merge inside xfuser/yunchang's ring flash attention,
 * reached from adapters/base.py:320 (usp_attn(None, q, k, v)) with the
 * per-block processor contract of adapters/cudnn_ring_attention.py:61-89.
 */
int dgxm_lse_merge(int32_t batch, int32_t rows, int32_t heads, int32_t head_dim,
                   int32_t n_parts, const void* const* parts_out, int32_t part_dtype,
                   const float* const* parts_lse, void* out, int32_t out_dtype, float* lse_out,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DGXM_SP_H */
