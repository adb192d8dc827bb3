/*
 * dgxm_sp.h -- C ABI of the B200 sequence-parallel attention path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*), returns an int status (DGXM_OK == 0), never aborts the
 * process, and waits on the device only for a bounded time.  A failed call
 * leaves a human-readable reason in dgxm_last_error_message() for the calling
 * thread.  Nothing here allocates device memory except dgxm_comm_create;
 * the ring entry point keeps its rotating blocks in the comm window and its
 * partial results in a caller-provided workspace.
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
/* 16-bit attention at head dim 128 runs on CTA pairs: clusters of two CTAs
 * on the two SMs of a TPC, each loading half of every K/V block, with one
 * thread of the pair issuing M256 tensor-core products for both.  This flag
 * runs it on single CTAs instead (a cross-check; results agree within the
 * attention tolerance).  e4m3, head dim 64, the single P release and devices
 * that cannot hold a cluster of two such CTAs always run on single CTAs. */
#define DGXM_ATTN_ONE_CTA 2
/* Release the probabilities of each 128-key block to the tensor core in
 * chunks, so P.V starts on the first chunk while the softmax computes the
 * rest: 0 keeps the library default (4 chunks; 2 for e4m3 inputs, whose
 * 32-key MMA steps allow no more), as do 2 and 4; 1 releases the whole block
 * at once (a cross-check).  Results agree within the attention tolerance
 * across chunk counts (the P.V steps accumulate in another order). */
#define DGXM_ATTN_P_CHUNKS_SHIFT 4
#define DGXM_ATTN_P_CHUNKS_MASK (7 << DGXM_ATTN_P_CHUNKS_SHIFT)
#define DGXM_ATTN_P_CHUNKS(n) ((n) << DGXM_ATTN_P_CHUNKS_SHIFT)

/* Version of this ABI; bumped on any incompatible change. */
int dgxm_abi_version(void);

/* Message describing the last failed call made on this thread ("" if none). */
const char* dgxm_last_error_message(void);

/* A strided copy (host <-> device or within either): height rows of width
 * bytes with row pitches dpitch / spitch, one copy-engine transfer on the
 * stream.  The head-group slices of a (B, L, H, D) tensor are such copies. */
int dgxm_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width,
                 int64_t height, void* stream);

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
  int32_t in_dtype;   /* DGXM_DTYPE_BF16, DGXM_DTYPE_F16 or DGXM_DTYPE_E4M3 */
  int32_t out_dtype;  /* DGXM_DTYPE_F32, or the inputs' 16-bit format (BF16 for E4M3) */
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

/* ------------------------------------------------------------ attention extras */
#define DGXM_MAX_BIAS_GROUPS 8

/*
 * Optional inputs of dgxm_attn_fwd_ext.
 *
 * key_keep / query_keep: bit i of word i/32 keeps key (query row) i; a key
 * with bit 0 is excluded from every softmax, a query row with bit 0 is
 * written as zeros (LSE -inf).  This is the exact pad-row exclusion of
 * adapters/usp_pad_exclusion.py:112-137 (attend the real rows, zero-restore
 * the pads) done inside the kernel instead of by index_select copies.
 * NULL keeps everything; a batch stride of 0 shares one mask.
 *
 * Query-group bias (adapters/usp_query_bias.py:109-130): query row r in
 * [bias_row_begin[g], bias_row_end[g]) adds
 * bias[g][b, h, r - bias_row_begin[g], key] to its scaled logits for keys
 * < bias_keys[g] (later keys carry no bias, extend_bias_keys at
 * adapters/usp_query_bias.py:95-106); rows in no group carry none.  fp32,
 * strides in elements; a stride of 0 broadcasts (a query-row stride of 0 is
 * one key row shared by the whole group).
 */
typedef struct dgxm_attn_extras {
  const uint32_t* key_keep;
  int64_t key_keep_batch_stride;   /* words */
  const uint32_t* query_keep;
  int64_t query_keep_batch_stride; /* words */
  int32_t n_bias_groups;
  int32_t bias_row_begin[DGXM_MAX_BIAS_GROUPS];
  int32_t bias_row_end[DGXM_MAX_BIAS_GROUPS];
  const float* bias[DGXM_MAX_BIAS_GROUPS];
  int64_t bias_stride[DGXM_MAX_BIAS_GROUPS][3]; /* batch, head, query row */
  int32_t bias_keys[DGXM_MAX_BIAS_GROUPS];
} dgxm_attn_extras;

/* Output routing of the fused inverse all-to-all (see dgxm_attn_fwd_routed).
 *
 * Replicated text (txt_rows > 0): the gathered axis holds txt_rows text rows
 * -- every rank holds the whole text and attends its own head slice of it --
 * before (txt_front = 1) or after (txt_front = 0) the world*seq_local image
 * rows, so q_len = txt_rows + world*seq_local.  Image rows route as above
 * (rank-major, seg0 must be 0).  Text output row i of query head h goes to
 * EVERY rank r: row i, head rank*q_heads + h of txt_peers[r], a (batch,
 * txt_rows, world*q_heads, head_dim) tensor with the row and head strides of
 * desc->o_stride and batch stride txt_rows * o_stride[1] -- the all-gather
 * over heads of the text output, done by the epilogue's stores. */
typedef struct dgxm_attn_route {
  void* o_peers[8];
  int32_t world;
  int32_t rank;
  int32_t seq_local;
  int32_t seg0;
  int32_t txt_rows;
  int32_t txt_front;
  void* txt_peers[8];
} dgxm_attn_route;

/*
 * dgxm_attn_fwd with optional extras and optional output routing (either may
 * be NULL; with a route, `o` is ignored).  The general entry behind the
 * drop-in's padded and biased calls.
 */
int dgxm_attn_fwd_ext(const dgxm_attn_desc* desc, const dgxm_attn_extras* extras,
                      const dgxm_attn_route* route, const void* q, const void* k, const void* v,
                      const float* q_descale, const float* k_descale, const float* v_descale,
                      void* o, float* lse, void* stream);

/* ------------------------------------------------------------ LSE merge */
/*
 * Merge n_parts partial attention results over disjoint key blocks:
 *   lse = log(sum_i exp(lse_i)),  out = sum_i exp(lse_i - lse) * out_i
 * in fp32.  parts_out[i] is (batch, rows, heads, head_dim) of part_dtype
 * (BF16, F16 or F32), contiguous; parts_lse[i] is fp32 (batch, heads, rows),
 * contiguous.  out is written in out_dtype (F32, or a 16-bit format: any for
 * F32 parts, the parts' own for 16-bit parts) with the same layout; lse_out
 * (may be NULL) is fp32 (batch, heads, rows).
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

/* ------------------------------------------------------------ communicator */
#define DGXM_MAX_WORLD 8
#define DGXM_IPC_HANDLE_BYTES 64

/* One rank's NVLink window: device memory on the current device that every
 * peer maps through a CUDA IPC handle (a plain peer mapping; no NVSwitch
 * group object is created).  Bound to one setup generation: a handle from a retired
 * generation is destroyed, never reused.
 *
 * Stands in for the process groups the reference builds in
 * actor/worker_env.py:313-327 (init_process_group("nccl") + xfuser
 * initialize_model_parallel) as far as the data path needs them; bootstrap
 * (handle exchange) still rides torch.distributed. */
typedef struct dgxm_comm dgxm_comm;

/* Allocate `bytes` (plus a 4 KB flag area) on the current device. */
int dgxm_comm_create(int32_t rank, int32_t world, int64_t bytes, uint64_t generation,
                     dgxm_comm** out);
/* Write this rank's DGXM_IPC_HANDLE_BYTES-byte window handle into `handle`. */
int dgxm_comm_export(dgxm_comm* comm, void* handle);
/* Map every peer window; `handles` holds world handles in rank order. */
int dgxm_comm_import(dgxm_comm* comm, const void* handles);
/* Base of `peer`'s usable window as addressable from this process. */
int dgxm_comm_window(dgxm_comm* comm, int32_t peer, void** ptr);
int64_t dgxm_comm_bytes(dgxm_comm* comm);
uint64_t dgxm_comm_generation(dgxm_comm* comm);
/* Stream-ordered barrier over all ranks of the comm: each rank releases a
 * flag in every peer window and waits (bounded, about one second) for every
 * peer's flag.  A wait that expires sets the device error word instead of
 * hanging.  Replaces the implicit synchronisation of the reference's NCCL
 * all_to_all.  The barrier count lives in device memory, so the barrier --
 * and the Ulysses step built on it (scatter, barrier, routed attention,
 * barrier) and dgxm_shared_amax_scale -- may be captured in a CUDA graph and
 * replayed; every rank must replay the same sequence.  The entries that
 * alternate window buffers on the host (ring, full-context, sequence gather)
 * are not for capture. */
int dgxm_comm_barrier(dgxm_comm* comm, void* stream);
/* Wall-clock budget of one barrier wait (default about one second). */
int dgxm_comm_set_timeout(dgxm_comm* comm, int32_t timeout_ms);
/* All-gather as peer stores: `bytes` from src land in every rank's window at
 * window_offset + rank*bytes (copy-engine peer copies), followed by a
 * barrier, so on return (stream order) every window holds all world slices
 * in rank order.  Replaces the cfg-group all_gather of the CFG split,
 * adapters/cfg_parallel.py:293-301 (and actor/dual_model_cfg.py:84). */
int dgxm_comm_allgather(dgxm_comm* comm, const void* src, int64_t bytes, int64_t window_offset,
                        void* stream);
/* Synchronise the device, unmap peers, free the window. */
int dgxm_comm_destroy(dgxm_comm* comm);

/* ------------------------------------------------------------ Ulysses all-to-all */
typedef struct dgxm_a2a_desc {
  int32_t n_tensors;  /* 1..3 tensors moved in one launch (q, k, v) */
  int32_t world;
  int32_t rank;
  int32_t batch;
  int32_t seq_local;  /* rows this rank holds before the scatter */
  int32_t heads;      /* all heads; heads % world == 0 */
  int32_t head_dim;
  int32_t dtype;
  int64_t src_stride[3][3]; /* per tensor: batch, row, head (elements) */
  /* Joint order.  0: the gathered axis is the rank-major concat of the local
   * rows.  seg0 > 0: each rank's local rows are [seg0 rows | seq_local - seg0
   * rows] (text then image) and the gathered axis lists every rank's first
   * segment, then every rank's second -- the stock key order that
   * adapters/usp_sequence_order.py:33-146 (RankMajorJointOrder) restores
   * with index copies; here the all-to-all writes rows straight there. */
  int32_t seg0;
} dgxm_a2a_desc;

/*
 * Sequence -> head all-to-all as direct peer stores.  src[t] is this rank's
 * (batch, seq_local, heads, head_dim) tensor t; dst[t*world + r] is rank r's
 * contiguous (batch, world*seq_local, heads/world, head_dim) receive tensor,
 * addressable from this rank (a comm window).  This rank writes head slice
 * [r*H/P, (r+1)*H/P) of its rows into rows [rank*seq_local, (rank+1)*seq_local)
 * of dst[t*world + r]: the rank-major gathered axis.  Follow with
 * dgxm_comm_barrier before any rank reads its receive tensors.
 *
 * Replaces yunchang SeqAllToAll4D.apply(pg, x, 2, 1) at
 * adapters/usp_full_axis.py:27-29 (and inside xfuser's call at
 * adapters/base.py:320).
 */
int dgxm_ulysses_scatter(const dgxm_a2a_desc* desc, const void* const* src, void* const* dst,
                         void* stream);

/*
 * The scatter of the joint image+text attention whose text every rank holds
 * in full (replicated, not sharded).  desc and src are the image rows, as for
 * dgxm_ulysses_scatter (seg0 must be 0).  txt[t] is this rank's whole
 * (batch, txt_rows, heads, head_dim) text tensor t, strides txt_stride[3*t ..
 * 3*t+2] (batch, row, head; elements).  dst[t*world + r] is rank r's
 * contiguous (batch, txt_rows + world*seq_local, heads/world, head_dim)
 * receive tensor: this rank's image rows land rank-major after
 * (txt_front = 1) or before (txt_front = 0) the text rows, and this rank
 * copies head slice [rank*H/P, (rank+1)*H/P) of its own text into its own
 * receive tensor, so no text crosses NVLink.  Follow with dgxm_comm_barrier.
 *
 * The key order is the unsharded [text | image] (or [image | text])
 * concatenation, the order of the single-process attention this replaces:
 * the joint attention of the CPU/gloo Ulysses case, image rows split by
 * sequence, text replicated, checked against one-process SDPA (the
 * SeqAllToAll4D call sites at adapters/usp_full_axis.py:27-29,40 around the
 * inner kernel of adapters/wan_ring_full_context.py:160-167).
 */
int dgxm_ulysses_scatter_joint(const dgxm_a2a_desc* desc, int32_t txt_rows, int32_t txt_front,
                               const void* const* txt, const int64_t* txt_stride,
                               const void* const* src, void* const* dst, void* stream);

/*
 * Head -> sequence (the inverse).  src is this rank's (batch, world*seq_local,
 * heads/world, head_dim) tensor (strides in desc->src_stride[0]); dst[r] is
 * rank r's contiguous (batch, seq_local, heads, head_dim) output.  Replaces
 * SeqAllToAll4D.apply(pg, out, 1, 2) at adapters/usp_full_axis.py:40.
 */
int dgxm_ulysses_gather(const dgxm_a2a_desc* desc, const void* src, void* const* dst,
                        void* stream);

/*
 * Attention whose epilogue performs the inverse all-to-all: output row i of
 * query head h goes to the rank owning gathered row i (rank-major, or the
 * joint order when seg0 > 0, see dgxm_a2a_desc), at that rank's local row,
 * head
 * rank*q_heads + h of that rank's (batch, seq_local, world*q_heads, head_dim)
 * tensor o_peers[owner] (strides desc->o_stride).  Everything else is
 * dgxm_attn_fwd; lse stays local.  No separate all-to-all kernel or permute
 * runs for the output.
 */
int dgxm_attn_fwd_routed(const dgxm_attn_desc* desc, const void* q, const void* k, const void* v,
                         const float* q_descale, const float* k_descale,
                         const float* v_descale, void* const* o_peers, int32_t world,
                         int32_t rank, int32_t seq_local, int32_t seg0, float* lse,
                         void* stream);

/* ------------------------------------------------------------ fused prologue */
#define DGXM_NORM_NONE 0
#define DGXM_NORM_HIDDEN 1 /* RMSNorm over all heads of a row (Wan norm_q / norm_k)   */
#define DGXM_NORM_HEAD 2   /* RMSNorm over each head's 128 values (Flux/Krea2 QKNorm) */

typedef struct dgxm_prologue_desc {
  int32_t world;
  int32_t rank;
  int32_t batch;
  int32_t seq_local;
  int32_t heads;    /* heads * 128 <= 6144 */
  int32_t head_dim; /* 128 */
  int32_t norm_mode;
  float eps;
  int64_t src_stride[3][3];  /* q, k, v: batch, row, head (elements), bf16 */
  int64_t rope_batch_stride; /* elements between batch items of the rope table; 0 = shared */
  int32_t seg0;              /* joint order, as in dgxm_a2a_desc */
} dgxm_prologue_desc;

/*
 * The Ulysses scatter with the per-token math the family forwards run right
 * before the attention seam fused in: RMSNorm of q and k (weights bf16, NULL
 * for none), then RoPE from `rope` -- fp32 (rows, head_dim/2, 2) cos/sin per
 * local row, rotating consecutive pairs (x0 c - x1 s, x0 s + x1 c) -- and the
 * head-sliced peer stores of dgxm_ulysses_scatter (dst as there).  V moves
 * unchanged.  Replaces the separate norm / apply_rope1 / all-to-all / permute
 * ops of adapters/wan_family.py:70-73 followed by
 * adapters/usp_full_axis.py:27-29.
 */
int dgxm_qkv_prologue_scatter(const dgxm_prologue_desc* desc, const void* const* src,
                              const void* norm_q_w, const void* norm_k_w, const float* rope,
                              void* const* dst, void* stream);

/* ------------------------------------------------------------ FP8 inputs */
/*
 * Per-head e4m3 quantisation of a bf16 (batch, rows, heads, 128) tensor
 * (strides in elements): descale[h] = absmax over head h / 448 (fp32) and
 * out = e4m3(x / descale[h]), contiguous.  The inputs of dgxm_attn_fwd's
 * e4m3 path (FP8 config: per-head fp32 absmax scales).  After a Ulysses
 * scatter every head lives whole on one rank, so the scale needs no
 * cross-rank reduction.
 */
int dgxm_quantize_e4m3_per_head(int32_t batch, int32_t rows, int32_t heads, int32_t head_dim,
                                const void* x, const int64_t* stride, void* out, float* descale,
                                void* stream);

/*
 * The same with row keep bits (int32 words, bit l % 32 of word l / 32 keeps
 * row l; `keep_batch_stride` words between batch rows, 0 for one mask shared
 * by every batch row): rows whose bit is clear do not count toward a head's
 * absmax, and are still written (saturated to +-448 where they exceed it).
 * The scale is then the one an attention over the real rows alone would
 * quantise with -- the rows the reference's pad exclusion hands its inner
 * kernel (adapters/usp_pad_exclusion.py:112-137).
 */
int dgxm_quantize_e4m3_per_head_masked(int32_t batch, int32_t rows, int32_t heads,
                                       int32_t head_dim, const void* x, const int64_t* stride,
                                       const uint32_t* keep, int64_t keep_batch_stride, void* out,
                                       float* descale, void* stream);

/*
 * Up to three tensors (q, k and v of one attention) quantised by the same
 * launches, each item as in dgxm_quantize_e4m3_per_head_masked (keep may be
 * NULL).  Every item is checked before anything is launched.
 */
typedef struct dgxm_quant_item {
  int32_t batch, rows, heads, head_dim;
  const void* x;
  int64_t stride[3];             /* elements: batch, row, head */
  const uint32_t* keep;          /* NULL: every row counts toward the scale */
  int64_t keep_batch_stride;     /* words; 0 shares one mask over the batch */
  void* out;                     /* contiguous (batch, rows, heads, 128) e4m3 */
  float* descale;                /* heads fp32 */
} dgxm_quant_item;

int dgxm_quantize_e4m3_per_head_batch(int32_t n, const dgxm_quant_item* items, void* stream);

/* ------------------------------------------------------------ ring attention */
/*
 * Ring attention over the ranks of `comm` (the ring group): every rank holds
 * its own query rows and one key/value block; the blocks rotate over NVLink
 * (copy-engine peer copies into the next rank's window, overlapped with the
 * attention of the current block) and the R partial results are merged by
 * LSE in fp32.  Keys/values and the output must be contiguous (B, L, H, D);
 * lse (may be NULL) is contiguous fp32 (B, H, Lq).  The comm window needs
 * dgxm_ring_window_bytes(desc); `workspace` (scratch owned by the caller,
 * 256-byte aligned) needs dgxm_ring_workspace_bytes(desc, R).  bf16 or f16
 * inputs; e4m3 inputs go through dgxm_ring_attn_fwd_fp8.
 *
 * Replaces the ring loop of xfuser/yunchang that adapters/base.py:320 reaches
 * when the ring degree exceeds one (block contract:
 * adapters/cudnn_ring_attention.py:61-89).
 */
int64_t dgxm_ring_window_bytes(const dgxm_attn_desc* desc);
int64_t dgxm_ring_workspace_bytes(const dgxm_attn_desc* desc, int32_t ring_world);
int dgxm_ring_attn_fwd(dgxm_comm* comm, const dgxm_attn_desc* desc, const void* q, const void* k,
                       const void* v, void* o, float* lse, void* workspace,
                       int64_t workspace_bytes, void* stream);

/*
 * The same over e4m3 inputs (desc->in_dtype DGXM_DTYPE_E4M3, bf16 output):
 * q_descale are the per-head fp32 descales of this rank's query rows,
 * k_descale / v_descale those of this rank's key/value block.  Each block
 * rotates with the descales it was quantised with (they ride behind it in
 * the window slot), so every ring step attends one block under its own
 * per-head scales -- what an inner FP8 kernel that quantises its own inputs
 * sees when the reference's ring loop calls it block by block.  The partial
 * results stay fp32 and merge by LSE as in dgxm_ring_attn_fwd.
 */
int dgxm_ring_attn_fwd_fp8(dgxm_comm* comm, const dgxm_attn_desc* desc, const void* q,
                           const void* k, const void* v, const float* q_descale,
                           const float* k_descale, const float* v_descale, void* o, float* lse,
                           void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Ring attention that allocates nothing, for callers that cannot call
 * cudaMalloc at attention time: a host runtime whose device memory is all
 * owned by another allocator with a fixed budget (a request outside it
 * would break the budget or fail), or a caller on a latency-critical path
 * where cudaMalloc would synchronise the device.  It has no counterpart in
 * the reference (which always allocates through torch).
 *
 * Same contract as dgxm_ring_attn_fwd, except that the per-step partial
 * results live in one 32 MiB array of module memory on each device that
 * loads this library (held until the process exits) instead of a caller
 * workspace: shapes needing more than dgxm_ring_noalloc_max_bytes() of
 * scratch are refused with DGXM_ERR_INVALID.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress); make that first
 * call before any stream capture.  Every call on a device shares the array,
 * so calls whose work overlaps on the GPU race; nothing in it needs clearing,
 * since every step rewrites its whole partial result.  The comm (created
 * earlier with dgxm_comm_create) supplies the rotation buffers and streams.
 */
int64_t dgxm_ring_noalloc_max_bytes(void);
int dgxm_ring_attn_fwd_noalloc(dgxm_comm* comm, const dgxm_attn_desc* desc, const void* q,
                               const void* k, const void* v, void* o, float* lse, void* stream);

/* ------------------------------------------------------------ full-context ring */
/*
 * The Wan Ring2 full-context path (adapters/wan_ring_full_context.py:203-295
 * gather, :422-449 local-Q x full-KV flash call): each rank's K/V block
 * (B, L, H_kv, D) is stored over NVLink into rank-major slots
 * [rank*L, (rank+1)*L) of every rank's window, then this rank's Q attends the
 * whole (B, R*L) key axis in one call -- exact, no LSE merge.  desc describes
 * the LOCAL shapes (kv_len = L); o and lse are this rank's (B, Lq, H, D) and
 * (B, H, Lq).  bf16 or f16 inputs; any ring degree R = comm world <= 8.  The window
 * must hold dgxm_full_context_window_bytes(desc, R) (two alternating buffers,
 * so one barrier per call suffices).  Collective: every rank of the comm
 * calls it in the same order with the same shapes.
 */
int64_t dgxm_full_context_window_bytes(const dgxm_attn_desc* desc, int32_t world);
/*
 * The store half of the full-context gather, for callers that own their
 * destination buffers and order them themselves (no barrier): this rank's
 * K and V blocks (desc: batch, kv_len, kv_heads, head_dim 128, k/v strides,
 * in_dtype bf16 or f16) go into rank-major rows [rank*L, (rank+1)*L) of every
 * rank's contiguous (batch, world*L, kv_heads, head_dim) tensors dst_k[r] /
 * dst_v[r], all addressable from this rank.  The batch_isend_irecv exchange
 * of adapters/wan_ring_full_context.py:203-295 as one launch of stores.
 */
int dgxm_kv_gather_store(const dgxm_attn_desc* desc, int32_t world, int32_t rank, const void* k,
                         const void* v, void* const* dst_k, void* const* dst_v, void* stream);
int dgxm_full_context_attn_fwd(dgxm_comm* comm, const dgxm_attn_desc* desc, const void* q,
                               const void* k, const void* v, void* o, float* lse, void* stream);

/* ------------------------------------------------------------ sequence-shard collectives */
/*
 * sp_gather (adapters/base.py:126-131): every rank's contiguous chunk of
 * seq_local rows (rank r holds gathered rows [r*seq_local, (r+1)*seq_local))
 * is stored over NVLink into every rank's window at window_offset, as the
 * trimmed (batch, orig_len, row_bytes) tensor; rows at or past orig_len (the
 * divisibility pad of shard_seq, adapters/base.py:91-123) are not sent.  A
 * flag barrier follows, so on return (in stream order) each rank's own
 * window holds the whole trimmed tensor.  Rows, strides and the source are
 * 16-byte aligned.  Collective over the comm.
 */
typedef struct dgxm_seq_gather_desc {
  int32_t batch;
  int32_t seq_local;
  int32_t orig_len;
  int32_t row_bytes;
  int64_t src_batch_stride; /* bytes */
  int64_t src_row_stride;   /* bytes */
} dgxm_seq_gather_desc;

int dgxm_seq_allgather(dgxm_comm* comm, const dgxm_seq_gather_desc* desc, const void* src,
                       int64_t window_offset, void* stream);
/* The store half of dgxm_seq_allgather (no barrier), for callers that own the
 * destinations: this rank's rows into dst[r], rank r's trimmed (batch,
 * orig_len, row_bytes) buffer, for every r < world (16-byte aligned). */
int dgxm_seq_gather_store(const dgxm_seq_gather_desc* desc, int32_t world, int32_t rank,
                          const void* src, void* const* dst, void* stream);

/*
 * The shared NVFP4 activation scale (adapters/quant_activation_scale.py:
 * 222-246): amax(|x|) over this rank's (rows, cols) shard (row_stride in
 * elements), max-reduced over every rank of the comm (the sequence x CFG
 * ranks of one model call), written as fp32 to amax_out (may be NULL) and as
 * dtype(dtype(amax) * (1 / divisor)) to scale_out -- the divide in the
 * activation dtype, as comfy orders it.  dtype: DGXM_DTYPE_BF16, _F16 or
 * _F32.  NaN propagates; a barrier that gives up writes NaN and sets the
 * device error word.  Collective over the comm.
 */
int dgxm_shared_amax_scale(dgxm_comm* comm, const void* x, int64_t rows, int64_t cols,
                           int64_t row_stride, int32_t dtype, float divisor, void* scale_out,
                           float* amax_out, void* stream);

/* ------------------------------------------------------------ fused QKV projection */
/*
 * y = x W^T + bias for one token stream of this rank (x: m rows of k bf16
 * features, row stride x_row_stride elements; W: the Linear weight,
 * (3 * heads * 128, k) bf16 row-major; bias: 3 * heads * 128 bf16 or NULL),
 * rounded to bf16, then per head: q and k through the per-head RMSNorm
 * (norm_mode DGXM_NORM_HEAD: bf16(y * rsqrt(mean(y^2) + eps)) then
 * bf16(n * w), weights of 128 bf16 or NULL) and RoPE (rope: (seq_local, 64, 2)
 * fp32 cos/sin by local row, or NULL; x, W and rope 16-byte aligned; heads
 * even, two heads per tile; the kernel runs as clusters of two CTAs, and a
 * device that cannot hold one returns DGXM_ERR_CUDA), and every 128-wide
 * head row stored into
 * dst[t * world + r] -- rank r's contiguous (world * seq_local, heads/world,
 * 128) bf16 receive tensor t (0 q, 1 k, 2 v) -- at the gathered row of local
 * row row0 + i (joint order seg0 as in dgxm_a2a_desc).  One tcgen05 kernel:
 * the QKV Linear, the QKNorm and RoPE of the Flux/Krea2 blocks and the
 * sequence->head all-to-all (adapters/usp_full_axis.py:27-29).  Batch 1 per
 * call; the text and image streams of a joint block are two calls with their
 * own weights and row0.  Follow with dgxm_comm_barrier before any rank reads
 * its receive tensors.
 */
typedef struct dgxm_qkv_gemm_desc {
  int32_t world;
  int32_t rank;
  int32_t m;          /* rows of x in this call */
  int32_t k;          /* input features; a multiple of 8 */
  int32_t heads;      /* query heads (== key/value heads); heads % world == 0 */
  int32_t seq_local;  /* rows this rank holds over all streams */
  int32_t row0;       /* local row of x's first row */
  int32_t seg0;       /* joint order: leading rows per rank (0 = rank-major) */
  int32_t norm_mode;  /* DGXM_NORM_NONE or DGXM_NORM_HEAD */
  float eps;
  int64_t x_row_stride; /* elements; a multiple of 8 */
} dgxm_qkv_gemm_desc;

int dgxm_qkv_gemm_prologue_scatter(const dgxm_qkv_gemm_desc* desc, const void* x, const void* w_qkv,
                                   const void* bias, const void* norm_q_w, const void* norm_k_w,
                                   const float* rope, void* const* dst, void* stream);

/*
 * One token stream of dgxm_qkv_gemm_prologue_scatter_streams: its m rows of
 * x (row stride x_row_stride elements, a multiple of 8) at local row row0,
 * its Linear weight and bias, and its own per-head QKNorm weights (a joint
 * block's text and image streams each have theirs).
 */
typedef struct dgxm_qkv_stream {
  const void* x;
  const void* w_qkv;     /* (3 * heads * 128, k) bf16 */
  const void* bias;      /* 3 * heads * 128 bf16, or NULL */
  const void* norm_q_w;  /* 128 bf16, or NULL */
  const void* norm_k_w;
  int64_t x_row_stride;
  int32_t m;
  int32_t row0;
} dgxm_qkv_stream;

/*
 * dgxm_qkv_gemm_prologue_scatter for the text and image streams of a joint
 * block (n_streams 1 or 2) in one launch: the pair tiles of both projections
 * share one grid, so neither stream's partial last wave of tiles idles the
 * GPU.  desc gives what the streams share (world, rank, k, heads, seq_local,
 * seg0, norm_mode, eps); its m, row0 and x_row_stride are not read.  Each
 * head row is computed exactly as by one dgxm_qkv_gemm_prologue_scatter call
 * per stream.  Replaces the same reference calls (adapters/usp_full_axis.py:27-29
 * after the blocks' QKV Linear, QKNorm and RoPE).
 */
int dgxm_qkv_gemm_prologue_scatter_streams(const dgxm_qkv_gemm_desc* desc, int32_t n_streams,
                                           const dgxm_qkv_stream* streams, const float* rope,
                                           void* const* dst, void* stream);

/* ------------------------------------------------------------ CFG combine */
/*
 * out = uncond + (cond - uncond) * cfg_scale over n contiguous elements of
 * dtype (DGXM_DTYPE_F32, _BF16 or _F16), each operation rounded to dtype with
 * the scale taken as fp32 -- comfy's default cfg_function as the dual-model
 * CFG split runs it after its all-gather (actor/dual_model_cfg.py:75-94).
 * The three pointers are 16-byte aligned; out may alias cond or uncond.
 */
int dgxm_cfg_combine(const void* cond, const void* uncond, int64_t n, int32_t dtype,
                     double cfg_scale, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DGXM_SP_H */
