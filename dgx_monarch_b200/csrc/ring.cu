// Ring attention over the ranks of one comm: K/V blocks rotate over NVLink
// while the attention of the current block runs, then the per-block partial
// results are merged by log-sum-exp.
//
// Step t on rank r (R ranks, next = r+1 mod R):
//   side stream : copy the block r holds (its own at t = 0, else the one
//                 received at t-1) into next's window buffer t % 2 -- a
//                 copy-engine peer copy, so it uses no SMs;
//   main stream : attention(Q, block) -> fp32 partial out_t and lse_t;
//   join, then dgxm_comm_barrier: every rank's copy has landed and every
//   rank finished step t, so buffer (t+1) % 2 may be overwritten next.
// After R steps one closing barrier (so the next call's first copy cannot
// overwrite a block a neighbour still attends), then the LSE merge writes the
// output.  The block a rank attends at step t came from rank (r - t) mod R,
// the oracle's ring order.
//
// Replaces the ring loop of xfuser/yunchang reached from
// adapters/base.py:320 (usp_attn with ring degree > 1), with the per-block
// contract of adapters/cudnn_ring_attention.py:61-89 and an fp32 merge (the
// reason the reference carries a cuDNN ring processor at all,
// adapters/wan_ring_attention.py:1-9).

namespace dgxm {

static int64_t ring_block_bytes(const dgxm_attn_desc* d) {
  const int64_t eb = d->in_dtype == DGXM_DTYPE_E4M3 ? 1 : 2;
  return static_cast<int64_t>(d->batch) * d->kv_len * d->kv_heads * d->head_dim * eb;
}

static int64_t round256(int64_t x) { return (x + 255) / 256 * 256; }

// One window slot holds a K or V block; an e4m3 block carries its per-head
// fp32 descales right behind it, so they rotate with the block.
static int64_t ring_slot_bytes(const dgxm_attn_desc* d) {
  const int64_t descales = d->in_dtype == DGXM_DTYPE_E4M3 ? round256(int64_t(d->kv_heads) * 4) : 0;
  return round256(ring_block_bytes(d)) + descales;
}

static int64_t ring_part_bytes(const dgxm_attn_desc* d) {
  return round256(static_cast<int64_t>(d->batch) * d->q_len * d->q_heads * d->head_dim * 4);
}

static int64_t ring_lse_bytes(const dgxm_attn_desc* d) {
  return round256(static_cast<int64_t>(d->batch) * d->q_heads * d->q_len * 4);
}

static bool contiguous_bhld(const int64_t* s, const dgxm_attn_desc* d, int heads, int len) {
  return s[2] == d->head_dim && s[1] == static_cast<int64_t>(heads) * d->head_dim &&
         (d->batch == 1 || s[0] == static_cast<int64_t>(len) * heads * d->head_dim);
}

// The LSE merge writes (B, H, Lq) contiguously, so a strided lse is refused
// rather than scrambled.
static bool contiguous_bhl(const int64_t* s, const dgxm_attn_desc* d) {
  return s[2] == 1 && s[1] == d->q_len &&
         (d->batch == 1 || s[0] == static_cast<int64_t>(d->q_heads) * d->q_len);
}

// Every launch of a ring call goes to the current device, and the comm's
// window and streams live on the device it was created on.
static int check_comm_device(const dgxm_comm* c) {
  int dev = -1;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != c->device)
    return fail(DGXM_ERR_INVALID, "the current device is %d but the comm lives on device %d", dev,
                c->device);
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int64_t dgxm_ring_window_bytes(const dgxm_attn_desc* d) {
  if (d == nullptr) return -1;
  return 4 * dgxm::ring_slot_bytes(d);
}

extern "C" int64_t dgxm_ring_workspace_bytes(const dgxm_attn_desc* d, int32_t ring_world) {
  if (d == nullptr || ring_world < 1) return -1;
  return static_cast<int64_t>(ring_world) * (dgxm::ring_part_bytes(d) + dgxm::ring_lse_bytes(d));
}

namespace dgxm {

// The ring loop, partial results in `workspace` (any device memory of at
// least dgxm_ring_workspace_bytes, 256-byte aligned).  e4m3 inputs take
// per-head fp32 descales: q's for the local rows, k's and v's for this
// rank's block (each block keeps the scales it was quantised with).
static int ring_attn_impl(dgxm_comm* c, const dgxm_attn_desc* d, const void* q, const void* k,
                          const void* v, const float* q_descale, const float* k_descale,
                          const float* v_descale, void* o, float* lse, void* workspace,
                          int64_t workspace_bytes, void* stream) {
  if (c == nullptr || d == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or descriptor");
  if (int rc0 = check_comm_device(c)) return rc0;
  const int world = c->world;
  if (world > kMaxMergeParts)
    return fail(DGXM_ERR_UNSUPPORTED, "ring degree %d exceeds %d", world, kMaxMergeParts);
  // The layout rules hold at every ring degree, so a call that runs at one
  // degree runs at all of them.
  if (!contiguous_bhld(d->k_stride, d, d->kv_heads, d->kv_len) ||
      !contiguous_bhld(d->v_stride, d, d->kv_heads, d->kv_len))
    return fail(DGXM_ERR_INVALID, "ring attention needs contiguous (B, L, H, D) keys and values");
  if (!contiguous_bhld(d->o_stride, d, d->q_heads, d->q_len))
    return fail(DGXM_ERR_INVALID, "ring attention needs a contiguous (B, L, H, D) output");
  if (lse != nullptr && !contiguous_bhl(d->lse_stride, d))
    return fail(DGXM_ERR_INVALID, "ring attention needs a contiguous (B, H, L) lse");
  const bool fp8 = d->in_dtype == DGXM_DTYPE_E4M3;
  if (fp8 && (q_descale == nullptr || k_descale == nullptr || v_descale == nullptr))
    return fail(DGXM_ERR_INVALID, "e4m3 ring attention takes q, k and v descales (dgxm_ring_attn_fwd_fp8)");
  if (!fp8 && (q_descale != nullptr || k_descale != nullptr || v_descale != nullptr))
    return fail(DGXM_ERR_INVALID, "descales belong to e4m3 inputs only");
  if (world == 1) return dgxm_attn_fwd(d, q, k, v, q_descale, k_descale, v_descale, o, lse, stream);
  if (d->in_dtype != DGXM_DTYPE_BF16 && d->in_dtype != DGXM_DTYPE_F16 && !fp8)
    return fail(DGXM_ERR_UNSUPPORTED, "ring attention runs bf16, f16 or e4m3 inputs");
  const int64_t block = ring_block_bytes(d);
  const int64_t slot = ring_slot_bytes(d);
  const int64_t scales_at = round256(block);                       // descales inside a slot
  const int64_t scale_bytes = int64_t(d->kv_heads) * 4;
  if (4 * slot > c->bytes)
    return fail(DGXM_ERR_INVALID, "comm window of %lld bytes is smaller than the %lld the ring needs",
                (long long)c->bytes, (long long)(4 * slot));
  const int64_t need = dgxm_ring_workspace_bytes(d, world);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(DGXM_ERR_INVALID, "ring workspace of %lld bytes is smaller than %lld",
                (long long)workspace_bytes, (long long)need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(DGXM_ERR_INVALID, "ring workspace must be 256-byte aligned");
  for (int r = 0; r < world; ++r)
    if (c->peers[r] == nullptr) return fail(DGXM_ERR_STATE, "peer %d window is not mapped", r);
  if (c->side == nullptr) return fail(DGXM_ERR_STATE, "the comm has no copy stream (world 1?)");
  int rc = DGXM_OK;
  cudaStream_t main = static_cast<cudaStream_t>(stream);
  const int next = (c->rank + 1) % world;
  char* mine = c->local + kFlagBytes;
  char* theirs = c->peers[next] + kFlagBytes;
  char* parts_out = static_cast<char*>(workspace);
  char* parts_lse = parts_out + world * ring_part_bytes(d);
  const void* outs[kMaxMergeParts];
  const float* lses[kMaxMergeParts];

  dgxm_attn_desc step = *d;
  step.out_dtype = DGXM_DTYPE_F32;
  step.o_stride[0] = static_cast<int64_t>(d->q_len) * d->q_heads * d->head_dim;
  step.o_stride[1] = static_cast<int64_t>(d->q_heads) * d->head_dim;
  step.o_stride[2] = d->head_dim;
  step.lse_stride[0] = static_cast<int64_t>(d->q_heads) * d->q_len;
  step.lse_stride[1] = d->q_len;
  step.lse_stride[2] = 1;

  const char* cur_k = static_cast<const char*>(k);
  const char* cur_v = static_cast<const char*>(v);
  const float* cur_kd = k_descale;
  const float* cur_vd = v_descale;
  DGXM_CUDA_TRY(cudaEventRecord(c->ev_main, main));
  for (int t = 0; t < world; ++t) {
    const bool send = t < world - 1;
    const int buf = t % 2;
    if (send) {
      DGXM_CUDA_TRY(cudaStreamWaitEvent(c->side, c->ev_main, 0));
      DGXM_CUDA_TRY(cudaMemcpyAsync(theirs + (2 * buf) * slot, cur_k, block, cudaMemcpyDefault, c->side));
      DGXM_CUDA_TRY(cudaMemcpyAsync(theirs + (2 * buf + 1) * slot, cur_v, block, cudaMemcpyDefault, c->side));
      if (fp8) {
        DGXM_CUDA_TRY(cudaMemcpyAsync(theirs + (2 * buf) * slot + scales_at, cur_kd, scale_bytes,
                                      cudaMemcpyDefault, c->side));
        DGXM_CUDA_TRY(cudaMemcpyAsync(theirs + (2 * buf + 1) * slot + scales_at, cur_vd, scale_bytes,
                                      cudaMemcpyDefault, c->side));
      }
      DGXM_CUDA_TRY(cudaEventRecord(c->ev_side, c->side));
    }
    void* po = parts_out + t * ring_part_bytes(d);
    float* pl = reinterpret_cast<float*>(parts_lse + t * ring_lse_bytes(d));
    outs[t] = po;
    lses[t] = pl;
    rc = dgxm_attn_fwd(&step, q, cur_k, cur_v, q_descale, cur_kd, cur_vd, po, pl, main);
    if (rc) return rc;
    if (send) {
      DGXM_CUDA_TRY(cudaStreamWaitEvent(main, c->ev_side, 0));
      rc = dgxm_comm_barrier(c, main);
      if (rc) return rc;
      DGXM_CUDA_TRY(cudaEventRecord(c->ev_main, main));
      cur_k = mine + (2 * buf) * slot;
      cur_v = mine + (2 * buf + 1) * slot;
      if (fp8) {
        cur_kd = reinterpret_cast<const float*>(mine + (2 * buf) * slot + scales_at);
        cur_vd = reinterpret_cast<const float*>(mine + (2 * buf + 1) * slot + scales_at);
      }
    }
  }
  // The last step attends the block in this rank's buffer (R - 2) % 2, and the
  // next call's first copy into a neighbour's buffer 0 waits only on that
  // neighbour's own stream.  A closing barrier orders every rank's last
  // attention before any rank's next call can overwrite the buffer it reads.
  rc = dgxm_comm_barrier(c, main);
  if (rc) return rc;
  return dgxm_lse_merge(d->batch, d->q_len, d->q_heads, d->head_dim, world, outs, DGXM_DTYPE_F32,
                        lses, o, d->out_dtype, lse, stream);
}

}  // namespace dgxm

extern "C" int dgxm_ring_attn_fwd(dgxm_comm* c, const dgxm_attn_desc* d, const void* q,
                                  const void* k, const void* v, void* o, float* lse,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  return dgxm::ring_attn_impl(c, d, q, k, v, nullptr, nullptr, nullptr, o, lse, workspace,
                              workspace_bytes, stream);
}

extern "C" int dgxm_ring_attn_fwd_fp8(dgxm_comm* c, const dgxm_attn_desc* d, const void* q,
                                      const void* k, const void* v, const float* q_descale,
                                      const float* k_descale, const float* v_descale, void* o,
                                      float* lse, void* workspace, int64_t workspace_bytes,
                                      void* stream) {
  if (d != nullptr && d->in_dtype != DGXM_DTYPE_E4M3)
    return dgxm::fail(DGXM_ERR_INVALID, "dgxm_ring_attn_fwd_fp8 takes e4m3 inputs");
  return dgxm::ring_attn_impl(c, d, q, k, v, q_descale, k_descale, v_descale, o, lse, workspace,
                              workspace_bytes, stream);
}

// ---------------------------------------------------------------- without allocation
// Partial results of dgxm_ring_attn_fwd_noalloc live in this module-scope
// array instead of a caller's workspace.  It is created when the library
// loads on a device and stays until the process exits; every call shares it.
namespace dgxm {

constexpr int64_t kRingStaticScratchBytes = int64_t(32) << 20;  // 32 MiB
static __device__ __align__(256) unsigned char g_ring_static_scratch[kRingStaticScratchBytes];

// The device address of the array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, looked up once per device (with that device current)
// and cached.
static int ring_static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  DGXM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(DGXM_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ring_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(ring scratch)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int64_t dgxm_ring_noalloc_max_bytes(void) { return dgxm::kRingStaticScratchBytes; }

extern "C" int dgxm_ring_attn_fwd_noalloc(dgxm_comm* c, const dgxm_attn_desc* d, const void* q,
                                          const void* k, const void* v, void* o, float* lse,
                                          void* stream) {
  using namespace dgxm;
  if (c == nullptr || d == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or descriptor");
  if (int rc0 = check_comm_device(c)) return rc0;
  // One rank attends its own block: no partial results, so no scratch.
  if (c->world == 1)
    return ring_attn_impl(c, d, q, k, v, nullptr, nullptr, nullptr, o, lse, nullptr, 0, stream);
  const int64_t need = dgxm_ring_workspace_bytes(d, c->world);
  if (need < 0 || need > kRingStaticScratchBytes)
    return fail(DGXM_ERR_INVALID,
                "ring attention of this shape needs %lld bytes of scratch; the allocation-free "
                "entry point holds at most %lld (32 MiB). Use dgxm_ring_attn_fwd with a workspace.",
                (long long)need, (long long)kRingStaticScratchBytes);
  void* scratch = nullptr;
  const int rc = ring_static_scratch(&scratch);
  if (rc != DGXM_OK) return rc;
  return ring_attn_impl(c, d, q, k, v, nullptr, nullptr, nullptr, o, lse, scratch,
                        kRingStaticScratchBytes, stream);
}
