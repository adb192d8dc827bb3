// Full-context ring attention: every rank gathers the whole key/value axis
// into its own window, then attends its local query rows against it in one
// kernel call -- no per-block partial results and no LSE merge.
//
// Replaces the Wan Ring2 full-context path of the reference
// (adapters/wan_ring_full_context.py:203-295 gathers each batch item's K/V
// into sequence-rank slots with batch_isend_irecv; :422-449 runs one ATen
// flash call of local Q against full K/V per batch item).  Here the gather is
// one kernel of NVLink peer stores for all batch items and both tensors, and
// any ring degree up to 8 is accepted (the reference's refusal of degrees
// other than 2 stays in the Python drop-in).
//
// Window layout (after the flag area), two buffers used on alternate calls:
//   [K_full | V_full] buffer 0, [K_full | V_full] buffer 1
// each (B, R*L, H_kv, D) contiguous, rank r's rows at [r*L, (r+1)*L) of every
// batch item (the rank-major slots of the reference).
//
// One barrier per call is enough with two buffers: a rank writes buffer
// (n+1)%2 only after passing barrier n, which every peer reaches after its
// attention of call n-1 -- the last reader of that buffer -- in stream order.

namespace dgxm {

struct KvGatherParams {
  const char* src[2];                 // local K, V (B, L, H, D), byte strides below
  int64_t s_sb[2], s_sl[2], s_sh[2];
  char* dst[2][DGXM_MAX_WORLD];       // K_full / V_full of each rank's window
  int world, rank;
  int batch, seq_local, heads, head_bytes;
};

// One thread loads 16 bytes of a head row once and stores them into every
// rank's window (its own first, then the peers in ring order).  A warp moves
// two consecutive 256-byte head rows, so loads and stores are coalesced.
__global__ void __launch_bounds__(256) kv_allgather_kernel(const __grid_constant__ KvGatherParams p) {
  const int chunks = p.head_bytes / 16;
  const int64_t per_tensor = static_cast<int64_t>(p.batch) * p.seq_local * p.heads * chunks;
  const int64_t total = 2 * per_tensor;
  const int64_t seq_full = static_cast<int64_t>(p.seq_local) * p.world;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = i >= per_tensor ? 1 : 0;
    int64_t rem = i - t * per_tensor;
    const int part = static_cast<int>(rem % chunks);
    rem /= chunks;
    const int h = static_cast<int>(rem % p.heads);
    rem /= p.heads;
    const int l = static_cast<int>(rem % p.seq_local);
    const int b = static_cast<int>(rem / p.seq_local);
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(
        p.src[t] + b * p.s_sb[t] + l * p.s_sl[t] + h * p.s_sh[t]) + part);
    const int64_t row = static_cast<int64_t>(b) * seq_full + static_cast<int64_t>(p.rank) * p.seq_local + l;
    const int64_t off = (row * p.heads + h) * p.head_bytes + part * 16;
    for (int j = 0; j < p.world; ++j) {
      const int r = (p.rank + j) % p.world;
      *reinterpret_cast<uint4*>(p.dst[t][r] + off) = val;
    }
  }
}

static int64_t full_kv_bytes(const dgxm_attn_desc* d, int world) {
  return static_cast<int64_t>(d->batch) * world * d->kv_len * d->kv_heads * d->head_dim * 2;
}

}  // namespace dgxm

extern "C" int64_t dgxm_full_context_window_bytes(const dgxm_attn_desc* d, int32_t world) {
  if (d == nullptr || world < 1) return -1;
  return 4 * dgxm::round256(dgxm::full_kv_bytes(d, world));
}

namespace dgxm {

// Checks of the local K/V blocks the gather reads (16-bit elements).
static int check_kv_block(const dgxm_attn_desc* d, const void* k, const void* v) {
  if (d->in_dtype != DGXM_DTYPE_BF16 && d->in_dtype != DGXM_DTYPE_F16)
    return fail(DGXM_ERR_UNSUPPORTED, "full-context ring attention runs bf16 or f16 inputs");
  if (d->head_dim != kHeadDim)
    return fail(DGXM_ERR_UNSUPPORTED, "head_dim %d is not supported (this build runs 128)",
                d->head_dim);
  if (d->batch <= 0 || d->kv_len <= 0 || d->kv_heads <= 0)
    return fail(DGXM_ERR_INVALID, "empty key/value block (batch=%d kv_len=%d kv_heads=%d)",
                d->batch, d->kv_len, d->kv_heads);
  if (k == nullptr || v == nullptr) return fail(DGXM_ERR_INVALID, "k and v must be non-NULL");
  const void* kv[2] = {k, v};
  const int64_t* strides[2] = {d->k_stride, d->v_stride};
  for (int t = 0; t < 2; ++t) {
    if (reinterpret_cast<uintptr_t>(kv[t]) % 16)
      return fail(DGXM_ERR_INVALID, "%s is not 16-byte aligned", t ? "v" : "k");
    for (int s = 0; s < 3; ++s)
      if ((strides[t][s] * 2) % 16)
        return fail(DGXM_ERR_INVALID, "%s strides must be multiples of 16 bytes", t ? "v" : "k");
  }
  return DGXM_OK;
}

// This rank's K and V blocks into rank-major slots of every rank's full K/V.
static int launch_kv_gather(const dgxm_attn_desc* d, int world, int rank, const void* k,
                            const void* v, char* const* dst_k, char* const* dst_v, cudaStream_t st) {
  const void* kv[2] = {k, v};
  const int64_t* strides[2] = {d->k_stride, d->v_stride};
  char* const* dst[2] = {dst_k, dst_v};
  KvGatherParams p;
  memset(&p, 0, sizeof(p));
  for (int t = 0; t < 2; ++t) {
    p.src[t] = static_cast<const char*>(kv[t]);
    p.s_sb[t] = strides[t][0] * 2;
    p.s_sl[t] = strides[t][1] * 2;
    p.s_sh[t] = strides[t][2] * 2;
    for (int r = 0; r < world; ++r) p.dst[t][r] = dst[t][r];
  }
  p.world = world;
  p.rank = rank;
  p.batch = d->batch;
  p.seq_local = d->kv_len;
  p.heads = d->kv_heads;
  p.head_bytes = d->head_dim * 2;
  const int64_t items = 2 * static_cast<int64_t>(d->batch) * d->kv_len * d->kv_heads * (p.head_bytes / 16);
  kv_allgather_kernel<<<grid_for(items, 256), 256, 0, st>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int dgxm_kv_gather_store(const dgxm_attn_desc* d, int32_t world, int32_t rank,
                                    const void* k, const void* v, void* const* dst_k,
                                    void* const* dst_v, void* stream) {
  using namespace dgxm;
  if (d == nullptr) return fail(DGXM_ERR_INVALID, "NULL descriptor");
  if (world < 1 || world > DGXM_MAX_WORLD || rank < 0 || rank >= world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", rank, world);
  if (int rc = check_kv_block(d, k, v)) return rc;
  if (dst_k == nullptr || dst_v == nullptr) return fail(DGXM_ERR_INVALID, "destination arrays are NULL");
  char* bk[DGXM_MAX_WORLD];
  char* bv[DGXM_MAX_WORLD];
  for (int r = 0; r < world; ++r) {
    if (dst_k[r] == nullptr || dst_v[r] == nullptr || reinterpret_cast<uintptr_t>(dst_k[r]) % 16 ||
        reinterpret_cast<uintptr_t>(dst_v[r]) % 16)
      return fail(DGXM_ERR_INVALID, "destination %d is NULL or not 16-byte aligned", r);
    bk[r] = static_cast<char*>(dst_k[r]);
    bv[r] = static_cast<char*>(dst_v[r]);
  }
  return launch_kv_gather(d, world, rank, k, v, bk, bv, static_cast<cudaStream_t>(stream));
}

extern "C" int dgxm_full_context_attn_fwd(dgxm_comm* c, const dgxm_attn_desc* d, const void* q,
                                          const void* k, const void* v, void* o, float* lse,
                                          void* stream) {
  using namespace dgxm;
  if (c == nullptr || d == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or descriptor");
  const int world = c->world;
  if (world == 1) return dgxm_attn_fwd(d, q, k, v, nullptr, nullptr, nullptr, o, lse, stream);
  if (int rc = check_kv_block(d, k, v)) return rc;
  const int64_t full = full_kv_bytes(d, world);
  const int64_t slot = round256(full);
  if (4 * slot > c->bytes)
    return fail(DGXM_ERR_INVALID, "comm window of %lld bytes is smaller than the %lld the "
                "full-context gather needs", (long long)c->bytes, (long long)(4 * slot));
  for (int r = 0; r < world; ++r)
    if (c->peers[r] == nullptr) return fail(DGXM_ERR_STATE, "peer %d window is not mapped", r);

  const int buf = static_cast<int>(c->fc_calls & 1u);
  char* bk[DGXM_MAX_WORLD];
  char* bv[DGXM_MAX_WORLD];
  for (int r = 0; r < world; ++r) {
    bk[r] = c->peers[r] + kFlagBytes + (2 * buf) * slot;
    bv[r] = c->peers[r] + kFlagBytes + (2 * buf + 1) * slot;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = launch_kv_gather(d, world, c->rank, k, v, bk, bv, st)) return rc;
  c->fc_calls += 1;
  int rc = dgxm_comm_barrier(c, stream);
  if (rc) return rc;

  dgxm_attn_desc full_desc = *d;
  full_desc.kv_len = d->kv_len * world;
  const int64_t row = static_cast<int64_t>(d->kv_heads) * d->head_dim;
  for (int64_t* s : {full_desc.k_stride, full_desc.v_stride}) {
    s[0] = full_desc.kv_len * row;
    s[1] = row;
    s[2] = d->head_dim;
  }
  char* mine = c->local + kFlagBytes;
  return dgxm_attn_fwd(&full_desc, q, mine + (2 * buf) * slot, mine + (2 * buf + 1) * slot, nullptr,
                       nullptr, nullptr, o, lse, stream);
}
