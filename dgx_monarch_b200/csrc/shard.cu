// Sequence-shard collectives over the peer windows: the all-gather behind
// sp_gather and the shared NVFP4 activation amax.
//
// sp_gather (adapters/base.py:126-131) all-gathers each rank's contiguous
// sequence chunk along the token axis and trims the divisibility pad.  Here
// each rank stores its rows straight into every rank's window, already in
// the trimmed (B, orig_len, row) layout (rows at or past orig_len -- the pad
// -- are never sent), then one flag barrier makes them visible.
//
// shared_activation_scale (adapters/quant_activation_scale.py:222-246)
// reduces the local amax(|x|) of each shard by a max all-reduce over the
// sequence and CFG groups, casts it to the activation dtype and divides by
// 448 * 6.  Here: one grid kernel takes the local amax (float bits,
// atomicMax), and one single-warp kernel publishes it into every rank's
// window, runs the flag barrier inline, and reduces the slots it received.
// The slots alternate by barrier-epoch parity: a rank publishes at epoch e
// only after passing barrier e-1, and every peer read its epoch e-2 slots
// inside the kernel that ran before it arrived at barrier e-1, so a slot is
// never overwritten unread.  The epoch comes from the device counter, so the
// exchange replays correctly inside a captured CUDA graph.

namespace dgxm {

// Flag-area layout (the first kFlagBytes of every window): barrier flags at
// byte 0 (one int per rank), amax slots at kAmaxSlots (two parities x 8
// ranks of fp32), this rank's local amax accumulator at kAmaxLocal, the
// barrier count at kEpochCounter.
constexpr int64_t kAmaxSlots = 2048;
constexpr int64_t kAmaxLocal = 3072;

struct SeqGatherParams {
  const char* src;           // (B, L, row) rows, byte strides below
  int64_t s_sb, s_sl;
  char* dst[DGXM_MAX_WORLD]; // (B, orig_len, row) contiguous on each rank
  int world, rank;
  int batch, seq_local, orig_len;
  int row_bytes;             // multiple of 16
};

// One thread moves 16 bytes of one row to every rank; a warp covers 512
// consecutive bytes of a row, so loads and stores are coalesced.
__global__ void __launch_bounds__(256) seq_allgather_kernel(const __grid_constant__ SeqGatherParams p) {
  const int chunks = p.row_bytes / 16;
  const int64_t total = static_cast<int64_t>(p.batch) * p.seq_local * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int part = static_cast<int>(i % chunks);
    const int64_t rem = i / chunks;
    const int l = static_cast<int>(rem % p.seq_local);
    const int b = static_cast<int>(rem / p.seq_local);
    const int64_t g = static_cast<int64_t>(p.rank) * p.seq_local + l;  // row on the gathered axis
    if (g >= p.orig_len) continue;  // a divisibility pad row: trimmed, never sent
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(p.src + b * p.s_sb + l * p.s_sl) + part);
    const int64_t off = (static_cast<int64_t>(b) * p.orig_len + g) * p.row_bytes + part * 16;
    for (int j = 0; j < p.world; ++j) {
      const int r = (p.rank + j) % p.world;
      *reinterpret_cast<uint4*>(p.dst[r] + off) = val;
    }
  }
}

struct AmaxParams {
  const char* x;       // (rows, cols), row stride in bytes
  int64_t rows, cols, row_stride;
  bool vec;            // rows and the base are 16-byte aligned: 16-byte loads
  unsigned int* local; // fp32 bits of the running max (non-negative: int order = float order)
};

// |v| as fp32 bits.  Non-negative floats order like their bit patterns, and
// a NaN's bits sit above +inf's, so an integer max propagates NaN as torch's
// amax does.
template <typename T>
__device__ __forceinline__ unsigned int abs_bits(T v);
template <>
__device__ __forceinline__ unsigned int abs_bits<__nv_bfloat16>(__nv_bfloat16 v) {
  return (static_cast<unsigned int>(__bfloat16_as_ushort(v)) & 0x7FFFu) << 16;
}
template <>
__device__ __forceinline__ unsigned int abs_bits<__half>(__half v) {
  return __float_as_uint(__half2float(v)) & 0x7FFFFFFFu;
}
template <>
__device__ __forceinline__ unsigned int abs_bits<float>(float v) {
  return __float_as_uint(v) & 0x7FFFFFFFu;
}

__device__ __forceinline__ unsigned int umax(unsigned int a, unsigned int b) { return a > b ? a : b; }

// Blocks stride over rows, threads over a row's 16-byte vectors (or its
// elements when unaligned); one atomicMax per block.
template <typename T>
__global__ void __launch_bounds__(256) amax_local_kernel(const __grid_constant__ AmaxParams p) {
  constexpr int kPerVec = 16 / sizeof(T);
  unsigned int m = 0;
  for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
    const char* row = p.x + r * p.row_stride;
    if (p.vec) {
      const int64_t nvec = p.cols / kPerVec;
      for (int64_t c = threadIdx.x; c < nvec; c += blockDim.x) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row) + c);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int j = 0; j < kPerVec; ++j) m = umax(m, abs_bits<T>(e[j]));
      }
    } else {
      for (int64_t c = threadIdx.x; c < p.cols; c += blockDim.x)
        m = umax(m, abs_bits<T>(reinterpret_cast<const T*>(row)[c]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = umax(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ unsigned int warp_max[8];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int b = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) b = umax(b, warp_max[w]);
    atomicMax(p.local, b);
  }
}

struct AmaxExchangeParams {
  char* peer_flag_area[DGXM_MAX_WORLD];  // every rank's flag area as seen here
  char* my_flag_area;
  int rank, world;
  long long wait_cycles;
  float inv_divisor;   // 1 / divisor, fp32 (the activation dtype's divide by a scalar)
  int dtype;           // output scale dtype
  void* scale_out;     // one element of `dtype`
  float* amax_out;     // the reduced amax, fp32 (may be NULL)
};

// One warp.  Lane i < world publishes this rank's amax into rank i's slot,
// then does rank i's half of the flag barrier (release its flag there,
// acquire the flag rank i left here), then reads the slot rank i filled here.
__global__ void amax_exchange_kernel(const __grid_constant__ AmaxExchangeParams p) {
  const int i = threadIdx.x;
  const int epoch = next_epoch(p.my_flag_area);
  const int parity = epoch & 1;
  float v = 0.f;
  bool ok = true;
  if (i < p.world) {
    const float mine = __uint_as_float(*reinterpret_cast<const unsigned int*>(p.my_flag_area + kAmaxLocal));
    float* slot = reinterpret_cast<float*>(p.peer_flag_area[i] + kAmaxSlots) + parity * DGXM_MAX_WORLD + p.rank;
    *reinterpret_cast<volatile float*>(slot) = mine;
    __threadfence_system();
    int* flag = reinterpret_cast<int*>(p.peer_flag_area[i]) + p.rank;
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
    const int* seen_at = reinterpret_cast<const int*>(p.my_flag_area) + i;
    const long long start = clock64();
    while (true) {
      int seen;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(seen) : "l"(seen_at) : "memory");
      if (seen - epoch >= 0) break;
      if (clock64() - start > p.wait_cycles) {
        report_device_error(kErrPeerTimeout);
        ok = false;
        break;
      }
      __nanosleep(64);
    }
    const float* got = reinterpret_cast<const float*>(p.my_flag_area + kAmaxSlots) + parity * DGXM_MAX_WORLD + i;
    v = *reinterpret_cast<const volatile float*>(got);
  }
  unsigned int m = __float_as_uint(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned int other = __shfl_xor_sync(0xffffffffu, m, o);
    m = other > m ? other : m;
  }
  const bool all_ok = __all_sync(0xffffffffu, ok);  // every lane has read the count
  if (i == 0) {
    *reinterpret_cast<volatile int*>(p.my_flag_area + kEpochCounter) = epoch;
    // A barrier that gave up leaves NaN, never a plausible scale.
    const float amax = all_ok ? __uint_as_float(m) : __int_as_float(0x7FC00000);
    if (p.amax_out != nullptr) *p.amax_out = amax;
    // amax.to(dtype) / divisor in the activation dtype: the cast, then the
    // fp32 product with the reciprocal, rounded once to the dtype.
    if (p.dtype == DGXM_DTYPE_BF16) {
      const float a = __bfloat162float(__float2bfloat16_rn(amax));
      *static_cast<__nv_bfloat16*>(p.scale_out) = __float2bfloat16_rn(a * p.inv_divisor);
    } else if (p.dtype == DGXM_DTYPE_F16) {
      const float a = __half2float(__float2half_rn(amax));
      *static_cast<__half*>(p.scale_out) = __float2half_rn(a * p.inv_divisor);
    } else {
      *static_cast<float*>(p.scale_out) = amax * p.inv_divisor;
    }
  }
}

}  // namespace dgxm

namespace dgxm {

// Checks shared by the collective and the store-only entry: 16-byte units.
static int check_seq_gather(const dgxm_seq_gather_desc* d, int world, const void* src) {
  if (d == nullptr || src == nullptr) return fail(DGXM_ERR_INVALID, "NULL descriptor or source");
  if (d->batch < 0 || d->seq_local < 0 || d->orig_len < 0 ||
      static_cast<int64_t>(d->seq_local) * world < d->orig_len)
    return fail(DGXM_ERR_INVALID, "orig_len %d exceeds %d ranks x %d local rows", d->orig_len, world,
                d->seq_local);
  if (d->row_bytes <= 0 || d->row_bytes % 16 || d->src_batch_stride % 16 || d->src_row_stride % 16 ||
      reinterpret_cast<uintptr_t>(src) % 16)
    return fail(DGXM_ERR_INVALID, "rows, strides and the source must be 16-byte aligned");
  return DGXM_OK;
}

// This rank's rows into every rank's trimmed (B, orig_len, row) buffer.
static int launch_seq_gather(const dgxm_seq_gather_desc* d, int world, int rank, const void* src,
                             char* const* dst, cudaStream_t st) {
  if (d->batch == 0 || d->seq_local == 0) return DGXM_OK;
  SeqGatherParams p;
  memset(&p, 0, sizeof(p));
  p.src = static_cast<const char*>(src);
  p.s_sb = d->src_batch_stride;
  p.s_sl = d->src_row_stride;
  for (int r = 0; r < world; ++r) p.dst[r] = dst[r];
  p.world = world;
  p.rank = rank;
  p.batch = d->batch;
  p.seq_local = d->seq_local;
  p.orig_len = d->orig_len;
  p.row_bytes = d->row_bytes;
  const int64_t items = static_cast<int64_t>(d->batch) * d->seq_local * (d->row_bytes / 16);
  seq_allgather_kernel<<<grid_for(items, 256), 256, 0, st>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int dgxm_seq_gather_store(const dgxm_seq_gather_desc* d, int32_t world, int32_t rank,
                                     const void* src, void* const* dst, void* stream) {
  using namespace dgxm;
  if (world < 1 || world > DGXM_MAX_WORLD || rank < 0 || rank >= world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", rank, world);
  if (int rc = check_seq_gather(d, world, src)) return rc;
  if (dst == nullptr) return fail(DGXM_ERR_INVALID, "destination array is NULL");
  char* bases[DGXM_MAX_WORLD];
  for (int r = 0; r < world; ++r) {
    if (dst[r] == nullptr || reinterpret_cast<uintptr_t>(dst[r]) % 16)
      return fail(DGXM_ERR_INVALID, "destination %d is NULL or not 16-byte aligned", r);
    bases[r] = static_cast<char*>(dst[r]);
  }
  return launch_seq_gather(d, world, rank, src, bases, static_cast<cudaStream_t>(stream));
}

extern "C" int dgxm_seq_allgather(dgxm_comm* c, const dgxm_seq_gather_desc* d, const void* src,
                                  int64_t window_offset, void* stream) {
  using namespace dgxm;
  if (c == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm");
  if (int rc = check_seq_gather(d, c->world, src)) return rc;
  if (window_offset < 0 || window_offset % 16)
    return fail(DGXM_ERR_INVALID, "window offset %lld is negative or not 16-byte aligned",
                (long long)window_offset);
  const int64_t need = static_cast<int64_t>(d->batch) * d->orig_len * d->row_bytes;
  if (window_offset + need > c->bytes)
    return fail(DGXM_ERR_INVALID, "gather of %lld bytes at offset %lld overflows the %lld-byte window",
                (long long)need, (long long)window_offset, (long long)c->bytes);
  char* bases[DGXM_MAX_WORLD];
  for (int r = 0; r < c->world; ++r) {
    if (c->peers[r] == nullptr) return fail(DGXM_ERR_STATE, "peer %d window is not mapped", r);
    bases[r] = c->peers[r] + kFlagBytes + window_offset;
  }
  if (int rc = launch_seq_gather(d, c->world, c->rank, src, bases, static_cast<cudaStream_t>(stream)))
    return rc;
  return dgxm_comm_barrier(c, stream);
}

extern "C" int dgxm_shared_amax_scale(dgxm_comm* c, const void* x, int64_t rows, int64_t cols,
                                      int64_t row_stride, int32_t dtype, float divisor,
                                      void* scale_out, float* amax_out, void* stream) {
  using namespace dgxm;
  if (c == nullptr || scale_out == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or scale output");
  if (rows < 0 || cols < 0 || (rows * cols > 0 && x == nullptr))
    return fail(DGXM_ERR_INVALID, "negative extent or NULL input");
  if (!(divisor > 0.f)) return fail(DGXM_ERR_INVALID, "divisor must be positive");
  const int eb = elt_bytes(dtype);
  if (eb == 0 || dtype == DGXM_DTYPE_E4M3)
    return fail(DGXM_ERR_UNSUPPORTED, "activation dtype %d is not supported (bf16, f16, f32)", dtype);
  if (rows > 1 && row_stride < cols) return fail(DGXM_ERR_INVALID, "row stride shorter than a row");
  if (c->world > DGXM_MAX_WORLD) return fail(DGXM_ERR_INVALID, "world %d too large", c->world);
  for (int r = 0; r < c->world; ++r)
    if (c->peers[r] == nullptr) return fail(DGXM_ERR_STATE, "peer %d window is not mapped", r);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int* local = reinterpret_cast<unsigned int*>(c->local + kAmaxLocal);
  DGXM_CUDA_TRY(cudaMemsetAsync(local, 0, sizeof(unsigned int), st));
  if (rows * cols > 0) {
    AmaxParams p;
    p.x = static_cast<const char*>(x);
    p.rows = rows;
    p.cols = cols;
    p.row_stride = row_stride * eb;
    p.vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && (cols * eb) % 16 == 0 &&
            (rows == 1 || (row_stride * eb) % 16 == 0);
    p.local = local;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = static_cast<int>(rows < 8LL * sms ? rows : 8LL * sms);
    if (dtype == DGXM_DTYPE_BF16)
      amax_local_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
    else if (dtype == DGXM_DTYPE_F16)
      amax_local_kernel<__half><<<grid, 256, 0, st>>>(p);
    else
      amax_local_kernel<float><<<grid, 256, 0, st>>>(p);
    DGXM_CUDA_TRY(cudaGetLastError());
  }
  AmaxExchangeParams e;
  memset(&e, 0, sizeof(e));
  for (int r = 0; r < c->world; ++r) e.peer_flag_area[r] = c->peers[r];
  e.my_flag_area = c->local;
  e.rank = c->rank;
  e.world = c->world;
  e.wait_cycles = c->wait_cycles;
  e.inv_divisor = 1.0f / divisor;
  e.dtype = dtype;
  e.scale_out = scale_out;
  e.amax_out = amax_out;
  amax_exchange_kernel<<<1, 32, 0, st>>>(e);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}
