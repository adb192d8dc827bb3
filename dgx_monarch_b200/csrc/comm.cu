// Peer windows over NVLink, the Ulysses all-to-all as direct peer stores, and
// a bounded device-side barrier.
//
// Each rank cudaMallocs one window in its own HBM and exports a CUDA IPC
// handle; every other rank maps it (a plain peer mapping, nothing switch-side),
// so a kernel on rank s can store straight into rank r's window over NVLink.
// The first 4 KB of a window hold barrier flags: slot i is written by rank i.
//
// Replaces yunchang's SeqAllToAll4D (reached from adapters/usp_full_axis.py:
// 27-29,40 and inside xfuser's USP call at adapters/base.py:320), which the
// reference runs as an NCCL all_to_all plus permute copies.
#include "common.h"
#include "device_error.cuh"
#include "ptx.cuh"

struct dgxm_comm {
  int rank;
  int world;
  int device;
  uint64_t generation;
  int64_t bytes;       // usable bytes after the flag area
  char* local;         // this rank's window base (cudaMalloc)
  char* peers[DGXM_MAX_WORLD];  // window bases as seen by this process
  bool opened[DGXM_MAX_WORLD];
  uint32_t fc_calls;   // full-context calls so far (their window buffer alternates)
  long long wait_cycles;  // barrier wait budget in SM clock cycles
  cudaStream_t side;      // ring: copy-engine stream (created on first use)
  cudaEvent_t ev_main, ev_side;
};

namespace dgxm {

constexpr int64_t kFlagBytes = 4096;
// This rank's barrier count, in its own flag area: every barrier-type kernel
// reads it, uses count + 1 as its epoch and stores that back, so the epochs
// live on the device and a captured CUDA graph advances them on each replay.
constexpr int64_t kEpochCounter = 3584;

__device__ __forceinline__ int next_epoch(const char* my_flag_area) {
  return *reinterpret_cast<const volatile int*>(my_flag_area + kEpochCounter) + 1;
}

// ------------------------------------------------------------------ barrier
struct BarrierParams {
  int* peer_flags[DGXM_MAX_WORLD];  // flag area of each rank's window
  int* my_flags;
  int rank, world;
  long long wait_cycles;
};

// One warp; lane i < world does this rank's half of the handshake with rank
// i: release the epoch into rank i's slot for this rank, acquire rank i's
// epoch from this rank's slot for it.
__global__ void comm_barrier_kernel(const __grid_constant__ BarrierParams p) {
  const int i = threadIdx.x;
  const int epoch = next_epoch(reinterpret_cast<const char*>(p.my_flags));
  if (i < p.world) {
    // Everything this rank wrote before this kernel (earlier kernels in the
    // stream) is performed before the flag below becomes visible.
    __threadfence_system();
    int* slot = p.peer_flags[i] + p.rank;
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(slot), "r"(epoch) : "memory");
    const int* mine = p.my_flags + i;
    const long long start = clock64();
    while (true) {
      int seen;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(seen) : "l"(mine) : "memory");
      if (seen - epoch >= 0) break;  // wrap-safe monotonic compare
      if (clock64() - start > p.wait_cycles) {
        report_device_error(kErrPeerTimeout);
        break;
      }
      __nanosleep(64);
    }
    __threadfence_system();
  }
  __syncwarp();  // every lane has read the count before it advances
  if (i == 0) *reinterpret_cast<volatile int*>(reinterpret_cast<char*>(p.my_flags) + kEpochCounter) = epoch;
}

// ------------------------------------------------------------------ all-to-all
struct ScatterParams {
  const char* src[3];                      // (B, Ls, H, D) per tensor
  char* dst[3][DGXM_MAX_WORLD];            // (B, world*Ls, H/world, D) on each rank
  int64_t s_sb[3], s_sl[3], s_sh[3];       // source strides, bytes
  int n_tensors, world, rank;
  int batch, seq_local, heads, head_bytes; // head_bytes = D * elt
  int seg0;                                // joint order: leading rows per rank (0 = rank-major)
  int64_t seq_full;                        // rows of each receive tensor
  int row_off;                             // first image row in it (after replicated text)
};

// Position on the gathered axis of local row l of rank r.  With seg0 == 0
// this is the rank-major concat [r*Ls + l]; with a two-segment local layout
// [seg0 rows | Ls - seg0 rows] it is the canonical order that lists every
// rank's first segment before every rank's second
// (adapters/usp_sequence_order.py:69-78).
__device__ __forceinline__ int64_t gathered_row(int r, int l, int seq_local, int world, int seg0) {
  if (seg0 == 0) return static_cast<int64_t>(r) * seq_local + l;
  if (l < seg0) return static_cast<int64_t>(r) * seg0 + l;
  const int seg1 = seq_local - seg0;
  return static_cast<int64_t>(world) * seg0 + static_cast<int64_t>(r) * seg1 + (l - seg0);
}

// Sequence -> head: this rank's rows, head slice of rank r -> rank r's
// gathered axis at rows [rank*Ls, (rank+1)*Ls).  One thread moves 16 bytes;
// a warp moves two consecutive 256-byte head rows, so loads and peer stores
// are both coalesced.
__global__ void __launch_bounds__(256) ulysses_scatter_kernel(const __grid_constant__ ScatterParams p) {
  const int chunks_per_head = p.head_bytes / 16;
  const int hl = p.heads / p.world;
  const int64_t per_tensor = static_cast<int64_t>(p.batch) * p.seq_local * p.heads * chunks_per_head;
  const int64_t total = per_tensor * p.n_tensors;
  const int64_t seq_full = p.seq_full;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / per_tensor);
    int64_t rem = i - t * per_tensor;
    const int part = static_cast<int>(rem % chunks_per_head);
    rem /= chunks_per_head;
    const int h = static_cast<int>(rem % p.heads);
    rem /= p.heads;
    const int l = static_cast<int>(rem % p.seq_local);
    const int b = static_cast<int>(rem / p.seq_local);
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(
        p.src[t] + b * p.s_sb[t] + l * p.s_sl[t] + h * p.s_sh[t]) + part);
    const int r = h / hl;
    const int hh = h - r * hl;
    const int64_t row = static_cast<int64_t>(b) * seq_full + p.row_off +
                        gathered_row(p.rank, l, p.seq_local, p.world, p.seg0);
    char* dst = p.dst[t][r] + (row * hl + hh) * p.head_bytes;
    reinterpret_cast<uint4*>(dst)[part] = val;
  }
}

// Replicated text: this rank's head slice [head0, head0 + hl) of its own
// whole (B, T, H, D) text goes into its own receive tensors at rows
// [row_off, row_off + T).  Local HBM to HBM, 16 bytes per thread.
struct TextSliceParams {
  const char* src[3];
  char* dst[3];
  int64_t s_sb[3], s_sl[3], s_sh[3];  // bytes
  int64_t d_sb;                       // bytes between batch items of a receive tensor
  int n_tensors, batch, rows, hl, head0, head_bytes, row_off;
};

__global__ void __launch_bounds__(256) text_head_slice_kernel(const __grid_constant__ TextSliceParams p) {
  const int chunks = p.head_bytes / 16;
  const int64_t per_tensor = static_cast<int64_t>(p.batch) * p.rows * p.hl * chunks;
  const int64_t total = per_tensor * p.n_tensors;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / per_tensor);
    int64_t rem = i - t * per_tensor;
    const int part = static_cast<int>(rem % chunks);
    rem /= chunks;
    const int hh = static_cast<int>(rem % p.hl);
    rem /= p.hl;
    const int l = static_cast<int>(rem % p.rows);
    const int b = static_cast<int>(rem / p.rows);
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(
        p.src[t] + b * p.s_sb[t] + l * p.s_sl[t] + (p.head0 + hh) * p.s_sh[t]) + part);
    char* dst = p.dst[t] + b * p.d_sb + ((static_cast<int64_t>(p.row_off) + l) * p.hl + hh) * p.head_bytes;
    reinterpret_cast<uint4*>(dst)[part] = val;
  }
}

// Head -> sequence (the inverse): this rank's (B, S, Hl, D) rows go back to
// the rank owning each sequence chunk, into head slice [rank*Hl, (rank+1)*Hl)
// of its (B, Ls, H, D) tensor.
struct GatherParams {
  const char* src;                     // (B, S, Hl, D), strides below
  char* dst[DGXM_MAX_WORLD];           // (B, Ls, H, D) contiguous on each rank
  int64_t s_sb, s_sl, s_sh;
  int world, rank;
  int batch, seq_local, heads, head_bytes;
  int seg0;
};

// Inverse of gathered_row: (owner rank, local row) of gathered row g.
__device__ __forceinline__ void owner_of_row(int64_t g, int seq_local, int world, int seg0, int* r,
                                             int* l) {
  if (seg0 == 0) {
    *r = static_cast<int>(g / seq_local);
    *l = static_cast<int>(g - static_cast<int64_t>(*r) * seq_local);
    return;
  }
  const int64_t head = static_cast<int64_t>(world) * seg0;
  if (g < head) {
    *r = static_cast<int>(g / seg0);
    *l = static_cast<int>(g - static_cast<int64_t>(*r) * seg0);
  } else {
    const int seg1 = seq_local - seg0;
    const int64_t t = g - head;
    *r = static_cast<int>(t / seg1);
    *l = seg0 + static_cast<int>(t - static_cast<int64_t>(*r) * seg1);
  }
}

__global__ void __launch_bounds__(256) ulysses_gather_kernel(const __grid_constant__ GatherParams p) {
  const int chunks_per_head = p.head_bytes / 16;
  const int hl = p.heads / p.world;
  const int64_t seq_full = static_cast<int64_t>(p.seq_local) * p.world;
  const int64_t total = static_cast<int64_t>(p.batch) * seq_full * hl * chunks_per_head;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t rem = i;
    const int part = static_cast<int>(rem % chunks_per_head);
    rem /= chunks_per_head;
    const int hh = static_cast<int>(rem % hl);
    rem /= hl;
    const int64_t l = rem % seq_full;
    const int b = static_cast<int>(rem / seq_full);
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(p.src + b * p.s_sb + l * p.s_sl + hh * p.s_sh) + part);
    int r, lr;
    owner_of_row(l, p.seq_local, p.world, p.seg0, &r, &lr);
    const int64_t row = static_cast<int64_t>(b) * p.seq_local + lr;
    char* dst = p.dst[r] + (row * p.heads + static_cast<int64_t>(p.rank) * hl + hh) * p.head_bytes;
    reinterpret_cast<uint4*>(dst)[part] = val;
  }
}

static int grid_for(int64_t work_items, int threads) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (work_items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

static int elt_bytes(int dtype) {
  switch (dtype) {
    case DGXM_DTYPE_BF16:
    case DGXM_DTYPE_F16: return 2;
    case DGXM_DTYPE_E4M3: return 1;
    case DGXM_DTYPE_F32: return 4;
    default: return 0;
  }
}

}  // namespace dgxm

// ------------------------------------------------------------------ C ABI
extern "C" int dgxm_comm_create(int32_t rank, int32_t world, int64_t bytes, uint64_t generation,
                                dgxm_comm** out) {
  using namespace dgxm;
  if (out == nullptr) return fail(DGXM_ERR_INVALID, "out handle pointer is NULL");
  *out = nullptr;
  if (world < 1 || world > DGXM_MAX_WORLD || rank < 0 || rank >= world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range (world <= %d)", rank, world,
                DGXM_MAX_WORLD);
  if (bytes < 0) return fail(DGXM_ERR_INVALID, "window size %lld is negative", (long long)bytes);
  dgxm_comm* c = new dgxm_comm();
  memset(c, 0, sizeof(*c));
  c->rank = rank;
  c->world = world;
  c->generation = generation;
  c->bytes = (bytes + 255) / 256 * 256;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->local), kFlagBytes + c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, kFlagBytes);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return cuda_fail(e, "dgxm_comm_create window allocation");
  }
  c->peers[rank] = c->local;
  c->opened[rank] = false;
  c->wait_cycles = kWaitBudgetCycles;
  if (world > 1) {
    // The copy-engine stream and events of ring attention, created with the
    // comm so that no attention call creates driver objects.
    e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_main, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_side, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      if (c->ev_main) cudaEventDestroy(c->ev_main);
      if (c->side) cudaStreamDestroy(c->side);
      cudaFree(c->local);
      delete c;
      return cuda_fail(e, "dgxm_comm_create stream/events");
    }
  }
  *out = c;
  return DGXM_OK;
}

extern "C" int dgxm_comm_set_timeout(dgxm_comm* c, int32_t timeout_ms) {
  using namespace dgxm;
  if (c == nullptr || timeout_ms <= 0) return fail(DGXM_ERR_INVALID, "NULL comm or non-positive timeout");
  int khz = 0;
  DGXM_CUDA_TRY(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, c->device));
  // Budget at the highest clock, so the wall-clock limit is never shorter
  // than asked.
  c->wait_cycles = static_cast<long long>(timeout_ms) * (khz > 0 ? khz : 2000000);
  return DGXM_OK;
}

extern "C" int dgxm_comm_export(dgxm_comm* c, void* handle) {
  using namespace dgxm;
  if (c == nullptr || handle == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or handle buffer");
  cudaIpcMemHandle_t h;
  DGXM_CUDA_TRY(cudaIpcGetMemHandle(&h, c->local));
  memcpy(handle, &h, sizeof(h));
  return DGXM_OK;
}

extern "C" int dgxm_comm_import(dgxm_comm* c, const void* handles) {
  using namespace dgxm;
  if (c == nullptr || handles == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or handles");
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->opened[r]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + r * DGXM_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    c->peers[r] = static_cast<char*>(p);
    c->opened[r] = true;
  }
  return DGXM_OK;
}

extern "C" int dgxm_comm_window(dgxm_comm* c, int32_t peer, void** ptr) {
  using namespace dgxm;
  if (c == nullptr || ptr == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or output pointer");
  if (peer < 0 || peer >= c->world) return fail(DGXM_ERR_INVALID, "peer %d out of range", peer);
  if (c->peers[peer] == nullptr)
    return fail(DGXM_ERR_STATE, "peer %d window is not mapped (call dgxm_comm_import)", peer);
  *ptr = c->peers[peer] + kFlagBytes;
  return DGXM_OK;
}

extern "C" int64_t dgxm_comm_bytes(dgxm_comm* c) { return c == nullptr ? -1 : c->bytes; }

extern "C" uint64_t dgxm_comm_generation(dgxm_comm* c) { return c == nullptr ? 0 : c->generation; }

extern "C" int dgxm_comm_barrier(dgxm_comm* c, void* stream) {
  using namespace dgxm;
  if (c == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm");
  if (c->world == 1) return DGXM_OK;
  BarrierParams p;
  memset(&p, 0, sizeof(p));
  for (int r = 0; r < c->world; ++r) {
    if (c->peers[r] == nullptr)
      return fail(DGXM_ERR_STATE, "peer %d window is not mapped (call dgxm_comm_import)", r);
    p.peer_flags[r] = reinterpret_cast<int*>(c->peers[r]);
  }
  p.my_flags = reinterpret_cast<int*>(c->local);
  p.rank = c->rank;
  p.world = c->world;
  p.wait_cycles = c->wait_cycles;
  comm_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

extern "C" int dgxm_comm_destroy(dgxm_comm* c) {
  using namespace dgxm;
  if (c == nullptr) return DGXM_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  if (c->side != nullptr) {
    if (c->ev_main) cudaEventDestroy(c->ev_main);
    if (c->ev_side) cudaEventDestroy(c->ev_side);
    cudaStreamDestroy(c->side);
  }
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) cudaIpcCloseMemHandle(c->peers[r]);
  cudaError_t e = cudaFree(c->local);
  if (prev >= 0) cudaSetDevice(prev);
  delete c;
  if (e != cudaSuccess) return cuda_fail(e, "dgxm_comm_destroy cudaFree");
  return DGXM_OK;
}

extern "C" int dgxm_comm_allgather(dgxm_comm* c, const void* src, int64_t bytes,
                                   int64_t window_offset, void* stream) {
  using namespace dgxm;
  if (c == nullptr || src == nullptr) return fail(DGXM_ERR_INVALID, "NULL comm or source");
  if (bytes < 0 || window_offset < 0 || window_offset % 16)
    return fail(DGXM_ERR_INVALID, "negative size or misaligned window offset");
  if (window_offset + bytes * c->world > c->bytes)
    return fail(DGXM_ERR_INVALID, "all-gather of %d x %lld bytes at offset %lld overflows the "
                "%lld-byte window", c->world, (long long)bytes, (long long)window_offset,
                (long long)c->bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < c->world; ++i) {
    // Start with the next peer so the copies of all ranks spread over links.
    const int r = (c->rank + i) % c->world;
    if (c->peers[r] == nullptr) return fail(DGXM_ERR_STATE, "peer %d window is not mapped", r);
    char* dst = c->peers[r] + kFlagBytes + window_offset + static_cast<int64_t>(c->rank) * bytes;
    if (bytes > 0) DGXM_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, st));
  }
  return dgxm_comm_barrier(c, stream);
}

namespace dgxm {

// Checks an all-to-all descriptor and fills the scatter parameters (the
// receive tensor holds world*seq_local rows, image rows from row 0).  The
// pointers are checked only when there are rows to move, as an empty shard
// may carry NULL tensors.
static int build_scatter(const dgxm_a2a_desc* d, const void* const* src, void* const* dst,
                         ScatterParams* p) {
  if (d == nullptr || src == nullptr || dst == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL all-to-all argument");
  if (d->n_tensors < 1 || d->n_tensors > 3)
    return fail(DGXM_ERR_INVALID, "all-to-all moves 1..3 tensors, got %d", d->n_tensors);
  if (d->world < 1 || d->world > DGXM_MAX_WORLD || d->rank < 0 || d->rank >= d->world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", d->rank, d->world);
  if (d->heads <= 0 || d->heads % d->world)
    return fail(DGXM_ERR_INVALID, "%d heads are not divisible by the Ulysses degree %d", d->heads,
                d->world);
  const int eb = elt_bytes(d->dtype);
  if (eb == 0) return fail(DGXM_ERR_UNSUPPORTED, "dtype %d is not supported", d->dtype);
  const int head_bytes = d->head_dim * eb;
  if (d->head_dim <= 0 || head_bytes % 16)
    return fail(DGXM_ERR_INVALID, "head row of %d bytes is not a multiple of 16", head_bytes);
  if (d->batch < 0 || d->seq_local < 0)
    return fail(DGXM_ERR_INVALID, "negative batch or sequence length");
  memset(p, 0, sizeof(*p));
  const bool rows = d->batch > 0 && d->seq_local > 0;
  for (int t = 0; t < d->n_tensors && rows; ++t) {
    if (src[t] == nullptr || reinterpret_cast<uintptr_t>(src[t]) % 16)
      return fail(DGXM_ERR_INVALID, "source tensor %d is NULL or not 16-byte aligned", t);
    p->src[t] = static_cast<const char*>(src[t]);
    p->s_sb[t] = d->src_stride[t][0] * eb;
    p->s_sl[t] = d->src_stride[t][1] * eb;
    p->s_sh[t] = d->src_stride[t][2] * eb;
    if (p->s_sb[t] % 16 || p->s_sl[t] % 16 || p->s_sh[t] % 16)
      return fail(DGXM_ERR_INVALID, "source tensor %d strides are not 16-byte multiples", t);
    for (int r = 0; r < d->world; ++r) {
      void* q = dst[t * d->world + r];
      if (q == nullptr || reinterpret_cast<uintptr_t>(q) % 16)
        return fail(DGXM_ERR_INVALID, "destination %d of tensor %d is NULL or misaligned", r, t);
      p->dst[t][r] = static_cast<char*>(q);
    }
  }
  p->n_tensors = d->n_tensors;
  p->world = d->world;
  p->rank = d->rank;
  p->batch = d->batch;
  p->seq_local = d->seq_local;
  p->heads = d->heads;
  p->head_bytes = head_bytes;
  if (d->seq_local > 0 &&
      (d->seg0 < 0 || d->seg0 >= d->seq_local || (d->seg0 > 0 && d->seq_local - d->seg0 < 1)))
    return fail(DGXM_ERR_INVALID, "joint segment of %d rows does not split %d local rows", d->seg0,
                d->seq_local);
  p->seg0 = d->seg0;
  p->seq_full = static_cast<int64_t>(d->seq_local) * d->world;
  p->row_off = 0;
  return DGXM_OK;
}

static int launch_scatter(const dgxm_a2a_desc* d, const ScatterParams& p, void* stream) {
  if (d->batch == 0 || d->seq_local == 0) return DGXM_OK;
  const int64_t work = static_cast<int64_t>(d->n_tensors) * d->batch * d->seq_local * d->heads * (p.head_bytes / 16);
  ulysses_scatter_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

}  // namespace dgxm

extern "C" int dgxm_ulysses_scatter(const dgxm_a2a_desc* d, const void* const* src,
                                    void* const* dst, void* stream) {
  using namespace dgxm;
  ScatterParams p;
  int rc = build_scatter(d, src, dst, &p);
  if (rc) return rc;
  return launch_scatter(d, p, stream);
}

extern "C" int dgxm_ulysses_scatter_joint(const dgxm_a2a_desc* d, int32_t txt_rows, int32_t txt_front,
                                          const void* const* txt, const int64_t* txt_stride,
                                          const void* const* src, void* const* dst, void* stream) {
  using namespace dgxm;
  ScatterParams p;
  int rc = build_scatter(d, src, dst, &p);
  if (rc) return rc;
  if (d->seg0 != 0)
    return fail(DGXM_ERR_INVALID, "replicated text needs the rank-major image order (seg0 = 0)");
  if (txt_rows < 0 || (txt_front != 0 && txt_front != 1))
    return fail(DGXM_ERR_INVALID, "text rows %d / front flag %d out of range", txt_rows, txt_front);
  p.seq_full = static_cast<int64_t>(d->seq_local) * d->world + txt_rows;
  p.row_off = txt_front ? txt_rows : 0;
  if ((rc = launch_scatter(d, p, stream))) return rc;
  if (txt_rows == 0 || d->batch == 0) return DGXM_OK;
  if (txt == nullptr || txt_stride == nullptr) return fail(DGXM_ERR_INVALID, "NULL text argument");
  const int eb = p.head_bytes / d->head_dim;
  TextSliceParams tp;
  memset(&tp, 0, sizeof(tp));
  for (int t = 0; t < d->n_tensors; ++t) {
    if (txt[t] == nullptr || reinterpret_cast<uintptr_t>(txt[t]) % 16)
      return fail(DGXM_ERR_INVALID, "text tensor %d is NULL or not 16-byte aligned", t);
    void* own = dst[t * d->world + d->rank];
    if (own == nullptr || reinterpret_cast<uintptr_t>(own) % 16)
      return fail(DGXM_ERR_INVALID, "receive tensor %d of this rank is NULL or misaligned", t);
    tp.src[t] = static_cast<const char*>(txt[t]);
    tp.s_sb[t] = txt_stride[3 * t] * eb;
    tp.s_sl[t] = txt_stride[3 * t + 1] * eb;
    tp.s_sh[t] = txt_stride[3 * t + 2] * eb;
    if (tp.s_sb[t] % 16 || tp.s_sl[t] % 16 || tp.s_sh[t] % 16)
      return fail(DGXM_ERR_INVALID, "text tensor %d strides are not 16-byte multiples", t);
    tp.dst[t] = static_cast<char*>(own);
  }
  tp.n_tensors = d->n_tensors;
  tp.batch = d->batch;
  tp.rows = txt_rows;
  tp.hl = d->heads / d->world;
  tp.head0 = d->rank * tp.hl;
  tp.head_bytes = p.head_bytes;
  tp.d_sb = p.seq_full * tp.hl * p.head_bytes;
  tp.row_off = txt_front ? 0 : d->seq_local * d->world;
  const int64_t work = static_cast<int64_t>(d->n_tensors) * d->batch * txt_rows * tp.hl * (p.head_bytes / 16);
  text_head_slice_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(tp);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}

extern "C" int dgxm_ulysses_gather(const dgxm_a2a_desc* d, const void* src, void* const* dst,
                                   void* stream) {
  using namespace dgxm;
  if (d == nullptr || src == nullptr || dst == nullptr)
    return fail(DGXM_ERR_INVALID, "NULL all-to-all argument");
  if (d->world < 1 || d->world > DGXM_MAX_WORLD || d->rank < 0 || d->rank >= d->world)
    return fail(DGXM_ERR_INVALID, "rank %d / world %d out of range", d->rank, d->world);
  if (d->heads <= 0 || d->heads % d->world)
    return fail(DGXM_ERR_INVALID, "%d heads are not divisible by the Ulysses degree %d", d->heads,
                d->world);
  const int eb = elt_bytes(d->dtype);
  if (eb == 0) return fail(DGXM_ERR_UNSUPPORTED, "dtype %d is not supported", d->dtype);
  const int head_bytes = d->head_dim * eb;
  if (d->head_dim <= 0 || head_bytes % 16)
    return fail(DGXM_ERR_INVALID, "head row of %d bytes is not a multiple of 16", head_bytes);
  if (d->batch == 0 || d->seq_local == 0) return DGXM_OK;
  GatherParams p;
  memset(&p, 0, sizeof(p));
  if (reinterpret_cast<uintptr_t>(src) % 16) return fail(DGXM_ERR_INVALID, "source misaligned");
  p.src = static_cast<const char*>(src);
  p.s_sb = d->src_stride[0][0] * eb;
  p.s_sl = d->src_stride[0][1] * eb;
  p.s_sh = d->src_stride[0][2] * eb;
  if (p.s_sb % 16 || p.s_sl % 16 || p.s_sh % 16)
    return fail(DGXM_ERR_INVALID, "source strides are not 16-byte multiples");
  for (int r = 0; r < d->world; ++r) {
    if (dst[r] == nullptr || reinterpret_cast<uintptr_t>(dst[r]) % 16)
      return fail(DGXM_ERR_INVALID, "destination %d is NULL or misaligned", r);
    p.dst[r] = static_cast<char*>(dst[r]);
  }
  p.world = d->world;
  p.rank = d->rank;
  p.batch = d->batch;
  p.seq_local = d->seq_local;
  p.heads = d->heads;
  p.head_bytes = head_bytes;
  if (d->seg0 < 0 || d->seg0 >= d->seq_local)
    return fail(DGXM_ERR_INVALID, "joint segment of %d rows does not split %d local rows", d->seg0,
                d->seq_local);
  p.seg0 = d->seg0;
  const int64_t work = static_cast<int64_t>(d->batch) * d->seq_local * d->heads * (head_bytes / 16);
  ulysses_gather_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  DGXM_CUDA_TRY(cudaGetLastError());
  return DGXM_OK;
}
