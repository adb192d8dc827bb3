// Single translation unit of libdgxm_sp.so.  The kernels share one device
// error word (device_error.cuh), so the library is built as one unit rather
// than with relocatable device code.
#include <math.h>
#include <string.h>

#include <mutex>

#include "capi.cu"
#include "attn_fwd.cu"
#include "lse_merge.cu"
#include "comm.cu"
#include "ring.cu"
#include "full_context.cu"
#include "shard.cu"
#include "cfg.cu"
#include "qkv_gemm.cu"
#include "prologue.cu"
