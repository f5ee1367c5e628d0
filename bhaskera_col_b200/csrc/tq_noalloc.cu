// tq_noalloc.cu — decode attention for callers that cannot allocate device
// memory.
//
// Some hosts call into this library from places where no allocator may be
// used: a serving runtime that owns every byte of device memory through its
// own pool and forbids cudaMalloc after start-up, or an engine that issues
// work from a context where allocation would block or fail.  Such callers
// cannot provide the workspace tq_decode_attn needs.  tq_decode_attn_noalloc
// runs the same kernels with their scratch in a fixed array compiled into
// this library instead.
//
// The array is a file-scope __device__ variable of kNoAllocScratchBytes
// (8 MiB).  Every GPU on which the library is loaded holds it until the
// process exits.  Host code cannot use the array's name as a device address,
// so the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture.  The cached address belongs to the
// device's current context: after cudaDeviceReset (or anything else that
// destroys the primary context) the library reloads at a new address and
// the cache is stale, so do not call these entry points again in such a
// process.  All calls on a device share the one array and it keeps the last
// call's contents: each call clears the status word the kernels report
// device-side errors through, and every other byte a call reads is written
// earlier in the same call (which is why a call must run all three phases:
// a phase-split sequence would read what an intervening call left there).
// Calls whose work overlaps on the GPU (different streams, or host threads
// racing on one device) race on the array; serialise them.
// tq_noalloc_status reads and clears the array's status word.
#include <mutex>

#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of this device's scratch array (looked up once per device).
static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("tq_decode_attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("tq_decode_attn_noalloc: device %d is beyond the %d supported", dev, kMaxDevices);
    return TQ_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("tq_decode_attn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return TQ_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return TQ_OK;
}

}  // namespace tq

using namespace tq;

extern "C" int32_t tq_decode_attn_noalloc(const tq_geom* g, const tq_tables* t,
                                          const tq_cache* c, const tq_decode_args* a,
                                          void* stream) {
  constexpr int kAll = TQ_PHASE_QPREP | TQ_PHASE_DECODE | TQ_PHASE_MERGE;
  if (a && a->phases != 0 && a->phases != kAll) {
    set_error("tq_decode_attn_noalloc: phases must be 0 (all): a later phase would read "
              "scratch that any other call on this device may have overwritten");
    return TQ_ERR_INVALID;
  }
  const size_t need = tq_decode_workspace_bytes(g, c, a);
  if (need == 0) {
    // argument errors are reported by the full check in tq_decode_attn below
    return tq_decode_attn(g, t, c, a, nullptr, 0, stream);
  }
  if (need > kNoAllocScratchBytes) {
    set_error("tq_decode_attn_noalloc: this call needs %zu bytes of scratch; the built-in "
              "array holds %zu (8 MiB). Use tq_decode_attn with a caller-provided workspace",
              need, kNoAllocScratchBytes);
    return TQ_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != TQ_OK) return rc;
  cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(uint32_t), (cudaStream_t)stream);
  if (e != cudaSuccess) {
    set_error("tq_decode_attn_noalloc: clearing the status word: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return tq_decode_attn(g, t, c, a, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int32_t tq_noalloc_status(uint32_t* status, void* stream) {
  if (!status) {
    set_error("tq_noalloc_status: NULL argument");
    return TQ_ERR_INVALID;
  }
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != TQ_OK) return rc;
  // the status word sits at the start of the array, as in a workspace
  return tq_workspace_status(scratch, status, stream);
}
