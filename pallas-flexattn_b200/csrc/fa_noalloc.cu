// fa_bwd_noalloc: the backward pass with its workspace in a static device array.
//
// Some callers cannot allocate device memory: a foreign-language host (cgo, JNI,
// ctypes) that is handed raw device pointers by a runtime owning the memory pool has no
// allocator handle, and a cudaMalloc of its own would bypass that pool's accounting and
// can fail once the pool has reserved most of the HBM.  This entry point serves them by
// running fa_bwd's unchanged kernel sequence on a workspace that lives in the library.
//
// The scratch is a file-scope __device__ array in this translation unit's CUDA module, so
// the driver reserves it when that module loads: on the first fa_bwd_noalloc call under
// lazy module loading (the CUDA 12 default), at context creation under eager loading.
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
//
// Per call, fa_bwd's preprocess step zeroes the fp32 dQ accumulator (a memset on the
// caller's stream; the only part that must start at zero) and writes delta and lse2
// before the fused kernel reads them, so no state carries from one call to the next.
// Calls that overlap on one device (several streams or host threads) share the array
// and race.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <mutex>

#include "fa_internal.h"
#include "flexattn.h"

namespace fa {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_addr[kMaxDevices];
std::mutex g_setup_mutex;

// Address of the scratch on the current device, resolved once per device.
int scratch_on_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  char msg[192];
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "fa_bwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return set_last_error(FA_ERR_CUDA, msg);
  }
  if (dev < 0 || dev >= kMaxDevices) {
    snprintf(msg, sizeof(msg), "fa_bwd_noalloc: device ordinal %d outside 0..%d", dev, kMaxDevices - 1);
    return set_last_error(FA_ERR_UNSUPPORTED, msg);
  }
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_addr[dev].load(std::memory_order_relaxed);
    if (!p) {
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        snprintf(msg, sizeof(msg), "fa_bwd_noalloc: cudaGetSymbolAddress of the static scratch on device %d: %s",
                 dev, cudaGetErrorString(e));
        return set_last_error(FA_ERR_CUDA, msg);
      }
      g_scratch_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return FA_OK;
}

}  // namespace
}  // namespace fa

extern "C" {

int fa_bwd_noalloc(const FaBwdParams* p, fa_stream_t stream) {
  if (!p) return fa::set_last_error(FA_ERR_INVALID, "fa_bwd_noalloc: NULL argument");
  // Shapes are validated by fa_bwd; only a well-formed shape is measured against the limit.
  if (p->B > 0 && p->H > 0 && p->Tq > 0 && p->D > 0) {
    size_t need = 0;
    int rc = fa_bwd_workspace_size(p, &need);
    if (rc) return rc;
    if (need > FA_NOALLOC_SCRATCH_BYTES) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "fa_bwd_noalloc: B=%d H=%d Tq=%d D=%d needs %zu bytes of workspace, more than the %zu-byte "
               "static scratch; use fa_bwd with a caller workspace",
               p->B, p->H, p->Tq, p->D, need, (size_t)FA_NOALLOC_SCRATCH_BYTES);
      return fa::set_last_error(FA_ERR_UNSUPPORTED, msg);
    }
  }
  void* scratch = nullptr;
  int rc = fa::scratch_on_current_device(&scratch);
  if (rc) return rc;
  return fa_bwd(p, scratch, FA_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
