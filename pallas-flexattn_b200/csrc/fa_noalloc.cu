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
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "fa_internal.h"
#include "flexattn.h"

namespace fa {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FA_NOALLOC_SCRATCH_BYTES];

// The device address of a __device__ symbol belongs to one CUDA context: the primary
// context of a device, or a context the host made itself (cuCtxCreate, common in cgo/JNI
// hosts), each load the module and place the array separately, and a context destroyed
// and re-created (cudaDeviceReset) may place it elsewhere.  The cache is therefore keyed
// by the context's process-unique ID (cuCtxGetId), never by the device number.
struct ScratchEntry {
  unsigned long long ctx_id;
  void* addr;
};
constexpr int kMaxContexts = 64;
ScratchEntry g_entries[kMaxContexts];
int g_n_entries = 0;
std::mutex g_mutex;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

int fail_cuda(const char* what, cudaError_t e) {
  char msg[192];
  snprintf(msg, sizeof(msg), "fa_bwd_noalloc: %s: %s", what, cudaGetErrorString(e));
  return set_last_error(FA_ERR_CUDA, msg);
}

// Address of the scratch in the calling thread's current context, resolved with
// cudaGetSymbolAddress (return code checked) the first time each context is seen.
int scratch_in_current_context(void** out) {
  static CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  void* p = nullptr;
  if (!get_current || !get_id) {  // no context identity available: resolve on every call
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return fail_cuda("cudaGetSymbolAddress of the static scratch", e);
    *out = p;
    return FA_OK;
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) {
    // No context is current yet: the runtime binds the device's primary context on its
    // first call, which is this lookup.
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return fail_cuda("cudaGetSymbolAddress of the static scratch", e);
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) {
      *out = p;
      return FA_OK;
    }
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return set_last_error(FA_ERR_CUDA, "fa_bwd_noalloc: cuCtxGetId failed");
  std::lock_guard<std::mutex> lock(g_mutex);
  for (int i = 0; i < g_n_entries; ++i)
    if (g_entries[i].ctx_id == id) {
      *out = g_entries[i].addr;
      return FA_OK;
    }
  if (!p) {
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return fail_cuda("cudaGetSymbolAddress of the static scratch", e);
  }
  if (g_n_entries < kMaxContexts) g_entries[g_n_entries++] = ScratchEntry{id, p};  // else: resolve again next time
  *out = p;
  return FA_OK;
}

}  // namespace
}  // namespace fa

extern "C" {

int fa_bwd_noalloc(const FaBwdParams* p, fa_stream_t stream) {
  // The same validation as fa_bwd first, so a malformed call gets fa_bwd's error; only a
  // well-formed shape is then measured against the scratch.
  int rc = fa::check_bwd_params(p);
  if (rc) return rc;
  size_t need = 0;
  if ((rc = fa_bwd_workspace_size(p, &need))) return rc;
  if (need > FA_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "fa_bwd_noalloc: B=%d H=%d Tq=%d D=%d needs %zu bytes of workspace, more than the %zu-byte "
             "static scratch; use fa_bwd with a caller workspace",
             p->B, p->H, p->Tq, p->D, need, (size_t)FA_NOALLOC_SCRATCH_BYTES);
    return fa::set_last_error(FA_ERR_UNSUPPORTED, msg);
  }
  void* scratch = nullptr;
  if ((rc = fa::scratch_in_current_context(&scratch))) return rc;
  return fa_bwd(p, scratch, FA_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
