// noalloc.cu -- ltxattn_fwd_noalloc: the forward for callers that cannot
// allocate device memory.
//
// ltxattn_fwd needs caller-provided scratch for two things: the rotated copies
// of q and k (when rotary tables are given) and, for short query sequences,
// the per-split partial outputs that the combine kernel merges.  Some callers
// cannot call cudaMalloc to provide it: a host whose device memory is owned
// entirely by another framework's allocator (the reference's tensors live in
// MLX's allocator, which hands out no raw scratch), or a render or serving
// loop that must not allocate between steps.  This entry point takes its
// scratch from a fixed array compiled into the library instead.
//
//  - The array is kNoAllocScratchBytes (32 MiB) of device memory.  Every GPU
//    that loads the library holds it until the process exits.
//  - Arguments whose scratch would exceed it are refused with
//    LTXATTN_ERR_WORKSPACE; the message gives the size needed.
//  - The array's device address is looked up once per device, on the first
//    call made with that device current (cudaGetSymbolAddress).  Make that
//    first call before any stream capture.
//  - Every call shares the one array, and it keeps whatever the last call
//    wrote.  Nothing in it needs to start at zero: every byte a call reads was
//    written earlier by the same call.  Calls whose executions overlap on the
//    GPU (different streams, or different host threads without ordering)
//    race on the array and corrupt each other's results; serialise them.
//  - No cudaMalloc, cudaFree or allocating library routine is called.
//  - The looked-up address belongs to the device's context at that first
//    call: after cudaDeviceReset (or any other teardown of the primary
//    context) in the same process it is stale, so the library must not be
//    used on that device again in that process.
#include <cstdio>
#include <mutex>

#include "../../include/ltxattn.h"
#include "ltxattn_internal.h"

namespace ltx {

int set_error_message(int status, const char* msg);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // not left behind for a later launch check to find
    return set_error_message(LTXATTN_ERR_CUDA, cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= kMaxDevices) return set_error_message(LTXATTN_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      char buf[256];
      snprintf(buf, sizeof buf, "cudaGetSymbolAddress of the no-alloc scratch failed: %s", cudaGetErrorString(e));
      return set_error_message(LTXATTN_ERR_CUDA, buf);
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LTXATTN_OK;
}

}  // namespace
}  // namespace ltx

extern "C" {

int ltxattn_fwd_noalloc(const ltxattn_fwd_args* args, void* stream) {
  if (args == nullptr) return ltx::set_error_message(LTXATTN_ERR_ARG, "args is NULL");
  const size_t need = ltxattn_fwd_workspace(args);
  if (need > ltx::kNoAllocScratchBytes) {
    char buf[256];
    snprintf(buf, sizeof buf,
             "ltxattn_fwd_noalloc: these arguments need %zu bytes of scratch, above the fixed %zu; "
             "use ltxattn_fwd with a caller-provided workspace",
             need, ltx::kNoAllocScratchBytes);
    return ltx::set_error_message(LTXATTN_ERR_WORKSPACE, buf);
  }
  ltxattn_fwd_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  if (need > 0) {
    void* scratch = nullptr;
    if (int rc = ltx::scratch_for_current_device(&scratch)) return rc;
    a.workspace = scratch;
    a.workspace_bytes = ltx::kNoAllocScratchBytes;
  }
  return ltxattn_fwd(&a, stream);
}

}  // extern "C"
