// fpa_fwd_noalloc: the forward pass for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc (or any allocator) at the point where they run the
// operator: code that runs inside another runtime's memory pool with no allocation hook, plugin hosts that hand
// over only the input and output buffers, or paths where an allocation would synchronise the device or fail
// after start-up (for instance when device memory is fully reserved by the host application). fpa_fwd needs a
// caller-provided workspace for its per-call scratch (the per-tile field statistics and the per-key vectors the
// attention kernel streams); this entry point instead uses a scratch array that is part of the library image:
// `g_fwd_scratch`, a file-scope __device__ array of kNoAllocScratchBytes. Every GPU that loads the library holds
// that array until the process exits.
//
// Host code cannot use `g_fwd_scratch` directly: in host code the name is only a host-side stand-in, not a
// device address. The device address is looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call made on that device; that first call should therefore come before any stream
// capture. All calls share the array and it keeps the last call's contents: the one word that must start at zero
// (the status word at its head) is cleared by the first kernel of every call, and every other byte a call reads
// is written earlier in the same call. Calls whose kernels overlap on the GPU (different streams, or different
// host threads, on one device) race on the array and must be serialised by the caller.
#include <cstdio>
#include <mutex>
#include <string>

#include "fpa_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = FPA_NOALLOC_SCRATCH_BYTES;  // 8 MiB

static __device__ __align__(256) unsigned char g_fwd_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_fwd_scratch on the current device (looked up on the first call per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fwd_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" FPA_API int fpa_fwd_noalloc(FpaFwdArgs* a, void* stream) {
  if (a == nullptr) return fpa_fwd(a, stream);  // reports the null argument block
  const size_t need = fpa_fwd_workspace_bytes(a->dtype, a->B, a->H, a->T, a->D, a->path);
  if (need == 0) return fpa_fwd(a, stream);  // invalid sizes: let fpa_fwd report them with its messages
  if (need > kNoAllocScratchBytes) {
    // Too large for the built-in scratch: nothing is launched.
    a->kernels_launched = 0;
    char msg[256];
    snprintf(msg, sizeof msg,
             "fpa_fwd_noalloc: this call needs %zu bytes of scratch, more than the %zu built into the library; "
             "call fpa_fwd with a workspace instead",
             need, kNoAllocScratchBytes);
    fpa::set_last_error(msg);
    return FPA_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) {
    a->kernels_launched = 0;
    fpa::set_last_error(std::string("fpa_fwd_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    return FPA_ERR_CUDA;
  }
  a->workspace = scratch;
  a->workspace_bytes = kNoAllocScratchBytes;
  return fpa_fwd(a, stream);
}
