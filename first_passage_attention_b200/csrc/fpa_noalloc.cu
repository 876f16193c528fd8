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
// device address. The device address belongs to the CUDA context that is current, so it is looked up with
// cudaGetSymbolAddress, with the caller's device and context current, on every call made outside stream capture
// (the lookup is cheap and allocates nothing once the array exists), and remembered per context for calls made
// during a capture, which cannot look it up. CUDA loads a module lazily by default (CUDA_MODULE_LOADING=LAZY), and
// this file's module holds no kernel, so the array itself is created by the first lookup in a context: a caller
// that must not allocate later makes that first lookup at start-up, either with a set-up call
// fpa_fwd_noalloc(NULL, stream) or with a first small forward, and before any stream capture. All calls share the
// array and it keeps the last call's contents: the one word that must start at zero (the status word at its head)
// is cleared by the first kernel of every call, and every other byte a call reads is written earlier in the same
// call. Calls whose kernels overlap on the GPU (different streams, or different host threads, on one device) race
// on the array and must be serialised by the caller.
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "fpa_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = FPA_NOALLOC_SCRATCH_BYTES;  // 8 MiB

static __device__ __align__(256) unsigned char g_fwd_scratch[kNoAllocScratchBytes];

std::mutex g_mutex;
struct Known {
  void* ctx;   // CUcontext current when the address was looked up
  void* addr;  // device address of g_fwd_scratch in that context
};
std::vector<Known> g_known;

typedef int (*CtxGetCurrentFn)(void**);  // cuCtxGetCurrent(CUcontext*) -> CUresult

void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of g_fwd_scratch in the current context. Outside stream capture it is looked up afresh (which
// also creates the array on the first lookup in a context); during a capture the address remembered for the
// current context is used, and a context that has none is an error.
cudaError_t scratch_address(cudaStream_t s, void** out, std::string* why) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);  // makes the device's primary context current if none is
  if (e != cudaSuccess) return e;
  void* ctx = current_context();
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(s, &cap);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_mutex);
  Known* known = nullptr;
  for (Known& k : g_known)
    if (k.ctx == ctx) known = &k;
  if (cap != cudaStreamCaptureStatusNone) {
    if (known == nullptr || ctx == nullptr) {
      *why = "the first fpa_fwd_noalloc call in a CUDA context must come before any stream capture";
      return cudaErrorStreamCaptureUnsupported;
    }
    *out = known->addr;
    return cudaSuccess;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_fwd_scratch);
  if (e != cudaSuccess) return e;
  if (known)
    known->addr = p;
  else
    g_known.push_back(Known{ctx, p});
  *out = p;
  return cudaSuccess;
}

}  // namespace

extern "C" FPA_API int fpa_fwd_noalloc(FpaFwdArgs* a, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a == nullptr) {
    // Set-up only: look the array up in the current context (creating it there) and launch nothing.
    void* scratch = nullptr;
    std::string why;
    const cudaError_t e = scratch_address(s, &scratch, &why);
    if (e != cudaSuccess) {
      fpa::set_last_error(std::string("fpa_fwd_noalloc: ") + (why.empty() ? cudaGetErrorString(e) : why));
      return FPA_ERR_CUDA;
    }
    return FPA_OK;
  }
  const size_t need = fpa::fwd_workspace_min_bytes(a->dtype, a->B, a->H, a->T, a->D, a->path);
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
  std::string why;
  const cudaError_t e = scratch_address(s, &scratch, &why);
  if (e != cudaSuccess) {
    a->kernels_launched = 0;
    fpa::set_last_error(std::string("fpa_fwd_noalloc: ") +
                        (why.empty() ? std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e) : why));
    return FPA_ERR_CUDA;
  }
  a->workspace = scratch;
  a->workspace_bytes = kNoAllocScratchBytes;
  return fpa_fwd(a, stream);
}
