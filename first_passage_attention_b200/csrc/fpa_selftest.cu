// fpa_selftest_wait_timeout: drives the bounded mbarrier wait of the tensor-core kernels to expiry.
//
// Every wait of the tcgen05 kernels goes through fpa::sm100::mbar_wait_limit: after the limit it records
// FPA_ERR_TIMEOUT and the call-site id in the workspace status word and returns false, and the kernel unwinds.
// In a correct build no wait of those kernels ever runs out, so this entry point exists to exercise that path on
// the GPU without faulting or hanging it: one warp initialises an mbarrier that nothing will ever arrive on, waits
// on it with the caller's (short) limit through the same function, and returns. The host then reads the status
// with fpa_workspace_status exactly as it would after a real call.
#include "fpa_sm100.cuh"
#include "fpa_internal.h"

namespace fpa {
namespace {

constexpr int kSelftestSite = 0x7e57;

__global__ void wait_timeout_kernel(int* status, unsigned long long limit_ns, int* returned) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_mbar_init();
  }
  __syncwarp();
  // Nothing arrives on `bar`: phase 0 never completes, so the wait can only end by its limit.
  const bool ok = sm100::mbar_wait_limit(&bar, 0, status, kSelftestSite, limit_ns);
  if (threadIdx.x == 0) *returned = ok ? 2 : 1;
}

}  // namespace
}  // namespace fpa

extern "C" FPA_API int fpa_selftest_wait_timeout(void* workspace, unsigned long long limit_ns, void* stream) {
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
    fpa::set_last_error("workspace must be a non-null 256-byte aligned device pointer");
    return FPA_ERR_WORKSPACE;
  }
  if (limit_ns == 0 || limit_ns > 1000000000ull) {
    fpa::set_last_error("limit_ns must be in (0, 1e9]");
    return FPA_ERR_INVALID_ARGUMENT;
  }
  int* status = static_cast<int*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, 2 * sizeof(int), s);
  if (e == cudaSuccess) {
    fpa::wait_timeout_kernel<<<1, 32, 0, s>>>(status, limit_ns, status + 1);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    fpa::set_last_error(std::string("fpa_selftest_wait_timeout: ") + cudaGetErrorString(e));
    return FPA_ERR_CUDA;
  }
  return FPA_OK;
}
