// The layer's field (kernel.py:502-509) in one pass each way: fpa_field_fwd / fpa_field_bwd (include/fpa.h).
//
// The fp32 projection of x gives, per batch b, position t and head h, an increment delta = proj[b, t, h] and
// offsets g = proj[b, t, H + h], hh = proj[b, t, 2H + h]. The walk is w_t = sum_{u <= t} delta_u and the field is
// phi = w + g, psi = w + hh, written [B, H, T] contiguous (the layout the operator reads). The backward maps dphi,
// dpsi [B, H, T] to the projection's gradient: d delta_t = sum_{u >= t} (dphi_u + dpsi_u), dg = dphi, dh = dpsi.
//
// One block per (h, b) walks the head's positions in chunks of 1024, one position per thread: a warp inclusive
// scan, a scan of the 32 warp totals and a running carry from the previous chunks. The order of every sum is fixed,
// so the results are deterministic.
#include <string>

#include "fpa_internal.h"

namespace fpa {
namespace {

constexpr int kFieldThreads = 1024;

// Inclusive sum over the block's threads in thread order (reverse = false) or in reverse thread order (reverse =
// true, thread 1023 first); `carry` is added to every result and updated to the block total plus carry.
__device__ __forceinline__ float block_scan(float x, bool reverse, float* warp_tot, float& carry) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int rl = reverse ? 31 - lane : lane;  // position in the scan order inside the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = reverse ? __shfl_down_sync(0xffffffffu, x, o) : __shfl_up_sync(0xffffffffu, x, o);
    if (rl >= o) x += y;
  }
  if (rl == 31) warp_tot[w] = x;
  __syncthreads();
  float before = carry;
  const int wr = reverse ? 31 - w : w;  // warp position in the scan order
  for (int v = 0; v < wr; ++v) before += warp_tot[reverse ? 31 - v : v];
  float total = carry;
  for (int v = 0; v < 32; ++v) total += warp_tot[v];
  __syncthreads();  // warp_tot is rewritten by the next chunk
  carry = total;
  return x + before;
}

__global__ void __launch_bounds__(kFieldThreads)
field_fwd_kernel(const float* __restrict__ proj, int64_t sb, int64_t st, int64_t sc, int H, int T,
                 float* __restrict__ phi, float* __restrict__ psi) {
  __shared__ float warp_tot[32];
  const int h = blockIdx.x, b = blockIdx.y;
  const float* base = proj + b * sb;
  const size_t out = (size_t(b) * H + h) * T;
  float carry = 0.f;
  for (int t0 = 0; t0 < T; t0 += kFieldThreads) {
    const int t = t0 + int(threadIdx.x);
    float d = 0.f, g = 0.f, hh = 0.f;
    if (t < T) {
      const float* row = base + int64_t(t) * st;
      d = row[int64_t(h) * sc];
      g = row[int64_t(H + h) * sc];
      hh = row[int64_t(2 * H + h) * sc];
    }
    const float w = block_scan(d, false, warp_tot, carry);
    if (t < T) {
      phi[out + t] = w + g;
      psi[out + t] = w + hh;
    }
  }
}

__global__ void __launch_bounds__(kFieldThreads)
field_bwd_kernel(const float* __restrict__ dphi, const float* __restrict__ dpsi, int H, int T,
                 float* __restrict__ dproj, int64_t sb, int64_t st, int64_t sc) {
  __shared__ float warp_tot[32];
  const int h = blockIdx.x, b = blockIdx.y;
  float* base = dproj + b * sb;
  const size_t in = (size_t(b) * H + h) * T;
  float carry = 0.f;
  const int nchunks = (T + kFieldThreads - 1) / kFieldThreads;
  for (int c = nchunks - 1; c >= 0; --c) {
    const int t = c * kFieldThreads + int(threadIdx.x);
    float gp = 0.f, gs = 0.f;
    if (t < T) {
      gp = dphi[in + t];
      gs = dpsi[in + t];
    }
    const float dd = block_scan(gp + gs, true, warp_tot, carry);  // sum over u >= t
    if (t < T) {
      float* row = base + int64_t(t) * st;
      row[int64_t(h) * sc] = dd;
      row[int64_t(H + h) * sc] = gp;
      row[int64_t(2 * H + h) * sc] = gs;
    }
  }
}

int field_check(const FpaFieldArgs* a) {
  if (a == nullptr) return FPA_ERR_INVALID_ARGUMENT;
  if (a->B <= 0 || a->T <= 0 || a->H <= 0) return FPA_ERR_INVALID_ARGUMENT;
  if (a->B > 65535 || a->H > 65535 || int64_t(a->B) * a->H * a->T > INT32_MAX) return FPA_ERR_UNSUPPORTED;
  return FPA_OK;
}

}  // namespace
}  // namespace fpa

extern "C" FPA_API int fpa_field_fwd(const FpaFieldArgs* a, void* stream) {
  int rc = fpa::field_check(a);
  if (rc) {
    fpa::set_last_error("fpa_field_fwd: B, T and H must be positive (B, H <= 65535, B * H * T < 2^31)");
    return rc;
  }
  if (!a->proj || !a->phi || !a->psi) {
    fpa::set_last_error("fpa_field_fwd: null tensor pointer");
    return FPA_ERR_INVALID_ARGUMENT;
  }
  fpa::field_fwd_kernel<<<dim3(a->H, a->B), fpa::kFieldThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      a->proj, a->proj_stride[0], a->proj_stride[1], a->proj_stride[2], a->H, a->T, a->phi, a->psi);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fpa::set_last_error(std::string("fpa_field_fwd: ") + cudaGetErrorString(e));
    return FPA_ERR_CUDA;
  }
  return FPA_OK;
}

extern "C" FPA_API int fpa_field_bwd(const FpaFieldArgs* a, void* stream) {
  int rc = fpa::field_check(a);
  if (rc) {
    fpa::set_last_error("fpa_field_bwd: B, T and H must be positive (B, H <= 65535, B * H * T < 2^31)");
    return rc;
  }
  if (!a->dphi || !a->dpsi || !a->dproj) {
    fpa::set_last_error("fpa_field_bwd: null tensor pointer");
    return FPA_ERR_INVALID_ARGUMENT;
  }
  fpa::field_bwd_kernel<<<dim3(a->H, a->B), fpa::kFieldThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      a->dphi, a->dpsi, a->H, a->T, a->dproj, a->dproj_stride[0], a->dproj_stride[1], a->dproj_stride[2]);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fpa::set_last_error(std::string("fpa_field_bwd: ") + cudaGetErrorString(e));
    return FPA_ERR_CUDA;
  }
  return FPA_OK;
}
