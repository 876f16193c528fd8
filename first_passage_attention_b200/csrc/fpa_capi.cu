// The C ABI of libfpa_b200 (include/fpa.h): argument checks, workspace carving and the sequence of launches.
#include <cstdio>
#include <cstring>
#include <string>

#include "fpa_internal.h"
#include "fpa_tc.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return FPA_ERR_CUDA;
}

bool pow2_ge16(int n) { return n >= 16 && (n & (n - 1)) == 0; }

// Mirrors the shape checks of kernel.py:469-486 (the caller has already matched q, k and v shapes).
int check_common(int dtype, int B, int H, int T, int D, float tau) {
  if (dtype != FPA_DTYPE_F16 && dtype != FPA_DTYPE_F32) return fail(FPA_ERR_INVALID_ARGUMENT, "q, k and v must all be fp16 or all fp32");
  if (B <= 0 || H <= 0 || T <= 0) return fail(FPA_ERR_INVALID_ARGUMENT, "q, k and v must have the same shape (B, H, T, D)");
  if (!pow2_ge16(D)) return fail(FPA_ERR_INVALID_ARGUMENT, "the head dimension and the block must be powers of two >= 16");
  if (D > 256) return fail(FPA_ERR_UNSUPPORTED, "head dimensions above 256 are not supported");
  // Per-head kernels run on a (tiles, H, B) grid, whose y and z extents stop at 65535; row indices are 32-bit.
  if (B > 65535 || H > 65535) return fail(FPA_ERR_UNSUPPORTED, "B and H above 65535 are not supported");
  if (int64_t(B) * H * T > INT32_MAX) return fail(FPA_ERR_UNSUPPORTED, "B * H * T above 2^31 - 1 is not supported");
  if (!(tau > 0.f)) return fail(FPA_ERR_INVALID_ARGUMENT, "tau must be positive");
  return FPA_OK;
}

int check_workspace(void* ws, size_t have, size_t need) {
  if (ws == nullptr || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(FPA_ERR_WORKSPACE, "workspace must be a non-null 256-byte aligned device pointer");
  if (have < need) return fail(FPA_ERR_WORKSPACE, "workspace is smaller than fpa_*_workspace_bytes requires");
  return FPA_OK;
}

bool tensor_path_ok(int dtype, int D) { return dtype == FPA_DTYPE_F16 && fpa::tc_supports(D); }

int pick_path(int requested, int dtype, int D) {
  if (requested == FPA_PATH_SIMT) return FPA_PATH_SIMT;
  if (requested == FPA_PATH_TENSOR) return tensor_path_ok(dtype, D) ? FPA_PATH_TENSOR : -1;
  return tensor_path_ok(dtype, D) ? FPA_PATH_TENSOR : FPA_PATH_SIMT;
}

int tile_of(int path) { return path == FPA_PATH_TENSOR ? fpa::kTcBT : fpa::kSimtBT; }

// Floats per tile pair of the TB array: both kv-passes write 8 per-warp partial sums (the O(NB^2) part-3 passes of
// the dphi combination reuse two of them).
int tb_parts_of(int path) { return path == FPA_PATH_TENSOR ? fpa::kTcTbParts : fpa::kSimtTbParts; }

// The backward follows the same choice as the forward: tensor cores for fp16 with a supported D, FFMA otherwise.
int bwd_path(int requested, int dtype, int D) { return pick_path(requested, dtype, D); }

// The forward's workspace without the key-range split's partial outputs: what fpa_fwd needs at least.
size_t fwd_ws_min(int dtype, int B, int H, int T, int D, int path) {
  fpa::Dims d = fpa::make_dims(B, H, T, D, tile_of(path));
  return fpa::kStatusBytes + fpa::stats_bytes(d) + (path == FPA_PATH_TENSOR ? fpa::keycols_bytes(d) : 0);
}

// What fpa_fwd_workspace_bytes reports: the minimum plus, on the tensor-core path, the partial outputs of the
// key-range split that small grids take on the current device.
size_t fwd_ws(int dtype, int B, int H, int T, int D, int path) {
  const size_t m = fwd_ws_min(dtype, B, H, T, D, path);
  return path == FPA_PATH_TENSOR ? m + fpa::tc_fwd_split_bytes(fpa::make_dims(B, H, T, D, tile_of(path))) : m;
}

size_t bwd_ws(int dtype, int B, int H, int T, int D, int path) {
  fpa::Dims d = fpa::make_dims(B, H, T, D, tile_of(path));
  return fpa::kStatusBytes + fpa::stats_bytes(d) + fpa::bwd_scratch_bytes(d, tb_parts_of(path)) +
         (path == FPA_PATH_TENSOR ? fpa::tc_bwd_extra_bytes(d) : 0);
}

}  // namespace

void fpa::set_last_error(const std::string& msg) { g_last_error = msg; }

size_t fpa::fwd_workspace_min_bytes(int dtype, int B, int H, int T, int D, int path) {
  if (check_common(dtype, B, H, T, D, 1.f) != FPA_OK) return 0;
  const int p = pick_path(path, dtype, D);
  return p < 0 ? 0 : fwd_ws_min(dtype, B, H, T, D, p);
}

extern "C" {

int fpa_abi_version(void) { return FPA_ABI_VERSION; }

size_t fpa_struct_size(int which) {
  return which == 0 ? sizeof(FpaFwdArgs) : which == 1 ? sizeof(FpaBwdArgs) : which == 2 ? sizeof(FpaFieldArgs) : 0;
}

size_t fpa_fwd_workspace_bytes(int dtype, int B, int H, int T, int D, int path) {
  if (check_common(dtype, B, H, T, D, 1.f) != FPA_OK) return 0;
  int p = pick_path(path, dtype, D);
  if (p < 0) return 0;
  return fwd_ws(dtype, B, H, T, D, p);
}

size_t fpa_bwd_workspace_bytes(int dtype, int B, int H, int T, int D, int path) {
  if (check_common(dtype, B, H, T, D, 1.f) != FPA_OK) return 0;
  int p = bwd_path(path, dtype, D);
  if (p < 0) return 0;
  return bwd_ws(dtype, B, H, T, D, p);
}

int fpa_fwd(FpaFwdArgs* a, void* stream) {
  if (a == nullptr) return fail(FPA_ERR_INVALID_ARGUMENT, "null argument block");
  a->kernels_launched = 0;
  int rc = check_common(a->dtype, a->B, a->H, a->T, a->D, a->tau);
  if (rc) return rc;
  if (!a->q || !a->k || !a->v || !a->phi || !a->psi || !a->beta || !a->o || !a->lse)
    return fail(FPA_ERR_INVALID_ARGUMENT, "null tensor pointer");
  int path = pick_path(a->path, a->dtype, a->D);
  if (path < 0) return fail(FPA_ERR_UNSUPPORTED, "the tensor-core path needs fp16 inputs and D in {16, 32, 64, 128}");
  rc = check_workspace(a->workspace, a->workspace_bytes, fwd_ws_min(a->dtype, a->B, a->H, a->T, a->D, path));
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  fpa::Dims d = fpa::make_dims(a->B, a->H, a->T, a->D, tile_of(path));
  char* ws = static_cast<char*>(a->workspace);
  int* status = reinterpret_cast<int*>(ws);
  fpa::Stats st = fpa::carve_stats(ws + fpa::kStatusBytes, d);
  fpa::KeyCols cols{nullptr, nullptr, nullptr};
  int* join_cnt = nullptr;  // the key-range split's per-tile counters, zeroed by the stats kernel
  const size_t used = fpa::kStatusBytes + fpa::stats_bytes(d) + fpa::keycols_bytes(d);
  if (path == FPA_PATH_TENSOR) {
    cols = fpa::carve_keycols(ws + fpa::kStatusBytes + fpa::stats_bytes(d), d);
    join_cnt = fpa::tc_fwd_split_counters(d, ws + used, a->workspace_bytes - used);
  }
  fpa::prof_mark(s, "stats");
  cudaError_t e = fpa::launch_stats(a->phi, a->psi, a->beta, d, a->tau, st, cols, 1, status, s, nullptr, nullptr,
                                    join_cnt, 1);
  if (e != cudaSuccess) return cuda_fail(e, "stats kernel");
  a->kernels_launched = 1;
  if (path == FPA_PATH_TENSOR) {
    int n = 0;
    fpa::prof_mark(s, "fwd_tc");
    rc = fpa::tc_fwd(*a, d, st, cols, ws + used, a->workspace_bytes - used, status, s, &n, &g_last_error);
    a->kernels_launched += n;
    if (rc) return rc;
  } else {
    fpa::prof_mark(s, "fwd_simt");
    e = fpa::simt_fwd_tiled(*a, d, st, s);
    if (e != cudaSuccess) return cuda_fail(e, "forward kernel");
    a->kernels_launched += 1;
  }
  fpa::prof_mark(s, nullptr);
  a->path_taken = path;
  return FPA_OK;
}

int fpa_bwd(FpaBwdArgs* a, void* stream) {
  if (a == nullptr) return fail(FPA_ERR_INVALID_ARGUMENT, "null argument block");
  a->kernels_launched = 0;
  int rc = check_common(a->dtype, a->B, a->H, a->T, a->D, a->tau);
  if (rc) return rc;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->phi || !a->psi || !a->beta || !a->dq ||
      !a->dk || !a->dv || !a->dphi || !a->dpsi || !a->dbeta)
    return fail(FPA_ERR_INVALID_ARGUMENT, "null tensor pointer");
  int path = bwd_path(a->path, a->dtype, a->D);
  if (path < 0) return fail(FPA_ERR_UNSUPPORTED, "the tensor-core path needs fp16 inputs and D in {16, 32, 64, 128}");
  rc = check_workspace(a->workspace, a->workspace_bytes, bwd_ws(a->dtype, a->B, a->H, a->T, a->D, path));
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  fpa::Dims d = fpa::make_dims(a->B, a->H, a->T, a->D, tile_of(path));
  int* status = static_cast<int*>(a->workspace);
  char* ws = static_cast<char*>(a->workspace) + fpa::kStatusBytes;
  fpa::Stats st = fpa::carve_stats(ws, d);
  fpa::BwdScratch sc = fpa::carve_bwd(ws + fpa::stats_bytes(d), d, tb_parts_of(path));
  int n = 0;
  cudaError_t e;
  if (path == FPA_PATH_TENSOR) {
    char* extra = ws + fpa::stats_bytes(d) + fpa::bwd_scratch_bytes(d, sc.tb_parts);
    int m = 0;
    rc = fpa::tc_bwd(*a, d, st, sc, extra, status, s, &m, &g_last_error);
    n += m;
    if (rc) {
      a->kernels_launched = n;
      return rc;
    }
  } else {
    fpa::prof_mark(s, "stats");
    e = fpa::launch_stats(a->phi, a->psi, a->beta, d, a->tau, st, fpa::KeyCols{nullptr, nullptr, nullptr}, 0, status,
                          s);
    if (e != cudaSuccess) return cuda_fail(e, "stats kernel");
    ++n;
    fpa::prof_mark(s, "delta");
    e = fpa::launch_delta(a->dtype, a->o, fpa::str4(a->o_stride), a->dout, fpa::str4(a->dout_stride), d, sc.delta,
                          nullptr, nullptr, s);
    if (e != cudaSuccess) return cuda_fail(e, "delta kernel");
    ++n;
    fpa::prof_mark(s, "bwd_simt");
    e = fpa::simt_bwd_tiled(*a, d, st, sc, s);
    if (e != cudaSuccess) return cuda_fail(e, "backward kernel");
    ++n;
  }
  fpa::prof_mark(s, "dphi");
  int nd = 0;
  e = fpa::launch_dphi(a->phi, a->beta, d, a->tau, st, sc, a->dphi, a->dbeta, s, &nd);  // also reduces dbeta
  if (e != cudaSuccess) return cuda_fail(e, "dphi kernel");
  n += nd;
  fpa::prof_mark(s, nullptr);
  a->kernels_launched = n;
  a->path_taken = path;
  return FPA_OK;
}

int fpa_workspace_status(void* workspace, void* stream) {
  if (workspace == nullptr) return fail(FPA_ERR_WORKSPACE, "null workspace");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the workspace status");
  if (v == 0) return FPA_OK;
  int zero = 0;
  e = cudaMemcpyAsync(workspace, &zero, sizeof(int), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  char buf[128];
  snprintf(buf, sizeof buf, "a bounded device-side wait expired (site %d)", v & 0xffff);
  g_last_error = buf;
  return v >> 16;
}

const char* fpa_status_string(int status) {
  switch (status) {
    case FPA_OK: return "ok";
    case FPA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FPA_ERR_UNSUPPORTED: return "unsupported configuration";
    case FPA_ERR_CUDA: return "CUDA error";
    case FPA_ERR_TIMEOUT: return "device-side wait timed out";
    case FPA_ERR_WORKSPACE: return "bad workspace";
    default: return "unknown status";
  }
}

const char* fpa_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
