// Host-side launchers shared between the translation units of libfpa_b200 (not part of the public ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "fpa_common.cuh"

namespace fpa {

struct Str4 {
  int64_t b, h, t, d;
};

inline Str4 str4(const int64_t s[4]) { return Str4{s[0], s[1], s[2], s[3]}; }

// Inputs of the per-query pairs of the tensor-core backward when the stats kernel builds them itself:
// qv4[t] = (-lse, -delta, PRE, prey) in the pair layout, delta_t = sum_d dO[t, d] O[t, d] (fp16 O and dO with
// unit innermost stride and 16-byte aligned rows).
struct QvIn {
  const __half* o;
  Str4 so;
  const __half* dout;
  Str4 sdo;
  const float* lse;
  float4* qv4;
  int D;
};

// Sizes shared by every kernel of one call. Tiles are BT positions; NB = ceil(T / BT); TP = NB * BT.
struct Dims {
  int B, H, T, D, BT, NB, TP;
  int BH() const { return B * H; }
};

inline Dims make_dims(int B, int H, int T, int D, int BT) {
  Dims d{B, H, T, D, BT, (T + BT - 1) / BT, 0};
  d.TP = d.NB * BT;
  return d;
}

// Profiling mark (fpa_profile.cu): when profiling is on, records an event on `s` that starts the timing of the
// kernel `name` launched next; name = nullptr ends the last kernel of a call. A no-op otherwise.
void prof_mark(cudaStream_t s, const char* name);
bool prof_on();  // per-kernel timing enabled (the library then launches everything on the caller's stream)

// cudaFuncSetAttribute(fn, MaxDynamicSharedMemorySize, bytes) on the current device, made once per (device,
// kernel) with the largest size asked for so far; later calls that ask for no more cost a lock and a lookup
// (fpa_tma.cu). Thread-safe.
cudaError_t allow_dynamic_smem(const void* fn, int bytes);

// Launches `kernel` on `s` with programmatic stream serialization: it may start while the previous kernel of the
// stream runs its last CTAs (see pdl_wait / pdl_launch_dependents in fpa_common.cuh, which the kernel must call).
template <typename... P, typename... A>
cudaError_t launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}

// Records the message that fpa_last_error returns on the calling thread (fpa_capi.cu).
void set_last_error(const std::string& msg);

// The least workspace fpa_fwd accepts for these sizes (fpa_fwd_workspace_bytes without the room for the
// forward's key-range split, which fpa_fwd then leaves out); 0 for invalid sizes (fpa_capi.cu).
size_t fwd_workspace_min_bytes(int dtype, int B, int H, int T, int D, int path);

// Workspace carving (all arrays 256-byte aligned, after the 256-byte status word).
size_t stats_bytes(const Dims& d);
size_t bwd_scratch_bytes(const Dims& d, int tb_parts);
Stats carve_stats(char* base, const Dims& d);
BwdScratch carve_bwd(char* base, const Dims& d, int tb_parts);

// fpa_aux.cu
size_t keycols_bytes(const Dims& d);
KeyCols carve_keycols(char* base, const Dims& d);
// cols_scaled = 1: the forward's b'-scaled key vectors; 0: raw (a = SUF - psi, psi, phi) for the backward.
// tile_cnt (optional): ncnt ints per (head, tile), [BH][NB][ncnt], set to zero (the join counters of the split
// kernels that follow).
cudaError_t launch_stats(const float* phi, const float* psi, const float* beta, const Dims& d, float tau,
                         const Stats& st, const KeyCols& cols, int cols_scaled, int* status, cudaStream_t s,
                         const Fact* fact = nullptr, const QvIn* qv = nullptr, int* tile_cnt = nullptr,
                         int ncnt = 0);
cudaError_t launch_delta(int dtype, const void* o, Str4 so, const void* dout, Str4 sdo, const Dims& d, float* delta,
                         const float* lse, float* lsep, cudaStream_t s);
cudaError_t launch_qv_pack(const float* lse, const float* delta, const float* pre, const float* prey, const Dims& d,
                           float4* qv4, cudaStream_t s);
// The stats kernel builds the per-query pairs itself (QvIn) when O and dO are fp16 with unit innermost stride and
// 16-byte aligned rows and D <= 128; otherwise launch_delta + launch_qv_pack.
bool qv_delta_fusable(int dtype, const void* o, Str4 so, const void* dout, Str4 sdo, const Dims& d);
cudaError_t launch_diag_dphi(const float* phi, const float* gd, const Dims& d, float tau, float* dphi4, cudaStream_t s);
// dphi_kernel, which also reduces dbeta; for long contexts dphi_part3_kernel first. Sets *launched.
cudaError_t launch_dphi(const float* phi, const float* beta, const Dims& d, float tau, const Stats& st,
                        const BwdScratch& sc, float* dphi, float* dbeta, cudaStream_t s, int* launched);

// The FFMA path (fp32, fp16 with D = 256, or path=SIMT): tiles of 64 positions, any supported D, fp16 or fp32.
constexpr int kSimtBT = 64;
// fpa_simt_fwd.cu: the register-tiled FFMA forward.
cudaError_t simt_fwd_tiled(const FpaFwdArgs& a, const Dims& d, const Stats& st, cudaStream_t s);
// fpa_simt_bwd.cu: the register-tiled FFMA backward (kv-pass and q-pass in one launch); its kv-pass writes
// kSimtTbParts per-warp partial sums per tile pair into the TB array.
constexpr int kSimtTbParts = 8;
cudaError_t simt_bwd_tiled(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s);

}  // namespace fpa
