// Shared device helpers and the workspace layout of the FPA kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fpa.h"

namespace fpa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kInf = __builtin_huge_valf();

// Device status word at the head of every workspace (see fpa_workspace_status). The first 256 bytes of a
// workspace are reserved for it so that the per-head arrays that follow stay 256-byte aligned.
constexpr size_t kStatusBytes = 256;

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// 2^x and log2(x) with the hardware approximations (PTX ex2.approx.ftz.f32 / lg2.approx.ftz.f32: about 2^-22
// relative error; subnormal results flush to zero; ex2(-inf) = +0, lg2(0) = -inf). One MUFU operation each.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 1/x with the hardware approximation (PTX rcp.approx.ftz.f32). One MUFU operation.
__device__ __forceinline__ float rcp_approx_f(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Programmatic dependent launch (launch_pdl in fpa_internal.h). A kernel launched that way may start while the
// kernel before it on the stream is still running, once every CTA of that kernel has called pdl_launch_dependents
// (or exited): its CTAs run their prologue (shared-memory carving, barrier set-up, TMEM allocation), then
// pdl_wait() blocks until the previous kernel has completed and its memory writes are visible. Every kernel
// launched that way calls pdl_wait() before its first global-memory access, and pdl_launch_dependents() only after
// it, so that no more than two kernels of a stream overlap. Both are no-ops for a kernel launched without the
// attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// log2(2^a + 2^b), with -inf + -inf = -inf (the stable base-2 log-add-exp of kernel.py:73-75).
__device__ __forceinline__ float lse2(float a, float b) {
  float m = fmaxf(a, b);
  if (m == -kInf) return m;
  return m + lg2(1.0f + ex2(fminf(a, b) - m));
}

// Sum over the `W` consecutive lanes of a group (W a power of two <= 32, groups aligned). Every lane of the group
// gets the bit-identical result: the butterfly pairs lanes symmetrically and float addition commutes.
template <int W>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Per-tile statistics of the field phi, for tiles of BT positions (kernel.py:84-100 computes the same quantities):
//   PRE_t  = min phi over [tile start, t]                      PREL_t = log2 sum 2^{a2} over [tile start, t]
//   SUF_s  = min phi over (s, tile end] (inf if empty)         SUFL_s = log2 sum 2^{a2} over (s, tile end]
//   BMIN_j = min phi over tile j                               BL_j   = log2 sum 2^{a2} over tile j
// with a2 = -phi * log2(e) / tau. Positions >= T are excluded (phi = +inf, a2 = -inf there).
struct Stats {
  float* pre;   // [BH][TP]
  float* suf;   // [BH][TP]
  float* prel;  // [BH][TP]
  float* sufl;  // [BH][TP]
  float* bmin;  // [BH][NB]
  float* bl;    // [BH][NB]
};

// Per-key vectors the tensor-core forward streams next to each key tile (float32, [BH][TP]), in the units of the
// log2-scaled logits (b' = beta * log2 e of the key's head):
//   a_s   = b' * min(SUF_s - psi_s, 0)   (the part of the bias that does not depend on the query)
//   psi_s = -b' * psi_s                   (negated, so the bias needs an add rather than a subtract)
//   phi_s = b' * phi_s                    (for the running extremum inside the diagonal tile)
// All three are 0 beyond T.
struct KeyCols {
  float* a;
  float* psi;
  float* phi;
};

// Factors that let the tensor-core backward form the soft-min denominators without a per-element exp2
// (float32; written by stats_kernel when `prey` is set):
//   prey_t = 2^{PREL_t - BL_j} for t in tile j, prer_j = BL_j - PREL_{first of j}
//   sufy_s = 2^{SUFL_s - SUFL_{first of j}} for s in tile j, sufr_j = SUFL_{first} - min_{SUFL_s > -inf} SUFL_s
struct Fact {
  float* prey;  // [BH][TP]
  float* sufy;  // [BH][TP]
  float* prer;  // [BH][NB]
  float* sufr;  // [BH][NB]
  // [BH][TP] per key, two keys c, c+1 (c even) per pair of float4 for packed f32x2 arithmetic:
  // kv4[c] = (SUF_c - psi_c, SUF_c1 - psi_c1, -psi_c, -psi_c1), kv4[c + 1] = (sufy_c, sufy_c1, SUFL_c, SUFL_c1)
  float4* kv4;
};

// Scratch of the backward pass (all float32, per head z = b*H + h).
struct BwdScratch {
  float* delta;  // [BH][TP]   rowsum(dO * O)
  float* w;      // [BH][TP]   soft-min partial sums per key, normalised by 2^{c_s} (part "key tile")
  float* dphi2;  // [BH][TP]   soft-min contribution of u in the query's tile
  float* dphi4;  // [BH][TP]   soft-min contribution of u in the diagonal tile
  float* tb;     // [BH][NB][NB][tb_parts] tile-pair totals, normalised by 2^{cmid}, as tb_sum partial sums
  float* dbeta;  // [BH][NB]   dbeta partial per key tile
  float* part3;  // [BH][NB]   long contexts: the strictly-between part of dphi per tile, before 2^{a2_u - c_U}
  int tb_parts;  // floats per tile pair (at least 2: the O(NB^2) part-3 passes reuse two of them)
  int tb_sum;    // partial sums per tile pair that the kv-pass writes (summed in a fixed order)
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Bounded-wait failure reporting: a kernel whose wait expires stores this code (first writer wins) and returns.
__device__ __forceinline__ void report_timeout(int* status, int where) {
  if (status) atomicCAS(status, 0, (FPA_ERR_TIMEOUT << 16) | (where & 0xffff));
}

}  // namespace fpa
