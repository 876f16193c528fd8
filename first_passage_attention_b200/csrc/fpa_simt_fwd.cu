// Register-tiled FFMA forward of the FPA operator: the fp32 path, and fp16 with a head dimension the tensor-core
// kernels do not cover (D = 256). Same decomposition as the tensor-core forward and the reference (kernel.py:104-162):
// one CTA per query tile of 64 rows, walking its key tiles from the diagonal backwards so that `mid` (the minimum of
// phi over the key tiles already passed) is a running minimum, with an online softmax.
//
// Work split (256 threads as 16 x 16): thread (ty, tx) owns rows 4 ty .. 4 ty + 3 of the query tile, and
//   * of S = Q K^T the 4 x 4 block of those rows and keys 4 tx .. 4 tx + 3: an outer product per head-dimension
//     index from the transposed Q and K tiles in shared memory (two 16-byte loads for 16 FMAs);
//   * of O += P V the columns (tx + 16 g) VW + e of those rows: per four keys, four 16-byte loads of P and one
//     VW-wide load of V per column group;
//   * the row maxima by four shuffles per tile over the 16 threads of a row (not per key); the row sums stay
//     per-thread partials, rescaled with O, and are added across the 16 threads once at the end.
// The range minimum of phi that the bias needs inside the diagonal tile, min over (s, t] for key s <= row t, is
// tabulated once per CTA in shared memory (one thread per row walking its keys downwards).
//
// For D <= 128 a CTA holds two such groups of 256 threads that share the query tile and take alternate key tiles
// (group 0 the diagonal tile and every second tile below it, group 1 the others), each with its own K, V and P
// tiles, running maximum, row sums and output block; group 1 hands its state to group 0 through shared memory at the
// end, which joins the two as the key-range split of the tensor-core forward does. The longest chain of key tiles a
// CTA walks is then half the query tile's, which bounds the forward at small batches.
#include "fpa_simt_tile.cuh"

namespace fpa {
namespace {

using tile::kFT;
using tile::kFThreads;
using tile::kPitch;
using tile::ld_vec;
using tile::load_rows;
using tile::vec_ok;


template <int D>
struct FwdTile {
  static constexpr int CPT = D / 16;             // output columns per thread
  static constexpr int VW = CPT >= 4 ? 4 : CPT;  // width of a column group
  static constexpr int NG = CPT / VW;            // column groups: columns (tx + 16 g) * VW + e
  static constexpr int NGRP = D <= 128 ? 2 : 1;  // groups of 256 threads taking alternate key tiles
  // Per group: Kt [D][kPitch], Vs [kFT][D], Ps [kFT][kPitch] (also the diagonal tile's range minima), then the
  // per-key psi, SUF and phi of the group's current key tile.
  static constexpr size_t GROUP_FLOATS = size_t(D) * kPitch + size_t(kFT) * D + size_t(kFT) * kPitch + 3 * kFT;
  // Qt [D][kPitch], then the groups.
  static constexpr size_t SMEM = (size_t(D) * kPitch + NGRP * GROUP_FLOATS) * 4;
};

// Barrier of the 256 threads of group g (named barrier g + 1; barrier 0 is __syncthreads).
__device__ __forceinline__ void group_sync(int g) {
  asm volatile("bar.sync %0, %1;" ::"r"(g + 1), "n"(kFThreads) : "memory");
}

template <typename TIn, int D, bool VEC>
__global__ void __launch_bounds__(kFThreads * FwdTile<D>::NGRP)
simt_fwd_tiled_kernel(const TIn* __restrict__ q, Str4 sq, const TIn* __restrict__ k, Str4 sk,
                      const TIn* __restrict__ v, Str4 sv, const float* __restrict__ phi,
                      const float* __restrict__ psi, const float* __restrict__ beta, Stats st, TIn* __restrict__ o,
                      Str4 so, float* __restrict__ lse, int H, int T, int NB, float scale2) {
  using F = FwdTile<D>;
  constexpr int VW = F::VW, NG = F::NG, NGRP = F::NGRP;
  extern __shared__ float smem[];
  const int grp = NGRP > 1 ? int(threadIdx.x) / kFThreads : 0;
  float* Qt = smem;
  float* Kt = Qt + D * kPitch + grp * F::GROUP_FLOATS;
  float* Vs = Kt + D * kPitch;
  float* Ps = Vs + kFT * D;
  float* psis = Ps + kFT * kPitch;
  float* sufs = psis + kFT;
  float* phis = sufs + kFT;
  auto gsync = [&] {
    if constexpr (NGRP > 1)
      group_sync(grp);
    else
      __syncthreads();
  };

  // 1-D grid of NB * B * H CTAs, tile rank major: the longest query tiles of every head first (kernel.py:108 orders
  // a head's tiles the same way), so that the hardware's in-order dispatch approximates longest-first scheduling.
  const int BH = int(gridDim.x) / NB;
  const int i = NB - 1 - int(blockIdx.x) / BH;
  const int z = int(blockIdx.x) % BH, b = z / H, h = z % H;
  const int tid = int(threadIdx.x) % kFThreads, ty = tid >> 4, tx = tid & 15;  // index within the group
  const size_t TP = size_t(NB) * kFT, zt = size_t(z) * T, zp = size_t(z) * TP;
  const float betal = beta[h] * kLog2e;

  // Q tile, transposed and pre-scaled by D^-1/2 log2 e (rows >= T read as zero), loaded by group 0 and shared.
  if (grp == 0) load_rows<TIn, D, true, VEC>(Qt, q + b * sq.b + h * sq.h, sq, i, T, scale2, tid);
  float pre[4];  // PRE_t of the thread's rows
#pragma unroll
  for (int a = 0; a < 4; ++a) pre[a] = st.pre[zp + size_t(i) * kFT + ty * 4 + a];

  auto load_tile = [&](int j) {
    load_rows<TIn, D, true, VEC>(Kt, k + b * sk.b + h * sk.h, sk, j, T, 1.f, tid);
    load_rows<TIn, D, false, VEC>(Vs, v + b * sv.b + h * sv.h, sv, j, T, 1.f, tid);
    if (tid < kFT) {
      const int s = j * kFT + tid;
      psis[tid] = s < T ? psi[zt + s] : 0.f;
      sufs[tid] = st.suf[zp + s];
      phis[tid] = s < T ? phi[zt + s] : kInf;
    }
  };

  float m[4], l[4], acc[4][NG][VW];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    m[a] = -kInf;
    l[a] = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int e = 0; e < VW; ++e) acc[a][g][e] = 0.f;
  }

  // One key tile: S block, bias (diag: range minima from the table in Ps; else SUF, mid and PRE), online softmax,
  // P to shared memory, O += P V.
  auto step = [&](int j, bool diag, float mid) {
    float sc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) sc[a][c] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(Qt + d * kPitch + ty * 4);
      const float4 kc = *reinterpret_cast<const float4*>(Kt + d * kPitch + tx * 4);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kc.x, kc.y, kc.z, kc.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) sc[a][c] = fmaf(qv[a], kv[c], sc[a][c]);
    }
    float mx[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int r = ty * 4 + a;
      float rm[4];
      if (diag) ld_vec<4>(rm, Ps + r * kPitch + tx * 4);  // min phi over (key, row] (+inf on the diagonal)
      const float cap = fminf(mid, pre[a]);
      mx[a] = -kInf;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int s = tx * 4 + c;
        float x;
        bool ok = true;
        if (diag) {
          x = rm[c] - psis[s];
          ok = s <= r && j * kFT + s < T;
        } else {
          x = fminf(sufs[s], cap) - psis[s];
        }
        sc[a][c] = ok ? fmaf(betal, fminf(x, 0.f), sc[a][c]) : -kInf;
        mx[a] = fmaxf(mx[a], sc[a][c]);
      }
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1)
#pragma unroll
      for (int a = 0; a < 4; ++a) mx[a] = fmaxf(mx[a], __shfl_xor_sync(0xffffffffu, mx[a], off));
    gsync();  // the range-minimum table (diagonal) is read; Ps takes P next
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float mn = fmaxf(m[a], mx[a]);
      const float alpha = m[a] == -kInf ? 0.f : ex2(m[a] - mn);
      m[a] = mn;
      float p[4], ls = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        p[c] = ex2(sc[a][c] - mn);  // -inf -> 0
        ls += p[c];
      }
      l[a] = fmaf(l[a], alpha, ls);
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int e = 0; e < VW; ++e) acc[a][g][e] *= alpha;
      *reinterpret_cast<float4*>(Ps + (ty * 4 + a) * kPitch + tx * 4) = make_float4(p[0], p[1], p[2], p[3]);
    }
    gsync();
#pragma unroll 2
    for (int s0 = 0; s0 < kFT; s0 += 4) {
      float pr[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a) ld_vec<4>(pr[a], Ps + (ty * 4 + a) * kPitch + s0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          float vv[VW];
          ld_vec<VW>(vv, Vs + (s0 + c) * D + (tx + 16 * g) * VW);
#pragma unroll
          for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int e = 0; e < VW; ++e) acc[a][g][e] = fmaf(pr[a][c], vv[e], acc[a][g][e]);
        }
      }
    }
  };

  // Group 0 takes the diagonal tile first: the range-minimum table min over (s, t] of phi, one thread per row t
  // walking its keys s = t, t - 1, ..., 0 (the bias of kernel.py:130-132 inside the tile).
  if (grp == 0) load_tile(i);
  __syncthreads();  // Q (shared by the groups) and group 0's diagonal tile are loaded
  if (grp == 0) {
    if (tid < kFT) {
      float x = kInf;
      float* row = Ps + tid * kPitch;
      row[tid] = kInf;
      for (int s = tid - 1; s >= 0; --s) {
        x = fminf(x, phis[s + 1]);
        row[s] = x;
      }
    }
    gsync();
    step(i, true, kInf);
  }
  // Earlier key tiles, walking back from the diagonal with mid = min phi over the tiles passed (kernel.py:143-159);
  // with two groups, tile j belongs to group (i - j) mod 2.
  float mid = kInf;
  for (int j = i - 1; j >= 0; --j) {
    if (NGRP == 1 || ((i - j) & 1) == grp) {
      gsync();  // the previous tile's V and P are read
      load_tile(j);
      gsync();
      step(j, false, mid);
    }
    mid = fminf(mid, st.bmin[size_t(z) * NB + j]);
  }

  // Row sums across the 16 threads of a row (per-thread partials until here).
#pragma unroll
  for (int off = 1; off < 16; off <<= 1)
#pragma unroll
    for (int a = 0; a < 4; ++a) l[a] += __shfl_xor_sync(0xffffffffu, l[a], off);
  if constexpr (NGRP > 1) {
    // Group 1 hands m, l and its output block to the thread of group 0 with the same rows and columns (through its
    // own tiles' space, strided by thread so that the accesses are conflict-free); M = max(m0, m1),
    // l = l0 2^(m0 - M) + l1 2^(m1 - M), O = O0 2^(m0 - M) + O1 2^(m1 - M). A group without tiles has m = -inf.
    constexpr int NV = 8 + 4 * NG * VW;
    static_assert(size_t(NV) * kFThreads <= F::GROUP_FLOATS, "group 1's tiles hold its hand-over");
    float* xch = smem + D * kPitch + F::GROUP_FLOATS;
    __syncthreads();  // group 1's tiles are read
    if (grp == 1) {
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        xch[a * kFThreads + tid] = m[a];
        xch[(4 + a) * kFThreads + tid] = l[a];
#pragma unroll
        for (int g = 0; g < NG; ++g)
#pragma unroll
          for (int e = 0; e < VW; ++e) xch[(8 + (a * NG + g) * VW + e) * kFThreads + tid] = acc[a][g][e];
      }
    }
    __syncthreads();
    if (grp == 1) return;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float m1 = xch[a * kFThreads + tid], l1 = xch[(4 + a) * kFThreads + tid];
      const float mm = fmaxf(m[a], m1);
      const float s0 = m[a] == -kInf ? 0.f : ex2(m[a] - mm), s1 = m1 == -kInf ? 0.f : ex2(m1 - mm);
      m[a] = mm;
      l[a] = l[a] * s0 + l1 * s1;
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int e = 0; e < VW; ++e)
          acc[a][g][e] = acc[a][g][e] * s0 + xch[(8 + (a * NG + g) * VW + e) * kFThreads + tid] * s1;
    }
  }

  // o = O / l and lse = m + log2 l (base 2, as the tensor-core path).
  TIn* ob = o + b * so.b + h * so.h;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int t = i * kFT + ty * 4 + a;
    if (t >= T) continue;
    const float inv = 1.f / l[a];
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int e = 0; e < VW; ++e)
        ob[int64_t(t) * so.t + int64_t((tx + 16 * g) * VW + e) * so.d] = from_f32<TIn>(acc[a][g][e] * inv);
    if (tx == 0) lse[zt + t] = m[a] + lg2(l[a]);
  }
}

template <typename TIn, int D>
cudaError_t launch_tiled(const FpaFwdArgs& a, const Dims& d, const Stats& st, cudaStream_t s) {
  const bool vec = vec_ok<TIn>(a.q, a.q_stride) && vec_ok<TIn>(a.k, a.k_stride) && vec_ok<TIn>(a.v, a.v_stride);
  auto fn = vec ? simt_fwd_tiled_kernel<TIn, D, true> : simt_fwd_tiled_kernel<TIn, D, false>;
  const size_t smem = FwdTile<D>::SMEM;
  if (smem > 48 * 1024) {
    const cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(fn), int(smem));
    if (e != cudaSuccess) return e;
  }
  fn<<<dim3(d.NB * d.B * d.H), kFThreads * FwdTile<D>::NGRP, smem, s>>>(
      (const TIn*)a.q, str4(a.q_stride), (const TIn*)a.k, str4(a.k_stride), (const TIn*)a.v, str4(a.v_stride),
      a.phi, a.psi, a.beta, st, (TIn*)a.o, str4(a.o_stride), a.lse, d.H, d.T, d.NB,
      float(1.0 / sqrt(double(D))) * kLog2e);
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_tiled_d(const FpaFwdArgs& a, const Dims& d, const Stats& st, cudaStream_t s) {
  switch (d.D) {
    case 16: return launch_tiled<TIn, 16>(a, d, st, s);
    case 32: return launch_tiled<TIn, 32>(a, d, st, s);
    case 64: return launch_tiled<TIn, 64>(a, d, st, s);
    case 128: return launch_tiled<TIn, 128>(a, d, st, s);
    case 256: return launch_tiled<TIn, 256>(a, d, st, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t simt_fwd_tiled(const FpaFwdArgs& a, const Dims& d, const Stats& st, cudaStream_t s) {
  return a.dtype == FPA_DTYPE_F16 ? launch_tiled_d<__half>(a, d, st, s) : launch_tiled_d<float>(a, d, st, s);
}

}  // namespace fpa
