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
  // Qt [D][kPitch], Kt [D][kPitch], Vs [kFT][D], Ps [kFT][kPitch] (also the diagonal tile's range minima), then the
  // per-key psi, SUF and phi of the current key tile.
  static constexpr size_t SMEM = (2 * size_t(D) * kPitch + size_t(kFT) * D + size_t(kFT) * kPitch + 3 * kFT) * 4;
};

template <typename TIn, int D, bool VEC>
__global__ void __launch_bounds__(kFThreads)
simt_fwd_tiled_kernel(const TIn* __restrict__ q, Str4 sq, const TIn* __restrict__ k, Str4 sk,
                      const TIn* __restrict__ v, Str4 sv, const float* __restrict__ phi,
                      const float* __restrict__ psi, const float* __restrict__ beta, Stats st, TIn* __restrict__ o,
                      Str4 so, float* __restrict__ lse, int H, int T, int NB, float scale2) {
  using F = FwdTile<D>;
  constexpr int VW = F::VW, NG = F::NG;
  extern __shared__ float smem[];
  float* Qt = smem;
  float* Kt = Qt + D * kPitch;
  float* Vs = Kt + D * kPitch;
  float* Ps = Vs + kFT * D;
  float* psis = Ps + kFT * kPitch;
  float* sufs = psis + kFT;
  float* phis = sufs + kFT;

  // 1-D grid of NB * B * H CTAs, tile rank major: the longest query tiles of every head first (kernel.py:108 orders
  // a head's tiles the same way), so that the hardware's in-order dispatch approximates longest-first scheduling.
  const int BH = int(gridDim.x) / NB;
  const int i = NB - 1 - int(blockIdx.x) / BH;
  const int z = int(blockIdx.x) % BH, b = z / H, h = z % H;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const size_t TP = size_t(NB) * kFT, zt = size_t(z) * T, zp = size_t(z) * TP;
  const float betal = beta[h] * kLog2e;

  // Q tile, transposed and pre-scaled by D^-1/2 log2 e (rows >= T read as zero).
  load_rows<TIn, D, true, VEC>(Qt, q + b * sq.b + h * sq.h, sq, i, T, scale2);
  float pre[4];  // PRE_t of the thread's rows
#pragma unroll
  for (int a = 0; a < 4; ++a) pre[a] = st.pre[zp + size_t(i) * kFT + ty * 4 + a];

  auto load_tile = [&](int j) {
    load_rows<TIn, D, true, VEC>(Kt, k + b * sk.b + h * sk.h, sk, j, T, 1.f);
    load_rows<TIn, D, false, VEC>(Vs, v + b * sv.b + h * sv.h, sv, j, T, 1.f);
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
    __syncthreads();  // the range-minimum table (diagonal) is read; Ps takes P next
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
    __syncthreads();
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

  // Diagonal tile first: the range-minimum table min over (s, t] of phi, one thread per row t walking its keys
  // s = t, t - 1, ..., 0 (the bias of kernel.py:130-132 inside the tile).
  load_tile(i);
  __syncthreads();
  if (tid < kFT) {
    float x = kInf;
    float* row = Ps + tid * kPitch;
    row[tid] = kInf;
    for (int s = tid - 1; s >= 0; --s) {
      x = fminf(x, phis[s + 1]);
      row[s] = x;
    }
  }
  __syncthreads();
  step(i, true, kInf);
  // Earlier key tiles, walking back from the diagonal with mid = min phi over the tiles passed (kernel.py:143-159).
  float mid = kInf;
  for (int j = i - 1; j >= 0; --j) {
    __syncthreads();  // the previous tile's V and P are read
    load_tile(j);
    __syncthreads();
    step(j, false, mid);
    mid = fminf(mid, st.bmin[size_t(z) * NB + j]);
  }

  // Row sums across the 16 threads of a row, then o = O / l and lse = m + log2 l (base 2, as the tensor-core path).
#pragma unroll
  for (int off = 1; off < 16; off <<= 1)
#pragma unroll
    for (int a = 0; a < 4; ++a) l[a] += __shfl_xor_sync(0xffffffffu, l[a], off);
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
  fn<<<dim3(d.NB * d.B * d.H), kFThreads, smem, s>>>(
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
