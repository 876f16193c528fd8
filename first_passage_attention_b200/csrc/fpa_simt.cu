// Row-per-thread-group FFMA backward kernels of the FPA operator, for D = 256, where the register-tiled backward
// (fpa_simt_bwd.cu) does not fit its four transposed tiles in shared memory: the fp32 path and fp16 at D = 256 (the
// forward of that path is fpa_simt_fwd.cu). Tiles of 64 positions; a group of TPR consecutive threads owns one query
// row (q-pass) or one key (kv-pass) and splits the head dimension between its lanes.
//
// The math follows the reference's tiled decomposition (kernel.py:178-265 kv-pass, 287-340 q-pass): for query t in
// tile i and key s in tile j < i the range (s, t] splits into (s, end of j], the tiles strictly between, and
// [start of i, t], so
//     min_{s<u<=t} phi_u = min(SUF_s, mid_ij, PRE_t),   Z_{s,t} = 2^{SUFL_s} + 2^{MIDL_ij} + 2^{PREL_t}.
// Inside the diagonal tile the range minimum is carried as a running minimum along the row.
#include "fpa_internal.h"

namespace fpa {

template <int D>
struct SimtShape {
  static constexpr int BT = kSimtBT;
  static constexpr int TPR = (D >= 64) ? D / 16 : 4;  // threads per row / key
  static constexpr int CPT = D / TPR;                 // head-dim columns per thread
  static constexpr int THREADS = BT * TPR;
};

template <typename TIn>
__device__ __forceinline__ void load_row(float* dst, const TIn* src, int64_t stride_d, int c0, int n, bool ok) {
#pragma unroll
  for (int c = 0; c < n; ++c) dst[c] = ok ? to_f32(src[int64_t(c0 + c) * stride_d]) : 0.f;
}

// Loads rows [j*BT, j*BT+BT) of a [.., T, D] operand into shared memory as float32 (zero beyond T).
template <typename TIn, int D, int THREADS>
__device__ __forceinline__ void load_tile(float* dst, const TIn* base, Str4 st, int j, int T) {
  constexpr int BT = kSimtBT;
  for (int e = threadIdx.x; e < BT * D; e += THREADS) {
    int r = e / D, c = e % D, t = j * BT + r;
    dst[e] = t < T ? to_f32(base[int64_t(t) * st.t + int64_t(c) * st.d]) : 0.f;
  }
}

// ------------------------------------------------------------------------------------------------ kv-pass ----
// Per key tile j: dK, dV, dpsi, the dbeta partial, the soft-min sums W (u in the key's tile) and TB (u strictly
// between the tiles), and the complete in-tile soft-min gradient DPHI4 of the diagonal tile.
template <typename TIn, int D>
__global__ void __launch_bounds__(SimtShape<D>::THREADS)
simt_bwd_kv_kernel(const TIn* __restrict__ q, Str4 sq, const TIn* __restrict__ k, Str4 sk,
                   const TIn* __restrict__ v, Str4 sv, const TIn* __restrict__ dout, Str4 sdo,
                   const float* __restrict__ lse, const float* __restrict__ phi, const float* __restrict__ psi,
                   const float* __restrict__ beta, Stats st, BwdScratch sc, TIn* __restrict__ dk, Str4 sdk,
                   TIn* __restrict__ dv, Str4 sdv, float* __restrict__ dpsi, int H, int T, int NB, float scale,
                   float il2) {
  using S = SimtShape<D>;
  constexpr int BT = S::BT, TPR = S::TPR, CPT = S::CPT, LD = BT + 1;
  extern __shared__ float smem[];
  float* Qs = smem;
  float* DOs = Qs + BT * D;
  float* lses = DOs + BT * D;
  float* dels = lses + BT;
  float* pres = dels + BT;
  float* prels = pres + BT;
  float* phis = prels + BT;
  float* Gd = phis + BT;   // [BT][BT+1]  g of the diagonal tile, then its soft-min contributions
  float* Ls = Gd + BT * LD;  // [BT][BT+1]  log2 partial sums inside the diagonal tile
  float* red = Ls + BT * LD; // [32]

  const int j = blockIdx.x;  // key tile 0 has the most query tiles: launched first
  const int z = blockIdx.z * gridDim.y + blockIdx.y, b = z / H, h = z % H;  // grid (NB, H, B)
  const int sl = threadIdx.x / TPR, sub = threadIdx.x % TPR, c0 = sub * CPT;
  const int s = j * BT + sl;
  const bool s_ok = s < T;
  const size_t TP = size_t(NB) * BT;
  const float bh = beta[h], betal = bh * kLog2e, scale2 = scale * kLog2e;

  float kr[CPT], vr[CPT], dkr[CPT], dvr[CPT];
  load_row(kr, k + b * sk.b + h * sk.h + int64_t(s_ok ? s : 0) * sk.t, sk.d, c0, CPT, s_ok);
  load_row(vr, v + b * sv.b + h * sv.h + int64_t(s_ok ? s : 0) * sv.t, sv.d, c0, CPT, s_ok);
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    kr[c] *= scale2;
    dkr[c] = 0.f;
    dvr[c] = 0.f;
  }
  const float psi_s = s_ok ? psi[size_t(z) * T + s] : 0.f;
  const float suf_s = st.suf[size_t(z) * TP + s];
  const float sufl_s = st.sufl[size_t(z) * TP + s];
  const float c2_s = suf_s < kInf ? -suf_s * il2 : -kInf;
  float gsum = 0.f, dbsum = 0.f, wsum = 0.f;
  float mid = kInf, midl = -kInf;

  for (int i = j; i < NB; ++i) {
    __syncthreads();
    load_tile<TIn, D, S::THREADS>(Qs, q + b * sq.b + h * sq.h, sq, i, T);
    load_tile<TIn, D, S::THREADS>(DOs, dout + b * sdo.b + h * sdo.h, sdo, i, T);
    for (int r = threadIdx.x; r < BT; r += S::THREADS) {
      int t = i * BT + r;
      bool ok = t < T;
      lses[r] = ok ? lse[size_t(z) * T + t] : 0.f;
      dels[r] = ok ? sc.delta[size_t(z) * TP + t] : 0.f;
      pres[r] = st.pre[size_t(z) * TP + t];
      prels[r] = st.prel[size_t(z) * TP + t];
      phis[r] = ok ? phi[size_t(z) * T + t] : kInf;
    }
    __syncthreads();
    if (i == j) {
      float rmin = kInf;
      for (int tl = 0; tl < BT; ++tl) {
        const int t = i * BT + tl;
        const float* qrow = Qs + tl * D + c0;
        const float* drow = DOs + tl * D + c0;
        float dot = 0.f, dpd = 0.f;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          dot = fmaf(kr[c], qrow[c], dot);
          dpd = fmaf(vr[c], drow[c], dpd);
        }
        dot = group_sum<TPR>(dot);
        dpd = group_sum<TPR>(dpd);
        if (tl > sl) rmin = fminf(rmin, phis[tl]);
        const float x = rmin - psi_s;  // +inf on and above the diagonal
        const float xm = fminf(x, 0.f);
        const bool valid = (tl >= sl) && (t < T) && s_ok;
        const float p = valid ? ex2(dot + betal * xm - lses[tl]) : 0.f;
        const float ds = p * (dpd - dels[tl]);
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          dvr[c] = fmaf(p, drow[c], dvr[c]);
          dkr[c] = fmaf(ds, qrow[c], dkr[c]);
        }
        const bool strict = valid && (tl > sl);
        const float g = (strict && x <= 0.f) ? ds : 0.f;
        gsum += g;
        dbsum += strict ? ds * xm : 0.f;
        if (sub == 0) Gd[sl * LD + tl] = g;
      }
      __syncthreads();
      // In-tile soft-min gradient (kernel.py:269-283 computes the same sums with scans): for key s,
      //   H(t) = g_ts + (Z_{s,t}/Z_{s,t+1}) H(t+1),  contribution to u = t: (2^{a2_t}/Z_{s,t}) H(t),
      // with Z_{s,t} = sum_{s<u<=t} 2^{a2_u} carried as L = log2 Z. Every factor lies in [0, 1].
      const int tend = min(BT, T - i * BT);
      if (sub == 0) {
        float L = -kInf;
        for (int tl = sl + 1; tl < tend; ++tl) {
          L = lse2(L, -phis[tl] * il2);
          Ls[sl * LD + tl] = L;
        }
        float Hh = 0.f;
        for (int tl = tend - 1; tl > sl; --tl) {
          if (tl < tend - 1) Hh *= ex2(Ls[sl * LD + tl] - Ls[sl * LD + tl + 1]);
          Hh += Gd[sl * LD + tl];
          Gd[sl * LD + tl] = ex2(-phis[tl] * il2 - Ls[sl * LD + tl]) * Hh;
        }
      }
      __syncthreads();
      if (sub == 0 && sl < tend) {
        float a4 = 0.f;
        for (int s2 = 0; s2 < sl; ++s2) a4 += Gd[s2 * LD + sl];
        sc.dphi4[size_t(z) * TP + i * BT + sl] = a4;
      }
    } else {
      const float cmid2 = mid < kInf ? -mid * il2 : -kInf;
      float rs = fmaxf(c2_s, cmid2);
      const bool vrs = rs > -kInf;
      rs = vrs ? rs : 0.f;
      const float sv_ = ex2(sufl_s - rs) + ex2(midl - rs);
      const float cap = fminf(suf_s, mid);
      float fsum = 0.f;
      for (int tl = 0; tl < BT; ++tl) {
        const int t = i * BT + tl;
        const float* qrow = Qs + tl * D + c0;
        const float* drow = DOs + tl * D + c0;
        float dot = 0.f, dpd = 0.f;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          dot = fmaf(kr[c], qrow[c], dot);
          dpd = fmaf(vr[c], drow[c], dpd);
        }
        dot = group_sum<TPR>(dot);
        dpd = group_sum<TPR>(dpd);
        const float x = fminf(cap, pres[tl]) - psi_s;
        const float xm = fminf(x, 0.f);
        const bool valid = (t < T) && s_ok;
        const float p = valid ? ex2(dot + betal * xm - lses[tl]) : 0.f;
        const float ds = p * (dpd - dels[tl]);
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          dvr[c] = fmaf(p, drow[c], dvr[c]);
          dkr[c] = fmaf(ds, qrow[c], dkr[c]);
        }
        const float g = (valid && x <= 0.f) ? ds : 0.f;
        gsum += g;
        dbsum += valid ? ds * xm : 0.f;
        fsum += g / (sv_ + ex2(prels[tl] - rs));
      }
      if (vrs) wsum += ex2(c2_s - rs) * fsum;
      if (i > j + 1) {
        float tp = (vrs && sub == 0) ? ex2(cmid2 - rs) * fsum : 0.f;
        tp = group_sum<32>(tp);
        const int warp = threadIdx.x >> 5, nw = S::THREADS >> 5;
        if ((threadIdx.x & 31) == 0) red[warp] = tp;
        __syncthreads();
        if (threadIdx.x == 0) {
          float tot = 0.f;
          for (int w = 0; w < nw; ++w) tot += red[w];
          sc.tb[((size_t(z) * NB + i) * NB + j) * sc.tb_parts] = tot;
        }
      }
      mid = fminf(mid, st.bmin[size_t(z) * NB + i]);
      midl = lse2(midl, st.bl[size_t(z) * NB + i]);
    }
  }
  if (s_ok) {
    TIn* dkrow = dk + b * sdk.b + h * sdk.h + int64_t(s) * sdk.t;
    TIn* dvrow = dv + b * sdv.b + h * sdv.h + int64_t(s) * sdv.t;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      dkrow[int64_t(c0 + c) * sdk.d] = from_f32<TIn>(dkr[c] * scale);
      dvrow[int64_t(c0 + c) * sdv.d] = from_f32<TIn>(dvr[c]);
    }
    if (sub == 0) {
      dpsi[size_t(z) * T + s] = -bh * gsum;
      sc.w[size_t(z) * TP + s] = wsum;
    }
  }
  // dbeta partial of this key tile, reduced in a fixed order.
  __syncthreads();
  float db = (sub == 0) ? dbsum : 0.f;
  db = group_sum<32>(db);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = db;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (S::THREADS >> 5); ++w) tot += red[w];
    sc.dbeta[size_t(z) * NB + j] = tot;
  }
}

// ------------------------------------------------------------------------------------------------- q-pass ----
// Per query tile i: dQ and the soft-min contribution of u in the query's own tile (DPHI2), from
//   r_t = sum_{s in earlier tiles} g_ts 2^{c_t} / Z_{s,t},  DPHI2_u = sum_{t>=u in tile} 2^{a2_u - c_t} r_t.
template <typename TIn, int D>
__global__ void __launch_bounds__(SimtShape<D>::THREADS)
simt_bwd_q_kernel(const TIn* __restrict__ q, Str4 sq, const TIn* __restrict__ k, Str4 sk,
                  const TIn* __restrict__ v, Str4 sv, const TIn* __restrict__ dout, Str4 sdo,
                  const float* __restrict__ lse, const float* __restrict__ phi, const float* __restrict__ psi,
                  const float* __restrict__ beta, Stats st, BwdScratch sc, TIn* __restrict__ dq, Str4 sdq, int H,
                  int T, int NB, float scale, float il2) {
  using S = SimtShape<D>;
  constexpr int BT = S::BT, TPR = S::TPR, CPT = S::CPT;
  extern __shared__ float smem[];
  float* Ks = smem;
  float* Vs = Ks + BT * D;
  float* psis = Vs + BT * D;
  float* phis = psis + BT;
  float* sufs = phis + BT;
  float* sufls = sufs + BT;
  float* rr = sufls + BT;
  float* c2t = rr + BT;

  const int i = NB - 1 - blockIdx.x;
  const int z = blockIdx.z * gridDim.y + blockIdx.y, b = z / H, h = z % H;  // grid (NB, H, B)
  const int tl = threadIdx.x / TPR, sub = threadIdx.x % TPR, c0 = sub * CPT;
  const int t = i * BT + tl;
  const bool t_ok = t < T;
  const size_t TP = size_t(NB) * BT;
  const float betal = beta[h] * kLog2e, scale2 = scale * kLog2e;

  float qr[CPT], dor[CPT], dqr[CPT];
  load_row(qr, q + b * sq.b + h * sq.h + int64_t(t_ok ? t : 0) * sq.t, sq.d, c0, CPT, t_ok);
  load_row(dor, dout + b * sdo.b + h * sdo.h + int64_t(t_ok ? t : 0) * sdo.t, sdo.d, c0, CPT, t_ok);
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    qr[c] *= scale2;
    dqr[c] = 0.f;
  }
  const float lse_t = t_ok ? lse[size_t(z) * T + t] : 0.f;
  const float del_t = t_ok ? sc.delta[size_t(z) * TP + t] : 0.f;
  const float pre_t = st.pre[size_t(z) * TP + t];
  const float prel_t = st.prel[size_t(z) * TP + t];
  const float c2_t = t_ok ? -pre_t * il2 : 0.f;
  const float bpre = t_ok ? ex2(prel_t - c2_t) : 1.f;
  float racc = 0.f;

  auto tile_in = [&](int j) {
    const size_t zb = size_t(z) * T;
    load_tile<TIn, D, S::THREADS>(Ks, k + b * sk.b + h * sk.h, sk, j, T);
    load_tile<TIn, D, S::THREADS>(Vs, v + b * sv.b + h * sv.h, sv, j, T);
    for (int r = threadIdx.x; r < BT; r += S::THREADS) {
      int s = j * BT + r;
      psis[r] = s < T ? psi[zb + s] : 0.f;
      phis[r] = s < T ? phi[zb + s] : kInf;
      sufs[r] = st.suf[size_t(z) * TP + s];
      sufls[r] = st.sufl[size_t(z) * TP + s];
    }
  };
  tile_in(i);
  __syncthreads();
  float rmin = kInf;
  for (int sl = BT - 1; sl >= 0; --sl) {
    const float* krow = Ks + sl * D + c0;
    const float* vrow = Vs + sl * D + c0;
    float dot = 0.f, dpd = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      dot = fmaf(qr[c], krow[c], dot);
      dpd = fmaf(dor[c], vrow[c], dpd);
    }
    dot = group_sum<TPR>(dot);
    dpd = group_sum<TPR>(dpd);
    const bool ok = (sl <= tl) && (i * BT + sl < T) && t_ok;
    const float x = rmin - psis[sl];
    const float p = ok ? ex2(dot + betal * fminf(x, 0.f) - lse_t) : 0.f;
    const float ds = p * (dpd - del_t);
#pragma unroll
    for (int c = 0; c < CPT; ++c) dqr[c] = fmaf(ds, krow[c], dqr[c]);
    if (sl <= tl) rmin = fminf(rmin, phis[sl]);
  }
  float mid = kInf, midl = -kInf;
  for (int j = i - 1; j >= 0; --j) {
    __syncthreads();
    tile_in(j);
    __syncthreads();
    const float mterm = ex2(midl - c2_t) + bpre;
    const float cap = fminf(mid, pre_t);
    for (int sl = 0; sl < BT; ++sl) {
      const float* krow = Ks + sl * D + c0;
      const float* vrow = Vs + sl * D + c0;
      float dot = 0.f, dpd = 0.f;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        dot = fmaf(qr[c], krow[c], dot);
        dpd = fmaf(dor[c], vrow[c], dpd);
      }
      dot = group_sum<TPR>(dot);
      dpd = group_sum<TPR>(dpd);
      const float x = fminf(sufs[sl], cap) - psis[sl];
      const float p = t_ok ? ex2(dot + betal * fminf(x, 0.f) - lse_t) : 0.f;
      const float ds = p * (dpd - del_t);
#pragma unroll
      for (int c = 0; c < CPT; ++c) dqr[c] = fmaf(ds, krow[c], dqr[c]);
      const float g = (t_ok && x <= 0.f) ? ds : 0.f;
      racc += g / (ex2(sufls[sl] - c2_t) + mterm);
    }
    mid = fminf(mid, st.bmin[size_t(z) * NB + j]);
    midl = lse2(midl, st.bl[size_t(z) * NB + j]);
  }
  if (t_ok) {
    TIn* row = dq + b * sdq.b + h * sdq.h + int64_t(t) * sdq.t;
#pragma unroll
    for (int c = 0; c < CPT; ++c) row[int64_t(c0 + c) * sdq.d] = from_f32<TIn>(dqr[c] * scale);
  }
  __syncthreads();
  if (sub == 0) {
    rr[tl] = racc;
    c2t[tl] = c2_t;
    phis[tl] = t_ok ? phi[size_t(z) * T + t] : kInf;  // the query tile's own field
  }
  __syncthreads();
  if (sub == 0 && t_ok) {
    const int tend = min(BT, T - i * BT);
    const float a2 = -phis[tl] * il2;
    float p2 = 0.f;
    for (int t2 = tl; t2 < tend; ++t2) p2 += ex2(a2 - c2t[t2]) * rr[t2];
    sc.dphi2[size_t(z) * TP + t] = p2;
  }
}

// ------------------------------------------------------------------------------------------------ launchers --
template <int D>
static size_t kv_smem() {
  return (2 * size_t(kSimtBT) * D + 5 * kSimtBT + 2 * size_t(kSimtBT) * (kSimtBT + 1) + 32) * sizeof(float);
}
template <int D>
static size_t q_smem() { return (2 * size_t(kSimtBT) * D + 6 * kSimtBT) * sizeof(float); }

template <typename F>
static cudaError_t allow_smem(F* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  return allow_dynamic_smem(reinterpret_cast<const void*>(fn), int(bytes));
}

template <typename TIn, int D>
static cudaError_t simt_kv_t(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc,
                             cudaStream_t s) {
  auto fn = simt_bwd_kv_kernel<TIn, D>;
  size_t smem = kv_smem<D>();
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  fn<<<dim3(d.NB, d.H, d.B), SimtShape<D>::THREADS, smem, s>>>(
      (const TIn*)a.q, str4(a.q_stride), (const TIn*)a.k, str4(a.k_stride), (const TIn*)a.v, str4(a.v_stride),
      (const TIn*)a.dout, str4(a.dout_stride), a.lse, a.phi, a.psi, a.beta, st, sc, (TIn*)a.dk, str4(a.dk_stride),
      (TIn*)a.dv, str4(a.dv_stride), a.dpsi, d.H, d.T, d.NB, float(1.0 / sqrt(double(D))), kLog2e / a.tau);
  return cudaGetLastError();
}

template <typename TIn, int D>
static cudaError_t simt_q_t(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc,
                            cudaStream_t s) {
  auto fn = simt_bwd_q_kernel<TIn, D>;
  size_t smem = q_smem<D>();
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  fn<<<dim3(d.NB, d.H, d.B), SimtShape<D>::THREADS, smem, s>>>(
      (const TIn*)a.q, str4(a.q_stride), (const TIn*)a.k, str4(a.k_stride), (const TIn*)a.v, str4(a.v_stride),
      (const TIn*)a.dout, str4(a.dout_stride), a.lse, a.phi, a.psi, a.beta, st, sc, (TIn*)a.dq, str4(a.dq_stride),
      d.H, d.T, d.NB, float(1.0 / sqrt(double(D))), kLog2e / a.tau);
  return cudaGetLastError();
}

template <int D>
static cudaError_t kv_f16(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc,
                          cudaStream_t s) {
  return simt_kv_t<__half, D>(a, d, st, sc, s);
}
template <int D>
static cudaError_t kv_f32(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc,
                          cudaStream_t s) {
  return simt_kv_t<float, D>(a, d, st, sc, s);
}
template <int D>
static cudaError_t q_f16(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s) {
  return simt_q_t<__half, D>(a, d, st, sc, s);
}
template <int D>
static cudaError_t q_f32(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s) {
  return simt_q_t<float, D>(a, d, st, sc, s);
}

cudaError_t simt_bwd_kv(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s) {
  if (d.D != 256) return cudaErrorInvalidValue;
  return a.dtype == FPA_DTYPE_F16 ? kv_f16<256>(a, d, st, sc, s) : kv_f32<256>(a, d, st, sc, s);
}

cudaError_t simt_bwd_q(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s) {
  if (d.D != 256) return cudaErrorInvalidValue;
  return a.dtype == FPA_DTYPE_F16 ? q_f16<256>(a, d, st, sc, s) : q_f32<256>(a, d, st, sc, s);
}

}  // namespace fpa
