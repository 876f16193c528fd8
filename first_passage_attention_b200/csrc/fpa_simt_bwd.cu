// Register-tiled FFMA backward of the FPA operator: the fp32 path, fp16 with D = 256 (which the tensor-core kernels
// do not cover) and fp16 wherever the FFMA path is asked for. One launch runs both passes of the reference's backward
// (kernel.py:178-265 kv-pass, 287-340 q-pass) as interleaved CTAs of a 1-D grid, tile rank major over all heads: kv-pass
// CTAs of key tiles 0, 1, ... alternate with q-pass CTAs of query tiles NB - 1, NB - 2, ..., so that the hardware's
// in-order dispatch starts the longest tiles of every head first and the tails of the two passes overlap.
//
// Work split (256 threads as 16 x 16, tiles of 64 positions): thread (ty, tx) owns
//   * of the score tiles (S^T, dP^T in the kv-pass, S, dP in the q-pass) the 4 x 4 block of rows 4 ty .. 4 ty + 3
//     and columns 4 tx .. 4 tx + 3: an outer product per head-dimension index from the transposed tiles in shared
//     memory (four 16-byte loads for 32 FMAs);
//   * of the gradient accumulators (dK and dV of its four keys, or dQ of its four queries) the columns tx + 16 g:
//     per four positions, one 16-byte load of each score row and one of the transposed operand's row per column.
// The CTA's own tile pair (K, V in the kv-pass; Q, dO in the q-pass) stays in shared memory, transposed; the other
// pair streams through it. For D <= 128 the streamed pair is one stage of all D columns. For D = 256 (four
// transposed 64 x 256 fp32 tiles would need 278 KB) it streams in stages of 64 columns, and two CTAs share each tile
// and pass: both compute the score tiles, each keeps the accumulators of one half of the columns (128 registers of
// dK and dV per thread otherwise), and the first also writes the per-key or per-query results.
// The field math is the one of the reference's tiled decomposition: off the diagonal tile the bias uses
// min(SUF_s, mid, PRE_t) and the soft-min sums Z = 2^SUFL + 2^MIDL + 2^PREL; inside it the range minimum over (s, t]
// comes from a table built once per CTA, and the kv-pass runs the in-tile soft-min recurrence (kernel.py:269-283)
// on the g values it leaves in shared memory.
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
struct BwdTile {
  static constexpr int NH = D <= 128 ? 1 : 2;   // CTAs per tile and pass (column halves of the accumulators)
  static constexpr int NC = D / NH;             // accumulator columns of a CTA
  static constexpr int CPT = NC / 16;           // accumulator columns per thread (tx + 16 g)
  static constexpr int DC = D <= 128 ? D : 64;  // columns of the streamed tile pair per shared-memory stage
  static constexpr int NCH = D / DC;            // stages of the score contraction
  // kv-pass: Kt, Vt [D][kPitch]; Qt, Dt [DC][kPitch]; Ps, Ds [kFT][kPitch]; per query lse, delta, PRE, PREL, phi;
  // per key psi; eight per-warp partial sums.
  static constexpr size_t KV_FLOATS =
      2 * size_t(D) * kPitch + 2 * size_t(DC) * kPitch + 2 * size_t(kFT) * kPitch + 6 * kFT + 8;
  // q-pass: Qt, Dt [D][kPitch]; Kt, Vt [DC][kPitch]; Ss [kFT][kPitch]; per key psi, phi, SUF, SUFL; per query r,
  // c2, phi.
  static constexpr size_t Q_FLOATS =
      2 * size_t(D) * kPitch + 2 * size_t(DC) * kPitch + size_t(kFT) * kPitch + 7 * kFT;
  static constexpr size_t SMEM = (KV_FLOATS > Q_FLOATS ? KV_FLOATS : Q_FLOATS) * 4;
};

struct BwdTiledArgs {
  const void *q, *k, *v, *dout;
  Str4 sq, sk, sv, sdo;
  const float *lse, *phi, *psi, *beta;
  void *dq, *dk, *dv;
  Str4 sdq, sdk, sdv;
  float* dpsi;
  int H, T, NB;
  float scale, il2;
};

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Adds x over the 16 threads of a row group (tx = lane & 15).
__device__ __forceinline__ float row16_sum(float x) {
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// Adds to the 4 x 4 blocks A = X Y^T and B = U W^T the contraction over DC head-dimension indices; X, U rows
// 4 ty .., Y, W rows 4 tx .., all four operands transposed ([DC][kPitch]) in shared memory.
template <int DC>
__device__ __forceinline__ void score_blocks(float (&A)[4][4], float (&Bm)[4][4], const float* Xt, const float* Yt,
                                             const float* Ut, const float* Wt, int ty, int tx) {
#pragma unroll 4
  for (int d = 0; d < DC; ++d) {
    const float4 x = lds4(Xt + d * kPitch + ty * 4), y = lds4(Yt + d * kPitch + tx * 4);
    const float4 u = lds4(Ut + d * kPitch + ty * 4), w = lds4(Wt + d * kPitch + tx * 4);
    const float xv[4] = {x.x, x.y, x.z, x.w}, yv[4] = {y.x, y.y, y.z, y.w};
    const float uv[4] = {u.x, u.y, u.z, u.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        A[a][c] = fmaf(xv[a], yv[c], A[a][c]);
        Bm[a][c] = fmaf(uv[a], wv[c], Bm[a][c]);
      }
  }
}

// ------------------------------------------------------------------------------------------------ kv-pass ----
// Key tile j: dK, dV, dpsi, the dbeta partial, the soft-min sums W (u in the key's tile) and TB (u strictly between
// the tiles, one partial per warp), and the in-tile soft-min gradient DPHI4 of the diagonal tile; the columns
// half * NC .. of dK and dV (the per-key results from half 0 only).
template <typename TIn, int D, bool VEC>
__device__ __forceinline__ void kv_pass(const BwdTiledArgs& A, const Stats& st, const BwdScratch& sc, float* smem,
                                        int j, int z, int half) {
  using BT = BwdTile<D>;
  constexpr int CPT = BT::CPT, DC = BT::DC, NCH = BT::NCH;
  float* Kt = smem;
  float* Vt = Kt + D * kPitch;
  float* Qt = Vt + D * kPitch;  // one stage of DC columns of the query tile's Q and dO
  float* Dt = Qt + DC * kPitch;
  float* Ps = Dt + DC * kPitch;  // P^T [key][query]; the range-minimum table before, log2 Z of the recurrence after
  float* Ds = Ps + kFT * kPitch;  // dS^T [key][query]; g and then the recurrence's contributions on the diagonal
  float* lses = Ds + kFT * kPitch;
  float* dels = lses + kFT;
  float* pres = dels + kFT;
  float* prels = pres + kFT;
  float* phis = prels + kFT;
  float* psik = phis + kFT;
  float* red = psik + kFT;

  const int H = A.H, T = A.T, NB = A.NB, b = z / H, h = z % H;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15, warp = tid >> 5;
  const size_t TP = size_t(NB) * kFT, zt = size_t(z) * T, zp = size_t(z) * TP;
  const float bh = A.beta[h], betal = bh * kLog2e, il2 = A.il2;
  const TIn* q = static_cast<const TIn*>(A.q) + b * A.sq.b + h * A.sq.h;
  const TIn* dout = static_cast<const TIn*>(A.dout) + b * A.sdo.b + h * A.sdo.h;

  // The key tile, transposed; K pre-scaled by D^-1/2 log2 e so that S^T comes out in base-2 logits.
  load_rows<TIn, D, true, VEC>(Kt, static_cast<const TIn*>(A.k) + b * A.sk.b + h * A.sk.h, A.sk, j, T,
                               A.scale * kLog2e);
  load_rows<TIn, D, true, VEC>(Vt, static_cast<const TIn*>(A.v) + b * A.sv.b + h * A.sv.h, A.sv, j, T, 1.f);
  if (tid < kFT) psik[tid] = j * kFT + tid < T ? A.psi[zt + j * kFT + tid] : 0.f;

  float psi_s[4], suf_s[4], sufl_s[4], c2_s[4], gsum[4], wsum[4];
  bool s_ok[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int s = j * kFT + ty * 4 + a;
    s_ok[a] = s < T;
    psi_s[a] = s_ok[a] ? A.psi[zt + s] : 0.f;
    suf_s[a] = st.suf[zp + s];
    sufl_s[a] = st.sufl[zp + s];
    c2_s[a] = suf_s[a] < kInf ? -suf_s[a] * il2 : -kInf;
    gsum[a] = wsum[a] = 0.f;
  }
  float dbsum = 0.f, mid = kInf, midl = -kInf;
  float dka[4][CPT], dva[4][CPT];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int g = 0; g < CPT; ++g) dka[a][g] = dva[a][g] = 0.f;

  // Stages of Q and dO in the order (first + 1, ..., first): the score contraction ends on the stage holding the
  // first DC of this CTA's accumulator columns, which the dK / dV update then starts from without a reload.
  const int first = half * (NCH / BT::NH);
  auto load_stage = [&](int i, int c) {
    load_rows<TIn, DC, true, VEC>(Qt, q + int64_t(c) * DC * A.sq.d, A.sq, i, T, 1.f);
    load_rows<TIn, DC, true, VEC>(Dt, dout + int64_t(c) * DC * A.sdo.d, A.sdo, i, T, 1.f);
  };

  for (int i = j; i < NB; ++i) {
    const bool diag = i == j;
    float sS[4][4], sP[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) sS[a][c] = sP[a][c] = 0.f;
#pragma unroll 1
    for (int k = 0; k < NCH; ++k) {
      const int c = (first + 1 + k) % NCH;
      __syncthreads();  // the previous stage (and, at k = 0, the previous query tile's Ps and Ds) are read
      load_stage(i, c);
      if (k == 0 && tid < kFT) {
        const int t = i * kFT + tid;
        const bool ok = t < T;
        lses[tid] = ok ? A.lse[zt + t] : 0.f;
        dels[tid] = ok ? sc.delta[zp + t] : 0.f;
        pres[tid] = st.pre[zp + t];
        prels[tid] = st.prel[zp + t];
        phis[tid] = ok ? A.phi[zt + t] : kInf;
      }
      __syncthreads();
      if (k == 0 && diag) {
        // Range-minimum table of the diagonal tile: Ps[s][t] = min phi over (s, t] for t > s, one thread per key.
        if (tid < kFT) {
          float x = kInf;
          float* row = Ps + tid * kPitch;
          for (int t = tid + 1; t < kFT; ++t) {
            x = fminf(x, phis[t]);
            row[t] = x;
          }
        }
        __syncthreads();
      }
      score_blocks<DC>(sS, sP, Kt + c * DC * kPitch, Qt, Vt + c * DC * kPitch, Dt, ty, tx);
    }

    // Per-key constants of this query tile (off the diagonal): rs normalises the soft-min sums.
    const float cmid2 = mid < kInf ? -mid * il2 : -kInf;
    float rs[4], svv[4], cap[4], fsum[4];
    bool vrs[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float r = fmaxf(c2_s[a], cmid2);
      vrs[a] = !diag && r > -kInf;
      rs[a] = vrs[a] ? r : 0.f;
      svv[a] = ex2(sufl_s[a] - rs[a]) + ex2(midl - rs[a]);
      cap[a] = fminf(suf_s[a], mid);
      fsum[a] = 0.f;
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int sl = ty * 4 + a;
      float rm[4];
      if (diag) ld_vec<4>(rm, Ps + sl * kPitch + tx * 4);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int tl = tx * 4 + c;
        const bool t_ok = i * kFT + tl < T;
        float x;
        bool valid, strict;
        if (diag) {
          x = (tl > sl ? rm[c] : kInf) - psi_s[a];
          valid = tl >= sl && t_ok && s_ok[a];
          strict = valid && tl > sl;
        } else {
          x = fminf(cap[a], pres[tl]) - psi_s[a];
          valid = t_ok && s_ok[a];
          strict = valid;
        }
        const float xm = fminf(x, 0.f);
        const float p = valid ? ex2(sS[a][c] + betal * xm - lses[tl]) : 0.f;
        const float ds = p * (sP[a][c] - dels[tl]);
        const float g = (strict && x <= 0.f) ? ds : 0.f;
        gsum[a] += g;
        dbsum += strict ? ds * xm : 0.f;
        if (!diag) fsum[a] += __fdividef(g, svv[a] + ex2(prels[tl] - rs[a]));
        sS[a][c] = p;
        sP[a][c] = ds;
      }
    }
    if (diag) __syncthreads();  // the range-minimum table is read; Ps takes P
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int sl = ty * 4 + a;
      *reinterpret_cast<float4*>(Ps + sl * kPitch + tx * 4) = make_float4(sS[a][0], sS[a][1], sS[a][2], sS[a][3]);
      *reinterpret_cast<float4*>(Ds + sl * kPitch + tx * 4) = make_float4(sP[a][0], sP[a][1], sP[a][2], sP[a][3]);
    }
    __syncthreads();
    // dV += P^T dO and dK += dS^T Q over the tile's 64 queries, one stage of DC columns at a time.
#pragma unroll
    for (int cc = 0; cc < CPT / (DC / 16); ++cc) {
      if (cc > 0) {
        __syncthreads();
        load_stage(i, first + cc);
        __syncthreads();
      }
#pragma unroll 2
      for (int t0 = 0; t0 < kFT; t0 += 4) {
        float pr[4][4], dr[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          ld_vec<4>(pr[a], Ps + (ty * 4 + a) * kPitch + t0);
          ld_vec<4>(dr[a], Ds + (ty * 4 + a) * kPitch + t0);
        }
#pragma unroll
        for (int gl = 0; gl < DC / 16; ++gl) {
          const int g = cc * (DC / 16) + gl;
          float dov[4], qv[4];
          ld_vec<4>(dov, Dt + (tx + 16 * gl) * kPitch + t0);
          ld_vec<4>(qv, Qt + (tx + 16 * gl) * kPitch + t0);
#pragma unroll
          for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              dva[a][g] = fmaf(pr[a][c], dov[c], dva[a][g]);
              dka[a][g] = fmaf(dr[a][c], qv[c], dka[a][g]);
            }
        }
      }
    }
    if (!diag) {
      float tp = 0.f;
#pragma unroll
      for (int a = 0; a < 4; ++a)
        if (vrs[a]) {
          wsum[a] += ex2(c2_s[a] - rs[a]) * fsum[a];
          tp += ex2(cmid2 - rs[a]) * fsum[a];
        }
      if (i > j + 1 && half == 0) {
        // Tile-pair total: one partial per warp, summed in a fixed order by the dphi kernel.
        tp = group_sum<32>(tp);
        if ((tid & 31) == 0) sc.tb[((size_t(z) * NB + i) * NB + j) * sc.tb_parts + warp] = tp;
      }
      mid = fminf(mid, st.bmin[size_t(z) * NB + i]);
      midl = lse2(midl, st.bl[size_t(z) * NB + i]);
    } else if (half == 0) {
      // In-tile soft-min gradient of the diagonal tile, one thread per key s: with Z_{s,t} = sum over s < u <= t
      // of 2^{a2_u} carried as L = log2 Z, H(t) = g_st + (Z_{s,t} / Z_{s,t+1}) H(t + 1) and the contribution to
      // u = t is (2^{a2_t} / Z_{s,t}) H(t); DPHI4_t sums the contributions over the keys s < t.
      __syncthreads();  // the dV / dK updates have read Ps and Ds
      const int tend = min(kFT, T - i * kFT);
      if (tid < kFT) {
        float* drow = Ds + tid * kPitch;
        float* lrow = Ps + tid * kPitch;
        const float ps = psik[tid];
        float rmin = kInf, L = -kInf;
        for (int tl = tid + 1; tl < tend; ++tl) {
          rmin = fminf(rmin, phis[tl]);
          drow[tl] = rmin - ps <= 0.f ? drow[tl] : 0.f;  // g: the minimum over (s, t] lies at or below psi_s
          L = lse2(L, -phis[tl] * il2);
          lrow[tl] = L;
        }
        float Hh = 0.f;
        for (int tl = tend - 1; tl > tid; --tl) {
          if (tl < tend - 1) Hh *= ex2(lrow[tl] - lrow[tl + 1]);
          Hh += drow[tl];
          drow[tl] = ex2(-phis[tl] * il2 - lrow[tl]) * Hh;
        }
      }
      __syncthreads();
      if (tid < tend) {
        float a4 = 0.f;
        for (int s2 = 0; s2 < tid; ++s2) a4 += Ds[s2 * kPitch + tid];
        sc.dphi4[zp + size_t(i) * kFT + tid] = a4;
      }
    }
  }

  TIn* dk = static_cast<TIn*>(A.dk) + b * A.sdk.b + h * A.sdk.h;
  TIn* dv = static_cast<TIn*>(A.dv) + b * A.sdv.b + h * A.sdv.h;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const float gs = row16_sum(gsum[a]), ws = row16_sum(wsum[a]);
    const int s = j * kFT + ty * 4 + a;
    if (!s_ok[a]) continue;
#pragma unroll
    for (int g = 0; g < CPT; ++g) {
      const int64_t col = half * BT::NC + tx + 16 * g;
      dk[int64_t(s) * A.sdk.t + col * A.sdk.d] = from_f32<TIn>(dka[a][g] * A.scale);
      dv[int64_t(s) * A.sdv.t + col * A.sdv.d] = from_f32<TIn>(dva[a][g]);
    }
    if (tx == 0 && half == 0) {
      A.dpsi[zt + s] = -bh * gs;
      sc.w[zp + s] = ws;
    }
  }
  if (half != 0) return;
  // dbeta partial of this key tile, reduced in a fixed order.
  dbsum = group_sum<32>(dbsum);
  if ((tid & 31) == 0) red[warp] = dbsum;
  __syncthreads();
  if (tid == 0) {
    float tot = 0.f;
    for (int w = 0; w < kFThreads / 32; ++w) tot += red[w];
    sc.dbeta[size_t(z) * NB + j] = tot;
  }
}

// ------------------------------------------------------------------------------------------------- q-pass ----
// Query tile i: dQ and the soft-min contribution of u in the query's own tile (DPHI2), from
//   r_t = sum_{s in earlier tiles} g_ts 2^{c_t} / Z_{s,t},  DPHI2_u = sum_{t >= u in tile} 2^{a2_u - c_t} r_t.
// The columns half * NC .. of dQ (DPHI2 from half 0 only).
template <typename TIn, int D, bool VEC>
__device__ __forceinline__ void q_pass(const BwdTiledArgs& A, const Stats& st, const BwdScratch& sc, float* smem,
                                       int i, int z, int half) {
  using BT = BwdTile<D>;
  constexpr int CPT = BT::CPT, DC = BT::DC, NCH = BT::NCH;
  float* Qt = smem;
  float* Dt = Qt + D * kPitch;
  float* Kt = Dt + D * kPitch;  // one stage of DC columns of the key tile's K and V
  float* Vt = Kt + DC * kPitch;
  float* Ss = Vt + DC * kPitch;  // dS [query][key]; the range-minimum table of the diagonal tile before
  float* psis = Ss + kFT * kPitch;
  float* phis = psis + kFT;
  float* sufs = phis + kFT;
  float* sufls = sufs + kFT;
  float* rr = sufls + kFT;
  float* c2t = rr + kFT;
  float* phq = c2t + kFT;

  const int H = A.H, T = A.T, NB = A.NB, b = z / H, h = z % H;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const size_t TP = size_t(NB) * kFT, zt = size_t(z) * T, zp = size_t(z) * TP;
  const float betal = A.beta[h] * kLog2e, il2 = A.il2;
  const TIn* k = static_cast<const TIn*>(A.k) + b * A.sk.b + h * A.sk.h;
  const TIn* v = static_cast<const TIn*>(A.v) + b * A.sv.b + h * A.sv.h;

  load_rows<TIn, D, true, VEC>(Qt, static_cast<const TIn*>(A.q) + b * A.sq.b + h * A.sq.h, A.sq, i, T,
                               A.scale * kLog2e);
  load_rows<TIn, D, true, VEC>(Dt, static_cast<const TIn*>(A.dout) + b * A.sdo.b + h * A.sdo.h, A.sdo, i, T, 1.f);

  float lse_t[4], del_t[4], pre_t[4], c2_t[4], bpre[4], racc[4];
  bool t_ok[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int t = i * kFT + ty * 4 + a;
    t_ok[a] = t < T;
    lse_t[a] = t_ok[a] ? A.lse[zt + t] : 0.f;
    del_t[a] = t_ok[a] ? sc.delta[zp + t] : 0.f;
    pre_t[a] = st.pre[zp + t];
    const float prel = st.prel[zp + t];
    c2_t[a] = t_ok[a] ? -pre_t[a] * il2 : 0.f;
    bpre[a] = t_ok[a] ? ex2(prel - c2_t[a]) : 1.f;
    racc[a] = 0.f;
  }
  float dqa[4][CPT];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int g = 0; g < CPT; ++g) dqa[a][g] = 0.f;
  float mid = kInf, midl = -kInf;

  // Stages of K and V in the order (first + 1, ..., first), as in the kv-pass.
  const int first = half * (NCH / BT::NH);
  auto load_stage = [&](int j, int c) {
    load_rows<TIn, DC, true, VEC>(Kt, k + int64_t(c) * DC * A.sk.d, A.sk, j, T, 1.f);
    load_rows<TIn, DC, true, VEC>(Vt, v + int64_t(c) * DC * A.sv.d, A.sv, j, T, 1.f);
  };

  // The diagonal tile first, then the earlier key tiles walking back with mid = min phi over the tiles passed.
  for (int j = i; j >= 0; --j) {
    const bool diag = j == i;
    float sS[4][4], sP[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) sS[a][c] = sP[a][c] = 0.f;
#pragma unroll 1
    for (int kk = 0; kk < NCH; ++kk) {
      const int c = (first + 1 + kk) % NCH;
      __syncthreads();  // the previous stage (and, at kk = 0, the previous key tile's Ss) are read
      load_stage(j, c);
      if (kk == 0 && tid < kFT) {
        const int s = j * kFT + tid;
        psis[tid] = s < T ? A.psi[zt + s] : 0.f;
        phis[tid] = s < T ? A.phi[zt + s] : kInf;
        sufs[tid] = st.suf[zp + s];
        sufls[tid] = st.sufl[zp + s];
      }
      __syncthreads();
      if (kk == 0 && diag) {
        // Range-minimum table: Ss[t][s] = min phi over (s, t] for s < t, one thread per query walking its keys down.
        if (tid < kFT) {
          float x = kInf;
          float* row = Ss + tid * kPitch;
          for (int s = tid - 1; s >= 0; --s) {
            x = fminf(x, phis[s + 1]);
            row[s] = x;
          }
        }
        __syncthreads();
      }
      score_blocks<DC>(sS, sP, Qt + c * DC * kPitch, Kt, Dt + c * DC * kPitch, Vt, ty, tx);
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int tl = ty * 4 + a;
      float rm[4];
      if (diag) ld_vec<4>(rm, Ss + tl * kPitch + tx * 4);
      const float cap = fminf(mid, pre_t[a]);
      const float mterm = ex2(midl - c2_t[a]) + bpre[a];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int sl = tx * 4 + c;
        float x;
        bool valid;
        if (diag) {
          x = (sl < tl ? rm[c] : kInf) - psis[sl];
          valid = sl <= tl && j * kFT + sl < T && t_ok[a];
        } else {
          x = fminf(sufs[sl], cap) - psis[sl];
          valid = t_ok[a];
        }
        const float p = valid ? ex2(sS[a][c] + betal * fminf(x, 0.f) - lse_t[a]) : 0.f;
        const float ds = p * (sP[a][c] - del_t[a]);
        if (!diag) {
          const float g = (valid && x <= 0.f) ? ds : 0.f;
          racc[a] += __fdividef(g, ex2(sufls[sl] - c2_t[a]) + mterm);
        }
        sP[a][c] = ds;
      }
    }
    if (diag) __syncthreads();  // the range-minimum table is read; Ss takes dS
#pragma unroll
    for (int a = 0; a < 4; ++a)
      *reinterpret_cast<float4*>(Ss + (ty * 4 + a) * kPitch + tx * 4) =
          make_float4(sP[a][0], sP[a][1], sP[a][2], sP[a][3]);
    __syncthreads();
    // dQ += dS K over the tile's 64 keys, one stage of DC columns at a time.
#pragma unroll
    for (int cc = 0; cc < CPT / (DC / 16); ++cc) {
      if (cc > 0) {
        __syncthreads();
        load_stage(j, first + cc);
        __syncthreads();
      }
#pragma unroll 2
      for (int s0 = 0; s0 < kFT; s0 += 4) {
        float dr[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a) ld_vec<4>(dr[a], Ss + (ty * 4 + a) * kPitch + s0);
#pragma unroll
        for (int gl = 0; gl < DC / 16; ++gl) {
          const int g = cc * (DC / 16) + gl;
          float kv[4];
          ld_vec<4>(kv, Kt + (tx + 16 * gl) * kPitch + s0);
#pragma unroll
          for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) dqa[a][g] = fmaf(dr[a][c], kv[c], dqa[a][g]);
        }
      }
    }
    if (!diag) {
      mid = fminf(mid, st.bmin[size_t(z) * NB + j]);
      midl = lse2(midl, st.bl[size_t(z) * NB + j]);
    }
  }

  TIn* dq = static_cast<TIn*>(A.dq) + b * A.sdq.b + h * A.sdq.h;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    racc[a] = row16_sum(racc[a]);
    const int t = i * kFT + ty * 4 + a;
    if (!t_ok[a]) continue;
#pragma unroll
    for (int g = 0; g < CPT; ++g)
      dq[int64_t(t) * A.sdq.t + int64_t(half * BT::NC + tx + 16 * g) * A.sdq.d] = from_f32<TIn>(dqa[a][g] * A.scale);
  }
  if (half != 0) return;
  if (tx == 0)
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int tl = ty * 4 + a, t = i * kFT + tl;
      rr[tl] = racc[a];
      c2t[tl] = c2_t[a];
      phq[tl] = t_ok[a] ? A.phi[zt + t] : kInf;  // the query tile's own field
    }
  __syncthreads();
  const int t = i * kFT + tid;
  if (tid < kFT && t < T) {
    const int tend = min(kFT, T - i * kFT);
    const float a2 = -phq[tid] * il2;
    float p2 = 0.f;
    for (int t2 = tid; t2 < tend; ++t2) p2 += ex2(a2 - c2t[t2]) * rr[t2];
    sc.dphi2[zp + t] = p2;
  }
}

template <typename TIn, int D, bool VEC>
__global__ void __launch_bounds__(kFThreads, D <= 64 ? 2 : 1)
simt_bwd_tiled_kernel(const BwdTiledArgs A, const Stats st, const BwdScratch sc) {
  extern __shared__ __align__(16) float smem[];
  constexpr int NH = BwdTile<D>::NH;
  const int BH = int(gridDim.x) / (2 * NH * A.NB);  // grid: 2 NH NB units (rank major) x B H heads
  const int u = int(blockIdx.x) / BH, z = int(blockIdx.x) % BH;
  const int half = (u >> 1) % NH, x = u / (2 * NH);
  if (u & 1)
    q_pass<TIn, D, VEC>(A, st, sc, smem, A.NB - 1 - x, z, half);
  else
    kv_pass<TIn, D, VEC>(A, st, sc, smem, x, z, half);
}

template <typename TIn, int D>
cudaError_t launch(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s) {
  const bool vec = vec_ok<TIn>(a.q, a.q_stride) && vec_ok<TIn>(a.k, a.k_stride) &&
                   vec_ok<TIn>(a.v, a.v_stride) && vec_ok<TIn>(a.dout, a.dout_stride);
  auto fn = vec ? simt_bwd_tiled_kernel<TIn, D, true> : simt_bwd_tiled_kernel<TIn, D, false>;
  const size_t smem = BwdTile<D>::SMEM;
  if (smem > 48 * 1024) {
    const cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(fn), int(smem));
    if (e != cudaSuccess) return e;
  }
  BwdTiledArgs A;
  A.q = a.q, A.k = a.k, A.v = a.v, A.dout = a.dout;
  A.sq = str4(a.q_stride), A.sk = str4(a.k_stride), A.sv = str4(a.v_stride), A.sdo = str4(a.dout_stride);
  A.lse = a.lse, A.phi = a.phi, A.psi = a.psi, A.beta = a.beta;
  A.dq = a.dq, A.dk = a.dk, A.dv = a.dv;
  A.sdq = str4(a.dq_stride), A.sdk = str4(a.dk_stride), A.sdv = str4(a.dv_stride);
  A.dpsi = a.dpsi;
  A.H = d.H, A.T = d.T, A.NB = d.NB;
  A.scale = float(1.0 / sqrt(double(d.D)));
  A.il2 = kLog2e / a.tau;
  fn<<<dim3(2 * BwdTile<D>::NH * d.NB * d.B * d.H), kFThreads, smem, s>>>(A, st, sc);
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_d(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, cudaStream_t s) {
  switch (d.D) {
    case 16: return launch<TIn, 16>(a, d, st, sc, s);
    case 32: return launch<TIn, 32>(a, d, st, sc, s);
    case 64: return launch<TIn, 64>(a, d, st, sc, s);
    case 128: return launch<TIn, 128>(a, d, st, sc, s);
    case 256: return launch<TIn, 256>(a, d, st, sc, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t simt_bwd_tiled(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc,
                           cudaStream_t s) {
  return a.dtype == FPA_DTYPE_F16 ? launch_d<__half>(a, d, st, sc, s) : launch_d<float>(a, d, st, sc, s);
}

}  // namespace fpa
