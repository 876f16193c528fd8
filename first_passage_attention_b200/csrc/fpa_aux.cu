// Small kernels around the attention passes: field statistics, delta = rowsum(dO * O), the final combination of
// the soft-min gradient of phi, and the batch/tile reduction of dbeta. All are deterministic (fixed summation order).
#include <cstdlib>

#include "fpa_internal.h"

namespace fpa {

size_t stats_bytes(const Dims& d) {
  size_t bh = size_t(d.BH());
  return 4 * align256(bh * d.TP * sizeof(float)) + 2 * align256(bh * d.NB * sizeof(float));
}

size_t bwd_scratch_bytes(const Dims& d, int tb_parts) {
  size_t bh = size_t(d.BH());
  return 4 * align256(bh * d.TP * sizeof(float)) + align256(bh * d.NB * d.NB * tb_parts * sizeof(float)) +
         2 * align256(bh * d.NB * sizeof(float));
}

static float* take(char*& p, size_t n_floats) {
  float* r = reinterpret_cast<float*>(p);
  p += align256(n_floats * sizeof(float));
  return r;
}

Stats carve_stats(char* base, const Dims& d) {
  size_t bh = size_t(d.BH());
  Stats s;
  s.pre = take(base, bh * d.TP);
  s.suf = take(base, bh * d.TP);
  s.prel = take(base, bh * d.TP);
  s.sufl = take(base, bh * d.TP);
  s.bmin = take(base, bh * d.NB);
  s.bl = take(base, bh * d.NB);
  return s;
}

BwdScratch carve_bwd(char* base, const Dims& d, int tb_parts) {
  size_t bh = size_t(d.BH());
  BwdScratch s;
  s.tb_parts = tb_parts;
  s.tb_sum = tb_parts;
  s.delta = take(base, bh * d.TP);
  s.w = take(base, bh * d.TP);
  s.dphi2 = take(base, bh * d.TP);
  s.dphi4 = take(base, bh * d.TP);
  s.tb = take(base, bh * d.NB * d.NB * tb_parts);
  s.dbeta = take(base, bh * d.NB);
  s.part3 = take(base, bh * d.NB);
  return s;
}

size_t keycols_bytes(const Dims& d) { return 3 * align256(size_t(d.BH()) * d.TP * sizeof(float)); }

KeyCols carve_keycols(char* base, const Dims& d) {
  size_t n = size_t(d.BH()) * d.TP;
  KeyCols c;
  c.a = take(base, n);
  c.psi = take(base, n);
  c.phi = take(base, n);
  return c;
}

// Block per (tile j, head z), one thread per position: warp-shuffle scans joined across warps through shared
// memory (kernel.py:84-100 computes the same per-tile statistics). It also clears the device status word of the
// call's workspace (the first launch of every call), and, when `cols.a` is set, writes the per-key vectors of the
// tensor-core forward. Positions >= T take phi = +inf (a2 = -inf) and do not enter any statistic.
// QV: the tensor-core backward's instantiation, which also forms delta and the per-query pairs (its rows of O and
// dO in flight cost registers that the forward's instantiation does not spend). Eight 128-thread blocks per SM: at
// configuration 2 (768 blocks) the whole grid is resident at once.
template <bool QV>
__global__ void __launch_bounds__(128, 8) stats_kernel(const float* __restrict__ phi, const float* __restrict__ psi, int BH, int T, int BT,
                             int NB, float il2, Stats st, KeyCols cols, int cols_scaled,
                             const float* __restrict__ beta, int H, Fact fact, int* status, QvIn qv, int* tile_cnt,
                             int ncnt) {
  __shared__ float wmin[32], wlse[32], smin[1024], slse[1024];
  pdl_wait();  // launched with launch_pdl: the previous kernel's writes are visible from here on
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, nw = BT >> 5;
  const int j = blockIdx.x, z = blockIdx.z * gridDim.y + blockIdx.y;  // grid (NB, H, B): z = b * H + h
  if (j == 0 && z == 0 && tid < 4 && status) status[tid] = 0;  // status word and the work-unit counters
  if (tid < ncnt) tile_cnt[(size_t(z) * NB + j) * ncnt + tid] = 0;  // the split kernels' per-tile join counters
  const int t = j * BT + tid;
  const size_t base = (size_t(z) * NB + j) * BT;
  // The global loads of the kernel are issued here, before any of them is used, so that few memory latencies cover
  // them all (the kernel is latency-bound at small sizes): phi, psi, lse and beta of this block's positions, and
  // for the tensor-core backward the rows of O and dO for delta_t = sum_d dO[t, d] O[t, d] (kernel.py:166-174).
  const bool need_psi = fact.kv4 != nullptr || cols.a != nullptr;
  const float p = t < T ? phi[size_t(z) * T + t] : kInf;
  const float y_psi = (need_psi && t < T) ? psi[size_t(z) * T + t] : 0.f;
  const float beta_h = (cols.a && cols_scaled) ? beta[z % H] : 0.f;
  float delta = 0.f, nlse = -kInf;
  if (QV && t < T) nlse = -qv.lse[size_t(z) * T + t];
  // delta in float32, read coalesced: each warp covers its 32 rows with groups of G = D/8 lanes, one 16-byte load
  // of O and of dO per lane per row (four rows' loads in flight at once), a fixed shuffle tree over the group, and
  // the row's owner thread picks the sum up from shared memory. Packed with -lse, PRE and prey at the end.
  __shared__ float sdelta[1024];
  if constexpr (QV) {
    const int G = qv.D / 8, rpi = 32 / G, sub = lane / G, part = lane % G;
    const int b = z / H, h = z % H;
    const __half* ob = qv.o + b * qv.so.b + h * qv.so.h + part * 8;
    const __half* db = qv.dout + b * qv.sdo.b + h * qv.sdo.h + part * 8;
    for (int it0 = 0; it0 < G; it0 += 4) {
      uint4 xo[4], xd[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int rr = w * 32 + (it0 + q) * rpi + sub, tt = j * BT + rr;
        xo[q] = make_uint4(0u, 0u, 0u, 0u);
        xd[q] = make_uint4(0u, 0u, 0u, 0u);
        if (it0 + q < G && tt < T) {
          xo[q] = *reinterpret_cast<const uint4*>(ob + int64_t(tt) * qv.so.t);
          xd[q] = *reinterpret_cast<const uint4*>(db + int64_t(tt) * qv.sdo.t);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (it0 + q >= G) break;
        const __half2* xh = reinterpret_cast<const __half2*>(&xo[q]);
        const __half2* yh = reinterpret_cast<const __half2*>(&xd[q]);
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 a2 = __half22float2(xh[e]), b2 = __half22float2(yh[e]);
          acc = fmaf(a2.x, b2.x, acc);
          acc = fmaf(a2.y, b2.y, acc);
        }
        for (int o = G >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (part == 0) sdelta[w * 32 + (it0 + q) * rpi + sub] = acc;
      }
    }
    __syncwarp();
    delta = sdelta[tid];  // this warp's rows only
  }
  const float a = t < T ? -p * il2 : -kInf;
  // inclusive prefix: PRE, PREL
  float pm = p, pl = a;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float qm = __shfl_up_sync(0xffffffffu, pm, o), ql = __shfl_up_sync(0xffffffffu, pl, o);
    if (lane >= o) {
      pm = fminf(pm, qm);
      pl = lse2(pl, ql);
    }
  }
  if (lane == 31) {
    wmin[w] = pm;
    wlse[w] = pl;
  }
  __syncthreads();
  for (int v = 0; v < w; ++v) {
    pm = fminf(pm, wmin[v]);
    pl = lse2(pl, wlse[v]);
  }
  st.pre[base + tid] = pm;
  st.prel[base + tid] = pl;
  if (tid == BT - 1) {
    st.bmin[size_t(z) * NB + j] = pm;
    st.bl[size_t(z) * NB + j] = pl;
  }
  __syncthreads();
  // inclusive suffix, then shifted by one: SUF_t, SUFL_t over (t, tile end]
  float sm = p, sl = a;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float qm = __shfl_down_sync(0xffffffffu, sm, o), ql = __shfl_down_sync(0xffffffffu, sl, o);
    if (lane + o < 32) {
      sm = fminf(sm, qm);
      sl = lse2(sl, ql);
    }
  }
  if (lane == 0) {
    wmin[w] = sm;
    wlse[w] = sl;
  }
  __syncthreads();
  for (int v = nw - 1; v > w; --v) {
    sm = fminf(sm, wmin[v]);
    sl = lse2(sl, wlse[v]);
  }
  smin[tid] = sm;
  slse[tid] = sl;
  __syncthreads();
  const float suf = tid + 1 < BT ? smin[tid + 1] : kInf;
  const float sufl = tid + 1 < BT ? slse[tid + 1] : -kInf;
  st.suf[base + tid] = suf;
  st.sufl[base + tid] = sufl;
  if (fact.prey) {
    // slse holds the inclusive suffix LSE: slse[0] = BL_j; the prefix LSE of the first position is a2 there;
    // the smallest finite exclusive suffix is at the second-to-last valid position (= a2 of the last one).
    const int lv = min(BT, T - j * BT) - 1;
    const float blj = slse[0];
    const float sufl0 = BT > 1 ? slse[1] : -kInf;
    fact.prey[base + tid] = t < T ? ex2(pl - blj) : 1.f;
    fact.sufy[base + tid] = ex2(sufl - sufl0);
    if (tid == 0) {
      fact.prer[size_t(z) * NB + j] = blj - pl;  // pl = PREL_first in thread 0
      fact.sufr[size_t(z) * NB + j] = lv >= 1 ? sufl0 - slse[lv] : 0.f;
    }
    if (fact.kv4) {
      // Pair layout: keys c, c+1 (c even) share kv4[c] and kv4[c + 1].
      const float y = y_psi;
      float* kv = reinterpret_cast<float*>(fact.kv4 + base + (tid & ~1)) + (tid & 1);
      kv[0] = t < T ? suf - y : kInf;
      kv[2] = -y;
      kv[4] = ex2(sufl - sufl0);
      kv[6] = sufl;
    }
    if (QV) {
      // Pair layout: queries c, c+1 (c even) share qv4[c] = (-lse, -delta) and qv4[c + 1] = (PRE, prey).
      float* qa = reinterpret_cast<float*>(qv.qv4 + base + (tid & ~1)) + (tid & 1);
      qa[0] = nlse;  // -inf beyond T
      qa[2] = t < T ? -delta : 0.f;
      qa[4] = pm;
      qa[6] = t < T ? ex2(pl - blj) : 1.f;
    }
  }
  if (cols.a) {
    const bool ok = t < T;
    const float y = y_psi;
    if (cols_scaled) {
      const float bl = beta_h * kLog2e;
      cols.a[base + tid] = ok ? bl * fminf(suf - y, 0.f) : 0.f;
      cols.psi[base + tid] = ok ? -bl * y : 0.f;
      cols.phi[base + tid] = ok ? bl * p : 0.f;
    } else {
      cols.a[base + tid] = ok ? suf - y : kInf;
      cols.psi[base + tid] = y;
      cols.phi[base + tid] = ok ? p : kInf;
    }
  }
}

cudaError_t launch_stats(const float* phi, const float* psi, const float* beta, const Dims& d, float tau,
                         const Stats& st, const KeyCols& cols, int cols_scaled, int* status, cudaStream_t s,
                         const Fact* fact, const QvIn* qv, int* tile_cnt, int ncnt) {
  const Fact f = fact ? *fact : Fact{nullptr, nullptr, nullptr, nullptr, nullptr};
  const QvIn q = qv ? *qv : QvIn{nullptr, Str4{0, 0, 0, 0}, nullptr, Str4{0, 0, 0, 0}, nullptr, nullptr, 0};
  return launch_pdl(qv ? stats_kernel<true> : stats_kernel<false>, dim3(d.NB, d.H, d.B), dim3(d.BT), 0, s, phi, psi,
                    d.BH(), d.T, d.BT, d.NB, kLog2e / tau, st, cols, cols_scaled, beta, d.H, f, status, q, tile_cnt,
                    tile_cnt ? ncnt : 0);
}

// delta_t = sum_d dO[t, d] * O[t, d] in float32 (kernel.py:166-174). One warp per row.
// When `lse` and `lsep` are set it also copies lse [BH][T] into the padded layout lsep [BH][TP], so the tensor-core
// backward can fetch whole tiles of it with bulk copies.
template <typename TIn>
__global__ void delta_kernel(const TIn* __restrict__ o, Str4 so, const TIn* __restrict__ dout, Str4 sdo, int H,
                             int T, int D, int TP, int rows, float* __restrict__ delta, const float* __restrict__ lse,
                             float* __restrict__ lsep) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  int z = warp / T, t = warp % T, b = z / H, h = z % H;
  const TIn* op = o + b * so.b + h * so.h + int64_t(t) * so.t;
  const TIn* dp = dout + b * sdo.b + h * sdo.h + int64_t(t) * sdo.t;
  float acc = 0.f;
  for (int c = lane; c < D; c += 32) acc += to_f32(op[c * so.d]) * to_f32(dp[c * sdo.d]);
  acc = group_sum<32>(acc);
  if (lane == 0) {
    delta[size_t(z) * TP + t] = acc;
    if (lsep) lsep[size_t(z) * TP + t] = lse[size_t(z) * T + t];
  }
}

// fp16 with unit innermost stride and 16-byte aligned rows: G = D / 8 lanes per row, 16-byte loads.
template <int G>
__global__ void delta_f16_vec_kernel(const __half* __restrict__ o, Str4 so, const __half* __restrict__ dout, Str4 sdo,
                                     int H, int T, int TP, int rows, float* __restrict__ delta,
                                     const float* __restrict__ lse, float* __restrict__ lsep) {
  const int gid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gid / G, part = gid % G;
  const bool ok = row < rows;
  float acc = 0.f;
  int z = 0, t = 0;
  if (ok) {
    z = row / T;
    t = row % T;
    const int b = z / H, h = z % H;
    const uint4 a = *reinterpret_cast<const uint4*>(o + b * so.b + h * so.h + int64_t(t) * so.t + part * 8);
    const uint4 c = *reinterpret_cast<const uint4*>(dout + b * sdo.b + h * sdo.h + int64_t(t) * sdo.t + part * 8);
    const __half2* ah = reinterpret_cast<const __half2*>(&a);
    const __half2* ch = reinterpret_cast<const __half2*>(&c);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 x = __half22float2(ah[q]), y = __half22float2(ch[q]);
      acc = fmaf(x.x, y.x, acc);
      acc = fmaf(x.y, y.y, acc);
    }
  }
  acc = group_sum<G>(acc);
  if (ok && part == 0) {
    delta[size_t(z) * TP + t] = acc;
    if (lsep) lsep[size_t(z) * TP + t] = lse[size_t(z) * T + t];
  }
}

static bool vec16_ok(const void* p, Str4 s) {
  return reinterpret_cast<uintptr_t>(p) % 16 == 0 && s.d == 1 && (s.t * 2) % 16 == 0 && (s.h * 2) % 16 == 0 &&
         (s.b * 2) % 16 == 0;
}

cudaError_t launch_delta(int dtype, const void* o, Str4 so, const void* dout, Str4 sdo, const Dims& d, float* delta,
                         const float* lse, float* lsep, cudaStream_t s) {
  int rows = d.BH() * d.T;
  if (dtype == FPA_DTYPE_F16 && d.D >= 16 && d.D <= 256 && vec16_ok(o, so) && vec16_ok(dout, sdo)) {
    const int G = d.D / 8;
    const int blocks = int((int64_t(rows) * G + 255) / 256);
    auto a = static_cast<const __half*>(o);
    auto c = static_cast<const __half*>(dout);
    switch (G) {
      case 2: delta_f16_vec_kernel<2><<<blocks, 256, 0, s>>>(a, so, c, sdo, d.H, d.T, d.TP, rows, delta, lse, lsep); break;
      case 4: delta_f16_vec_kernel<4><<<blocks, 256, 0, s>>>(a, so, c, sdo, d.H, d.T, d.TP, rows, delta, lse, lsep); break;
      case 8: delta_f16_vec_kernel<8><<<blocks, 256, 0, s>>>(a, so, c, sdo, d.H, d.T, d.TP, rows, delta, lse, lsep); break;
      case 16: delta_f16_vec_kernel<16><<<blocks, 256, 0, s>>>(a, so, c, sdo, d.H, d.T, d.TP, rows, delta, lse, lsep); break;
      default: delta_f16_vec_kernel<32><<<blocks, 256, 0, s>>>(a, so, c, sdo, d.H, d.T, d.TP, rows, delta, lse, lsep); break;
    }
    return cudaGetLastError();
  }
  int blocks = (rows * 32 + 255) / 256;
  if (dtype == FPA_DTYPE_F16)
    delta_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)o, so, (const __half*)dout, sdo, d.H, d.T, d.D,
                                                d.TP, rows, delta, lse, lsep);
  else
    delta_kernel<float><<<blocks, 256, 0, s>>>((const float*)o, so, (const float*)dout, sdo, d.H, d.T, d.D, d.TP,
                                               rows, delta, lse, lsep);
  return cudaGetLastError();
}

// Per-query vectors of the tensor-core backward, two queries t, t+1 (t even) per pair of float4 so the kv-pass
// reads them as operands of packed f32x2 arithmetic:
//   qv4[t] = (-lse_t, -lse_t1, -delta_t, -delta_t1),  qv4[t + 1] = (PRE_t, PRE_t1, prey_t, prey_t1);
// beyond T: lse = +inf, delta = 0, prey = 1, so padded queries get P = 0. One thread per pair.
__global__ void qv_pack_kernel(const float* __restrict__ lse, const float* __restrict__ delta,
                               const float* __restrict__ pre, const float* __restrict__ prey, int T, int TP, int n,
                               float4* __restrict__ qv4) {
  const int pidx = blockIdx.x * blockDim.x + threadIdx.x;  // pair index over [BH][TP / 2]
  if (2 * pidx >= n) return;
  const int idx = 2 * pidx;
  const int z = idx / TP, t = idx % TP;
  const bool ok0 = t < T, ok1 = t + 1 < T;
  const size_t lz = size_t(z) * T;
  qv4[idx] = make_float4(ok0 ? -lse[lz + t] : -kInf, ok1 ? -lse[lz + t + 1] : -kInf, ok0 ? -delta[idx] : 0.f,
                         ok1 ? -delta[idx + 1] : 0.f);
  qv4[idx + 1] = make_float4(pre[idx], pre[idx + 1], ok0 ? prey[idx] : 1.f, ok1 ? prey[idx + 1] : 1.f);
}


bool qv_delta_fusable(int dtype, const void* o, Str4 so, const void* dout, Str4 sdo, const Dims& d) {
  return dtype == FPA_DTYPE_F16 && d.D >= 16 && d.D <= 128 && vec16_ok(o, so) && vec16_ok(dout, sdo);
}


cudaError_t launch_qv_pack(const float* lse, const float* delta, const float* pre, const float* prey, const Dims& d,
                           float4* qv4, cudaStream_t s) {
  const int n = d.BH() * d.TP;  // TP is a multiple of 128, so pairs never straddle heads
  qv_pack_kernel<<<(n / 2 + 255) / 256, 256, 0, s>>>(lse, delta, pre, prey, d.T, d.TP, n, qv4);
  return cudaGetLastError();
}

// Deterministic block sum of one value per thread (blockDim.x a multiple of 32, at most 1024). All threads must call.
__device__ float block_sum(float v, float* red) {
  v = group_sum<32>(v);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < nw; ++w) r += red[w];
  return r;  // valid in thread 0
}

// Part 3 of the dphi combination, u strictly between the key's tile j and the query's tile i (kernel.py:352-364),
// for every tile U of one head in O(NB^2) work, for long contexts (dphi_kernel sums all pairs j < U < i for each U,
// O(NB^3) per head, which is cheaper up to a few hundred tiles because it spreads over NB blocks per head):
//   S_U = sum_{j < U < i} 2^{c_U - M(j, i)} TB[i][j],   M(j, i) = max_{j < n < i} c_n,   c_n = -BMIN_n * il2,
// so that part3_u = 2^{a2_u - c_U} S_U (dphi_kernel). With X[i][j] = TB[i][j] at scale 2^{-M(j, i)}, three passes
// in one block per head, each over many independent items:
//   pass 1, every pair (i, j), i >= j + 2: the pair's partial sums (fixed order) and -M(j, i) (two lookups in a
//           sparse table of range maxima) go into the pair's first two floats;
//   pass 2, one warp per key tile j: the suffix sums C_j(U) = sum_{i > U} X[i][j] (a warp scan per 32 pairs with a
//           carry), stored at pair (U + 1, j);
//   pass 3, one warp per tile U: S_U 2^{-c_U} = sum_{j < U} C_j(U), lane-strided and then a fixed shuffle tree.
// Sums of terms at different scales are kept as (m, v) = v 2^m with a running maximum; c_U - M(j, i) <= 0, so
// nothing overflows. Fixed orders throughout: deterministic.
constexpr int kPart3CubicMaxNB = 256;

__device__ __forceinline__ void join_mv(float& m, float& v, float m2, float v2) {
  const float mm = fmaxf(m, m2);
  v = mm == -kInf ? 0.f : v * ex2(m - mm) + v2 * ex2(m2 - mm);
  m = mm;
}

__global__ void dphi_part3_kernel(const float* __restrict__ bmin, int NB, int LV, float il2, BwdScratch sc) {
  extern __shared__ float rmq[];  // [LV][NB]: rmq[l][n] = max c over tiles n .. n + 2^l - 1
  pdl_wait();  // launched with launch_pdl after the backward passes
  pdl_launch_dependents();
  const int z = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nwarps = blockDim.x >> 5;
  for (int n = tid; n < NB; n += blockDim.x) rmq[n] = -bmin[size_t(z) * NB + n] * il2;
  __syncthreads();
  for (int l = 1; l < LV; ++l) {
    for (int n = tid; n + (1 << l) <= NB; n += blockDim.x)
      rmq[l * NB + n] = fmaxf(rmq[(l - 1) * NB + n], rmq[(l - 1) * NB + n + (1 << (l - 1))]);
    __syncthreads();
  }
  const int np = sc.tb_parts;
  float* tbz = sc.tb + size_t(z) * NB * NB * np;
  // pass 1
  for (int q = tid; q < NB * NB; q += blockDim.x) {
    const int i = q / NB, j = q % NB;
    if (i < j + 2) continue;
    float* pp = tbz + size_t(q) * np;
    float v = 0.f;
    if (sc.tb_sum == 8) {
      const float4 x = reinterpret_cast<const float4*>(pp)[0], y = reinterpret_cast<const float4*>(pp)[1];
      v = (((x.x + x.y) + x.z) + x.w) + (((y.x + y.y) + y.z) + y.w);
    } else {
      for (int k = 0; k < sc.tb_sum; ++k) v += pp[k];
    }
    const int lo = j + 1, len = i - 1 - lo + 1, l = 31 - __clz(len);
    const float mx = fmaxf(rmq[l * NB + lo], rmq[l * NB + i - (1 << l)]);
    pp[0] = v;
    pp[1] = -mx;
  }
  __syncthreads();
  // pass 2: column j holds pairs i = NB-1 .. j+2 (descending); lane k of a 32-pair chunk takes i = top - k
  for (int j = wid; j + 2 < NB; j += nwarps) {
    float cm = -kInf, cv = 0.f;  // carry: the sum over the pairs above this chunk
    for (int top = NB - 1; top >= j + 2; top -= 32) {
      const int i = top - lane;
      const bool in = i >= j + 2;
      float* pp = tbz + (size_t(in ? i : j + 2) * NB + j) * np;
      float m = in ? pp[1] : -kInf, v = in ? pp[0] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive scan over the lanes below (larger i first)
        const float m2 = __shfl_up_sync(0xffffffffu, m, o), v2 = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) join_mv(m, v, m2, v2);
      }
      join_mv(m, v, cm, cv);
      if (in) {
        pp[0] = v;  // C_j(i - 1)
        pp[1] = m;
      }
      cm = __shfl_sync(0xffffffffu, m, 31);
      cv = __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  // pass 3
  for (int U = wid; U < NB; U += nwarps) {
    float m = -kInf, v = 0.f;
    if (U >= 1 && U + 2 <= NB)
      for (int j = lane; j < U; j += 32) {
        const float* pp = tbz + (size_t(U + 1) * NB + j) * np;
        join_mv(m, v, pp[1], pp[0]);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), v2 = __shfl_xor_sync(0xffffffffu, v, o);
      join_mv(m, v, m2, v2);
    }
    if (lane == 0) sc.part3[size_t(z) * NB + U] = v == 0.f ? 0.f : v * ex2(m + rmq[U]);
  }
}

// Final soft-min gradient of phi for tile U of head z (kernel.py:344-370 combines the same four parts):
//   part1_u = sum_{s<u in U, SUF_s<inf} 2^{a2_u - c_s} W_s            (u in the key's tile)
//   dphi2_u                                                            (u in the query's tile)
//   dphi4_u                                                            (u in the diagonal tile with both)
//   part3_u = 2^{a2_u - c_U} sum_{j<U<i} 2^{c_U - cmid_ij} TB[i][j]     (u in a tile strictly between)
// dphi_u = beta * (part1 + dphi2 + dphi4 + part3). Block: BT threads (one per position of the tile).
__global__ void dphi_kernel(const float* __restrict__ phi, const float* __restrict__ beta, int B, int H, int T,
                            int BT, int NB, float il2, Stats st, BwdScratch sc, float* __restrict__ dphi,
                            float* __restrict__ dbeta, int part3_ready) {
  pdl_wait();  // launched with launch_pdl after the backward passes (and the join of the forked q-pass)
  pdl_launch_dependents();
  extern __shared__ float sm[];
  float* cb = sm;           // [NB] max of a2 per tile
  float* A = cb + NB;       // [NB] A[j] = max cb over (j, U]
  float* Bv = A + NB;       // [NB] B[i] = max cb over [U, i)
  float* Ws = Bv + NB;      // [BT]
  float* c2s = Ws + BT;     // [BT]
  float* red = c2s + BT;    // [32]
  const int U = blockIdx.x, z = blockIdx.z * gridDim.y + blockIdx.y, h = z % H;  // grid (NB, H, B)
  const int tid = threadIdx.x;
  const size_t TP = size_t(NB) * BT;
  const int u = U * BT + tid;
  // The per-position inputs of the final sum are loaded first, with the tile statistics below, so that their
  // latency passes during the scans (the kernel is latency-bound at small sizes).
  const bool own = tid < BT && u < T;
  const size_t pu = size_t(z) * TP + u;
  const float phi_u = own ? phi[size_t(z) * T + u] : 0.f;
  const float d2 = own ? sc.dphi2[pu] : 0.f, d4 = own ? sc.dphi4[pu] : 0.f;
  const float beta_h = beta[h];
  for (int n = tid; n < NB; n += blockDim.x) cb[n] = -st.bmin[size_t(z) * NB + n] * il2;
  {
    float w = 0.f, c2 = -kInf;
    if (tid < BT) {
      float suf = st.suf[size_t(z) * TP + u];
      c2 = suf < kInf ? -suf * il2 : -kInf;
      w = sc.w[size_t(z) * TP + u];
      Ws[tid] = w;
      c2s[tid] = c2;
    }
  }
  __syncthreads();
  if (!part3_ready && tid == 0) {
    float m = -kInf;
    for (int j = U - 1; j >= 0; --j) {  // A[j] = max cb over tiles j+1 .. U
      m = fmaxf(m, cb[j + 1]);
      A[j] = m;
    }
    m = -kInf;
    for (int i = U + 1; i < NB; ++i) {  // B[i] = max cb over tiles U .. i-1
      m = fmaxf(m, cb[i - 1]);
      Bv[i] = m;
    }
  }
  __syncthreads();
  // part3 (kernel.py:352-364) partial sums over the tile pairs (i, j), j < U < i, spread over the threads (fixed
  // assignment); each pair's total joins its tb_sum partial sums in order. Long contexts: dphi_part3_kernel.
  float s3 = 0.f;
  if (!part3_ready && U > 0 && U < NB - 1) {
    const float cU = cb[U];
    const int np = sc.tb_parts, npairs = (NB - 1 - U) * U;
    for (int pi = tid; pi < npairs; pi += blockDim.x) {
      const int i = U + 1 + pi / U, j = pi % U;
      const float* part = sc.tb + ((size_t(z) * NB + i) * NB + j) * np;
      float tbij = 0.f;
      if (sc.tb_sum == 8) {
        const float4 u = reinterpret_cast<const float4*>(part)[0], v = reinterpret_cast<const float4*>(part)[1];
        tbij = (((u.x + u.y) + u.z) + u.w) + (((v.x + v.y) + v.z) + v.w);
      } else {
        for (int q = 0; q < sc.tb_sum; ++q) tbij += part[q];
      }
      s3 += ex2(cU - fmaxf(A[j], Bv[i])) * tbij;
    }
  }
  float S = block_sum(s3, red);
  if (tid == 0) red[0] = part3_ready ? sc.part3[size_t(z) * NB + U] : S;
  __syncthreads();
  S = red[0];
  // part1 as an exclusive scan over s of W_s 2^{-c_s} kept as (m, v) = v 2^m with a running maximum m (the
  // partial sums span any range); then part1_u = v 2^{m + a2_u}, where m + a2_u <= 0 since SUF_s <= phi_u.
  // Fixed shuffle tree within warps, warp totals joined in order: deterministic.
  float pm = -kInf, pv = 0.f;
  if (tid < BT && c2s[tid] > -kInf) {
    pm = -c2s[tid];
    pv = Ws[tid];
  }
  auto join = [](float m1, float v1, float m2, float v2, float& mo, float& vo) {
    const float m = fmaxf(m1, m2);
    mo = m;
    vo = m == -kInf ? 0.f : v1 * ex2(m1 - m) + v2 * ex2(m2 - m);
  };
  const int lane = tid & 31, wq = tid >> 5, nwq = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {  // inclusive scan within the warp
    const float qm = __shfl_up_sync(0xffffffffu, pm, o), qv = __shfl_up_sync(0xffffffffu, pv, o);
    if (lane >= o) join(qm, qv, pm, pv, pm, pv);
  }
  __syncthreads();
  if (lane == 31) {
    red[wq] = pm;
    red[8 + wq] = pv;
  }
  __syncthreads();
  float bm = -kInf, bv = 0.f;  // total of the warps before this one
  for (int w = 0; w < wq && w < nwq; ++w) join(bm, bv, red[w], red[8 + w], bm, bv);
  // exclusive: the inclusive value of the previous lane, joined after the earlier warps' total
  float em = __shfl_up_sync(0xffffffffu, pm, 1), ev = __shfl_up_sync(0xffffffffu, pv, 1);
  if (lane == 0) {
    em = -kInf;
    ev = 0.f;
  }
  join(bm, bv, em, ev, em, ev);
  if (own) {
    const float a2 = -phi_u * il2;
    const float part1 = em == -kInf ? 0.f : ev * ex2(em + a2);
    const float part3 = (U > 0 && U < NB - 1) ? ex2(a2 - cb[U]) * S : 0.f;
    dphi[size_t(z) * T + u] = beta_h * (part1 + d2 + d4 + part3);
  }
  // dbeta[h]: the kv-pass's parts summed over the batch and the key tiles, by the first warp of the blocks
  // (U = 0, b = 0), strided over the lanes and then a fixed shuffle tree (kernel.py:450: dbeta.sum((0, 2))).
  if (U == 0 && z < H && tid < 32) {
    const int n = B * NB;
    float acc = 0.f;
    for (int e = tid; e < n; e += 32) acc += sc.dbeta[(size_t(e / NB) * H + h) * NB + e % NB];
    acc = group_sum<32>(acc);
    if (tid == 0) dbeta[h] = acc;
  }
}

cudaError_t launch_dphi(const float* phi, const float* beta, const Dims& d, float tau, const Stats& st,
                        const BwdScratch& sc, float* dphi, float* dbeta, cudaStream_t s, int* launched) {
  // Beyond kPart3CubicMaxNB tiles (or with FPA_B200_DPHI_QUADRATIC set, which the tests use to reach it at small
  // sizes) dphi_part3_kernel evaluates the strictly-between part first, in O(NB^2).
  const bool quadratic = d.NB > kPart3CubicMaxNB || std::getenv("FPA_B200_DPHI_QUADRATIC") != nullptr;
  *launched = 0;
  if (quadratic) {
    int lv = 1;
    while ((1 << lv) <= d.NB) ++lv;  // levels of the range-maximum table: 2^(lv - 1) <= NB < 2^lv
    const size_t smem3 = size_t(lv) * d.NB * sizeof(float);
    if (smem3 > 48 * 1024) {
      cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(dphi_part3_kernel), int(smem3));
      if (e != cudaSuccess) return e;
    }
    cudaError_t e = launch_pdl(dphi_part3_kernel, dim3(d.BH()), dim3(1024), smem3, s, st.bmin, d.NB, lv,
                               kLog2e / tau, sc);
    if (e != cudaSuccess) return e;
    *launched += 1;
  }
  int threads = d.BT < 32 ? 32 : d.BT;
  size_t smem = (3 * size_t(d.NB) + 2 * d.BT + 32) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(dphi_kernel), int(smem));
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = launch_pdl(dphi_kernel, dim3(d.NB, d.H, d.B), dim3(threads), smem, s, phi, beta, d.B, d.H, d.T,
                             d.BT, d.NB, kLog2e / tau, st, sc, dphi, dbeta, quadratic ? 1 : 0);
  if (e == cudaSuccess) *launched += 1;
  return e;
}

// In-tile soft-min gradient of the diagonal tiles from their stored g (the tensor-core backward writes
// g_ts = dS_ts [x_ts <= 0] of each diagonal tile to `gd` [BH][NB][128][128], indexed [key s][query t]). For key s
// and Z_{s,t} = sum_{s<u<=t} 2^{a2_u} (kernel.py:269-283 evaluates the same sums with scans), with
// w_t = 2^{a2_t} / Z_{s,t} in (0, 1]:
//   H(t) = g_ts + (1 - w_{t+1}) H(t+1)    (Z_{s,t} / Z_{s,t+1} = 1 - w_{t+1}),   contribution to u = t: w_t H(t).
// Thread = key: w_t for all t of the tile stays in registers; the forward pass keeps Z as a scaled sum with its
// running maximum (one exp2 and one reciprocal per step), the reverse pass needs no transcendental. A warp's keys
// lie in [32 w, 32 w + 32), so it skips the 32-position blocks before its first key. The contributions are summed
// per u in a fixed order.
constexpr int kDiagBT = 128;

__global__ void __launch_bounds__(kDiagBT)
diag_dphi_kernel(const float* __restrict__ phi, const float* __restrict__ gd, int T, int NB, float il2,
                 float* __restrict__ dphi4) {
  constexpr int BT = kDiagBT, LD = BT + 1;
  extern __shared__ float dsm[];
  pdl_wait();  // launched with launch_pdl after the kv-pass, whose stored g it reads
  pdl_launch_dependents();
  float* G = dsm;           // [BT][BT+1]
  float* a2 = G + BT * LD;  // [BT]
  const int j = blockIdx.x, z = blockIdx.z * gridDim.y + blockIdx.y, sl = threadIdx.x, wq = sl >> 5;  // grid (NB, H, B)
  const size_t TP = size_t(NB) * BT;
  const float4* g4 = reinterpret_cast<const float4*>(gd + (size_t(z) * NB + j) * BT * BT);
  // All 32 loads of the thread in flight before the first store (the tile is 64 KB).
  {
    float4 v[BT * BT / 4 / BT];
#pragma unroll
    for (int q = 0; q < BT / 4; ++q) v[q] = g4[sl + q * BT];
#pragma unroll
    for (int q = 0; q < BT / 4; ++q) {
      const int e = sl + q * BT, row = (4 * e) / BT, col = (4 * e) % BT;
      G[row * LD + col] = v[q].x;
      G[row * LD + col + 1] = v[q].y;
      G[row * LD + col + 2] = v[q].z;
      G[row * LD + col + 3] = v[q].w;
    }
  }
  const int p0 = j * BT;
  a2[sl] = p0 + sl < T ? -phi[size_t(z) * T + p0 + sl] * il2 : -kInf;
  __syncthreads();
  const int tend = min(BT, T - p0);
  float w[BT];
  // Forward: Z_{s,t} = zz 2^{mz} over t = s+1 .. tend-1.
  float mz = -kInf, zz = 0.f;
#pragma unroll
  for (int tb = 0; tb < BT / 32; ++tb) {
    if (tb < wq) continue;  // warp-uniform
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int t = 32 * tb + i;
      const float at = a2[t];
      const float d = at - mz;
      const bool up = d > 0.f;
      const float e = ex2(-fabsf(d));  // d = +inf on the first term: e = 0
      const bool on = t > sl && t < tend;
      const float znew = up ? fmaf(zz, e, 1.f) : zz + e;
      const float term = up ? 1.f : e;
      zz = on ? znew : zz;
      mz = (on && up) ? at : mz;
      w[t] = on ? term * rcp_approx_f(znew) : 0.f;
    }
  }
  // Reverse: H and the contributions, written over g in place.
  float Hh = 0.f, wn = 0.f;  // w_{t+1}
#pragma unroll
  for (int tb = BT / 32 - 1; tb >= 0; --tb) {
    if (tb < wq) continue;  // warp-uniform
#pragma unroll
    for (int i = 31; i >= 0; --i) {
      const int t = 32 * tb + i;
      const bool on = t > sl && t < tend;
      const float hn = fmaf(1.f - wn, Hh, G[sl * LD + t]);
      Hh = on ? hn : 0.f;
      if (on) G[sl * LD + t] = w[t] * Hh;
      wn = w[t];
    }
  }
  __syncthreads();
  if (sl < tend) {
    // Four interleaved partial sums (keys s2 = 0, 1, 2, 3 mod 4), joined in a fixed order.
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int s2 = 0;
    for (; s2 + 4 <= sl; s2 += 4) {
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] += G[(s2 + q) * LD + sl];
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
      if (s2 + q < sl) acc[q] += G[(s2 + q) * LD + sl];
    dphi4[size_t(z) * TP + p0 + sl] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
}

cudaError_t launch_diag_dphi(const float* phi, const float* gd, const Dims& d, float tau, float* dphi4, cudaStream_t s) {
  if (d.BT != kDiagBT) return cudaErrorInvalidValue;
  const int smem = (kDiagBT * (kDiagBT + 1) + kDiagBT) * int(sizeof(float));
  cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(diag_dphi_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(diag_dphi_kernel, dim3(d.NB, d.H, d.B), dim3(kDiagBT), smem, s, phi, gd, d.T, d.NB, kLog2e / tau,
                    dphi4);
}


}  // namespace fpa
