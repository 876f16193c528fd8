// Tensor-core forward pass of FPA for sm_100a (fp16 q, k, v; fp32 accumulation).
//
// One CTA computes two query tiles of 128 rows (i0 = 2m, i1 = 2m + 1) of one head and walks their key tiles from
// the diagonal backwards (the order of kernel.py:104-162), so that the minimum of phi over the key tiles already
// passed, `mid`, is a running minimum. Warp roles (384 threads; warps 10-11 only hand their registers to the softmax groups):
//   warps 0-3  softmax group 0 (query tile i0; thread = row = TMEM lane)
//   warps 4-7  softmax group 1 (query tile i1)
//   warp  8    TMA producer: Q tiles once, then K, V tiles and the per-key vectors through an NS-stage ring
//   warp  9    MMA issuer (one thread): S_x = Q_x K^T into TMEM, O_x += P_x V with P_x read from TMEM
// TMEM (512 columns): NSLOT slots of 128 columns for S (three for D <= 64, two for D = 128), then O0 and O1 (D
// each). The jobs (key step k, group x) run in order n = 0, 1, ...; job n uses slot n % NSLOT, so the S of a
// group's next key tile is computed while it still works on the current one. P (fp16, packed two per column)
// overwrites the first 64 columns of its slot after the softmax has read S.
//
// The bias of query t (tile i) and key s (tile j) in log2 units is b' * min(0, x_ts), b' = beta * log2 e, with
//   off-diagonal (j < i):  b' min(0, x_ts) = min(b' a_s, b' min(mid_ij, PRE_t) - b' psi_s),  a_s = min(SUF_s - psi_s, 0)
//   diagonal (j == i):     x_ts = min_{s<u<=t} phi_u - psi_s, a running minimum along the row (keys descending);
// the per-key terms come pre-scaled by b' (stats_kernel), and for b' < 0 every minimum becomes a maximum.
// The online softmax rescales O lazily: the running maximum only moves when it grows by more than 8 (log2), so P
// stays below 2^8 and most tiles need no O correction.
//
// Synchronisation (all mbarriers, every wait bounded by fpa::sm100::mbar_wait):
//   q_full              producer -> MMA       (TMA bytes)
//   k_full[s], v_full[s] producer -> MMA, softmax (TMA / bulk bytes)
//   kv_empty[s]         MMA commit -> producer (stage s free again)
//   s_full[slot]        MMA commit -> softmax (S of the slot's job ready)
//   p_full[slot]        softmax (128 arrivals) -> MMA (P of the slot's job in TMEM, O_x corrected)
//   o_ready[x]          MMA commit -> softmax x (the group's previous O_x += P V completed: O_x may be rescaled)
//   o_done[x]           MMA commit -> softmax x (final O_x complete)
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <queue>
#include <type_traits>
#include <vector>

#include "fpa_sm100.cuh"
#include "fpa_tc.h"

namespace fpa {
using namespace sm100;

namespace {

constexpr int kBT = kTcBT;
constexpr int kThreads = 384;
constexpr int kWarpProducer = 8;
constexpr int kWarpMma = 9;
constexpr float kRescaleThreshold = 8.0f;

template <int D>
struct TcFwdCfg {
  static constexpr int BOXC = D >= 64 ? 64 : D;   // head-dim columns per TMA box (one swizzle row)
  static constexpr int NBOX = D / BOXC;           // boxes per [128 x D] tile
  static constexpr int SWB = BOXC * 2;            // bytes per row inside a box = swizzle width
  static constexpr int BOXB = kBT * SWB;          // bytes per box
  static constexpr int TILEB = NBOX * BOXB;       // bytes per [128 x D] tile
  static constexpr uint32_t SW = SWB == 128 ? kSwizzle128 : (SWB == 64 ? kSwizzle64 : kSwizzle32);
  static constexpr int NS = D >= 128 ? 2 : 3;     // K/V ring stages
  static constexpr int COLB = kBT * 4;            // bytes of one per-key vector
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * TILEB;
  static constexpr int OFF_V = OFF_K + NS * TILEB;
  static constexpr int OFF_COL = OFF_V + NS * TILEB;  // per stage: a, psi, phi
  static constexpr int OFF_BAR = OFF_COL + NS * 3 * COLB;
  static constexpr int NSLOT = D <= 64 ? 3 : 2;  // TMEM slots for S / P
  static constexpr int NBAR = 1 + 3 * NS + 2 * NSLOT + 2 + 2 + 1;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + TMEM slot + alignment slack
  static constexpr uint32_t IDESC_S = idesc_f16(kBT, kBT, 0);
  static constexpr uint32_t IDESC_O = idesc_f16(kBT, D, 1);
  static constexpr int COL_O = NSLOT * kBT;
  static_assert(COL_O + 2 * D <= 512, "TMEM columns");
  static constexpr int REG_LO = D >= 64 ? 40 : 24, REG_HI = D >= 64 ? 232 : 240;
  static_assert(128 * REG_LO + 256 * REG_HI == kThreads * 168, "register split");
};

struct TcFwdParams {
  const float* cola;   // [BH][TP]
  const float* colpsi;
  const float* colphi;
  const float* pre;    // [BH][TP]
  const float* bmin;   // [BH][NB]
  const float* beta;   // [H]
  __half* o;
  int64_t o_sb, o_sh, o_st;
  float* lse;          // [BH][T]
  int* status;
  int B, H, T, NB, TP, NPAIR;
  float scale2;        // D^-1/2 * log2(e)
};

// Key-range split of the one-tile kernel (L = 0: none): chunk c of query tile i covers key tiles i - c L down to
// max(0, i - c L - L + 1); a head's IPH chunks are numbered with i descending, c ascending. Query tiles with more
// than one chunk leave their unnormalised output in po [z * IPH + chunk][D / 4][128] (float4 groups of columns,
// rows innermost, so that a warp's stores and loads are coalesced) with the row maximum pm and row sum pl
// [z * IPH + chunk][128], and count themselves in cnt [z][i] (zeroed by the stats kernel); the chunk that counts
// last joins them. A separate kernel argument, so that the two-tile kernel's parameters stay as they are.
struct FwdSplitParams {
  int L, IPH;
  float4* po;
  float* pm;
  float* pl;
  int* cnt;
};

// AND of v over the 256 softmax threads of the one-tile kernel (named barrier 1; all of them call it).
__device__ __forceinline__ bool softmax_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

// With kEmuEvery > 0, every kEmuEvery-th pair of columns takes its exponentials on the FMA pipe instead of the
// MUFU unit (16 exp2 per clock per SM against 128 FMA lanes). Off by default: measured on B200 at configuration 2
// the forward is not MUFU-bound yet (no gain at 1/5 or 1/3 of the pairs) and the polynomial adds 1e-4 to lse.
#ifndef FPA_EMU_EVERY
#define FPA_EMU_EVERY 0
#endif
constexpr int kEmuEvery = FPA_EMU_EVERY;

// 2^x for a pair, on the FMA/ALU pipes: x = n + f with n = rint(x) (the 1.5 * 2^23 rounding trick), f in
// [-0.5, 0.5]; 2^f from a degree-3 polynomial fitted for this file by a reweighted least-squares minimax on
// [-0.5, 0.5] (max relative error 7.5e-5, below the fp16 rounding of P); 2^n is added to the exponent field.
// x is clamped at -125 so the exponent field of the result stays >= 1 for every f (2^-125 rounds to 0 in fp16).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 nf = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(nf, make_float2(-1.f, -1.f), x);
  float2 q = __ffma2_rn(make_float2(0.055171627551317215f, 0.055171627551317215f), f,
                        make_float2(0.2426111400127411f, 0.2426111400127411f));
  q = __ffma2_rn(q, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  q = __ffma2_rn(q, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  // Unsigned arithmetic: the shift drops the high bits of t, leaving n << 23 modulo 2^32.
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
tc_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
              const __grid_constant__ CUtensorMap tv, const TcFwdParams p) {
  using C = TcFwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base (the swizzle atoms of the UMMA operands), kept as an offset from smem_raw so the
  // compiler still sees shared-memory pointers.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + C::NS;
  uint64_t* kv_empty = v_full + C::NS;
  uint64_t* s_full = kv_empty + C::NS;  // [NSLOT]
  uint64_t* p_full = s_full + C::NSLOT;  // [NSLOT]
  uint64_t* o_ready = p_full + C::NSLOT;  // [2]
  uint64_t* o_done = o_ready + 2;        // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-d grid in longest-first order: all heads' pair NPAIR-1 (the most key tiles), then NPAIR-2, ... so the block
  // scheduler performs a longest-processing-time-first list schedule over the SMs.
  const int nbh = p.B * p.H;
  const int m = p.NPAIR - 1 - int(blockIdx.x) / nbh;
  const int z = int(blockIdx.x) % nbh, b = z / p.H, h = z % p.H;
  const int i0 = 2 * m, i1 = 2 * m + 1;
  const bool has1 = i1 < p.NB;
  const int jtop = has1 ? i1 : i0;
  const int nsteps = jtop + 1;
  const int k0 = has1 ? 1 : 0;  // first step in which query tile i0 takes part
  // Jobs in order: with both tiles (k, x) = (0, 1), (1, 0), (1, 1), (2, 0), ...; with one tile (k, 0).
  const int njobs = has1 ? 2 * nsteps - 1 : nsteps;
  auto job_k = [&](int n) { return has1 ? (n + 1) >> 1 : n; };
  auto job_x = [&](int n) { return has1 ? (n + 1) & 1 : 0; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int sl = 0; sl < C::NSLOT; ++sl) {
      mbar_init(s_full + sl, 1);
      mbar_init(p_full + sl, 128);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(o_ready + x, 1);
      mbar_init(o_done + x, 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched after the stats kernel with launch_pdl: the prologue above overlapped its last blocks.
  pdl_wait();
  pdl_launch_dependents();

  // Register split (per warpgroup): the launch gives 168 per thread; the producer/MMA group keeps C::REG_LO and
  // each softmax group takes C::REG_HI (128*40 + 256*232 = 128*24 + 256*240 = 384*168). With 224 the softmax
  // rows spilled to local memory.
  if (warp >= 8) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::REG_LO) : "memory");
  if (warp == kWarpProducer) {
    // The whole warp runs the loop (converged, uniform operands); one elected lane issues each copy.
    if (elect_one()) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
    }
    __syncwarp();
    uint8_t* sq = smem + C::OFF_Q;
    if (elect_one()) {
      mbar_expect_tx(q_full, (has1 ? 2 : 1) * C::TILEB);
      for (int bx = 0; bx < C::NBOX; ++bx) {
        tma_load_4d(sq + bx * C::BOXB, &tq, bx * C::BOXC, i0 * kBT, h, b, q_full);
        if (has1) tma_load_4d(sq + C::TILEB + bx * C::BOXB, &tq, bx * C::BOXC, i1 * kBT, h, b, q_full);
      }
    }
    __syncwarp();
    bool ok = true;
    const size_t colbase = size_t(z) * p.TP;
    for (int k = 0; k < nsteps && ok; ++k) {
      const int st = k % C::NS, j = jtop - k;
      if (k >= C::NS) ok = mbar_wait(kv_empty + st, ((k / C::NS) - 1) & 1, p.status, 1);
      if (!ok) break;
      uint8_t* sk = smem + C::OFF_K + st * C::TILEB;
      uint8_t* sv = smem + C::OFF_V + st * C::TILEB;
      uint8_t* sc = smem + C::OFF_COL + st * 3 * C::COLB;
      if (elect_one()) {
        mbar_expect_tx(k_full + st, C::TILEB + 3 * C::COLB);
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(sk + bx * C::BOXB, &tk, bx * C::BOXC, j * kBT, h, b, k_full + st);
        bulk_load(sc, p.cola + colbase + size_t(j) * kBT, C::COLB, k_full + st);
        bulk_load(sc + C::COLB, p.colpsi + colbase + size_t(j) * kBT, C::COLB, k_full + st);
        bulk_load(sc + 2 * C::COLB, p.colphi + colbase + size_t(j) * kBT, C::COLB, k_full + st);
        mbar_expect_tx(v_full + st, C::TILEB);
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(sv + bx * C::BOXB, &tv, bx * C::BOXC, j * kBT, h, b, v_full + st);
      }
      __syncwarp();
    }
    // Drain: wait (bounded) until the copies this warp issued have landed before the CTA may exit.
    mbar_wait(q_full, 0, p.status, 2);
    for (int k = (nsteps > C::NS ? nsteps - C::NS : 0); k < nsteps; ++k) {
      mbar_wait(k_full + k % C::NS, (k / C::NS) & 1, p.status, 3);
      mbar_wait(v_full + k % C::NS, (k / C::NS) & 1, p.status, 4);
    }
  } else if (warp == kWarpMma) {
    {  // The whole warp runs the loop (its waits included); one elected lane issues the MMAs and commits. The
       // descriptors are built once: each MMA then costs an add to the low word of its operands' descriptors.
      const bool leader = elect_one();
      constexpr uint32_t HI = desc_hi(8 * C::SWB, C::SW);
      const uint32_t lq = desc_lo(smem_u32(smem + C::OFF_Q), 16);
      const uint32_t lk = desc_lo(smem_u32(smem + C::OFF_K), 16);
      const uint32_t lv = desc_lo(smem_u32(smem + C::OFF_V), C::BOXB);
      auto issue_s = [&](int n) {  // S of job n into its slot
        const int x = job_x(n), st = job_k(n) % C::NS;
        const uint32_t la = lq + uint32_t(x * (C::TILEB >> 4)), lb = lk + uint32_t(st * (C::TILEB >> 4));
        const uint32_t dcol = tmem + (n % C::NSLOT) * kBT;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            constexpr int PER = C::SWB / 32;  // K-steps per swizzle row
            const uint32_t off = uint32_t(((kk / PER) * C::BOXB + (kk % PER) * 32) >> 4);
            mma_ss(dcol, desc_make(la + off, HI), desc_make(lb + off, HI), C::IDESC_S, kk > 0);
          }
          mma_commit(s_full + n % C::NSLOT);
        }
        __syncwarp();
      };
      auto issue_pv = [&](int n, bool acc) {  // O_x += P V of job n
        const int x = job_x(n), st = job_k(n) % C::NS;
        const uint32_t lb = lv + uint32_t(st * (C::TILEB >> 4));
        const uint32_t acol = tmem + (n % C::NSLOT) * kBT, dcol = tmem + C::COL_O + x * D;
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < kBT / 16; ++kk)
            mma_ts(dcol, acol + kk * 8, desc_make(lb + uint32_t((kk * 16 * C::SWB) >> 4), HI), C::IDESC_O,
                   (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, p.status, 10);
      int kload = -1, vload = -1;  // key steps whose K (V) stage is known to be loaded: up to kload (vload)
      auto need_k = [&](int kt) {
        if (ok && kt > kload) {
          ok = mbar_wait(k_full + kt % C::NS, (kt / C::NS) & 1, p.status, 11);
          kload = kt;
          tc_fence_after();
        }
        return ok;
      };
      tc_fence_after();
      for (int n = 0; n < C::NSLOT && n < njobs; ++n)
        if (need_k(job_k(n))) issue_s(n);
      for (int n = 0; n < njobs && ok; ++n) {
        const int k = job_k(n), x = job_x(n), st = k % C::NS;
        if (k > vload) {
          ok = mbar_wait(v_full + st, (k / C::NS) & 1, p.status, 12);
          vload = k;
          if (!ok) break;
        }
        ok = mbar_wait(p_full + n % C::NSLOT, (n / C::NSLOT) & 1, p.status, 13);
        if (!ok) break;
        tc_fence_after();
        issue_pv(n, x == 0 ? k > k0 : k > 0);
        if (leader) {
          mma_commit(o_ready + x);
          if (x == 1 || !has1) mma_commit(kv_empty + st);  // last job of key step k
        }
        __syncwarp();
        const int m = n + C::NSLOT;
        if (m < njobs && need_k(job_k(m))) issue_s(m);
      }
      mma_commit_w(o_done + 0);
      mma_commit_w(o_done + 1);
      // Drain: every MMA issued by this warp has completed before TMEM can be released.
      mma_commit_w(drain);
      mbar_wait(drain, 0, p.status, 16);
    }
  } else if (warp < 8) {
    // ----------------------------------------------------------------------------------- softmax groups ----
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::REG_HI) : "memory");
    const int x = warp >> 2, wr = warp & 3;
    const int r = wr * 32 + lane;
    const int i = x == 0 ? i0 : i1;
    const bool active_wg = (x == 0) || has1;
    const int t = i * kBT + r;
    const uint32_t tl = tmem + (uint32_t(wr * 32) << 16);
    const uint32_t col_o = C::COL_O + x * D;
    const float betal = p.beta[h] * kLog2e;
    const float pre_t = p.pre[size_t(z) * p.TP + t];
    const float* bmin = p.bmin + size_t(z) * p.NB;
    // The row sum is kept as two parts, keys [0, 64) and [64, 128) of every tile, added at the end: the same
    // order of additions as the one-tile kernel below, so both kernels give bit-identical results.
    float mrow = -kInf, lrow = 0.f, lrow2 = 0.f, mid = kInf;
    int cnt = 0;
    bool ok = active_wg;
    const int kfirst = x == 0 ? k0 : 0;
    // The bias in log2 units is b' * min(0, x) with b' = beta * log2 e. For b' >= 0 that is a minimum of the
    // pre-scaled per-key terms; for b' < 0 every minimum becomes a maximum (NEG).
    auto run = [&](auto neg_tag) {
      constexpr bool NEG = decltype(neg_tag)::value;
      auto ext = [](float a, float b2) { return NEG ? fmaxf(a, b2) : fminf(a, b2); };
      const float2 sc2 = make_float2(p.scale2, p.scale2);
      for (int k = kfirst; k < nsteps && ok; ++k) {
        const int j = jtop - k, st = k % C::NS;
        const int n = has1 ? 2 * k - 1 + x : k, slot = n % C::NSLOT;  // this group's job at step k
        const uint32_t col_s = slot * kBT;
        ok = mbar_wait(k_full + st, (k / C::NS) & 1, p.status, 20);
        if (ok) ok = mbar_wait(s_full + slot, (n / C::NSLOT) & 1, p.status, 21);
        if (!ok) break;
        tc_fence_after();
        float s[kBT];
#pragma unroll
        for (int c = 0; c < kBT / 32; ++c) tmem_ld32(tl + col_s + c * 32, s + c * 32);
        tmem_ld_wait();
        const float* cA = reinterpret_cast<const float*>(smem + C::OFF_COL + st * 3 * C::COLB);  // b'*min(SUF-psi,0)
        const float* cE = cA + kBT;                                                               // -b'*psi
        const float* cF = cA + 2 * kBT;                                                           // b'*phi
        if (j == i) {
          // Diagonal tile: keys from the row down; rr = extremum of b'*phi over (key, row] (+-inf when empty).
          float rr = NEG ? -kInf : kInf;
          const int lim = min(r, p.T - 1 - j * kBT);  // last valid key of this row
#pragma unroll
          for (int c = kBT - 1; c >= 0; --c) {
            const float bias = ext(0.f, rr + cE[c]);
            const float v = fmaf(s[c], p.scale2, bias);
            s[c] = c <= lim ? v : -kInf;
            if (c <= r) rr = ext(rr, cF[c]);
          }
        } else {
          // Off the diagonal: bias = ext(a_s, b' * min(mid, PRE_t) - b' * psi_s), two keys per packed op.
          const float R = betal * fminf(mid, pre_t);
          const float2 R2 = make_float2(R, R);
#pragma unroll
          for (int c = 0; c < kBT; c += 2) {
            const float2 e2 = *reinterpret_cast<const float2*>(cE + c);
            const float2 a2 = *reinterpret_cast<const float2*>(cA + c);
            const float2 tt = __fadd2_rn(R2, e2);
            const float2 bias = make_float2(ext(a2.x, tt.x), ext(a2.y, tt.y));
            const float2 v = __ffma2_rn(make_float2(s[c], s[c + 1]), sc2, bias);
            s[c] = v.x;
            s[c + 1] = v.y;
          }
          mid = fminf(mid, bmin[j]);  // tile j lies strictly between the next key tile and tile i
        }
        float m4[4] = {fmaxf(s[0], s[4]), fmaxf(s[1], s[5]), fmaxf(s[2], s[6]), fmaxf(s[3], s[7])};
#pragma unroll
        for (int c = 8; c < kBT; c += 8) {
          m4[0] = fmax3f(m4[0], s[c], s[c + 4]);
          m4[1] = fmax3f(m4[1], s[c + 1], s[c + 5]);
          m4[2] = fmax3f(m4[2], s[c + 2], s[c + 6]);
          m4[3] = fmax3f(m4[3], s[c + 3], s[c + 7]);
        }
        const float mt = fmaxf(fmax3f(m4[0], m4[1], m4[2]), m4[3]);
        // Lazy rescaling of the running maximum.
        const float mnew = fmaxf(mrow, mt);
        bool need = false;
        float alpha = 1.f;
        if (cnt == 0) {
          mrow = mnew;
        } else if (mnew > mrow + kRescaleThreshold) {
          need = true;
          alpha = ex2(mrow - mnew);
          mrow = mnew;
        }
        // The group's previous O += P V must be complete before O is touched (and before this job's P is handed on).
        if (cnt > 0) {
          ok = mbar_wait(o_ready + x, (cnt - 1) & 1, p.status, 23);
          if (!ok) break;
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, need)) {
          lrow *= alpha;
          lrow2 *= alpha;
#pragma unroll
          for (int c = 0; c < D; c += 16) {
            float o[16];
            tmem_ld16(tl + col_o + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] *= alpha;
            tmem_st16(tl + col_o + c, reinterpret_cast<const uint32_t*>(o));
          }
        }
        const float2 nm2 = make_float2(-mrow, -mrow);
        float2 ls = make_float2(0.f, 0.f), ls2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c0 = 0; c0 < kBT; c0 += 32) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 xx = __fadd2_rn(make_float2(s[c0 + e], s[c0 + e + 1]), nm2);
            const bool emu = kEmuEvery > 0 && ((c0 + e) / 2) % (kEmuEvery > 0 ? kEmuEvery : 1) == 0;
            const float2 pp = emu ? ex2_poly2(xx) : make_float2(ex2(xx.x), ex2(xx.y));
            if (c0 < kBT / 2)
              ls = __fadd2_rn(ls, pp);
            else
              ls2 = __fadd2_rn(ls2, pp);
            pk[e / 2] = pack_half2(pp.x, pp.y);
          }
          tmem_st16(tl + col_s + c0 / 2, pk);
        }
        lrow += ls.x + ls.y;
        lrow2 += ls2.x + ls2.y;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full + slot);
        ++cnt;
      }
    };
    if (betal < 0.f)
      run(std::true_type{});
    else
      run(std::false_type{});
    if (ok && active_wg) ok = mbar_wait(o_done + x, 0, p.status, 22);
    if (ok && active_wg) {
      tc_fence_after();
      lrow += lrow2;
      const float inv = 1.f / lrow;
      const bool store = t < p.T;
      __half* orow = p.o + b * p.o_sb + h * p.o_sh + int64_t(store ? t : 0) * p.o_st;
#pragma unroll
      for (int c = 0; c < D; c += 16) {
        float o[16];
        tmem_ld16(tl + col_o + c, o);
        tmem_ld_wait();
        if (store) {
          uint4 w0, w1;
          w0.x = pack_half2(o[0] * inv, o[1] * inv);
          w0.y = pack_half2(o[2] * inv, o[3] * inv);
          w0.z = pack_half2(o[4] * inv, o[5] * inv);
          w0.w = pack_half2(o[6] * inv, o[7] * inv);
          w1.x = pack_half2(o[8] * inv, o[9] * inv);
          w1.y = pack_half2(o[10] * inv, o[11] * inv);
          w1.z = pack_half2(o[12] * inv, o[13] * inv);
          w1.w = pack_half2(o[14] * inv, o[15] * inv);
          reinterpret_cast<uint4*>(orow + c)[0] = w0;
          reinterpret_cast<uint4*>(orow + c)[1] = w1;
        }
      }
      if (store) p.lse[size_t(z) * p.T + t] = mrow + lg2(lrow);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------------------
// One query tile per CTA, two CTAs per SM, each row shared by two threads (D <= 64).
//
// The CTA takes query tile i of one head and walks its key tiles j = i, i - 1, ..., 0 (the diagonal first, as
// above). It holds 256 TMEM columns: S [0, 128), P [128, 192) (fp16 pairs), O [192, 192 + D). Two CTAs share an
// SM, so one CTA's prologue, pipeline fill and epilogue run while the other computes, and single-tile CTAs balance
// over the SMs better than two-tile ones (and fill more of them when a GPU holds few heads). S has one slot: the
// softmax hands it back (s_free) as soon as it has read S, and the MMA warp computes the next S meanwhile; P has
// columns of its own and is rewritten only after the previous P V has completed (o_ready).
// Each S row is shared by two softmax threads, one per half of the key columns (threads of warps w and w + 4 see
// the same TMEM lanes), which doubles the warps per SM sub-partition that take turns hiding each other's latency.
// The halves agree on the row maximum through shared memory once per key tile (a 64-thread named barrier per
// lane quadrant, whose 64 threads meet on an mbarrier of their own), keep their own partial row sums and rescale
// their own half of O.
// Warps (384 threads): 0-3 and 4-7 the two halves (thread = row = TMEM lane), 8 TMA producer, 9 MMA issuer, 10-11
// only complete the third warpgroup (setmaxnreg acts per warpgroup).
//
// Synchronisation (all mbarriers, every wait bounded):
//   q_full                     producer -> MMA
//   k_full[s], v_full[s]       producer -> MMA, softmax (K, V tiles and the per-key vectors of stage s)
//   kv_empty[s]                MMA commit -> producer (stage s free again)
//   s_full                     MMA commit -> softmax (S of the next key tile ready)
//   s_free                     softmax (256 arrivals) -> MMA (S read: the slot may take the next S)
//   p_full                     softmax (256 arrivals) -> MMA (P in TMEM, O corrected)
//   o_ready                    MMA commit -> softmax (the previous O += P V completed)
//   o_done                     MMA commit -> softmax (final O complete)
//   x_pair[q]                  the two softmax threads of each row of lane quadrant q (64 arrivals): row maxima
//                              (once per key tile) and the partial row sums (once at the end) exchanged
constexpr int kThreads1 = 384;
constexpr int kSoftmaxThreads1 = 256;
constexpr int kWarpProducer1 = 8;
constexpr int kWarpMma1 = 9;
constexpr int kHalf = kBT / 2;  // key columns per softmax thread

template <int D>
struct Fwd1Cfg {
  static constexpr int BOXC = D >= 64 ? 64 : D;
  static constexpr int NBOX = D / BOXC;
  static constexpr int SWB = BOXC * 2;
  static constexpr int BOXB = kBT * SWB;
  static constexpr int TILEB = NBOX * BOXB;
  static constexpr uint32_t SW = SWB == 128 ? kSwizzle128 : (SWB == 64 ? kSwizzle64 : kSwizzle32);
  static constexpr int NS = 2;                      // K/V ring stages
  static constexpr int COLB = kBT * 4;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILEB;
  static constexpr int OFF_V = OFF_K + NS * TILEB;
  static constexpr int OFF_COL = OFF_V + NS * TILEB;  // per stage: a, psi, phi
  static constexpr int OFF_X = OFF_COL + NS * 3 * COLB;  // row maxima of the halves [2 parities][2 halves][128]
  static constexpr int OFF_BAR = OFF_X + 2 * 2 * kBT * 4;
  static constexpr int NBAR = 1 + 3 * NS + 6 + 4;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int COL_S = 0, COL_P = kBT, COL_O = kBT + kBT / 2;
  static constexpr int TMEM_COLS = 256;
  static constexpr uint32_t IDESC_S = idesc_f16(kBT, kBT, 0);
  static constexpr uint32_t IDESC_O = idesc_f16(kBT, D, 1);
  static_assert(D <= 64 && COL_O + D <= TMEM_COLS, "TMEM columns");
  static_assert(2 * SMEM <= 228 * 1024, "two CTAs per SM");
};

template <int D>
__global__ void __launch_bounds__(kThreads1, 2)
tc_fwd1_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const TcFwdParams p, const FwdSplitParams sp) {
  using C = Fwd1Cfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + C::NS;
  uint64_t* kv_empty = v_full + C::NS;
  uint64_t* s_full = kv_empty + C::NS;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_free + 1;
  uint64_t* o_ready = p_full + 1;
  uint64_t* o_done = o_ready + 1;
  uint64_t* drain = o_done + 1;
  uint64_t* x_pair = drain + 1;  // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_pair + 4);
  float* xmax = reinterpret_cast<float*>(smem + C::OFF_X);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-d grid in longest-first order: every head's last query tile (the most key tiles) first. With a key-range
  // split the CTA takes one chunk: key tiles jhi, jhi - 1, ..., jlo of query tile i.
  const int nbh = p.B * p.H;
  const int z = int(blockIdx.x) % nbh, b = z / p.H, h = z % p.H;
  int i = p.NB - 1 - int(blockIdx.x) / nbh, jhi = i, jlo = 0, slot = -1;
  if (sp.L > 0) {
    const int u0 = int(blockIdx.x) / nbh;
    int u = u0;
    for (i = p.NB - 1; i > 0; --i) {
      const int nc = (i + sp.L) / sp.L;
      if (u < nc) break;
      u -= nc;
    }
    jhi = i - u * sp.L;
    jlo = max(0, jhi - sp.L + 1);
    if (i >= sp.L) slot = z * sp.IPH + u0;  // more than one chunk: partial output
  }
  const int nsteps = jhi - jlo + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, kSoftmaxThreads1);
    mbar_init(p_full, kSoftmaxThreads1);
    mbar_init(o_ready, 1);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    for (int qq = 0; qq < 4; ++qq) mbar_init(x_pair + qq, 64);
    fence_mbar_init();
  }
  if (warp == kWarpMma1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched after the stats kernel with launch_pdl: the prologue above overlapped its last blocks.
  pdl_wait();
  pdl_launch_dependents();

  // Register split: 80 per thread at launch (two CTAs per SM); the softmax warpgroups take 104, the third 32.
  if (warp >= 8) asm volatile("setmaxnreg.dec.sync.aligned.u32 32;" ::: "memory");
  if (warp == kWarpProducer1) {
    if (elect_one()) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
    }
    __syncwarp();
    uint8_t* sq = smem + C::OFF_Q;
    if (elect_one()) {
      mbar_expect_tx(q_full, C::TILEB);
      for (int bx = 0; bx < C::NBOX; ++bx) tma_load_4d(sq + bx * C::BOXB, &tq, bx * C::BOXC, i * kBT, h, b, q_full);
    }
    __syncwarp();
    bool ok = true;
    const size_t colbase = size_t(z) * p.TP;
    for (int k = 0; k < nsteps && ok; ++k) {
      const int st = k % C::NS, j = jhi - k;
      if (k >= C::NS) ok = mbar_wait(kv_empty + st, ((k / C::NS) - 1) & 1, p.status, 31);
      if (!ok) break;
      uint8_t* sk = smem + C::OFF_K + st * C::TILEB;
      uint8_t* sv = smem + C::OFF_V + st * C::TILEB;
      uint8_t* sc = smem + C::OFF_COL + st * 3 * C::COLB;
      if (elect_one()) {
        mbar_expect_tx(k_full + st, C::TILEB + 3 * C::COLB);
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(sk + bx * C::BOXB, &tk, bx * C::BOXC, j * kBT, h, b, k_full + st);
        bulk_load(sc, p.cola + colbase + size_t(j) * kBT, C::COLB, k_full + st);
        bulk_load(sc + C::COLB, p.colpsi + colbase + size_t(j) * kBT, C::COLB, k_full + st);
        bulk_load(sc + 2 * C::COLB, p.colphi + colbase + size_t(j) * kBT, C::COLB, k_full + st);
        mbar_expect_tx(v_full + st, C::TILEB);
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_4d(sv + bx * C::BOXB, &tv, bx * C::BOXC, j * kBT, h, b, v_full + st);
      }
      __syncwarp();
    }
    // Drain: wait (bounded) until the copies this warp issued have landed before the CTA may exit.
    mbar_wait(q_full, 0, p.status, 32);
    for (int k = (nsteps > C::NS ? nsteps - C::NS : 0); k < nsteps; ++k) {
      mbar_wait(k_full + k % C::NS, (k / C::NS) & 1, p.status, 33);
      mbar_wait(v_full + k % C::NS, (k / C::NS) & 1, p.status, 34);
    }
  } else if (warp == kWarpMma1) {
    // The whole warp runs the loop; one elected lane issues the MMAs and commits, from descriptors built once.
    const bool leader = elect_one();
    constexpr uint32_t HI = desc_hi(8 * C::SWB, C::SW);
    const uint32_t lq = desc_lo(smem_u32(smem + C::OFF_Q), 16);
    const uint32_t lk = desc_lo(smem_u32(smem + C::OFF_K), 16);
    const uint32_t lv = desc_lo(smem_u32(smem + C::OFF_V), C::BOXB);
    auto issue_s = [&](int k) {  // S = Q K^T of key step k into the S slot
      const uint32_t lb = lk + uint32_t((k % C::NS) * (C::TILEB >> 4));
      if (leader) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr int PER = C::SWB / 32;
          const uint32_t off = uint32_t(((kk / PER) * C::BOXB + (kk % PER) * 32) >> 4);
          mma_ss(tmem + C::COL_S, desc_make(lq + off, HI), desc_make(lb + off, HI), C::IDESC_S, kk > 0);
        }
        mma_commit(s_full);
      }
      __syncwarp();
    };
    auto issue_pv = [&](int k) {  // O += P V of key step k, then the commits that release O and the K/V stage
      const uint32_t lb = lv + uint32_t((k % C::NS) * (C::TILEB >> 4));
      if (leader) {
#pragma unroll
        for (int kk = 0; kk < kBT / 16; ++kk)
          mma_ts(tmem + C::COL_O, tmem + C::COL_P + kk * 8, desc_make(lb + uint32_t((kk * 16 * C::SWB) >> 4), HI),
                 C::IDESC_O, (k > 0 || kk > 0) ? 1u : 0u);
        mma_commit(o_ready);
        mma_commit(kv_empty + k % C::NS);
      }
      __syncwarp();
    };
    bool ok = mbar_wait(q_full, 0, p.status, 40);
    if (ok) ok = mbar_wait(k_full, 0, p.status, 41);
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int k = 0; k < nsteps && ok; ++k) {
      if (k + 1 < nsteps) {
        // The next S as soon as the softmax has read this one out of the slot (K of step k + 1 was released by
        // the P V of step k - 1, already issued).
        ok = mbar_wait(s_free, k & 1, p.status, 42);
        if (ok) ok = mbar_wait(k_full + (k + 1) % C::NS, ((k + 1) / C::NS) & 1, p.status, 43);
        if (!ok) break;
        tc_fence_after();
        issue_s(k + 1);
      }
      ok = mbar_wait(p_full, k & 1, p.status, 44);
      if (ok) ok = mbar_wait(v_full + k % C::NS, (k / C::NS) & 1, p.status, 45);
      if (!ok) break;
      tc_fence_after();
      issue_pv(k);
    }
    mma_commit_w(o_done);
    // Drain: every MMA issued by this warp has completed before TMEM can be released.
    mma_commit_w(drain);
    mbar_wait(drain, 0, p.status, 46);
  } else if (warp < 8) {
    // ------------------------------------------------------------------------------------------- softmax ----
    asm volatile("setmaxnreg.inc.sync.aligned.u32 104;" ::: "memory");
    const int q = warp & 3, half = warp >> 2;
    const int r = q * 32 + lane;
    const int t = i * kBT + r;
    const int c0h = half * kHalf;  // first key column of this thread's half
    const uint32_t tl = tmem + (uint32_t(q * 32) << 16);
    const float betal = p.beta[h] * kLog2e;
    const float pre_t = p.pre[size_t(z) * p.TP + t];
    const float* bmin = p.bmin + size_t(z) * p.NB;
    float mrow = -kInf, lrow = 0.f, mid = kInf;  // lrow: this half's part of the row sum
    for (int jj = jhi + 1; jj < i; ++jj) mid = fminf(mid, bmin[jj]);  // a chunk below the diagonal
    bool ok = true;
    // Exchange with the other half of the row through buffer `buf` ([2][128]) at exchange number `ph`: publish
    // v, meet on x_pair[q] (bounded wait), return the partner's value.
    auto exchange = [&](float* buf, float v, int ph) {
      buf[half * kBT + r] = v;
      mbar_arrive(x_pair + q);
      ok = ok && mbar_wait(x_pair + q, ph & 1, p.status, 54);
      return buf[(1 - half) * kBT + r];
    };
    auto run = [&](auto neg_tag) {
      constexpr bool NEG = decltype(neg_tag)::value;
      auto ext = [](float a, float b2) { return NEG ? fmaxf(a, b2) : fminf(a, b2); };
      const float2 sc2 = make_float2(p.scale2, p.scale2);
      for (int k = 0; k < nsteps && ok; ++k) {
        const int j = jhi - k, st = k % C::NS;
        ok = mbar_wait(k_full + st, (k / C::NS) & 1, p.status, 50);
        if (ok) ok = mbar_wait(s_full, k & 1, p.status, 51);
        if (!ok) break;
        tc_fence_after();
        float s[kHalf];
        tmem_ld32(tl + C::COL_S + c0h, s);
        tmem_ld32(tl + C::COL_S + c0h + 32, s + 32);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(s_free);  // the slot may take the next S now
        const float* cA = reinterpret_cast<const float*>(smem + C::OFF_COL + st * 3 * C::COLB) + c0h;
        const float* cE = cA + kBT;       // -b'*psi
        const float* cF = cA + 2 * kBT;   // b'*phi
        if (j == i) {
          // Diagonal tile: keys from the row down; rr = extremum of b'*phi over (key, row] (+-inf when empty). The
          // lower half starts from the extremum over the upper half's keys up to the row.
          float rr = NEG ? -kInf : kInf;
          if (half == 0) {
#pragma unroll 8
            for (int c = 0; c < kHalf; ++c)
              if (kHalf + c <= r) rr = ext(rr, cF[kHalf + c]);
          }
          const int lim = min(r, p.T - 1 - j * kBT) - c0h;  // last valid key of this row, in this half
          const int rh = r - c0h;
#pragma unroll
          for (int c = kHalf - 1; c >= 0; --c) {
            const float bias = ext(0.f, rr + cE[c]);
            const float v = fmaf(s[c], p.scale2, bias);
            s[c] = c <= lim ? v : -kInf;
            if (c <= rh) rr = ext(rr, cF[c]);
          }
        } else {
          // Off the diagonal: bias = ext(a_s, b' * min(mid, PRE_t) - b' * psi_s), two keys per packed op.
          const float R = betal * fminf(mid, pre_t);
          const float2 R2 = make_float2(R, R);
#pragma unroll
          for (int c = 0; c < kHalf; c += 2) {
            const float2 e2 = *reinterpret_cast<const float2*>(cE + c);
            const float2 a2 = *reinterpret_cast<const float2*>(cA + c);
            const float2 tt = __fadd2_rn(R2, e2);
            const float2 bias = make_float2(ext(a2.x, tt.x), ext(a2.y, tt.y));
            const float2 v = __ffma2_rn(make_float2(s[c], s[c + 1]), sc2, bias);
            s[c] = v.x;
            s[c + 1] = v.y;
          }
          mid = fminf(mid, bmin[j]);  // tile j lies strictly between the next key tile and tile i
        }
        float m4[4] = {fmaxf(s[0], s[4]), fmaxf(s[1], s[5]), fmaxf(s[2], s[6]), fmaxf(s[3], s[7])};
#pragma unroll
        for (int c = 8; c < kHalf; c += 8) {
          m4[0] = fmax3f(m4[0], s[c], s[c + 4]);
          m4[1] = fmax3f(m4[1], s[c + 1], s[c + 5]);
          m4[2] = fmax3f(m4[2], s[c + 2], s[c + 6]);
          m4[3] = fmax3f(m4[3], s[c + 3], s[c + 7]);
        }
        // The row maximum: each half publishes its own, then both read the other's (double-buffered by key step,
        // so a half that runs one step ahead never overwrites a value its partner has yet to read).
        const float mh = fmaxf(fmax3f(m4[0], m4[1], m4[2]), m4[3]);
        const float mt = fmaxf(mh, exchange(xmax + (k & 1) * 2 * kBT, mh, k));
        if (!ok) break;
        // Lazy rescaling of the running maximum (both halves of a row take the same decision).
        const float mnew = fmaxf(mrow, mt);
        bool need = false;
        float alpha = 1.f;
        if (k == 0) {
          mrow = mnew;
        } else if (mnew > mrow + kRescaleThreshold) {
          need = true;
          alpha = ex2(mrow - mnew);
          mrow = mnew;
        }
        // The previous O += P V must be complete before O is touched and before P is rewritten.
        if (k > 0) {
          ok = mbar_wait(o_ready, (k - 1) & 1, p.status, 53);
          if (!ok) break;
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, need)) {  // this half's columns of O
          lrow *= alpha;
#pragma unroll
          for (int c = 0; c < D / 2; c += 8) {
            float o[8];
            tmem_ld8(tl + C::COL_O + half * (D / 2) + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] *= alpha;
            tmem_st8(tl + C::COL_O + half * (D / 2) + c, reinterpret_cast<const uint32_t*>(o));
          }
        }
        const float2 nm2 = make_float2(-mrow, -mrow);
        float2 ls = make_float2(0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < kHalf; cc += 32) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 xx = __fadd2_rn(make_float2(s[cc + e], s[cc + e + 1]), nm2);
            const float2 pp = make_float2(ex2(xx.x), ex2(xx.y));
            ls = __fadd2_rn(ls, pp);
            pk[e / 2] = pack_half2(pp.x, pp.y);
          }
          tmem_st16(tl + C::COL_P + (c0h + cc) / 2, pk);
        }
        lrow += ls.x + ls.y;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full);
      }
    };
    if (betal < 0.f)
      run(std::true_type{});
    else
      run(std::false_type{});
    // The row sum is the two halves' parts; the halves share it through the row-maximum buffer.
    float l = lrow;
    if (ok) l += exchange(xmax + (nsteps & 1) * 2 * kBT, lrow, nsteps);
    if (ok) ok = mbar_wait(o_done, 0, p.status, 52);
    ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the TMEM loads below are warp-collective
    if (slot >= 0) {
      // One chunk of several: the unnormalised output, row maximum and row sum, made visible (fence) before the
      // chunk counts itself; the chunk that counts last joins all chunks of query tile i in chunk order (the same
      // order whichever chunk that is): M = max of the row maxima, l = sum of l_c 2^(m_c - M), O = sum of
      // O_c 2^(m_c - M), then o = O / l and lse = M + log2 l as the unsplit kernel writes them. Every softmax
      // thread reaches the barriers below (a timed-out wait leaves ok false but no thread behind).
      if (ok) {
        tc_fence_after();
        float4* pcol = sp.po + size_t(slot) * (D / 4) * kBT + (half * (D / 8)) * kBT + r;
#pragma unroll
        for (int c = 0; c < D / 2; c += 8) {
          float o[8];
          tmem_ld8(tl + C::COL_O + half * (D / 2) + c, o);
          tmem_ld_wait();
          pcol[(c / 4) * kBT] = make_float4(o[0], o[1], o[2], o[3]);
          pcol[(c / 4 + 1) * kBT] = make_float4(o[4], o[5], o[6], o[7]);
        }
        if (half == 0) {
          sp.pm[size_t(slot) * kBT + r] = mrow;
          sp.pl[size_t(slot) * kBT + r] = l;
        }
        __threadfence();
      }
      const int nc = (i + sp.L) / sp.L;
      uint32_t* join = tmem_slot + 1;
      if (softmax_all(ok) && threadIdx.x == 0) join[0] = atomicAdd(sp.cnt + size_t(z) * p.NB + i, 1) == nc - 1;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (join[0] && ok) {
        __threadfence();
        int base = 0;  // chunks of the query tiles after i
        for (int ii = p.NB - 1; ii > i; --ii) base += (ii + sp.L) / sp.L;
        const size_t s0 = size_t(z) * sp.IPH + base;
        float M = -kInf;
        for (int c = 0; c < nc; ++c) M = fmaxf(M, __ldcg(sp.pm + (s0 + c) * kBT + r));
        float lt = 0.f, acc[D / 2];
#pragma unroll
        for (int e = 0; e < D / 2; ++e) acc[e] = 0.f;
        for (int c = 0; c < nc; ++c) {
          const float w = ex2(__ldcg(sp.pm + (s0 + c) * kBT + r) - M);
          lt = fmaf(__ldcg(sp.pl + (s0 + c) * kBT + r), w, lt);
          const float4* src = sp.po + ((s0 + c) * (D / 4) + half * (D / 8)) * kBT + r;
#pragma unroll
          for (int e = 0; e < D / 8; ++e) {
            const float4 v = __ldcg(src + e * kBT);
            acc[4 * e] = fmaf(v.x, w, acc[4 * e]);
            acc[4 * e + 1] = fmaf(v.y, w, acc[4 * e + 1]);
            acc[4 * e + 2] = fmaf(v.z, w, acc[4 * e + 2]);
            acc[4 * e + 3] = fmaf(v.w, w, acc[4 * e + 3]);
          }
        }
        if (t < p.T) {
          const float inv = 1.f / lt;
          __half* orow = p.o + b * p.o_sb + h * p.o_sh + int64_t(t) * p.o_st + half * (D / 2);
#pragma unroll
          for (int e = 0; e < D / 2; e += 8) {
            uint4 w0;
            w0.x = pack_half2(acc[e] * inv, acc[e + 1] * inv);
            w0.y = pack_half2(acc[e + 2] * inv, acc[e + 3] * inv);
            w0.z = pack_half2(acc[e + 4] * inv, acc[e + 5] * inv);
            w0.w = pack_half2(acc[e + 6] * inv, acc[e + 7] * inv);
            reinterpret_cast<uint4*>(orow + e)[0] = w0;
          }
          if (half == 0) p.lse[size_t(z) * p.T + t] = M + lg2(lt);
        }
      }
    } else if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;
      const bool store = t < p.T;
      __half* orow = p.o + b * p.o_sb + h * p.o_sh + int64_t(store ? t : 0) * p.o_st + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 2; c += 8) {
        float o[8];
        tmem_ld8(tl + C::COL_O + half * (D / 2) + c, o);
        tmem_ld_wait();
        if (store) {
          uint4 w0;
          w0.x = pack_half2(o[0] * inv, o[1] * inv);
          w0.y = pack_half2(o[2] * inv, o[3] * inv);
          w0.z = pack_half2(o[4] * inv, o[5] * inv);
          w0.w = pack_half2(o[6] * inv, o[7] * inv);
          reinterpret_cast<uint4*>(orow + c)[0] = w0;
        }
      }
      if (store && half == 0) p.lse[size_t(z) * p.T + t] = mrow + lg2(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Chunks per head with chunks of L key tiles: query tile i has ceil((i + 1) / L) of them.
int chunks_per_head(int NB, int L) {
  int n = 0;
  for (int i = 0; i < NB; ++i) n += (i + L) / L;
  return n;
}

TcFwdParams fwd_params(const FpaFwdArgs& a, const Dims& d, const Stats& st, const KeyCols& cols, int* status) {
  TcFwdParams p;
  p.cola = cols.a;
  p.colpsi = cols.psi;
  p.colphi = cols.phi;
  p.pre = st.pre;
  p.bmin = st.bmin;
  p.beta = a.beta;
  p.o = static_cast<__half*>(a.o);
  p.o_sb = a.o_stride[0];
  p.o_sh = a.o_stride[1];
  p.o_st = a.o_stride[2];
  p.lse = a.lse;
  p.status = status;
  p.B = d.B;
  p.H = d.H;
  p.T = d.T;
  p.NB = d.NB;
  p.TP = d.TP;
  p.NPAIR = 0;
  p.scale2 = float(1.0 / sqrt(double(d.D))) * kLog2e;
  return p;
}

// One-tile forward (with sp.L > 0, the chunks of the key-range split, joined in the kernel). Sets *launched.
template <int D>
int launch1(const FpaFwdArgs& a, const Dims& d, const Stats& st, const KeyCols& cols, const FwdSplit& sp,
            char* split_ws, int* status, cudaStream_t s, int* launched, std::string* err) {
  using C = Fwd1Cfg<D>;
  CUtensorMap mq, mk, mv;
  if (!make_tile_map(&mq, a.q, a.q_stride, d.B, d.H, d.T, D) || !make_tile_map(&mk, a.k, a.k_stride, d.B, d.H, d.T, D) ||
      !make_tile_map(&mv, a.v, a.v_stride, d.B, d.H, d.T, D)) {
    *err = "cuTensorMapEncodeTiled failed for q, k or v";
    return FPA_ERR_CUDA;
  }
  auto fn = tc_fwd1_kernel<D>;
  cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(fn), C::SMEM);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core forward: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  const TcFwdParams p = fwd_params(a, d, st, cols, status);
  FwdSplitParams q{0, 0, nullptr, nullptr, nullptr, nullptr};
  int grid = d.NB * d.BH();
  if (sp.L > 0) {
    const size_t n = size_t(d.BH()) * sp.items_per_head * kBT;
    const size_t nc = align256(size_t(d.BH()) * d.NB * sizeof(int));
    q.L = sp.L;
    q.IPH = sp.items_per_head;
    q.cnt = reinterpret_cast<int*>(split_ws);
    q.po = reinterpret_cast<float4*>(split_ws + nc);
    q.pm = reinterpret_cast<float*>(split_ws + nc + align256(n * D * sizeof(float)));
    q.pl = q.pm + align256(n * sizeof(float)) / sizeof(float);
    grid = sp.items_per_head * d.BH();
  }
  e = launch_pdl(fn, dim3(grid), dim3(kThreads1), C::SMEM, s, mq, mk, mv, p, q);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core forward launch: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  *launched = 1;
  return FPA_OK;
}

template <int D>
int launch(const FpaFwdArgs& a, const Dims& d, const Stats& st, const KeyCols& cols, int* status, cudaStream_t s,
           int* launched, std::string* err) {
  using C = TcFwdCfg<D>;
  CUtensorMap mq, mk, mv;
  if (!make_tile_map(&mq, a.q, a.q_stride, d.B, d.H, d.T, D) || !make_tile_map(&mk, a.k, a.k_stride, d.B, d.H, d.T, D) ||
      !make_tile_map(&mv, a.v, a.v_stride, d.B, d.H, d.T, D)) {
    *err = "cuTensorMapEncodeTiled failed for q, k or v";
    return FPA_ERR_CUDA;
  }
  auto fn = tc_fwd_kernel<D>;
  cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(fn), C::SMEM);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core forward: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  TcFwdParams p = fwd_params(a, d, st, cols, status);
  p.NPAIR = (d.NB + 1) / 2;
  e = launch_pdl(fn, dim3(p.NPAIR * d.BH()), dim3(kThreads), C::SMEM, s, mq, mk, mv, p);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core forward launch: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  *launched = 1;
  return FPA_OK;
}

// D <= 64: the two-tile kernel while its grid fills the SMs (two query tiles per CTA share every K and V tile
// they load, half the L2 traffic); below that the one-tile kernel (twice as many CTAs, two per SM).
bool use_one_tile(const Dims& d) { return d.D <= 64 && int64_t((d.NB + 1) / 2) * d.BH() < sm_count(); }

// FPA_B200_FWD_SPLIT: unset (or any text that is not a number) for the planned split, 0 for none, L >= 2 for
// chunks of L key tiles wherever the one-tile kernel runs (a tuning switch; L is capped below NB).
int split_env() {
  const char* e = getenv("FPA_B200_FWD_SPLIT");
  if (e == nullptr || *e == 0) return -1;
  char* end = nullptr;
  const long v = strtol(e, &end, 10);
  return (*end == 0 && v >= 0 && v < (1 << 20)) ? int(v) : -1;
}

}  // namespace

bool tc_supports(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

namespace {

// Plans already made, by (NB, heads, SM slots): the list-schedule model below costs the host far more than a launch,
// and a call asks for its plan several times (workspace size, join counters, launch).
struct PlanEntry {
  int NB, BH, slots;
  FwdSplit sp;
};
std::mutex g_plan_mu;
std::vector<PlanEntry> g_plans;

}  // namespace

FwdSplit tc_fwd_split_plan(const Dims& d) {
  FwdSplit sp;
  const int forced = split_env();
  if (!tc_supports(d.D) || !use_one_tile(d) || d.NB < 4 || forced == 0 || forced == 1) return sp;
  if (forced > 1) {
    if (forced < d.NB) {
      sp.L = forced;
      sp.items_per_head = chunks_per_head(d.NB, forced);
    }
    return sp;
  }
  // The one-tile grid (NB CTAs per head, the longest NB key tiles) leaves CTA slots (two per SM) idle. Pick the chunk
  // length whose grid finishes first under a list schedule of its CTAs, in launch order, on the slots, each CTA
  // costing its key tiles plus kChunkCost tiles for its prologue, pipeline fill and epilogue (fitted to chunk-length
  // sweeps on B200 at 6 and 12 heads of T = 2048); ties keep the longer chunks (fewer partial outputs) or no split.
  constexpr int kChunkCost = 2;
  const int slots = 2 * sm_count();
  {
    std::lock_guard<std::mutex> lock(g_plan_mu);
    for (const PlanEntry& e : g_plans)
      if (e.NB == d.NB && e.BH == d.BH() && e.slots == slots) return e.sp;
  }
  auto finish = [&](int L) {  // L = NB: the unsplit grid
    std::priority_queue<int, std::vector<int>, std::greater<int>> free_at;
    for (int q = 0; q < slots; ++q) free_at.push(0);
    int end = 0;
    for (int i = d.NB - 1; i >= 0; --i)      // launch order: query tile descending, then chunk, then head
      for (int c = 0; c * L <= i; ++c) {
        const int len = std::min(L, i + 1 - c * L) + kChunkCost;
        for (int z = 0; z < d.BH(); ++z) {
          const int t = free_at.top() + len;
          free_at.pop();
          free_at.push(t);
          end = std::max(end, t);
        }
      }
    return end;
  };
  int best = finish(d.NB);
  for (int L = d.NB - 1; L >= 2; --L) {
    const int f = finish(L);
    if (f < best) {
      best = f;
      sp.L = L;
      sp.items_per_head = chunks_per_head(d.NB, L);
    }
  }
  std::lock_guard<std::mutex> lock(g_plan_mu);
  if (g_plans.size() >= 256) g_plans.clear();  // bounded: shapes seldom vary that much
  g_plans.push_back(PlanEntry{d.NB, d.BH(), slots, sp});
  return sp;
}

size_t tc_fwd_split_bytes(const Dims& d) {
  const FwdSplit sp = tc_fwd_split_plan(d);
  if (sp.L == 0) return 0;
  const size_t n = size_t(d.BH()) * sp.items_per_head * kBT;
  return align256(size_t(d.BH()) * d.NB * sizeof(int)) + align256(n * d.D * sizeof(float)) +
         2 * align256(n * sizeof(float));
}

int* tc_fwd_split_counters(const Dims& d, char* split_ws, size_t split_avail) {
  if (!use_one_tile(d) || tc_fwd_split_plan(d).L == 0 || split_avail < tc_fwd_split_bytes(d)) return nullptr;
  return reinterpret_cast<int*>(split_ws);
}

int tc_fwd(const FpaFwdArgs& a, const Dims& d, const Stats& st, const KeyCols& cols, char* split_ws,
           size_t split_avail, int* status, cudaStream_t s, int* launched, std::string* err) {
  *launched = 0;
  if (!tma_layout_ok(a.q, a.q_stride) || !tma_layout_ok(a.k, a.k_stride) || !tma_layout_ok(a.v, a.v_stride)) {
    *err = "the tensor-core path needs q, k, v with unit innermost stride and 16-byte aligned rows";
    return FPA_ERR_UNSUPPORTED;
  }
  if (a.o_stride[3] != 1 || (a.o_stride[2] * 2) % 16 || reinterpret_cast<uintptr_t>(a.o) % 16) {
    *err = "the tensor-core path needs o with unit innermost stride and 16-byte aligned rows";
    return FPA_ERR_UNSUPPORTED;
  }
  const bool one = use_one_tile(d);
  FwdSplit sp;
  if (one) {
    sp = tc_fwd_split_plan(d);
    if (sp.L > 0 && split_avail < tc_fwd_split_bytes(d)) sp = FwdSplit{};  // a workspace sized without the split
  }
  switch (d.D) {
    case 16:
      return one ? launch1<16>(a, d, st, cols, sp, split_ws, status, s, launched, err)
                 : launch<16>(a, d, st, cols, status, s, launched, err);
    case 32:
      return one ? launch1<32>(a, d, st, cols, sp, split_ws, status, s, launched, err)
                 : launch<32>(a, d, st, cols, status, s, launched, err);
    case 64:
      return one ? launch1<64>(a, d, st, cols, sp, split_ws, status, s, launched, err)
                 : launch<64>(a, d, st, cols, status, s, launched, err);
    case 128: return launch<128>(a, d, st, cols, status, s, launched, err);
    default: *err = "unsupported head dimension for the tensor-core path"; return FPA_ERR_UNSUPPORTED;
  }
}

}  // namespace fpa
