// Tensor-core backward pass of FPA for sm_100a (fp16 operands, fp32 accumulation), in two deterministic passes
// with the decomposition of the reference's backward (kernel.py:178-265 kv-pass, 287-340 q-pass):
//
//   tc_bwd_kv_kernel  persistent, one CTA per SM taking key tiles j (128 keys) of one head as work units; per
//                     unit, query tiles i = j .. NB-1:
//                     S^T = K Q^T and dP^T = V dO^T into TMEM; thread = key computes P^T, dS^T (fp16, back into
//                     TMEM over S^T and dP^T), then dV += P^T dO and dK += dS^T Q on the tensor cores. Also dpsi,
//                     the dbeta partial, the soft-min sums W (u in the key's tile) and TB (u strictly between the
//                     tiles), and the in-tile soft-min of the diagonal tile (warps 2-3; for D = 128 its g is stored
//                     for diag_dphi_kernel).
//   tc_bwd_q_kernel   persistent, one CTA per SM taking query tiles i of one head as work units; per unit, key
//                     tiles j = i .. 0: S = Q K^T, dP = dO V^T; thread = query computes dS (fp16, into its own TMEM
//                     columns) and dQ += dS K; also r_t and from it the soft-min part with u in the query's tile
//                     (DPHI2).
//
// Warp roles (384 threads): warp 0 issues the MMAs (whole warp, one elected lane issues), warp 1 is the TMA
// producer (work-unit ids, the stationary tiles, streamed tiles and their per-row vectors through a ring of
// stages), warps 2-3 run the kv-pass's diagonal soft-min and otherwise hand registers to the row groups
// (setmaxnreg). Warps 4-7 and 8-11 are two row groups (thread = TMEM lane); group g
// owns columns [64 g, 64 g + 64) of every S / dP tile and runs on its own barriers; S and dP live in TMEM slots
// that rotate over the jobs (tile, group), so the products of a group's next tile are computed while it works on
// the current one. Every mbarrier wait is bounded (fpa::sm100::mbar_wait).
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "fpa_sm100.cuh"
#include "fpa_tc.h"

namespace fpa {
using namespace sm100;

namespace {

constexpr int kBT = kTcBT;
constexpr int kThreads = 384;
// The MMA and producer warps come first: the warp schedulers favour older warps, and these two must issue promptly
// while the row warps sharing their schedulers are busy.
constexpr int kWarpMma = 0;
constexpr int kWarpProducer = 1;
constexpr int kRowWarp0 = 4;  // row warps 4..11
constexpr int kRowThreads = 256;    // two row groups of 128
constexpr int kGroupThreads = 128;
constexpr int kHalf = kBT / 2;      // columns of one row group
constexpr int kNamedBarRows = 1;    // bar.sync id used by the 256 row threads
constexpr int kNamedBarDiag = 2;    // bar.sync id used by the 64 threads of warps 2-3 (diagonal soft-min)
constexpr int kUQ = 4;              // persistent passes: depth of the ring of work-unit ids

// Shared-memory layout of one [128 x D] fp16 tile as TMA writes it: boxes of 128 rows x min(64, D) columns with
// the swizzle of the box row width.
template <int D>
struct TileLayout {
  static constexpr int BOXC = D >= 64 ? 64 : D;
  static constexpr int NBOX = D / BOXC;
  static constexpr int SWB = BOXC * 2;
  static constexpr int BOXB = kBT * SWB;
  static constexpr int TILEB = NBOX * BOXB;
  static constexpr uint32_t SW = SWB == 128 ? kSwizzle128 : (SWB == 64 ? kSwizzle64 : kSwizzle32);
  static constexpr uint32_t IDESC_S = idesc_f16(kBT, kHalf, 0);  // 128 rows x one group's 64 columns
  static constexpr uint32_t IDESC_ACC = idesc_f16(kBT, D, 1);
};

// Per-pass configuration. TMEM holds NSLOT slots of 128 columns, each the job of one row group for one tile (its
// 64 columns of S, then its 64 columns of dP); job n = 2 k + g (tile k, group g) uses slot n % NSLOT, so with three
// slots the products of a group's next tile are computed while it still works on the current one. The
// accumulators follow the slots (dV, dK for the kv-pass; dQ for the q-pass), then the two stationary operands
// (D/2 columns each) when they fit in the 512 columns; otherwise those are read from shared memory.
template <int D, bool KV>
struct TcBwdCfg : TileLayout<D> {
  using L = TileLayout<D>;
  static constexpr int NSLOT = D <= 64 ? 3 : 2;
  static constexpr int NS = NSLOT;  // shared-memory stages of the streamed tiles
  static constexpr int COL_A1 = 128 * NSLOT, COL_A2 = COL_A1 + D;
  static constexpr int COL_X = COL_A1 + (KV ? 2 : 1) * D;
  static constexpr bool AT = COL_X + D <= 512;
  static constexpr int NSTAT = AT ? 0 : 2;  // stationary tiles kept in shared memory
  static constexpr int VECB = kBT * 4;
  static constexpr int VECSTAGE = 4 * VECB + 2 * VECB;  // float4 per row + two float vectors, per stage
  static constexpr int OFF_A = 0;                       // stationary operand 1 (when !AT)
  static constexpr int OFF_B = L::TILEB;                // stationary operand 2 (when !AT)
  static constexpr int OFF_S1 = NSTAT * L::TILEB;       // streamed operand 1 [NS]
  static constexpr int OFF_S2 = OFF_S1 + NS * L::TILEB;  // streamed operand 2 [NS]
  static constexpr int OFF_X = OFF_S2 + NS * L::TILEB;   // the next unit's stationary tiles (TMA staging; AT)
  static constexpr int OFF_VEC = OFF_X + (AT ? 2 * L::TILEB : 0);  // [NS][VECSTAGE]
  static constexpr int OFF_RED = OFF_VEC + NS * VECSTAGE;  // 32 + 4 * 128 floats of row-group scratch
  static constexpr int OFF_G = OFF_RED + (32 + 4 * kBT) * 4;
  // kv: a_full, st_full[NS], st_empty[NS], s_full[NSLOT], p_full[NSLOT], acc_done, acc_free, drain, at_full,
  // x_full, x_empty, g_full, g_free, u_full[kUQ], u_empty[kUQ], s_last (the q-pass uses a subset)
  static constexpr int NBAR = 2 * NS + 2 * NSLOT + 10 + 2 * kUQ;
  // kv-pass: the diagonal tile's g ([128][129] fp32) and a2 of its positions (with 2^{a2 - max}) stay in shared
  // memory, where warps 2-3 run the in-tile soft-min while the row groups go on, when that fits (all D but 128).
  static constexpr int GLD = kBT + 1;
  static constexpr int GBYTES = (kBT * GLD + 2 * kBT + 4) * 4;  // g, a2, 2^{a2 - M}, max / min
  static constexpr bool FUSEDIAG = KV && OFF_G + GBYTES + NBAR * 8 + 64 + 1024 <= 227 * 1024;
  static constexpr int OFF_BAR = OFF_G + (FUSEDIAG ? GBYTES : 0);
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 64 + 1024;  // + the TMEM address and the unit ring
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(KV || AT, "the q-pass keeps Q and dO in TMEM");
};

struct TcBwdParams {
  // per-head [BH][TP] arrays (padded, tiles of 128)
  const float4* qv4;   // per query: (lse or +inf beyond T, delta or 0, PRE, prey)
  const float4* kv4;   // per key: (SUF - psi, psi, sufy, SUFL)
  const float* delta;
  const float* pre;
  const float* prel;
  const float* suf;
  const float* sufl;
  const float* bmin;   // [BH][NB]
  const float* bl;     // [BH][NB]
  const float* xs;     // SUF - psi (raw key vectors)
  const float* psi;    // psi
  const float* phi;    // phi (+inf beyond T)
  const float* beta;   // [H]
  const float* prey;   // 2^{PREL_t - BL_tile}
  const float* sufy;   // 2^{SUFL_s - SUFL_first of tile}
  const float* prer;   // [BH][NB] BL - PREL_first
  const float* sufr;   // [BH][NB] SUFL_first - min finite SUFL
  // outputs
  // inputs read row by row into TMEM (the stationary MMA operands)
  const __half* q;
  const __half* k;
  const __half* v;
  const __half* dout;
  int64_t q_s[3], k_s[3], v_s[3], do_s[3];  // b, h, t strides (d stride 1)
  __half* dq;
  __half* dk;
  __half* dv;
  int64_t dq_s[3], dk_s[3], dv_s[3];  // b, h, t strides (d stride 1)
  float* dpsi;         // [BH][T]
  float* w;            // [BH][TP]
  float* tb;           // [BH][NB][NB][kTcTbParts]
  float* dbeta;        // [BH][NB]
  float* gd;           // [BH][NB][128][128] (when the kv-pass does not run the diagonal soft-min itself)
  float* dphi4;        // [BH][TP]
  float* dphi2;        // [BH][TP]
  int* status;
  int* sched;          // [2] work-unit counters (kv-pass, q-pass), zeroed by the stats kernel
  int B, H, T, NB, TP;
  float scale, scale2, il2;
};

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void rows_sync() { asm volatile("bar.sync %0, 256;" ::"r"(kNamedBarRows) : "memory"); }

// Deterministic sum over the 256 row threads (fixed shuffle tree, then the 8 warp partials in a fixed order). All
// 256 threads call it; the result is returned to every thread.
__device__ __forceinline__ float rows_sum(float v, float* red) {
  v = group_sum<32>(v);
  const int w = (threadIdx.x >> 5) - kRowWarp0;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  rows_sync();
  const float r = ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
  rows_sync();
  return r;
}

// Register split per warpgroup (the launch gives 168 per thread): the producer/MMA warpgroup keeps 88 (96 for
// D = 128, whose MMA warp issues from shared-memory descriptors) and the two row groups take the rest,
// 128 * 88 + 256 * 208 = 128 * 96 + 256 * 200 = 384 * 168.
template <int D>
__device__ __forceinline__ void regs_producer() {
  if constexpr (D == 128)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 96;" ::: "memory");
  else
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
}
template <int D>
__device__ __forceinline__ void regs_rows() {
  if constexpr (D == 128)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 200;" ::: "memory");
  else
    asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
}

// The descriptor of the same operand layout `off` bytes further on: the start address is the low 14-bit field
// (address >> 4) and shared-memory addresses stay below 2^18, so the offset adds to the low word without a carry.
// Built once per operand, each K-step then costs one integer add in the MMA warp.
__device__ __forceinline__ uint64_t desc_at(uint64_t d, uint32_t off) {
  return (d & 0xFFFFFFFF00000000ull) | uint32_t(uint32_t(d) + (off >> 4));
}

// D[128 x 64] = A[128 x D] * B[64 x D]^T, both K-major in shared memory; `b` points at the group's first B row.
template <int D>
__device__ __forceinline__ void issue_ss_half(uint32_t d, uint32_t a, uint32_t b) {
  using C = TileLayout<D>;
  const uint64_t da = smem_desc(a, 16, 8 * C::SWB, C::SW), db = smem_desc(b, 16, 8 * C::SWB, C::SW);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk / (C::SWB / 32)) * C::BOXB + (kk % (C::SWB / 32)) * 32;
    mma_ss_w(d, desc_at(da, off), desc_at(db, off), C::IDESC_S, kk > 0);
  }
}

// D[128 x D] (+)= A[128 x 64 from TMEM, fp16 packed] * B[64 x D from smem, N-contiguous], for row group g: A holds
// the group's 64 columns and B its 64 rows (rows 64 g .. 64 g + 63 of the tile). The K-step kk of A (16 values,
// 8 packed columns) sits at column a_tmem + 16 kk: the row groups write it over the first half of the 16 fp32
// columns they read it from, so no column is overwritten before it is read.
template <int D>
__device__ __forceinline__ void issue_ts_half(uint32_t d, uint32_t a_tmem, uint32_t b, int g, bool acc) {
  using C = TileLayout<D>;
  const uint64_t db = smem_desc(b + g * kHalf * C::SWB, C::BOXB, 8 * C::SWB, C::SW);
#pragma unroll
  for (int kk = 0; kk < kHalf / 16; ++kk)
    mma_ts_w(d, a_tmem + kk * 16, desc_at(db, kk * 16 * C::SWB), C::IDESC_ACC, (acc || kk > 0) ? 1u : 0u);
}

// D[128 x 64] = A[128 x D from TMEM] * B[64 x D]^T (B K-major in shared memory, `b` at the group's first row).
// A is packed densely, two fp16 per 32-bit column in K order: K-step kk (16 values) at columns a_tmem + 8 kk.
template <int D>
__device__ __forceinline__ void issue_ts_k(uint32_t d, uint32_t a_tmem, uint32_t b) {
  using C = TileLayout<D>;
  const uint64_t db = smem_desc(b, 16, 8 * C::SWB, C::SW);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk / (C::SWB / 32)) * C::BOXB + (kk % (C::SWB / 32)) * 32;
    mma_ts_w(d, a_tmem + 8 * kk, desc_at(db, off), C::IDESC_S, kk > 0);
  }
}

// One row of a staged [128 x D] fp16 tile (as TMA wrote it) into this thread's TMEM lane, D/2 columns from `taddr`
// (the packing issue_ts_k expects: two fp16 per 32-bit column in K order). Warp-collective.
template <int D>
__device__ __forceinline__ void stage_row_to_tmem(uint32_t taddr, const uint8_t* tile, int r) {
  using L = TileLayout<D>;
  constexpr int CPB = L::SWB / 16;  // 16-byte chunks per box row; the TMA swizzle permutes them by row
  uint32_t u[D / 2];
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    const uint32_t o = uint32_t(r * L::SWB + (c % CPB) * 16);
    const uint32_t sw = o ^ (((o >> 7) & uint32_t(CPB - 1)) << 4);
    const uint4 x = *reinterpret_cast<const uint4*>(tile + (c / CPB) * L::BOXB + sw);
    u[4 * c] = x.x;
    u[4 * c + 1] = x.y;
    u[4 * c + 2] = x.z;
    u[4 * c + 3] = x.w;
  }
  if constexpr (D == 16) {
    tmem_st8(taddr, u);
  } else if constexpr (D == 32) {
    tmem_st16(taddr, u);
  } else {
#pragma unroll
    for (int c = 0; c < D / 2; c += 32) tmem_st32(taddr + c, u + c);
  }
}

// AND of `v` over the `n` threads of named barrier `id` (all of them call it).
__device__ __forceinline__ bool bar_all(bool v, int id, int n) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool rows_all(bool v) { return bar_all(v, kNamedBarRows, kRowThreads); }  // 256 row threads
__device__ __forceinline__ bool diag_all(bool v) { return bar_all(v, kNamedBarDiag, 64); }  // warps 2-3

// ------------------------------------------------------------------------------------------------ kv-pass ----
// Persistent, like the q-pass: work units are key tiles j of one head (longest first) taken from a counter. The
// producer stages each unit's K and V tiles by TMA (or, when K and V stay in shared memory, loads them there once
// the previous unit's products are complete); at a unit boundary the row threads copy the next unit's K and V rows
// into TMEM and then read the finished unit's dV and dK out, so the next unit's first products are computed
// meanwhile. The diagonal tile comes first in each unit; its soft-min runs on warps 2-3 during the rest of the
// unit, and the next unit's diagonal tile waits until they are done with G.
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
tc_bwd_kv_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                 const TcBwdParams p) {
  using C = TcBwdCfg<D, true>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* a_full = bars;  // K and V of the unit in shared memory (when they do not fit in TMEM)
  uint64_t* st_full = bars + 1;
  uint64_t* st_empty = st_full + C::NS;
  uint64_t* s_full = st_empty + C::NS;     // [NSLOT] S and dP of the job in the slot are ready
  uint64_t* p_full = s_full + C::NSLOT;    // [NSLOT] the group of the job in the slot has written its P / dS
  uint64_t* acc_done = p_full + C::NSLOT;  // every MMA of the unit has completed (dV, dK final)
  uint64_t* acc_free = acc_done + 1;       // the row threads have read dV and dK out of TMEM
  uint64_t* drain = acc_free + 1;
  uint64_t* at_full = drain + 1;  // K and V rows of the unit in TMEM
  uint64_t* x_full = at_full + 1;  // K and V tiles of the unit in the staging buffer
  uint64_t* x_empty = x_full + 1;  // the row threads have copied the staging buffer
  uint64_t* g_full = x_empty + 1;  // the diagonal tile's g is in shared memory (fused diagonal soft-min)
  uint64_t* g_free = g_full + 1;   // warps 2-3 are done with it
  uint64_t* u_full = g_free + 1;   // [kUQ] unit ids handed from the producer to the other warps
  uint64_t* u_empty = u_full + kUQ;
  uint64_t* s_last = u_empty + kUQ;  // once per unit: its last S^T / dP^T products are complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_last + 1);
  int* uq = reinterpret_cast<int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbh = p.B * p.H;
  const int nunits = p.NB * nbh;
  // K and V as TMEM operands of S^T and dP^T (both stationary) when the columns fit.
  constexpr bool AT = C::AT;
  constexpr int COL_K = C::COL_X, COL_V = COL_K + D / 2;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(st_full + s, 1);
      mbar_init(st_empty + s, 1);
    }
    for (int x = 0; x < C::NSLOT; ++x) {
      mbar_init(s_full + x, 1);
      mbar_init(p_full + x, kGroupThreads);
    }
    mbar_init(acc_done, 1);
    mbar_init(acc_free, kRowThreads);
    mbar_init(drain, 1);
    mbar_init(at_full, kRowThreads);
    mbar_init(x_full, 1);
    mbar_init(x_empty, kRowThreads);
    mbar_init(g_full, kRowThreads);
    mbar_init(g_free, 64);
    for (int x = 0; x < kUQ; ++x) {
      mbar_init(u_full + x, 1);
      mbar_init(u_empty + x, 1 + kRowThreads / 32 + (C::FUSEDIAG ? 2 : 0));  // MMA, row and soft-min warps
    }
    mbar_init(s_last, 1);
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
  if (warp < kRowWarp0) regs_producer<D>();

  if (warp == kWarpProducer) {
    if (elect_one()) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&tdo);
    }
    __syncwarp();
    bool ok = true;
    int gk = 0, nx = 0;  // tiles and staged units issued so far
    for (int u = 0; ok; ++u) {
      const int us = u % kUQ;
      if (u >= kUQ) ok = mbar_wait(u_empty + us, ((u / kUQ) - 1) & 1, p.status, 134);
      if (!ok) break;
      int x = 0;
      if (lane == 0) {
        x = atomicAdd(p.sched, 1);
        uq[us] = x;
        mbar_arrive(u_full + us);
      }
      x = __shfl_sync(0xffffffffu, x, 0);
      if (x >= nunits) break;
      const int j = x / nbh, z = x % nbh, b = z / p.H, h = z % p.H;
      const size_t zb = size_t(z) * p.TP;
      const int nsteps = p.NB - j;
      if constexpr (AT) {
        if (nx > 0) ok = mbar_wait(x_empty, (nx - 1) & 1, p.status, 131);
        if (!ok) break;
        if (elect_one()) {
          mbar_expect_tx(x_full, 2 * C::TILEB);
          for (int bx = 0; bx < C::NBOX; ++bx) {
            tma_load_4d(smem + C::OFF_X + bx * C::BOXB, &tk, bx * C::BOXC, j * kBT, h, b, x_full);
            tma_load_4d(smem + C::OFF_X + C::TILEB + bx * C::BOXB, &tv, bx * C::BOXC, j * kBT, h, b, x_full);
          }
        }
        __syncwarp();
        ++nx;
      }
      // Without room in TMEM, K and V go to shared memory as soon as the previous unit's last S^T / dP^T products
      // (the last readers of that memory) are complete, ahead of the unit's tiles: that happens while the rows
      // still work on the previous unit's last tiles, so the copy is hidden behind them. s_last completes once per
      // unit and is waited here in unit order, and its next phase needs this unit's K and V, so the parity test
      // cannot see an older phase. The wait needs nothing from this warp: every tile of the previous unit has been
      // issued.
      if constexpr (!AT) {
        if (u > 0) ok = mbar_wait(s_last, (u - 1) & 1, p.status, 102);
        if (!ok) break;
        if (elect_one()) {
          mbar_expect_tx(a_full, 2 * C::TILEB);
          for (int bx = 0; bx < C::NBOX; ++bx) {
            tma_load_4d(smem + C::OFF_A + bx * C::BOXB, &tk, bx * C::BOXC, j * kBT, h, b, a_full);
            tma_load_4d(smem + C::OFF_B + bx * C::BOXB, &tv, bx * C::BOXC, j * kBT, h, b, a_full);
          }
        }
        __syncwarp();
        ++nx;
      }
      for (int k = 0; k < nsteps && ok; ++k) {
        const int st = gk % C::NS, i = j + k;
        if (gk >= C::NS) ok = mbar_wait(st_empty + st, ((gk / C::NS) - 1) & 1, p.status, 101);
        if (!ok) break;
        if (elect_one()) {
          uint8_t* vec = smem + C::OFF_VEC + st * C::VECSTAGE;
          mbar_expect_tx(st_full + st, 2 * C::TILEB + 6 * C::VECB);
          for (int bx = 0; bx < C::NBOX; ++bx) {
            tma_load_4d(smem + C::OFF_S1 + st * C::TILEB + bx * C::BOXB, &tq, bx * C::BOXC, i * kBT, h, b,
                        st_full + st);
            tma_load_4d(smem + C::OFF_S2 + st * C::TILEB + bx * C::BOXB, &tdo, bx * C::BOXC, i * kBT, h, b,
                        st_full + st);
          }
          const size_t off = zb + size_t(i) * kBT;
          bulk_load(vec, p.qv4 + off, 4 * C::VECB, st_full + st);
          bulk_load(vec + 4 * C::VECB, p.prel + off, C::VECB, st_full + st);
          bulk_load(vec + 5 * C::VECB, p.phi + off, C::VECB, st_full + st);
        }
        __syncwarp();
        ++gk;
      }
    }
    // Nothing may land in shared memory after the CTA exits: wait for the last copies issued.
    for (int q = (gk > C::NS ? gk - C::NS : 0); q < gk; ++q) mbar_wait(st_full + q % C::NS, (q / C::NS) & 1, p.status, 103);
    if (nx > 0) mbar_wait(AT ? x_full : a_full, (nx - 1) & 1, p.status, 104);
  } else if (warp == kWarpMma) {
    // Jobs n = 2 k + g of a unit in order (query tile k, row group g = query columns [64 g, 64 g + 64)); with gn
    // jobs before the unit, S^T and dP^T of job n go into slot (gn + n) % NSLOT; once the group has written P^T and
    // dS^T there, dV += P^T dO and dK += dS^T Q over its 64 queries, then the products of job n + NSLOT into the
    // same slot (tcgen05.mma from one thread execute in order, so the reads come first). The first products of a
    // unit overwrite dV and dK, so they wait until the rows have read the previous unit's.
    const uint32_t sa = smem_u32(smem + C::OFF_A), sb = smem_u32(smem + C::OFF_B);
    const uint32_t s1 = smem_u32(smem + C::OFF_S1), s2 = smem_u32(smem + C::OFF_S2);
    bool ok = true;
    int gn = 0, gk = 0, loaded = -1;
    for (int u = 0; ok; ++u) {
      const int us = u % kUQ;
      ok = mbar_wait(u_full + us, (u / kUQ) & 1, p.status, 132);
      if (!ok) break;
      const int x = uq[us];
      __syncwarp();
      if (lane == 0) mbar_arrive(u_empty + us);
      if (x >= nunits) break;
      const int njobs = 2 * (p.NB - x / nbh);
      auto need_tile = [&](int kt) {
        const int gt = gk + kt;
        if (ok && gt > loaded) {
          ok = mbar_wait(st_full + gt % C::NS, (gt / C::NS) & 1, p.status, 111);
          loaded = gt;
          tc_fence_after();
        }
        return ok;
      };
      auto issue_s = [&](int n) {
        const int g = n & 1, st = (gk + (n >> 1)) % C::NS, sl = (gn + n) % C::NSLOT;
        const uint32_t dcol = tmem + sl * 128;
        const uint32_t bq = s1 + st * C::TILEB + g * kHalf * C::SWB, bdo = s2 + st * C::TILEB + g * kHalf * C::SWB;
        if constexpr (AT) {
          issue_ts_k<D>(dcol, tmem + COL_K, bq);              // S^T  = K Q^T
          issue_ts_k<D>(dcol + kHalf, tmem + COL_V, bdo);     // dP^T = V dO^T
        } else {
          issue_ss_half<D>(dcol, sa, bq);
          issue_ss_half<D>(dcol + kHalf, sb, bdo);
        }
        mma_commit_w(s_full + sl);
        if (n == njobs - 1) mma_commit_w(s_last);
      };
      ok = AT ? mbar_wait(at_full, u & 1, p.status, 115) : mbar_wait(a_full, u & 1, p.status, 110);
      tc_fence_after();
      for (int n = 0; n < C::NSLOT && n < njobs; ++n)
        if (need_tile(n >> 1)) issue_s(n);
      for (int n = 0; n < njobs && ok; ++n) {
        const int g = n & 1, st = (gk + (n >> 1)) % C::NS, sl = (gn + n) % C::NSLOT;
        ok = mbar_wait(p_full + sl, ((gn + n) / C::NSLOT) & 1, p.status, 112);
        if (ok && n == 0 && u > 0) ok = mbar_wait(acc_free, (u - 1) & 1, p.status, 116);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acol = tmem + sl * 128;
        issue_ts_half<D>(tmem + C::COL_A1, acol, s2 + st * C::TILEB, g, n > 0);          // dV += P^T dO
        issue_ts_half<D>(tmem + C::COL_A2, acol + kHalf, s1 + st * C::TILEB, g, n > 0);  // dK += dS^T Q
        if (g == 1) mma_commit_w(st_empty + st);
        const int m = n + C::NSLOT;
        if (m < njobs && need_tile(m >> 1)) issue_s(m);
      }
      mma_commit_w(acc_done);
      gn += njobs;
      gk += njobs / 2;
    }
    mma_commit_w(drain);
    mbar_wait(drain, 0, p.status, 114);
  } else if (C::FUSEDIAG && (warp == 2 || warp == 3)) {
    // ---- In-tile soft-min of the diagonal tile (DPHI4), concurrent with the row groups (kernel.py:269-283
    // evaluates the same sums with scans). For key s, Z_{s,t} = sum_{s<u<=t} 2^{a2_u}, and g_ts at G[s][t]
    // (t > s), the contribution to position u is
    //   2^{a2_u} K_s(u),  K_s(u) = sum_{t>=u} g_ts / Z_{s,t}.
    // Fast path, when the tile's a2 spans at most kSpan: with E_u = 2^{a2_u - M} (M the tile maximum, so
    // E_u >= 2^-kSpan stays a normal float), S_{s,t} = Z_{s,t} 2^-M is a running sum, one reciprocal per pair
    // gives R_ts = g_ts / S_{s,t} (in place of g), a suffix sum along t gives K (in place of R), and the column sums
    // times E_u give DPHI4_u. Every term E_u g_ts / S_{s,t} is at most |g_ts| (u lies in the window).
    // Otherwise the running-maximum form: w_t = 2^{a2_t} / Z_{s,t} in (0, 1] and
    //   H(t) = g_ts + (1 - w_{t+1}) H(t+1),  contribution to u = t: w_t H(t)   (Z_{s,t} / Z_{s,t+1} = 1 - w_{t+1}),
    // with w_t of key s kept at G[t][s] (below the diagonal, unused by g).
    // Each of the 64 threads takes keys wt and 127 - wt (equal work), then positions wt and 127 - wt for the column
    // sums. Both passes run in blocks of kRun positions whose shared-memory operands are loaded into registers
    // first, so only the add/FMA chain is serial; positions past the end of a chain load neutral values and store
    // nothing.
    constexpr int LD = C::GLD;
    constexpr int kRun = 8;
    constexpr float kSpan = 64.f;
    float* G = reinterpret_cast<float*>(smem + C::OFF_G);
    float* a2s = G + kBT * LD;
    float* es = a2s + kBT;
    float* mm = es + kBT;  // per-warp maximum and minimum of a2 over the tile's positions
    const int wt = threadIdx.x - 64;
    bool ok = true;
    for (int u = 0;; ++u) {
      const int us = u % kUQ;
      int x = nunits;
      if (ok) ok = mbar_wait(u_full + us, (u / kUQ) & 1, p.status, 133);
      if (ok) x = uq[us];
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(u_empty + us);
      if (!diag_all(ok && x < nunits)) break;
      const int j = x / nbh, z = x % nbh;
      const size_t zb = size_t(z) * p.TP;
      const int tend = min(kBT, p.T - j * kBT);
      float vmax = -kInf, vmin = kInf;
      for (int t = wt; t < kBT; t += 64) {
        const float a = -p.phi[zb + size_t(j) * kBT + t] * p.il2;  // phi = +inf beyond T
        a2s[t] = a;
        if (t < tend) {
          vmax = fmaxf(vmax, a);
          vmin = fminf(vmin, a);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
        vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
      }
      if (lane == 0) {
        mm[2 * (warp - 2)] = vmax;
        mm[2 * (warp - 2) + 1] = vmin;
      }
      asm volatile("bar.sync %0, 64;" ::"r"(kNamedBarDiag) : "memory");
      const float M = fmaxf(mm[0], mm[2]);
      const bool fast = M - fminf(mm[1], mm[3]) <= kSpan;  // the same for all 64 threads
      if (fast) {
        for (int t = wt; t < kBT; t += 64) es[t] = t < tend ? ex2(a2s[t] - M) : 0.f;
        asm volatile("bar.sync %0, 64;" ::"r"(kNamedBarDiag) : "memory");
      }
      ok = mbar_wait(g_full, u & 1, p.status, 130);
      if (ok && fast) {
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          const int s = q == 0 ? wt : kBT - 1 - wt;
          float* row = G + s * LD;
          float S = 0.f;
#pragma unroll 1
          for (int t0 = s + 1; t0 < tend; t0 += kRun) {
            float ev[kRun], gv[kRun];
#pragma unroll
            for (int e = 0; e < kRun; ++e) {
              const bool in = t0 + e < tend;
              ev[e] = in ? es[t0 + e] : 0.f;
              gv[e] = in ? row[t0 + e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < kRun; ++e) {
              S += ev[e];
              gv[e] *= rcp_approx(S);
            }
#pragma unroll
            for (int e = 0; e < kRun; ++e)
              if (t0 + e < tend) row[t0 + e] = gv[e];
          }
          float K = 0.f;
#pragma unroll 1
          for (int t1 = tend - 1; t1 > s; t1 -= kRun) {
            float rv[kRun];
#pragma unroll
            for (int e = 0; e < kRun; ++e) rv[e] = t1 - e > s ? row[t1 - e] : 0.f;
#pragma unroll
            for (int e = 0; e < kRun; ++e) {
              K += rv[e];
              rv[e] = K;
            }
#pragma unroll
            for (int e = 0; e < kRun; ++e)
              if (t1 - e > s) row[t1 - e] = rv[e];
          }
        }
      } else if (ok) {
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          const int s = q == 0 ? wt : kBT - 1 - wt;
          float mz = -kInf, zz = 0.f;
#pragma unroll 1
          for (int t0 = s + 1; t0 < tend; t0 += kRun) {
            float at[kRun], wv[kRun];
#pragma unroll
            for (int e = 0; e < kRun; ++e) at[e] = t0 + e < tend ? a2s[t0 + e] : -kInf;
#pragma unroll
            for (int e = 0; e < kRun; ++e) {
              const float dd = at[e] - mz;
              const bool up = dd > 0.f;
              const float ee = ex2(-fabsf(dd));
              zz = fmaf(zz, up ? ee : 1.f, up ? 1.f : ee);
              mz = fmaxf(mz, at[e]);
              wv[e] = (up ? 1.f : ee) * rcp_approx(zz);
            }
#pragma unroll
            for (int e = 0; e < kRun; ++e)
              if (t0 + e < tend) G[(t0 + e) * LD + s] = wv[e];
          }
          float H = 0.f, wn = 0.f;
#pragma unroll 1
          for (int t1 = tend - 1; t1 > s; t1 -= kRun) {
            float w[kRun], g[kRun];
#pragma unroll
            for (int e = 0; e < kRun; ++e) {
              const bool in = t1 - e > s;
              w[e] = in ? G[(t1 - e) * LD + s] : 0.f;
              g[e] = in ? G[s * LD + t1 - e] : 0.f;
            }
#pragma unroll
            for (int e = 0; e < kRun; ++e) {
              H = fmaf(1.f - wn, H, g[e]);
              g[e] = w[e] * H;
              wn = w[e];
            }
#pragma unroll
            for (int e = 0; e < kRun; ++e)
              if (t1 - e > s) G[s * LD + t1 - e] = g[e];
          }
        }
      }
      asm volatile("bar.sync %0, 64;" ::"r"(kNamedBarDiag) : "memory");
      if (ok) {
#pragma unroll 1
        for (int q = 0; q < 2; ++q) {
          const int u = q == 0 ? wt : kBT - 1 - wt;
          if (u < tend) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};  // keys s = 0, 1, 2, 3 mod 4, joined in a fixed order
            int s2 = 0;
            for (; s2 + 4 <= u; s2 += 4) {
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[e] += G[(s2 + e) * LD + u];
            }
#pragma unroll
            for (int e = 0; e < 3; ++e)
              if (s2 + e < u) acc[e] += G[(s2 + e) * LD + u];
            const float col = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            p.dphi4[zb + size_t(j) * kBT + u] = fast ? es[u] * col : col;
          }
        }
      }
      asm volatile("bar.sync %0, 64;" ::"r"(kNamedBarDiag) : "memory");  // G, a2s, es, mm are reused
      mbar_arrive(g_free);
    }
  } else if (warp >= kRowWarp0) {
    regs_rows<D>();
    const int grp = (warp - kRowWarp0) >> 2, wr = warp & 3;
    const int r = wr * 32 + lane;  // key within the tile = TMEM lane
    const int cb = grp * kHalf;    // this group's query columns [cb, cb + 64)
    const uint32_t tl = tmem + (uint32_t(wr * 32) << 16);
    constexpr int DH = D >= 32 ? D / 2 : D;  // head-dim columns of dV and dK stored by each group
    const float2 sc2 = make_float2(p.scale2, p.scale2);
    float* xg = red + 32;
    float* xw = red + 32 + kBT;
    bool ok = true;
    int gn = 0, gk = 0;
    // The finished unit, written out after the next unit's K and V rows are in TMEM.
    bool have_prev = false, pv_done = false, pv_ok = false;
    int pv_s = 0, pv_j = 0, pv_b = 0, pv_h = 0, pv_z = 0;
    float pv_g = 0.f, pv_db = 0.f, pv_w = 0.f, pv_bh = 0.f;
    for (int u = 0;; ++u) {
      const int us = u % kUQ;
      int x = nunits;
      if (ok) ok = mbar_wait(u_full + us, (u / kUQ) & 1, p.status, 124);
      if (ok) x = uq[us];
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(u_empty + us);
      const bool more = rows_all(ok && x < nunits);
      const int j = more ? x / nbh : 0;
      const int z = more ? x % nbh : 0, b = z / p.H, h = z % p.H;
      const size_t zb = size_t(z) * p.TP;
      const int s = j * kBT + r;
      const bool s_ok = more && s < p.T;
      // The unit's per-key and first per-tile scalars, loaded first so that their latency passes during the copy
      // below and the previous unit's write-out.
      float bh = 0.f, psi_s = 0.f, xs_s = 0.f, suf_s = 0.f, sufl_s = 0.f, bl_n = 0.f, bmin_n = 0.f, prer_n = 0.f;
      if (more) {
        bh = p.beta[h];
        psi_s = p.psi[zb + s];
        xs_s = p.xs[zb + s];  // SUF_s - psi_s (+inf for the last key of the tile)
        suf_s = p.suf[zb + s];
        sufl_s = p.sufl[zb + s];
        bl_n = p.bl[size_t(z) * p.NB + j];
        bmin_n = p.bmin[size_t(z) * p.NB + j];
        prer_n = p.prer[size_t(z) * p.NB + j];
      }
      if constexpr (AT) {
        // The previous unit's last S^T / dP^T products (the last readers of the K and V columns) are complete:
        // s_last is waited in unit order, and its next phase needs this unit's K and V.
        if (have_prev && ok) ok = mbar_wait(s_last, (u - 1) & 1, p.status, 127);
        if (more) {
          // Group 0 copies the key's row of K, group 1 its row of V, into TMEM.
          ok = ok && mbar_wait(x_full, u & 1, p.status, 125);
          if (ok) {
            stage_row_to_tmem<D>(tl + (grp == 0 ? COL_K : COL_V), smem + C::OFF_X + grp * C::TILEB, r);
            tmem_st_wait();
          }
          tc_fence_before();
          mbar_arrive(at_full);
          mbar_arrive(x_empty);
        }
      }
      if (have_prev) {
        // dV and dK of the finished unit out of TMEM (its MMAs have completed); the MMA warp may then start this
        // unit's.
        if (pv_done && !mbar_wait(acc_done, (u - 1) & 1, p.status, 122)) pv_done = pv_ok = ok = false;
        pv_done = __all_sync(0xffffffffu, pv_done);  // warp-uniform: the TMEM loads below are warp-collective
        if (pv_done) {
          tc_fence_after();
          __half* dvrow = p.dv + pv_b * p.dv_s[0] + pv_h * p.dv_s[1] + int64_t(pv_s) * p.dv_s[2];
          __half* dkrow = p.dk + pv_b * p.dk_s[0] + pv_h * p.dk_s[1] + int64_t(pv_s) * p.dk_s[2];
          if (D >= 32 || grp == 0) {
#pragma unroll
            for (int c = grp * DH; c < grp * DH + DH; c += 16) {
              float a1[16], a2[16];
              tmem_ld16(tl + C::COL_A1 + c, a1);
              tmem_ld16(tl + C::COL_A2 + c, a2);
              tmem_ld_wait();
              if (pv_ok) {
                uint32_t u1[8], u2[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  u1[e] = pack_half2(a1[2 * e], a1[2 * e + 1]);
                  u2[e] = pack_half2(a2[2 * e] * p.scale, a2[2 * e + 1] * p.scale);
                }
                reinterpret_cast<uint4*>(dvrow + c)[0] = make_uint4(u1[0], u1[1], u1[2], u1[3]);
                reinterpret_cast<uint4*>(dvrow + c)[1] = make_uint4(u1[4], u1[5], u1[6], u1[7]);
                reinterpret_cast<uint4*>(dkrow + c)[0] = make_uint4(u2[0], u2[1], u2[2], u2[3]);
                reinterpret_cast<uint4*>(dkrow + c)[1] = make_uint4(u2[4], u2[5], u2[6], u2[7]);
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(acc_free);
        // Join the two groups' per-key sums (fixed order: group 0 + group 1).
        if (grp == 1) {
          xg[r] = pv_g;
          xw[r] = pv_w;
        }
        rows_sync();
        if (pv_ok && grp == 0) {
          p.dpsi[size_t(pv_z) * p.T + pv_s] = -pv_bh * (pv_g + xg[r]);
          p.w[size_t(pv_z) * p.TP + pv_s] = pv_w + xw[r];
        }
        const float db = rows_sum(pv_db, red);  // xg, xw are next written after rows_all
        if (threadIdx.x == kRowWarp0 * 32) p.dbeta[size_t(pv_z) * p.NB + pv_j] = db;
      }
      if (!more) break;

      const int nsteps = p.NB - j;
      const float betal = bh * kLog2e;
      const float c2_s = suf_s < kInf ? -suf_s * p.il2 : -kInf;
      const float* bmin = p.bmin + size_t(z) * p.NB;
      const float* bl = p.bl + size_t(z) * p.NB;
      const float2 bet2 = make_float2(betal, betal);
      const float2 npsi2 = make_float2(-psi_s, -psi_s);
      float gsum = 0.f, dbsum = 0.f, wsum = 0.f;
      float2 gsum2 = make_float2(0.f, 0.f), dbsum2 = make_float2(0.f, 0.f);
      float mid = kInf, midl = -kInf;
      // Per-tile scalars of query tile i (those of the first tile were loaded above), loaded one tile ahead so
      // their latency hides behind the element work.
      const float* prer = p.prer + size_t(z) * p.NB;
      for (int k = 0; k < nsteps && ok; ++k) {
        const int gt = gk + k, st = gt % C::NS, i = j + k;
        const float bli = bl_n, bmini = bmin_n, preri = prer_n;
        if (i + 1 < p.NB) {
          bl_n = bl[i + 1];
          bmin_n = bmin[i + 1];
          prer_n = prer[i + 1];
        }
        const int n = gn + 2 * k + grp, slot = n % C::NSLOT;
        ok = mbar_wait(st_full + st, (gt / C::NS) & 1, p.status, 120);
        if (ok) ok = mbar_wait(s_full + slot, (n / C::NSLOT) & 1, p.status, 121);
        if (!ok) break;
        tc_fence_after();
        // TMEM addresses of this job's S and dP columns, offset so that column c of the tile (cb <= c < cb + 64)
        // is at tS + c and tP + c (unsigned wrap-around keeps the sums exact).
        const uint32_t tS = tl + uint32_t(slot * 128) - uint32_t(cb), tP = tS + kHalf;
        const uint8_t* vbase = smem + C::OFF_VEC + st * C::VECSTAGE;
        const float4* QV = reinterpret_cast<const float4*>(vbase);  // query pairs: (-lse, -delta), (PRE, prey)
        const float* vprel = reinterpret_cast<const float*>(vbase + 4 * C::VECB);
        const float* vphi = reinterpret_cast<const float*>(vbase + 5 * C::VECB);
        const bool diag = k == 0;
        const float cmid2 = mid < kInf ? -mid * p.il2 : -kInf;
        float rs = fmaxf(c2_s, cmid2);
        const bool vrs = !diag && rs > -kInf;
        rs = vrs ? rs : 0.f;
        const float sv_ = ex2(sufl_s - rs) + ex2(midl - rs);
        // 2^{PREL_t - rs} = prey_t * 2^{BL_i - rs} when both factors stay in range (no exp2 per element).
        // Warp-uniform: the chunk body holds warp-collective TMEM loads and stores, so the whole warp takes the
        // factorised path or none of it does. Keys without a soft-min sum on this tile (!vrs: the last key of the
        // tile on the first tile past the diagonal) discard their denominators, so they take either path.
        const bool fact = __all_sync(0xffffffffu, !vrs || (preri <= 120.f && bli - rs <= 120.f));
        const float xfac = (fact && vrs) ? ex2(bli - rs) : 0.f;
        const float2 xf2 = make_float2(xfac, xfac), sv2 = make_float2(sv_, sv_);
        const int tvalid = p.T - i * kBT;  // queries c < tvalid exist (padded ones carry lse = +inf: P = 0)
        // Off the diagonal x_ts = min(a_s, PRE_t - psi_s) with a_s = min(SUF_s - psi_s, mid - psi_s): x_ts <= 0 iff
        // a_s <= 0 or PRE_t <= psi_s, and min(x_ts, 0) = min(min(a_s, 0), PRE_t - psi_s).
        const float a_s = fminf(xs_s, mid - psi_s);
        const float am = fminf(a_s, 0.f);
        const bool pa = a_s <= 0.f;
        // Diagonal tile: rr = min phi over (key, query]; the second group starts from the minimum over (key, 63].
        float rr = kInf;
        if (diag && grp == 1)
          for (int c = 0; c < kHalf; ++c)
            if (c > r) rr = fminf(rr, vphi[c]);
        float2 fsum2 = make_float2(0.f, 0.f);
        float* grow = C::FUSEDIAG ? nullptr : p.gd + ((size_t(z) * p.NB + j) * kBT + r) * kBT;
        // 16 query columns per chunk: load S^T and dP^T, compute, write P^T and dS^T (fp16) over the first 8 of
        // those 16 columns. DIAG and FACT are compile-time so the element loop has no branches; off the diagonal
        // two queries are handled per step with packed f32x2 arithmetic.
        auto chunk = [&](int c0, float(&sS)[16], float(&sP)[16], auto diag_tag, auto fact_tag) {
          constexpr bool DIAG = decltype(diag_tag)::value;
          constexpr bool FACT = decltype(fact_tag)::value;
          uint32_t ppk[8], dpk[8];
          if constexpr (DIAG) {
            float gb[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int c = c0 + e;
              const float4 va = QV[c0 + (e & ~1)];
              const float nl = (e & 1) ? va.y : va.x, nd = (e & 1) ? va.w : va.z;
              rr = c > r ? fminf(rr, vphi[c]) : rr;
              const float x = rr - psi_s;  // +inf for c <= r
              const float xm = fminf(x, 0.f);
              const float sv = fmaf(sS[e], p.scale2, betal * xm);
              const bool valid = s_ok && c >= r && c < tvalid;
              const float pp = valid ? ex2(sv + nl) : 0.f;
              const float ds = valid ? pp * (sP[e] + nd) : 0.f;
              const float g = x <= 0.f ? ds : 0.f;
              gsum += g;
              dbsum = fmaf(ds, xm, dbsum);
              gb[e] = g;
              sS[e] = pp;
              sP[e] = ds;
            }
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              ppk[e / 2] = pack_half2(sS[e], sS[e + 1]);
              dpk[e / 2] = pack_half2(sP[e], sP[e + 1]);
            }
            if constexpr (C::FUSEDIAG) {
              float* grs = reinterpret_cast<float*>(smem + C::OFF_G) + r * C::GLD + c0;
#pragma unroll
              for (int e = 0; e < 16; ++e) grs[e] = gb[e];
            } else {
              float4* dst = reinterpret_cast<float4*>(grow + c0);
#pragma unroll
              for (int q = 0; q < 4; ++q) dst[q] = make_float4(gb[4 * q], gb[4 * q + 1], gb[4 * q + 2], gb[4 * q + 3]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float4 va = QV[c0 + e];      // (-lse_c, -lse_c1, -delta_c, -delta_c1)
              const float4 vb = QV[c0 + e + 1];  // (PRE_c, PRE_c1, prey_c, prey_c1)
              const float2 dd = __fadd2_rn(make_float2(vb.x, vb.y), npsi2);
              const float2 xm = make_float2(fminf(am, dd.x), fminf(am, dd.y));
              const bool in0 = pa || dd.x <= 0.f, in1 = pa || dd.y <= 0.f;
              const float2 sv = __ffma2_rn(make_float2(sS[e], sS[e + 1]), sc2,
                                           __ffma2_rn(bet2, xm, make_float2(va.x, va.y)));
              const float2 pp = make_float2(ex2(sv.x), ex2(sv.y));
              const float2 ds = __fmul2_rn(pp, __fadd2_rn(make_float2(sP[e], sP[e + 1]), make_float2(va.z, va.w)));
              const float2 g = make_float2(in0 ? ds.x : 0.f, in1 ? ds.y : 0.f);
              gsum2 = __fadd2_rn(gsum2, g);
              dbsum2 = __ffma2_rn(ds, xm, dbsum2);
              float2 den;
              if constexpr (FACT)
                den = __ffma2_rn(make_float2(vb.z, vb.w), xf2, sv2);
              else
                den = make_float2(sv_ + ex2(vprel[c0 + e] - rs), sv_ + ex2(vprel[c0 + e + 1] - rs));
              fsum2 = __ffma2_rn(g, make_float2(rcp_approx(den.x), rcp_approx(den.y)), fsum2);
              ppk[e / 2] = pack_half2(pp.x, pp.y);
              dpk[e / 2] = pack_half2(ds.x, ds.y);
            }
          }
          tmem_st8(tS + c0, ppk);
          tmem_st8(tP + c0, dpk);
        };
        // The group's four chunks, ascending, with the TMEM loads of the next chunk in flight during the current one.
        auto tile = [&](auto diag_tag, auto fact_tag) {
          float sA[16], pA[16], sB[16], pB[16];
          tmem_ld16(tS + cb, sA);
          tmem_ld16(tP + cb, pA);
          tmem_ld_wait_regs(sA, pA);
#pragma unroll
          for (int q = 0; q < kHalf / 16; q += 2) {
            const int c0 = cb + 16 * q;
            tmem_ld16(tS + c0 + 16, sB);
            tmem_ld16(tP + c0 + 16, pB);
            chunk(c0, sA, pA, diag_tag, fact_tag);
            tmem_ld_wait_regs(sB, pB);
            if (q + 2 < kHalf / 16) {
              tmem_ld16(tS + c0 + 32, sA);
              tmem_ld16(tP + c0 + 32, pA);
            }
            chunk(c0 + 16, sB, pB, diag_tag, fact_tag);
            if (q + 2 < kHalf / 16) tmem_ld_wait_regs(sA, pA);
          }
        };
        if (diag) {
          // The diagonal tile writes its g into G: the soft-min warps must be done with the previous unit's.
          if (C::FUSEDIAG && u > 0) ok = mbar_wait(g_free, (u - 1) & 1, p.status, 123);
          if (!ok) break;
          tile(std::true_type{}, std::false_type{});
        }
        else if (fact)
          tile(std::false_type{}, std::true_type{});
        else
          tile(std::false_type{}, std::false_type{});
        if (C::FUSEDIAG && diag) mbar_arrive(g_full);  // release: the g columns written above
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full + slot);
        if (!diag) {
          const float fsum = vrs ? fsum2.x + fsum2.y : 0.f;
          if (vrs) wsum += ex2(c2_s - rs) * fsum;
          if (i > j + 1) {
            // Tile-pair total: one partial per warp (8 per pair), summed in a fixed order by the dphi kernel.
            const float tot = group_sum<32>(vrs ? ex2(cmid2 - rs) * fsum : 0.f);
            if (lane == 0) p.tb[((size_t(z) * p.NB + i) * p.NB + j) * kTcTbParts + (warp - kRowWarp0)] = tot;
          }
          mid = fminf(mid, bmini);
          midl = lse2(midl, bli);
        }
      }
      gsum += gsum2.x + gsum2.y;
      dbsum += dbsum2.x + dbsum2.y;
      have_prev = true;
      pv_done = ok;
      pv_ok = s_ok && ok;
      pv_s = s;
      pv_j = j;
      pv_b = b;
      pv_h = h;
      pv_z = z;
      pv_g = gsum;
      pv_db = dbsum;
      pv_w = wsum;
      pv_bh = bh;
      gn += 2 * nsteps;
      gk += nsteps;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------- q-pass ----
// Persistent: one CTA per SM takes work units (query tile i of one head; longest first) from a counter in the
// workspace until none is left. The producer stages each unit's Q and dO tiles by TMA while the previous unit runs;
// at a unit boundary the row threads read dQ out of TMEM, copy the next unit's Q and dO rows from the staging buffer
// into TMEM, and only then store dQ and DPHI2 of the finished unit, so the next unit's first products are computed
// meanwhile. Jobs, tiles and units are numbered across units, which sets every slot, stage and barrier phase.
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
tc_bwd_q_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                const TcBwdParams p) {
  using C = TcBwdCfg<D, false>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* st_full = bars;
  uint64_t* st_empty = st_full + C::NS;
  uint64_t* s_full = st_empty + C::NS;  // [NSLOT] S and dP of the job in the slot are ready
  uint64_t* p_full = s_full + C::NSLOT;  // [NSLOT] the group of the job in the slot has written its dS
  uint64_t* acc_done = p_full + C::NSLOT;  // every MMA of the unit has completed (dQ final)
  uint64_t* acc_free = acc_done + 1;       // the row threads have read dQ out of TMEM
  uint64_t* drain = acc_free + 1;
  uint64_t* at_full = drain + 1;  // the unit's Q and dO rows are in TMEM
  uint64_t* x_full = at_full + 1;  // the unit's Q and dO tiles are in the staging buffer
  uint64_t* x_empty = x_full + 1;  // the row threads have copied the staging buffer
  uint64_t* u_full = x_empty + 1;  // [kUQ] unit ids handed from the producer to the MMA warp and the rows
  uint64_t* u_empty = u_full + kUQ;
  uint64_t* s_last = u_empty + kUQ;  // once per unit: its last S / dP products are complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_last + 1);
  int* uq = reinterpret_cast<int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nbh = p.B * p.H;
  const int nunits = p.NB * nbh;
  // Q and dO (stationary) as TMEM operands of S and dP.
  constexpr int COL_Q = C::COL_X, COL_DO = COL_Q + D / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(st_full + s, 1);
      mbar_init(st_empty + s, 1);
    }
    for (int x = 0; x < C::NSLOT; ++x) {
      mbar_init(s_full + x, 1);
      mbar_init(p_full + x, kGroupThreads);
    }
    mbar_init(acc_done, 1);
    mbar_init(acc_free, kRowThreads);
    mbar_init(drain, 1);
    mbar_init(at_full, kRowThreads);
    mbar_init(x_full, 1);
    mbar_init(x_empty, kRowThreads);
    for (int x = 0; x < kUQ; ++x) {
      mbar_init(u_full + x, 1);
      mbar_init(u_empty + x, 1 + kRowThreads / 32);  // the MMA warp and each row warp
    }
    mbar_init(s_last, 1);
    fence_mbar_init();
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < kRowWarp0) regs_producer<D>();

  if (warp == kWarpProducer) {
    if (elect_one()) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&tdo);
    }
    __syncwarp();
    bool ok = true;
    int gk = 0, nx = 0;  // tiles and staged units issued so far
    for (int u = 0; ok; ++u) {
      const int us = u % kUQ;
      if (u >= kUQ) ok = mbar_wait(u_empty + us, ((u / kUQ) - 1) & 1, p.status, 230);
      if (!ok) break;
      int x = 0;
      if (lane == 0) {
        x = atomicAdd(p.sched + 1, 1);
        uq[us] = x;
        mbar_arrive(u_full + us);
      }
      x = __shfl_sync(0xffffffffu, x, 0);
      if (x >= nunits) break;
      const int i = p.NB - 1 - x / nbh, z = x % nbh, b = z / p.H, h = z % p.H;
      const size_t zb = size_t(z) * p.TP;
      if (nx > 0) ok = mbar_wait(x_empty, (nx - 1) & 1, p.status, 231);
      if (!ok) break;
      if (elect_one()) {
        mbar_expect_tx(x_full, 2 * C::TILEB);
        for (int bx = 0; bx < C::NBOX; ++bx) {
          tma_load_4d(smem + C::OFF_X + bx * C::BOXB, &tq, bx * C::BOXC, i * kBT, h, b, x_full);
          tma_load_4d(smem + C::OFF_X + C::TILEB + bx * C::BOXB, &tdo, bx * C::BOXC, i * kBT, h, b, x_full);
        }
      }
      __syncwarp();
      ++nx;
      for (int k = 0; k <= i && ok; ++k, ++gk) {
        const int st = gk % C::NS, j = i - k;
        if (gk >= C::NS) ok = mbar_wait(st_empty + st, ((gk / C::NS) - 1) & 1, p.status, 201);
        if (!ok) break;
        if (elect_one()) {
          uint8_t* vec = smem + C::OFF_VEC + st * C::VECSTAGE;
          mbar_expect_tx(st_full + st, 2 * C::TILEB + 5 * C::VECB);
          for (int bx = 0; bx < C::NBOX; ++bx) {
            tma_load_4d(smem + C::OFF_S1 + st * C::TILEB + bx * C::BOXB, &tk, bx * C::BOXC, j * kBT, h, b,
                        st_full + st);
            tma_load_4d(smem + C::OFF_S2 + st * C::TILEB + bx * C::BOXB, &tv, bx * C::BOXC, j * kBT, h, b,
                        st_full + st);
          }
          const size_t off = zb + size_t(j) * kBT;
          bulk_load(vec, p.kv4 + off, 4 * C::VECB, st_full + st);
          bulk_load(vec + 4 * C::VECB, p.phi + off, C::VECB, st_full + st);
        }
        __syncwarp();
      }
    }
    // Nothing may land in shared memory after the CTA exits: wait for the last copies issued.
    for (int q = (gk > C::NS ? gk - C::NS : 0); q < gk; ++q) mbar_wait(st_full + q % C::NS, (q / C::NS) & 1, p.status, 203);
    if (nx > 0) mbar_wait(x_full, (nx - 1) & 1, p.status, 204);
  } else if (warp == kWarpMma) {
    // Jobs n = 2 k + g of a unit in order (key tile k, row group g = key columns [64 g, 64 g + 64)); with gn jobs
    // before the unit, S and dP of job n go into slot (gn + n) % NSLOT; once the group has written dS there,
    // dQ += dS K over its 64 keys, then the products of job n + NSLOT into the same slot (in issue order, so the
    // read of dS comes first). The first dQ product of a unit overwrites dQ, so it waits until the rows have read
    // the previous unit's.
    const uint32_t s1 = smem_u32(smem + C::OFF_S1), s2 = smem_u32(smem + C::OFF_S2);
    bool ok = true;
    int gn = 0, gk = 0, loaded = -1;
    for (int u = 0; ok; ++u) {
      const int us = u % kUQ;
      ok = mbar_wait(u_full + us, (u / kUQ) & 1, p.status, 232);
      if (!ok) break;
      const int x = uq[us];
      __syncwarp();
      if (lane == 0) mbar_arrive(u_empty + us);
      if (x >= nunits) break;
      const int i = p.NB - 1 - x / nbh;
      const int njobs = 2 * (i + 1);
      auto need_tile = [&](int kt) {
        const int gt = gk + kt;
        if (ok && gt > loaded) {
          ok = mbar_wait(st_full + gt % C::NS, (gt / C::NS) & 1, p.status, 211);
          loaded = gt;
          tc_fence_after();
        }
        return ok;
      };
      auto issue_s = [&](int n) {
        const int g = n & 1, st = (gk + (n >> 1)) % C::NS, sl = (gn + n) % C::NSLOT;
        const uint32_t dcol = tmem + sl * 128;
        issue_ts_k<D>(dcol, tmem + COL_Q, s1 + st * C::TILEB + g * kHalf * C::SWB);           // S  = Q K^T
        issue_ts_k<D>(dcol + kHalf, tmem + COL_DO, s2 + st * C::TILEB + g * kHalf * C::SWB);  // dP = dO V^T
        mma_commit_w(s_full + sl);
        if (n == njobs - 1) mma_commit_w(s_last);
      };
      ok = mbar_wait(at_full, u & 1, p.status, 210);
      tc_fence_after();
      for (int n = 0; n < C::NSLOT && n < njobs; ++n)
        if (need_tile(n >> 1)) issue_s(n);
      for (int n = 0; n < njobs && ok; ++n) {
        const int g = n & 1, st = (gk + (n >> 1)) % C::NS, sl = (gn + n) % C::NSLOT;
        ok = mbar_wait(p_full + sl, ((gn + n) / C::NSLOT) & 1, p.status, 212);
        if (ok && n == 0 && u > 0) ok = mbar_wait(acc_free, (u - 1) & 1, p.status, 215);
        if (!ok) break;
        tc_fence_after();
        issue_ts_half<D>(tmem + C::COL_A1, tmem + sl * 128 + kHalf, s1 + st * C::TILEB, g, n > 0);
        if (g == 1) mma_commit_w(st_empty + st);
        const int m = n + C::NSLOT;
        if (m < njobs && need_tile(m >> 1)) issue_s(m);
      }
      mma_commit_w(acc_done);
      gn += njobs;
      gk += njobs / 2;
    }
    mma_commit_w(drain);
    mbar_wait(drain, 0, p.status, 214);
  } else if (warp >= kRowWarp0) {
    regs_rows<D>();
    const int grp = (warp - kRowWarp0) >> 2, wr = warp & 3;
    const int r = wr * 32 + lane;  // query within the tile = TMEM lane
    const int cb = grp * kHalf;    // this group's key columns [cb, cb + 64)
    const uint32_t tl = tmem + (uint32_t(wr * 32) << 16);
    constexpr int DH = D >= 32 ? D / 2 : D;  // head-dim columns of dQ stored by each group
    const float2 sc2 = make_float2(p.scale2, p.scale2);
    float* rx = red + 32;
    float* rsh = red + 32 + kBT;
    float* csh = red + 32 + 2 * kBT;
    bool ok = true;
    int gn = 0, gk = 0;
    // The finished unit, read out and written after the next unit's Q and dO rows are in TMEM.
    bool have_prev = false, pv_done = false;
    int pv_t = 0, pv_i = 0, pv_b = 0, pv_h = 0;
    size_t pv_zb = 0;
    bool pv_ok = false;
    float pv_racc = 0.f, pv_c2 = 0.f, pv_a2 = 0.f;
    for (int u = 0;; ++u) {
      const int us = u % kUQ;
      int x = nunits;
      if (ok) ok = mbar_wait(u_full + us, (u / kUQ) & 1, p.status, 233);
      if (ok) x = uq[us];
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(u_empty + us);
      const bool more = rows_all(ok && x < nunits);
      const int i = more ? p.NB - 1 - x / nbh : 0;
      const int z = more ? x % nbh : 0, b = z / p.H, h = z % p.H;
      const size_t zb = size_t(z) * p.TP;
      const int t = i * kBT + r;
      const bool t_ok = more && t < p.T;
      // The unit's per-query and per-tile scalars, loaded first so that their latency passes during the copy below
      // and the previous unit's write-out.
      float2 nl_nd = make_float2(0.f, 0.f);
      float pre_t = 0.f, prel_t = 0.f, phi_t = 0.f, beta_h = 0.f, bl_n = 0.f, bmin_n = 0.f, sufr_n = 0.f,
            sufl0_n = 0.f;
      if (more) {
        const float* own = reinterpret_cast<const float*>(p.qv4 + zb + (t & ~1));  // (-lse, -delta) pair of t
        nl_nd = make_float2(own[t & 1], own[2 + (t & 1)]);  // -lse is -inf beyond T
        pre_t = p.pre[zb + t];
        prel_t = p.prel[zb + t];
        phi_t = p.phi[zb + t];
        beta_h = p.beta[h];
        bl_n = p.bl[size_t(z) * p.NB + i];
        bmin_n = p.bmin[size_t(z) * p.NB + i];
        sufr_n = p.sufr[size_t(z) * p.NB + i];
        sufl0_n = p.sufl[zb + size_t(i) * kBT];
      }
      // The previous unit's last S / dP products (the last readers of the Q and dO columns) are complete: s_last
      // is waited in unit order, and its next phase needs this unit's Q and dO.
      if (have_prev && ok) ok = mbar_wait(s_last, (u - 1) & 1, p.status, 235);
      if (more) {
        // Group 0 copies the query's row of Q, group 1 its row of dO, into TMEM.
        ok = ok && mbar_wait(x_full, u & 1, p.status, 234);
        if (ok) {
          stage_row_to_tmem<D>(tl + (grp == 0 ? COL_Q : COL_DO), smem + C::OFF_X + grp * C::TILEB, r);
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(at_full);
        mbar_arrive(x_empty);
      }
      if (have_prev) {
        // dQ of the finished unit out of TMEM (its MMAs have completed); the MMA warp may then start this unit's.
        float dqv[DH];
        bool done = pv_done && mbar_wait(acc_done, (u - 1) & 1, p.status, 222);
        done = __all_sync(0xffffffffu, done);  // warp-uniform: the TMEM loads below are warp-collective
        if (done) {
          tc_fence_after();
          if (D >= 32 || grp == 0) {
#pragma unroll
            for (int c = 0; c < DH; c += 16) tmem_ld16(tl + C::COL_A1 + grp * DH + c, dqv + c);
            tmem_ld_wait();
          }
        }
        tc_fence_before();
        mbar_arrive(acc_free);
        if (!done) ok = false;
        if (done && pv_ok && (D >= 32 || grp == 0)) {
          __half* dqrow = p.dq + pv_b * p.dq_s[0] + pv_h * p.dq_s[1] + int64_t(pv_t) * p.dq_s[2] + grp * DH;
#pragma unroll
          for (int c = 0; c < DH; c += 8) {
            uint32_t w4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) w4[e] = pack_half2(dqv[c + 2 * e] * p.scale, dqv[c + 2 * e + 1] * p.scale);
            reinterpret_cast<uint4*>(dqrow + c)[0] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
        // DPHI2_u = sum_{t >= u in this tile} 2^{a2_u - c2_t} r_t  (u in the query's own tile), with r_t joining
        // the two groups' partial sums in a fixed order. PRE is non-increasing within the tile, so
        //   DPHI2_u = 2^{a2_u - c2_u} Q_u,  Q_u = r_u + f_u Q_{u+1},  f_u = 2^{c2_u - c2_{u+1}} <= 1,
        // a linear recurrence that contracts; the first row warp solves it: four positions per lane, then a suffix
        // scan of the lanes' affine maps Q_{4l} = A + B Q_{4l+4}.
        if (grp == 1) rx[r] = pv_racc;
        rows_sync();
        if (grp == 0) {
          rsh[r] = pv_racc + rx[r];
          csh[r] = pv_c2;
        }
        rows_sync();
        if (warp == kRowWarp0) {
          const int tend = min(kBT, p.T - pv_i * kBT);
          float rv[4], fv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int u = 4 * lane + e;
            rv[e] = u < tend ? rsh[u] : 0.f;
            fv[e] = u + 1 < tend ? ex2(csh[u] - csh[u + 1]) : 0.f;
          }
          float A = rv[3], Bm = fv[3];
#pragma unroll
          for (int e = 2; e >= 0; --e) {
            A = fmaf(fv[e], A, rv[e]);
            Bm *= fv[e];
          }
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const float A2 = __shfl_down_sync(0xffffffffu, A, o), B2 = __shfl_down_sync(0xffffffffu, Bm, o);
            if (lane + o < 32) {
              A = fmaf(Bm, A2, A);
              Bm *= B2;
            }
          }
          float qn = __shfl_down_sync(0xffffffffu, A, 1);  // Q_{4l+4}
          if (lane == 31) qn = 0.f;
#pragma unroll
          for (int e = 3; e >= 0; --e) {
            qn = fmaf(fv[e], qn, rv[e]);
            rsh[4 * lane + e] = qn;
          }
        }
        rows_sync();
        // rsh, csh and rx are next written after the rows_all of the next unit.
        if (grp == 0 && pv_ok) p.dphi2[pv_zb + pv_t] = ex2(pv_a2 - pv_c2) * rsh[r];
      }
      if (!more) break;

      const int nsteps = i + 1;
      const float betal = beta_h * kLog2e;
      const float nlse = nl_nd.x, ndel = nl_nd.y;
      const float c2_t = t_ok ? -pre_t * p.il2 : 0.f;
      const float bpre = t_ok ? ex2(prel_t - c2_t) : 1.f;
      const float a2_t = t_ok ? -phi_t * p.il2 : 0.f;  // for DPHI2 of this unit
      const float* bmin = p.bmin + size_t(z) * p.NB;
      const float* bl = p.bl + size_t(z) * p.NB;
      const float2 bet2 = make_float2(betal, betal);
      const float2 nlse2 = make_float2(nlse, nlse), ndel2 = make_float2(ndel, ndel);
      float2 racc2 = make_float2(0.f, 0.f);
      float mid = kInf, midl = -kInf;
      // Per-tile scalars of key tile j (those of the first tile were loaded above), loaded one tile ahead so their
      // latency hides behind the element work.
      const float* sufr = p.sufr + size_t(z) * p.NB;
      for (int k = 0; k < nsteps && ok; ++k) {
        const int gt = gk + k, st = gt % C::NS, j = i - k;
        const float blj = bl_n, bminj = bmin_n, sufrj = sufr_n, sufl0 = sufl0_n;
        if (j > 0) {
          bl_n = bl[j - 1];
          bmin_n = bmin[j - 1];
          sufr_n = sufr[j - 1];
          sufl0_n = p.sufl[zb + size_t(j - 1) * kBT];
        }
        const int n = gn + 2 * k + grp, slot = n % C::NSLOT;
        ok = mbar_wait(st_full + st, (gt / C::NS) & 1, p.status, 220);
        if (ok) ok = mbar_wait(s_full + slot, (n / C::NSLOT) & 1, p.status, 221);
        if (!ok) break;
        tc_fence_after();
        // TMEM addresses of this job's S and dP columns, offset so that column c of the tile (cb <= c < cb + 64)
        // is at tS + c and tP + c (unsigned wrap-around keeps the sums exact).
        const uint32_t tS = tl + uint32_t(slot * 128) - uint32_t(cb), tP = tS + kHalf;
        const uint8_t* vbase = smem + C::OFF_VEC + st * C::VECSTAGE;
        const float4* KV = reinterpret_cast<const float4*>(vbase);  // key pairs: (SUF - psi, -psi), (sufy, SUFL)
        const float* vphi = reinterpret_cast<const float*>(vbase + 4 * C::VECB);
        const bool diag = k == 0;
        const float cap = fminf(mid, pre_t);
        const float mterm = ex2(midl - c2_t) + bpre;
        // 2^{SUFL_s - c2_t} = sufy_s * 2^{SUFL_first - c2_t} when both factors stay in range.
        // Warp-uniform (the chunk body holds warp-collective TMEM loads and stores). Rows beyond T take either path.
        const bool fact = __all_sync(0xffffffffu, !diag && (!t_ok || (sufrj <= 120.f && sufl0 - c2_t <= 120.f)));
        const float yfac = (fact && t_ok) ? ex2(sufl0 - c2_t) : 0.f;
        const float2 cap2 = make_float2(cap, cap), yf2 = make_float2(yfac, yfac), mt2 = make_float2(mterm, mterm);
        const int kvalid = p.T - j * kBT;  // keys c < kvalid exist
        // Diagonal tile, keys descending: rr = min phi over (key, query]; the first group starts from the minimum
        // over the second group's keys up to the query, [64, query].
        float rr = kInf;
        if (diag && grp == 0)
          for (int c = kHalf; c < kBT; ++c)
            if (c <= r) rr = fminf(rr, vphi[c]);
        // 16 key columns per chunk: load S and dP, compute dS (fp16) and write it over the first 8 of those 16 dP
        // columns. DIAG and FACT are compile-time so the element loop has no branches; off the diagonal two keys
        // are handled per step with packed f32x2 arithmetic.
        auto chunk = [&](int c0, float(&sS)[16], float(&sP)[16], auto diag_tag, auto fact_tag) {
          constexpr bool DIAG = decltype(diag_tag)::value;
          constexpr bool FACT = decltype(fact_tag)::value;
          uint32_t dpk[8];
          if constexpr (DIAG) {
#pragma unroll
            for (int e = 15; e >= 0; --e) {
              const int c = c0 + e;
              const float4 va = KV[c0 + (e & ~1)];
              const float npsi = (e & 1) ? va.w : va.z;
              const float x = rr + npsi;  // +inf at c == r
              rr = c <= r ? fminf(rr, vphi[c]) : rr;
              const float xm = fminf(x, 0.f);
              const float sv = fmaf(sS[e], p.scale2, betal * xm);
              const bool valid = c <= r && c < kvalid;
              sP[e] = valid ? ex2(sv + nlse) * (sP[e] + ndel) : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 16; e += 2) dpk[e / 2] = pack_half2(sP[e], sP[e + 1]);
          } else {
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float4 va = KV[c0 + e];      // (SUF_c - psi_c, SUF_c1 - psi_c1, -psi_c, -psi_c1)
              const float4 vb = KV[c0 + e + 1];  // (sufy_c, sufy_c1, SUFL_c, SUFL_c1)
              const float2 dd = __fadd2_rn(cap2, make_float2(va.z, va.w));
              const float2 x = make_float2(fminf(va.x, dd.x), fminf(va.y, dd.y));
              const float2 xm = make_float2(fminf(x.x, 0.f), fminf(x.y, 0.f));
              const float2 sv = __ffma2_rn(make_float2(sS[e], sS[e + 1]), sc2, __ffma2_rn(bet2, xm, nlse2));
              const float2 pp = make_float2(ex2(sv.x), ex2(sv.y));
              const float2 ds = __fmul2_rn(pp, __fadd2_rn(make_float2(sP[e], sP[e + 1]), ndel2));
              const float2 g = make_float2(x.x <= 0.f ? ds.x : 0.f, x.y <= 0.f ? ds.y : 0.f);
              float2 den;
              if constexpr (FACT)
                den = __ffma2_rn(make_float2(vb.x, vb.y), yf2, mt2);
              else
                den = make_float2(ex2(vb.z - c2_t) + mterm, ex2(vb.w - c2_t) + mterm);
              racc2 = __ffma2_rn(g, make_float2(rcp_approx(den.x), rcp_approx(den.y)), racc2);
              dpk[e / 2] = pack_half2(ds.x, ds.y);
            }
          }
          tmem_st8(tP + c0, dpk);
        };
        // The group's four chunks, descending, with the TMEM loads of the next chunk in flight during the current
        // one.
        auto tile = [&](auto diag_tag, auto fact_tag) {
          float sA[16], pA[16], sB[16], pB[16];
          const int top = cb + kHalf - 16;
          tmem_ld16(tS + top, sA);
          tmem_ld16(tP + top, pA);
          tmem_ld_wait_regs(sA, pA);
#pragma unroll
          for (int q = 0; q < kHalf / 16; q += 2) {
            const int c0 = top - 16 * q;
            tmem_ld16(tS + c0 - 16, sB);
            tmem_ld16(tP + c0 - 16, pB);
            chunk(c0, sA, pA, diag_tag, fact_tag);
            tmem_ld_wait_regs(sB, pB);
            if (q + 2 < kHalf / 16) {
              tmem_ld16(tS + c0 - 32, sA);
              tmem_ld16(tP + c0 - 32, pA);
            }
            chunk(c0 - 16, sB, pB, diag_tag, fact_tag);
            if (q + 2 < kHalf / 16) tmem_ld_wait_regs(sA, pA);
          }
        };
        if (diag)
          tile(std::true_type{}, std::false_type{});
        else if (fact)
          tile(std::false_type{}, std::true_type{});
        else
          tile(std::false_type{}, std::false_type{});
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full + slot);
        if (!diag) {
          mid = fminf(mid, bminj);
          midl = lse2(midl, blj);
        }
      }
      have_prev = true;
      pv_done = ok;
      pv_t = t;
      pv_i = i;
      pv_b = b;
      pv_h = h;
      pv_zb = zb;
      pv_ok = t_ok && ok;
      pv_racc = racc2.x + racc2.y;
      pv_c2 = c2_t;
      pv_a2 = a2_t;
      gn += 2 * nsteps;
      gk += nsteps;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// The q-pass depends on nothing the kv-pass writes, so it runs on an auxiliary stream forked from the caller's
// stream: its persistent CTAs take over the SMs that the kv-pass's last units leave idle. One auxiliary stream and
// pair of events per calling stream and device, created on first use (under stream capture with the thread's
// capture mode relaxed for the creation calls, which touch no captured work); when none can be had, both passes
// run on the caller's stream.
struct Fork {
  cudaStream_t caller;
  int dev;
  cudaStream_t aux;
  cudaEvent_t fork, join;
};

bool fork_of(cudaStream_t s, Fork* out) {
  static std::mutex mu;
  static Fork table[32];
  static int n = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (table[i].caller == s && table[i].dev == dev) {
      *out = table[i];
      return true;
    }
  if (n == 32) return false;
  Fork f{s, dev, nullptr, nullptr, nullptr};
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  bool ok = cudaStreamCreateWithFlags(&f.aux, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&f.join, cudaEventDisableTiming) == cudaSuccess;
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (!ok) {
    cudaGetLastError();
    return false;
  }
  table[n++] = f;
  *out = f;
  return true;
}

template <int D>
int launch_bwd(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, const KeyCols& cols,
               const Fact& fact, float* gd, const float4* qv4, int* sched, int* status, cudaStream_t s,
               std::string* err) {
  using CK = TcBwdCfg<D, true>;
  using CQ = TcBwdCfg<D, false>;
  CUtensorMap mq, mk, mv, mdo;
  if (!make_tile_map(&mq, a.q, a.q_stride, d.B, d.H, d.T, D) || !make_tile_map(&mk, a.k, a.k_stride, d.B, d.H, d.T, D) ||
      !make_tile_map(&mv, a.v, a.v_stride, d.B, d.H, d.T, D) ||
      !make_tile_map(&mdo, a.dout, a.dout_stride, d.B, d.H, d.T, D)) {
    *err = "cuTensorMapEncodeTiled failed for q, k, v or do";
    return FPA_ERR_CUDA;
  }
  TcBwdParams p;
  p.qv4 = qv4;
  p.kv4 = fact.kv4;
  p.delta = sc.delta;
  p.pre = st.pre;
  p.prel = st.prel;
  p.suf = st.suf;
  p.sufl = st.sufl;
  p.bmin = st.bmin;
  p.bl = st.bl;
  p.xs = cols.a;
  p.psi = cols.psi;
  p.phi = cols.phi;
  p.beta = a.beta;
  p.prey = fact.prey;
  p.sufy = fact.sufy;
  p.prer = fact.prer;
  p.sufr = fact.sufr;
  p.q = static_cast<const __half*>(a.q);
  p.k = static_cast<const __half*>(a.k);
  p.v = static_cast<const __half*>(a.v);
  p.dout = static_cast<const __half*>(a.dout);
  p.dq = static_cast<__half*>(a.dq);
  p.dk = static_cast<__half*>(a.dk);
  p.dv = static_cast<__half*>(a.dv);
  for (int q = 0; q < 3; ++q) {
    p.q_s[q] = a.q_stride[q];
    p.k_s[q] = a.k_stride[q];
    p.v_s[q] = a.v_stride[q];
    p.do_s[q] = a.dout_stride[q];
    p.dq_s[q] = a.dq_stride[q];
    p.dk_s[q] = a.dk_stride[q];
    p.dv_s[q] = a.dv_stride[q];
  }
  p.dpsi = a.dpsi;
  p.w = sc.w;
  p.tb = sc.tb;
  p.dbeta = sc.dbeta;
  p.gd = gd;
  p.dphi4 = sc.dphi4;
  p.dphi2 = sc.dphi2;
  p.status = status;
  p.sched = sched;
  p.B = d.B;
  p.H = d.H;
  p.T = d.T;
  p.NB = d.NB;
  p.TP = d.TP;
  p.scale = float(1.0 / sqrt(double(D)));
  p.scale2 = p.scale * kLog2e;
  p.il2 = kLog2e / a.tau;
  auto kv = tc_bwd_kv_kernel<D>;
  auto qk = tc_bwd_q_kernel<D>;
  const int smem_kv = std::max(CK::SMEM, kPersistentMinSmem), smem_q = std::max(CQ::SMEM, kPersistentMinSmem);
  cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(kv), smem_kv);
  if (e == cudaSuccess) e = allow_dynamic_smem(reinterpret_cast<const void*>(qk), smem_q);
  if (e != cudaSuccess) {
    *err = std::string("tensor-core backward: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  const int grid = d.NB * d.BH();
  const int pgrid = std::min(grid, sm_count());  // persistent; the stats kernel zeroed the unit counters
  Fork f;
  const bool forked = !prof_on() && fork_of(s, &f);  // per-kernel timing needs one stream
  cudaStream_t sq = s;
  if (forked) {
    e = cudaEventRecord(f.fork, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(f.aux, f.fork, 0);
    if (e != cudaSuccess) {
      *err = std::string("tensor-core backward fork: ") + cudaGetErrorString(e);
      return FPA_ERR_CUDA;
    }
    sq = f.aux;
  }
  prof_mark(s, "bwd_kv_tc");
  e = launch_pdl(kv, dim3(pgrid), dim3(kThreads), smem_kv, s, mq, mk, mv, mdo, p);
  if (e == cudaSuccess && !CK::FUSEDIAG) {
    prof_mark(s, "diag_dphi");
    e = launch_diag_dphi(a.phi, gd, d, a.tau, sc.dphi4, s);
  }
  if (e == cudaSuccess) {
    prof_mark(s, "bwd_q_tc");
    qk<<<pgrid, kThreads, smem_q, sq>>>(mq, mk, mv, mdo, p);
    e = cudaGetLastError();
  }
  if (forked) {  // join even after a failed launch, so that no capture is left with a dangling fork
    const cudaError_t e2 = cudaEventRecord(f.join, f.aux);
    const cudaError_t e3 = e2 == cudaSuccess ? cudaStreamWaitEvent(s, f.join, 0) : e2;
    if (e == cudaSuccess) e = e3;
  }
  if (e != cudaSuccess) {
    *err = std::string("tensor-core backward launch: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  return FPA_OK;
}

}  // namespace

// Whether the kv-pass runs the diagonal soft-min itself (else the stored g goes through diag_dphi_kernel).
bool kv_fuses_diag(int D) {
  switch (D) {
    case 16: return TcBwdCfg<16, true>::FUSEDIAG;
    case 32: return TcBwdCfg<32, true>::FUSEDIAG;
    case 64: return TcBwdCfg<64, true>::FUSEDIAG;
    default: return TcBwdCfg<128, true>::FUSEDIAG;
  }
}

size_t gd_bytes(const Dims& d) {
  return kv_fuses_diag(d.D) ? 0 : align256(size_t(d.BH()) * d.NB * size_t(kBT) * kBT * sizeof(float));
}

size_t tc_bwd_extra_bytes(const Dims& d) {
  const size_t bh = size_t(d.BH());
  return keycols_bytes(d) + gd_bytes(d) +
         2 * align256(bh * d.TP * sizeof(float4)) + 2 * align256(bh * d.TP * sizeof(float)) +
         2 * align256(bh * d.NB * sizeof(float));
}

int tc_bwd(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, char* extra, int* status,
           cudaStream_t s, int* launched, std::string* err) {
  *launched = 0;
  if (!tma_layout_ok(a.q, a.q_stride) || !tma_layout_ok(a.k, a.k_stride) || !tma_layout_ok(a.v, a.v_stride) ||
      !tma_layout_ok(a.dout, a.dout_stride)) {
    *err = "the tensor-core path needs q, k, v, do with unit innermost stride and 16-byte aligned rows";
    return FPA_ERR_UNSUPPORTED;
  }
  for (const void* ptr : {a.dq, a.dk, a.dv})
    if (reinterpret_cast<uintptr_t>(ptr) % 16) {
      *err = "the tensor-core path needs 16-byte aligned dq, dk, dv";
      return FPA_ERR_UNSUPPORTED;
    }
  if (a.dq_stride[3] != 1 || a.dk_stride[3] != 1 || a.dv_stride[3] != 1 || (a.dq_stride[2] * 2) % 16 ||
      (a.dk_stride[2] * 2) % 16 || (a.dv_stride[2] * 2) % 16) {
    *err = "the tensor-core path needs dq, dk, dv with unit innermost stride and 16-byte aligned rows";
    return FPA_ERR_UNSUPPORTED;
  }
  const size_t bh = size_t(d.BH());
  KeyCols cols = carve_keycols(extra, d);
  float* gd = kv_fuses_diag(d.D) ? nullptr : reinterpret_cast<float*>(extra + keycols_bytes(d));
  char* q = extra + keycols_bytes(d) + gd_bytes(d);
  float4* qv4 = reinterpret_cast<float4*>(q);
  q += align256(bh * d.TP * sizeof(float4));
  Fact fact;
  fact.kv4 = reinterpret_cast<float4*>(q);
  q += align256(bh * d.TP * sizeof(float4));
  fact.prey = reinterpret_cast<float*>(q);
  q += align256(bh * d.TP * 4);
  fact.sufy = reinterpret_cast<float*>(q);
  q += align256(bh * d.TP * 4);
  fact.prer = reinterpret_cast<float*>(q);
  q += align256(bh * d.NB * 4);
  fact.sufr = reinterpret_cast<float*>(q);
  // Raw key vectors, the factorisation arrays and the per-query pairs (filled by the stats kernel; with O and dO
  // not fp16 and vector-aligned, the pairs by the delta and packing kernels).
  const bool fused = qv_delta_fusable(a.dtype, a.o, str4(a.o_stride), a.dout, str4(a.dout_stride), d);
  const QvIn qin{static_cast<const __half*>(a.o), str4(a.o_stride), static_cast<const __half*>(a.dout),
                 str4(a.dout_stride), a.lse, qv4, d.D};
  prof_mark(s, "stats");
  cudaError_t e =
      launch_stats(a.phi, a.psi, a.beta, d, a.tau, st, cols, 0, status, s, &fact, fused ? &qin : nullptr);
  int nprep = 1;
  if (!fused) {
    if (e == cudaSuccess) {
      prof_mark(s, "delta");
      e = launch_delta(a.dtype, a.o, str4(a.o_stride), a.dout, str4(a.dout_stride), d, sc.delta, nullptr, nullptr, s);
    }
    if (e == cudaSuccess) {
      prof_mark(s, "qv_pack");
      e = launch_qv_pack(a.lse, sc.delta, st.pre, fact.prey, d, qv4, s);
    }
    nprep += 2;
  }
  if (e != cudaSuccess) {
    *err = std::string("tensor-core backward prologue: ") + cudaGetErrorString(e);
    return FPA_ERR_CUDA;
  }
  int rc;
  switch (d.D) {
    case 16: rc = launch_bwd<16>(a, d, st, sc, cols, fact, gd, qv4, status + kSchedKv, status, s, err); break;
    case 32: rc = launch_bwd<32>(a, d, st, sc, cols, fact, gd, qv4, status + kSchedKv, status, s, err); break;
    case 64: rc = launch_bwd<64>(a, d, st, sc, cols, fact, gd, qv4, status + kSchedKv, status, s, err); break;
    case 128: rc = launch_bwd<128>(a, d, st, sc, cols, fact, gd, qv4, status + kSchedKv, status, s, err); break;
    default: *err = "unsupported head dimension for the tensor-core path"; return FPA_ERR_UNSUPPORTED;
  }
  if (rc == FPA_OK) *launched = nprep + (kv_fuses_diag(d.D) ? 2 : 3);  // stats, [delta, pack], kv, [diag], q
  return rc;
}

}  // namespace fpa
