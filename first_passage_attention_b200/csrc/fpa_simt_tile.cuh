// Tile loaders shared by the register-tiled FFMA kernels (fpa_simt_fwd.cu, fpa_simt_bwd.cu): 64-position tiles of a
// [B, H, T, D] operand staged in shared memory as float32, transposed ([D][kPitch]) for the outer-product
// contractions or row-major ([64][D]), 256 threads per CTA.
#pragma once

#include "fpa_internal.h"

namespace fpa {
namespace tile {

constexpr int kFT = kSimtBT;       // positions per tile (the FFMA path's field statistics use the same tiles)
constexpr int kFThreads = 256;     // 16 x 16
constexpr int kPitch = kFT + 4;    // row pitch of the transposed Q / K tiles, of P and of the range-minimum table

template <int VW>
__device__ __forceinline__ void ld_vec(float (&v)[VW], const float* p) {
  if constexpr (VW == 4) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
  } else if constexpr (VW == 2) {
    const float2 x = *reinterpret_cast<const float2*>(p);
    v[0] = x.x, v[1] = x.y;
  } else {
    v[0] = p[0];
  }
}

// Four consecutive elements (columns d0 .. d0 + 3) of row t of a [.., T, D] operand as float32, zero when !ok. VEC:
// unit column stride and 16-byte (fp32) / 8-byte (fp16) aligned rows, one vector load; otherwise four scalar loads.
template <typename TIn, bool VEC>
__device__ __forceinline__ void load4(float (&x)[4], const TIn* base, Str4 st, int t, int d0, bool ok) {
  if (!ok) {
    x[0] = x[1] = x[2] = x[3] = 0.f;
    return;
  }
  const TIn* p = base + int64_t(t) * st.t + int64_t(d0) * st.d;
  if constexpr (VEC && sizeof(TIn) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
  } else if constexpr (VEC) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    x[0] = a.x, x[1] = a.y, x[2] = c.x, x[3] = c.y;
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) x[c] = to_f32(p[int64_t(c) * st.d]);
  }
}

// Rows j*64 .. j*64 + 63 of a [.., T, D] operand into shared memory as float32 (rows >= T as zero), times `scale`:
// TRANS, transposed to [D][kPitch] (thread -> (row, four columns), consecutive threads on consecutive rows, so the
// scalar stores hit consecutive banks); otherwise row-major [64][D] (consecutive threads on consecutive columns).
// Every load of a batch is issued before the first store, so one memory latency covers the batch.
// `tid` is the thread's index among the kFThreads threads that share the load.
template <typename TIn, int D, bool TRANS, bool VEC>
__device__ __forceinline__ void load_rows(float* dst, const TIn* base, Str4 st, int j, int T, float scale,
                                          int tid = threadIdx.x) {
  constexpr int NCH = kFT * D / 4 / kFThreads;  // chunks of four per thread (D / 16)
  constexpr int BATCH = NCH < 8 ? NCH : 8;
#pragma unroll
  for (int c0 = 0; c0 < NCH; c0 += BATCH) {
    float x[BATCH][4];
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int e = tid + (c0 + q) * kFThreads;
      const int r = TRANS ? e % kFT : e / (D / 4), d0 = TRANS ? (e / kFT) * 4 : (e % (D / 4)) * 4;
      load4<TIn, VEC>(x[q], base, st, j * kFT + r, d0, j * kFT + r < T);
    }
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int e = tid + (c0 + q) * kFThreads;
      const int r = TRANS ? e % kFT : e / (D / 4), d0 = TRANS ? (e / kFT) * 4 : (e % (D / 4)) * 4;
      if (TRANS) {
#pragma unroll
        for (int c = 0; c < 4; ++c) dst[(d0 + c) * kPitch + r] = x[q][c] * scale;
      } else {
        *reinterpret_cast<float4*>(dst + r * D + d0) =
            make_float4(x[q][0] * scale, x[q][1] * scale, x[q][2] * scale, x[q][3] * scale);
      }
    }
  }
}

// Whether q, k, v can be read four columns per vector load: unit column stride, row and head/batch strides that keep
// every row start aligned to the vector (16 bytes fp32, 8 bytes fp16), aligned bases.
template <typename TIn>
inline bool vec_ok(const void* p, const int64_t st[4]) {
  constexpr int64_t A = 4 * int64_t(sizeof(TIn));
  if (st[3] != 1 || reinterpret_cast<uintptr_t>(p) % A) return false;
  for (int i = 0; i < 3; ++i)
    if ((st[i] * int64_t(sizeof(TIn))) % A) return false;
  return true;
}

}  // namespace tile
}  // namespace fpa
