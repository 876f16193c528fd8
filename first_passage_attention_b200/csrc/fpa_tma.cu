// Host-side TMA tensor maps and device queries for the tensor-core kernels.
#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

#include "fpa_tc.h"

namespace fpa {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && cache[dev] > 0) return cache[dev];
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64) cache[dev] = n;
  return n;
}

cudaError_t allow_dynamic_smem(const void* fn, int bytes) {
  struct Entry {
    int dev;
    const void* fn;
    int bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (Entry& x : done)
    if (x.dev == dev && x.fn == fn) {
      if (x.bytes >= bytes) return cudaSuccess;
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e == cudaSuccess) x.bytes = bytes;
      return e;
    }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.push_back(Entry{dev, fn, bytes});
  return e;
}

bool tma_layout_ok(const void* p, const int64_t st[4]) {
  if (reinterpret_cast<uintptr_t>(p) % 16) return false;
  if (st[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if ((st[i] * 2) % 16 || st[i] <= 0) return false;
  return true;
}

namespace {

// The last tensor maps made, keyed by everything the encoding depends on (a map is a pure function of its base,
// sizes and strides): a training loop passes the same buffers call after call, and each encoding costs the host
// about as much as a kernel launch.
struct MapKey {
  const void* base;
  int64_t s0, s1, s2;
  int B, H, T, D;
  bool operator==(const MapKey& o) const {
    return base == o.base && s0 == o.s0 && s1 == o.s1 && s2 == o.s2 && B == o.B && H == o.H && T == o.T && D == o.D;
  }
};
constexpr int kMapCache = 32;
std::mutex g_map_mu;
MapKey g_map_key[kMapCache];
CUtensorMap g_map_val[kMapCache];
int g_map_n = 0, g_map_next = 0;

}  // namespace

bool make_tile_map(CUtensorMap* map, const void* base, const int64_t st[4], int B, int H, int T, int D) {
  const MapKey key{base, st[0], st[1], st[2], B, H, T, D};
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    for (int i = 0; i < g_map_n; ++i)
      if (g_map_key[i] == key) {
        *map = g_map_val[i];
        return true;
      }
  }
  auto fn = encode_fn();
  if (!fn) return false;
  const int boxc = D >= 64 ? 64 : D;
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(T), cuuint64_t(H), cuuint64_t(B)};
  cuuint64_t strides[3] = {cuuint64_t(st[2]) * 2, cuuint64_t(st[1]) * 2, cuuint64_t(st[0]) * 2};
  cuuint32_t box[4] = {cuuint32_t(boxc), cuuint32_t(kTcBT), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMapSwizzle sw = boxc == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : boxc == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                       : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(g_map_mu);
  g_map_key[g_map_next] = key;
  g_map_val[g_map_next] = *map;
  g_map_next = (g_map_next + 1) % kMapCache;
  if (g_map_n < kMapCache) ++g_map_n;
  return true;
}

}  // namespace fpa
