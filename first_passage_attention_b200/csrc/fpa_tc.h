// Tensor-core (tcgen05 / TMEM / TMA) kernels for sm_100a.
#pragma once

#include <cuda.h>

#include <string>

#include "fpa_internal.h"

namespace fpa {

constexpr int kTcBT = 128;      // positions per tile of the tensor-core kernels (the MMA M and N)
constexpr int kTcTbParts = 8;  // per-warp partial sums of each tile-pair total of the tensor-core kv-pass

bool tc_supports(int D);

// Streaming multiprocessors of the current device (the grid of the persistent kernels).
int sm_count();

// Persistent kernels ask for at least this much shared memory, so that two of them (the kv- and q-pass running
// concurrently) never share an SM and wait for each other's 512 TMEM columns.
constexpr int kPersistentMinSmem = 116 * 1024;

// The 256-byte status block at the head of a workspace: word 0 is the status word, words 1-2 are the work-unit
// counters of the persistent kv-pass and q-pass; the stats kernel that precedes them zeroes words 0-3.
constexpr int kSchedKv = 1;

// True if a [B, H, T, D] fp16 operand with these element strides can be read by TMA as it is (innermost stride 1,
// 16-byte aligned base and strides).
bool tma_layout_ok(const void* p, const int64_t st[4]);

// Tensor map of a [B, H, T, D] fp16 operand: boxes of [128 rows x min(64, D) columns] with the swizzle whose width
// is one box row (128 B for D >= 64, 64 B for D = 32, 32 B for D = 16); rows >= T read as zero.
bool make_tile_map(CUtensorMap* map, const void* base, const int64_t st[4], int B, int H, int T, int D);

// Key-range split of the forward for grids too small to fill the SMs: each query tile's key tiles, from the
// diagonal down, go in chunks of L tiles to separate CTAs (`items_per_head` CTAs per head), whose unnormalised
// outputs the chunk that finishes last joins in chunk order. L = 0: no split. Depends on the current device's SM
// count. FPA_B200_FWD_SPLIT=0 in the environment turns it off (the results then do not depend on how many heads a
// call holds: a head computes bit for bit the same alone or inside a larger batch); FPA_B200_FWD_SPLIT=L (L >= 2)
// sets the chunk length wherever the one-tile kernel runs.
struct FwdSplit {
  int L = 0, items_per_head = 0;
};
FwdSplit tc_fwd_split_plan(const Dims& d);
size_t tc_fwd_split_bytes(const Dims& d);  // workspace for the chunks' partial outputs (0 without a split)
// The split's per-tile join counters ([BH][NB] ints at the head of split_ws, which the stats kernel zeroes), or
// nullptr when this call runs unsplit (no split planned, or split_avail short of tc_fwd_split_bytes).
int* tc_fwd_split_counters(const Dims& d, char* split_ws, size_t split_avail);

// Forward pass on the tensor cores; `status` is the device status word of the workspace and `split_ws` the
// `split_avail` bytes after the key vectors. The key-range split runs only when split_avail covers
// tc_fwd_split_bytes(d); otherwise the unsplit kernels run (same results up to the order of the additions).
// Sets *launched to the number of kernels launched. Returns an FpaStatus; on failure writes a message into *err.
int tc_fwd(const FpaFwdArgs& a, const Dims& d, const Stats& st, const KeyCols& cols, char* split_ws,
           size_t split_avail, int* status, cudaStream_t s, int* launched, std::string* err);

// Backward pass on the tensor cores (fp16). `extra` is tc_bwd_extra_bytes(d) bytes of workspace (raw key vectors,
// the stored g of the diagonal tiles, a padded copy of lse). Launches the field statistics, delta, the kv-pass,
// the diagonal soft-min and the q-pass; the caller then runs the dphi combination and the dbeta reduction.
size_t tc_bwd_extra_bytes(const Dims& d);
int tc_bwd(const FpaBwdArgs& a, const Dims& d, const Stats& st, const BwdScratch& sc, char* extra, int* status,
           cudaStream_t s, int* launched, std::string* err);

}  // namespace fpa
