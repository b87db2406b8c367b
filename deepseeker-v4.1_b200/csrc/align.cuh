// Device sort-and-pad of (token, slot) pairs by expert (moe_align.cu), shared by
// the public ds_moe_align entry point and the grouped expert FFN (grouped.cu).
#pragma once

#include "ds_common.cuh"

namespace ds {
namespace align {

constexpr int kMaxExperts = 1024;

struct Out {
  int32_t* sorted_ids;   // [capacity] flat pair index per padded position, sentinel = m * k
  int32_t* expert_ids;   // [capacity / block] expert of each block, or null
  int32_t* n_pad;        // [1] padded length; -1 when an id is out of range
  int32_t* pos_of_pair;  // [m * k] padded position of each pair (-1 = dropped), or null
  int32_t* blk_tile;     // [capacity / block] tile of each block, or null
  int4* tiles;           // [max tiles] {expert, first row, rows, 0}, or null
  int32_t* n_tiles;      // [1], or null
  int tile_rows;         // rows per tile (a multiple of block) when tiles != null
};

// Padded capacity for m*k pairs over E experts: every non-empty expert adds
// at most block - 1 sentinel rows.
inline int64_t capacity(int64_t mk, int E, int block) {
  return mk + (mk < E ? mk : (int64_t)E) * (block - 1);
}

inline int64_t max_tiles(int64_t mk, int E, int block, int tile_rows) {
  return capacity(mk, E, block) / tile_rows + (mk < E ? mk : (int64_t)E) + 1;
}

// allow_dropped: ids < 0 are skipped (pos_of_pair = -1) instead of rejected.
int launch(const int32_t* ids, int64_t mk, int E, int block, int allow_dropped, const Out& o, cudaStream_t st);

}  // namespace align
}  // namespace ds
