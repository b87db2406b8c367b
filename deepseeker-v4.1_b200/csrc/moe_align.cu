// Sort-and-pad of flat (token, top-k slot) positions by expert, on the device.
//
// Contract (src/deepseeker/moe_align.py:21-46, align_block_size): flatten
// topk_ids[M, K] row-major; group flat positions by expert, keeping their
// order (stable); pad each expert's run with the sentinel M*K up to a
// multiple of block_size; concatenate experts in id order; report the expert
// of every block and the padded length.
//
// One CTA of 32 warps.  Warp w owns a contiguous segment of the flat array:
// pass 1 counts its ids per expert (match_any groups equal ids inside the
// warp), a block scan turns the per-expert totals into padded run offsets and
// the per-segment counts into within-run offsets, and pass 2 re-reads the
// segment in order and writes each position at run offset + segment offset +
// rank among equal ids of earlier lanes -- the stable order of the reference.
#include "align.cuh"

namespace ds {
namespace align {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

// Exclusive prefix sum over the CTA (one value per thread); *total gets the sum.
__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = warp_sums[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, d);
      if (lane >= d) s += y;
    }
    warp_sums[lane] = s;  // inclusive
  }
  __syncthreads();
  const int before = warp == 0 ? 0 : warp_sums[warp - 1];
  const int r = before + x - v;
  *total = warp_sums[kWarps - 1];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    align_kernel(const int32_t* __restrict__ ids, int mk, int E, int block, int allow_dropped, Out o) {
  extern __shared__ int sm[];
  int* hist = sm;                 // [kWarps][E]: per-segment counts, then within-run offsets
  int* off = hist + kWarps * E;   // [E + 1] padded run offsets
  int* cnt = off + (E + 1);       // [E] pairs per expert
  int* toff = cnt + E;            // [E + 1] tile offsets
  __shared__ int warp_sums[kWarps];
  __shared__ int bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) bad = 0;
  for (int i = tid; i < kWarps * E; i += kThreads) hist[i] = 0;
  __syncthreads();

  const int chunk = (((mk + kWarps - 1) / kWarps) + 31) & ~31;
  const int begin = warp * chunk;
  const int end = min(mk, begin + chunk);
  // pass 1: counts per (segment, expert)
  for (int base = begin; base < end; base += 32) {
    const int i = base + lane;
    const bool valid = i < end;
    const int e = valid ? ids[i] : -1;
    const bool ok = valid && e >= 0 && e < E;
    if (valid && !ok && !(allow_dropped && e < 0)) bad = 1;
    const unsigned m = __match_any_sync(0xffffffffu, ok ? e : -1);
    if (ok && lane == __ffs(m) - 1) hist[warp * E + e] += __popc(m);
  }
  __syncthreads();
  if (bad) {
    if (tid == 0) {
      *o.n_pad = -1;
      if (o.n_tiles) *o.n_tiles = 0;
    }
    return;
  }
  // per-expert totals; segment counts -> offsets inside the expert's run
  int padded = 0, ntile = 0;
  for (int e = tid; e < E; e += kThreads) {  // E <= kThreads: at most one expert per thread
    int run = 0;
    for (int s = 0; s < kWarps; ++s) {
      const int c = hist[s * E + e];
      hist[s * E + e] = run;
      run += c;
    }
    cnt[e] = run;
    padded = (run + block - 1) / block * block;
    ntile = o.tiles ? (padded + o.tile_rows - 1) / o.tile_rows : 0;
  }
  int total = 0, ttotal = 0;
  const int ex = block_exclusive_scan(padded, warp_sums, &total);
  const int tx = block_exclusive_scan(ntile, warp_sums, &ttotal);
  if (tid < E) {
    off[tid] = ex;
    toff[tid] = tx;
  }
  if (tid == 0) {
    off[E] = total;
    toff[E] = ttotal;
  }
  __syncthreads();
  // pass 2: stable placement
  for (int base = begin; base < end; base += 32) {
    const int i = base + lane;
    const bool valid = i < end;
    const int e = valid ? ids[i] : -1;
    const bool ok = valid && e >= 0 && e < E;
    const unsigned m = __match_any_sync(0xffffffffu, ok ? e : -1);
    int pos = -1;
    if (ok) {
      const unsigned lt = (1u << lane) - 1u;
      pos = off[e] + hist[warp * E + e] + __popc(m & lt);
      o.sorted_ids[pos] = i;
    }
    if (valid && o.pos_of_pair) o.pos_of_pair[i] = pos;
    __syncwarp();
    if (ok && lane == __ffs(m) - 1) hist[warp * E + e] += __popc(m);
    __syncwarp();
  }
  // sentinel padding, expert of each block, tiles
  for (int e = tid; e < E; e += kThreads) {
    const int o0 = off[e], p = off[e + 1] - o0, c = cnt[e];
    for (int r = c; r < p; ++r) o.sorted_ids[o0 + r] = mk;
    if (o.expert_ids)
      for (int b = o0 / block; b < (o0 + p) / block; ++b) o.expert_ids[b] = e;
    if (o.tiles) {
      const int nt = (p + o.tile_rows - 1) / o.tile_rows;
      for (int t = 0; t < nt; ++t) {
        const int row0 = o0 + t * o.tile_rows;
        const int rows = min(o.tile_rows, p - t * o.tile_rows);
        o.tiles[toff[e] + t] = make_int4(e, row0, rows, 0);
        if (o.blk_tile)
          for (int b = row0 / block; b < (row0 + rows) / block; ++b) o.blk_tile[b] = toff[e] + t;
      }
    }
  }
  if (tid == 0) {
    *o.n_pad = off[E];
    if (o.n_tiles) *o.n_tiles = toff[E];
  }
}

}  // namespace

int launch(const int32_t* ids, int64_t mk, int E, int block, int allow_dropped, const Out& o, cudaStream_t st) {
  DS_REQUIRE(E >= 1 && E <= kMaxExperts, DS_ENOTSUP, "moe_align: n_experts must be in [1, %d]", kMaxExperts);
  DS_REQUIRE(block >= 1, DS_EINVAL, "moe_align: block_size must be >= 1");
  DS_REQUIRE(mk >= 0 && capacity(mk, E, block) < (int64_t)1 << 31, DS_EINVAL, "moe_align: too many pairs");
  DS_REQUIRE(o.tiles == nullptr || (o.tile_rows > 0 && o.tile_rows % block == 0), DS_EINVAL,
             "moe_align: tile_rows must be a positive multiple of block");
  const size_t smem = ((size_t)kWarps * E + 3 * (size_t)E + 2) * sizeof(int);
  DS_CHECK_CUDA(cudaFuncSetAttribute(align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  align_kernel<<<1, kThreads, smem, st>>>(ids, (int)mk, E, block, allow_dropped, o);
  DS_CHECK_LAUNCH("align_kernel");
  return DS_OK;
}

}  // namespace align
}  // namespace ds

extern "C" int ds_moe_align_capacity(int64_t m, int k, int n_experts, int block, int64_t* sorted_cap,
                                     int64_t* blocks_cap) {
  DS_REQUIRE(m >= 0 && k >= 0, DS_EINVAL, "moe_align_capacity: negative shape");
  DS_REQUIRE(block >= 1 && n_experts >= 1, DS_EINVAL, "block_size and num_experts must be >= 1");
  DS_REQUIRE(sorted_cap && blocks_cap, DS_EINVAL, "moe_align_capacity: null output");
  const int64_t cap = ds::align::capacity(m * k, n_experts, block);
  *sorted_cap = cap;
  *blocks_cap = cap / block;
  return DS_OK;
}

extern "C" int ds_moe_align(const int32_t* topk_ids, int64_t m, int k, int n_experts, int block, int32_t* sorted_ids,
                            int64_t sorted_cap, int32_t* expert_ids, int64_t blocks_cap, int32_t* n_pad,
                            void* stream) {
  DS_REQUIRE(m >= 0 && k >= 0, DS_EINVAL, "moe_align: negative shape");
  DS_REQUIRE(block >= 1 && n_experts >= 1, DS_EINVAL, "block_size and num_experts must be >= 1");
  DS_REQUIRE(n_pad != nullptr && (m * k == 0 || (topk_ids && sorted_ids && expert_ids)), DS_EINVAL,
             "moe_align: null pointer");
  const int64_t cap = ds::align::capacity(m * k, n_experts, block);
  DS_REQUIRE(sorted_cap >= cap && blocks_cap >= cap / block, DS_EINVAL,
             "moe_align: outputs hold %lld / %lld entries, need %lld / %lld", (long long)sorted_cap,
             (long long)blocks_cap, (long long)cap, (long long)(cap / block));
  ds::align::Out o = {};
  o.sorted_ids = sorted_ids;
  o.expert_ids = expert_ids;
  o.n_pad = n_pad;
  return ds::align::launch(topk_ids, m * k, n_experts, block, 0, o, static_cast<cudaStream_t>(stream));
}
