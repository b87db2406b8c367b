// Batched grouped expert FFN, FP4 throughput mode: FP4 banks (with their
// tensor-core scale atoms) times activations quantised to FP4 as well, on
// tcgen05 kind::mxf4 block-scaled MMAs (A = packed e2m1 weights, B = packed
// e2m1 activations, ue8m0 scales per 32, f32 accumulate, K = 64 per MMA).
//
// The parity mode of the grouped path (grouped.cu) carries x as two e4m3
// pieces and h as three, which multiplies the MMA work; this mode rounds x
// and h to a single e2m1 value per element with a per-32 scale that maps the
// block maximum into (3, 6], so every weight byte meets one MMA.  Its results
// differ from the exact layer by the FP4 rounding of x and h (rel-L2 of
// order 0.1), and match an emulation that rounds x and h the same way at the
// f32 level.  Same layer contract otherwise (moe_layer's expert loop,
// src/deepseeker/mlx_forward.py:388-419 with route_before_down; grouped.py:
// 34-56 without).
//
// Launch sequence (one stream): align (tiles of <= 96 rows) -> xquant (each
// padded row's x as packed e2m1 + scale atoms) -> gate/up GEMM (epilogue:
// SwiGLU, route weight, h as packed e2m1 + scale atoms) -> down GEMM (f32
// rows) -> combine (grouped.cuh).  GEMM roles per CTA (persistent, one CTA
// per SM, 576 threads): warp 0 TMA producer (one 128-byte K chunk = 256
// codes per stage: weight tiles of 128 rows, the tile's activation rows,
// six or four scale atoms), warp 1 MMA issuer (an elected lane of a
// warp-uniform loop), warps 2-5 stage the scale atoms into tensor memory,
// warps 6-17 drain the double-buffered accumulators (three warps per lane
// quarter, every third 16-column group).  Every wait is bounded.
#include <algorithm>

#include "align.cuh"
#include "grouped.cuh"
#include "tc5.cuh"

namespace ds {
namespace grouped {
namespace {

using namespace ds::ptx;

// Token rows per tile (MMA N <= 96): the widest tile whose two accumulator
// buffers (gate and up: 2 x 96 columns each) and the scale ring (4 stages x 6
// atoms x 4 columns) fit in the 512 tensor-memory columns of an SM.
constexpr int kFR = 96;
constexpr int kFEpiPerQ = 3;         // epilogue warps per tensor-memory lane quarter
constexpr int kFEpiWarps = 4 * kFEpiPerQ;
constexpr int kFEpi0 = 6;            // warps 6..17: epilogue
constexpr int kFThreads = 32 * (kFEpi0 + kFEpiWarps);
constexpr int kChunkBytes = 16384;   // one weight tile chunk: 128 rows x 128 B (256 codes)

template <int MODE>
struct FC;
// gate/up: A = W1 and W3 tiles, B = x (kFR rows), atoms: W1 x2, W3 x2, x x2.
template <>
struct FC<GATEUP> {
  static constexpr int kMats = 2, kStages = 4, kAtoms = 6;
  static constexpr int kA = kMats * kChunkBytes;            // 32 KB
  static constexpr int kB = kFR * 128;                      // 12 KB
  static constexpr int kStage = kA + kB;
  static constexpr int kAcc = kMats * kFR;                  // tensor-memory columns per accumulator buffer
  static constexpr int kTmemCols = 512;
};
// down: A = W2 tile, B = h (kFR rows), atoms: W2 x2, h x2.
template <>
struct FC<DOWN> {
  static constexpr int kMats = 1, kStages = 6, kAtoms = 4;
  static constexpr int kA = kChunkBytes;
  static constexpr int kB = kFR * 128;
  static constexpr int kStage = kA + kB;
  static constexpr int kAcc = kFR;
  static constexpr int kTmemCols = 512;
};
static_assert(2 * FC<GATEUP>::kAcc + FC<GATEUP>::kStages * FC<GATEUP>::kAtoms * 4 <= FC<GATEUP>::kTmemCols,
              "gate/up tensor memory");
static_assert(2 * FC<DOWN>::kAcc + FC<DOWN>::kStages * FC<DOWN>::kAtoms * 4 <= FC<DOWN>::kTmemCols,
              "down tensor memory");
static_assert(kFR % 16 == 0 && kFR <= 128, "tile rows: a multiple of 16 within one scale atom");
static_assert(FC<GATEUP>::kStage % 1024 == 0 && FC<DOWN>::kStage % 1024 == 0 && FC<GATEUP>::kA % 1024 == 0,
              "128-byte swizzled tiles start on 1024-byte boundaries");

template <int MODE>
constexpr size_t f_smem() {
  return 1024 + (size_t)FC<MODE>::kStages * (FC<MODE>::kStage + FC<MODE>::kAtoms * kSfAtom);
}
static_assert(f_smem<GATEUP>() <= 225 * 1024 && f_smem<DOWN>() <= 225 * 1024, "dynamic shared memory");

struct FParams {
  CUtensorMap a0, a1, b;      // packed FP4 weights (gate/up: W1, W3; down: W2), packed activations
  const uint8_t* sfa0;        // weight scale atoms [E][rows/128][K/128][512] (W1 or W2)
  const uint8_t* sfa1;        // W3 (gate/up)
  const uint8_t* sfb;         // activation scale atoms [tiles][K/128][512]
  const int4* tiles;
  const int32_t* n_tiles;
  const int32_t* sorted_ids;
  const float* topk_w;
  uint8_t* hq;                // gate/up output: h packed [cap][I/2]
  uint8_t* sfh;               // gate/up output: h scale atoms [tiles][I/128][512]
  float* y;                   // down output [cap][H] f32
  int* err;
  int H, I, mk;
  float limit;
  int gate_in_h;
};

// x (bf16) -> packed e2m1 with per-32 scales; B row = the padded row's place
// in its tile.  One warp per row, one lane per 32-element block.
__global__ void __launch_bounds__(256) fp4x_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const int32_t* __restrict__ sorted_ids,
                                                         const int32_t* __restrict__ n_pad,
                                                         const int32_t* __restrict__ blk_tile,
                                                         const int4* __restrict__ tiles, int mk, int k, int H,
                                                         uint8_t* __restrict__ xq, uint8_t* __restrict__ sfx) {
  const int lane = threadIdx.x & 31;
  const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int np = *n_pad;
  const int KC = H / 128;
  for (int row = w0; row < np; row += nw) {
    const int pr = sorted_ids[row];
    const int tile = blk_tile[row / kBlock];
    const int r = row - tiles[tile].y;
    for (int blk = lane; blk < H / 32; blk += 32) {
      float v[32];
      if (pr < mk) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(pr / k) * H + blk * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 u = src[c];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            v[c * 8 + 2 * d] = __uint_as_float(w[d] << 16);
            v[c * 8 + 2 * d + 1] = __uint_as_float(w[d] & 0xFFFF0000u);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.0f;
      }
      float a = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) a = fmaxf(a, fabsf(v[j]));
      const int sc = tc5::e2m1_block_scale(a);
      const float inv = inv_scale_of(sc);
      uint32_t words[4];
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b)
          word |= tc5::f32x2_to_e2m1x2(v[wd * 8 + 2 * b] * inv, v[wd * 8 + 2 * b + 1] * inv) << (8 * b);
        words[wd] = word;
      }
      *reinterpret_cast<uint4*>(xq + (size_t)row * (H / 2) + blk * 16) =
          make_uint4(words[0], words[1], words[2], words[3]);
      sfx[((size_t)tile * KC + blk / 4) * kSfAtom + atom_off(r, blk & 3)] = (uint8_t)sc;
    }
  }
}

// Epilogue of one item (tile x 128 weight rows), thread = one weight row
// (lane quarter q, lane); the kFEpiPerQ warps of a quarter take every
// kFEpiPerQ-th group of 16 token columns (part = 0 .. kFEpiPerQ - 1).  gate/up: the 32 lanes are 32 consecutive
// intermediate rows = one 32-block of the down projection's K, so h of each
// token is quantised to e2m1 across the warp (block maximum by one warp
// max-reduction of |h|'s bits: non-negative floats order as their bits; a
// NaN counts as 0, as a maximum tree of fmaxf would skip it).
// Route weights of an epilogue warp's token columns (route weight inside h),
// loaded before the accumulator wait: column (part + kFEpiPerQ gi) * 16 + c
// of the warp's group gi (0 or 1) is lane gi * 16 + c of the result.
static_assert(kFR <= 2 * 16 * kFEpiPerQ, "at most two 16-column groups per epilogue warp");
__device__ __forceinline__ float f_route_weights(const FParams& p, int N, int row0, int part, int lane) {
  if (!p.gate_in_h) return 1.0f;
  const int c = (part + kFEpiPerQ * (lane >> 4)) * 16 + (lane & 15);
  if (c >= N) return 1.0f;
  const int pr = p.sorted_ids[row0 + c];
  return pr < p.mk ? p.topk_w[pr] : 0.0f;
}

template <int MODE>
__device__ __forceinline__ void f_epilogue(const FParams& p, uint32_t dacc, int N, int row0, int tile, int mt, int q,
                                           int lane, int part, float wa) {
  if (MODE == GATEUP) {
    const int I = p.I;
    const int i = mt * 128 + q * 32 + lane;
    uint8_t* sf = p.sfh + ((size_t)tile * (I / 128) + mt) * kSfAtom;
    for (int n0 = 16 * part, gi = 0; n0 < N; n0 += 16 * kFEpiPerQ, ++gi) {
      float gv[16], uv[16];
      tc5::ld_x16_nowait(dacc + n0, gv);
      tc5::ld_x16_nowait(dacc + kFR + n0, uv);
      tc5::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float h = silu_glu(gv[j], uv[j], p.limit);
        if (p.gate_in_h) h *= __shfl_sync(0xffffffffu, wa, gi * 16 + j);
        const float ah = fabsf(h);
        const float am = __uint_as_float(__reduce_max_sync(0xffffffffu, ah == ah ? __float_as_uint(ah) : 0u));
        const int sc = tc5::e2m1_block_scale(am);
        const uint32_t code = tc5::f32x2_to_e2m1x2(h * inv_scale_of(sc), 0.0f) & 0xFu;
        const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
        if ((lane & 1) == 0) p.hq[(size_t)(row0 + n0 + j) * (I / 2) + i / 2] = (uint8_t)(code | (hi << 4));
        if (lane == 0) sf[atom_off(n0 + j, q)] = (uint8_t)sc;
      }
    }
  } else {
    const int hrow = mt * 128 + q * 32 + lane;
    for (int n0 = 16 * part; n0 < N; n0 += 16 * kFEpiPerQ) {
      float v[16];
      tc5::ld_x16_nowait(dacc + n0, v);
      tc5::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) p.y[(size_t)(row0 + n0 + j) * p.H + hrow] = v[j];
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kFThreads, 1) fp4_gemm_kernel(const __grid_constant__ FParams p) {
  using C = FC<MODE>;
  constexpr int S = C::kStages, NA = C::kAtoms;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ops = smem;                        // S x [A chunk(s)][B chunk], 128-byte swizzled
  uint8_t* sfs = smem + S * C::kStage;        // S x NA scale atoms
  __shared__ __align__(8) uint64_t full[S], sfready[S], empty[S], accfull[2], accempty[2], done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_out = MODE == GATEUP ? p.I : p.H;
  const int K = MODE == GATEUP ? p.H : p.I;
  const int MT = rows_out / 128, KC = K / 256, KC128 = K / 128;
  const int n_items = *p.n_tiles * MT;
  if ((int)blockIdx.x >= n_items) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&sfready[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], kFEpiWarps);
    }
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc5::alloc(&tmem_base, C::kTmemCols);
  __syncthreads();
  tc5::fence_after();
  const uint32_t tb = tmem_base;
  const uint32_t tsf0 = tb + 2 * C::kAcc;     // scale atoms: NA x 4 columns per stage
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t wpol = policy_evict_first();
      int g = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int tile = item / MT, mt = item % MT;
        const int4 td = p.tiles[tile];
        const int e = td.x, row0 = td.y;
        const size_t atom_a = ((size_t)e * MT + mt) * KC128;
        for (int kc = 0; kc < KC; ++kc, ++g) {
          const int s = g % S;
          if (g >= S && !wait_or_abort(&empty[s], ((g / S) - 1) & 1, abort, p.err)) goto drain;
          uint8_t* st = ops + s * C::kStage;
          uint8_t* sf = sfs + s * NA * kSfAtom;
          mbar_arrive_expect_tx(&full[s], C::kStage + NA * kSfAtom);
          tma_load_3d_hint(st, &p.a0, 0, e * rows_out + mt * 128, kc, &full[s], wpol);
          bulk_g2s(sf, p.sfa0 + (atom_a + 2 * kc) * kSfAtom, 2 * kSfAtom, &full[s]);
          if (MODE == GATEUP) {
            tma_load_3d_hint(st + kChunkBytes, &p.a1, 0, e * rows_out + mt * 128, kc, &full[s], wpol);
            bulk_g2s(sf + 2 * kSfAtom, p.sfa1 + (atom_a + 2 * kc) * kSfAtom, 2 * kSfAtom, &full[s]);
          }
          tma_load_3d(st + C::kA, &p.b, 0, row0, kc, &full[s]);
          bulk_g2s(sf + (NA - 2) * kSfAtom, p.sfb + ((size_t)tile * KC128 + 2 * kc) * kSfAtom, 2 * kSfAtom,
                   &full[s]);
        }
      }
    drain:
      // never leave with copies in flight into this CTA's shared memory
      for (int j = g - S < 0 ? 0 : g - S; j < g; ++j) mbar_wait_bounded(&full[j % S], (j / S) & 1, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Warp-uniform loop, one elected lane issues.  A stage is one 128-byte K
    // chunk (256 codes) = four K = 64 steps; step kk uses scale atom kk / 2
    // of the stage and the byte pair kk % 2 of its words (scale_vec::2X).
    // A K step of 32 B adds 2 to a descriptor's 16-byte address field.
    {
      int g = 0, li = 0;
      const uint64_t ops_desc = tc5::sdesc_sw128(smem_u32(ops));
      for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
        const int N = p.tiles[item / MT].z;
        const uint32_t idesc[2] = {tc5::idesc_mxf4(N, 0), tc5::idesc_mxf4(N, 2)};
        const int b = li & 1;
        if (li >= 2 && !warp_wait(&accempty[b], ((li >> 1) - 1) & 1, abort, p.err)) break;
        tc5::fence_after();
        const uint32_t dacc = tb + b * C::kAcc;
        for (int kc = 0; kc < KC; ++kc, ++g) {
          const int s = g % S;
          // the stagers arrive on sfready after the stage's copies landed
          if (!warp_wait(&sfready[s], (g / S) & 1, abort, p.err)) goto mma_out;
          tc5::fence_after();
          if (elect_one()) {
            const uint64_t ad = ops_desc + (uint64_t)((s * C::kStage) >> 4);
            const uint64_t bd = ad + (uint64_t)(C::kA >> 4);
            const uint32_t tsf = tsf0 + s * NA * 4;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t sfb = tsf + 4 * (NA - 2 + (kk >> 1));
              const uint32_t acc = (kc | kk) != 0;
              tc5::mma_mxf4(dacc, ad + 2 * kk, bd + 2 * kk, idesc[kk & 1], tsf + 4 * (kk >> 1), sfb, acc);
              if (MODE == GATEUP)
                tc5::mma_mxf4(dacc + kFR, ad + (kChunkBytes >> 4) + 2 * kk, bd + 2 * kk, idesc[kk & 1],
                              tsf + 4 * (2 + (kk >> 1)), sfb, acc);
            }
            tc5::commit(&empty[s]);
          }
          __syncwarp();
        }
        if (elect_one()) tc5::commit(&accfull[b]);
        __syncwarp();
      }
    mma_out:
      // all issued MMAs complete before the tensor memory is released
      if (elect_one()) {
        tc5::commit(&done);
        mbar_wait_bounded(&done, 0, 1000000000ull);
      }
      __syncwarp();
    }
  } else if (warp < kFEpi0) {
    // ------------------------------------------------------------ scale staging
    const int q = warp & 3;
    int g = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      for (int kc = 0; kc < KC; ++kc, ++g) {
        const int s = g % S;
        if (!warp_wait(&full[s], (g / S) & 1, abort, p.err)) goto sf_out;
        const uint4* src = reinterpret_cast<const uint4*>(sfs + s * NA * kSfAtom);
        const uint32_t t = tc5::lane_quarter(tsf0 + s * NA * 4, q);
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          const uint4 v = src[a * 32 + lane];
          tc5::st_x4(t + 4 * a, v.x, v.y, v.z, v.w);
        }
        tc5::wait_st();
        tc5::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfready[s]);
      }
    }
  sf_out:;
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3, part = (warp - kFEpi0) >> 2;
    int li = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
      const int tile = item / MT, mt = item % MT;
      const int4 td = p.tiles[tile];
      const int b = li & 1;
      const float wa = MODE == GATEUP ? f_route_weights(p, td.z, td.y, part, lane) : 1.0f;
      if (!warp_wait(&accfull[b], (li >> 1) & 1, abort, p.err)) break;
      tc5::fence_after();
      f_epilogue<MODE>(p, tc5::lane_quarter(tb + b * C::kAcc, q), td.z, td.y, tile, mt, q, lane, part, wa);
      tc5::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[b]);
    }
  }
  tc5::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc5::fence_after();
    tc5::dealloc(tb, C::kTmemCols);
  }
}

}  // namespace

// ---------------------------------------------------------------- host side

namespace {

// Packed FP4 rows [rows][K/2 B] viewed as {128 B, rows, K/256 chunks}; a box
// is one chunk of box_rows rows, 128-byte swizzle.
bool map_packed(CUtensorMap* m, const void* base, uint64_t rows, uint64_t K, uint32_t box_rows) {
  const cuuint64_t dims[3] = {128, rows, K / 256};
  const cuuint64_t strides[2] = {K / 2, 128};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct FLayout {
  int64_t mk, cap, max_tiles;
  size_t ints, sorted, pos, blk, tiles, xq, sfx, hq, sfh, y, total;
};

FLayout f_layout(const DsMoeDesc* d, int64_t T) {
  FLayout L;
  L.mk = T * d->top_k;
  L.cap = align::capacity(L.mk, d->n_experts, kBlock);
  L.max_tiles = align::max_tiles(L.mk, d->n_experts, kBlock, kFR);
  const size_t H = d->hidden, I = d->inter, NT = L.max_tiles;
  size_t o = 0;
  L.ints = o;   o += up(256);
  L.sorted = o; o += up(L.cap * 4);
  L.pos = o;    o += up(L.mk * 4);
  L.blk = o;    o += up(L.cap / kBlock * 4);
  L.tiles = o;  o += up(NT * 16);
  L.xq = o;     o += up(L.cap * H / 2);
  L.sfx = o;    o += up(NT * (H / 128) * kSfAtom);
  L.hq = o;     o += up(L.cap * I / 2);
  L.sfh = o;    o += up(NT * (I / 128) * kSfAtom);
  L.y = o;      o += up(L.cap * H * 4);
  L.total = o;
  return L;
}

int f_validate(const DsMoeDesc* d, int64_t T) {
  DS_REQUIRE(d != nullptr, DS_EINVAL, "grouped_ffn_fp4: null descriptor");
  DS_REQUIRE(T >= 1 && d->top_k >= 1 && T * d->top_k < ((int64_t)1 << 30), DS_EINVAL,
             "grouped_ffn_fp4: tokens and top_k must be >= 1");
  DS_REQUIRE(d->w1.format == DS_FMT_FP4 && d->w3.format == DS_FMT_FP4 && d->w2.format == DS_FMT_FP4, DS_ENOTSUP,
             "grouped_ffn_fp4: expert banks must be FP4");
  DS_REQUIRE(d->w1.scales_tc && d->w3.scales_tc && d->w2.scales_tc, DS_EINVAL,
             "grouped_ffn_fp4: the banks need their tensor-core scale atoms (ds_fp4_scale_atoms)");
  DS_REQUIRE(d->n_experts >= 1 && d->n_experts <= align::kMaxExperts, DS_ENOTSUP,
             "grouped_ffn_fp4: n_experts must be in [1, %d]", align::kMaxExperts);
  DS_REQUIRE(d->hidden % 256 == 0 && d->inter % 256 == 0 && d->hidden > 0 && d->inter > 0, DS_EINVAL,
             "grouped_ffn_fp4: hidden and inter must be positive multiples of 256");
  const int E = d->n_experts, H = d->hidden, I = d->inter;
  DS_REQUIRE(d->w1.n_experts == E && d->w1.rows == I && d->w1.cols == H && d->w3.n_experts == E &&
                 d->w3.rows == I && d->w3.cols == H && d->w2.n_experts == E && d->w2.rows == H && d->w2.cols == I,
             DS_EINVAL, "grouped_ffn_fp4: bank shapes do not match the descriptor");
  DS_REQUIRE(ds::aligned(d->w1.data, 16) && ds::aligned(d->w3.data, 16) && ds::aligned(d->w2.data, 16) &&
                 ds::aligned(d->w1.scales_tc, 16) && ds::aligned(d->w3.scales_tc, 16) &&
                 ds::aligned(d->w2.scales_tc, 16),
             DS_EALIGN, "grouped_ffn_fp4: packed data and scale atoms 16-byte aligned");
  DS_REQUIRE(!(d->shared_w1 || d->shared_w3 || d->shared_w2), DS_ENOTSUP,
             "grouped_ffn_fp4: the shared expert is not part of the grouped call");
  DS_REQUIRE((int64_t)E * I < ((int64_t)1 << 31) && (int64_t)E * H < ((int64_t)1 << 31), DS_EINVAL,
             "grouped_ffn_fp4: bank too large");
  return DS_OK;
}

}  // namespace

}  // namespace grouped
}  // namespace ds

using namespace ds::grouped;

extern "C" int ds_grouped_ffn_fp4_workspace_size(const DsMoeDesc* desc, int64_t tokens, size_t* bytes) {
  int st = f_validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(bytes != nullptr, DS_EINVAL, "grouped_ffn_fp4_workspace_size: null output");
  *bytes = f_layout(desc, tokens).total;
  return DS_OK;
}

extern "C" int ds_grouped_ffn_fp4(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                                  const int32_t* topk_ids, const float* topk_w, void* out, int out_dtype,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  int st = f_validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(x_dtype == DS_BF16, DS_ENOTSUP, "grouped_ffn_fp4: x must be bf16");
  DS_REQUIRE(out_dtype == DS_BF16 || out_dtype == DS_F32, DS_EINVAL,
             "grouped_ffn_fp4: out_dtype must be bf16 or f32");
  DS_REQUIRE(x && topk_ids && topk_w && out && workspace, DS_EINVAL, "grouped_ffn_fp4: null pointer");
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 16) && ds::aligned(workspace, 256), DS_EALIGN,
             "grouped_ffn_fp4: x/out 16-byte and workspace 256-byte aligned");
  const FLayout L = f_layout(desc, tokens);
  DS_REQUIRE(workspace_bytes >= L.total, DS_EINVAL, "grouped_ffn_fp4: workspace %zu bytes < required %zu",
             workspace_bytes, L.total);
  DS_REQUIRE(encode_fn() != nullptr, DS_ECUDA, "grouped_ffn_fp4: cuTensorMapEncodeTiled unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  int32_t* ints = reinterpret_cast<int32_t*>(ws + L.ints);  // [0] n_pad, [1] n_tiles, [2] error bits
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + L.sorted);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + L.pos);
  int32_t* blk = reinterpret_cast<int32_t*>(ws + L.blk);
  int4* tiles = reinterpret_cast<int4*>(ws + L.tiles);
  uint8_t* xq = reinterpret_cast<uint8_t*>(ws + L.xq);
  uint8_t* sfx = reinterpret_cast<uint8_t*>(ws + L.sfx);
  uint8_t* hq = reinterpret_cast<uint8_t*>(ws + L.hq);
  uint8_t* sfh = reinterpret_cast<uint8_t*>(ws + L.sfh);
  float* y = reinterpret_cast<float*>(ws + L.y);
  const int E = desc->n_experts, H = desc->hidden, I = desc->inter, k = desc->top_k;

  DS_CHECK_CUDA(cudaMemsetAsync(ints, 0, 256, s));
  ds::align::Out ao = {};
  ao.sorted_ids = sorted;
  ao.n_pad = ints;
  ao.pos_of_pair = pos;
  ao.blk_tile = blk;
  ao.tiles = tiles;
  ao.n_tiles = ints + 1;
  ao.tile_rows = kFR;
  if ((st = ds::align::launch(topk_ids, L.mk, E, kBlock, 1, ao, s)) != DS_OK) return st;
  const int sms = ds::sm_count();
  fp4x_quant_kernel<<<sms * 4, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), sorted, ints, blk, tiles,
                                            (int)L.mk, k, H, xq, sfx);
  DS_CHECK_LAUNCH("fp4x_quant_kernel");

  FParams p;
  memset(&p, 0, sizeof(p));
  p.tiles = tiles;
  p.n_tiles = ints + 1;
  p.sorted_ids = sorted;
  p.topk_w = topk_w;
  p.hq = hq;
  p.sfh = sfh;
  p.y = y;
  p.err = ints + 2;
  p.H = H;
  p.I = I;
  p.mk = (int)L.mk;
  p.limit = desc->swiglu_limit;
  p.gate_in_h = desc->route_before_down ? 1 : 0;
  bool ok = map_packed(&p.a0, desc->w1.data, (uint64_t)E * I, H, 128) &&
            map_packed(&p.a1, desc->w3.data, (uint64_t)E * I, H, 128) &&
            map_packed(&p.b, xq, (uint64_t)L.cap, H, kFR);
  DS_REQUIRE(ok, DS_ECUDA, "grouped_ffn_fp4: tensor map encoding failed (gate/up)");
  p.sfa0 = static_cast<const uint8_t*>(desc->w1.scales_tc);
  p.sfa1 = static_cast<const uint8_t*>(desc->w3.scales_tc);
  p.sfb = sfx;
  const int grid_a = (int)std::min<int64_t>(sms, L.max_tiles * (I / 128));
  const int grid_b = (int)std::min<int64_t>(sms, L.max_tiles * (H / 128));
  DS_CHECK_CUDA(cudaFuncSetAttribute(fp4_gemm_kernel<GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)f_smem<GATEUP>()));
  fp4_gemm_kernel<GATEUP><<<grid_a, kFThreads, f_smem<GATEUP>(), s>>>(p);
  DS_CHECK_LAUNCH("fp4_gemm_kernel<gate/up>");

  ok = map_packed(&p.a0, desc->w2.data, (uint64_t)E * H, I, 128) && map_packed(&p.b, hq, (uint64_t)L.cap, I, kFR);
  DS_REQUIRE(ok, DS_ECUDA, "grouped_ffn_fp4: tensor map encoding failed (down)");
  p.a1 = p.a0;
  p.sfa0 = static_cast<const uint8_t*>(desc->w2.scales_tc);
  p.sfa1 = nullptr;
  p.sfb = sfh;
  DS_CHECK_CUDA(cudaFuncSetAttribute(fp4_gemm_kernel<DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)f_smem<DOWN>()));
  fp4_gemm_kernel<DOWN><<<grid_b, kFThreads, f_smem<DOWN>(), s>>>(p);
  DS_CHECK_LAUNCH("fp4_gemm_kernel<down>");

  return launch_combine(y, pos, topk_w, ints, ints + 2, k, H, desc->route_before_down ? 0 : 1, out, out_dtype,
                        tokens, s);
}

namespace ds {
namespace grouped {

}  // namespace grouped
}  // namespace ds
