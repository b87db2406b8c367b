// Batched grouped expert FFN (prefill, MTP verification): tokens routed to FP4
// experts are sorted into per-expert runs and pushed through tcgen05
// block-scaled MMAs (kind::mxf8f6f4, A = e2m1 weights, B = e4m3 activations,
// ue8m0 scales per 32 elements, f32 accumulate in tensor memory).
//
// Replaces the per-expert loop of grouped_swiglu / moe_layer
//   (src/deepseeker/grouped.py:34-56, src/deepseeker/mlx_forward.py:388-419)
// for FP4 expert banks.  Launch sequence on one stream, no host sync:
//   1. align   : stable sort of (token, slot) pairs by expert, runs padded to
//                16 rows, cut into tiles of <= 64 rows (moe_align.cu);
//   2. xquant  : every padded row gets its token's x as two e4m3 pieces
//                (hi + lo, each with its own per-32 ue8m0 scale): a bf16
//                value has 8 significant bits, each piece carries 4, so
//                hi + lo reproduces x (exactly, unless an element is below
//                2^-13 of its block maximum);
//   3. gate/up : D_gate = W1 X^T and D_up = W3 X^T per (tile, 128 rows of I);
//                epilogue h = silu(min(g, L)) * clip(u, +-L) [* route weight],
//                written as three e4m3 pieces (about 14 significant bits
//                relative to the block maximum) with per-32 ue8m0 scales;
//   4. down    : Y = W2 H^T per (tile, 128 rows of the hidden size), f32 rows;
//   5. combine : out[t] = sum over t's slots (in top-k order) of
//                [route weight *] Y[row of the pair], cast to x's dtype.
//
// GEMM kernels (one template, two modes) are persistent, one CTA per SM,
// warp-specialised: warp 0 issues TMA loads into a stage ring, warp 1 issues
// the MMAs (one thread) and owns the tensor memory, warps 2-5 copy the stage's
// scale atoms from shared memory into tensor memory (tcgen05.st, one warp per
// lane quarter), warps 6-17 drain the double-buffered accumulators (three
// warps per lane quarter, every third group of 16 token columns).
// Every wait is bounded; a timeout sets an error bit and an abort flag that
// makes every other role leave its loop.
#include <algorithm>

#include "align.cuh"
#include "grouped.cuh"
#include "tc5.cuh"

namespace ds {
namespace grouped {
namespace {

using namespace ds::ptx;

constexpr int kTileRows = 64;   // token rows per tile (MMA N <= 64)
constexpr int kEpiPerQ = 3;    // epilogue warps per tensor-memory lane quarter
constexpr int kEpiWarps = 4 * kEpiPerQ;
constexpr int kEpiWarp0 = 6;  // warps 2..5 stage scales, 6..17 run the epilogue
constexpr int kWarps = kEpiWarp0 + kEpiWarps;
constexpr int kThreads = kWarps * 32;
constexpr int kSfStage = 4 * kSfAtom;         // scale atoms of one stage
constexpr int kHPieces = 3, kXPieces = 2;
constexpr uint32_t kTxBytes = 34816;          // per stage, both modes (see Cfg)

template <int MODE>
struct Cfg;
// gate/up: A = 128 rows of W1 and 128 rows of W3 (two accumulators), B = x hi/lo.
// per stage: A 2 x 8 KB packed (2 x 16 KB in shared memory), B 2 x 8 KB, scales 2 KB.
template <>
struct Cfg<GATEUP> {
  static constexpr int kStages = 4, kPieces = kXPieces;
  static constexpr int kAStage = 2 * 16384;
  static constexpr int kBPiece = kTileRows * 128;
  static constexpr int kStage = kAStage + kPieces * kBPiece;
  static constexpr int kAcc = 2 * kTileRows;  // tensor-memory columns per accumulator buffer
  static constexpr int kTmemCols = 512;
};
// down: A = 128 rows of W2, B = h in three pieces.
// per stage: A 8 KB packed (16 KB in shared memory), B 3 x 8 KB, scales 2 KB.
template <>
struct Cfg<DOWN> {
  static constexpr int kStages = 5, kPieces = kHPieces;
  static constexpr int kAStage = 16384;
  static constexpr int kBPiece = kTileRows * 128;
  static constexpr int kStage = kAStage + kPieces * kBPiece;
  static constexpr int kAcc = kTileRows;
  static constexpr int kTmemCols = 256;
};

template <int MODE>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)Cfg<MODE>::kStages * (Cfg<MODE>::kStage + kSfStage);
}

struct Params {
  CUtensorMap a0, a1, b;      // weights (gate/up: W1, W3; down: W2 in a0), activation pieces
  const uint8_t* sfa;         // prepared weight scales
  const uint8_t* sfb;         // activation piece scales, per tile
  const int4* tiles;          // {expert, first row, rows, 0}
  const int32_t* n_tiles;
  const int32_t* sorted_ids;  // padded row -> pair (sentinel = mk)
  const float* topk_w;        // [mk]
  uint8_t* hq;                // gate/up output pieces [cap][3][I]
  uint8_t* sfh;               // gate/up output scales [tiles][I/128][3][512]
  float* y;                   // down output [cap][H] f32
  int* err;
  int H, I, mk;
  float limit;
  int gate_in_h;              // route weight applied to h (before the down projection)
};

// Route weights of an epilogue warp's token columns (route weight inside h),
// loaded before the accumulator wait: column (part + kEpiPerQ gi) * 16 + c of
// the warp's column group gi (0 or 1) is lane gi * 16 + c of the result.
static_assert(kTileRows <= 2 * 16 * kEpiPerQ, "at most two 16-column groups per epilogue warp");
__device__ __forceinline__ float route_weights(const Params& p, int N, int row0, int part, int lane) {
  if (!p.gate_in_h) return 1.0f;
  const int c = (part + kEpiPerQ * (lane >> 4)) * 16 + (lane & 15);
  if (c >= N) return 1.0f;
  const int pr = p.sorted_ids[row0 + c];
  return pr < p.mk ? p.topk_w[pr] : 0.0f;
}

// Epilogue of one item, thread = one weight row (lane quarter q, lane); the
// kEpiPerQ warps of a quarter take every kEpiPerQ-th group of 16 token
// columns (part).  gate/up: the block maximum of |h| over the warp's 32
// consecutive intermediate rows by one warp max-reduction of its bits
// (non-negative floats order as their bits; a NaN counts as 0, as a maximum
// tree of fmaxf would skip it).
template <int MODE>
__device__ __forceinline__ void epilogue(const Params& p, uint32_t dacc, int N, int row0, int tile, int mt, int q,
                                         int lane, int part, float wa) {
  if (MODE == GATEUP) {
    const int KC2 = p.I / 128;
    const int i = mt * 128 + q * 32 + lane;  // intermediate index held by this lane
    for (int n0 = 16 * part, gi = 0; n0 < N; n0 += 16 * kEpiPerQ, ++gi) {
      float gv[16], uv[16];
      tc5::ld_x16_nowait(dacc + n0, gv);
      tc5::ld_x16_nowait(dacc + kTileRows + n0, uv);
      tc5::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        float h[2];
        int ef[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          h[c] = silu_glu(gv[j + c], uv[j + c], p.limit);
          if (p.gate_in_h) h[c] *= __shfl_sync(0xffffffffu, wa, gi * 16 + j + c);
          const float a = fabsf(h[c]);
          ef[c] = (int)(__reduce_max_sync(0xffffffffu, a == a ? __float_as_uint(a) : 0u) >> 23);
        }
        const int n = n0 + j;
        uint8_t* dst0 = p.hq + (size_t)(row0 + n) * kHPieces * p.I + i;
        uint8_t* dst1 = dst0 + (size_t)kHPieces * p.I;
        float r0 = h[0], r1 = h[1];
#pragma unroll
        for (int pc = 0; pc < kHPieces; ++pc) {
          const int s0 = piece_scale(ef[0], pc), s1 = piece_scale(ef[1], pc);
          const uint32_t bb = tc5::f32x2_to_e4m3x2(r0 * inv_scale_of(s0), r1 * inv_scale_of(s1));
          float v0, v1;
          tc5::e4m3x2_to_f32x2(bb, v0, v1);
          r0 = fmaf(-v0, scale_of(s0), r0);
          r1 = fmaf(-v1, scale_of(s1), r1);
          dst0[pc * p.I] = (uint8_t)(bb & 0xFFu);
          dst1[pc * p.I] = (uint8_t)(bb >> 8);
          if (lane == 0) {
            uint8_t* sf = p.sfh + (((size_t)tile * KC2 + mt) * kHPieces + pc) * kSfAtom;
            sf[atom_off(n, q)] = (uint8_t)s0;
            sf[atom_off(n + 1, q)] = (uint8_t)s1;
          }
        }
      }
    }
  } else {
    const int hrow = mt * 128 + q * 32 + lane;
    for (int n0 = 16 * part; n0 < N; n0 += 16 * kEpiPerQ) {
      float v[16];
      tc5::ld_x16_nowait(dacc + n0, v);
      tc5::wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) p.y[(size_t)(row0 + n0 + j) * p.H + hrow] = v[j];
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Params p) {
  using C = Cfg<MODE>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ops = smem;
  uint8_t* sfs = smem + S * C::kStage;
  __shared__ __align__(8) uint64_t full[S], sfready[S], empty[S], accfull[2], accempty[2], done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int MT = MODE == GATEUP ? p.I / 128 : p.H / 128;
  const int KC = MODE == GATEUP ? p.H / 128 : p.I / 128;
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
      mbar_init(&accempty[b], kEpiWarps);
    }
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc5::alloc(&tmem_base, C::kTmemCols);
  __syncthreads();
  tc5::fence_after();
  const uint32_t tb = tmem_base;
  const uint32_t tsf0 = tb + 2 * C::kAcc;  // scale ring: 16 columns per stage
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int g = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int tile = item / MT, mt = item % MT;
        const int4 td = p.tiles[tile];
        const int e = td.x, row0 = td.y;
        for (int kc = 0; kc < KC; ++kc, ++g) {
          const int s = g % S;
          if (g >= S && !wait_or_abort(&empty[s], ((g / S) - 1) & 1, abort, p.err)) goto drain;
          uint8_t* sa = ops + s * C::kStage;
          uint8_t* sb = sa + C::kAStage;
          uint8_t* sf = sfs + s * kSfStage;
          mbar_arrive_expect_tx(&full[s], kTxBytes);
          if (MODE == GATEUP) {
            tma_load_3d(sa, &p.a0, 0, e * p.I + mt * 128, kc, &full[s]);
            tma_load_3d(sa + 16384, &p.a1, 0, e * p.I + mt * 128, kc, &full[s]);
            bulk_g2s(sf, p.sfa + ((size_t)(e * MT + mt) * KC + kc) * (2 * kSfAtom), 2 * kSfAtom, &full[s]);
            bulk_g2s(sf + 2 * kSfAtom, p.sfb + ((size_t)tile * KC + kc) * (kXPieces * kSfAtom),
                     kXPieces * kSfAtom, &full[s]);
          } else {
            tma_load_3d(sa, &p.a0, 0, e * p.H + mt * 128, kc, &full[s]);
            bulk_g2s(sf, p.sfa + ((size_t)(e * MT + mt) * KC + kc) * kSfAtom, kSfAtom, &full[s]);
            bulk_g2s(sf + kSfAtom, p.sfb + ((size_t)tile * KC + kc) * (kHPieces * kSfAtom), kHPieces * kSfAtom,
                     &full[s]);
          }
#pragma unroll
          for (int pc = 0; pc < C::kPieces; ++pc)
            tma_load_3d(sb + pc * C::kBPiece, &p.b, 0, row0, pc * KC + kc, &full[s]);
        }
      }
    drain:
      // never leave with copies in flight into this CTA's shared memory
      for (int j = g - S < 0 ? 0 : g - S; j < g; ++j) mbar_wait_bounded(&full[j % S], (j / S) & 1, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (warp-uniform waits and operands); one
    // elected lane issues.  Descriptors are formed once: a K step of 32
    // advances a start address by 32 B = 2 units of the descriptor's
    // address field (shared memory addresses stay below 256 KB: no carry).
    {
      int g = 0, li = 0;
      const uint64_t ops_desc = tc5::sdesc_sw128(smem_u32(ops));
      for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
        const int tile = item / MT;
        const int N = p.tiles[tile].z;
        uint32_t idesc[4];
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) idesc[sub] = tc5::idesc_e2m1_e4m3(N, sub);
        const int b = li & 1;
        if (li >= 2 && !warp_wait(&accempty[b], ((li >> 1) - 1) & 1, abort, p.err)) break;
        tc5::fence_after();
        const uint32_t dacc = tb + b * C::kAcc;
        for (int kc = 0; kc < KC; ++kc, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          // the stagers arrive on sfready after they have seen the stage's
          // copies land, so waiting for sfready covers the copies too
          if (!warp_wait(&sfready[s], ph, abort, p.err)) goto mma_out;
          tc5::fence_after();
          if (elect_one()) {
            const uint64_t ad = ops_desc + (uint64_t)((s * C::kStage) >> 4);
            const uint64_t bd = ad + (uint64_t)(C::kAStage >> 4);
            const uint32_t tsf = tsf0 + s * 16;
#pragma unroll
            for (int sub = 0; sub < 4; ++sub) {
#pragma unroll
              for (int pc = 0; pc < C::kPieces; ++pc) {
                const uint64_t bdp = bd + (uint64_t)((pc * C::kBPiece) >> 4) + 2 * sub;
                const uint32_t acc = (kc | sub | pc) != 0;
                if (MODE == GATEUP) {
                  tc5::mma_mxf8f6f4(dacc, ad + 2 * sub, bdp, idesc[sub], tsf, tsf + 8 + 4 * pc, acc);
                  tc5::mma_mxf8f6f4(dacc + kTileRows, ad + (16384 >> 4) + 2 * sub, bdp, idesc[sub], tsf + 4,
                                    tsf + 8 + 4 * pc, acc);
                } else {
                  tc5::mma_mxf8f6f4(dacc, ad + 2 * sub, bdp, idesc[sub], tsf, tsf + 4 + 4 * pc, acc);
                }
              }
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
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ scale staging
    const int q = warp & 3;
    int g = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      for (int kc = 0; kc < KC; ++kc, ++g) {
        const int s = g % S;
        if (!warp_wait(&full[s], (g / S) & 1, abort, p.err)) goto sf_out;
        const uint4* src = reinterpret_cast<const uint4*>(sfs + s * kSfStage);
        const uint32_t t = tc5::lane_quarter(tsf0 + s * 16, q);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
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
    const int q = warp & 3, part = (warp - kEpiWarp0) >> 2;
    int li = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
      const int tile = item / MT, mt = item % MT;
      const int4 td = p.tiles[tile];
      const int b = li & 1;
      const float wa = MODE == GATEUP ? route_weights(p, td.z, td.y, part, lane) : 1.0f;
      if (!warp_wait(&accfull[b], (li >> 1) & 1, abort, p.err)) break;
      tc5::fence_after();
      epilogue<MODE>(p, tc5::lane_quarter(tb + b * C::kAcc, q), td.z, td.y, tile, mt, q, lane, part, wa);
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

// Every padded row gets its token's x (bf16) as hi/lo e4m3 pieces; sentinel
// rows are zero.  One warp per row, one lane per 32-element block.
__global__ void __launch_bounds__(256) xquant_kernel(const __nv_bfloat16* __restrict__ x,
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
    uint8_t* dst = xq + (size_t)row * kXPieces * H;
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
      const int ef = (int)(__float_as_uint(a) >> 23);
      const int s0 = piece_scale(ef, 0), s1 = piece_scale(ef, 1);
      uint32_t hi[8], lo[8];
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        uint32_t bh = 0, bl = 0;
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          const uint32_t b0 = tc5::f32x2_to_e4m3x2(v[j + c] * inv_scale_of(s0), v[j + c + 1] * inv_scale_of(s0));
          float q0, q1;
          tc5::e4m3x2_to_f32x2(b0, q0, q1);
          const float r0 = fmaf(-q0, scale_of(s0), v[j + c]), r1 = fmaf(-q1, scale_of(s0), v[j + c + 1]);
          const uint32_t b1 = tc5::f32x2_to_e4m3x2(r0 * inv_scale_of(s1), r1 * inv_scale_of(s1));
          bh |= b0 << (8 * c);
          bl |= b1 << (8 * c);
        }
        hi[j / 4] = bh;
        lo[j / 4] = bl;
      }
      uint4* dh = reinterpret_cast<uint4*>(dst + blk * 32);
      uint4* dl = reinterpret_cast<uint4*>(dst + H + blk * 32);
      dh[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      dh[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
      dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
      uint8_t* sf = sfx + ((size_t)tile * KC + blk / 4) * kXPieces * kSfAtom;
      sf[atom_off(r, blk & 3)] = (uint8_t)s0;
      sf[kSfAtom + atom_off(r, blk & 3)] = (uint8_t)s1;
    }
  }
}

// Scale re-layout: [E][rows][K/32] ue8m0 -> [E][rows/128][K/128][mats][512-byte atom],
// atom byte (r%32)*16 + (r/32)*4 + kb holds k-block kb of row r.  With two
// matrices (W1, W3) their atoms of the same (tile, chunk) are adjacent.
__global__ void prep_scales_kernel(const uint8_t* __restrict__ s0, const uint8_t* __restrict__ s1, int mats,
                                   int64_t n_words, int rows, int K, uint32_t* __restrict__ out) {
  const int RT = rows / 128, KC = K / 128, KB = K / 32;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < n_words;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int wi = (int)(w & 127);
    int64_t a = w >> 7;
    const int mat = (int)(a % mats);
    a /= mats;
    const int kc = (int)(a % KC);
    a /= KC;
    const int rt = (int)(a % RT);
    const int64_t e = a / RT;
    const int row = rt * 128 + (wi >> 2) + 32 * (wi & 3);
    const uint8_t* src = (mat ? s1 : s0) + ((size_t)e * rows + row) * KB + kc * 4;
    out[w] = *reinterpret_cast<const uint32_t*>(src);
  }
}

// ---------------------------------------------------------------- host side

// FP4 weights [rows][K/2] as e2m1 codes with 16U4_ALIGN16B (16 codes -> 16
// bytes of shared memory), viewed as {128 codes, rows, K/128 chunks}.
bool map_fp4(CUtensorMap* m, const void* base, uint64_t rows, uint64_t K, uint32_t box_rows) {
  const cuuint64_t dims[3] = {128, rows, K / 128};
  const cuuint64_t strides[2] = {K / 2, 64};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Layout {
  int64_t mk, cap, max_tiles;
  size_t ints, sorted, pos, blk, tiles, xq, sfx, hq, sfh, y, total;
};

Layout layout(const DsMoeDesc* d, int64_t T) {
  Layout L;
  L.mk = T * d->top_k;
  L.cap = align::capacity(L.mk, d->n_experts, kBlock);
  L.max_tiles = align::max_tiles(L.mk, d->n_experts, kBlock, kTileRows);
  const size_t H = d->hidden, I = d->inter;
  size_t o = 0;
  L.ints = o;   o += up(256);
  L.sorted = o; o += up(L.cap * 4);
  L.pos = o;    o += up(L.mk * 4);
  L.blk = o;    o += up(L.cap / kBlock * 4);
  L.tiles = o;  o += up(L.max_tiles * 16);
  L.xq = o;     o += up(L.cap * kXPieces * H);
  L.sfx = o;    o += up(L.max_tiles * (H / 128) * kXPieces * kSfAtom);
  L.hq = o;     o += up(L.cap * kHPieces * I);
  L.sfh = o;    o += up(L.max_tiles * (I / 128) * kHPieces * kSfAtom);
  L.y = o;      o += up(L.cap * H * 4);
  L.total = o;
  return L;
}

bool is_q3(const DsMoeDesc* d) { return d != nullptr && d->w1.format == DS_FMT_Q3; }

int validate(const DsMoeDesc* d, int64_t T) {
  DS_REQUIRE(d != nullptr, DS_EINVAL, "grouped_ffn: null descriptor");
  DS_REQUIRE(T >= 1 && d->top_k >= 1 && T * d->top_k < ((int64_t)1 << 30), DS_EINVAL,
             "grouped_ffn: tokens and top_k must be >= 1");
  if (is_q3(d)) return q3_validate(d);
  DS_REQUIRE(d->w1.format == DS_FMT_FP4 && d->w3.format == DS_FMT_FP4 && d->w2.format == DS_FMT_FP4, DS_ENOTSUP,
             "grouped_ffn: expert banks must be all FP4 or all Q3");
  DS_REQUIRE(d->n_experts >= 1 && d->n_experts <= align::kMaxExperts, DS_ENOTSUP,
             "grouped_ffn: n_experts must be in [1, %d]", align::kMaxExperts);
  DS_REQUIRE(d->hidden % 128 == 0 && d->inter % 128 == 0 && d->hidden > 0 && d->inter > 0, DS_EINVAL,
             "grouped_ffn: hidden and inter must be positive multiples of 128");
  const int E = d->n_experts, H = d->hidden, I = d->inter;
  DS_REQUIRE(d->w1.n_experts == E && d->w1.rows == I && d->w1.cols == H && d->w3.n_experts == E &&
                 d->w3.rows == I && d->w3.cols == H && d->w2.n_experts == E && d->w2.rows == H && d->w2.cols == I,
             DS_EINVAL, "grouped_ffn: bank shapes do not match the descriptor");
  DS_REQUIRE(d->w1.data && d->w3.data && d->w2.data && d->w1.scales && d->w3.scales && d->w2.scales, DS_EINVAL,
             "grouped_ffn: null bank pointer");
  DS_REQUIRE(ds::aligned(d->w1.data, 32) && ds::aligned(d->w3.data, 32) && ds::aligned(d->w2.data, 32) &&
                 ds::aligned(d->w1.scales, 4) && ds::aligned(d->w3.scales, 4) && ds::aligned(d->w2.scales, 4),
             DS_EALIGN, "grouped_ffn: FP4 data 32-byte and scales 4-byte aligned");
  DS_REQUIRE(!(d->shared_w1 || d->shared_w3 || d->shared_w2), DS_ENOTSUP,
             "grouped_ffn: the shared expert is not part of the grouped call");
  DS_REQUIRE((int64_t)E * I < ((int64_t)1 << 31) && (int64_t)E * H < ((int64_t)1 << 31), DS_EINVAL,
             "grouped_ffn: bank too large");
  return DS_OK;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

bool map_pieces(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_combine(const float* y, const int32_t* pos, const float* topk_w, const int32_t* n_pad, int* err, int k,
                   int H, int route_after, void* out, int out_dtype, int64_t tokens, cudaStream_t s) {
  if (out_dtype == DS_F32)
    combine_kernel<float><<<(unsigned)tokens, 256, 0, s>>>(y, pos, topk_w, n_pad, err, k, H, route_after,
                                                            static_cast<float*>(out));
  else
    combine_kernel<__nv_bfloat16><<<(unsigned)tokens, 256, 0, s>>>(y, pos, topk_w, n_pad, err, k, H, route_after,
                                                                    static_cast<__nv_bfloat16*>(out));
  DS_CHECK_LAUNCH("combine_kernel");
  return DS_OK;
}

}  // namespace grouped
}  // namespace ds

using namespace ds::grouped;

extern "C" int ds_grouped_scales_size(const DsMoeDesc* desc, size_t* w13_bytes, size_t* w2_bytes) {
  int st = validate(desc, 1);
  if (st != DS_OK) return st;
  DS_REQUIRE(w13_bytes && w2_bytes, DS_EINVAL, "grouped_scales_size: null output");
  if (is_q3(desc)) {   // q3 banks are read as stored
    *w13_bytes = *w2_bytes = 0;
    return DS_OK;
  }
  const size_t E = desc->n_experts, H = desc->hidden, I = desc->inter;
  *w13_bytes = E * (I / 128) * (H / 128) * 2 * kSfAtom;
  *w2_bytes = E * (H / 128) * (I / 128) * kSfAtom;
  return DS_OK;
}

extern "C" int ds_grouped_prepare_scales(const DsMoeDesc* desc, void* w13_sf, void* w2_sf, void* stream) {
  int st = validate(desc, 1);
  if (st != DS_OK) return st;
  if (is_q3(desc)) return DS_OK;
  DS_REQUIRE(w13_sf && w2_sf && ds::aligned(w13_sf, 16) && ds::aligned(w2_sf, 16), DS_EALIGN,
             "grouped_prepare_scales: outputs must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int E = desc->n_experts, H = desc->hidden, I = desc->inter;
  const int64_t w13 = (int64_t)E * (I / 128) * (H / 128) * 2 * 128;
  const int64_t w2 = (int64_t)E * (H / 128) * (I / 128) * 128;
  const int grid = ds::sm_count() * 4;
  prep_scales_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(desc->w1.scales),
                                          static_cast<const uint8_t*>(desc->w3.scales), 2, w13, I, H,
                                          static_cast<uint32_t*>(w13_sf));
  DS_CHECK_LAUNCH("prep_scales_kernel (w13)");
  prep_scales_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(desc->w2.scales), nullptr, 1, w2, H, I,
                                          static_cast<uint32_t*>(w2_sf));
  DS_CHECK_LAUNCH("prep_scales_kernel (w2)");
  return DS_OK;
}

extern "C" int ds_fp4_scale_atoms(const void* scales, int64_t n_experts, int rows, int cols, void* atoms,
                                  void* stream) {
  DS_REQUIRE(scales && atoms, DS_EINVAL, "fp4_scale_atoms: null pointer");
  DS_REQUIRE(n_experts >= 1 && rows > 0 && cols > 0 && rows % 128 == 0 && cols % 128 == 0, DS_EINVAL,
             "fp4_scale_atoms: rows and cols must be positive multiples of 128");
  DS_REQUIRE(ds::aligned(scales, 4) && ds::aligned(atoms, 16), DS_EALIGN,
             "fp4_scale_atoms: scales 4-byte, atoms 16-byte aligned");
  const int64_t words = n_experts * (rows / 128) * (cols / 128) * 128;
  prep_scales_kernel<<<ds::sm_count() * 4, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(scales), nullptr, 1, words, rows, cols, static_cast<uint32_t*>(atoms));
  DS_CHECK_LAUNCH("prep_scales_kernel (atoms)");
  return DS_OK;
}

extern "C" int ds_grouped_ffn_workspace_size(const DsMoeDesc* desc, int64_t tokens, size_t* bytes) {
  int st = validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(bytes != nullptr, DS_EINVAL, "grouped_ffn_workspace_size: null output");
  *bytes = is_q3(desc) ? q3_workspace_bytes(desc, tokens) : layout(desc, tokens).total;
  return DS_OK;
}

extern "C" int ds_grouped_ffn(const DsMoeDesc* desc, const void* w13_sf, const void* w2_sf, const void* x,
                              int x_dtype, int64_t tokens, const int32_t* topk_ids, const float* topk_w, void* out,
                              int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int st = validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(x_dtype == DS_BF16, DS_ENOTSUP, "grouped_ffn: x must be bf16");
  DS_REQUIRE(out_dtype == DS_BF16 || out_dtype == DS_F32, DS_EINVAL, "grouped_ffn: out_dtype must be bf16 or f32");
  if (is_q3(desc))
    return q3_ffn(desc, x, tokens, topk_ids, topk_w, out, out_dtype, workspace, workspace_bytes,
                  static_cast<cudaStream_t>(stream));
  DS_REQUIRE(w13_sf && w2_sf && x && topk_ids && topk_w && out && workspace, DS_EINVAL,
             "grouped_ffn: null pointer");
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 16) && ds::aligned(workspace, 256) &&
                 ds::aligned(w13_sf, 16) && ds::aligned(w2_sf, 16),
             DS_EALIGN, "grouped_ffn: x/out/scales 16-byte and workspace 256-byte aligned");
  const Layout L = layout(desc, tokens);
  DS_REQUIRE(workspace_bytes >= L.total, DS_EINVAL, "grouped_ffn: workspace %zu bytes < required %zu",
             workspace_bytes, L.total);
  DS_REQUIRE(encode_fn() != nullptr, DS_ECUDA, "grouped_ffn: cuTensorMapEncodeTiled unavailable");
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
  ao.tile_rows = kTileRows;
  if ((st = ds::align::launch(topk_ids, L.mk, E, kBlock, 1, ao, s)) != DS_OK) return st;

  xquant_kernel<<<ds::sm_count() * 4, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), sorted, ints, blk, tiles,
                                                    (int)L.mk, k, H, xq, sfx);
  DS_CHECK_LAUNCH("xquant_kernel");

  Params p;
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
  bool ok = map_fp4(&p.a0, desc->w1.data, (uint64_t)E * I, H, 128) &&
            map_fp4(&p.a1, desc->w3.data, (uint64_t)E * I, H, 128) &&
            map_pieces(&p.b, xq, L.cap, (uint64_t)kXPieces * H, kTileRows);
  DS_REQUIRE(ok, DS_ECUDA, "grouped_ffn: tensor map encoding failed (gate/up)");
  p.sfa = static_cast<const uint8_t*>(w13_sf);
  p.sfb = sfx;
  const int sms = ds::sm_count();
  const int64_t items_a = L.max_tiles * (I / 128), items_b = L.max_tiles * (H / 128);
  const int grid_a = (int)std::min<int64_t>(sms, items_a), grid_b = (int)std::min<int64_t>(sms, items_b);
  DS_CHECK_CUDA(cudaFuncSetAttribute(gemm_kernel<GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem_bytes<GATEUP>()));
  gemm_kernel<GATEUP><<<grid_a, kThreads, smem_bytes<GATEUP>(), s>>>(p);
  DS_CHECK_LAUNCH("gemm_kernel<gate/up>");

  ok = map_fp4(&p.a0, desc->w2.data, (uint64_t)E * H, I, 128) &&
       map_pieces(&p.b, hq, L.cap, (uint64_t)kHPieces * I, kTileRows);
  DS_REQUIRE(ok, DS_ECUDA, "grouped_ffn: tensor map encoding failed (down)");
  p.sfa = static_cast<const uint8_t*>(w2_sf);
  p.sfb = sfh;
  DS_CHECK_CUDA(cudaFuncSetAttribute(gemm_kernel<DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem_bytes<DOWN>()));
  gemm_kernel<DOWN><<<grid_b, kThreads, smem_bytes<DOWN>(), s>>>(p);
  DS_CHECK_LAUNCH("gemm_kernel<down>");

  return launch_combine(y, pos, topk_w, ints, ints + 2, k, H, desc->route_before_down ? 0 : 1, out, out_dtype,
                        tokens, s);
}
