// Batched grouped expert FFN over q3 banks (3-bit affine codes, group 64, f16
// scale and bias per group) on tcgen05 block-scaled MMAs.
//
// Replaces the per-expert loop of moe_layer / gather_pinned_contributions for
// q3 banks (src/deepseeker/mlx_forward.py:99-101 qmm with biases, 187-193
// gather_qmm with group_size 64 and bits 3, 388-419 the loop).
//
// The codes are dequantised in shared memory exactly: a code q in 0..7
// becomes the e4m3 byte of q (every integer 0..7 is an e4m3 value), so the
// MMA computes D_g = sum over the group's 64 K of q * a for the activation a.
// The group's f16 scale s and bias b enter per group in the epilogue:
//   y = sum_g s_g * D_g + b_g * A_g,   A_g = the sum of the group's activations,
// which equals sum_k (s q + b) a with the weights never rounded.
//
// Launch sequence (one stream, no host sync):
//   1. align   : expert runs padded to 16 rows, cut into tiles of 16 rows;
//   2. xquant  : every padded row's x as two e4m3 pieces (hi + lo reproduce a
//                bf16 value), per-32 ue8m0 scales, and per-64 sums of x;
//   3. gate/up : per (tile, 128 rows of I): W1 and W3 codes converted to e4m3
//                in shared memory, one accumulator per 64-group and matrix;
//                the epilogue adds s * D + b * X per group into f32 sums, then
//                writes h = silu(min(g, L)) * clip(u, +-L) [* route weight]
//                as three e4m3 pieces with per-32 scales and h's 32-row sums;
//   4. down    : the same over W2 with h's three pieces, f32 rows out;
//   5. combine : shared with the FP4 path.
//
// Persistent GEMM kernels, one CTA per SM, 448 threads: warp 0 issues TMA
// copies into a ring (each weight row's 48 code bytes per 128-wide K stage,
// the tile's activation pieces, their scale atom), warp 1 issues the MMAs and
// owns tensor memory, warps 2-9 convert codes to e4m3 in the 128-byte-swizzled
// operand layout (two per scheduler: the conversion is ALU work with short
// dependency chains) and warps 2-5 also stage the activation scale atom in
// tensor memory, warps 10-13 run the epilogue.  B operand row `pieces * t + p` holds piece p of the
// tile's token t, so one MMA covers every piece.  The accumulators of a whole
// stage (both groups) form one tensor-memory buffer with one commit / wait /
// release, and three or four such buffers let the MMAs run ahead of the
// epilogue: the group-by-group handshake was what paced the pipeline.  Every wait is bounded; a
// timeout sets an error bit and an abort flag that ends every role.
#include <algorithm>

#include "align.cuh"
#include "grouped.cuh"
#include "tc5.cuh"

namespace ds {
namespace grouped {
namespace {

using namespace ds::ptx;

constexpr int kQR = 16;              // token rows per tile
constexpr int kQThreads = 448;       // 14 warps
constexpr int kConvWarps = 8;        // warps 2..9
constexpr int kEpiWarp0 = 10;        // warps 10..13
constexpr int kRowBytes = 48;        // code bytes of one weight row per 128-wide K stage (2 groups x 24 B)
constexpr int kConv = 16384;         // one matrix's converted stage: 128 rows x 128 e4m3 bytes
constexpr int kCS = 3;               // converted stages
constexpr int kXP = 2, kHP = 3;      // pieces per x row, per h row
constexpr int kSmemMax = 227 * 1024;

template <int MODE>
struct QC;
// gate/up: A = 128 rows of W1 and of W3, B = x pieces of 16 tokens (32 rows).
template <>
struct QC<GATEUP> {
  static constexpr int kMats = 2, kPieces = kXP, kStages = 6, kNB = 3;
  static constexpr int kB = kPieces * kQR * 128;            // 4 KB
  static constexpr int kW = kMats * 128 * kRowBytes;        // 12 KB
  static constexpr int kGroupCols = kMats * kPieces * kQR;  // 64 tensor-memory columns per 64-group
  static constexpr int kAccCols = 2 * kGroupCols;           // 128 per stage buffer (two groups)
};
// down: A = 128 rows of W2, B = h pieces of 16 tokens (48 rows).
template <>
struct QC<DOWN> {
  static constexpr int kMats = 1, kPieces = kHP, kStages = 8, kNB = 4;
  static constexpr int kB = kPieces * kQR * 128;            // 6 KB
  static constexpr int kW = kMats * 128 * kRowBytes;        // 6 KB
  static constexpr int kGroupCols = kMats * kPieces * kQR;  // 48
  static constexpr int kAccCols = 2 * kGroupCols;           // 96
};
static_assert(QC<GATEUP>::kNB * QC<GATEUP>::kAccCols <= 384 && QC<DOWN>::kNB * QC<DOWN>::kAccCols <= 384,
              "accumulators overlap the scale columns");
constexpr uint32_t kTmemA = 384;     // constant A scale atom (every byte 127: scale 1)
constexpr uint32_t kTmemB = 388;     // activation scale atoms, 4 columns per converted stage

// Dynamic shared memory of one GEMM launch whose reduction size is K.
template <int MODE>
size_t q3_smem(int K) {
  using C = QC<MODE>;
  return 1024 + (size_t)kCS * C::kMats * kConv + (size_t)C::kStages * (C::kB + C::kW + kSfAtom) +
         2 * (size_t)(K / 64) * kQR * sizeof(float);
}

struct QParams {
  CUtensorMap w[2];          // code rows, UINT8 {K*3/8 B, rows}, box {48 B, 128 rows} (gate/up: W1, W3; down: W2)
  CUtensorMap b;             // activation pieces, UINT8 {128 B, pieces*cap rows, K/128}, box {128 B, pieces*32}
  const __half* sc[2];       // bank scales [E*rows][K/64]
  const __half* bi[2];       // bank biases
  const uint8_t* sfb;        // piece scale atoms [tiles][K/128][512]
  const float* asum;         // gate/up: x 64-sums [tiles][K/64][32]; down: h 32-sums [tiles][K/32][32]
  const int4* tiles;         // {expert, first row, rows, 0}
  const int32_t* n_tiles;
  const int32_t* sorted_ids; // padded row -> pair (sentinel = mk)
  const float* topk_w;       // [mk]
  uint8_t* hq;               // gate/up output: h pieces [cap][3][I]
  uint8_t* sfh;              // gate/up output: their scale atoms [tiles][I/128][512]
  float* hsum;               // gate/up output: h 32-row sums [tiles][I/32][32]
  float* y;                  // down output [cap][H] f32
  int* err;
  int H, I, mk;
  float limit;
  int gate_in_h;             // route weight applied to h (before the down projection)
};

// 2-bit fields in bits 0-7 and 16-23 -> the low two bits of 4-bit nibbles
// (bits 0-15 and 16-31 of the result, field j of a half in nibble j).
__device__ __forceinline__ uint32_t spread2(uint32_t x) {
  x = (x | (x << 4)) & 0x0F0F0F0Fu;
  return (x | (x << 2)) & 0x33333333u;
}
// 1-bit fields in bits 0-3 and 16-19 -> bit 2 of the nibbles.
__device__ __forceinline__ uint32_t spread1(uint32_t h) {
  h = (h | (h << 6)) & 0x03030303u;
  return ((h | (h << 3)) & 0x11111111u) << 2;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// 16 consecutive codes of one 64-group -> 16 e4m3 bytes in element order.
// L = the group's low word for these elements (two low bits of element j at
// bits 2j and of element 8+j at bits 16+2j), Hh = its high word shifted so
// that bit j / 16+j hold bit 2 of element j / 8+j.  The selector nibbles are
// the codes, and prmt looks each up in the e4m3 table of 0..7.
__device__ __forceinline__ uint4 codes16_to_e4m3(uint32_t L, uint32_t Hh) {
  constexpr uint32_t kLut03 = 0x44403800u;   // e4m3 of 0, 1, 2, 3
  constexpr uint32_t kLut47 = 0x4E4C4A48u;   // e4m3 of 4, 5, 6, 7
  const uint32_t a = spread2(L & 0x00FF00FFu) | spread1(Hh & 0x000F000Fu);                 // 0-3 | 8-11
  const uint32_t b = spread2((L >> 8) & 0x00FF00FFu) | spread1((Hh >> 4) & 0x000F000Fu);   // 4-7 | 12-15
  return make_uint4(prmt(kLut03, kLut47, a), prmt(kLut03, kLut47, b), prmt(kLut03, kLut47, a >> 16),
                    prmt(kLut03, kLut47, b >> 16));
}

__device__ __forceinline__ float f16_half(uint32_t w, int hi) {
  return __half2float(__ushort_as_half((unsigned short)(hi ? (w >> 16) : (w & 0xFFFFu))));
}

// Every padded row gets its token's x (bf16) as hi/lo e4m3 pieces (B rows
// 2r and 2r + 1 of its tile), their scales, and the f32 sum of every 64-group
// of x (the bias term of the gate/up projections); sentinel rows are zero.
// One warp per row, one lane per 32-element block.
__global__ void __launch_bounds__(256) q3_xquant_kernel(const __nv_bfloat16* __restrict__ x,
                                                        const int32_t* __restrict__ sorted_ids,
                                                        const int32_t* __restrict__ n_pad,
                                                        const int32_t* __restrict__ blk_tile,
                                                        const int4* __restrict__ tiles, int mk, int k, int H,
                                                        uint8_t* __restrict__ xq, uint8_t* __restrict__ sfx,
                                                        float* __restrict__ xsum) {
  const int lane = threadIdx.x & 31;
  const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int np = *n_pad;
  const int KC = H / 128, nb = H / 32, G = H / 64;
  for (int row = w0; row < np; row += nw) {
    const int pr = sorted_ids[row];
    const int tile = blk_tile[row / kBlock];
    const int r = row - tiles[tile].y;
    uint8_t* dst = xq + (size_t)row * kXP * H;
    for (int base = 0; base < nb; base += 32) {
      const int blk = base + lane;
      const bool act = blk < nb;   // nb is even: both blocks of a 64-group are active or neither
      float v[32];
      if (act && pr < mk) {
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
      float a = 0.0f, bs = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        a = fmaxf(a, fabsf(v[j]));
        bs += v[j];
      }
      // the 64-group sum: even block first, the same value in both lanes
      const float other = __shfl_xor_sync(0xffffffffu, bs, 1);
      const float gsum = (lane & 1) ? other + bs : bs + other;
      if (!act) continue;
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
      uint8_t* sf = sfx + ((size_t)tile * KC + blk / 4) * kSfAtom;
      sf[atom_off(2 * r, blk & 3)] = (uint8_t)s0;
      sf[atom_off(2 * r + 1, blk & 3)] = (uint8_t)s1;
      if ((lane & 1) == 0) xsum[((size_t)tile * G + blk / 2) * kQR + r] = gsum;
    }
  }
}

// Epilogue of one item (tile x 128 weight rows) for a tile of Z = 16 token
// rows.  Thread = one weight row of the item (lane quarter q, lane).  Per
// stage (two 64-groups, one accumulator buffer `stage % kNB`): read each
// group's accumulators (pieces summed), add s * D + b * A with the row's f16
// scale / bias and the tile's activation sums `asm_` ([G][16] in shared
// memory).  `stage` counts stages over the CTA's items.  Returns false on abort.
template <int MODE, int Z>
__device__ bool q3_epilogue(const QParams& p, const float* asm_, int tile, int mt, int4 td, int q, int lane, int KC,
                            uint32_t tb, int& stage, uint64_t* accfull, uint64_t* accempty, volatile int* abort) {
  using C = QC<MODE>;
  constexpr int NB = C::kNB, MATS = C::kMats;
  if (*abort) return false;
  const int rows_out = MODE == GATEUP ? p.I : p.H;
  const int G = 2 * KC;
  const int row = mt * 128 + q * 32 + lane;                  // output row of the matrix
  const size_t wrow = (size_t)td.x * rows_out + row;         // row of the bank
  // scale / bias words of a stage (two groups, f16 each) of this row, two
  // stages ahead of their use; 4-byte aligned as G is even
  const uint32_t* s0p = reinterpret_cast<const uint32_t*>(p.sc[0] + wrow * G);
  const uint32_t* b0p = reinterpret_cast<const uint32_t*>(p.bi[0] + wrow * G);
  const uint32_t* s1p = reinterpret_cast<const uint32_t*>(p.sc[MATS - 1] + wrow * G);
  const uint32_t* b1p = reinterpret_cast<const uint32_t*>(p.bi[MATS - 1] + wrow * G);
  uint32_t cur[4] = {0, 0, 0, 0}, nx1[4] = {0, 0, 0, 0}, nx2[4] = {0, 0, 0, 0};
  auto load_sb = [&](int kc, uint32_t(&o)[4]) {
    if (kc < KC) {
      o[0] = __ldg(s0p + kc);
      o[1] = __ldg(b0p + kc);
      if (MATS > 1) {
        o[2] = __ldg(s1p + kc);
        o[3] = __ldg(b1p + kc);
      }
    }
  };
  load_sb(0, cur);
  load_sb(1, nx1);
  load_sb(2, nx2);
  float acc0[Z], acc1[Z];
#pragma unroll
  for (int t = 0; t < Z; ++t) acc0[t] = acc1[t] = 0.0f;
  for (int kc = 0; kc < KC; ++kc, ++stage) {
    const int a = stage % NB;
    if (!warp_wait(&accfull[a], (stage / NB) & 1, abort, p.err)) return false;
    tc5::fence_after();
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const uint32_t dacc = tc5::lane_quarter(tb + a * C::kAccCols + gg * C::kGroupCols, q);
      const float* X = asm_ + (2 * kc + gg) * kQR;
      const float s0 = f16_half(cur[0], gg), b0 = f16_half(cur[1], gg);
      if (MODE == GATEUP) {
        const float s1 = f16_half(cur[2], gg), b1 = f16_half(cur[3], gg);
#pragma unroll
        for (int t0 = 0; t0 < Z; t0 += 8) {
          float v0[16], v1[16];
          tc5::ld_x16_nowait(dacc + 2 * t0, v0);                    // W1: columns 2t (hi), 2t + 1 (lo)
          tc5::ld_x16_nowait(dacc + kXP * kQR + 2 * t0, v1);        // W3
          tc5::wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xs = X[t0 + j];
            acc0[t0 + j] = fmaf(s0, v0[2 * j] + v0[2 * j + 1], fmaf(b0, xs, acc0[t0 + j]));
            acc1[t0 + j] = fmaf(s1, v1[2 * j] + v1[2 * j + 1], fmaf(b1, xs, acc1[t0 + j]));
          }
        }
      } else {
        float v[48];
        tc5::ld_x16_nowait(dacc, *reinterpret_cast<float(*)[16]>(v));
        tc5::ld_x16_nowait(dacc + 16, *reinterpret_cast<float(*)[16]>(v + 16));
        tc5::ld_x16_nowait(dacc + 32, *reinterpret_cast<float(*)[16]>(v + 32));
        tc5::wait_ld();
#pragma unroll
        for (int j = 0; j < Z; ++j)
          acc0[j] = fmaf(s0, (v[3 * j] + v[3 * j + 1]) + v[3 * j + 2], fmaf(b0, X[j], acc0[j]));
      }
    }
    tc5::fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&accempty[a]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      cur[i] = nx1[i];
      nx1[i] = nx2[i];
    }
    load_sb(kc + 3, nx2);
  }

  if (MODE == DOWN) {
#pragma unroll
    for (int t = 0; t < Z; ++t) p.y[(size_t)(td.y + t) * p.H + row] = acc0[t];
    return true;
  }
  // gate/up: h, its three e4m3 pieces (B rows 3t + pc of the down launch;
  // the 32 lanes are one 32-block of the down projection's K) and its sums
  const int I = p.I, KC2 = I / 128;
  float h[Z];
#pragma unroll
  for (int t = 0; t < Z; ++t) {
    float w = 1.0f;
    if (p.gate_in_h) {
      const int pr = p.sorted_ids[td.y + t];
      w = pr < p.mk ? p.topk_w[pr] : 0.0f;
    }
    h[t] = silu_glu(acc0[t], acc1[t], p.limit) * w;
  }
  uint8_t* sf = p.sfh + ((size_t)tile * KC2 + mt) * kSfAtom;
#pragma unroll
  for (int t = 0; t < Z; t += 2) {
    int ef[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float am = fabsf(h[t + c]);
#pragma unroll
      for (int d = 16; d; d >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, d));
      ef[c] = (int)(__float_as_uint(am) >> 23);
    }
    uint8_t* dst0 = p.hq + (size_t)(td.y + t) * kHP * I + row;
    uint8_t* dst1 = dst0 + (size_t)kHP * I;
    float r0 = h[t], r1 = h[t + 1];
#pragma unroll
    for (int pc = 0; pc < kHP; ++pc) {
      const int e0 = piece_scale(ef[0], pc), e1 = piece_scale(ef[1], pc);
      const uint32_t bb = tc5::f32x2_to_e4m3x2(r0 * inv_scale_of(e0), r1 * inv_scale_of(e1));
      float v0, v1;
      tc5::e4m3x2_to_f32x2(bb, v0, v1);
      r0 = fmaf(-v0, scale_of(e0), r0);
      r1 = fmaf(-v1, scale_of(e1), r1);
      dst0[(size_t)pc * I] = (uint8_t)(bb & 0xFFu);
      dst1[(size_t)pc * I] = (uint8_t)(bb >> 8);
      if (lane == 0) {
        sf[atom_off(kHP * t + pc, q)] = (uint8_t)e0;
        sf[atom_off(kHP * (t + 1) + pc, q)] = (uint8_t)e1;
      }
    }
  }
  float* hs = p.hsum + ((size_t)tile * (I / 32) + mt * 4 + q) * kQR;
#pragma unroll
  for (int t = 0; t < Z; ++t) {
    float v = h[t];
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    if (lane == 0) hs[t] = v;
  }
  return true;
}

template <int MODE>
__global__ void __launch_bounds__(kQThreads, 1) q3_gemm_kernel(const __grid_constant__ QParams p) {
  using C = QC<MODE>;
  constexpr int S = C::kStages, NB = C::kNB, MATS = C::kMats, PC = C::kPieces;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* conv = smem;                                       // kCS x MATS x 16 KB (SW128 A operands)
  uint8_t* bsm = conv + kCS * MATS * kConv;                   // S x kB (SW128 B operands)
  uint8_t* wsm = bsm + S * C::kB;                             // S x kW (raw code rows)
  uint8_t* sfs = wsm + S * C::kW;                             // S x 512 (B scale atoms)
  float* sums = reinterpret_cast<float*>(sfs + S * kSfAtom);  // 2 x G x 32 (activation sums per item)
  __shared__ __align__(8) uint64_t full[S], empty[S], cfull[kCS], cempty[kCS], accfull[NB], accempty[NB], done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_out = MODE == GATEUP ? p.I : p.H;
  const int K = MODE == GATEUP ? p.H : p.I;
  const int MT = rows_out / 128, KC = K / 128, G = K / 64;
  const int n_items = *p.n_tiles * MT;
  if ((int)blockIdx.x >= n_items) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int c = 0; c < kCS; ++c) {
      mbar_init(&cfull[c], kConvWarps);
      mbar_init(&cempty[c], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 4);
    }
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc5::alloc(&tmem_base, 512);
  __syncthreads();
  tc5::fence_after();
  const uint32_t tb = tmem_base;
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t wpol = policy_evict_first();   // codes are read once per call
      int g = 0;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int tile = item / MT, mt = item % MT;
        const int4 td = p.tiles[tile];
        for (int kc = 0; kc < KC; ++kc, ++g) {
          const int s = g % S;
          if (g >= S && !wait_or_abort(&empty[s], ((g / S) - 1) & 1, abort, p.err)) goto drain;
          mbar_arrive_expect_tx(&full[s], C::kW + C::kB + kSfAtom);
#pragma unroll
          for (int m = 0; m < MATS; ++m)
            tma_load_2d_hint(wsm + s * C::kW + m * 128 * kRowBytes, &p.w[m], kc * kRowBytes,
                             td.x * rows_out + mt * 128, &full[s], wpol);
          tma_load_3d(bsm + s * C::kB, &p.b, 0, td.y * PC, kc, &full[s]);
          bulk_g2s(sfs + s * kSfAtom, p.sfb + ((size_t)tile * KC + kc) * kSfAtom, kSfAtom, &full[s]);
        }
      }
    drain:
      // never leave with copies in flight into this CTA's shared memory
      for (int j = g - S < 0 ? 0 : g - S; j < g; ++j) mbar_wait_bounded(&full[j % S], (j / S) & 1, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Per stage (K = 128, two 64-groups): accumulator buffer g % NB, one
    // fresh accumulator per group and matrix, two K steps of 32 each.  The
    // whole warp runs the loop (warp-uniform waits and operands); one
    // elected lane issues.
    {
      int g = 0;
      const uint32_t conv0 = smem_u32(conv), b0 = smem_u32(bsm);
      // descriptors: a K step of 32 advances the start address by 32 B = 2
      // units of the descriptor's address field (no carry: shared memory
      // addresses stay below 256 KB)
      const uint64_t ad_base = tc5::sdesc_sw128(conv0), bd_base = tc5::sdesc_sw128(b0);
      const uint32_t sfa = tb + kTmemA;
      for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int N = PC * p.tiles[item / MT].z;
        uint32_t idesc[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) idesc[kk] = tc5::idesc_e4m3_e4m3(N, kk);
        for (int kc = 0; kc < KC; ++kc, ++g) {
          const int s = g % S, c = g % kCS;
          // the converters arrive on cfull after they have seen the stage's
          // copies land, so waiting for cfull covers the copies too
          if (!warp_wait(&cfull[c], (g / kCS) & 1, abort, p.err)) goto mma_out;
          tc5::fence_after();
          const int a = g % NB;
          if (g >= NB) {
            if (!warp_wait(&accempty[a], ((g / NB) - 1) & 1, abort, p.err)) goto mma_out;
            tc5::fence_after();
          }
          if (elect_one()) {
            const uint64_t ad = ad_base + (uint64_t)((c * MATS * kConv) >> 4);
            const uint64_t bd = bd_base + (uint64_t)((s * C::kB) >> 4);
            const uint32_t d0 = tb + a * C::kAccCols, sfb = tb + kTmemB + 4 * c;
#pragma unroll
            for (int gg = 0; gg < 2; ++gg)
#pragma unroll
              for (int m = 0; m < MATS; ++m)
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                  const int kk = 2 * gg + ks;
                  tc5::mma_mxf8f6f4(d0 + gg * C::kGroupCols + m * PC * kQR, ad + (m * kConv >> 4) + 2 * kk,
                                    bd + 2 * kk, idesc[kk], sfa, sfb, ks);
                }
            tc5::commit(&accfull[a]);
          }
          __syncwarp();
          if (elect_one()) {
            tc5::commit(&empty[s]);
            tc5::commit(&cempty[c]);
          }
          __syncwarp();
        }
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
    // ------------------------------------------------------------ converters
    // warp 2 + cw: rows (cw % 4) * 32 + lane of the 128-row tile; gate/up:
    // matrix cw / 4 (W1, W3); down: group cw / 4 of the stage (chunks 4 part
    // .. 4 part + 3).  Warps 2-5 (one per lane quarter) also write the scale
    // atoms into tensor memory.
    const int cw = warp - 2, part = cw >> 2;
    const int q = warp & 3;
    const int r = (cw & 3) * 32 + lane;
    const bool stager = cw < 4;
    if (stager) {
      tc5::st_x4(tc5::lane_quarter(tb + kTmemA, q), 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
      tc5::wait_st();
    }
    int g = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      for (int kc = 0; kc < KC; ++kc, ++g) {
        const int s = g % S, c = g % kCS;
        if (!warp_wait(&full[s], (g / S) & 1, abort, p.err)) goto cv_out;
        if (g >= kCS && !warp_wait(&cempty[c], ((g / kCS) - 1) & 1, abort, p.err)) goto cv_out;
        {
          const int m = MATS > 1 ? part : 0;
          const uint4* src = reinterpret_cast<const uint4*>(wsm + s * C::kW + (m * 128 + r) * kRowBytes);
          uint8_t* dst = conv + (c * MATS + m) * kConv + r * 128;
          if (MATS > 1) {   // the whole row: both groups
            const uint4 u0 = src[0], u1 = src[1], u2 = src[2];
            const uint32_t wd[12] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w, u2.x, u2.y, u2.z, u2.w};
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {   // 16 codes each: group ch / 4, low word ch % 4
              const int gg = ch >> 2, w = ch & 3;
              const uint32_t Hh = wd[gg * 6 + 4 + (w >> 1)] >> (8 * (w & 1));
              *reinterpret_cast<uint4*>(dst + ((ch ^ (r & 7)) << 4)) = codes16_to_e4m3(wd[gg * 6 + w], Hh);
            }
          } else {          // one group of the row: six words at byte 24 * part
            const uint2* s2 = reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(src) + 24 * part);
            const uint2 a0 = s2[0], a1 = s2[1], a2 = s2[2];
            const uint32_t wd[6] = {a0.x, a0.y, a1.x, a1.y, a2.x, a2.y};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const int ch = 4 * part + w;
              const uint32_t Hh = wd[4 + (w >> 1)] >> (8 * (w & 1));
              *reinterpret_cast<uint4*>(dst + ((ch ^ (r & 7)) << 4)) = codes16_to_e4m3(wd[w], Hh);
            }
          }
        }
        if (stager) {
          const uint4 v = reinterpret_cast<const uint4*>(sfs + s * kSfAtom)[lane];
          tc5::st_x4(tc5::lane_quarter(tb + kTmemB + 4 * c, q), v.x, v.y, v.z, v.w);
          tc5::wait_st();
        }
        fence_proxy_async_smem();
        tc5::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&cfull[c]);
      }
    }
  cv_out:;
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int et = threadIdx.x - kEpiWarp0 * 32;   // 0..127
    int stage = 0, li = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
      const int tile = item / MT, mt = item % MT;
      const int4 td = p.tiles[tile];
      // the tile's activation sums, double-buffered over items (a warp
      // reaches item li + 2 only after every warp passed item li + 1's barrier)
      float* sm = sums + (li & 1) * G * kQR;
      if (MODE == GATEUP) {
        const float4* src = reinterpret_cast<const float4*>(p.asum + (size_t)tile * G * kQR);
        for (int i = et; i < G * kQR / 4; i += 128) reinterpret_cast<float4*>(sm)[i] = src[i];
      } else {
        const float* src = p.asum + (size_t)tile * (2 * G) * kQR;   // 32-row block sums of h
        for (int i = et; i < G * kQR; i += 128) {
          const int gq = i / kQR, t = i % kQR;
          sm[i] = src[(2 * gq) * kQR + t] + src[(2 * gq + 1) * kQR + t];
        }
      }
      bar_sync(1, 128);
      // after an abort every item returns at once, but the loop goes on so
      // that the four warps meet the same number of item barriers
      q3_epilogue<MODE, kQR>(p, sm, tile, mt, td, q, lane, KC, tb, stage, accfull, accempty, abort);
    }
  }
  tc5::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc5::fence_after();
    tc5::dealloc(tb, 512);
  }
}

}  // namespace

// ---------------------------------------------------------------- host side

namespace {

// q3 code rows [rows][K*3/8 B] as a 2-D UINT8 tensor; a box is one 128-wide K
// stage (48 B) of 128 rows.
bool map_codes(CUtensorMap* m, const void* base, uint64_t rows, uint64_t K) {
  const cuuint64_t dims[2] = {K * 3 / 8, rows};
  const cuuint64_t strides[1] = {K * 3 / 8};
  const cuuint32_t box[2] = {kRowBytes, 128};
  const cuuint32_t es[2] = {1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct QLayout {
  int64_t mk, cap, max_tiles;
  size_t ints, sorted, pos, blk, tiles, xq, sfx, xs, hq, sfh, hs, y, total;
};

QLayout q3_layout(const DsMoeDesc* d, int64_t T) {
  QLayout L;
  L.mk = T * d->top_k;
  L.cap = align::capacity(L.mk, d->n_experts, kBlock);
  L.max_tiles = align::max_tiles(L.mk, d->n_experts, kBlock, kQR);
  const size_t H = d->hidden, I = d->inter, NT = L.max_tiles;
  size_t o = 0;
  L.ints = o;   o += up(256);
  L.sorted = o; o += up(L.cap * 4);
  L.pos = o;    o += up(L.mk * 4);
  L.blk = o;    o += up(L.cap / kBlock * 4);
  L.tiles = o;  o += up(NT * 16);
  L.xq = o;     o += up(L.cap * kXP * H);
  L.sfx = o;    o += up(NT * (H / 128) * kSfAtom);
  L.xs = o;     o += up(NT * (H / 64) * kQR * 4);
  L.hq = o;     o += up(L.cap * kHP * I);
  L.sfh = o;    o += up(NT * (I / 128) * kSfAtom);
  L.hs = o;     o += up(NT * (I / 32) * kQR * 4);
  L.y = o;      o += up(L.cap * H * 4);
  L.total = o;
  return L;
}

}  // namespace

int q3_validate(const DsMoeDesc* d) {
  DS_REQUIRE(d->w1.format == DS_FMT_Q3 && d->w3.format == DS_FMT_Q3 && d->w2.format == DS_FMT_Q3, DS_ENOTSUP,
             "grouped_ffn: expert banks must be all FP4 or all Q3");
  DS_REQUIRE(d->n_experts >= 1 && d->n_experts <= align::kMaxExperts, DS_ENOTSUP,
             "grouped_ffn: n_experts must be in [1, %d]", align::kMaxExperts);
  DS_REQUIRE(d->hidden % 128 == 0 && d->inter % 128 == 0 && d->hidden > 0 && d->inter > 0, DS_EINVAL,
             "grouped_ffn: hidden and inter must be positive multiples of 128");
  const int E = d->n_experts, H = d->hidden, I = d->inter;
  DS_REQUIRE(d->w1.n_experts == E && d->w1.rows == I && d->w1.cols == H && d->w3.n_experts == E &&
                 d->w3.rows == I && d->w3.cols == H && d->w2.n_experts == E && d->w2.rows == H && d->w2.cols == I,
             DS_EINVAL, "grouped_ffn: bank shapes do not match the descriptor");
  const DsExpertBank* banks[3] = {&d->w1, &d->w3, &d->w2};
  for (const DsExpertBank* b : banks) {
    DS_REQUIRE(b->data && b->scales && b->biases, DS_EINVAL, "grouped_ffn: null q3 bank pointer");
    DS_REQUIRE(ds::aligned(b->data, 16) && ds::aligned(b->scales, 4) && ds::aligned(b->biases, 4), DS_EALIGN,
               "grouped_ffn: q3 words 16-byte, scales and biases 4-byte aligned");
  }
  DS_REQUIRE(!(d->shared_w1 || d->shared_w3 || d->shared_w2), DS_ENOTSUP,
             "grouped_ffn: the shared expert is not part of the grouped call");
  DS_REQUIRE((int64_t)E * I < ((int64_t)1 << 31) && (int64_t)E * H < ((int64_t)1 << 31), DS_EINVAL,
             "grouped_ffn: bank too large");
  DS_REQUIRE(q3_smem<GATEUP>(H) <= (size_t)kSmemMax && q3_smem<DOWN>(I) <= (size_t)kSmemMax, DS_ENOTSUP,
             "grouped_ffn: q3 banks need hidden <= %d and inter <= %d", (int)((kSmemMax - q3_smem<GATEUP>(0)) / 2),
             (int)((kSmemMax - q3_smem<DOWN>(0)) / 2));
  return DS_OK;
}

size_t q3_workspace_bytes(const DsMoeDesc* d, int64_t T) { return q3_layout(d, T).total; }

int q3_ffn(const DsMoeDesc* d, const void* x, int64_t tokens, const int32_t* topk_ids, const float* topk_w,
           void* out, int out_dtype, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  DS_REQUIRE(x && topk_ids && topk_w && out && workspace, DS_EINVAL, "grouped_ffn: null pointer");
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 16) && ds::aligned(workspace, 256), DS_EALIGN,
             "grouped_ffn: x/out 16-byte and workspace 256-byte aligned");
  const QLayout L = q3_layout(d, tokens);
  DS_REQUIRE(workspace_bytes >= L.total, DS_EINVAL, "grouped_ffn: workspace %zu bytes < required %zu",
             workspace_bytes, L.total);
  DS_REQUIRE(encode_fn() != nullptr, DS_ECUDA, "grouped_ffn: cuTensorMapEncodeTiled unavailable");
  char* ws = static_cast<char*>(workspace);
  int32_t* ints = reinterpret_cast<int32_t*>(ws + L.ints);  // [0] n_pad, [1] n_tiles, [2] error bits
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + L.sorted);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + L.pos);
  int32_t* blk = reinterpret_cast<int32_t*>(ws + L.blk);
  int4* tiles = reinterpret_cast<int4*>(ws + L.tiles);
  uint8_t* xq = reinterpret_cast<uint8_t*>(ws + L.xq);
  uint8_t* sfx = reinterpret_cast<uint8_t*>(ws + L.sfx);
  float* xs = reinterpret_cast<float*>(ws + L.xs);
  uint8_t* hq = reinterpret_cast<uint8_t*>(ws + L.hq);
  uint8_t* sfh = reinterpret_cast<uint8_t*>(ws + L.sfh);
  float* hs = reinterpret_cast<float*>(ws + L.hs);
  float* y = reinterpret_cast<float*>(ws + L.y);
  const int E = d->n_experts, H = d->hidden, I = d->inter, k = d->top_k;

  DS_CHECK_CUDA(cudaMemsetAsync(ints, 0, 256, s));
  align::Out ao = {};
  ao.sorted_ids = sorted;
  ao.n_pad = ints;
  ao.pos_of_pair = pos;
  ao.blk_tile = blk;
  ao.tiles = tiles;
  ao.n_tiles = ints + 1;
  ao.tile_rows = kQR;
  int st = align::launch(topk_ids, L.mk, E, kBlock, 1, ao, s);
  if (st != DS_OK) return st;

  const int sms = ds::sm_count();
  q3_xquant_kernel<<<sms * 4, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), sorted, ints, blk, tiles,
                                           (int)L.mk, k, H, xq, sfx, xs);
  DS_CHECK_LAUNCH("q3_xquant_kernel");

  QParams p;
  memset(&p, 0, sizeof(p));
  p.tiles = tiles;
  p.n_tiles = ints + 1;
  p.sorted_ids = sorted;
  p.topk_w = topk_w;
  p.hq = hq;
  p.sfh = sfh;
  p.hsum = hs;
  p.y = y;
  p.err = ints + 2;
  p.H = H;
  p.I = I;
  p.mk = (int)L.mk;
  p.limit = d->swiglu_limit;
  p.gate_in_h = d->route_before_down ? 1 : 0;

  bool ok = map_codes(&p.w[0], d->w1.data, (uint64_t)E * I, H) && map_codes(&p.w[1], d->w3.data, (uint64_t)E * I, H) &&
            map_pieces(&p.b, xq, (uint64_t)kXP * L.cap, H, kXP * kQR);
  DS_REQUIRE(ok, DS_ECUDA, "grouped_ffn: tensor map encoding failed (q3 gate/up)");
  p.sc[0] = static_cast<const __half*>(d->w1.scales);
  p.bi[0] = static_cast<const __half*>(d->w1.biases);
  p.sc[1] = static_cast<const __half*>(d->w3.scales);
  p.bi[1] = static_cast<const __half*>(d->w3.biases);
  p.sfb = sfx;
  p.asum = xs;
  const int grid_a = (int)std::min<int64_t>(sms, L.max_tiles * (I / 128));
  const int grid_b = (int)std::min<int64_t>(sms, L.max_tiles * (H / 128));
  const size_t sm_a = q3_smem<GATEUP>(H), sm_b = q3_smem<DOWN>(I);
  DS_CHECK_CUDA(cudaFuncSetAttribute(q3_gemm_kernel<GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_a));
  q3_gemm_kernel<GATEUP><<<grid_a, kQThreads, sm_a, s>>>(p);
  DS_CHECK_LAUNCH("q3_gemm_kernel<gate/up>");

  ok = map_codes(&p.w[0], d->w2.data, (uint64_t)E * H, I) && map_pieces(&p.b, hq, (uint64_t)kHP * L.cap, I, kHP * kQR);
  DS_REQUIRE(ok, DS_ECUDA, "grouped_ffn: tensor map encoding failed (q3 down)");
  p.w[1] = p.w[0];
  p.sc[0] = p.sc[1] = static_cast<const __half*>(d->w2.scales);
  p.bi[0] = p.bi[1] = static_cast<const __half*>(d->w2.biases);
  p.sfb = sfh;
  p.asum = hs;
  DS_CHECK_CUDA(cudaFuncSetAttribute(q3_gemm_kernel<DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_b));
  q3_gemm_kernel<DOWN><<<grid_b, kQThreads, sm_b, s>>>(p);
  DS_CHECK_LAUNCH("q3_gemm_kernel<down>");

  return launch_combine(y, pos, topk_w, ints, ints + 2, k, H, d->route_before_down ? 0 : 1, out, out_dtype, tokens,
                        s);
}

}  // namespace grouped
}  // namespace ds
