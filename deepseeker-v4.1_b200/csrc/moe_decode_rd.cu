// Single-token routed-expert MoE layer, register-dequant path: FP4 routed
// experts (checkpoint layout, no prepared scale atoms needed) + optional bf16
// shared expert, bf16 x, one token, SwiGLU clamp on.  One cooperative
// persistent kernel per layer, one CTA per SM, every warp independent:
//
// Streaming.  A warp's unit of work is 16 weight rows x 4 K-groups of 128
// elements (4 KB of FP4) or 16 rows x 128 bf16 elements (4 KB).  Each lane
// loads 16 bytes of two rows per group straight from HBM into registers
// (coalesced 128-bit loads, L2 evict-first), and reloads each group's
// registers with the next unit's bytes as soon as it has consumed them, so
// every warp keeps about one unit in flight without a shared-memory ring.
//
// Dot products: mma.sync m16n8k16 f16 with f32 accumulate, A = the weights
// decoded in registers, B = the activation laid out so that column n of the
// 16x8 B tile only carries the K elements of lane group t = n, i.e. of ONE
// 32-element weight block: C[row][n] is the dot product of that row with
// that block, and each block's ue8m0 scale (times the activation block's
// power-of-two scale) multiplies its own f32 partial.  The FP4 decode is split
// between two units of the SM: one word of every four goes through the
// hardware e2m1 -> f16x2 conversion (exact values), the other three through
// integer ops (code c -> f16 bits sign << 15 | magnitude << 9, i.e. the value
// times 2^-14, exact for every code including the subnormal 0.5) into a
// second accumulator that is rescaled by 2^14.  Dequant and products are
// exact, accumulation is f32.  bf16 x enters as f16 scaled per 32-block by a
// power of two (exact); the SwiGLU intermediate h as an f16 hi + lo pair
// (~22 significant bits) scaled per slot from its bound |h| <= L max(L, 0.28) |gate|
// (columns 0-3 hi, 4-7 lo).  The shared expert's bf16 weights feed bf16 MMAs
// directly (x exact; its h as three bf16 pieces).
//
// Phase A (gate/up): tasks of 8 rows of W1 and the same 8 rows of W3 over the
//   full K (a routed expert), or over a K quarter (the shared expert, whose
//   rows are 4x wider); every CTA takes the same share of both kinds.  A
//   routed task finishes h for its 8 rows (clamps, route weight) and writes
//   them as MMA-ready pieces; a shared quarter writes its partial sums.  The
//   down projection's weights of this CTA are prefetched into L2 at the
//   start (the gate/up phase leaves HBM bandwidth to spare).
// Grid barrier (bounded spin).  Before it, every CTA issues its first
//   phase-B unit's loads.
// Phase B (down + combine): each CTA sums the shared quarters into h_s (its
//   bf16 pieces), then owns a contiguous range of ~H/G output rows: all
//   routed slots' W2 rows and the shared W2 rows of that range, so the
//   combine (routed slots in ascending expert id, then the shared output
//   rounded to bf16, reference mlx_forward.py:388-419 /
//   mlx_runner.py:776-781) happens in the CTA with no further pass.
//
// Control words (the grid barrier) live in the workspace's reserved block
// [256, kWsReserved), where no path writes anything else; they must be zero
// before the first call and are left zero by every call that completes.
// The barrier wait is bounded by %globaltimer (2 s); on expiry the kernel
// sets kErrWaitTimeout in the error word and stops waiting.
#include <algorithm>

#include "moe_decode.cuh"
#include "ptx.cuh"

namespace ds {
namespace decode {
namespace {

using namespace ds::ptx;

constexpr int kWarps = 16;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxSlotsRd = 32;
constexpr int kMaxTasksPerCta = 256;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kZeroBytes = 128;
constexpr int kCvtWords = 1;  // words (of four per 16-byte group) decoded by the conversion unit

struct RdParams {
  const uint8_t* w1;  // FP4 [E][I][H/2]
  const uint8_t* w3;
  const uint8_t* w2;  // FP4 [E][H][I/2]
  const uint8_t* s1;  // ue8m0 [E][I][H/32]
  const uint8_t* s3;
  const uint8_t* s2;  // ue8m0 [E][H][I/32]
  const uint8_t* sw1; // bf16 [Is][H] (null: no shared expert)
  const uint8_t* sw3;
  const uint8_t* sw2; // bf16 [H][Is]
  const __nv_bfloat16* x;
  const int32_t* ids;
  const float* gates;
  void* out;
  __half* hq;         // [kMaxSlotsRd][I/32][2 pieces][32] f16, element order of piece_pos16
  float2* part_sh;    // [4][Is] (gate, up) partial sums of the shared expert's K quarters
  unsigned* ctl;      // [0] arrive, [1] depart
  int* err;
  int H, I, E, Is, k;
  int out_f32;
  float limit;
  uint32_t smem_a_part, smem_b_hq, smem_b_hsp, smem_b_part;  // byte offsets
};

// ---------------------------------------------------------------- small helpers

__device__ __forceinline__ uint4 ldg_stream(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ uint32_t ldg_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ float silu_clamped(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

// 2^e as an f32 for e in [-126, 127]
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Exponent that maps a block whose largest magnitude has f32 bits m into
// [2^14, 2^15), f16's last full binade but one (0 for an all-zero or
// non-finite block).
__device__ __forceinline__ int f16_block_shift(uint32_t m) {
  if (m == 0u || m >= 0x7F800000u) return 0;
  const int e = m < 0x00800000u ? -127 : (int)(m >> 23) - 127;
  return max(-126, min(126, 14 - e));
}

// Exponent bits of ue8m0 byte 0 / byte 1 of w as an f32 (2^(b-127) for b in
// 1..254; byte 0 gives 0, byte 255 gives inf: a NaN-coded block makes the
// sums it enters non-finite).
__device__ __forceinline__ float ue8m0_lo(uint32_t w) { return __uint_as_float((w << 23) & 0x7F800000u); }
__device__ __forceinline__ float ue8m0_hi(uint32_t w) { return __uint_as_float((w << 15) & 0x7F800000u); }

// Integer decode of the eight e2m1 codes of w (nibble k = element k) into
// four f16x2 registers: P_k = (element k, element k + 4), each the code's
// value times 2^-14 (f16 bits sign << 15 | (e1 e0 m) << 9).
__device__ __forceinline__ void e2m1x8_to_f16x2_int(uint32_t w, uint32_t (&p)[4]) {
  p[0] = ((w << 9) & 0x0E000E00u) | ((w << 12) & 0x80008000u);
  p[1] = ((w << 5) & 0x0E000E00u) | ((w << 8) & 0x80008000u);
  p[2] = ((w << 1) & 0x0E000E00u) | ((w << 4) & 0x80008000u);
  p[3] = ((w >> 3) & 0x0E000E00u) | (w & 0x80008000u);
}

// Slot (in f16 units) of element e (0..31) of a block in an activation piece:
// per group of eight, the pair order in which that word's weight registers
// meet the K dimension -- natural order for words decoded by the conversion
// unit, (0, 4, 1, 5, 2, 6, 3, 7) for words decoded by integer ops.
__device__ __forceinline__ int piece_pos16(int e) {
  const int j = e >> 3, r = e & 7;
  return 8 * j + (j < kCvtWords ? r : 2 * (r & 3) + (r >> 2));
}

// x / d for small x by a multiply-high (m = ceil(2^32 / d)); exact for
// x < 2^32 / d, which holds for every index divided here.
struct FastDiv {
  uint32_t m;
  int d;
  __device__ __forceinline__ explicit FastDiv(int dd) : d(dd) {
    m = dd > 1 ? (uint32_t)(0xFFFFFFFFull / (uint64_t)dd + 1ull) : 0u;
  }
  __device__ __forceinline__ int div(int x) const { return d > 1 ? (int)__umulhi((uint32_t)x, m) : x; }
};

// ---------------------------------------------------------------- units

enum UnitKind : int { kShared = 0, kRouted = 1, kNone = 2 };

// One unit of a warp: 16 weight rows (lane (g, t) streams rows g and g + 8)
// x up to 4 K-groups of 128 elements (FP4) or 4 chunks of 32 elements (bf16).
struct Unit {
  int kind;
  const uint8_t* ra;   // this lane's 16 bytes of row g at the unit's first group (null: zeros)
  const uint8_t* rb;   // the same for row g + 8
  const uint8_t* sra;  // ue8m0 bytes of row g at the unit's first group (FP4)
  const uint8_t* srb;
  int nkg;             // groups in this unit: 1..4 (0: no unit)
  int kabs;            // FP4: absolute index of its first K-group; bf16: first element
  int slot;
  int idx;             // unit index inside the CTA (partial-sum slot)
};

// Weight registers: slot j holds group (FP4) or chunk (bf16) j of rows g and
// g + 8 and, for FP4, their four ue8m0 bytes of that group.
struct Buf {
  uint4 a[4], b[4];
  uint32_t sa[4], sb[4];
};

// Issue the loads of group j of unit u into slot j (zeros past the unit).
__device__ __forceinline__ void load_slot(Buf& f, const Unit& u, int j, uint64_t pol) {
  const bool on = j < u.nkg;
  f.a[j] = (on && u.ra) ? ldg_stream(u.ra + 64 * j, pol) : make_uint4(0u, 0u, 0u, 0u);
  f.b[j] = (on && u.rb) ? ldg_stream(u.rb + 64 * j, pol) : make_uint4(0u, 0u, 0u, 0u);
  const bool sc = on && u.kind == kRouted;
  f.sa[j] = (sc && u.ra) ? ldg_u32(u.sra + 4 * j) : 0x7F7F7F7Fu;
  f.sb[j] = (sc && u.rb) ? ldg_u32(u.srb + 4 * j) : 0x7F7F7F7Fu;
}

// FP4 group (this lane's 32-element block of rows g and g + 8): decode, eight
// MMAs against the lane's 64-byte B source bp (word j's activations at
// bp + 16 j), then this lane's two blocks' scales into acc0 / acc1 (rows g /
// g + 8).  f0 / f1: activation scales of blocks blk0 and blk0 + 1 of the
// group.  `scale` false: the lane's columns are empty (skip the scales, whose
// NaN code would otherwise turn 0 into NaN).
__device__ __forceinline__ void fp4_group(const uint4 qa, const uint4 qb, uint32_t sa, uint32_t sb,
                                          const uint8_t* bp, float f0, float f1, int blk0, bool scale,
                                          float& acc0, float& acc1) {
  const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
  const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
  float cx[4] = {0.f, 0.f, 0.f, 0.f};  // words decoded by the conversion unit: true values
  float cy[4] = {0.f, 0.f, 0.f, 0.f};  // words decoded by integer ops: values times 2^-14
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t pa[4], pb[4];
    if (j < kCvtWords) {
      e2m1x8_to_f16x2(wa[j], pa);
      e2m1x8_to_f16x2(wb[j], pb);
    } else {
      e2m1x8_to_f16x2_int(wa[j], pa);
      e2m1x8_to_f16x2_int(wb[j], pb);
    }
    const uint4 xv = lds128(bp + 16 * j);
    const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]};
    const uint32_t a1[4] = {pa[2], pb[2], pa[3], pb[3]};
    if (j < kCvtWords) {
      mma_f16(cx, a0, xv.x, xv.y, cx);
      mma_f16(cx, a1, xv.z, xv.w, cx);
    } else {
      mma_f16(cy, a0, xv.x, xv.y, cy);
      mma_f16(cy, a1, xv.z, xv.w, cy);
    }
  }
  if (scale) {
    sa >>= 8 * blk0;
    sb >>= 8 * blk0;
    acc0 = fmaf(fmaf(cy[0], 16384.0f, cx[0]), ue8m0_lo(sa) * f0, acc0);
    acc0 = fmaf(fmaf(cy[1], 16384.0f, cx[1]), ue8m0_hi(sa) * f1, acc0);
    acc1 = fmaf(fmaf(cy[2], 16384.0f, cx[2]), ue8m0_lo(sb) * f0, acc1);
    acc1 = fmaf(fmaf(cy[3], 16384.0f, cx[3]), ue8m0_hi(sb) * f1, acc1);
  }
}

// bf16 chunk (32 elements of rows g and g + 8): two MMAs into c, B = xv.
__device__ __forceinline__ void bf16_chunk(const uint4 qa, const uint4 qb, const uint4 xv, float (&c)[4]) {
  const uint32_t a0[4] = {qa.x, qb.x, qa.y, qb.y};
  const uint32_t a1[4] = {qa.z, qb.z, qa.w, qb.w};
  mma_bf16(c, a0, xv.x, xv.y, c);
  mma_bf16(c, a1, xv.z, xv.w, c);
}

// ---------------------------------------------------------------- the kernel

struct Slots1 {
  int count;
  int expert[kMaxSlotsRd];
  float gate[kMaxSlotsRd];
  float hmul[kMaxSlotsRd];  // power of two that puts the slot's |h| bound under 2^15
  float hdiv[kMaxSlotsRd];  // its inverse
};

__global__ void __launch_bounds__(kThreads, 1) rd_kernel(const RdParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ Slots1 slots;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = gridDim.x, c = blockIdx.x;
  const int H = p.H, I = p.I, Is = p.Is;
  const bool has_sh = p.sw1 != nullptr;
  const uint64_t pol = policy_evict_first();

  unsigned char* zero = smem;                                     // kZeroBytes of zeros
  unsigned char* xb = smem + kZeroBytes;                          // x bf16 [H]
  unsigned char* xq = xb + 2 * H;                                 // x f16 [H/32][32] (piece_pos16 order)
  float* xsc = reinterpret_cast<float*>(xq + 2 * H);              // [H/32]
  float2* part_a = reinterpret_cast<float2*>(smem + p.smem_a_part);
  unsigned char* hq = smem + p.smem_b_hq;                         // [S][I/32][2][32] f16
  unsigned char* hsp = smem + p.smem_b_hsp;                       // [3][Is] bf16
  float* part_b = reinterpret_cast<float*>(smem + p.smem_b_part); // [units][16]
  const uint8_t* my_zero = zero;

  // ---- prologue: slots (warp 0), x staging (all warps)
  if (tid < kZeroBytes / 4) reinterpret_cast<uint32_t*>(zero)[tid] = 0u;
  if (tid == 0) s_abort = 0;
  if (warp == 0) {
    int id = -1;
    float gt = 0.f;
    if (lane < p.k) {
      id = p.ids[lane];
      gt = p.gates[lane];
      if (id >= p.E) {
        atomicOr(p.err, kErrExpertRange);
        id = -1;
      }
      if (id < 0) id = -1;
    }
    const unsigned same = __match_any_sync(0xffffffffu, id);
    const bool first = id >= 0 && (__ffs(same) - 1) == lane;
    const unsigned firsts = __ballot_sync(0xffffffffu, first);
    int rank = 0;
    for (int j = 0; j < 32; ++j) {
      const int idj = __shfl_sync(0xffffffffu, id, j);
      rank += ((firsts >> j) & 1u) && idj < id;
    }
    if (first) {
      slots.expert[rank] = id;
      slots.gate[rank] = gt;
      // |h| <= L max(L, 0.28) |gate|: |silu(min(g, L))| <= max(L, 0.28), |clip(u)| <= L
      const float bound = p.limit * fmaxf(p.limit, 0.2785f) * gt;
      const int sh = f16_block_shift(__float_as_uint(bound) & 0x7FFFFFFFu);
      slots.hmul[rank] = exp2i(sh);
      slots.hdiv[rank] = exp2i(-sh);
    }
    if (lane == 0) slots.count = __popc(firsts);
  }
  for (int b = warp; b < H / 32; b += kWarps) {
    const __nv_bfloat16 v = p.x[32 * b + lane];
    reinterpret_cast<__nv_bfloat16*>(xb)[32 * b + lane] = v;
    const float f = __bfloat162float(v);
    const int se = f16_block_shift(__reduce_max_sync(0xffffffffu, __float_as_uint(f) & 0x7FFFFFFFu));
    reinterpret_cast<__half*>(xq)[32 * b + piece_pos16(lane)] = __float2half_rn(f * exp2i(se));
    if (lane == 0) xsc[b] = exp2i(-se);
  }
  __syncthreads();
  const int S = slots.count;

  // ---- phase B geometry (known now): output rows [n0, n1) of this CTA
  const int n0 = (int)((int64_t)c * H / G), n1 = (int)((int64_t)(c + 1) * H / G);
  const int nkgb = I / 128;
  const int ups = (nkgb + 3) / 4;                // routed units per (tile, slot)
  const int ush = has_sh ? Is / 128 : 0;         // shared units per tile (128-wide K slices)
  const int upt_b = S * ups + ush;               // units per tile
  const int ntiles = (n1 - n0 + 15) / 16;
  const int nub = ntiles * upt_b;

  // the down projection's weights of this CTA's rows into L2 while the
  // gate/up phase (compute-bound) leaves HBM bandwidth to spare
  if (tid < S) {
    const size_t e = slots.expert[tid];
    prefetch_l2(p.w2 + (e * H + n0) * (I / 2), (uint32_t)((n1 - n0) * (I / 2)));
    const size_t soff = (e * H + n0) * (I / 32), sbytes = (size_t)(n1 - n0) * (I / 32);
    if (soff % 16 == 0 && sbytes % 16 == 0) prefetch_l2(p.s2 + soff, (uint32_t)sbytes);
  } else if (tid == kMaxSlotsRd && has_sh) {
    prefetch_l2(p.sw2 + (size_t)n0 * Is * 2, (uint32_t)((size_t)(n1 - n0) * Is * 2));
  }

  // ---- phase A: every CTA takes the same share of shared-expert tasks and
  // of routed tasks (the two kinds cost different compute per byte): local
  // task tl < nsc is shared task s0 + tl, the others routed task r0 + tl - nsc
  const int upt = H / 512;                       // units per task
  const int n_sh = has_sh ? 4 * (Is / 8) : 0;
  const int n_rt = S * (I / 8);
  const int s0 = (int)((int64_t)c * n_sh / G), nsc = (int)((int64_t)(c + 1) * n_sh / G) - s0;
  const int r0 = (int)((int64_t)c * n_rt / G), nrc = (int)((int64_t)(c + 1) * n_rt / G) - r0;
  const int ntl = nsc + nrc;
  const int nua = ntl * upt;
  const FastDiv div_upt(upt), div_i8(I / 8);

  auto unit_a = [&](int u) -> Unit {
    Unit d;
    d.idx = u;
    d.slot = 0;
    d.ra = d.rb = d.sra = d.srb = nullptr;
    d.kind = kNone;
    d.nkg = 0;
    d.kabs = 0;
    if (u >= nua) return d;
    const int tl = div_upt.div(u), part = u - tl * upt;
    d.nkg = 4;
    if (tl < nsc) {
      const int task = s0 + tl;
      const int pg = task >> 2, q = task & 3;
      const int row = 8 * pg + g;
      const int k0 = q * (H / 4) + part * 128;
      d.kind = kShared;
      d.kabs = k0;
      d.ra = p.sw1 + ((size_t)row * H + k0 + 8 * t) * 2;
      d.rb = p.sw3 + ((size_t)row * H + k0 + 8 * t) * 2;
    } else {
      const int rt = r0 + tl - nsc;
      const int sl = div_i8.div(rt), pg = rt - sl * (I / 8);
      const size_t row = (size_t)slots.expert[sl] * I + 8 * pg + g;
      const int kg0 = part * 4;
      d.kind = kRouted;
      d.slot = sl;
      d.kabs = kg0;
      d.ra = p.w1 + row * (H / 2) + 64 * kg0 + 16 * t;
      d.rb = p.w3 + row * (H / 2) + 64 * kg0 + 16 * t;
      d.sra = p.s1 + row * (H / 32) + 4 * kg0;
      d.srb = p.s3 + row * (H / 32) + 4 * kg0;
    }
    return d;
  };

  // Walk this warp's units; group kg of the next unit is loaded into slot kg
  // as soon as the current unit has consumed it.
  {
    // B sources: routed column n = g' < 4 carries block n of a group (x has
    // one piece, columns 4-7 stay empty); the shared expert's column 0 x itself
    const bool rvalid = g == t;
    Buf f;
    Unit cur = unit_a(warp);
#pragma unroll
    for (int j = 0; j < 4; ++j) load_slot(f, cur, j, pol);
    for (int u = warp; u < nua; u += kWarps) {
      const Unit nxt = unit_a(u + kWarps);
      if (cur.kind == kRouted) {
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int kg = 0; kg < 4; ++kg) {
          const int kga = cur.kabs + kg;
          const int blk0 = 2 * (t & 1);
          fp4_group(f.a[kg], f.b[kg], f.sa[kg], f.sb[kg], rvalid ? xq + (size_t)(4 * kga + t) * 64 : my_zero,
                    xsc[4 * kga + blk0], xsc[4 * kga + blk0 + 1], blk0, t < 2, acc0, acc1);
          load_slot(f, nxt, kg, pol);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        if (t == 0) part_a[cur.idx * 8 + g] = make_float2(acc0, acc1);
      } else {
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
        const unsigned char* xsrc = (g == 0) ? xb + 2 * (cur.kabs + 8 * t) : my_zero;
        const int step = (g == 0) ? 64 : 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          bf16_chunk(f.a[j], f.b[j], lds128(xsrc + step * j), cc);
          load_slot(f, nxt, j, pol);
        }
        if (t == 0) part_a[cur.idx * 8 + g] = make_float2(cc[0], cc[2]);
      }
      cur = nxt;
    }
  }
  __syncthreads();

  // ---- phase A epilogue: routed h of every routed task (MMA-ready pieces),
  // partial sums of every shared quarter
  for (int i = tid; i < ntl * 8; i += kThreads) {
    const int tl = i >> 3, r = i & 7;
    float G1 = 0.f, U1 = 0.f;
    for (int q = 0; q < upt; ++q) {
      const float2 v = part_a[(tl * upt + q) * 8 + r];
      G1 += v.x;
      U1 += v.y;
    }
    if (tl < nsc) {
      const int task = s0 + tl;
      p.part_sh[(size_t)(task & 3) * Is + 8 * (task >> 2) + r] = make_float2(G1, U1);
    } else {
      const int rt = r0 + tl - nsc;
      const int sl = rt / (I / 8), pg = rt - sl * (I / 8);
      const float h = silu_clamped(G1, U1, p.limit) * slots.gate[sl] * slots.hmul[sl];
      const __half hi = __float2half_rn(h);
      const __half lo = __float2half_rn(h - __half2float(hi));
      __half* dst = p.hq + ((size_t)sl * (I / 32) + (pg >> 2)) * 64;
      const int pos = piece_pos16(8 * (pg & 3) + r);
      dst[pos] = hi;
      dst[32 + pos] = lo;
    }
  }

  // ---- phase B: first units' loads, then the grid barrier
  const FastDiv div_uptb(upt_b), div_ups(ups);
  auto unit_b = [&](int u) -> Unit {
    Unit d;
    d.idx = u;
    d.slot = 0;
    d.sra = d.srb = nullptr;
    d.ra = d.rb = nullptr;
    d.kind = kNone;
    d.nkg = 0;
    d.kabs = 0;
    if (u >= nub) return d;
    const int tile = div_uptb.div(u), r = u - tile * upt_b;
    const int row0 = n0 + 16 * tile + g, row1 = row0 + 8;
    if (r < S * ups) {
      const int sl = div_ups.div(r), kq = r - sl * ups;
      const int kg0 = 4 * kq;
      d.kind = kRouted;
      d.slot = sl;
      d.kabs = kg0;
      d.nkg = min(4, nkgb - kg0);
      const size_t e = slots.expert[sl];
      if (row0 < n1) {
        d.ra = p.w2 + (e * H + row0) * (I / 2) + 64 * kg0 + 16 * t;
        d.sra = p.s2 + (e * H + row0) * (I / 32) + 4 * kg0;
      }
      if (row1 < n1) {
        d.rb = p.w2 + (e * H + row1) * (I / 2) + 64 * kg0 + 16 * t;
        d.srb = p.s2 + (e * H + row1) * (I / 32) + 4 * kg0;
      }
    } else {
      const int k0 = (r - S * ups) * 128;
      d.kind = kShared;
      d.kabs = k0;
      d.nkg = 4;
      if (row0 < n1) d.ra = p.sw2 + ((size_t)row0 * Is + k0 + 8 * t) * 2;
      if (row1 < n1) d.rb = p.sw2 + ((size_t)row1 * Is + k0 + 8 * t) * 2;
    }
    return d;
  };
  Buf fb;
  Unit curb = unit_b(warp);
#pragma unroll
  for (int j = 0; j < 4; ++j) load_slot(fb, curb, j, pol);

  __syncthreads();
  if (tid == 0) {
    __threadfence();   // release this CTA's h pieces and shared partials
    atomicAdd(&p.ctl[0], 1u);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire(&p.ctl[0]) < (unsigned)G) {
      __nanosleep(64);
      if (globaltimer_ns() - t0 > kWaitNs) {
        atomicOr(p.err, kErrWaitTimeout);
        s_abort = 1;
        break;
      }
    }
    if (!s_abort && atomicAdd(&p.ctl[1], 1u) == (unsigned)G - 1u) {
      atomicExch(&p.ctl[0], 0u);
      atomicExch(&p.ctl[1], 0u);
    }
  }
  __syncthreads();
  if (s_abort) return;

  // ---- phase B prologue: routed h pieces into shared memory; the shared
  // expert's h from its four quarters, as three bf16 pieces
  {
    const int nq = S * (I / 32) * 128 / 16;
    const uint4* src = reinterpret_cast<const uint4*>(p.hq);
    for (int i = tid; i < nq; i += kThreads) reinterpret_cast<uint4*>(hq)[i] = __ldcg(src + i);
    if (has_sh) {
      __nv_bfloat16* d3 = reinterpret_cast<__nv_bfloat16*>(hsp);
      for (int i = tid; i < Is; i += kThreads) {
        float G1 = 0.f, U1 = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 v = __ldcg(&p.part_sh[(size_t)q * Is + i]);
          G1 += v.x;
          U1 += v.y;
        }
        const float h = silu_clamped(G1, U1, 10.0f);   // the shared expert always clamps at 10
        const __nv_bfloat16 hi = __float2bfloat16_rn(h);
        const float r1 = h - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        d3[i] = hi;
        d3[Is + i] = mid;
        d3[2 * Is + i] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
      }
    }
  }
  __syncthreads();

  {
    // B sources: routed column n = g' carries block n & 3 of a group, piece
    // n >> 2 (0: hi, 1: lo) of h; the shared expert's columns 0-2 its three
    // bf16 pieces
    const bool rvalid = (g & 3) == t;
    const int rpiece = g >> 2;
    for (int u = warp; u < nub; u += kWarps) {
      const Unit nxt = unit_b(u + kWarps);
      if (curb.kind == kRouted) {
        float acc0 = 0.f, acc1 = 0.f;
        const unsigned char* hbase = hq + (size_t)curb.slot * (I / 32) * 128;
        const float hs = slots.hdiv[curb.slot];
#pragma unroll
        for (int kg = 0; kg < 4; ++kg) {
          if (kg < curb.nkg) {
            const int kga = curb.kabs + kg;
            fp4_group(fb.a[kg], fb.b[kg], fb.sa[kg], fb.sb[kg],
                      rvalid ? hbase + (size_t)((4 * kga + t) * 2 + rpiece) * 64 : my_zero, hs, hs, 2 * (t & 1),
                      true, acc0, acc1);
          }
          load_slot(fb, nxt, kg, pol);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        if (t == 0) {
          part_b[curb.idx * 16 + g] = acc0;
          part_b[curb.idx * 16 + g + 8] = acc1;
        }
      } else {
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
        const bool bvalid = g < 3;
        const unsigned char* src = bvalid ? hsp + ((size_t)g * Is + curb.kabs + 8 * t) * 2 : my_zero;
        const int step = bvalid ? 64 : 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          bf16_chunk(fb.a[j], fb.b[j], lds128(src + step * j), cc);
          load_slot(fb, nxt, j, pol);
        }
        float v0 = cc[0] + cc[1], v1 = cc[2] + cc[3];
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        if (t == 0) {
          part_b[curb.idx * 16 + g] = v0;
          part_b[curb.idx * 16 + g + 8] = v1;
        }
      }
      curb = nxt;
    }
  }
  __syncthreads();

  // ---- combine: routed slots in ascending expert id, then the shared expert
  for (int n = n0 + tid; n < n1; n += kThreads) {
    const int tile = (n - n0) >> 4, rr = (n - n0) & 15;
    const float* pb = part_b + (size_t)tile * upt_b * 16 + rr;
    float routed = 0.f;
    for (int s = 0; s < S; ++s) {
      float v = 0.f;
      for (int q = 0; q < ups; ++q) v += pb[(s * ups + q) * 16];
      routed += v;
    }
    float sh = 0.f;
    for (int q = 0; q < ush; ++q) sh += pb[(S * ups + q) * 16];
    if (has_sh) routed += __bfloat162float(__float2bfloat16_rn(sh));
    if (p.out_f32)
      static_cast<float*>(p.out)[n] = routed;
    else
      static_cast<__nv_bfloat16*>(p.out)[n] = __float2bfloat16_rn(routed);
  }
}

struct RdLayout {
  size_t hq, part_sh, ctl, total;
  uint32_t a_part, b_hq, b_hsp, b_part, smem;
};

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

RdLayout rd_layout(const DsMoeDesc& d) {
  RdLayout L;
  const size_t H = d.hidden, I = d.inter, Is = d.shared_w1 ? d.shared_inter : 0;
  const int S = std::min(d.top_k, d.n_experts);
  L.ctl = 256;   // grid-barrier words in the reserved block after the error word
  size_t o = kWsReserved;
  L.hq = o;      o += up256((size_t)kMaxSlotsRd * (I / 32) * 128);
  L.part_sh = o; o += up256(4 * Is * 8 + 8);
  L.total = o;
  // shared memory (one union for phase A and phase B after the zero block)
  const int G = ds::sm_count();
  const int upt = (int)(H / 512);
  const int n_sh = Is ? 4 * (int)(Is / 8) : 0, n_rt = S * (int)(I / 8);
  const int tasks_cta = (n_sh + G - 1) / G + (n_rt + G - 1) / G;
  uint32_t a = kZeroBytes + 4 * (uint32_t)H + 4 * (uint32_t)(H / 32);
  a = (a + 15) / 16 * 16;
  L.a_part = a;
  a += (uint32_t)tasks_cta * upt * 8 * 8;
  uint32_t b = kZeroBytes;
  L.b_hq = b;
  b += (uint32_t)(S * (I / 32) * 128);
  L.b_hsp = b;
  b += (uint32_t)(3 * Is * 2);
  b = (b + 15) / 16 * 16;
  L.b_part = b;
  const int rows_cta = (int)((H + G - 1) / G) + 1;
  const int ntiles = (rows_cta + 15) / 16;
  const int ups = (int)((I / 128 + 3) / 4);
  b += (uint32_t)(ntiles * (S * ups + (Is ? (int)(Is / 128) : 0)) * 16 * 4);
  L.smem = std::max(a, b);
  return L;
}

}  // namespace

bool rd_supported(const DecodeArgs& a) {
  const DsMoeDesc& d = a.d;
  if (a.x_f32 || a.tokens != 1 || d.w1.format != DS_FMT_FP4) return false;
  if (!d.route_before_down || !(d.swiglu_limit > 0.0f)) return false;   // h scale from the clamp bound
  if (a.out_sh != nullptr || a.sh_w2_ld != 0 || a.sh_row0 != 0 || a.sh_row1 != (1 << 30)) return false;
  if (d.hidden % 512 != 0 || d.inter % 128 != 0 || d.top_k > kMaxSlotsRd) return false;
  const bool sh = d.shared_w1 != nullptr;
  if (sh && d.shared_inter % 128 != 0) return false;
  if (!ds::aligned(a.x, 16) || !ds::aligned(d.w1.data, 16) || !ds::aligned(d.w3.data, 16) ||
      !ds::aligned(d.w2.data, 16) || !ds::aligned(d.w1.scales, 4) || !ds::aligned(d.w3.scales, 4) ||
      !ds::aligned(d.w2.scales, 4))
    return false;
  if (sh && (!ds::aligned(d.shared_w1, 16) || !ds::aligned(d.shared_w3, 16) || !ds::aligned(d.shared_w2, 16)))
    return false;
  const RdLayout L = rd_layout(d);
  const int G = ds::sm_count();
  const int n_sh = sh ? 4 * (d.shared_inter / 8) : 0, n_rt = std::min(d.top_k, d.n_experts) * (d.inter / 8);
  if ((n_sh + G - 1) / G + (n_rt + G - 1) / G > kMaxTasksPerCta) return false;
  if (d.hidden < G) return false;   // every CTA owns at least one output row
  return L.smem <= 200 * 1024;
}

size_t rd_workspace_bytes(const DsMoeDesc& d) { return rd_layout(d).total; }

size_t rd_control_bytes(const DsMoeDesc&) { return kWsReserved; }

int launch_rd(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const DsMoeDesc& d = a.d;
  const RdLayout L = rd_layout(d);
  DS_REQUIRE(workspace_bytes >= L.total, DS_EINVAL, "moe_decode: workspace %zu bytes < %zu (register-dequant path)",
             workspace_bytes, L.total);
  char* ws = static_cast<char*>(workspace);
  RdParams p;
  p.w1 = static_cast<const uint8_t*>(d.w1.data);
  p.w3 = static_cast<const uint8_t*>(d.w3.data);
  p.w2 = static_cast<const uint8_t*>(d.w2.data);
  p.s1 = static_cast<const uint8_t*>(d.w1.scales);
  p.s3 = static_cast<const uint8_t*>(d.w3.scales);
  p.s2 = static_cast<const uint8_t*>(d.w2.scales);
  const bool sh = d.shared_w1 != nullptr;
  p.sw1 = sh ? static_cast<const uint8_t*>(d.shared_w1) : nullptr;
  p.sw3 = sh ? static_cast<const uint8_t*>(d.shared_w3) : nullptr;
  p.sw2 = sh ? static_cast<const uint8_t*>(d.shared_w2) : nullptr;
  p.x = static_cast<const __nv_bfloat16*>(a.x);
  p.ids = a.ids;
  p.gates = a.gates;
  p.out = a.out;
  p.hq = reinterpret_cast<__half*>(ws + L.hq);
  p.part_sh = reinterpret_cast<float2*>(ws + L.part_sh);
  p.ctl = reinterpret_cast<unsigned*>(ws + L.ctl);
  p.err = a.err;
  p.H = d.hidden;
  p.I = d.inter;
  p.E = d.n_experts;
  p.Is = sh ? d.shared_inter : 0;
  p.k = d.top_k;
  p.out_f32 = d.out_f32 ? 1 : 0;
  p.limit = d.swiglu_limit;
  p.smem_a_part = L.a_part;
  p.smem_b_hq = L.b_hq;
  p.smem_b_hsp = L.b_hsp;
  p.smem_b_part = L.b_part;
  static const cudaError_t attr_rc =
      cudaFuncSetAttribute(rd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  DS_CHECK_CUDA(attr_rc);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ds::sm_count());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, rd_kernel, p));
  return DS_OK;
}

}  // namespace decode
}  // namespace ds
