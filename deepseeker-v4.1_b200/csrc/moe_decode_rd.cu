// Single-token routed-expert MoE layer, register-dequant path: FP4 routed
// experts (checkpoint layout, no prepared scale atoms needed) + optional bf16
// shared expert, bf16 x, one token.  One cooperative persistent kernel per
// layer, one CTA per SM, every warp independent:
//
// Streaming.  A warp's unit of work is 16 weight rows x 4 K-groups of 128
// elements (4 KB of FP4 or bf16 weights).  Each lane loads 16 bytes of two
// rows per K-group straight from HBM into registers (coalesced 128-bit
// loads, L2 evict-first), two units in flight per warp (double buffer).  No
// shared-memory staging ring and no producer/consumer hand-off: the
// bytes-in-flight come from every warp issuing its next unit's loads before
// it computes the current one.
//
// Dot products.  FP4 codes become e4m3 bytes in registers with integer ops
// alone (code c -> ((c&7)<<2) | ((c&8)<<4), the value times 2^-6, exact for
// every code including the subnormal 0.5), the A fragments of mma.sync
// m16n8k32 e4m3 (f32 accumulate).  The B operand is the activation laid out
// so that column n of the 32x8 B tile only carries the K elements of lane
// group t = n, i.e. of ONE 32-element weight block: C[row][n] is then the dot
// product of that row with that block, and each block's ue8m0 scale (times
// the activation block's power-of-two scale) multiplies its own f32 partial.
// Dequant is exact, products are exact, accumulation is f32.  Activations
// enter as e4m3 pieces of a per-32-block power-of-two scaling: bf16 x as two
// pieces (exactly), the SwiGLU intermediate h as four (~16 significant bits,
// two MMA chains), in columns 0-3 / 4-7.  The shared expert's bf16 weights
// feed bf16 MMAs directly (x exact; its h as three bf16 pieces).
//
// Phase A (gate/up): tasks of 8 rows of W1 and the same 8 rows of W3 over the
//   full K (a routed expert), or over a K quarter (the shared expert, whose
//   rows are 4x wider); each CTA takes a contiguous range of tasks, so h of a
//   routed task is finished inside the CTA (SwiGLU clamps, route weight); the
//   four quarters of a shared task are summed by the CTA that finishes last,
//   and each 32-row block of a routed h is cut into its e4m3 pieces by the
//   CTA that delivers its last 8 rows (arrival counters), once for all CTAs.
// Grid barrier (bounded spin).  Before it, every CTA prefetches its phase-B
//   weights into L2 and issues its first phase-B unit's loads.
// Phase B (down + combine): each CTA owns a contiguous range of ~H/G output
//   rows: all routed slots' W2 rows and the shared W2 rows of that range, so
//   the combine (routed slots in ascending expert id, then the shared output
//   rounded to bf16, reference mlx_forward.py:388-419 / mlx_runner.py:776-781)
//   happens in the CTA with no further pass.
//
// Control words (grid barrier, shared-task counters) live in the workspace's
// reserved block [256, kWsReserved), where no path writes anything else; they
// must be zero before the first call and are left zero by every call that
// completes.  Every wait is bounded by %globaltimer (2 s); on expiry the
// kernel sets kErrWaitTimeout in the error word and stops waiting.
#include <cuda_fp8.h>

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
  float* h_r;         // [kMaxSlotsRd][I] f32
  uint8_t* hq8;       // [kMaxSlotsRd][I/32][4 pieces][32] e4m3 (piece byte order)
  float* hsc;         // [kMaxSlotsRd][I/32] scale of each block's pieces (incl. 2^6)
  float* h_s;         // [Is] f32
  __nv_bfloat16* hsp; // [3][Is] bf16 pieces of h_s
  float2* part_sh;    // [4][Is]
  unsigned* ctl;      // [0] arrive, [1] depart, [2 + pg] shared-task arrivals,
                      // [2 + Is/8 + slot*(I/32) + blk] routed h-block arrivals
  int* err;
  int H, I, E, Is, k;
  int out_f32;
  float limit;
  uint32_t smem_a_part, smem_b_hq, smem_b_hsc, smem_b_hsp, smem_b_part;  // byte offsets
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


// e4m3 bytes (value = e2m1 * 2^-6) of the low / high nibbles of the four
// bytes of w: code c -> sign (c & 8) << 4 | magnitude (c & 7) << 2.
__device__ __forceinline__ uint32_t fp4lo_e4m3(uint32_t w) {
  return ((w << 2) & 0x1C1C1C1Cu) | ((w << 4) & 0x80808080u);
}
__device__ __forceinline__ uint32_t fp4hi_e4m3(uint32_t w) {
  return ((w >> 2) & 0x1C1C1C1Cu) | (w & 0x80808080u);
}

// D += A(16x32, e4m3, row) * B(32x8, e4m3, col), f32 accumulate.
__device__ __forceinline__ void mma_e4m3(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Exponent bits of ue8m0 byte i (0..3) of w as an f32 (2^(b-127) for b in
// 1..254; byte 0 gives 0, byte 255 gives inf: a NaN-coded block makes the
// sums it enters non-finite).
__device__ __forceinline__ float ue8m0_lo(uint32_t w) { return __uint_as_float((w << 23) & 0x7F800000u); }
__device__ __forceinline__ float ue8m0_hi(uint32_t w) { return __uint_as_float((w << 15) & 0x7F800000u); }

// Byte position of element j (0..31) inside a 32-byte e4m3 piece: per group
// of eight elements, the four even ones then the four odd ones -- the order
// in which lane group t's B registers meet the low / high nibbles of a word.
__device__ __forceinline__ int piece_pos(int j) { return (j >> 3) * 8 + (j & 1) * 4 + ((j & 7) >> 1); }

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float from_e4m3(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3)));
}

// Element j of a 32-block (one per lane): scale the block so that its largest
// magnitude lands in [2^7, 2^8) and write `np` e4m3 pieces (each the
// rounding of what the earlier ones left) to dst[p * 32 + piece_pos(j)];
// returns the factor that undoes the scaling times 2^6 (the e2m1 -> e4m3
// offset of the weights).
__device__ __forceinline__ float split_e4m3(float v, int np, uint8_t* dst, int lane) {
  const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(v) & 0x7FFFFFFFu);
  int se = 0;
  if (m != 0u && m < 0x7F800000u) {
    const int e = m < 0x00800000u ? -127 : (int)(m >> 23) - 127;
    se = max(-120, min(120, 7 - e));
  }
  float r = v * __uint_as_float((uint32_t)(se + 127) << 23);
  const int pos = piece_pos(lane);
  for (int p = 0; p < np; ++p) {
    const uint8_t q = to_e4m3(r);
    dst[p * 32 + pos] = q;
    r -= from_e4m3(q);
  }
  return __uint_as_float((uint32_t)(6 - se + 127) << 23);
}

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

// FP4 group: decode the two rows' 32 + 32 codes into e4m3 A fragments, NCH
// chains of four MMAs against the lane's B sources bp[ch] (two accumulators
// for overlap), then this lane's two blocks' scales: acc0 / acc1 gather the
// partials of rows g / g + 8.  f0 / f1: activation scales of blocks blk0 and
// blk0 + 1 of the group.
template <int NCH>
__device__ __forceinline__ void fp4_group(const uint4 qa, const uint4 qb, uint32_t sa, uint32_t sb,
                                          const uint8_t* const (&bp)[NCH], float f0, float f1, int blk0,
                                          float& acc0, float& acc1) {
  const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
  const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
  uint32_t A[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    A[j][0] = fp4lo_e4m3(wa[j]);
    A[j][1] = fp4lo_e4m3(wb[j]);
    A[j][2] = fp4hi_e4m3(wa[j]);
    A[j][3] = fp4hi_e4m3(wb[j]);
  }
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    const uint4 q0 = lds128(bp[ch]), q1 = lds128(bp[ch] + 16);
    mma_e4m3(c0, A[0], q0.x, q0.y);
    mma_e4m3(c1, A[1], q0.z, q0.w);
    mma_e4m3(c0, A[2], q1.x, q1.y);
    mma_e4m3(c1, A[3], q1.z, q1.w);
  }
  sa >>= 8 * blk0;
  sb >>= 8 * blk0;
  acc0 = fmaf(c0[0] + c1[0], ue8m0_lo(sa) * f0, acc0);
  acc0 = fmaf(c0[1] + c1[1], ue8m0_hi(sa) * f1, acc0);
  acc1 = fmaf(c0[2] + c1[2], ue8m0_lo(sb) * f0, acc1);
  acc1 = fmaf(c0[3] + c1[3], ue8m0_hi(sb) * f1, acc1);
}

// bf16 chunk (32 elements of rows g and g + 8): two MMAs into c, B = xv.
__device__ __forceinline__ void bf16_chunk(const uint4 qa, const uint4 qb, const uint4 xv, float (&c)[4]) {
  const uint32_t a0[4] = {qa.x, qb.x, qa.y, qb.y};
  const uint32_t a1[4] = {qa.z, qb.z, qa.w, qb.w};
  mma_bf16(c, a0, xv.x, xv.y, c);
  mma_bf16(c, a1, xv.z, xv.w, c);
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

// ---------------------------------------------------------------- the kernel

struct Slots1 {
  int count;
  int expert[kMaxSlotsRd];
  float gate[kMaxSlotsRd];
};

__global__ void __launch_bounds__(kThreads, 1) rd_kernel(const RdParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ Slots1 slots;
  __shared__ int s_last[kMaxTasksPerCta];
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = gridDim.x, c = blockIdx.x;
  const int H = p.H, I = p.I, Is = p.Is;
  const bool has_sh = p.sw1 != nullptr;
  const uint64_t pol = policy_evict_first();

  unsigned char* zero = smem;                                     // kZeroBytes of zeros
  unsigned char* xb = smem + kZeroBytes;                          // x bf16 [H]
  unsigned char* xq = xb + 2 * H;                                 // x e4m3 [H/32][2 pieces][32]
  float* xsc = reinterpret_cast<float*>(xq + 2 * H);              // [H/32]
  float2* part_a = reinterpret_cast<float2*>(smem + p.smem_a_part);
  unsigned char* hq = smem + p.smem_b_hq;                         // [S][I/32][4][32] e4m3
  float* hsc = reinterpret_cast<float*>(smem + p.smem_b_hsc);     // [S][I/32]
  unsigned char* hsp = smem + p.smem_b_hsp;                       // [3][Is] bf16
  float* part_b = reinterpret_cast<float*>(smem + p.smem_b_part); // [units][16]

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
    }
    if (lane == 0) slots.count = __popc(firsts);
  }
  for (int b = warp; b < H / 32; b += kWarps) {
    const __nv_bfloat16 v = p.x[32 * b + lane];
    reinterpret_cast<__nv_bfloat16*>(xb)[32 * b + lane] = v;
    const float sc = split_e4m3(__bfloat162float(v), 2, xq + 64 * b, lane);   // bf16: two pieces are exact
    if (lane == 0) xsc[b] = sc;
  }
  __syncthreads();
  const int S = slots.count;

  // ---- phase A: task list [shared quarters][routed pair groups]
  const int upt = H / 512;                       // units per task
  const int n_sh = has_sh ? 4 * (Is / 8) : 0;
  const int n_rt = S * (I / 8);
  const int n_tasks = n_sh + n_rt;
  (void)n_tasks;
  // every CTA takes the same share of shared-expert tasks and of routed tasks
  // (the two kinds cost different compute per byte): local task tl < nsc is
  // shared task s0 + tl, the others routed task r0 + tl - nsc
  const int s0 = (int)((int64_t)c * n_sh / G), nsc = (int)((int64_t)(c + 1) * n_sh / G) - s0;
  const int r0 = (int)((int64_t)c * n_rt / G), nrc = (int)((int64_t)(c + 1) * n_rt / G) - r0;
  const int ntl = nsc + nrc;
  auto task_of = [&](int tl) { return tl < nsc ? s0 + tl : n_sh + r0 + (tl - nsc); };
  const int nua = ntl * upt;
  const uint8_t* my_zero = zero;

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
    const int tq = div_upt.div(u);
    const int task = task_of(tq), part = u - tq * upt;
    d.nkg = 4;
    if (task < n_sh) {
      const int pg = task >> 2, q = task & 3;
      const int row = 8 * pg + g;
      const int k0 = q * (H / 4) + part * 128;
      d.kind = kShared;
      d.kabs = k0;
      d.ra = p.sw1 + ((size_t)row * H + k0 + 8 * t) * 2;
      d.rb = p.sw3 + ((size_t)row * H + k0 + 8 * t) * 2;
    } else {
      const int rt = task - n_sh;
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
    // B sources: routed columns n = g' carry block t' = n & 3 of a group,
    // piece n >> 2 of x; the shared expert's column 0 carries x itself
    const bool rvalid = (g & 3) == t;
    const int rpiece = g >> 2;
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
          const uint8_t* bp[1] = {rvalid ? xq + (size_t)((4 * kga + t) * 2 + rpiece) * 32 : my_zero};
          const int blk0 = 2 * (t & 1);
          fp4_group<1>(f.a[kg], f.b[kg], f.sa[kg], f.sb[kg], bp, xsc[4 * kga + blk0], xsc[4 * kga + blk0 + 1],
                       blk0, acc0, acc1);
          load_slot(f, nxt, kg, pol);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
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

  // ---- phase A epilogue: h of every task of this CTA
  for (int i = tid; i < ntl * 8; i += kThreads) {
    const int tl = i >> 3, r = i & 7, task = task_of(tl);
    float G1 = 0.f, U1 = 0.f;
    for (int q = 0; q < upt; ++q) {
      const float2 v = part_a[(tl * upt + q) * 8 + r];
      G1 += v.x;
      U1 += v.y;
    }
    if (task < n_sh) {
      const int pg = task >> 2, qq = task & 3;
      p.part_sh[(size_t)qq * Is + 8 * pg + r] = make_float2(G1, U1);
    } else {
      const int rt = task - n_sh;
      const int s = rt / (I / 8), pg = rt - s * (I / 8);
      p.h_r[(size_t)s * I + 8 * pg + r] = silu_clamped(G1, U1, p.limit) * slots.gate[s];
    }
  }
  __syncthreads();
  // Arrivals: a shared pair group is complete with its fourth quarter, a
  // routed h block (32 rows) with its fourth pair group; the CTA that
  // completes one finishes it for everybody.
  unsigned* ctl_sh = p.ctl + 2;
  unsigned* ctl_blk = p.ctl + 2 + Is / 8;
  for (int tl = tid; tl < ntl; tl += kThreads) {
    const int task = task_of(tl);
    __threadfence();   // release this CTA's rows of the task (written before the barrier above)
    if (task < n_sh) {
      s_last[tl] = atomicAdd(&ctl_sh[task >> 2], 1u) == 3u;
    } else {
      const int rt = task - n_sh;
      const int sl = rt / (I / 8), pg = rt - sl * (I / 8);
      s_last[tl] = atomicAdd(&ctl_blk[sl * (I / 32) + (pg >> 2)], 1u) == 3u;
    }
  }
  __syncthreads();
  for (int tl = warp; tl < ntl; tl += kWarps) {
    if (!s_last[tl]) continue;
    __threadfence();   // acquire: the other CTAs' rows of this task
    const int task = task_of(tl);
    if (task < n_sh) {
      // shared pair group: h of its 8 rows from the four quarters, and its bf16 pieces
      const int pg = task >> 2;
      if (lane < 8) {
        float G1 = 0.f, U1 = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 v = __ldcg(&p.part_sh[(size_t)q * Is + 8 * pg + lane]);
          G1 += v.x;
          U1 += v.y;
        }
        const int row = 8 * pg + lane;
        const float h = silu_clamped(G1, U1, 10.0f);   // the shared expert always clamps at 10
        const __nv_bfloat16 hi = __float2bfloat16_rn(h);
        const float r1 = h - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        p.hsp[row] = hi;
        p.hsp[Is + row] = mid;
        p.hsp[2 * Is + row] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
        if (lane == 0) ctl_sh[pg] = 0u;
      }
    } else {
      // routed h block: four e4m3 pieces of its 32 values and their scale
      const int rt = task - n_sh;
      const int sl = rt / (I / 8), blk = (rt - sl * (I / 8)) >> 2;
      const size_t bi = (size_t)sl * (I / 32) + blk;
      const float v = __ldcg(&p.h_r[(size_t)sl * I + 32 * blk + lane]);
      const float sc = split_e4m3(v, 4, p.hq8 + bi * 128, lane);
      if (lane == 0) {
        p.hsc[bi] = sc;
        ctl_blk[bi] = 0u;
      }
    }
  }

  // ---- phase B geometry: output rows [n0, n1) of this CTA
  const int n0 = (int)((int64_t)c * H / G), n1 = (int)((int64_t)(c + 1) * H / G);
  const int nkgb = I / 128;
  const int ups = (nkgb + 3) / 4;                // routed units per (tile, slot)
  const int ush = has_sh ? Is / 128 : 0;         // shared units per tile (128-wide K slices)
  const int upt_b = S * ups + ush;               // units per tile
  const int ntiles = (n1 - n0 + 15) / 16;
  const int nub = ntiles * upt_b;

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

  // L2 prefetch of this CTA's phase-B weights, then its first units' loads
  if (tid < S) {
    const size_t e = slots.expert[tid];
    prefetch_l2(p.w2 + (e * H + n0) * (I / 2), (uint32_t)((n1 - n0) * (I / 2)));
    const size_t soff = (e * H + n0) * (I / 32), sbytes = (size_t)(n1 - n0) * (I / 32);
    if (soff % 16 == 0 && sbytes % 16 == 0) prefetch_l2(p.s2 + soff, (uint32_t)sbytes);
  } else if (tid == kMaxSlotsRd && has_sh) {
    prefetch_l2(p.sw2 + (size_t)n0 * Is * 2, (uint32_t)((size_t)(n1 - n0) * Is * 2));
  }
  Buf fb;
  Unit curb = unit_b(warp);
#pragma unroll
  for (int j = 0; j < 4; ++j) load_slot(fb, curb, j, pol);

  // ---- grid barrier (h of every CTA visible afterwards)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
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

  // ---- phase B prologue: the prepared activation pieces into shared memory
  {
    const int nq = S * (I / 32) * 128 / 16;
    const uint4* src = reinterpret_cast<const uint4*>(p.hq8);
    for (int i = tid; i < nq; i += kThreads) reinterpret_cast<uint4*>(hq)[i] = __ldcg(src + i);
    for (int i = tid; i < S * (I / 32); i += kThreads) hsc[i] = __ldcg(&p.hsc[i]);
    if (has_sh) {
      const uint4* s3 = reinterpret_cast<const uint4*>(p.hsp);
      for (int i = tid; i < 3 * Is * 2 / 16; i += kThreads) reinterpret_cast<uint4*>(hsp)[i] = __ldcg(s3 + i);
    }
  }
  __syncthreads();

  {
    // B sources: routed chain ch carries pieces 2ch (columns 0-3) and
    // 2ch + 1 (columns 4-7) of h; the shared expert's columns 0-2 its three
    // bf16 pieces
    const bool rvalid = (g & 3) == t;
    const int rpiece = g >> 2;
    for (int u = warp; u < nub; u += kWarps) {
      const Unit nxt = unit_b(u + kWarps);
      if (curb.kind == kRouted) {
        float acc0 = 0.f, acc1 = 0.f;
        const unsigned char* hbase = hq + (size_t)curb.slot * (I / 32) * 128;
        const float* sbase = hsc + (size_t)curb.slot * (I / 32);
#pragma unroll
        for (int kg = 0; kg < 4; ++kg) {
          if (kg < curb.nkg) {
            const int kga = curb.kabs + kg;
            const uint8_t* bp[2] = {rvalid ? hbase + (size_t)((4 * kga + t) * 4 + rpiece) * 32 : my_zero,
                                    rvalid ? hbase + (size_t)((4 * kga + t) * 4 + 2 + rpiece) * 32 : my_zero};
            const int blk0 = 2 * (t & 1);
            fp4_group<2>(fb.a[kg], fb.b[kg], fb.sa[kg], fb.sb[kg], bp, sbase[4 * kga + blk0],
                         sbase[4 * kga + blk0 + 1], blk0, acc0, acc1);
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
  size_t h_r, hq8, hsc, h_s, hsp, part_sh, ctl, total;
  uint32_t a_part, b_hq, b_hsc, b_hsp, b_part, smem;
};

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

RdLayout rd_layout(const DsMoeDesc& d) {
  RdLayout L;
  const size_t H = d.hidden, I = d.inter, Is = d.shared_w1 ? d.shared_inter : 0;
  const int S = std::min(d.top_k, d.n_experts);
  L.ctl = 256;   // control words in the reserved block after the error word
  size_t o = kWsReserved;
  L.h_r = o;     o += up256((size_t)kMaxSlotsRd * I * 4);
  L.hq8 = o;     o += up256((size_t)kMaxSlotsRd * (I / 32) * 128);
  L.hsc = o;     o += up256((size_t)kMaxSlotsRd * (I / 32) * 4);
  L.h_s = o;     o += up256(Is * 4 + 4);
  L.hsp = o;     o += up256(3 * Is * 2 + 16);
  L.part_sh = o; o += up256(4 * Is * 8 + 8);
  L.total = o;
  // shared memory (one union for phase A and phase B after the zero block)
  const int G = ds::sm_count();
  const int upt = (int)(H / 512);
  const int n_tasks = (Is ? 4 * (int)(Is / 8) : 0) + S * (int)(I / 8);
  const int tasks_cta = (n_tasks + G - 1) / G + 1;
  uint32_t a = kZeroBytes + 4 * (uint32_t)H + 4 * (uint32_t)(H / 32);
  a = (a + 15) / 16 * 16;
  L.a_part = a;
  a += (uint32_t)tasks_cta * upt * 8 * 8;
  uint32_t b = kZeroBytes;
  L.b_hq = b;
  b += (uint32_t)(S * (I / 32) * 128);
  L.b_hsc = b;
  b += (uint32_t)(S * (I / 32) * 4);
  b = (b + 15) / 16 * 16;
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
  if (!d.route_before_down) return false;
  if (a.out_sh != nullptr || a.sh_w2_ld != 0 || a.sh_row0 != 0 || a.sh_row1 != (1 << 30)) return false;
  if (d.hidden % 512 != 0 || d.inter % 128 != 0 || d.top_k > kMaxSlotsRd) return false;
  const bool sh = d.shared_w1 != nullptr;
  if (sh && d.shared_inter % 128 != 0) return false;
  const size_t words = 2 + (sh ? d.shared_inter / 8 : 0) +
                       (size_t)std::min(d.top_k, d.n_experts) * (d.inter / 32);
  if (256 + 4 * words > kWsReserved) return false;  // the control words fit the reserved block
  if (!ds::aligned(a.x, 16) || !ds::aligned(d.w1.data, 16) || !ds::aligned(d.w3.data, 16) ||
      !ds::aligned(d.w2.data, 16) || !ds::aligned(d.w1.scales, 4) || !ds::aligned(d.w3.scales, 4) ||
      !ds::aligned(d.w2.scales, 4))
    return false;
  if (sh && (!ds::aligned(d.shared_w1, 16) || !ds::aligned(d.shared_w3, 16) || !ds::aligned(d.shared_w2, 16)))
    return false;
  const RdLayout L = rd_layout(d);
  const int G = ds::sm_count();
  const int n_tasks = (sh ? 4 * (d.shared_inter / 8) : 0) + std::min(d.top_k, d.n_experts) * (d.inter / 8);
  if ((n_tasks + G - 1) / G + 1 > kMaxTasksPerCta) return false;
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
  p.h_r = reinterpret_cast<float*>(ws + L.h_r);
  p.hq8 = reinterpret_cast<uint8_t*>(ws + L.hq8);
  p.hsc = reinterpret_cast<float*>(ws + L.hsc);
  p.h_s = reinterpret_cast<float*>(ws + L.h_s);
  p.hsp = reinterpret_cast<__nv_bfloat16*>(ws + L.hsp);
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
  p.smem_b_hsc = L.b_hsc;
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
