// Decode MoE layer (1..8 tokens, FP4 routed banks with prepared scale atoms,
// bf16 x, optional bf16 shared expert) on tcgen05 tensor cores.
//
// Same contract as the other decode kernels (moe_layer's expert loop,
// src/deepseeker/mlx_forward.py:388-419; shared add mlx_runner.py:776-781):
// for every distinct routed expert e (ascending id),
// h = silu(min(x W1e^T, L)) * clip(x W3e^T, +-L) * gate, out += h W2e^T; plus
// the shared expert, its output rounded to bf16 before the add.
//
// Launch chain (programmatic dependent launch between the kernels):
//   prep    : distinct experts of the batch ("slots", ascending), the gate of
//             every (slot, token), and x as six e2m1 pieces per token with
//             per-32 ue8m0 scales (each piece re-scaled to the block maximum
//             of the remaining residual: about 12-14 significant bits);
//   gate/up : persistent tcgen05 kernel over items of 64 KB of weights:
//             shared-expert tiles first (bf16, kind::f16, B = x itself -- no
//             dependency on prep, so they stream while prep runs), then the
//             routed FP4 tiles (kind::mxf4 block-scaled: A = the packed
//             weights as stored, B = the x pieces, one MMA row per piece);
//             every item is 128 weight rows x a K slice, its f32 partial sum
//             goes to a workspace slot;
//   h       : sums the K slices, applies SiLU/clamp/gate, writes h as six
//             e2m1 pieces (routed) or bf16 hi/lo (shared); it lets the down
//             launch be scheduled before it waits for gate/up;
//   down    : the same kernel over W2 tiles (its producer prefetches weight
//             stages before waiting for the previous grid);
//   combine : adds the slots in ascending expert order and the shared expert
//             rounded to bf16, writes bf16 rows.
//
// kind::mxf4 reads FP4 operands packed (two codes per byte) with the 128-byte
// swizzle, so the weights go from HBM to shared memory unchanged (128-byte
// TMA rows: 256 codes) and a stage of shared memory holds exactly its HBM
// bytes; the ring holds as many 40 KB stages as fit (5 for up to 2 tokens:
// 160 KB of weights in flight per SM).  A stage is freed only when its MMAs
// complete, so the ring's turnaround (TMA landing, scale staging, MMA issue
// and completion) sets the per-SM stream rate.  Roles per CTA: TMA producer,
// two single-thread MMA issuers (even / odd items, four accumulator buffers
// in tensor memory), four stager warps (scale atoms into tensor memory, one
// warp per lane quarter), four epilogue warps.  Every wait is bounded; a
// timeout sets kErrWaitTimeout and an abort flag that ends every role.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "moe_decode.cuh"
#include "ptx.cuh"
#include "route.cuh"
#include "tc5.cuh"

namespace ds {
namespace decode {
namespace {

using namespace ds::ptx;

constexpr int kThreads = 352;                  // 11 warps
constexpr int kMaxStages = 8;
constexpr int kAcc = 4;                        // accumulator buffers (64 tensor-memory columns each)
static_assert(64 * kAcc + 32 * kMaxStages <= 512, "accumulators + scale ring exceed tensor memory");
constexpr int kASlot = 32768;                  // 2 chunks x 128 rows x 128 B (FP4 K = 512 packed, or bf16 K = 128)
constexpr int kSfSlot = 4096;                  // 4 weight atoms + 4 activation atoms
constexpr int kAtom = 512;
constexpr int kPieces = 6;                     // e2m1 pieces per activation row
constexpr int kPieceRows = 8 * kPieces;        // piece rows per slot (8 tokens max)
constexpr int kStagesPerItem = 2;              // 64 KB of weights per item
constexpr int kMaxSlots5 = 64;
constexpr int kMaxT = 8;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr size_t kSmemMax = 225 * 1024;   // dynamic shared memory cap (leaves room for the static part)

enum { PH_GATEUP = 0, PH_DOWN = 1 };

// Workspace (byte offsets, 256-aligned; built on the host by t5_layout).
struct T5Layout {
  size_t ints, slot_expert, gate, xq, sfx, part_a, part_as, hq, sfh, hb, part_b, part_bs, total;
  int KPa, KPas, KPb, KPbs;  // K slices per item kind
};

struct T5Params {
  CUtensorMap w[2];   // routed packed FP4 (gate/up: W1, W3; down: W2 in w[0]), UINT8 {128 B, rows, K/256}
  CUtensorMap s[2];   // shared bf16 (gate/up: sW1, sW3; down: sW2), UINT8 {128 B, rows, 2K/128}
  CUtensorMap bq;     // routed B operand pieces (packed e2m1), UINT8 {128 B, rows, K/256}
  CUtensorMap bs;     // shared B operand bf16, UINT8 {128 B, rows, 2K/128}
  const uint8_t* sfa[2];      // weight scale atoms [E][rows/128][K/128][512]
  const uint8_t* sfb;         // B-operand scale atoms
  size_t sfb_slot_stride;     // bytes between slots of sfb (0: shared by all slots)
  const int32_t* slot_expert;
  const int32_t* n_slots;
  float* part;                // routed partials
  float* part_sh;             // shared partials
  int* err;
  int T, phase, n_sh_items;
  int rows_r, rows_s;         // output rows of a routed / shared matrix
  int K_r, K_s;               // input features of a routed / shared matrix
  int KP_r, KP_s;             // K slices per routed / shared item
  int N_r;                    // MMA N of routed items (piece rows rounded up to 16)
  int bq_rows_per_slot;       // rows of the routed B operand per slot (0 gate/up: x pieces shared)
  int nst;                    // stages in the ring
  int stage_bytes;            // A slot + B slot + scale slot
  int b_slot;                 // bytes of the B slot (N_r rows x 2 chunks x 128 B, >= 4 KB)
  const float* slot_gate;     // [kMaxSlots5][kMaxT]
  uint8_t* hq;                // gate/up output: routed h pieces [slot][48][I/2]
  uint8_t* sfh;               // gate/up output: their scale atoms [slot][I/128][512]
  __nv_bfloat16* hb;          // gate/up output: shared h hi/lo [16][Is]
  void* out;                  // down output [T][H]: bf16, or f32 when out_f32
  int out_f32;
  int sh_t0, sh_t1;           // output rows that receive the shared expert
  float* out_sh;              // non-null: shared expert sum [T][H] f32 goes here, unrounded
  float limit;
};

// Bounded wait: suspended try_waits (the thread resumes when the phase
// completes), an abort check and a %globaltimer limit between them.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      *abort = 1;
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_or_abort(bar, parity, abort, err) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok != 0;
}

struct Item {
  int shared, slot, m, rt, kp;
};

__device__ __forceinline__ Item decode_item(const T5Params& p, int idx) {
  Item it;
  const int mats = p.phase == PH_GATEUP ? 2 : 1;
  if (idx < p.n_sh_items) {
    const int RT = p.rows_s / 128;
    it.shared = 1;
    it.slot = 0;
    it.kp = idx % p.KP_s;
    idx /= p.KP_s;
    it.rt = idx % RT;
    it.m = idx / RT;
  } else {
    idx -= p.n_sh_items;
    const int RT = p.rows_r / 128;
    it.shared = 0;
    it.kp = idx % p.KP_r;
    idx /= p.KP_r;
    it.rt = idx % RT;
    idx /= RT;
    it.m = idx % mats;
    it.slot = idx / mats;
  }
  return it;
}

__device__ __forceinline__ float silu_glu(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

// ue8m0 byte of the scale that maps a block maximum `amax` into (3, 6] (the
// top of the e2m1 range): 2^(E-2) when the maximum's mantissa is <= 1.5,
// else 2^(E-1).  Zero blocks get scale 1.
__device__ __forceinline__ int e2m1_scale(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const int ef = (int)(b >> 23);
  if (ef == 0) return 127;
  const int s = (b & 0x7FFFFFu) <= 0x400000u ? ef - 2 : ef - 1;
  return min(max(s, 1), 253);
}
__device__ __forceinline__ float scale_of(int sfb) { return __uint_as_float((uint32_t)sfb << 23); }
__device__ __forceinline__ float inv_scale_of(int sfb) { return __uint_as_float((uint32_t)(254 - sfb) << 23); }
__device__ __forceinline__ int atom_off(int r, int kb) { return (r & 31) * 16 + (r >> 5) * 4 + kb; }

// ------------------------------------------------------------------ tails (one warp, 32 rows, kT tokens)
// Partial sums live in L2 ([...][rows][kT] f32); they are read with .cg loads
// in batches so that up to 32 are in flight per lane (one L2 round trip for
// the usual slice counts), and summed in slice order starting from 0.

// sa = sum_j a[j * stride + 0..kT), sb likewise, j < n.
template <int kT>
__device__ __forceinline__ void sum_two(const float* a, const float* b, size_t stride, int n, float (&sa)[kT],
                                        float (&sb)[kT]) {
  constexpr int kC = kT >= 16 ? 1 : 16 / kT;
#pragma unroll
  for (int t = 0; t < kT; ++t) sa[t] = sb[t] = 0.0f;
  for (int j0 = 0; j0 < n; j0 += kC) {
    float va[kC][kT], vb[kC][kT];
#pragma unroll
    for (int c = 0; c < kC; ++c)
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        const bool ok = j0 + c < n;
        va[c][t] = ok ? __ldcg(a + (size_t)(j0 + c) * stride + t) : 0.0f;
        vb[c][t] = ok ? __ldcg(b + (size_t)(j0 + c) * stride + t) : 0.0f;
      }
#pragma unroll
    for (int c = 0; c < kC; ++c)
      if (j0 + c < n) {
#pragma unroll
        for (int t = 0; t < kT; ++t) {
          sa[t] += va[c][t];
          sb[t] += vb[c][t];
        }
      }
  }
}

// h of one routed slot for rows r0 + lane of I (one 32-row block) as e2m1
// pieces: sums the K slices of the gate/up partials, SiLU/clamp, route gate.
template <int kT>
__device__ void tail_h_routed(const T5Params& p, int slot, int r0, int lane) {
  const int I = p.rows_r, KP = p.KP_r;
  const int i = r0 + lane;
  float g[kT], u[kT];
  sum_two<kT>(p.part + (((size_t)slot * 2 + 0) * KP * I + i) * kT, p.part + (((size_t)slot * 2 + 1) * KP * I + i) * kT,
              (size_t)I * kT, KP, g, u);
  uint8_t* hq = p.hq + (size_t)slot * kPieceRows * (I / 2);
  uint8_t* sf = p.sfh + ((size_t)slot * (I / 128) + r0 / 128) * kAtom;
  float gates[kT];   // the slot's gates, loaded together (uniform over the warp)
#pragma unroll
  for (int t = 0; t < kT; ++t) gates[t] = p.slot_gate[slot * kMaxT + t];
#pragma unroll 1
  for (int t = 0; t < kT; ++t) {
    const float gate = gates[t];
    if (gate == 0.0f) {
      // a token not routed to this slot: h = 0 exactly, i.e. zero codes in
      // every piece and the scale byte e2m1_scale(0) = 127
#pragma unroll 1
      for (int pc = 0; pc < kPieces; ++pc) {
        const int row = t * kPieces + pc;
        if ((lane & 1) == 0) hq[(size_t)row * (I / 2) + i / 2] = 0;
        if (lane == 0) sf[atom_off(row, (r0 & 127) >> 5)] = (uint8_t)127;
      }
      continue;
    }
    float r = silu_glu(g[t], u[t], p.limit) * gate;
#pragma unroll 1
    for (int pc = 0; pc < kPieces; ++pc) {
      // block maximum of |r| over the warp's 32 rows: one max-reduction of
      // the bits (non-negative floats order as their bits; NaN counts as 0,
      // as a maximum tree of fmaxf would skip it)
      const float ar = fabsf(r);
      const float am = __uint_as_float(__reduce_max_sync(0xffffffffu, ar == ar ? __float_as_uint(ar) : 0u));
      const int sc = e2m1_scale(am);
      const uint32_t code = tc5::f32x2_to_e2m1x2(r * inv_scale_of(sc), 0.0f) & 0xFu;
      float q0, q1;
      tc5::e2m1x2_to_f32x2(code, q0, q1);
      r = fmaf(-q0, scale_of(sc), r);
      const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
      const int row = t * kPieces + pc;
      if ((lane & 1) == 0) hq[(size_t)row * (I / 2) + i / 2] = (uint8_t)(code | (hi << 4));
      if (lane == 0) sf[atom_off(row, (r0 & 127) >> 5)] = (uint8_t)sc;
    }
  }
}

// Shared-expert h for rows r0 + lane of Is as bf16 hi/lo (rows 2t, 2t+1).
template <int kT>
__device__ void tail_h_shared(const T5Params& p, int r0, int lane) {
  const int Is = p.rows_s, KP = p.KP_s;
  const int i = r0 + lane;
  float g[kT], u[kT];
  sum_two<kT>(p.part_sh + (size_t)i * kT, p.part_sh + ((size_t)KP * Is + i) * kT, (size_t)Is * kT, KP, g, u);
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    // the shared expert always clamps at 10 (src/deepseeker/mlx_runner.py:776-781)
    const float h = silu_glu(g[t], u[t], 10.0f);
    const __nv_bfloat16 hi = __float2bfloat16_rn(h);
    p.hb[(size_t)(2 * t) * Is + i] = hi;
    p.hb[(size_t)(2 * t + 1) * Is + i] = __float2bfloat16_rn(h - __bfloat162float(hi));
  }
}

// Output rows r0 + lane of H: routed slots in ascending expert order (each
// slot's K slices summed in order, then added), then the shared expert's K
// slices summed and rounded to bf16.
template <int kT>
__device__ void tail_combine(const T5Params& p, int r0, int lane) {
  const int H = p.rows_r, KP = p.KP_r, KPs = p.n_sh_items ? p.KP_s : 0;
  const int h = r0 + lane;
  const int nr = *p.n_slots * KP, n = nr + KPs;
  // partial j: routed (slot j / KP, K slice j % KP) for j < nr, then the
  // shared K slices; both arrays have H * kT floats per slice
  const size_t stride = (size_t)H * kT;
  const float* pr = p.part + (size_t)h * kT;
  const float* ps = p.part_sh + (size_t)h * kT;
  constexpr int kC = kT >= 32 ? 1 : 32 / kT;
  float acc[kT], es[kT], sh[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) acc[t] = es[t] = sh[t] = 0.0f;
  int kp = 0;
  for (int j0 = 0; j0 < n; j0 += kC) {
    float v[kC][kT];
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      const int j = j0 + c;
      const float* src = j < nr ? pr + (size_t)j * stride : ps + (size_t)(j - nr) * stride;
#pragma unroll
      for (int t = 0; t < kT; ++t) v[c][t] = j < n ? __ldcg(src + t) : 0.0f;
    }
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      const int j = j0 + c;
      if (j < nr) {
#pragma unroll
        for (int t = 0; t < kT; ++t) es[t] = (kp == 0 ? 0.0f : es[t]) + v[c][t];
        if (++kp == KP) {
          kp = 0;
#pragma unroll
          for (int t = 0; t < kT; ++t) acc[t] += es[t];
        }
      } else if (j < n) {
#pragma unroll
        for (int t = 0; t < kT; ++t) sh[t] += v[c][t];
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    if (KPs && (p.out_sh != nullptr || (t >= p.sh_t0 && t < p.sh_t1))) {
      if (p.out_sh != nullptr) p.out_sh[(size_t)t * H + h] = sh[t];
      else acc[t] += __bfloat162float(__float2bfloat16_rn(sh[t]));
    }
    if (p.out_f32) static_cast<float*>(p.out)[(size_t)t * H + h] = acc[t];
    else static_cast<__nv_bfloat16*>(p.out)[(size_t)t * H + h] = __float2bfloat16_rn(acc[t]);
  }
}

// CALL(K) with K = the token count as a compile-time constant (1..8).
#define DS_T5_FOR_T(T, CALL)  \
  switch (T) {                \
    case 1: CALL(1); break;   \
    case 2: CALL(2); break;   \
    case 3: CALL(3); break;   \
    case 4: CALL(4); break;   \
    case 5: CALL(5); break;   \
    case 6: CALL(6); break;   \
    case 7: CALL(7); break;   \
    default: CALL(8); break;  \
  }

// ------------------------------------------------------------------ gate/up and down GEMM kernel

__global__ void __launch_bounds__(kThreads, 1) t5_gemm_kernel(const __grid_constant__ T5Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ring = smem;                          // nst x [A 32 KB][B b_slot][SF 4 KB]
  __shared__ __align__(8) uint64_t full[kMaxStages], staged[kMaxStages], empty[kMaxStages], accfull[kAcc], accempty[kAcc],
      done[2];
  const int S = p.nst;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&staged[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 4);
    }
    mbar_init(&done[0], 1);
    mbar_init(&done[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc5::alloc(&tmem_base, 512);
  __syncthreads();
  tc5::fence_after();
  const uint32_t tb = tmem_base;                 // D buffers at columns 0, 64, 128, 192; scale ring from 256
  const uint32_t tsf0 = tb + 64 * kAcc;          // 32 columns per stage
  volatile int* abort = &abort_flag;
  // the down phase consumes what the gate/up launch produced; its producer
  // first prefetches weight tiles, every other role waits right away
  if (p.phase == PH_DOWN && warp != 0) wait_prior_grid();
  // gate/up: shared items need nothing from prep; routed items do
  int n_items = p.n_sh_items;
  bool routed_known = false;
  auto know_routed = [&]() {
    if (!routed_known) {
      if (p.phase == PH_GATEUP || warp == 0) wait_prior_grid();
      const int mats = p.phase == PH_GATEUP ? 2 : 1;
      n_items = p.n_sh_items + *p.n_slots * mats * (p.rows_r / 128) * p.KP_r;
      routed_known = true;
    }
  };
  if (p.n_sh_items == 0 || (p.phase == PH_DOWN && warp != 0)) know_routed();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int g = 0;
      const uint64_t wpol = policy_evict_first();   // weights: read once per step
      // down: issue the weight half of the first stages of this CTA's shared
      // items before waiting for the gate/up grid; their activation halves
      // (h, produced by that grid) follow after the wait
      int pre = 0;
      if (p.phase == PH_DOWN) {
        for (int item = blockIdx.x; item < p.n_sh_items && pre < S; item += gridDim.x) {
          const Item it = decode_item(p, item);
          for (int j = 0; j < kStagesPerItem && pre < S; ++j, ++pre) {
            mbar_arrive_expect_tx(&full[pre], kASlot + 2 * 16 * 128);
            tma_load_3d_hint(ring + pre * p.stage_bytes, &p.s[it.m], 0, it.rt * 128,
                             2 * (it.kp * kStagesPerItem + j), &full[pre], wpol);
          }
        }
        know_routed();
      }
      for (int item = blockIdx.x;; item += gridDim.x) {
        if (item >= n_items) {
          know_routed();
          if (item >= n_items) break;
        }
        const Item it = decode_item(p, item);
        int e = 0;
        if (!it.shared) e = p.slot_expert[it.slot];
        for (int j = 0; j < kStagesPerItem; ++j, ++g) {
          const int s = g % S;
          if (g >= S && !wait_or_abort(&empty[s], ((g / S) - 1) & 1, abort, p.err)) goto drain;
          uint8_t* sa = ring + s * p.stage_bytes;
          uint8_t* sb = sa + kASlot;
          uint8_t* sf = sb + p.b_slot;
          const int kc = it.kp * kStagesPerItem + j;  // stage index along K (two 128-byte chunks each)
          if (it.shared) {
            if (g >= pre) {
              mbar_arrive_expect_tx(&full[s], kASlot + 2 * 16 * 128);
              tma_load_3d_hint(sa, &p.s[it.m], 0, it.rt * 128, 2 * kc, &full[s], wpol);
            }
            tma_load_3d(sb, &p.bs, 0, 0, 2 * kc, &full[s]);
          } else {
            mbar_arrive_expect_tx(&full[s], kASlot + 2 * p.N_r * 128 + kSfSlot);
            tma_load_3d_hint(sa, &p.w[it.m], 0, e * p.rows_r + it.rt * 128, 2 * kc, &full[s], wpol);
            tma_load_3d(sb, &p.bq, 0, it.slot * p.bq_rows_per_slot, 2 * kc, &full[s]);
            const int KC = p.K_r / 128;
            bulk_g2s_hint(sf, p.sfa[it.m] + (((size_t)e * (p.rows_r / 128) + it.rt) * KC + 4 * kc) * kAtom,
                          4 * kAtom, &full[s], wpol);
            bulk_g2s(sf + 4 * kAtom, p.sfb + it.slot * p.sfb_slot_stride + (size_t)(4 * kc) * kAtom, 4 * kAtom,
                     &full[s]);
          }
        }
      }
    drain:
      for (int j = g - S < 0 ? 0 : g - S; j < g; ++j) mbar_wait_bounded(&full[j % S], (j / S) & 1, 200000000ull);
    }
  } else if (warp == 1 || warp == 10) {
    // ---------------------------------------------------------------- MMA issuers
    // Two threads issue the MMAs, alternating items (warp 1: even local
    // items, warp 10: odd), so that one thread's waits and issue latency
    // overlap the other's MMAs in the tensor pipe.  Each item has its own
    // accumulator buffer (item % kAcc) and ring stages g = item * 2 + j.  A
    // thread starts waiting on stage g only after it has seen stage g - 3
    // staged (its previous item), and the stagers stage in ring order, so
    // with S >= 3 the slot's previous phase (stage g - S) has completed and
    // the parity wait cannot alias.  Each issuer warp runs its loop
    // warp-uniformly and one elected lane issues, with the descriptors
    // formed once per stage: a K step of 32 B adds 2 to the descriptor's
    // 16-byte address field (shared memory stays below 256 KB: no carry).
    {
      const int par = warp == 1 ? 0 : 1;
      int li = 0;
      const uint64_t ring_desc = tc5::sdesc_sw128(smem_u32(ring));
      const uint32_t idesc_sh = tc5::idesc_bf16(16);
      uint32_t idesc_r[2];
      idesc_r[0] = tc5::idesc_mxf4(p.N_r, 0);
      idesc_r[1] = tc5::idesc_mxf4(p.N_r, 2);
      const uint32_t bchunk16 = ((uint32_t)p.N_r * 128) >> 4;
      for (int item = blockIdx.x;; item += gridDim.x, ++li) {
        if (item >= n_items) {
          know_routed();
          if (item >= n_items) break;
        }
        if ((li & 1) != par) continue;
        const bool shared = item < p.n_sh_items;
        const int b = li % kAcc;
        if (li >= kAcc && !warp_wait(&accempty[b], ((li / kAcc) - 1) & 1, abort, p.err)) break;
        const uint32_t dacc = tb + b * 64;
        for (int j = 0; j < kStagesPerItem; ++j) {
          const int g = li * kStagesPerItem + j, s = g % S, ph = (g / S) & 1;
          if (!warp_wait(&staged[s], ph, abort, p.err)) goto mma_out;
          tc5::fence_after();
          if (elect_one()) {
            const uint64_t ad = ring_desc + (uint64_t)(((uint32_t)s * p.stage_bytes) >> 4);
            const uint64_t bd = ad + (uint64_t)(kASlot >> 4);
            const uint32_t tsf = tsf0 + s * 32;
            if (shared) {
#pragma unroll
              for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int sub = 0; sub < 4; ++sub)
                  tc5::mma_bf16(dacc, ad + (c * 16384 >> 4) + 2 * sub, bd + (c * 16 * 128 >> 4) + 2 * sub, idesc_sh,
                                (j | c | sub) != 0);
            } else {
              // each 128-byte row chunk = 256 codes = 4 MMAs of K = 64; scale word 2c + kk/2, byte pair kk%2
#pragma unroll
              for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  tc5::mma_mxf4(dacc, ad + (c * 16384 >> 4) + 2 * kk, bd + c * bchunk16 + 2 * kk, idesc_r[kk & 1],
                                tsf + 4 * (2 * c + (kk >> 1)), tsf + 16 + 4 * (2 * c + (kk >> 1)), (j | c | kk) != 0);
            }
            tc5::commit(&empty[s]);
          }
          __syncwarp();
        }
        if (elect_one()) tc5::commit(&accfull[b]);
        __syncwarp();
      }
    mma_out:
      if (elect_one()) {
        tc5::commit(&done[par]);
        mbar_wait_bounded(&done[par], 0, 1000000000ull);
      }
      __syncwarp();
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- stagers
    const int q = warp & 3;
    int s = 0, ph = 0;
    for (int item = blockIdx.x;; item += gridDim.x) {
      if (item >= n_items) {
        know_routed();
        if (item >= n_items) break;
      }
      const bool shared = item < p.n_sh_items;
      for (int j = 0; j < kStagesPerItem; ++j) {
        if (!warp_wait(&full[s], ph, abort, p.err)) goto st_out;
        if (!shared) {
          const uint4* sf = reinterpret_cast<const uint4*>(ring + s * p.stage_bytes + kASlot + p.b_slot);
          const uint32_t t = tc5::lane_quarter(tsf0 + s * 32, q);
#pragma unroll
          for (int a = 0; a < 8; ++a) {
            const uint4 v = sf[a * 32 + lane];
            tc5::st_x4(t + 4 * a, v.x, v.y, v.z, v.w);
          }
          tc5::wait_st();
        }
        tc5::fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&staged[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  st_out:;
  } else if (warp < 10) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    int li = 0;
    for (int item = blockIdx.x;; item += gridDim.x, ++li) {
      if (item >= n_items) {
        know_routed();
        if (item >= n_items) break;
      }
      const Item it = decode_item(p, item);
      const int b = li % kAcc;
      if (!warp_wait(&accfull[b], (li / kAcc) & 1, abort, p.err)) break;
      tc5::fence_after();
      const uint32_t dacc = tc5::lane_quarter(tb + b * 64, q);
      float v[48];
      tc5::ld_x16_nowait(dacc, *reinterpret_cast<float(*)[16]>(v));
      if (!it.shared && p.N_r > 16) tc5::ld_x16_nowait(dacc + 16, *reinterpret_cast<float(*)[16]>(v + 16));
      if (!it.shared && p.N_r > 32) tc5::ld_x16_nowait(dacc + 32, *reinterpret_cast<float(*)[16]>(v + 32));
      tc5::wait_ld();
      tc5::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[b]);
      const int row = it.rt * 128 + q * 32 + lane;
      const int T = p.T;
      if (it.shared) {
        float* dst = p.phase == PH_GATEUP
                         ? p.part_sh + (((size_t)it.m * p.KP_s + it.kp) * p.rows_s + row) * T
                         : p.part_sh + ((size_t)it.kp * p.rows_s + row) * T;
        for (int t = 0; t < T; ++t) dst[t] = p.phase == PH_GATEUP ? v[t] : v[2 * t] + v[2 * t + 1];
      } else {
        float* dst = p.phase == PH_GATEUP
                         ? p.part + ((((size_t)it.slot * 2 + it.m) * p.KP_r + it.kp) * p.rows_r + row) * T
                         : p.part + (((size_t)it.slot * p.KP_r + it.kp) * p.rows_r + row) * T;
        for (int t = 0; t < T; ++t) {
          float acc = 0.0f;
#pragma unroll
          for (int pc = 0; pc < kPieces; ++pc) acc += v[kPieces * t + pc];
          dst[t] = acc;
        }
      }

    }
  }
  tc5::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc5::fence_after();
    tc5::dealloc(tb, 512);
  }
}

// h between the two GEMM launches: one CTA per 128-row tile of one slot
// (the last grid row is the shared expert), one row per thread.  The down
// launch may be scheduled right away: it waits for this grid before it reads
// h, and its producer streams weights meanwhile.
__global__ void __launch_bounds__(128) t5_h_kernel(const __grid_constant__ T5Params p) {
  launch_dependents();
  wait_prior_grid();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * 128 + warp * 32;
  if (blockIdx.y == gridDim.y - 1) {
    if (p.n_sh_items && r0 < p.rows_s) {
#define DS_T5_CALL(K) tail_h_shared<K>(p, r0, lane)
      DS_T5_FOR_T(p.T, DS_T5_CALL)
#undef DS_T5_CALL
    }
  } else if ((int)blockIdx.y < *p.n_slots && r0 < p.rows_r) {
    const int slot = blockIdx.y;
#define DS_T5_CALL(K) tail_h_routed<K>(p, slot, r0, lane)
    DS_T5_FOR_T(p.T, DS_T5_CALL)
#undef DS_T5_CALL
  }
}

// Output rows after the down launch: one row per thread.
__global__ void __launch_bounds__(128) t5_combine_kernel(const __grid_constant__ T5Params p) {
  launch_dependents();
  wait_prior_grid();
  const int r0 = blockIdx.x * 128 + (threadIdx.x >> 5) * 32, lane = threadIdx.x & 31;
#define DS_T5_CALL(K) tail_combine<K>(p, r0, lane)
  DS_T5_FOR_T(p.T, DS_T5_CALL)
#undef DS_T5_CALL
}

// ------------------------------------------------------------------ prep: slots, gates, x pieces

struct PrepArgs {
  const __nv_bfloat16* x;
  const int32_t* ids;     // [T, k] routing (written here when the kernel routes)
  const float* gates;     // [T, k]
  // routing inside the kernel (template kRoutePer > 0): logits [T, E], the
  // score bias (or null), the router kind and scale
  const float* logits;
  const float* route_bias;
  int route_kind;
  float route_scale;
  int T, k, H, E;
  int32_t* n_slots;
  int32_t* slot_expert;   // [kMaxSlots5]
  float* slot_gate;       // [kMaxSlots5][kMaxT]
  uint8_t* xq;            // [48 piece rows][H/2] packed e2m1 (row t*6+p: piece p of token t)
  uint8_t* sfx;           // [H/128][512]
  int* err;
};

// Block 0 builds the slot list; blocks 1.. make the x pieces, in parallel.
// kRoutePer > 0: block 0 first routes the T tokens itself (warp t routes
// token t from its logits, ds::route::route_row_warp, with the router
// kernel's results bit for bit) and writes ids / gates for the caller;
// 0: it reads the caller's routing.
template <int kRoutePer>
__global__ void __launch_bounds__(256) t5_prep_kernel(PrepArgs a) {
  wait_prior_grid();
  launch_dependents();
  if (blockIdx.x == 0) {
    __shared__ int ids[kMaxEntries];
    __shared__ float gts[kMaxEntries];
    __shared__ uint32_t present[32];
    __shared__ int word_base[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n = a.T * a.k;
    if constexpr (kRoutePer > 0) {
      if (warp < a.T) {
        int e;
        float g;
        ds::route::route_row_warp<kRoutePer>(a.logits + (size_t)warp * a.E, a.route_bias, a.E, a.k, a.route_kind,
                                             a.route_scale, lane, e, g);
        if (lane < a.k) {
          ids[warp * a.k + lane] = e;
          gts[warp * a.k + lane] = g;
          const_cast<int32_t*>(a.ids)[warp * a.k + lane] = e;
          const_cast<float*>(a.gates)[warp * a.k + lane] = g;
        }
      }
    } else {
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        ids[j] = a.ids[j];
        gts[j] = a.gates[j];
      }
    }
    __syncthreads();
    if (warp != 0) return;
    // distinct valid experts, ascending; one warp, at most 128 entries, no
    // serial scan: a bitmap of the experts present (E <= 1024: 32 words),
    // a warp scan of its word counts gives every expert's slot, and each
    // entry writes its gate if it is its token's first slot for that expert
    present[lane] = 0u;
    __syncwarp();
    for (int j = lane; j < n; j += 32) {
      int e = ids[j];
      if (e >= a.E) {
        atomicOr(a.err, kErrExpertRange);
        e = -1;
      }
      ids[j] = e;
      if (e >= 0) atomicOr(&present[e >> 5], 1u << (e & 31));
    }
    __syncwarp();
    const uint32_t word = present[lane];
    int incl = __popc(word);
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    word_base[lane] = incl - __popc(word);
    const int count = __shfl_sync(0xffffffffu, incl, 31);
    for (uint32_t w = word; w; w &= w - 1) {
      const int b = __ffs(w) - 1;
      a.slot_expert[word_base[lane] + __popc(word & ((1u << b) - 1u))] = lane * 32 + b;
    }
    for (int q = lane; q < count * a.T; q += 32) a.slot_gate[(q / a.T) * kMaxT + q % a.T] = 0.0f;
    __syncwarp();
    for (int j = lane; j < n; j += 32) {
      const int e = ids[j];
      if (e < 0) continue;
      const int t = j / a.k, c = j % a.k;
      bool first_in_token = true;
      for (int c2 = 0; c2 < c; ++c2) first_in_token &= ids[t * a.k + c2] != e;
      if (!first_in_token) continue;
      const int rank = word_base[e >> 5] + __popc(present[e >> 5] & ((1u << (e & 31)) - 1u));
      a.slot_gate[rank * kMaxT + t] = gts[j];
    }
    if (lane == 0) *a.n_slots = count;
    return;
  }
  // x pieces (blocks 1..): 8 threads per (token, 32-block), 4 consecutive
  // elements each (the block maximum by three xor shuffles inside the
  // aligned 8-lane group); piece rows t * kPieces + p
  const int nb = a.H / 32;
  const int tid = (blockIdx.x - 1) * blockDim.x + threadIdx.x;
  for (int w = tid; w < a.T * nb * 8; w += (gridDim.x - 1) * blockDim.x) {
    const int grp = w >> 3, sub = w & 7;
    const int t = grp / nb, blk = grp % nb;
    float v[4];
    {
      const uint2 u = *reinterpret_cast<const uint2*>(a.x + (size_t)t * a.H + blk * 32 + sub * 4);
      v[0] = __uint_as_float(u.x << 16);
      v[1] = __uint_as_float(u.x & 0xFFFF0000u);
      v[2] = __uint_as_float(u.y << 16);
      v[3] = __uint_as_float(u.y & 0xFFFF0000u);
    }
    uint8_t* sf = a.sfx + (size_t)(blk / 4) * kAtom;
#pragma unroll 1
    for (int pc = 0; pc < kPieces; ++pc) {
      float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
      const int sc = e2m1_scale(am);
      const float inv = inv_scale_of(sc), scl = scale_of(sc);
      uint32_t half = 0;
#pragma unroll
      for (int c = 0; c < 4; c += 2) {
        const uint32_t b = tc5::f32x2_to_e2m1x2(v[c] * inv, v[c + 1] * inv);
        float q0, q1;
        tc5::e2m1x2_to_f32x2(b, q0, q1);
        v[c] = fmaf(-q0, scl, v[c]);
        v[c + 1] = fmaf(-q1, scl, v[c + 1]);
        half |= b << (4 * c);
      }
      const int row = t * kPieces + pc;
      *reinterpret_cast<uint16_t*>(a.xq + (size_t)row * (a.H / 2) + blk * 16 + sub * 2) = (uint16_t)half;
      if (sub == 0) sf[atom_off(row, blk & 3)] = (uint8_t)sc;
    }
  }
}

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn5() {
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

// Rows of `row_bytes` bytes viewed as {128 B, rows, row_bytes / 128}, box {128, box_rows, box_chunks}.
bool map3(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows,
          uint32_t box_chunks, bool swizzle) {
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {128, box_rows, box_chunks};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode_fn5()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Same with a row stride wider than the rows (a column slice of a matrix).
bool map3s(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint64_t stride_bytes,
           uint32_t box_rows, uint32_t box_chunks) {
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {stride_bytes, 128};
  const cuuint32_t box[3] = {128, box_rows, box_chunks};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode_fn5()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

// Tensor maps of one call that do not depend on x, cached by what they
// encode (bank pointers, geometry, workspace, tokens, slots): a layer keeps
// its banks and a decode loop its workspace, so steady state encodes only
// the x map.
struct MapSet {
  const void* key[12];
  int geo[8];
  CUtensorMap w1, w3, w2, sw1, sw3, sw2, xq, hq, hb;
};
constexpr int kMapCache = 32;
std::mutex g_map_mu;
MapSet g_maps[kMapCache];
int g_map_n = 0, g_map_next = 0;

bool same_key(const MapSet& m, const void* const* k, const int* geo) {
  return memcmp(m.key, k, sizeof(m.key)) == 0 && memcmp(m.geo, geo, sizeof(m.geo)) == 0;
}

T5Layout t5_layout(const DsMoeDesc& d, int T) {
  T5Layout L;
  const size_t H = d.hidden, I = d.inter, Is = d.shared_w1 ? d.shared_inter : 0;
  const int S = std::min<int>(T * d.top_k, d.n_experts);
  L.KPa = (int)(H / (512 * kStagesPerItem));
  L.KPas = (int)(H / (128 * kStagesPerItem));
  L.KPb = (int)(I / (512 * kStagesPerItem));
  L.KPbs = Is ? (int)(Is / (128 * kStagesPerItem)) : 0;
  size_t o = 0;
  L.ints = o;        o = kWsReserved;            // [0] error word, [1] slot count; reserved block
  L.slot_expert = o; o += up256(kMaxSlots5 * 4);
  L.gate = o;        o += up256(kMaxSlots5 * kMaxT * 4);
  L.xq = o;          o += up256(kPieceRows * H / 2);
  L.sfx = o;         o += up256((H / 128) * kAtom);
  L.part_a = o;      o += up256((size_t)S * 2 * L.KPa * I * T * 4);
  L.part_as = o;     o += up256((size_t)2 * L.KPas * Is * T * 4);
  L.hq = o;          o += up256((size_t)S * kPieceRows * I / 2);
  L.sfh = o;         o += up256((size_t)S * (I / 128) * kAtom);
  L.hb = o;          o += up256(16 * Is * 2);
  L.part_b = o;      o += up256((size_t)S * L.KPb * H * T * 4);
  L.part_bs = o;     o += up256((size_t)L.KPbs * H * T * 4);
  L.total = o;
  return L;
}

}  // namespace

bool t5_supported(const DecodeArgs& a) {
  const DsMoeDesc& d = a.d;
  if (a.x_f32 || d.w1.format != DS_FMT_FP4 || a.tokens < 1 || a.tokens > kMaxT) return false;
  if (!d.w1.scales_tc || !d.w3.scales_tc || !d.w2.scales_tc) return false;
  if (d.hidden % 1024 != 0 || d.inter % 1024 != 0) return false;
  if (d.top_k > 16 || a.max_slots > kMaxSlots5 || d.n_experts > 1024) return false;   // prep's 1024-bit expert map
  if ((uint64_t)d.n_experts * d.inter >= (1ull << 31) || (uint64_t)d.n_experts * d.hidden >= (1ull << 31)) return false;
  const bool sh = d.shared_w1 != nullptr;
  if (sh && (d.shared_inter % 256 != 0)) return false;
  if (!ds::aligned(a.x, 16) || !ds::aligned(d.w1.data, 16) || !ds::aligned(d.w3.data, 16) ||
      !ds::aligned(d.w2.data, 16) || !ds::aligned(d.w1.scales_tc, 16) || !ds::aligned(d.w3.scales_tc, 16) ||
      !ds::aligned(d.w2.scales_tc, 16))
    return false;
  if (sh && (!ds::aligned(d.shared_w1, 16) || !ds::aligned(d.shared_w3, 16) || !ds::aligned(d.shared_w2, 16)))
    return false;
  return encode_fn5() != nullptr;
}

size_t t5_workspace_bytes(const DsMoeDesc& d, int tokens) { return t5_layout(d, tokens).total; }

int launch_t5(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const DsMoeDesc& d = a.d;
  const int T = a.tokens, H = d.hidden, I = d.inter, E = d.n_experts;
  const bool sh = d.shared_w1 != nullptr;
  const int Is = sh ? d.shared_inter : 0;
  const T5Layout L = t5_layout(d, T);
  DS_REQUIRE(workspace_bytes >= L.total, DS_EINVAL, "moe_decode: workspace %zu bytes < %zu (tensor-core path)",
             workspace_bytes, L.total);
  char* ws = static_cast<char*>(workspace);
  int32_t* ints = reinterpret_cast<int32_t*>(ws + L.ints);   // [0] error bits, [1] n_slots
  int32_t* slot_expert = reinterpret_cast<int32_t*>(ws + L.slot_expert);
  float* slot_gate = reinterpret_cast<float*>(ws + L.gate);
  uint8_t* xq = reinterpret_cast<uint8_t*>(ws + L.xq);
  uint8_t* sfx = reinterpret_cast<uint8_t*>(ws + L.sfx);
  float* part_a = reinterpret_cast<float*>(ws + L.part_a);
  float* part_as = reinterpret_cast<float*>(ws + L.part_as);
  uint8_t* hq = reinterpret_cast<uint8_t*>(ws + L.hq);
  uint8_t* sfh = reinterpret_cast<uint8_t*>(ws + L.sfh);
  __nv_bfloat16* hb = reinterpret_cast<__nv_bfloat16*>(ws + L.hb);
  float* part_b = reinterpret_cast<float*>(ws + L.part_b);
  float* part_bs = reinterpret_cast<float*>(ws + L.part_bs);
  int* err = a.err;
  const int S = a.max_slots;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;

  // 1. prep
  PrepArgs pa;
  pa.x = static_cast<const __nv_bfloat16*>(a.x);
  pa.ids = a.ids;
  pa.gates = a.gates;
  pa.logits = a.logits;
  pa.route_bias = a.route_bias;
  pa.route_kind = a.route_kind;
  pa.route_scale = a.route_scale;
  pa.T = T;
  pa.k = d.top_k;
  pa.H = H;
  pa.E = E;
  pa.n_slots = ints + 1;
  pa.slot_expert = slot_expert;
  pa.slot_gate = slot_gate;
  pa.xq = xq;
  pa.sfx = sfx;
  pa.err = err;
  cfg.gridDim = dim3(1 + std::max(1, (T * (H / 4) + 255) / 256));   // slot-list block + piece blocks
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  if (!a.logits) {
    DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_prep_kernel<0>, pa));
  } else {
    const int per = (E + 31) / 32;     // experts per lane of a routing warp (E <= 1024)
    if (per <= 2) DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_prep_kernel<2>, pa));
    else if (per <= 4) DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_prep_kernel<4>, pa));
    else if (per <= 8) DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_prep_kernel<8>, pa));
    else if (per <= 16) DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_prep_kernel<16>, pa));
    else DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_prep_kernel<32>, pa));
  }

  // 2. gate/up
  T5Params p;
  memset(&p, 0, sizeof(p));
  const int NB = (kPieces * T + 15) / 16 * 16;   // piece rows of the batch, MMA N
  MapSet ms;
  {
    const void* key[12] = {d.w1.data, d.w3.data, d.w2.data, d.shared_w1, d.shared_w3, d.shared_w2,
                           workspace, nullptr, nullptr, nullptr, nullptr, nullptr};
    const int sh_ld = a.sh_w2_ld > 0 ? a.sh_w2_ld : Is;
    const int geo[8] = {H, I, E, Is, T, S, sh_ld, 0};
    int dev = 0;
    cudaGetDevice(&dev);
    key[7] = reinterpret_cast<const void*>((uintptr_t)dev + 1);
    std::lock_guard<std::mutex> lock(g_map_mu);
    int hit = -1;
    for (int i = 0; i < g_map_n; ++i)
      if (same_key(g_maps[i], key, geo)) hit = i;
    if (hit >= 0) {
      ms = g_maps[hit];
    } else {
      memset(&ms, 0, sizeof(ms));
      memcpy(ms.key, key, sizeof(key));
      memcpy(ms.geo, geo, sizeof(geo));
      bool ok = map3(&ms.w1, d.w1.data, (uint64_t)E * I, H / 2, 128, 2, true) &&
                map3(&ms.w3, d.w3.data, (uint64_t)E * I, H / 2, 128, 2, true) &&
                map3(&ms.w2, d.w2.data, (uint64_t)E * H, I / 2, 128, 2, true) &&
                map3(&ms.xq, xq, kPieceRows, H / 2, NB, 2, true) &&
                map3(&ms.hq, hq, (uint64_t)S * kPieceRows, I / 2, NB, 2, true) &&
                (!sh || (map3(&ms.sw1, d.shared_w1, Is, (uint64_t)H * 2, 128, 2, true) &&
                         map3(&ms.sw3, d.shared_w3, Is, (uint64_t)H * 2, 128, 2, true) &&
                         map3s(&ms.sw2, d.shared_w2, H, (uint64_t)Is * 2, (uint64_t)sh_ld * 2, 128, 2) &&
                         map3(&ms.hb, hb, 16, (uint64_t)Is * 2, 16, 2, true)));
      DS_REQUIRE(ok, DS_ECUDA, "moe_decode: tensor map encoding failed (tensor-core path)");
      const int slot = g_map_n < kMapCache ? g_map_n++ : (g_map_next++ % kMapCache);
      g_maps[slot] = ms;
    }
  }
  p.w[0] = ms.w1;
  p.w[1] = ms.w3;
  p.bq = ms.xq;
  if (sh) {
    p.s[0] = ms.sw1;
    p.s[1] = ms.sw3;
    DS_REQUIRE(map3(&p.bs, a.x, T, (uint64_t)H * 2, 16, 2, true), DS_ECUDA,
               "moe_decode: tensor map encoding failed (x)");
  }
  p.sfa[0] = static_cast<const uint8_t*>(d.w1.scales_tc);
  p.sfa[1] = static_cast<const uint8_t*>(d.w3.scales_tc);
  p.sfb = sfx;
  p.sfb_slot_stride = 0;
  p.slot_expert = slot_expert;
  p.n_slots = ints + 1;
  p.part = part_a;
  p.part_sh = part_as;
  p.err = err;
  p.T = T;
  p.phase = PH_GATEUP;
  p.rows_r = I;
  p.rows_s = Is;
  p.K_r = H;
  p.K_s = H;
  p.KP_r = L.KPa;
  p.KP_s = L.KPas;
  p.N_r = NB;
  p.bq_rows_per_slot = 0;
  p.b_slot = std::max(4096, NB * 2 * 128);
  p.stage_bytes = kASlot + p.b_slot + kSfSlot;
  p.nst = std::min<int>(kMaxStages, (int)((kSmemMax - 1024) / p.stage_bytes));
  DS_REQUIRE(p.nst >= 3, DS_ENOTSUP, "moe_decode: ring of %d stages (needs 3)", p.nst);
  const size_t smem = 1024 + (size_t)p.nst * p.stage_bytes;
  p.n_sh_items = sh ? 2 * (Is / 128) * L.KPas : 0;
  p.slot_gate = slot_gate;
  p.hq = hq;
  p.sfh = sfh;
  p.hb = hb;
  p.out = a.out;
  p.out_f32 = d.out_f32 ? 1 : 0;
  p.sh_t0 = a.sh_row0;
  p.sh_t1 = a.sh_row1;
  p.out_sh = a.out_sh;
  p.limit = d.swiglu_limit;
  static const cudaError_t attr_rc =
      cudaFuncSetAttribute(t5_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemMax);
  DS_CHECK_CUDA(attr_rc);
  cfg.gridDim = dim3(ds::sm_count());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_gemm_kernel, p));

  // 3. h
  cfg.gridDim = dim3(std::max(I, Is) / 128, S + 1);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_h_kernel, p));

  // 4. down
  T5Params q = p;
  q.w[0] = ms.w2;
  q.bq = ms.hq;
  if (sh) {
    q.s[0] = ms.sw2;
    q.bs = ms.hb;
  }
  q.sfa[0] = static_cast<const uint8_t*>(d.w2.scales_tc);
  q.sfa[1] = nullptr;
  q.sfb = sfh;
  q.sfb_slot_stride = (size_t)(I / 128) * kAtom;
  q.part = part_b;
  q.part_sh = part_bs;
  q.phase = PH_DOWN;
  q.rows_r = H;
  q.rows_s = H;
  q.K_r = I;
  q.K_s = Is;
  q.KP_r = L.KPb;
  q.KP_s = L.KPbs;
  q.N_r = NB;
  q.bq_rows_per_slot = kPieceRows;
  q.n_sh_items = sh ? (H / 128) * L.KPbs : 0;
  cfg.gridDim = dim3(ds::sm_count());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_gemm_kernel, q));

  // 5. combine
  cfg.gridDim = dim3(H / 128);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, t5_combine_kernel, q));

  return DS_OK;
}

}  // namespace decode
}  // namespace ds
