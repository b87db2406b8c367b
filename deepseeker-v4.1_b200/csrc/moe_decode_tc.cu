// Single-token (B = 1) routed-expert MoE layer: warp-specialised, TMA
// pipelined, tensor-core decode.  FP4 routed experts (checkpoint layout) +
// optional bf16 shared expert; geometry checked by tc_supported(), everything
// else goes to the generic path in moe_decode.cu.
//
// Both kernels are persistent (one CTA per SM, 1 + 16 warps):
//   warp 0, lane 0   producer: streams weight tiles HBM -> shared memory with
//                    tiled TMA tensor copies into a ring of stages (mbarrier
//                    full/empty handshake).  FP4 rows arrive as one 3-D box
//                    [128 B][rows][K/256 chunks] per matrix with the 128-byte
//                    swizzle, so a whole 8- or 16-row tile is one copy and the
//                    consumers' fragment reads are bank-conflict free.  (The
//                    bulk-copy unit costs ~100 cycles per copy, so per-row
//                    copies cannot reach HBM bandwidth; one box per matrix can.)
//   warps 1..16      consumers: each owns a K slice of the current tile,
//                    decodes e2m1 codes straight into mma.sync A fragments
//                    (cvt.rn.f16x2.e2m1x2; low nibble = even element), runs
//                    m16n8k16 with the activations as the B fragment and
//                    applies the ue8m0 block scale per 32-element block on the
//                    f32 accumulator.  A cross-warp reduction finishes a unit.
//
// Kernel A (gate/up): tile = 8 rows of W1 + the same 8 rows of W3 of one
//   routed expert (m16 rows 0-7 gate, 8-15 up), full K; or a 1024-wide K
//   slice of 8+8 shared-expert rows.  x is staged once per CTA as f16 scaled
//   by an exact power of two (x is bf16: 8 significant bits, so its products
//   with e2m1 values are exact in f32) and as raw bf16 for the shared expert.
//   Epilogue: h = silu(min(g, L)) * clip(u, -L, L) * gate, stored in f32.
// Kernel B (down + combine): unit = 16 output rows; tiles = pairs of routed
//   slots (16 rows of W2 each, full K = I) then 1024-wide K slices of the
//   shared W2.  h is staged per CTA as f16 hi + lo (routed, power-of-two
//   scaled) and bf16 hi + lo (shared); hi and lo ride in B-fragment columns 0
//   and 1 of the same MMA, so the split costs no extra tensor-core work and h
//   keeps ~22 (16) significant bits.  out = bf16(routed + f32(bf16(shared)))
//   as in the reference (src/deepseeker/mlx_forward.py:409-419).
//
// Launch chain on the stream: router -> A -> B with programmatic dependent
// launch: A's shared-expert tiles stream while the router runs; A lets B start
// once routing is resolved, and B streams W2 tiles while A finishes (B's
// consumers wait for A's h with griddepcontrol.wait).
//
// Every wait is bounded (2 s of %globaltimer); on expiry the kernel records
// kErrWaitTimeout in the workspace error word and stops.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <mutex>
#include <unordered_map>

#include "moe_decode.cuh"
#include "ptx.cuh"

namespace ds {
namespace decode {
namespace {

using namespace ds::ptx;

constexpr int kCW = 16;                     // consumer warps
constexpr int kThreads = 32 * (kCW + 1);    // 544
constexpr int kConsumerThreads = 32 * kCW;  // 512
constexpr int kMaxStages = 8;
constexpr int kKTile = 1024;                // bf16 K slice per shared tile (2048 B)
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kMaxSlots = 32;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kRing = 8;                    // reduction buffers in flight (> stages + 1)
constexpr int kRedBytesA = kRing * kCW * 8 * 8;   // [ring][warp][row 0..7] float2 (gate, up)
constexpr int kRedBytesB = kRing * kCW * 8 * 16;  // [ring][warp][row 0..7] float4

struct Geo {
  int H, I, Is, shared, max_slots;
  // kernel A (tile: 8 + 8 rows)
  uint32_t a_data, a_scales, a_stage;  // bytes of one data box, one scale box, stage stride
  int a_stages;
  uint32_t a_x16_off, a_xb_off, a_red_off, a_total;
  // kernel B (tile: 2 slots x 16 rows)
  uint32_t b_data, b_scales, b_stage;
  int b_stages;
  uint32_t b_hh_off, b_hl_off, b_sh_off, b_red_off, b_total;
};

struct alignas(64) TcParams {
  CUtensorMap w1d, w3d, w1s, w3s, sw1, sw3;  // kernel A
  CUtensorMap w2d, w2s, sw2;                 // kernel B
  DecodeArgs a;
  Geo g;
};

struct SlotInfo {
  int count;
  int expert[kMaxSlots];
  float gate[kMaxSlots];
};

// Distinct routed experts of the single token in ascending id, each with the
// gate of its first slot (src/deepseeker/mlx_forward.py:394-404).  Executed by
// a whole warp (top_k <= 32): one load per lane, duplicates found with
// __match_any_sync, ranks by counting smaller distinct ids.
__device__ void build_slots_warp(const DecodeArgs& a, SlotInfo& s, int lane) {
  const int k = a.d.top_k;
  int id = -1;
  float gt = 0.f;
  if (lane < k) {
    id = a.ids[lane];
    gt = a.gates[lane];
    if (id >= a.d.n_experts) {
      atomicOr(a.err, kErrExpertRange);
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
    s.expert[rank] = id;
    s.gate[rank] = gt;
  }
  if (lane == 0) s.count = __popc(firsts);
  __syncwarp();
}

__device__ __forceinline__ float silu_glu(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u);
}

// ------------------------------------------------------------------ work lists

// Kernel A items of CTA b.  Shared units (8+8 rows, KTs K-slices each) go
// round-robin first; routed units (one tile each) first top up the CTAs that
// got one shared unit fewer, then go round-robin, so per-CTA tile counts
// differ by at most one.
struct ListA {
  int G, b, KTs, Us, ups, rem, ns, Ur, p1, p2;
  __device__ void init(int G_, int b_, int KTs_, int Us_, int ups_) {
    G = G_, b = b_, KTs = KTs_, Us = Us_, ups = ups_;
    rem = Us % G;
    ns = KTs * (Us > b ? (Us - b + G - 1) / G : 0);
    Ur = p1 = p2 = 0;
  }
  __device__ void set_routed(int D) {
    Ur = D * ups;
    p1 = 0;
    if (b >= rem) {
      const int lo = KTs * (b - rem);
      p1 = max(0, min(KTs, Ur - lo));
    }
    const int start = KTs * (G - rem) + b;
    p2 = Ur > start ? (Ur - start + G - 1) / G : 0;
  }
  __device__ int total() const { return ns + p1 + p2; }
  // kind 0 = shared (unit x, K slice y), 1 = routed (slot x, row block y)
  __device__ void at(int i, int& kind, int& x, int& y) const {
    if (i < ns) {
      kind = 0;
      x = b + (i / KTs) * G;
      y = i % KTs;
      return;
    }
    int r;
    if (i < ns + p1) r = KTs * (b - rem) + (i - ns);
    else r = KTs * (G - rem) + b + (i - ns - p1) * G;
    kind = 1;
    x = r / ups;
    y = r % ups;
  }
};

// ------------------------------------------------------------------ fragments

// e2m1 word (8 codes) of rows g and g+8 -> two k16 MMAs.  Lane (g, t) holds
// word t of the 16-byte block of both rows; the codes map to the MMA k slots
// (2t, 2t+1, 2t+8, 2t+9) of two k16 steps, and the B fragment carries the
// activations of the same K positions (8t .. 8t+7 of the block).
__device__ __forceinline__ void fp4_word_mma(uint32_t wg, uint32_t w8, uint4 bv, float (&d0)[4], float (&d1)[4]) {
  uint32_t hg[4], h8[4];
  e2m1x8_to_f16x2(wg, hg);
  e2m1x8_to_f16x2(w8, h8);
  const uint32_t a0[4] = {hg[0], h8[0], hg[1], h8[1]};
  const uint32_t a1[4] = {hg[2], h8[2], hg[3], h8[3]};
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  mma_f16(d0, a0, bv.x, bv.y, z);  // two independent k16 halves: no MMA -> MMA dependency
  mma_f16(d1, a1, bv.z, bv.w, z);
}

// ue8m0 byte i (0..3) of w -> 2^(b-127), valid for b in 1..254 (exponent field
// placement); tiles holding 0x00 or 0xFF bytes use ds::u8m0_value instead.
__device__ __forceinline__ float scale_fast(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0u, 0x0444u | ((uint32_t)i << 12)) >> 1);
}

__device__ __forceinline__ bool has_special_byte(uint2 v) {
  return (__vcmpeq4(v.x, 0u) | __vcmpeq4(v.x, 0xFFFFFFFFu) | __vcmpeq4(v.y, 0u) | __vcmpeq4(v.y, 0xFFFFFFFFu)) != 0u;
}

__device__ __forceinline__ float scale_at(uint2 v, int i, bool exact) {
  const uint32_t w = i < 4 ? v.x : v.y;
  return exact ? u8m0_value((w >> (8 * (i & 3))) & 0xFFu) : scale_fast(w, i & 3);
}

// Deterministic cross-warp reduction without a CTA barrier: each consumer
// warp deposits its row partials in ring slot `buf` and bumps a counter; the
// last warp to arrive sums the slots in warp order and runs the epilogue.
__device__ __forceinline__ bool arrive_last(int* cnt, int buf, int lane) {
  __threadfence_block();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(&cnt[buf], 1) == kCW - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) __threadfence_block();
  return last != 0;
}

// ============================================================== kernel A

__global__ void __launch_bounds__(kThreads, 1) moe_tc_gate_up(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t slots_bar;
  __shared__ SlotInfo slots;
  __shared__ float xred[kCW];
  __shared__ int red_cnt[kRing];

  uint8_t* smem = align1k(smem_raw);
  const DecodeArgs& a = p.a;
  const Geo& g = p.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = g.a_stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kCW);
    }
    mbar_init(&slots_bar, 1);
    for (int r = 0; r < kRing; ++r) red_cnt[r] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  ListA L;
  L.init(gridDim.x, blockIdx.x, g.H / kKTile, g.shared ? g.Is / 8 : 0, g.I / 8);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // lane 0 issues the copies; the whole warp joins to build the slot list
    if (lane == 0) {
      prefetch_tensormap(&p.w1d);
      prefetch_tensormap(&p.w3d);
      prefetch_tensormap(&p.w1s);
      prefetch_tensormap(&p.w3s);
      if (g.shared) {
        prefetch_tensormap(&p.sw1);
        prefetch_tensormap(&p.sw3);
      }
    }
    bool ok = true;
    // shared-expert tiles do not depend on the routing: issue them first
    for (int i = 0; i < L.ns && ok; ++i) {
      if (lane == 0) {
        const int stage = i % S, use = i / S;
        if (use > 0 && !mbar_wait_bounded(&empty_bar[stage], (use - 1) & 1, kWaitNs)) {
          atomicOr(a.err, kErrWaitTimeout);
          ok = false;
        } else {
          uint8_t* dst = smem + (size_t)stage * g.a_stage;
          int kind, x, y;
          L.at(i, kind, x, y);
          mbar_arrive_expect_tx(&full_bar[stage], 2u * 8u * kKTile * 2u);
          tma_load_3d(dst, &p.sw1, 0, x * 8, y * 16, &full_bar[stage]);
          tma_load_3d(dst + g.a_data, &p.sw3, 0, x * 8, y * 16, &full_bar[stage]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    wait_prior_grid();  // routing (previous kernel) complete and visible
    build_slots_warp(a, slots, lane);
    L.set_routed(slots.count);
    if (lane == 0) {
      launch_dependents();  // the down kernel may start streaming W2
      mbar_arrive(&slots_bar);
    }
    if (lane != 0 || !ok) return;
    for (int i = L.ns; i < L.total(); ++i) {
      const int stage = i % S, use = i / S;
      if (use > 0 && !mbar_wait_bounded(&empty_bar[stage], (use - 1) & 1, kWaitNs)) {
        atomicOr(a.err, kErrWaitTimeout);
        break;
      }
      uint8_t* dst = smem + (size_t)stage * g.a_stage;
      int kind, x, y;
      L.at(i, kind, x, y);
      const int row = slots.expert[x] * g.I + y * 8;
      mbar_arrive_expect_tx(&full_bar[stage], 2u * (g.a_data + g.a_scales));
      tma_load_3d(dst, &p.w1d, 0, row, 0, &full_bar[stage]);
      tma_load_3d(dst + g.a_data, &p.w3d, 0, row, 0, &full_bar[stage]);
      tma_load_2d(dst + 2 * g.a_data, &p.w1s, 0, row, &full_bar[stage]);
      tma_load_2d(dst + 2 * g.a_data + g.a_scales, &p.w3s, 0, row, &full_bar[stage]);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int tid = threadIdx.x - 32;
  const int gq = lane >> 2, t = lane & 3;
  __half* x16 = reinterpret_cast<__half*>(smem + g.a_x16_off);
  __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(smem + g.a_xb_off);
  const __nv_bfloat16* xin = static_cast<const __nv_bfloat16*>(a.x);

  // x may be written by the preceding kernel: wait for it (the producer keeps
  // streaming shared-expert weights meanwhile).
  wait_prior_grid();
  // x staging: exact power-of-two scale so that max|x| lands in [2^14, 2^15)
  float m = 0.f;
  for (int k = tid; k < g.H; k += kConsumerThreads) m = fmaxf(m, fabsf(__bfloat162float(xin[k])));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) xred[cw] = m;
  bar_sync(1, kConsumerThreads);
  float mx = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) mx = fmaxf(mx, xred[w]);
  const int pe = (mx > 0.f && isfinite(mx)) ? 14 - ilogbf(mx) : 0;
  const float xs = ldexpf(1.0f, pe), xinv = ldexpf(1.0f, -pe);
  for (int k = tid; k < g.H; k += kConsumerThreads) {
    const __nv_bfloat16 v = xin[k];
    x16[k] = __float2half_rn(__bfloat162float(v) * xs);
    xb[k] = v;
  }
  bar_sync(1, kConsumerThreads);

  const int nbw = g.H / 32 / kCW;  // FP4 blocks per warp (multiple of 8)
  const uint32_t srow = g.H / 32;   // scale bytes per row
  float2* red = reinterpret_cast<float2*>(smem + g.a_red_off);  // [ring][warp][8]
  float acc0 = 0.f, acc2 = 0.f;     // gate / up row gq (column 0), routed tile
  float accs[4] = {0.f, 0.f, 0.f, 0.f};
  int unit = 0;
  bool have = false;
  for (int i = 0;; ++i) {
    if (i == L.ns && !have) {
      if (!mbar_wait_bounded(&slots_bar, 0, kWaitNs)) {
        atomicOr(a.err, kErrWaitTimeout);
        break;
      }
      L.set_routed(slots.count);
      have = true;
    }
    if (i >= L.total()) break;
    const int stage = i % S, use = i / S;
    if (!mbar_wait_bounded(&full_bar[stage], use & 1, kWaitNs)) {
      atomicOr(a.err, kErrWaitTimeout);
      break;
    }
    const uint8_t* st = smem + (size_t)stage * g.a_stage;
    int kind, x, y;
    L.at(i, kind, x, y);
    if (kind == 0) {
      // shared bf16 tile: this warp's 64-wide K slice, 4 k16 steps; every
      // lane supplies x, so all B columns are equal and column 0 is used.
      const uint8_t* top = st;
      const uint8_t* bot = st + g.a_data;
#pragma unroll
      for (int j = 0; j < kKTile / kCW / 16; ++j) {
        const int k0 = cw * (kKTile / kCW) + j * 16;
        const int xo = (k0 + 4 * t) * 2;
        const uint2 wa = *reinterpret_cast<const uint2*>(top + swz128(gq, xo, 8));
        const uint2 wb = *reinterpret_cast<const uint2*>(bot + swz128(gq, xo, 8));
        const uint2 xv = *reinterpret_cast<const uint2*>(xb + y * kKTile + k0 + 4 * t);
        const uint32_t af[4] = {wa.x, wb.x, wa.y, wb.y};
        mma_bf16(accs, af, xv.x, xv.y, accs);
      }
    } else {
      acc0 = acc2 = 0.f;
      const uint8_t* top = st;
      const uint8_t* bot = st + g.a_data;
      const uint8_t* s1 = st + 2 * g.a_data;
      const uint8_t* s3 = s1 + g.a_scales;
      for (int c = 0; c < nbw; c += 8) {
        const int bg = cw * nbw + c;  // first of 8 blocks = one 128-byte chunk column
        const uint32_t rowoff = (uint32_t)(((bg >> 3) * 8 + gq) * 128 + 4 * t) ^ (uint32_t)(gq << 4);
        const uint2 sg = *reinterpret_cast<const uint2*>(s1 + gq * srow + bg);
        const uint2 su = *reinterpret_cast<const uint2*>(s3 + gq * srow + bg);
        const bool exact = __any_sync(0xffffffffu, has_special_byte(sg) || has_special_byte(su));
        // two batches of 4 blocks: all shared-memory loads of a batch are
        // issued before its conversions and MMAs (independent chains)
#pragma unroll
        for (int h4 = 0; h4 < 8; h4 += 4) {
          uint32_t wg[4], w8[4];
          uint4 xv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t off = rowoff ^ (uint32_t)((h4 + q) << 4);
            wg[q] = *reinterpret_cast<const uint32_t*>(top + off);
            w8[q] = *reinterpret_cast<const uint32_t*>(bot + off);
            xv[q] = *reinterpret_cast<const uint4*>(x16 + (bg + h4 + q) * 32 + t * 8);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float d0[4], d1[4];
            fp4_word_mma(wg[q], w8[q], xv[q], d0, d1);
            float sgv, suv;
            if (!exact) {
              sgv = scale_fast(h4 == 0 ? sg.x : sg.y, q);
              suv = scale_fast(h4 == 0 ? su.x : su.y, q);
            } else {
              sgv = scale_at(sg, h4 + q, true);
              suv = scale_at(su, h4 + q, true);
            }
            acc0 = fmaf(sgv, d0[0] + d1[0], acc0);
            acc2 = fmaf(suv, d0[2] + d1[2], acc2);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);

    const bool unit_done = (kind == 1) || (y == L.KTs - 1);
    if (unit_done) {
      const int buf = unit % kRing;
      if (t == 0) red[(buf * kCW + cw) * 8 + gq] = kind == 1 ? make_float2(acc0, acc2) : make_float2(accs[0], accs[2]);
      if (arrive_last(red_cnt, buf, lane)) {
        if (t == 0) {
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int w = 0; w < kCW; ++w) {
            const float2 v = red[(buf * kCW + w) * 8 + gq];
            gs += v.x;
            us += v.y;
          }
          float hv;
          int slot_index;
          if (kind == 1) {
            hv = silu_glu(gs * xinv, us * xinv, a.d.swiglu_limit) * slots.gate[x];
            slot_index = x;
          } else {
            hv = silu_glu(gs, us, 10.0f);
            slot_index = g.max_slots;
          }
          const int n = (kind == 1 ? y : x) * 8 + gq;
          a.h[(size_t)slot_index * a.h_stride + n] = hv;
        }
        __syncwarp();
        if (lane == 0) red_cnt[buf] = 0;
      }
      ++unit;
      if (kind == 0) accs[0] = accs[1] = accs[2] = accs[3] = 0.f;
    }
  }
}

// ============================================================== kernel B

__global__ void __launch_bounds__(kThreads, 1) moe_tc_down(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t slots_bar;
  __shared__ SlotInfo slots;
  __shared__ float hred[kCW];
  __shared__ int red_cnt[kRing];

  uint8_t* smem = align1k(smem_raw);
  const DecodeArgs& a = p.a;
  const Geo& g = p.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = g.b_stages;
  const int G = gridDim.x, b = blockIdx.x;
  const int units = g.H / 16;
  const int my_units = units > b ? (units - b + G - 1) / G : 0;
  const int KTb = g.shared ? g.Is / kKTile : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kCW);
    }
    mbar_init(&slots_bar, 1);
    for (int r = 0; r < kRing; ++r) red_cnt[r] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Routing is complete: the gate/up kernel triggers this launch only after
    // its own wait on the router.
    if (lane == 0) {
      prefetch_tensormap(&p.w2d);
      prefetch_tensormap(&p.w2s);
      if (g.shared) prefetch_tensormap(&p.sw2);
    }
    build_slots_warp(a, slots, lane);
    if (lane != 0) return;
    mbar_arrive(&slots_bar);
    const int D = slots.count;
    const int np = (D + 1) / 2;
    const int per_unit = np + KTb;
    const int total = my_units * per_unit;
    for (int i = 0; i < total; ++i) {
      const int stage = i % S, use = i / S;
      if (use > 0 && !mbar_wait_bounded(&empty_bar[stage], (use - 1) & 1, kWaitNs)) {
        atomicOr(a.err, kErrWaitTimeout);
        break;
      }
      const int rb = b + (i / per_unit) * G;
      const int j = i % per_unit;
      uint8_t* dst = smem + (size_t)stage * g.b_stage;
      if (j < np) {
        const int s0 = 2 * j, nsl = min(2, D - s0);
        mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)nsl * (g.b_data + g.b_scales));
        for (int q = 0; q < nsl; ++q) {
          const int row = slots.expert[s0 + q] * g.H + rb * 16;
          tma_load_3d(dst + q * g.b_data, &p.w2d, 0, row, 0, &full_bar[stage]);
          tma_load_2d(dst + 2 * g.b_data + q * g.b_scales, &p.w2s, 0, row, &full_bar[stage]);
        }
      } else {
        const int kt = j - np;
        mbar_arrive_expect_tx(&full_bar[stage], 16u * kKTile * 2u);
        tma_load_3d(dst, &p.sw2, 0, rb * 16, kt * 16, &full_bar[stage]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int tid = threadIdx.x - 32;
  const int gq = lane >> 2, t = lane & 3;
  if (!mbar_wait_bounded(&slots_bar, 0, kWaitNs)) {
    atomicOr(a.err, kErrWaitTimeout);
    return;
  }
  const int D = slots.count;
  const int np = (D + 1) / 2;
  const int per_unit = np + KTb;

  // h of the gate/up kernel: wait for it, then stage hi/lo halves.
  wait_prior_grid();
  if (per_unit == 0) {  // nothing routed and no shared expert: the layer output is zero
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    for (int u = 0; u < my_units; ++u)
      if (tid < 16) out[(b + u * G) * 16 + tid] = __float2bfloat16_rn(0.0f);
    return;
  }
  __half* hh = reinterpret_cast<__half*>(smem + g.b_hh_off);   // [slot][I]
  __half* hl = reinterpret_cast<__half*>(smem + g.b_hl_off);   // [slot][I]
  __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(smem + g.b_sh_off);  // [2][Is] hi, lo
  // h rows are h_stride apart and I is a multiple of 4, so a float4 never
  // straddles two slots.  Each thread keeps up to kHVec float4 of h in
  // registers (one global round trip), the block agrees on max|h|, and the
  // registers are converted to f16 hi/lo; larger D * I falls back to a
  // second (L2-hit) pass.
  constexpr int kHVec = 8;
  const int nvec = D * g.I / 4;
  float4 hv4[kHVec];
  float m = 0.f;
#pragma unroll
  for (int r = 0; r < kHVec; ++r) {
    const int v = tid + r * kConsumerThreads;
    hv4[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < nvec) {
      const int k = 4 * v, s = k / g.I, c = k - s * g.I;
      hv4[r] = *reinterpret_cast<const float4*>(a.h + (size_t)s * a.h_stride + c);
    }
  }
#pragma unroll
  for (int r = 0; r < kHVec; ++r)
    m = fmaxf(m, fmaxf(fmaxf(fabsf(hv4[r].x), fabsf(hv4[r].y)), fmaxf(fabsf(hv4[r].z), fabsf(hv4[r].w))));
  for (int v = tid + kHVec * kConsumerThreads; v < nvec; v += kConsumerThreads) {
    const int k = 4 * v, s = k / g.I, c = k - s * g.I;
    const float4 f = *reinterpret_cast<const float4*>(a.h + (size_t)s * a.h_stride + c);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) hred[cw] = m;
  bar_sync(1, kConsumerThreads);
  float mx = 0.f;
#pragma unroll
  for (int w = 0; w < kCW; ++w) mx = fmaxf(mx, hred[w]);
  const int pe = (mx > 0.f && isfinite(mx)) ? 14 - ilogbf(mx) : 0;
  const float hsc = ldexpf(1.0f, pe), hinv = ldexpf(1.0f, -pe);
  auto store_hilo = [&](int k, float4 f) {
    const float fv[4] = {f.x * hsc, f.y * hsc, f.z * hsc, f.w * hsc};
    uint32_t hi2[2], lo2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const __half2 hi = __floats2half2_rn(fv[2 * e], fv[2 * e + 1]);
      const float2 hf = __half22float2(hi);
      const __half2 lo = __floats2half2_rn(fv[2 * e] - hf.x, fv[2 * e + 1] - hf.y);
      hi2[e] = *reinterpret_cast<const uint32_t*>(&hi);
      lo2[e] = *reinterpret_cast<const uint32_t*>(&lo);
    }
    *reinterpret_cast<uint2*>(hh + k) = make_uint2(hi2[0], hi2[1]);
    *reinterpret_cast<uint2*>(hl + k) = make_uint2(lo2[0], lo2[1]);
  };
#pragma unroll
  for (int r = 0; r < kHVec; ++r) {
    const int v = tid + r * kConsumerThreads;
    if (v < nvec) store_hilo(4 * v, hv4[r]);
  }
  for (int v = tid + kHVec * kConsumerThreads; v < nvec; v += kConsumerThreads) {
    const int k = 4 * v, s = k / g.I, c = k - s * g.I;
    store_hilo(k, *reinterpret_cast<const float4*>(a.h + (size_t)s * a.h_stride + c));
  }
  if (g.shared) {
    for (int k = tid; k < g.Is; k += kConsumerThreads) {
      const float v = a.h[(size_t)g.max_slots * a.h_stride + k];
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      sh[k] = hi;
      sh[g.Is + k] = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
  }
  bar_sync(1, kConsumerThreads);

  // B fragment columns: lanes with even groupID supply the hi half, odd the
  // lo half, so column 0 = hi and column 1 = lo (the rest duplicate them).
  const int nbw = g.I / 32 / (kCW / 2);  // 8 warps per slot of a pair
  const uint32_t srow = g.I / 32;
  float4* red = reinterpret_cast<float4*>(smem + g.b_red_off);  // [ring][warp][8]
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float accs[4] = {0.f, 0.f, 0.f, 0.f};
  int unit = 0;
  const int total = my_units * per_unit;
  for (int i = 0; i < total; ++i) {
    const int stage = i % S, use = i / S;
    if (!mbar_wait_bounded(&full_bar[stage], use & 1, kWaitNs)) {
      atomicOr(a.err, kErrWaitTimeout);
      break;
    }
    const int rb = b + (i / per_unit) * G;
    const int j = i % per_unit;
    const uint8_t* st = smem + (size_t)stage * g.b_stage;
    if (j < np) {
      const int q = cw / (kCW / 2), kq = cw % (kCW / 2);
      const int s = 2 * j + q;
      if (s < D) {
        const uint8_t* dat = st + q * g.b_data;
        const uint8_t* sc = st + 2 * g.b_data + q * g.b_scales;
        const __half* hsrc = ((gq & 1) ? hl : hh) + (size_t)s * g.I;
        for (int c = 0; c < nbw; c += 8) {
          const int bg = kq * nbw + c;
          // rows gq and gq+8 of the 16-row box share the swizzle key gq
          const uint32_t rowoff = (uint32_t)(((bg >> 3) * 16 + gq) * 128 + 4 * t) ^ (uint32_t)(gq << 4);
          const uint2 s0v = *reinterpret_cast<const uint2*>(sc + gq * srow + bg);
          const uint2 s8v = *reinterpret_cast<const uint2*>(sc + (gq + 8) * srow + bg);
          const bool exact = __any_sync(0xffffffffu, has_special_byte(s0v) || has_special_byte(s8v));
#pragma unroll
          for (int h4 = 0; h4 < 8; h4 += 4) {
            uint32_t wg[4], w8[4];
            uint4 hv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t off = rowoff ^ (uint32_t)((h4 + q) << 4);
              wg[q] = *reinterpret_cast<const uint32_t*>(dat + off);
              w8[q] = *reinterpret_cast<const uint32_t*>(dat + off + 8 * 128);
              hv[q] = *reinterpret_cast<const uint4*>(hsrc + (bg + h4 + q) * 32 + t * 8);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float d0[4], d1[4];
              fp4_word_mma(wg[q], w8[q], hv[q], d0, d1);
              float s0, s8;
              if (!exact) {
                s0 = scale_fast(h4 == 0 ? s0v.x : s0v.y, q);
                s8 = scale_fast(h4 == 0 ? s8v.x : s8v.y, q);
              } else {
                s0 = scale_at(s0v, h4 + q, true);
                s8 = scale_at(s8v, h4 + q, true);
              }
              acc[0] = fmaf(s0, d0[0] + d1[0], acc[0]);
              acc[1] = fmaf(s0, d0[1] + d1[1], acc[1]);
              acc[2] = fmaf(s8, d0[2] + d1[2], acc[2]);
              acc[3] = fmaf(s8, d0[3] + d1[3], acc[3]);
            }
          }
        }
      }
    } else {
      const int kt = j - np;
      const __nv_bfloat16* hsrc = sh + ((gq & 1) ? g.Is : 0) + kt * kKTile;
#pragma unroll
      for (int jj = 0; jj < kKTile / kCW / 16; ++jj) {
        const int k0 = cw * (kKTile / kCW) + jj * 16;
        const int xo = (k0 + 4 * t) * 2;
        const uint2 wa = *reinterpret_cast<const uint2*>(st + swz128(gq, xo, 16));
        const uint2 wb = *reinterpret_cast<const uint2*>(st + swz128(gq + 8, xo, 16));
        const uint2 hv = *reinterpret_cast<const uint2*>(hsrc + k0 + 4 * t);
        const uint32_t af[4] = {wa.x, wb.x, wa.y, wb.y};
        mma_bf16(accs, af, hv.x, hv.y, accs);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);

    if (j == per_unit - 1) {
      const int buf = unit % kRing;
      if (t == 0)
        red[(buf * kCW + cw) * 8 + gq] =
            make_float4(acc[0] + acc[1], acc[2] + acc[3], accs[0] + accs[1], accs[2] + accs[3]);
      if (arrive_last(red_cnt, buf, lane)) {
        if (t == 0) {
          float r0 = 0.f, r8 = 0.f, s0 = 0.f, s8 = 0.f;
#pragma unroll
          for (int w = 0; w < kCW; ++w) {
            const float4 v = red[(buf * kCW + w) * 8 + gq];
            r0 += v.x;
            r8 += v.y;
            s0 += v.z;
            s8 += v.w;
          }
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
          float o0 = r0 * hinv, o8 = r8 * hinv;
          if (g.shared) {
            o0 += __bfloat162float(__float2bfloat16_rn(s0));
            o8 += __bfloat162float(__float2bfloat16_rn(s8));
          }
          out[rb * 16 + gq] = __float2bfloat16_rn(o0);
          out[rb * 16 + gq + 8] = __float2bfloat16_rn(o8);
        }
        __syncwarp();
        if (lane == 0) red_cnt[buf] = 0;
      }
      ++unit;
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      accs[0] = accs[1] = accs[2] = accs[3] = 0.f;
    }
  }
}

// ============================================================== host side

uint32_t round_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

Geo make_geo(const DecodeArgs& a) {
  Geo g{};
  g.H = a.d.hidden;
  g.I = a.d.inter;
  g.shared = a.d.shared_w1 != nullptr;
  g.Is = g.shared ? a.d.shared_inter : 0;
  g.max_slots = a.max_slots;
  const uint32_t sh_box = 8u * kKTile * 2u;  // 8 rows x 2048 B
  // kernel A: [W1 box][W3 box][W1 scales][W3 scales]; shared: [SW1 box][SW3 box]
  g.a_data = std::max<uint32_t>(8u * (g.H / 2), sh_box);
  g.a_scales = 8u * (g.H / 32);
  g.a_stage = round_up(2 * g.a_data + 2 * g.a_scales, 1024);
  const uint32_t a_fixed = 1024 + (uint32_t)g.H * 4 + kRedBytesA;
  g.a_stages = std::min<int>(kMaxStages, (int)((kSmemLimit - 1024 - (int)a_fixed) / (int)g.a_stage));
  g.a_x16_off = g.a_stages * g.a_stage;
  g.a_xb_off = g.a_x16_off + g.H * 2;
  g.a_red_off = round_up(g.a_xb_off + g.H * 2, 16);
  g.a_total = g.a_red_off + kRedBytesA + 1024;  // + alignment slack
  // kernel B: [slot0 box][slot1 box][slot0 scales][slot1 scales]; shared: [SW2 box 16 rows]
  g.b_data = std::max<uint32_t>(16u * (g.I / 2), 0u);
  g.b_scales = 16u * (g.I / 32);
  g.b_stage = round_up(std::max<uint32_t>(2 * g.b_data + 2 * g.b_scales, 2 * sh_box), 1024);
  const uint32_t h_bytes = (uint32_t)g.max_slots * g.I * 4 + (uint32_t)g.Is * 4;
  const uint32_t b_fixed = 1024 + h_bytes + kRedBytesB;
  g.b_stages = std::min<int>(kMaxStages, (int)((kSmemLimit - 1024 - (int)b_fixed) / (int)g.b_stage));
  g.b_hh_off = g.b_stages * g.b_stage;
  g.b_hl_off = g.b_hh_off + (uint32_t)g.max_slots * g.I * 2;
  g.b_sh_off = g.b_hl_off + (uint32_t)g.max_slots * g.I * 2;
  g.b_red_off = round_up(g.b_sh_off + (uint32_t)g.Is * 4, 16);
  g.b_total = g.b_red_off + kRedBytesB + 1024;
  return g;
}

// ---- tensor maps (driver entry point resolved through the runtime; no -lcuda)

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

// Rows of `row_bytes` bytes (multiple of 128) viewed as [128 B][rows][row_bytes/128]
// with the 128-byte swizzle; box = 128 B x box_rows x box_chunks.
bool map_rows_swizzled(CUtensorMap* m, const void* base, uint64_t rows, uint32_t row_bytes, uint32_t box_rows,
                       uint32_t box_chunks) {
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {128, box_rows, box_chunks};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Plain rows (scales): box = row_bytes x box_rows, no swizzle.
bool map_rows_plain(CUtensorMap* m, const void* base, uint64_t rows, uint32_t row_bytes, uint32_t box_rows) {
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {row_bytes, box_rows};
  const cuuint32_t es[2] = {1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct MapKey {
  const void* p[9];
  int geo[6];
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = 1469598103934665603ull;
    const unsigned char* b = reinterpret_cast<const unsigned char*>(&k);
    for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
  }
};
struct Maps {
  CUtensorMap w1d, w3d, w1s, w3s, sw1, sw3, w2d, w2s, sw2;
};

// Encode the tensor maps of a layer (pure host work, no allocation).
int encode_maps(const DecodeArgs& a, Maps& m) {
  const DsMoeDesc& d = a.d;
  DS_REQUIRE(encode_fn() != nullptr, DS_ECUDA, "moe_decode: cuTensorMapEncodeTiled unavailable");
  memset(&m, 0, sizeof(m));
  const uint64_t E = d.n_experts, H = d.hidden, I = d.inter;
  bool ok = map_rows_swizzled(&m.w1d, d.w1.data, E * I, H / 2, 8, H / 256) &&
            map_rows_swizzled(&m.w3d, d.w3.data, E * I, H / 2, 8, H / 256) &&
            map_rows_plain(&m.w1s, d.w1.scales, E * I, H / 32, 8) &&
            map_rows_plain(&m.w3s, d.w3.scales, E * I, H / 32, 8) &&
            map_rows_swizzled(&m.w2d, d.w2.data, E * H, I / 2, 16, I / 256) &&
            map_rows_plain(&m.w2s, d.w2.scales, E * H, I / 32, 16);
  if (ok && d.shared_w1) {
    const uint64_t Is = d.shared_inter;
    ok = map_rows_swizzled(&m.sw1, d.shared_w1, Is, H * 2, 8, 16) &&
         map_rows_swizzled(&m.sw3, d.shared_w3, Is, H * 2, 8, 16) &&
         map_rows_swizzled(&m.sw2, d.shared_w2, H, Is * 2, 16, 16);
  }
  DS_REQUIRE(ok, DS_ECUDA, "moe_decode: tensor map encoding failed");
  return DS_OK;
}

// Encode (or fetch cached) tensor maps for a layer.  Resident banks keep
// their addresses, so a small cache makes the per-call cost a hash lookup.
int get_maps(const DecodeArgs& a, Maps& out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, Maps, MapKeyHash> cache;
  const DsMoeDesc& d = a.d;
  MapKey key;
  memset(&key, 0, sizeof(key));
  key.p[0] = d.w1.data, key.p[1] = d.w3.data, key.p[2] = d.w2.data;
  key.p[3] = d.w1.scales, key.p[4] = d.w3.scales, key.p[5] = d.w2.scales;
  key.p[6] = d.shared_w1, key.p[7] = d.shared_w3, key.p[8] = d.shared_w2;
  key.geo[0] = d.hidden, key.geo[1] = d.inter, key.geo[2] = d.n_experts, key.geo[3] = d.shared_inter;
  int dev = 0;
  cudaGetDevice(&dev);
  key.geo[4] = dev;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    out = it->second;
    return DS_OK;
  }
  Maps m;
  const int rc = encode_maps(a, m);
  if (rc != DS_OK) return rc;
  if (cache.size() > 256) cache.clear();
  cache.emplace(key, m);
  out = m;
  return DS_OK;
}

int launch_with_maps(const DecodeArgs& a, const Maps& m, cudaStream_t st) {
  TcParams p;
  memset(&p, 0, sizeof(p));
  p.w1d = m.w1d, p.w3d = m.w3d, p.w1s = m.w1s, p.w3s = m.w3s, p.sw1 = m.sw1, p.sw3 = m.sw3;
  p.w2d = m.w2d, p.w2s = m.w2s, p.sw2 = m.sw2;
  p.a = a;
  p.g = make_geo(a);
  DS_CHECK_CUDA(cudaFuncSetAttribute(moe_tc_gate_up, cudaFuncAttributeMaxDynamicSharedMemorySize, p.g.a_total));
  DS_CHECK_CUDA(cudaFuncSetAttribute(moe_tc_down, cudaFuncAttributeMaxDynamicSharedMemorySize, p.g.b_total));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(ds::sm_count());
  cfg.dynamicSmemBytes = p.g.a_total;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, moe_tc_gate_up, p));
  cfg.gridDim = dim3(std::min(ds::sm_count(), p.g.H / 16));
  cfg.dynamicSmemBytes = p.g.b_total;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, moe_tc_down, p));
  return DS_OK;
}

}  // namespace

bool tc_supported(const DecodeArgs& a) {
  const DsMoeDesc& d = a.d;
  if (a.tokens != 1 || a.x_f32 || d.w1.format != DS_FMT_FP4) return false;
  if (a.max_slots > kMaxSlots || d.top_k > 32) return false;
  // FP4 rows in whole 128-byte chunks, scale rows within one TMA box (<= 256 B),
  // 8 blocks per consumer warp, whole bf16 K slices.
  if (d.hidden % 4096 != 0 || d.hidden > 8192) return false;
  if (d.inter % 2048 != 0 || d.inter > 8192) return false;
  if ((uint64_t)d.n_experts * d.inter >= (1ull << 31) || (uint64_t)d.n_experts * d.hidden >= (1ull << 31)) return false;
  const bool sh = d.shared_w1 != nullptr;
  if (sh && (d.shared_inter % kKTile != 0 || d.shared_inter % 8 != 0)) return false;
  const Geo g = make_geo(a);
  if (g.a_stages < 2 || g.b_stages < 2 || g.a_stages > kRing - 2 || g.b_stages > kRing - 2) return false;
  if (g.a_total > (uint32_t)kSmemLimit || g.b_total > (uint32_t)kSmemLimit) return false;
  // TMA global addresses must be 16-byte aligned (strides are multiples of 16 by the checks above)
  if (!ds::aligned(d.w1.data, 16) || !ds::aligned(d.w3.data, 16) || !ds::aligned(d.w2.data, 16) ||
      !ds::aligned(d.w1.scales, 16) || !ds::aligned(d.w3.scales, 16) || !ds::aligned(d.w2.scales, 16))
    return false;
  if (sh && (!ds::aligned(d.shared_w1, 16) || !ds::aligned(d.shared_w3, 16) || !ds::aligned(d.shared_w2, 16)))
    return false;
  return encode_fn() != nullptr;
}

int launch_tc(const DecodeArgs& a, cudaStream_t st) {
  Maps m;
  const int rc = get_maps(a, m);
  if (rc != DS_OK) return rc;
  return launch_with_maps(a, m, st);
}

int launch_tc_uncached(const DecodeArgs& a, cudaStream_t st) {
  Maps m;
  const int rc = encode_maps(a, m);
  if (rc != DS_OK) return rc;
  return launch_with_maps(a, m, st);
}

}  // namespace decode
}  // namespace ds
