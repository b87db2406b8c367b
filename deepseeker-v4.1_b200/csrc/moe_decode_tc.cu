// Single-token (B = 1) routed-expert MoE layer: warp-specialised, bulk-copy
// pipelined, tensor-core decode.  FP4 routed experts + optional bf16 shared
// expert; geometry checked by tc_supported(), everything else goes to the
// generic path in moe_decode.cu.
//
// Both kernels are persistent (one CTA per SM, 9 warps):
//   warp 0, lane 0   producer: streams weight tiles HBM -> shared memory with
//                    1-D cp.async.bulk row copies into a ring of stages
//                    (mbarrier full/empty handshake).  Rows are padded in
//                    shared memory so the consumers' fragment reads are
//                    bank-conflict free.
//   warps 1..8       consumers: each owns a K slice of the current tile,
//                    decodes e2m1 codes straight into mma.sync A fragments
//                    (cvt.rn.f16x2.e2m1x2; code order low nibble first), runs
//                    m16n8k16 with the activations as the B fragment and
//                    applies the ue8m0 block scale per 32-element block on the
//                    f32 accumulator.  A cross-warp reduction finishes a unit.
//
// Kernel A (gate/up): tile = 8 rows of W1 and the same 8 rows of W3 of one
//   routed expert (m16 rows 0-7 gate, 8-15 up), full K; or a 1024-wide K
//   slice of 8+8 shared-expert rows.  x is staged once per CTA as f16 scaled
//   by an exact power of two (x is bf16: 8 significant bits, so the products
//   with e2m1 values are exact in f32) and as raw bf16 for the shared expert.
//   Epilogue: h = silu(min(g, L)) * clip(u, -L, L) * gate, stored f32.
// Kernel B (down + combine): unit = 16 output rows; tiles = pairs of routed
//   slots (16 rows of W2 each, full K = I) then 1024-wide K slices of the
//   shared W2.  h is staged per CTA as f16 hi + lo (routed, scaled by a power
//   of two) and bf16 hi + lo (shared): ~22 / 16 significant bits, so the down
//   projection is not limited by a bf16 rounding of h.  out = bf16(routed +
//   f32(bf16(shared))) as in the reference (mlx_forward.py:409-419).
//
// Launch chain on the stream: router -> A -> B with programmatic dependent
// launch: A's prologue and its shared-expert tiles overlap the router; A lets
// B start once routing is resolved, and B streams W2 tiles while A finishes
// (B's consumers wait for A's h with griddepcontrol.wait).
//
// Every wait is bounded (2 s of %globaltimer); on expiry the kernel records
// kErrWaitTimeout in the workspace error word and stops.
#include "moe_decode.cuh"
#include "ptx.cuh"

namespace ds {
namespace decode {
namespace {

using namespace ds::ptx;

constexpr int kCW = 8;                      // consumer warps
constexpr int kThreads = 32 * (kCW + 1);    // 288
constexpr int kConsumerThreads = 32 * kCW;  // 256
constexpr int kMaxStages = 8;
constexpr int kKTile = 1024;                // bf16 K slice per shared tile
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kMaxSlots = 32;
constexpr uint32_t kFp4Pad = 16;            // smem row padding (bytes)
constexpr uint32_t kBf16Pad = 32;
constexpr int kSmemLimit = 227 * 1024;

struct Geo {
  int H, I, Is, shared, max_slots;
  // kernel A
  uint32_t a_ds, a_ss, a_sc_off, a_stage;  // data stride, scale stride, scale offset, stage bytes
  int a_stages;
  uint32_t a_x16_off, a_xb_off, a_red_off, a_total;
  // kernel B
  uint32_t b_ds, b_ss, b_slot, b_stage;    // data stride, scale stride, per-slot bytes, stage bytes
  int b_stages;
  uint32_t b_hh_off, b_hl_off, b_sh_off, b_red_off, b_total;
  uint32_t sh_stride;                      // bf16 row stride in shared tiles
};

struct TcArgs {
  DecodeArgs a;
  Geo g;
};

struct SlotInfo {
  int count;
  int expert[kMaxSlots];
  float gate[kMaxSlots];
};

// Distinct routed experts of the single token in ascending id, each with the
// gate of its first slot (src/deepseeker/mlx_forward.py:394-404).
__device__ void build_slots_t1(const DecodeArgs& a, SlotInfo& s) {
  int cnt = 0;
  const int k = a.d.top_k;
  for (int i = 0; i < k; ++i) {
    const int id = a.ids[i];
    if (id >= a.d.n_experts) {
      atomicOr(a.err, kErrExpertRange);
      continue;
    }
    if (id < 0) continue;
    bool dup = false;
    for (int j = 0; j < cnt; ++j) dup |= (s.expert[j] == id);
    if (dup) continue;
    const float gt = a.gates[i];
    int p = cnt;
    while (p > 0 && s.expert[p - 1] > id) {
      s.expert[p] = s.expert[p - 1];
      s.gate[p] = s.gate[p - 1];
      --p;
    }
    s.expert[p] = id;
    s.gate[p] = gt;
    ++cnt;
  }
  s.count = cnt;
}

__device__ __forceinline__ float silu_glu(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
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
  // kind 0 = shared (unit u, slice kt), 1 = routed (slot, rb)
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

// One FP4 block (32 codes along K) of an m16 tile -> f32 partial (4 lanes'
// worth of C fragment), scaled by the rows' ue8m0 scales and accumulated.
// Lane (g, t) reads word t of rows g and g+8; the 8 codes of that word feed
// two k16 MMAs whose B fragments are x[32*blk + 8t .. 8t+7] (same mapping).
__device__ __forceinline__ void fp4_block_mma(const uint8_t* dat, uint32_t ds_, const uint8_t* sc, uint32_t ss,
                                              int blk, int gq, int t, uint4 xv, float (&acc)[4]) {
  const uint32_t wg = *reinterpret_cast<const uint32_t*>(dat + gq * ds_ + blk * 16 + t * 4);
  const uint32_t w8 = *reinterpret_cast<const uint32_t*>(dat + (gq + 8) * ds_ + blk * 16 + t * 4);
  uint32_t hg[4], h8[4];
  e2m1x8_to_f16x2(wg, hg);
  e2m1x8_to_f16x2(w8, h8);
  const uint32_t a0[4] = {hg[0], h8[0], hg[1], h8[1]};
  const uint32_t a1[4] = {hg[2], h8[2], hg[3], h8[3]};
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  float tmp[4];
  mma_f16(tmp, a0, xv.x, xv.y, z);
  mma_f16(tmp, a1, xv.z, xv.w, tmp);
  const float s0 = u8m0_value(sc[gq * ss + blk]);
  const float s8 = u8m0_value(sc[(gq + 8) * ss + blk]);
  acc[0] = fmaf(s0, tmp[0], acc[0]);
  acc[1] = fmaf(s0, tmp[1], acc[1]);
  acc[2] = fmaf(s8, tmp[2], acc[2]);
  acc[3] = fmaf(s8, tmp[3], acc[3]);
}

// Same with the activation split in two f16 halves (hi + lo): four MMAs.
__device__ __forceinline__ void fp4_block_mma2(const uint8_t* dat, uint32_t ds_, const uint8_t* sc, uint32_t ss,
                                               int blk, int gq, int t, uint4 hv, uint4 lv, float (&acc)[4]) {
  const uint32_t wg = *reinterpret_cast<const uint32_t*>(dat + gq * ds_ + blk * 16 + t * 4);
  const uint32_t w8 = *reinterpret_cast<const uint32_t*>(dat + (gq + 8) * ds_ + blk * 16 + t * 4);
  uint32_t hg[4], h8[4];
  e2m1x8_to_f16x2(wg, hg);
  e2m1x8_to_f16x2(w8, h8);
  const uint32_t a0[4] = {hg[0], h8[0], hg[1], h8[1]};
  const uint32_t a1[4] = {hg[2], h8[2], hg[3], h8[3]};
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  float tmp[4];
  mma_f16(tmp, a0, hv.x, hv.y, z);
  mma_f16(tmp, a0, lv.x, lv.y, tmp);
  mma_f16(tmp, a1, hv.z, hv.w, tmp);
  mma_f16(tmp, a1, lv.z, lv.w, tmp);
  const float s0 = u8m0_value(sc[gq * ss + blk]);
  const float s8 = u8m0_value(sc[(gq + 8) * ss + blk]);
  acc[0] = fmaf(s0, tmp[0], acc[0]);
  acc[1] = fmaf(s0, tmp[1], acc[1]);
  acc[2] = fmaf(s8, tmp[2], acc[2]);
  acc[3] = fmaf(s8, tmp[3], acc[3]);
}

// ============================================================== kernel A

__global__ void __launch_bounds__(kThreads, 1) moe_tc_gate_up(const TcArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t slots_bar;
  __shared__ SlotInfo slots;
  __shared__ float xred[kCW];

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
    fence_barrier_init();
  }
  __syncthreads();

  ListA L;
  L.init(gridDim.x, blockIdx.x, g.H / kKTile, g.shared ? g.Is / 8 : 0, g.I / 8);

  if (warp == 0) {
    if (lane != 0) return;
    // ------------------------------------------------------------ producer
    const DsExpertBank& w1 = a.d.w1;
    const DsExpertBank& w3 = a.d.w3;
    const uint32_t drow = g.H / 2, srow = g.H / 32;
    bool have = false;
    for (int i = 0;; ++i) {
      if (i == L.ns && !have) {
        wait_prior_grid();  // routing (previous kernel) complete and visible
        build_slots_t1(a, slots);
        L.set_routed(slots.count);
        launch_dependents();  // the down kernel may start streaming W2
        mbar_arrive(&slots_bar);
        have = true;
      }
      if (i >= L.total()) break;
      const int stage = i % S, use = i / S;
      if (use > 0 && !mbar_wait_bounded(&empty_bar[stage], (use - 1) & 1, kWaitNs)) {
        atomicOr(a.err, kErrWaitTimeout);
        break;
      }
      uint8_t* dst = smem + (size_t)stage * g.a_stage;
      int kind, x, y;
      L.at(i, kind, x, y);
      if (kind == 0) {
        // shared expert: rows x*8 .. x*8+7 of W1 and W3, K slice y
        const size_t koff = (size_t)y * kKTile * 2;
        mbar_arrive_expect_tx(&full_bar[stage], 16u * kKTile * 2);
        for (int r = 0; r < 8; ++r) {
          const size_t n = (size_t)x * 8 + r;
          bulk_g2s(dst + r * g.sh_stride, static_cast<const uint8_t*>(a.d.shared_w1) + n * g.H * 2 + koff,
                   kKTile * 2, &full_bar[stage]);
          bulk_g2s(dst + (8 + r) * g.sh_stride, static_cast<const uint8_t*>(a.d.shared_w3) + n * g.H * 2 + koff,
                   kKTile * 2, &full_bar[stage]);
        }
      } else {
        const int e = slots.expert[x];
        mbar_arrive_expect_tx(&full_bar[stage], 16u * (drow + srow));
        for (int r = 0; r < 8; ++r) {
          const size_t row = (size_t)e * g.I + (size_t)y * 8 + r;
          bulk_g2s(dst + r * g.a_ds, static_cast<const uint8_t*>(w1.data) + row * drow, drow, &full_bar[stage]);
          bulk_g2s(dst + (8 + r) * g.a_ds, static_cast<const uint8_t*>(w3.data) + row * drow, drow,
                   &full_bar[stage]);
          bulk_g2s(dst + g.a_sc_off + r * g.a_ss, static_cast<const uint8_t*>(w1.scales) + row * srow, srow,
                   &full_bar[stage]);
          bulk_g2s(dst + g.a_sc_off + (8 + r) * g.a_ss, static_cast<const uint8_t*>(w3.scales) + row * srow, srow,
                   &full_bar[stage]);
        }
      }
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

  const int NB = g.H / 32, nbw = NB / kCW;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float accs[4] = {0.f, 0.f, 0.f, 0.f};
  int red_buf = 0;
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
      // shared bf16 tile: 8 k16 steps of this warp's 128-wide slice
#pragma unroll 4
      for (int j = 0; j < 8; ++j) {
        const int k0 = cw * 128 + j * 16;
        const uint2 wa = *reinterpret_cast<const uint2*>(st + gq * g.sh_stride + (k0 + 4 * t) * 2);
        const uint2 wb = *reinterpret_cast<const uint2*>(st + (gq + 8) * g.sh_stride + (k0 + 4 * t) * 2);
        uint2 xv = make_uint2(0u, 0u);
        if (gq == 0) xv = *reinterpret_cast<const uint2*>(xb + y * kKTile + k0 + 4 * t);
        const uint32_t af[4] = {wa.x, wb.x, wa.y, wb.y};
        mma_bf16(accs, af, xv.x, xv.y, accs);
      }
    } else {
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      const uint8_t* sc = st + g.a_sc_off;
#pragma unroll 4
      for (int bb = 0; bb < nbw; ++bb) {
        const int blk = cw * nbw + bb;
        uint4 xv = make_uint4(0u, 0u, 0u, 0u);
        if (gq == 0) xv = *reinterpret_cast<const uint4*>(x16 + blk * 32 + t * 8);
        fp4_block_mma(st, g.a_ds, sc, g.a_ss, blk, gq, t, xv, acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);

    const bool unit_done = (kind == 1) || (y == L.KTs - 1);
    if (unit_done) {
      float* red = reinterpret_cast<float*>(smem + g.a_red_off) + red_buf * (kCW * 32 * 4);
      const float* src = kind == 1 ? acc : accs;
      reinterpret_cast<float4*>(red)[cw * 32 + lane] = make_float4(src[0], src[1], src[2], src[3]);
      bar_sync(1, kConsumerThreads);
      if (cw == 0 && t == 0) {
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) {
          const float4 v = reinterpret_cast<const float4*>(red)[w * 32 + lane];
          gs += v.x;
          us += v.z;
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
      red_buf ^= 1;
      if (kind == 0) accs[0] = accs[1] = accs[2] = accs[3] = 0.f;
    }
  }
}

// ============================================================== kernel B

__global__ void __launch_bounds__(kThreads, 1) moe_tc_down(const TcArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(8) uint64_t slots_bar;
  __shared__ SlotInfo slots;
  __shared__ float hred[kCW];

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
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane != 0) return;
    // ------------------------------------------------------------ producer
    // Routing is complete: the gate/up kernel triggers this launch only after
    // its own wait on the router.
    build_slots_t1(a, slots);
    mbar_arrive(&slots_bar);
    const int D = slots.count;
    const int np = (D + 1) / 2;
    const int per_unit = np + KTb;
    const DsExpertBank& w2 = a.d.w2;
    const uint32_t drow = g.I / 2, srow = g.I / 32;
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
        mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)nsl * 16u * (drow + srow));
        for (int q = 0; q < nsl; ++q) {
          const int e = slots.expert[s0 + q];
          uint8_t* d0 = dst + q * g.b_slot;
          for (int r = 0; r < 16; ++r) {
            const size_t row = (size_t)e * g.H + (size_t)rb * 16 + r;
            bulk_g2s(d0 + r * g.b_ds, static_cast<const uint8_t*>(w2.data) + row * drow, drow, &full_bar[stage]);
            bulk_g2s(d0 + 16 * g.b_ds + r * g.b_ss, static_cast<const uint8_t*>(w2.scales) + row * srow, srow,
                     &full_bar[stage]);
          }
        }
      } else {
        const int kt = j - np;
        mbar_arrive_expect_tx(&full_bar[stage], 16u * kKTile * 2);
        for (int r = 0; r < 16; ++r) {
          const size_t n = (size_t)rb * 16 + r;
          bulk_g2s(dst + r * g.sh_stride,
                   static_cast<const uint8_t*>(a.d.shared_w2) + (n * g.Is + (size_t)kt * kKTile) * 2, kKTile * 2,
                   &full_bar[stage]);
        }
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
  float m = 0.f;
  for (int k = tid; k < D * g.I; k += kConsumerThreads) {
    const int s = k / g.I, c = k - s * g.I;
    m = fmaxf(m, fabsf(a.h[(size_t)s * a.h_stride + c]));
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
  for (int k = tid; k < D * g.I; k += kConsumerThreads) {
    const int s = k / g.I, c = k - s * g.I;
    const float v = a.h[(size_t)s * a.h_stride + c] * hsc;
    const __half hi = __float2half_rn(v);
    hh[k] = hi;
    hl[k] = __float2half_rn(v - __half2float(hi));
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

  const int NB = g.I / 32, nbw = NB / 4;  // 4 warps per slot
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float accs[4] = {0.f, 0.f, 0.f, 0.f};
  int red_buf = 0;
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
      const int q = cw >> 2, kq = cw & 3;
      const int s = 2 * j + q;
      if (s < D) {
        const uint8_t* dat = st + q * g.b_slot;
        const uint8_t* sc = dat + 16 * g.b_ds;
        const __half* hhs = hh + (size_t)s * g.I;
        const __half* hls = hl + (size_t)s * g.I;
#pragma unroll 4
        for (int bb = 0; bb < nbw; ++bb) {
          const int blk = kq * nbw + bb;
          uint4 hv = make_uint4(0u, 0u, 0u, 0u), lv = make_uint4(0u, 0u, 0u, 0u);
          if (gq == 0) {
            hv = *reinterpret_cast<const uint4*>(hhs + blk * 32 + t * 8);
            lv = *reinterpret_cast<const uint4*>(hls + blk * 32 + t * 8);
          }
          fp4_block_mma2(dat, g.b_ds, sc, g.b_ss, blk, gq, t, hv, lv, acc);
        }
      }
    } else {
      const int kt = j - np;
#pragma unroll 4
      for (int jj = 0; jj < 8; ++jj) {
        const int k0 = cw * 128 + jj * 16;
        const uint2 wa = *reinterpret_cast<const uint2*>(st + gq * g.sh_stride + (k0 + 4 * t) * 2);
        const uint2 wb = *reinterpret_cast<const uint2*>(st + (gq + 8) * g.sh_stride + (k0 + 4 * t) * 2);
        uint2 hv = make_uint2(0u, 0u), lv = make_uint2(0u, 0u);
        if (gq == 0) {
          hv = *reinterpret_cast<const uint2*>(sh + kt * kKTile + k0 + 4 * t);
          lv = *reinterpret_cast<const uint2*>(sh + g.Is + kt * kKTile + k0 + 4 * t);
        }
        const uint32_t af[4] = {wa.x, wb.x, wa.y, wb.y};
        mma_bf16(accs, af, hv.x, hv.y, accs);
        mma_bf16(accs, af, lv.x, lv.y, accs);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);

    if (j == per_unit - 1) {
      float* red = reinterpret_cast<float*>(smem + g.b_red_off) + red_buf * (kCW * 32 * 8);
      reinterpret_cast<float4*>(red)[(cw * 32 + lane) * 2] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      reinterpret_cast<float4*>(red)[(cw * 32 + lane) * 2 + 1] = make_float4(accs[0], accs[1], accs[2], accs[3]);
      bar_sync(1, kConsumerThreads);
      if (cw == 0 && t == 0) {
        float r0 = 0.f, r8 = 0.f, s0 = 0.f, s8 = 0.f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) {
          const float4 v = reinterpret_cast<const float4*>(red)[(w * 32 + lane) * 2];
          const float4 u = reinterpret_cast<const float4*>(red)[(w * 32 + lane) * 2 + 1];
          r0 += v.x;
          r8 += v.z;
          s0 += u.x;
          s8 += u.z;
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
      red_buf ^= 1;
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      accs[0] = accs[1] = accs[2] = accs[3] = 0.f;
    }
  }
}

Geo make_geo(const DecodeArgs& a) {
  Geo g{};
  g.H = a.d.hidden;
  g.I = a.d.inter;
  g.shared = a.d.shared_w1 != nullptr;
  g.Is = g.shared ? a.d.shared_inter : 0;
  g.max_slots = a.max_slots;
  g.sh_stride = kKTile * 2 + kBf16Pad;
  // kernel A
  g.a_ds = g.H / 2 + kFp4Pad;
  g.a_ss = g.H / 32 + kFp4Pad;
  g.a_sc_off = 16 * g.a_ds;
  g.a_stage = std::max<uint32_t>(16 * (g.a_ds + g.a_ss), 16 * g.sh_stride);
  g.a_stage = (g.a_stage + 127) / 128 * 128;
  const uint32_t a_fixed = (uint32_t)g.H * 2 * 2 + 2 * kCW * 32 * 16 + 256;
  g.a_stages = std::min<int>(kMaxStages, (int)((kSmemLimit - a_fixed) / g.a_stage));
  g.a_x16_off = g.a_stages * g.a_stage;
  g.a_xb_off = g.a_x16_off + g.H * 2;
  g.a_red_off = g.a_xb_off + g.H * 2;
  g.a_total = g.a_red_off + 2 * kCW * 32 * 16;
  // kernel B
  g.b_ds = g.I / 2 + kFp4Pad;
  g.b_ss = g.I / 32 + kFp4Pad;
  g.b_slot = 16 * (g.b_ds + g.b_ss);
  g.b_stage = std::max<uint32_t>(2 * g.b_slot, 16 * g.sh_stride);
  g.b_stage = (g.b_stage + 127) / 128 * 128;
  const uint32_t h_bytes = (uint32_t)g.max_slots * g.I * 4 + (uint32_t)g.Is * 4;
  const uint32_t b_fixed = h_bytes + 2 * kCW * 32 * 32 + 256;
  g.b_stages = std::min<int>(kMaxStages, (int)((kSmemLimit - (int)b_fixed) / (int)g.b_stage));
  g.b_hh_off = g.b_stages * g.b_stage;
  g.b_hl_off = g.b_hh_off + (uint32_t)g.max_slots * g.I * 2;
  g.b_sh_off = g.b_hl_off + (uint32_t)g.max_slots * g.I * 2;
  g.b_red_off = g.b_sh_off + (uint32_t)g.Is * 4;
  g.b_red_off = (g.b_red_off + 15) / 16 * 16;
  g.b_total = g.b_red_off + 2 * kCW * 32 * 32;
  return g;
}

}  // namespace

bool tc_supported(const DecodeArgs& a) {
  const DsMoeDesc& d = a.d;
  if (a.tokens != 1 || a.x_f32 || d.w1.format != DS_FMT_FP4) return false;
  if (a.max_slots > kMaxSlots) return false;
  if (d.hidden % 1024 || d.inter % 512) return false;  // 16-byte scale rows, K slices per warp
  const bool sh = d.shared_w1 != nullptr;
  if (sh && (d.shared_inter % 1024)) return false;
  const Geo g = make_geo(a);
  if (g.a_stages < 2 || g.b_stages < 2) return false;
  if (g.a_total > (uint32_t)kSmemLimit || g.b_total > (uint32_t)kSmemLimit) return false;
  // bulk copies need 16-byte aligned sources
  if (!ds::aligned(d.w1.data, 16) || !ds::aligned(d.w3.data, 16) || !ds::aligned(d.w2.data, 16) ||
      !ds::aligned(d.w1.scales, 16) || !ds::aligned(d.w3.scales, 16) || !ds::aligned(d.w2.scales, 16))
    return false;
  if (sh && (!ds::aligned(d.shared_w1, 16) || !ds::aligned(d.shared_w3, 16) || !ds::aligned(d.shared_w2, 16)))
    return false;
  return true;
}

int launch_tc(const DecodeArgs& a, cudaStream_t st) {
  TcArgs p;
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

}  // namespace decode
}  // namespace ds
