// Decode MoE layer for 3-bit affine (q3) routed experts + the bf16 shared
// expert, 1..8 tokens, bf16 x, on CUDA cores with integer dot products.
//
// Every weight byte is read once per call:
//   * a CTA owns 64 output rows of one matrix (pair) at a time (8 per warp,
//     4 lanes per row); lane j of a row takes the 128-element segments
//     j, j+4, j+8, ... of the row (48 bytes of codes = three 16-byte loads,
//     plus one f16x2 of scales and one of biases);
//   * activations enter as int8 pieces per 64-value group: v ~ sx * (hi +
//     lo / 256), sx = max|v| / 127, hi = rint(v / sx), lo = rint(256 (v - sx
//     hi) / sx), i.e. about 15 significant bits, plus the group sum X of v;
//   * the planar q3 layout yields two codes per shift-and-mask in the two
//     16-bit halves of a register, which multiply two int8 pieces in one
//     dp2a (int16 x int8 pairs into an int32); a group contributes
//     s * sx * (Dhi + Dlo / 256) + b * X to its row;
//   * gate/up writes h (SwiGLU clamps, route weight before the down
//     projection) straight into pieces: the 64 rows of a work item are one
//     64-value group of the down projection's input;
//   * down sums two slots per work item into f32 partials; the combine
//     kernel adds the partials in slot order and the shared expert's output
//     rounded to bf16 (the reference's order).
// The shared expert (bf16) runs on f32 FMAs in the same kernels.  Three
// kernels chained with programmatic dependent launch.  The reference
// computes the layer with MLX's quantized_matmul over dequantised groups
// (src/deepseeker/mlx_forward.py:93-101, 257-419): w = f32(scale) q +
// f32(bias); the group math is regrouped here and the activations carry
// ~15 bits, which changes the result at the 1e-5 level.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "deepseeker_b200.h"
#include "ds_common.cuh"
#include "moe_decode.cuh"
#include "ptx.cuh"

namespace ds {
namespace decode {
namespace {

constexpr int kQT = 256;           // threads per CTA
constexpr int kRowsCta = 64;       // output rows per work item = one q3 group of the next projection
constexpr int kChunk = 2;          // routed slots per down work item
constexpr int kPk = 32;            // words of one (token, group) piece block: 16 hi + 16 lo
constexpr int kPkPad = 36;         // its stride in shared memory (16 bytes of padding: no bank conflicts)
constexpr int kShGU = 4;           // K quarters of a shared-expert gate/up item (partial g and u sums)
constexpr int kShDn = 2;           // K halves of a shared-expert down item (partial outputs)

__host__ __device__ constexpr int padded(int K) { return K + (K >> 7) * 4; }
__device__ __forceinline__ int pidx(int k) { return k + ((k >> 7) << 2); }

struct Q3Args {
  DecodeArgs a;
  uint32_t* hpk;     // routed h pieces [max_slots][T][I / 64][kPk]
  float2* hsx;       // routed h (sx, X) [max_slots][T][I / 64]
  float* hsh;        // shared gate/up partial sums [kShGU][T][2][Is] f32 (g, u)
  float* part;       // [max_chunks + kShDn][T][H] (chunks max_chunks..: shared expert halves)
  int max_chunks;
};

__device__ __forceinline__ float silu_glu_q3(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

// Codes of elements 16 wi + j (low half) and 16 wi + 8 + j (high half) of a
// group in the planar layout of oracle/q3.py: low word wi bits 2j / 16+2j,
// high word hw = word 4 + wi / 2 bits v8 + j / 16 + v8 + j (v8 = 8 (wi & 1)),
// the high bit moved to bit 2 by a compile-time shift once unrolled.
__device__ __forceinline__ uint32_t codes2(uint32_t lo, uint32_t hw, int v8, int j) {
  const int sh = v8 + j - 2;
  const uint32_t hb = (sh >= 0 ? (hw >> sh) : (hw << -sh)) & 0x00040004u;
  return ((lo >> (2 * j)) & 0x00030003u) | hb;
}

// Piece block of 16 values (one wi of a group): word p (p = 0..3) holds the
// int8 pieces of elements [16wi + 2p, 16wi + 8 + 2p, 16wi + 2p + 1,
// 16wi + 8 + 2p + 1], the operand order of dp2a.lo / dp2a.hi against the
// code pairs of j = 2p and j = 2p + 1.
__device__ __forceinline__ void make_pieces16(const float (&v)[16], float amax, uint32_t (&hi)[4], uint32_t (&lo)[4],
                                              float& sx) {
  sx = amax / 127.0f;
  const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
  int qh[16], ql[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int h = __float2int_rn(v[i] * inv);
    const float r = fmaf(-(float)h, sx, v[i]);
    const int l = __float2int_rn(r * (256.0f * inv));
    qh[i] = h;
    ql[i] = max(-127, min(127, l));
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int e0 = 2 * p, e1 = 8 + 2 * p, e2 = 2 * p + 1, e3 = 8 + 2 * p + 1;
    hi[p] = (uint32_t)(qh[e0] & 0xFF) | ((uint32_t)(qh[e1] & 0xFF) << 8) | ((uint32_t)(qh[e2] & 0xFF) << 16) |
            ((uint32_t)(qh[e3] & 0xFF) << 24);
    lo[p] = (uint32_t)(ql[e0] & 0xFF) | ((uint32_t)(ql[e1] & 0xFF) << 8) | ((uint32_t)(ql[e2] & 0xFF) << 16) |
            ((uint32_t)(ql[e3] & 0xFF) << 24);
  }
}

// Pieces of T rows of K bf16 values (row stride src_stride) into blocks
// dst[t][g] (stride kPkPad words) and (sx, X) into sxx[t][g].  A quad of
// threads builds one group (one wi each); the loop bound is a multiple of
// 32, so whole warps take part in the quad shuffles.
__device__ void pieces_rows_bf16(const __nv_bfloat16* src, int T, int K, int src_stride, uint32_t* dst, float2* sxx) {
  const int G = K / 64, n = T * G * 4;
  for (int i = threadIdx.x; i < (n + 31) / 32 * 32; i += blockDim.x) {
    const bool live = i < n;
    const int wi = i & 3, tg = live ? (i >> 2) : 0, t = tg / G, g = tg % G;
    float v[16];
    const uint4* p = reinterpret_cast<const uint4*>(src + (size_t)t * src_stride + 64 * g + 16 * wi);
    const uint4 a = p[0], b = p[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      v[2 * k] = __uint_as_float(w[k] << 16);
      v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
    float am = 0.0f, sum = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      am = fmaxf(am, fabsf(v[k]));
      sum += v[k];
    }
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    uint32_t hi[4], lo[4];
    float sx;
    make_pieces16(v, am, hi, lo, sx);
    if (live) {
      uint32_t* d = dst + (size_t)tg * kPkPad;
      *reinterpret_cast<uint4*>(d + 4 * wi) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(d + 16 + 4 * wi) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      if (wi == 0) sxx[tg] = make_float2(sx, sum);
    }
  }
}

// One group of 64 codes against the pieces block pk (hi words 0..15, lo
// 16..31): returns Dhi + Dlo / 256 (exact integers, then one f32 step).
__device__ __forceinline__ float group_dot(const uint32_t (&w)[6], const uint32_t* pk) {
  int dh = 0, dl = 0;
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    const uint4 h = *reinterpret_cast<const uint4*>(pk + 4 * wi);
    const uint4 l = *reinterpret_cast<const uint4*>(pk + 16 + 4 * wi);
    const uint32_t hv[4] = {h.x, h.y, h.z, h.w}, lv[4] = {l.x, l.y, l.z, l.w};
    const uint32_t lw = w[wi], hw = w[4 + (wi >> 1)];
    const int v8 = (wi & 1) * 8;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int c0 = (int)codes2(lw, hw, v8, 2 * p), c1 = (int)codes2(lw, hw, v8, 2 * p + 1);
      dh = __dp2a_lo(c0, (int)hv[p], dh);
      dh = __dp2a_hi(c1, (int)hv[p], dh);
      dl = __dp2a_lo(c0, (int)lv[p], dl);
      dl = __dp2a_hi(c1, (int)lv[p], dl);
    }
  }
  return (float)dh + (float)dl * (1.0f / 256.0f);
}

__device__ __forceinline__ void words_of(const uint4& u0, const uint4& u1, const uint4& u2, uint32_t (&g0)[6],
                                         uint32_t (&g1)[6]) {
  g0[0] = u0.x; g0[1] = u0.y; g0[2] = u0.z; g0[3] = u0.w; g0[4] = u1.x; g0[5] = u1.y;
  g1[0] = u1.z; g1[1] = u1.w; g1[2] = u2.x; g1[3] = u2.y; g1[4] = u2.z; g1[5] = u2.w;
}

// sum of the 4 lanes of a row (lanes 4r .. 4r+3), fixed order
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// bf16 row segment (32 values = four 16-byte words) dot bf16 values (four
// 16-byte words, read through L1)
__device__ __forceinline__ float bf16_dot32_bf16(const uint4 (&v)[4], const uint4* xg) {
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 xv = __ldg(xg + c);
    const uint32_t aw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s = fmaf(__uint_as_float(aw[k] << 16), __uint_as_float(xw[k] << 16), s);
      s = fmaf(__uint_as_float(aw[k] & 0xFFFF0000u), __uint_as_float(xw[k] & 0xFFFF0000u), s);
    }
  }
  return s;
}

// bf16 row segment (32 values = four 16-byte words) dot f32 values xs[0..31]
__device__ __forceinline__ float bf16_dot32(const uint4 (&v)[4], const float* xs) {
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 xa = *reinterpret_cast<const float4*>(xs + 8 * c);
    const float4 xb = *reinterpret_cast<const float4*>(xs + 8 * c + 4);
    const uint32_t aw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    const float xx[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s = fmaf(__uint_as_float(aw[k] << 16), xx[2 * k], s);
      s = fmaf(__uint_as_float(aw[k] & 0xFFFF0000u), xx[2 * k + 1], s);
    }
  }
  return s;
}

// ------------------------------------------------------------------ gate/up

template <int NT>
__global__ void __launch_bounds__(kQT, 2) q3_gate_up_kernel(const Q3Args q) {
  ptx::wait_prior_grid();
  ptx::launch_dependents();
  const DecodeArgs& a = q.a;
  extern __shared__ float4 smem4[];
  __shared__ Slots slots;
  __shared__ float hrow[8][kRowsCta];            // h of the item's 64 rows per token
  const int H = a.d.hidden, I = a.d.inter, T = a.tokens, G = H / 64;
  const bool has_shared = a.d.shared_w1 != nullptr;
  const int Is = has_shared ? a.d.shared_inter : 0;
  uint32_t* xpk = reinterpret_cast<uint32_t*>(smem4);                     // [T][G][kPkPad]
  float2* xsx = reinterpret_cast<float2*>(xpk + (size_t)T * G * kPkPad);  // [T][G]
  pieces_rows_bf16(static_cast<const __nv_bfloat16*>(a.x), T, H, H, xpk, xsx);
  build_slots(a, slots);                         // ends with __syncthreads

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 3;
  const int r_in = warp * 8 + (lane >> 2);       // row within the item
  const int D = slots.count;
  const int rb_r = I / kRowsCta, rb_s = Is / kRowsCta;
  // shared-expert items cover a quarter of K each, so that they weigh about
  // what a routed item weighs (bf16 rows are 5.3x the bytes of q3 rows)
  const int items = D * rb_r + rb_s * kShGU;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const bool routed = item < D * rb_r;
    float acc1[NT], acc3[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc1[t] = acc3[t] = 0.0f;
    int slot, rb;
    uint32_t mask;
    if (routed) {
      slot = item / rb_r;
      rb = item % rb_r;
      mask = slots.mask[slot];
      const int e = slots.expert[slot];
      const size_t rbytes = (size_t)H * 3 / 8;
      const size_t r = (size_t)e * I + rb * kRowsCta + r_in;
      const uint8_t* w1 = static_cast<const uint8_t*>(a.d.w1.data) + r * rbytes;
      const uint8_t* w3 = static_cast<const uint8_t*>(a.d.w3.data) + r * rbytes;
      const __half2* s1 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w1.scales) + r * G);
      const __half2* b1 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w1.biases) + r * G);
      const __half2* s3 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w3.scales) + r * G);
      const __half2* b3 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w3.biases) + r * G);
      for (int seg = j; seg < H / 128; seg += 4) {
        const uint4* p1 = reinterpret_cast<const uint4*>(w1 + (size_t)seg * 48);
        const uint4* p3 = reinterpret_cast<const uint4*>(w3 + (size_t)seg * 48);
        const uint4 u10 = __ldcs(p1), u11 = __ldcs(p1 + 1), u12 = __ldcs(p1 + 2);
        const uint4 u30 = __ldcs(p3), u31 = __ldcs(p3 + 1), u32 = __ldcs(p3 + 2);
        const float2 sc1 = __half22float2(__ldcs(s1 + seg)), bi1 = __half22float2(__ldcs(b1 + seg));
        const float2 sc3 = __half22float2(__ldcs(s3 + seg)), bi3 = __half22float2(__ldcs(b3 + seg));
        uint32_t g10[6], g11[6], g30[6], g31[6];
        words_of(u10, u11, u12, g10, g11);
        words_of(u30, u31, u32, g30, g31);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int g = 2 * seg + hh;
          const float sa = hh ? sc1.y : sc1.x, ba = hh ? bi1.y : bi1.x;
          const float sb = hh ? sc3.y : sc3.x, bb = hh ? bi3.y : bi3.x;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (!((mask >> t) & 1u)) continue;
            const uint32_t* pk = xpk + ((size_t)t * G + g) * kPkPad;
            const float2 sxx = xsx[t * G + g];
            const float d1 = group_dot(hh ? g11 : g10, pk), d3 = group_dot(hh ? g31 : g30, pk);
            acc1[t] = fmaf(sa * sxx.x, d1, fmaf(ba, sxx.y, acc1[t]));
            acc3[t] = fmaf(sb * sxx.x, d3, fmaf(bb, sxx.y, acc3[t]));
          }
        }
      }
    } else {
      // shared expert (bf16 rows of H), all tokens, f32 FMAs, K quarter kq
      slot = -1;
      rb = (item - D * rb_r) / kShGU;
      const int kq = (item - D * rb_r) % kShGU;
      mask = (1u << T) - 1u;
      const int row = rb * kRowsCta + r_in;
      const uint4* w1 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.d.shared_w1) +
                                                       (size_t)row * H);
      const uint4* w3 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.d.shared_w3) +
                                                       (size_t)row * H);
      const int nseg = H / 32 / kShGU;
      for (int seg = kq * nseg + j; seg < (kq + 1) * nseg; seg += 4) {
        uint4 v1[4], v3[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v1[c] = __ldcs(w1 + seg * 4 + c);
          v3[c] = __ldcs(w3 + seg * 4 + c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= T) continue;
          const uint4* xg = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) + (size_t)t * H) +
                            seg * 4;
          acc1[t] += bf16_dot32_bf16(v1, xg);
          acc3[t] += bf16_dot32_bf16(v3, xg);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc1[t] = quad_sum(acc1[t]);
      acc3[t] = quad_sum(acc3[t]);
    }
    if (!routed) {
      // partial g and u of K quarter kq; the down kernel sums the quarters
      // in order and applies the SwiGLU when it stages h
      if (j == 0) {
        const int kq = (item - D * rb_r) % kShGU;
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < T) {
            float* hp = q.hsh + ((size_t)(kq * T + t) * 2) * Is + rb * kRowsCta + r_in;
            hp[0] = acc1[t];
            hp[Is] = acc3[t];
          }
      }
      continue;
    }
    // routed: h of the 64 rows -> smem -> one piece block per token (the
    // rows are group rb of the down projection's input)
    if (j == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= T) continue;
        float hv = 0.0f;
        if ((mask >> t) & 1u) {
          hv = silu_glu_q3(acc1[t], acc3[t], a.d.swiglu_limit);
          if (a.d.route_before_down) hv *= slots.gate[slot][t];
        }
        hrow[t][r_in] = hv;
      }
    }
    __syncthreads();
    // T x 4 threads (quads) build the token blocks; the bound is a multiple
    // of 32 so whole warps take part in the quad shuffles
    for (int i = threadIdx.x; i < ((T * 4 + 31) / 32) * 32; i += blockDim.x) {
      const bool live = i < T * 4;
      const int t = live ? (i >> 2) : 0, wi = i & 3;
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = hrow[t][16 * wi + k];
      float am = 0.0f, sum = 0.0f;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        am = fmaxf(am, fabsf(v[k]));
        sum += v[k];
      }
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      uint32_t hi[4], lo[4];
      float sx;
      make_pieces16(v, am, hi, lo, sx);
      if (live) {
        const size_t blk = ((size_t)slot * T + t) * (I / 64) + rb;
        uint32_t* d = q.hpk + blk * kPk;
        *reinterpret_cast<uint4*>(d + 4 * wi) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(d + 16 + 4 * wi) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        if (wi == 0) q.hsx[blk] = make_float2(sx, sum);
      }
    }
    __syncthreads();                             // hrow is rewritten by the next item
  }
}

// ------------------------------------------------------------------ down

template <int NT>
__global__ void __launch_bounds__(kQT, 2) q3_down_kernel(const Q3Args q) {
  ptx::wait_prior_grid();
  ptx::launch_dependents();
  const DecodeArgs& a = q.a;
  extern __shared__ float4 smem4[];
  __shared__ Slots slots;
  build_slots(a, slots);
  const int H = a.d.hidden, I = a.d.inter, T = a.tokens, G = I / 64;
  const bool has_shared = a.d.shared_w2 != nullptr;
  const int Is = has_shared ? a.d.shared_inter : 0;
  const int Isp = padded(Is);
  uint32_t* hpk = reinterpret_cast<uint32_t*>(smem4);                              // [kChunk][T][G][kPkPad]
  float2* hsx = reinterpret_cast<float2*>(hpk + (size_t)kChunk * T * G * kPkPad);  // [kChunk][T][G]
  float* hs = reinterpret_cast<float*>(smem4);                                     // shared items: [T][Isp]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 3;
  const int D = slots.count;
  const int n_chunks = (D + kChunk - 1) / kChunk;
  const int n_rb = H / kRowsCta;
  const int items = (n_chunks + (has_shared ? kShDn : 0)) * n_rb;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int c = item / n_rb, rb = item % n_rb;
    const bool routed = c < n_chunks;
    const int hf = routed ? 0 : c - n_chunks;    // shared expert: K half
    const int row = rb * kRowsCta + warp * 8 + (lane >> 2);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    __syncthreads();                             // previous item's readers are done with the staging area
    if (routed) {
      const int nsl = min(kChunk, D - c * kChunk);
      const int nblk = nsl * T * G;
      const uint32_t* src = q.hpk + (size_t)c * kChunk * T * G * kPk;
      for (int i = threadIdx.x; i < nblk * (kPk / 4); i += blockDim.x) {
        const int blk = i / (kPk / 4), w4 = i % (kPk / 4);
        *reinterpret_cast<uint4*>(hpk + (size_t)blk * kPkPad + 4 * w4) =
            *reinterpret_cast<const uint4*>(src + (size_t)blk * kPk + 4 * w4);
      }
      for (int i = threadIdx.x; i < nblk; i += blockDim.x) hsx[i] = q.hsx[(size_t)c * kChunk * T * G + i];
    } else {
      // h of the shared expert = SwiGLU of the K-quarter sums (in order)
      for (int i = threadIdx.x; i < T * (Is / 4); i += blockDim.x) {
        const int t = i / (Is / 4), k = (i % (Is / 4)) * 4;
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
        for (int kq = 0; kq < kShGU; ++kq) {
          const float* hp = q.hsh + ((size_t)(kq * T + t) * 2) * Is + k;
          const float4 gg = *reinterpret_cast<const float4*>(hp);
          const float4 uu = *reinterpret_cast<const float4*>(hp + Is);
          g.x += gg.x; g.y += gg.y; g.z += gg.z; g.w += gg.w;
          u.x += uu.x; u.y += uu.y; u.z += uu.z; u.w += uu.w;
        }
        *reinterpret_cast<float4*>(hs + t * Isp + pidx(k)) =
            make_float4(silu_glu_q3(g.x, u.x, 10.0f), silu_glu_q3(g.y, u.y, 10.0f), silu_glu_q3(g.z, u.z, 10.0f),
                        silu_glu_q3(g.w, u.w, 10.0f));
      }
    }
    __syncthreads();
    if (routed) {
      for (int ci = 0; ci < kChunk && c * kChunk + ci < D; ++ci) {
        const int slot = c * kChunk + ci;
        const uint32_t mask = slots.mask[slot];
        const int e = slots.expert[slot];
        const size_t r = (size_t)e * H + row;
        const uint8_t* w = static_cast<const uint8_t*>(a.d.w2.data) + r * ((size_t)I * 3 / 8);
        const __half2* sc = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w2.scales) + r * G);
        const __half2* bi = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w2.biases) + r * G);
        float part[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) part[t] = 0.0f;
        for (int seg = j; seg < I / 128; seg += 4) {
          const uint4* p = reinterpret_cast<const uint4*>(w + (size_t)seg * 48);
          const uint4 u0 = __ldcs(p), u1 = __ldcs(p + 1), u2 = __ldcs(p + 2);
          const float2 s2 = __half22float2(__ldcs(sc + seg)), b2 = __half22float2(__ldcs(bi + seg));
          uint32_t g0[6], g1[6];
          words_of(u0, u1, u2, g0, g1);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int g = 2 * seg + hh;
            const float s = hh ? s2.y : s2.x, b = hh ? b2.y : b2.x;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (!((mask >> t) & 1u)) continue;
              const size_t blk = ((size_t)ci * T + t) * G + g;
              const float2 sxy = hsx[blk];
              const float d = group_dot(hh ? g1 : g0, hpk + blk * kPkPad);
              part[t] = fmaf(s * sxy.x, d, fmaf(b, sxy.y, part[t]));
            }
          }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (!((mask >> t) & 1u)) continue;
          // route_before_down == 0: the gate multiplies the down output
          acc[t] += a.d.route_before_down ? part[t] : part[t] * slots.gate[slot][t];
        }
      }
    } else {
      // row stride of W2: the full shared inter when this call holds a
      // column slice of it (expert-parallel ranks), else Is
      const size_t ld = a.sh_w2_ld > 0 ? (size_t)a.sh_w2_ld : (size_t)Is;
      const uint4* w = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.d.shared_w2) + row * ld);
      const int nseg = Is / 32 / kShDn;
      for (int seg = hf * nseg + j; seg < (hf + 1) * nseg; seg += 4) {
        uint4 v[4];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) v[cc] = __ldcs(w + seg * 4 + cc);
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < T) acc[t] += bf16_dot32(v, hs + t * Isp + pidx(32 * seg));
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = quad_sum(acc[t]);
    if (j == 0) {
      const int cc = routed ? c : q.max_chunks + hf;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < T) q.part[((size_t)cc * T + t) * H + row] = acc[t];
    }
  }
}

// ------------------------------------------------------------------ combine

__global__ void __launch_bounds__(kQT) q3_combine_kernel(const Q3Args q) {
  ptx::wait_prior_grid();
  ptx::launch_dependents();
  const DecodeArgs& a = q.a;
  __shared__ Slots slots;
  build_slots(a, slots);
  const int H = a.d.hidden, T = a.tokens;
  const int n_chunks = (slots.count + kChunk - 1) / kChunk;
  const bool has_shared = a.d.shared_w2 != nullptr;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * H) return;
  const int t = i / H, n = i % H;
  float acc = 0.0f;
  for (int c = 0; c < n_chunks; ++c) acc += q.part[((size_t)c * T + t) * H + n];
  if (has_shared) {
    float sh = 0.0f;
    for (int hf = 0; hf < kShDn; ++hf) sh += q.part[((size_t)(q.max_chunks + hf) * T + t) * H + n];
    if (a.out_sh != nullptr) a.out_sh[i] = sh;                  // summed over ranks by the caller
    else if (t >= a.sh_row0 && t < a.sh_row1) acc += __bfloat162float(__float2bfloat16_rn(sh));
  }
  if (a.d.out_f32) static_cast<float*>(a.out)[i] = acc;
  else static_cast<__nv_bfloat16*>(a.out)[i] = __float2bfloat16_rn(acc);
}

struct Q3Layout {
  size_t hpk, hsx, hsh, part, total;
  int max_chunks;
};

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

Q3Layout q3_layout(const DsMoeDesc& d, int T) {
  Q3Layout L;
  const int S = std::min(T * d.top_k, d.n_experts);
  const int Is = d.shared_w1 ? d.shared_inter : 0;
  L.max_chunks = (S + kChunk - 1) / kChunk;
  const size_t blocks = (size_t)L.max_chunks * kChunk * T * (d.inter / 64);
  size_t o = kWsReserved;                         // error word (offset 0), reserved control block
  L.hpk = o;  o += up256(blocks * kPk * 4);
  L.hsx = o;  o += up256(blocks * sizeof(float2));
  L.hsh = o;  o += up256((size_t)kShGU * T * 2 * Is * 4);
  L.part = o; o += up256((size_t)(L.max_chunks + kShDn) * T * d.hidden * 4);
  L.total = o;
  return L;
}

size_t smem_gate_up(const DsMoeDesc& d, int T) {
  const int G = d.hidden / 64;
  return (size_t)T * G * kPkPad * 4 + (size_t)T * G * sizeof(float2);
}

size_t smem_down(const DsMoeDesc& d, int T) {
  const int Is = d.shared_w1 ? d.shared_inter : 0;
  const int G = d.inter / 64;
  const size_t routed = (size_t)kChunk * T * G * kPkPad * 4 + (size_t)kChunk * T * G * sizeof(float2);
  return std::max(routed, (size_t)T * padded(Is) * 4);
}

template <int NT>
int launch_nt(const Q3Args& q, cudaStream_t st) {
  const DsMoeDesc& d = q.a.d;
  const int T = q.a.tokens;
  const size_t sm_a = smem_gate_up(d, T), sm_b = smem_down(d, T);
  static std::mutex mu;
  static bool configured = false;
  static int occ_a = 1, occ_b = 1;
  static size_t cfg_a = 0, cfg_b = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured) {
      DS_CHECK_CUDA(cudaFuncSetAttribute(q3_gate_up_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024));
      DS_CHECK_CUDA(cudaFuncSetAttribute(q3_down_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024));
      configured = true;
    }
    if (cfg_a != sm_a) {
      DS_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_a, q3_gate_up_kernel<NT>, kQT, sm_a));
      cfg_a = sm_a;
    }
    if (cfg_b != sm_b) {
      DS_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_b, q3_down_kernel<NT>, kQT, sm_b));
      cfg_b = sm_b;
    }
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(kQT);
  cfg.gridDim = dim3(ds::sm_count() * std::max(1, occ_a));
  cfg.dynamicSmemBytes = sm_a;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, q3_gate_up_kernel<NT>, q));
  cfg.gridDim = dim3(ds::sm_count() * std::max(1, occ_b));
  cfg.dynamicSmemBytes = sm_b;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, q3_down_kernel<NT>, q));
  cfg.gridDim = dim3((T * d.hidden + kQT - 1) / kQT);
  cfg.dynamicSmemBytes = 0;
  DS_CHECK_CUDA(cudaLaunchKernelEx(&cfg, q3_combine_kernel, q));
  return DS_OK;
}

}  // namespace

bool q3_supported(const DecodeArgs& a) {
  const DsMoeDesc& d = a.d;
  if (a.x_f32 || d.w1.format != DS_FMT_Q3 || a.tokens < 1 || a.tokens > 8) return false;
  if (d.hidden % 128 != 0 || d.inter % 128 != 0) return false;
  const bool sh = d.shared_w1 != nullptr;
  if (sh && (d.shared_inter % 128 != 0)) return false;
  if (!ds::aligned(a.x, 16) || !ds::aligned(d.w1.data, 16) || !ds::aligned(d.w3.data, 16) ||
      !ds::aligned(d.w2.data, 16))
    return false;
  for (const DsExpertBank* b : {&d.w1, &d.w3, &d.w2})
    if (!ds::aligned(b->scales, 4) || !ds::aligned(b->biases, 4)) return false;
  if (sh && (!ds::aligned(d.shared_w1, 16) || !ds::aligned(d.shared_w3, 16) || !ds::aligned(d.shared_w2, 16)))
    return false;
  if (smem_gate_up(d, a.tokens) > 200 * 1024 || smem_down(d, a.tokens) > 200 * 1024) return false;
  return true;
}

size_t q3_workspace_bytes(const DsMoeDesc& d, int tokens) { return q3_layout(d, tokens).total; }

int launch_q3(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const Q3Layout L = q3_layout(a.d, a.tokens);
  DS_REQUIRE(workspace_bytes >= L.total, DS_EINVAL, "moe_decode: workspace %zu bytes < %zu (q3 path)",
             workspace_bytes, L.total);
  char* ws = static_cast<char*>(workspace);
  Q3Args q;
  q.a = a;
  q.a.err = reinterpret_cast<int*>(ws);
  q.a.max_slots = std::min(a.tokens * a.d.top_k, a.d.n_experts);
  q.hpk = reinterpret_cast<uint32_t*>(ws + L.hpk);
  q.hsx = reinterpret_cast<float2*>(ws + L.hsx);
  q.hsh = reinterpret_cast<float*>(ws + L.hsh);
  q.part = reinterpret_cast<float*>(ws + L.part);
  q.max_chunks = L.max_chunks;
  if (a.tokens == 1) return launch_nt<1>(q, st);
  if (a.tokens == 2) return launch_nt<2>(q, st);
  if (a.tokens <= 4) return launch_nt<4>(q, st);
  return launch_nt<8>(q, st);
}

}  // namespace decode
}  // namespace ds
