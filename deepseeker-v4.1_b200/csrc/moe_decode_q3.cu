// Decode MoE layer for 3-bit affine (q3) routed experts + the bf16 shared
// expert, 1..8 tokens, bf16 x, on CUDA cores.
//
// Every weight byte is read once per call and the dot products run at the
// rate the bytes arrive:
//   * a CTA owns 64 output rows of one matrix pair at a time (8 per warp,
//     4 lanes per row); lane j of a row takes the 128-element segments
//     j, j+4, j+8, ... of the row (48 bytes of codes = three 16-byte loads,
//     plus one f16x2 of scales and of biases), so a warp's loads cover whole
//     rows and the four lanes of a row read different 512-byte stretches of
//     the staged activations (padded by 16 bytes per 128 values: no bank
//     conflicts);
//   * two codes come out of the planar q3 layout per shift-and-mask into the
//     two halves of an f16x2 whose bits are those of 1024 + q; one f16x2
//     subtraction of 1024 leaves q exactly, widened to f32;
//   * the group term is s * sum(q x) + b * sum(x) (sums over the 64 values of
//     the group, the activation sums computed once per call);
//   * gate/up writes h (SwiGLU clamps, route weight before the down
//     projection) per (slot, token, row); down sums two slots per work item
//     into f32 partials; the combine kernel adds the partials in slot order
//     and the shared expert's output rounded to bf16 (the reference's order).
// Three kernels chained with programmatic dependent launch.  The reference
// computes the same layer with MLX's quantized_matmul over dequantised
// groups (src/deepseeker/mlx_forward.py:93-101, 257-419); the group math
// w = f32(scale) q + f32(bias) is regrouped here, which changes float
// rounding only.
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
constexpr int kRowsCta = 64;       // output rows per work item (8 warps x 8 rows)
constexpr int kChunk = 2;          // routed slots per down work item

__host__ __device__ constexpr int padded(int K) { return K + (K >> 7) * 4; }
__device__ __forceinline__ int pidx(int k) { return k + ((k >> 7) << 2); }

struct Q3Args {
  DecodeArgs a;
  float* h;          // [max_slots + 1][T][h_stride] (row max_slots: shared expert)
  float* part;       // [max_chunks + 1][T][H] (chunk max_chunks: shared expert)
  int h_stride, max_chunks;
};

__device__ __forceinline__ float silu_glu_q3(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

// q (exact, as f32) for the 16 codes of low word wi of a group: out[j] = element
// 16 wi + j, out[8 + j] = element 16 wi + 8 + j (planar layout of
// oracle/q3.py).  hw = high word 4 + wi / 2, v8 = 8 (wi & 1); bits v8 + j
// and 16 + v8 + j of hw move to bits 2 and 18 (a right or left shift by a
// compile-time amount once unrolled).
__device__ __forceinline__ void codes16(uint32_t lo, uint32_t hw, int v8, float (&out)[16]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int sh = v8 + j - 2;
    const uint32_t hb = sh >= 0 ? (hw >> sh) : (hw << -sh);
    const uint32_t bits = ((lo >> (2 * j)) & 0x00030003u) | (hb & 0x00040004u) | 0x64006400u;
    const float2 f = __half22float2(__hsub2(*reinterpret_cast<const __half2*>(&bits), __float2half2_rn(1024.0f)));
    out[j] = f.x;
    out[8 + j] = f.y;
  }
}

// Group of 64: S1[t] += sum q1 x_t, S3[t] += sum q3 x_t for
// the tokens in mask; xg = group start in token 0's padded row.
template <int NT>
__device__ __forceinline__ void group_pair(const uint32_t (&w1)[6], const uint32_t (&w3)[6], const float* xg,
                                           int xstride, uint32_t mask, float (&S1)[NT], float (&S3)[NT]) {
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    float f1[16], f3[16];
    codes16(w1[wi], w1[4 + (wi >> 1)], (wi & 1) * 8, f1);
    codes16(w3[wi], w3[4 + (wi >> 1)], (wi & 1) * 8, f3);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (!((mask >> t) & 1u)) continue;
      const float4* xv = reinterpret_cast<const float4*>(xg + t * xstride) + 4 * wi;
      const float4 a = xv[0], b = xv[1], c = xv[2], d = xv[3];
      const float x[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
      float s1 = S1[t], s3 = S3[t];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        s1 = fmaf(f1[j], x[j], s1);
        s3 = fmaf(f3[j], x[j], s3);
      }
      S1[t] = s1;
      S3[t] = s3;
    }
  }
}

// Group of 64: D[t] += sum q h_t (down projection).
template <int NT>
__device__ __forceinline__ void group_one(const uint32_t (&w)[6], const float* hg, int hstride, uint32_t mask,
                                          float (&D)[NT]) {
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    float f[16];
    codes16(w[wi], w[4 + (wi >> 1)], (wi & 1) * 8, f);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (!((mask >> t) & 1u)) continue;
      const float4* hv = reinterpret_cast<const float4*>(hg + t * hstride) + 4 * wi;
      const float4 a = hv[0], b = hv[1], c = hv[2], d = hv[3];
      const float x[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
      float s = D[t];
#pragma unroll
      for (int j = 0; j < 16; ++j) s = fmaf(f[j], x[j], s);
      D[t] = s;
    }
  }
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

// T rows of K f32 values -> padded smem rows + group sums (64 per group).
__device__ void stage_rows(const float* src, int T, int K, int src_stride, float* dst, float* gsum) {
  const int Kp = padded(K);
  for (int i = threadIdx.x; i < T * (K / 4); i += blockDim.x) {
    const int t = i / (K / 4), k = (i % (K / 4)) * 4;
    *reinterpret_cast<float4*>(dst + t * Kp + pidx(k)) =
        *reinterpret_cast<const float4*>(src + (size_t)t * src_stride + k);
  }
  __syncthreads();
  if (gsum != nullptr)
    for (int i = threadIdx.x; i < T * (K / 64); i += blockDim.x) {
      const int t = i / (K / 64), g = i % (K / 64);
      const float* p = dst + t * Kp + pidx(64 * g);
      float s = 0.0f;
      for (int k = 0; k < 64; ++k) s += p[k];
      gsum[i] = s;
    }
}

// ------------------------------------------------------------------ gate/up

template <int NT>
__global__ void __launch_bounds__(kQT, 2) q3_gate_up_kernel(const Q3Args q) {
  ptx::wait_prior_grid();
  ptx::launch_dependents();
  const DecodeArgs& a = q.a;
  extern __shared__ float4 smem4[];
  __shared__ Slots slots;
  const int H = a.d.hidden, I = a.d.inter, T = a.tokens, Hp = padded(H);
  float* xs = reinterpret_cast<float*>(smem4);   // [T][Hp]
  float* xsum = xs + T * Hp;                     // [T][H / 64]
  {
    // bf16 x -> padded f32 rows
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x);
    for (int i = threadIdx.x; i < T * (H / 8); i += blockDim.x) {
      const int t = i / (H / 8), k = (i % (H / 8)) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)t * H + k);
      float* d = xs + t * Hp + pidx(k);
      *reinterpret_cast<float4*>(d) = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                                  __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
      *reinterpret_cast<float4*>(d + 4) = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xFFFF0000u),
                                                      __uint_as_float(u.w << 16), __uint_as_float(u.w & 0xFFFF0000u));
    }
  }
  build_slots(a, slots);                         // ends with __syncthreads
  for (int i = threadIdx.x; i < T * (H / 64); i += blockDim.x) {
    const int t = i / (H / 64), g = i % (H / 64);
    const float* p = xs + t * Hp + pidx(64 * g);
    float s = 0.0f;
    for (int k = 0; k < 64; ++k) s += p[k];
    xsum[i] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 3;
  const int D = slots.count;
  const bool has_shared = a.d.shared_w1 != nullptr;
  const int Is = has_shared ? a.d.shared_inter : 0;
  const int rb_r = I / kRowsCta, rb_s = Is / kRowsCta;
  const int items = D * rb_r + rb_s;
  const uint32_t all = (1u << T) - 1u;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const bool routed = item < D * rb_r;
    float acc1[NT], acc3[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc1[t] = acc3[t] = 0.0f;
    int slot, row;
    uint32_t mask;
    if (routed) {
      slot = item / rb_r;
      row = (item % rb_r) * kRowsCta + warp * 8 + (lane >> 2);
      mask = slots.mask[slot];
      const int e = slots.expert[slot];
      const size_t rbytes = (size_t)H * 3 / 8;
      const size_t r = (size_t)e * I + row;
      const uint8_t* w1 = static_cast<const uint8_t*>(a.d.w1.data) + r * rbytes;
      const uint8_t* w3 = static_cast<const uint8_t*>(a.d.w3.data) + r * rbytes;
      const __half2* s1 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w1.scales) + r * (H / 64));
      const __half2* b1 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w1.biases) + r * (H / 64));
      const __half2* s3 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w3.scales) + r * (H / 64));
      const __half2* b3 = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w3.biases) + r * (H / 64));
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
        for (int h = 0; h < 2; ++h) {
          const int g = 2 * seg + h;
          float S1[NT], S3[NT];
#pragma unroll
          for (int t = 0; t < NT; ++t) S1[t] = S3[t] = 0.0f;
          group_pair<NT>(h ? g11 : g10, h ? g31 : g30, xs + pidx(64 * g), Hp, mask, S1, S3);
          const float sa = h ? sc1.y : sc1.x, ba = h ? bi1.y : bi1.x;
          const float sb = h ? sc3.y : sc3.x, bb = h ? bi3.y : bi3.x;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (!((mask >> t) & 1u)) continue;
            const float X = xsum[t * (H / 64) + g];
            acc1[t] = fmaf(sa, S1[t], fmaf(ba, X, acc1[t]));
            acc3[t] = fmaf(sb, S3[t], fmaf(bb, X, acc3[t]));
          }
        }
      }
    } else {
      // shared expert (bf16 rows of H), all tokens
      slot = a.max_slots;
      row = (item - D * rb_r) * kRowsCta + warp * 8 + (lane >> 2);
      mask = all;
      const uint4* w1 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.d.shared_w1) +
                                                       (size_t)row * H);
      const uint4* w3 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.d.shared_w3) +
                                                       (size_t)row * H);
      for (int seg = j; seg < H / 32; seg += 4) {       // 32 values = four 16-byte loads per matrix
        uint4 v1[4], v3[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v1[c] = __ldcs(w1 + seg * 4 + c);
          v3[c] = __ldcs(w3 + seg * 4 + c);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= T) continue;
          const float4* xv = reinterpret_cast<const float4*>(xs + t * Hp + pidx(32 * seg));
          float s1 = acc1[t], s3 = acc3[t];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 xa = xv[2 * c], xb = xv[2 * c + 1];
            const uint32_t a1[4] = {v1[c].x, v1[c].y, v1[c].z, v1[c].w};
            const uint32_t a3[4] = {v3[c].x, v3[c].y, v3[c].z, v3[c].w};
            const float xx[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              s1 = fmaf(__uint_as_float(a1[k] << 16), xx[2 * k], s1);
              s1 = fmaf(__uint_as_float(a1[k] & 0xFFFF0000u), xx[2 * k + 1], s1);
              s3 = fmaf(__uint_as_float(a3[k] << 16), xx[2 * k], s3);
              s3 = fmaf(__uint_as_float(a3[k] & 0xFFFF0000u), xx[2 * k + 1], s3);
            }
          }
          acc1[t] = s1;
          acc3[t] = s3;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc1[t] = quad_sum(acc1[t]);
      acc3[t] = quad_sum(acc3[t]);
    }
    if (j == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= T) continue;
        float hv = 0.0f;
        if ((mask >> t) & 1u) {
          hv = silu_glu_q3(acc1[t], acc3[t], routed ? a.d.swiglu_limit : 10.0f);
          if (routed && a.d.route_before_down) hv *= slots.gate[slot][t];
        }
        q.h[((size_t)slot * T + t) * q.h_stride + row] = hv;
      }
    }
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
  const int H = a.d.hidden, I = a.d.inter, T = a.tokens;
  const bool has_shared = a.d.shared_w2 != nullptr;
  const int Is = has_shared ? a.d.shared_inter : 0;
  const int Ip = padded(I), Isp = padded(Is);
  float* hs = reinterpret_cast<float*>(smem4);   // routed: [kChunk][T][Ip]; shared: [T][Isp]
  float* ysum = hs + kChunk * T * Ip;            // [kChunk][T][I / 64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 3;
  const int D = slots.count;
  const int n_chunks = (D + kChunk - 1) / kChunk;
  const int n_rb = H / kRowsCta;
  const int items = (n_chunks + (has_shared ? 1 : 0)) * n_rb;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int c = item / n_rb, rb = item % n_rb;
    const bool routed = c < n_chunks;
    const int row = rb * kRowsCta + warp * 8 + (lane >> 2);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    __syncthreads();                             // previous item's readers are done with hs
    if (routed) {
      for (int ci = 0; ci < kChunk && c * kChunk + ci < D; ++ci)
        stage_rows(q.h + (size_t)(c * kChunk + ci) * T * q.h_stride, T, I, q.h_stride, hs + ci * T * Ip,
                   ysum + ci * T * (I / 64));
    } else {
      stage_rows(q.h + (size_t)a.max_slots * T * q.h_stride, T, Is, q.h_stride, hs, nullptr);
    }
    __syncthreads();
    if (routed) {
      for (int ci = 0; ci < kChunk && c * kChunk + ci < D; ++ci) {
        const int slot = c * kChunk + ci;
        const uint32_t mask = slots.mask[slot];
        const int e = slots.expert[slot];
        const size_t r = (size_t)e * H + row;
        const uint8_t* w = static_cast<const uint8_t*>(a.d.w2.data) + r * ((size_t)I * 3 / 8);
        const __half2* sc = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w2.scales) + r * (I / 64));
        const __half2* bi = reinterpret_cast<const __half2*>(static_cast<const __half*>(a.d.w2.biases) + r * (I / 64));
        const float* hsl = hs + ci * T * Ip;
        const float* ysl = ysum + ci * T * (I / 64);
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
            float Dq[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) Dq[t] = 0.0f;
            group_one<NT>(hh ? g1 : g0, hsl + pidx(64 * g), Ip, mask, Dq);
            const float s = hh ? s2.y : s2.x, b = hh ? b2.y : b2.x;
#pragma unroll
            for (int t = 0; t < NT; ++t)
              if ((mask >> t) & 1u) part[t] = fmaf(s, Dq[t], fmaf(b, ysl[t * (I / 64) + g], part[t]));
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
      const uint4* w = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.d.shared_w2) +
                                                      (size_t)row * Is);
      for (int seg = j; seg < Is / 32; seg += 4) {
        uint4 v[4];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) v[cc] = __ldcs(w + seg * 4 + cc);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= T) continue;
          const float4* hv = reinterpret_cast<const float4*>(hs + t * Isp + pidx(32 * seg));
          float s = acc[t];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const float4 xa = hv[2 * cc], xb = hv[2 * cc + 1];
            const uint32_t aw[4] = {v[cc].x, v[cc].y, v[cc].z, v[cc].w};
            const float xx[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              s = fmaf(__uint_as_float(aw[k] << 16), xx[2 * k], s);
              s = fmaf(__uint_as_float(aw[k] & 0xFFFF0000u), xx[2 * k + 1], s);
            }
          }
          acc[t] = s;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = quad_sum(acc[t]);
    if (j == 0) {
      const int cc = routed ? c : q.max_chunks;
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
  if (has_shared)
    acc += __bfloat162float(__float2bfloat16_rn(q.part[((size_t)q.max_chunks * T + t) * H + n]));
  if (a.d.out_f32) static_cast<float*>(a.out)[i] = acc;
  else static_cast<__nv_bfloat16*>(a.out)[i] = __float2bfloat16_rn(acc);
}

struct Q3Layout {
  size_t h, part, total;
  int h_stride, max_chunks;
};

Q3Layout q3_layout(const DsMoeDesc& d, int T) {
  Q3Layout L;
  const int S = std::min(T * d.top_k, d.n_experts);
  const int Is = d.shared_w1 ? d.shared_inter : 0;
  L.h_stride = std::max(d.inter, Is);
  L.max_chunks = (S + kChunk - 1) / kChunk;
  size_t o = 256;                                 // error word etc.
  L.h = o;
  o += ((size_t)(S + 1) * T * L.h_stride * 4 + 255) / 256 * 256;
  L.part = o;
  o += ((size_t)(L.max_chunks + 1) * T * d.hidden * 4 + 255) / 256 * 256;
  L.total = o;
  return L;
}

size_t smem_gate_up(const DsMoeDesc& d, int T) { return (size_t)T * padded(d.hidden) * 4 + (size_t)T * (d.hidden / 64) * 4; }

size_t smem_down(const DsMoeDesc& d, int T) {
  const int Is = d.shared_w1 ? d.shared_inter : 0;
  const size_t routed = (size_t)kChunk * T * padded(d.inter) * 4 + (size_t)kChunk * T * (d.inter / 64) * 4;
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
  if (d.hidden % 128 != 0 || d.inter % 128 != 0 || d.hidden % kRowsCta != 0 || d.inter % kRowsCta != 0) return false;
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
  Q3Args q;
  q.a = a;
  q.a.err = static_cast<int*>(workspace);
  q.a.max_slots = std::min(a.tokens * a.d.top_k, a.d.n_experts);
  q.h = reinterpret_cast<float*>(static_cast<char*>(workspace) + L.h);
  q.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + L.part);
  q.h_stride = L.h_stride;
  q.max_chunks = L.max_chunks;
  if (a.tokens == 1) return launch_nt<1>(q, st);
  if (a.tokens == 2) return launch_nt<2>(q, st);
  if (a.tokens <= 4) return launch_nt<4>(q, st);
  return launch_nt<8>(q, st);
}

}  // namespace decode
}  // namespace ds
