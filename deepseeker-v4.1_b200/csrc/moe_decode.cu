// Fused routed-expert MoE layer for decode (tokens <= 8), FP4 / Q3 routed
// experts + optional BF16 shared expert.
//
// Two launches per layer on the caller's stream:
//   A (gate/up): work item = (routed slot | shared, block of 16 rows).  Each
//     warp owns 2 rows of W1 and the same 2 rows of W3, streams them with
//     coalesced 128-bit (FP4/BF16) or 64-bit (Q3) loads straight into
//     registers, dequantises in registers, dots them against x (f32, staged
//     once per CTA in shared memory), reduces with warp shuffles and applies
//     the SwiGLU epilogue: h = silu(min(g, L)) * clip(u, -L, L) * gate.
//     h goes to the workspace in f32 (never rounded to bf16).
//   B (down + combine): work item = block of 16 output rows.  The CTA stages
//     every slot's h in shared memory; each warp owns 2 output rows and walks
//     the routed slots in ascending expert id, then the shared expert, with
//     the weight loads of later (slot, chunk) tasks in flight while earlier
//     ones are reduced.  out = bf16(sum_routed + f32(bf16(shared))).
//
// Distinct experts: every CTA rebuilds the ascending list of distinct routed
// experts and the per-(slot, token) gates from topk_ids (<= 128 entries) in
// shared memory, so no host round trip and no extra launch is needed.
//
// Weight loads use the streaming cache hint (__ldcs): every weight byte is
// read exactly once per layer.
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "moe_decode.cuh"

namespace {

using ds::decode::DecodeArgs;
using ds::decode::kMaxEntries;
using ds::decode::kMaxTokens;
using ds::decode::Slots;
using ds::decode::build_slots;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerWarp = 2;
constexpr int kRowsPerItem = kWarps * kRowsPerWarp;  // 16
constexpr int kSmemBudget = 200 * 1024;              // dynamic smem cap per CTA

// ---------------------------------------------------------------- staging

// f32 staging with a float4-unit swizzle: unit u lives at u ^ ((u >> 3) & 7).
// A lane reading the 8 (FP4) or 2 (BF16) consecutive units of its chunk then
// hits distinct banks across each quarter warp.
__device__ __forceinline__ int swz(int u) { return u ^ ((u >> 3) & 7); }

__device__ __forceinline__ float4 ld_unit(const float* base, int u) {
  return reinterpret_cast<const float4*>(base)[swz(u)];
}

__device__ __forceinline__ void st_unit(float* base, int u, float4 v) {
  reinterpret_cast<float4*>(base)[swz(u)] = v;
}

// ---------------------------------------------------------------- decode helpers

__device__ __forceinline__ void e2m1x8(uint32_t w, float (&f)[8]) {
  uint32_t h[4];
  asm("{ .reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3; }"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
    f[2 * i] = p.x;      // low nibble = even element
    f[2 * i + 1] = p.y;  // high nibble = odd element
  }
}

// dot of one 16-byte FP4 chunk (32 codes) with x units [8c, 8c+8)
__device__ __forceinline__ float fp4_chunk_dot(const uint4 w, const float* xs, int c) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float f[8];
    e2m1x8(words[i], f);
    const float4 xa = ld_unit(xs, 8 * c + 2 * i);
    const float4 xb = ld_unit(xs, 8 * c + 2 * i + 1);
    s0 = fmaf(f[0], xa.x, s0);
    s1 = fmaf(f[1], xa.y, s1);
    s0 = fmaf(f[2], xa.z, s0);
    s1 = fmaf(f[3], xa.w, s1);
    s0 = fmaf(f[4], xb.x, s0);
    s1 = fmaf(f[5], xb.y, s1);
    s0 = fmaf(f[6], xb.z, s0);
    s1 = fmaf(f[7], xb.w, s1);
  }
  return s0 + s1;
}

// dot of one 16-byte BF16 chunk (8 values) with x units [2c, 2c+2)
__device__ __forceinline__ float bf16_chunk_dot(const uint4 w, const float* xs, int c) {
  const float4 xa = ld_unit(xs, 2 * c);
  const float4 xb = ld_unit(xs, 2 * c + 1);
  float s0 = __uint_as_float(w.x << 16) * xa.x;
  float s1 = __uint_as_float(w.x & 0xFFFF0000u) * xa.y;
  s0 = fmaf(__uint_as_float(w.y << 16), xa.z, s0);
  s1 = fmaf(__uint_as_float(w.y & 0xFFFF0000u), xa.w, s1);
  s0 = fmaf(__uint_as_float(w.z << 16), xb.x, s0);
  s1 = fmaf(__uint_as_float(w.z & 0xFFFF0000u), xb.y, s1);
  s0 = fmaf(__uint_as_float(w.w << 16), xb.z, s0);
  s1 = fmaf(__uint_as_float(w.w & 0xFFFF0000u), xb.w, s1);
  return s0 + s1;
}

struct Q3Chunk {
  uint2 a, b, c;  // six words of one 64-element group
};

// sum_e q_e * x_e over one Q3 group (64 codes) with x units [16g, 16g+16);
// q_e is rebuilt exactly as f16 (1024 + q) - 1024 in f32.
__device__ __forceinline__ float q3_chunk_qdot(const Q3Chunk& q, const float* xs, int g) {
  const uint32_t lo[4] = {q.a.x, q.a.y, q.b.x, q.b.y};
  const uint32_t hi[2] = {q.c.x, q.c.y};
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t hw = hi[w >> 1];
    const int v = w & 1;
    // elements 16w + j (x unit 4w + j/4) and 16w + 8 + j (x unit 4w + 2 + j/4)
    const float4 x0 = ld_unit(xs, 16 * g + 4 * w);
    const float4 x1 = ld_unit(xs, 16 * g + 4 * w + 1);
    const float4 x2 = ld_unit(xs, 16 * g + 4 * w + 2);
    const float4 x3 = ld_unit(xs, 16 * g + 4 * w + 3);
    const float xa[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    const float xb[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t lo2 = (lo[w] >> (2 * j)) & 0x00030003u;
      const int hs = 8 * v + j;
      const uint32_t hi2 = ((hw >> hs) & 0x00010001u) << 2;
      const uint32_t bits = lo2 | hi2 | 0x64006400u;  // f16x2 of 1024 + q
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&bits));
      s0 = fmaf(f.x - 1024.0f, xa[j], s0);
      s1 = fmaf(f.y - 1024.0f, xb[j], s1);
    }
  }
  return s0 + s1;
}

// sum of x over group g (units 16g..16g+15)
__device__ __forceinline__ float x_group_sum(const float* xs, int g) {
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const float4 v = ld_unit(xs, 16 * g + u);
    s += (v.x + v.y) + (v.z + v.w);
  }
  return s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float silu_glu(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

// ---------------------------------------------------------------- per-warp row dots

// acc[r][t] += sum_k W_r[k] * xs_t[k] for NR rows of a quantised/bf16 matrix.
// Rows with a null data pointer are skipped (contribute 0).
template <int FMT, int NR, int NT>
struct RowDot;

template <int NR, int NT>
struct RowDot<DS_FMT_FP4, NR, NT> {
  static constexpr int U = 4;  // chunks per lane in flight, per row
  __device__ static void run(const uint8_t* const (&data)[NR], const uint8_t* const (&sc)[NR],
                             int K, const float* xs, int xstride, uint32_t tmask,
                             float (&acc)[NR][NT]) {
    const int lane = threadIdx.x & 31;
    const int nch = K / 32;
    for (int c0 = 0; c0 < nch; c0 += 32 * U) {
      uint4 w[NR][U];
      uint32_t sb[NR][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + lane + 32 * u;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          if (c < nch && data[r]) {
            w[r][u] = __ldcs(reinterpret_cast<const uint4*>(data[r]) + c);
            sb[r][u] = __ldcs(sc[r] + c);
          } else {
            w[r][u] = make_uint4(0u, 0u, 0u, 0u);
            sb[r][u] = 127u;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + lane + 32 * u;
        if (c < nch) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if ((tmask >> t) & 1u) {
#pragma unroll
              for (int r = 0; r < NR; ++r) {
                const float p = fp4_chunk_dot(w[r][u], xs + t * xstride, c);
                acc[r][t] = fmaf(p, ds::u8m0_value(sb[r][u]), acc[r][t]);
              }
            }
          }
        }
      }
    }
  }
};

template <int NR, int NT>
struct RowDot<DS_FMT_BF16, NR, NT> {
  static constexpr int U = 4;
  __device__ static void run(const uint8_t* const (&data)[NR], const uint8_t* const (&)[NR], int K,
                             const float* xs, int xstride, uint32_t tmask, float (&acc)[NR][NT]) {
    const int lane = threadIdx.x & 31;
    const int nch = K / 8;
    for (int c0 = 0; c0 < nch; c0 += 32 * U) {
      uint4 w[NR][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + lane + 32 * u;
#pragma unroll
        for (int r = 0; r < NR; ++r)
          w[r][u] = (c < nch && data[r]) ? __ldcs(reinterpret_cast<const uint4*>(data[r]) + c)
                                         : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + lane + 32 * u;
        if (c < nch) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if ((tmask >> t) & 1u) {
#pragma unroll
              for (int r = 0; r < NR; ++r) acc[r][t] += bf16_chunk_dot(w[r][u], xs + t * xstride, c);
            }
          }
        }
      }
    }
  }
};

// Q3: data = u32 words of the row, sc = f16 scales of the row; the matching
// biases pointer is sc + bias_off (biases live in a separate bank).
template <int NR, int NT>
struct RowDotQ3 {
  static constexpr int U = 2;
  __device__ static void run(const uint8_t* const (&data)[NR], const __half* const (&sc)[NR],
                             const __half* const (&bi)[NR], int K, const float* xs, int xstride,
                             const float* xg, uint32_t tmask, float (&acc)[NR][NT]) {
    const int lane = threadIdx.x & 31;
    const int ng = K / 64;
    for (int g0 = 0; g0 < ng; g0 += 32 * U) {
      Q3Chunk q[NR][U];
      float s[NR][U], b[NR][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int g = g0 + lane + 32 * u;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          if (g < ng && data[r]) {
            const uint2* p = reinterpret_cast<const uint2*>(data[r] + (size_t)g * 24);
            q[r][u].a = __ldcs(p);
            q[r][u].b = __ldcs(p + 1);
            q[r][u].c = __ldcs(p + 2);
            s[r][u] = __half2float(__ldcs(reinterpret_cast<const __half*>(sc[r]) + g));
            b[r][u] = __half2float(__ldcs(reinterpret_cast<const __half*>(bi[r]) + g));
          } else {
            q[r][u].a = q[r][u].b = q[r][u].c = make_uint2(0u, 0u);
            s[r][u] = 0.f;
            b[r][u] = 0.f;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int g = g0 + lane + 32 * u;
        if (g < ng) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if ((tmask >> t) & 1u) {
              const float xsum = xg[t * (K / 64) + g];
#pragma unroll
              for (int r = 0; r < NR; ++r) {
                const float qd = q3_chunk_qdot(q[r][u], xs + t * xstride, g);
                acc[r][t] = fmaf(s[r][u], qd, fmaf(b[r][u], xsum, acc[r][t]));
              }
            }
          }
        }
      }
    }
  }
};

// Pointers of row n of expert e in a bank.
struct RowPtr {
  const uint8_t* data;
  const uint8_t* sc;   // FP4 scales (u8) or Q3 scales (f16)
  const uint8_t* bi;   // Q3 biases (f16)
};

__device__ __forceinline__ RowPtr bank_row(const DsExpertBank& b, int e, int n) {
  RowPtr p{nullptr, nullptr, nullptr};
  const size_t row = (size_t)e * b.rows + n;
  const size_t K = (size_t)b.cols;
  if (b.format == DS_FMT_FP4) {
    p.data = static_cast<const uint8_t*>(b.data) + row * (K / 2);
    p.sc = static_cast<const uint8_t*>(b.scales) + row * (K / 32);
  } else if (b.format == DS_FMT_Q3) {
    p.data = static_cast<const uint8_t*>(b.data) + row * (K * 3 / 8);
    p.sc = static_cast<const uint8_t*>(b.scales) + row * (K / 64) * 2;
    p.bi = static_cast<const uint8_t*>(b.biases) + row * (K / 64) * 2;
  }
  return p;
}

// Stage T rows of a [T, K] bf16 or f32 matrix into swizzled f32 smem.
__device__ void stage_bf16(const __nv_bfloat16* src, int T, int K, float* dst) {
  const int units = K / 4;
  for (int i = threadIdx.x; i < T * units; i += blockDim.x) {
    const int t = i / units, u = i - t * units;
    const uint2 v = *reinterpret_cast<const uint2*>(src + (size_t)t * K + 4 * u);
    float4 f = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                           __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
    st_unit(dst + (size_t)t * K, u, f);
  }
}

__device__ void stage_f32(const float* src, int T, int K, int src_stride, float* dst) {
  const int units = K / 4;
  for (int i = threadIdx.x; i < T * units; i += blockDim.x) {
    const int t = i / units, u = i - t * units;
    st_unit(dst + (size_t)t * K, u, *reinterpret_cast<const float4*>(src + (size_t)t * src_stride + 4 * u));
  }
}

// Per-token group sums of x (Q3 bias term): xg[t][g] = sum over group g.
__device__ void stage_group_sums(const float* xs, int T, int K, float* xg) {
  const int ng = K / 64;
  for (int i = threadIdx.x; i < T * ng; i += blockDim.x) {
    const int t = i / ng, g = i - t * ng;
    xg[i] = x_group_sum(xs + (size_t)t * K, g);
  }
}

// ============================================================== kernel A

template <int FMT, int NT>
__global__ void __launch_bounds__(kThreads, 1) moe_gate_up_kernel(const DecodeArgs a) {
  extern __shared__ float4 smem4[];
  __shared__ Slots slots;
  const int H = a.d.hidden, I = a.d.inter;
  const int T = a.tokens;
  float* xs = reinterpret_cast<float*>(smem4);  // [T][H]
  float* xg = xs + (size_t)T * H;                // [T][H/64] (Q3 only)

  if (a.x_f32)
    stage_f32(static_cast<const float*>(a.x), T, H, H, xs);
  else
    stage_bf16(static_cast<const __nv_bfloat16*>(a.x), T, H, xs);
  build_slots(a, slots);  // ends with __syncthreads
  if (FMT == DS_FMT_Q3) {
    stage_group_sums(xs, T, H, xg);
    __syncthreads();
  }
  const int D = slots.count;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb_routed = (I + kRowsPerItem - 1) / kRowsPerItem;
  const bool has_shared = a.d.shared_w1 != nullptr;
  const int Is = a.d.shared_inter;
  const int nb_shared = has_shared ? (Is + kRowsPerItem - 1) / kRowsPerItem : 0;
  const int items = a.max_slots * nb_routed + nb_shared;

  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const bool routed = item < a.max_slots * nb_routed;
    int slot, rb;
    if (routed) {
      slot = item / nb_routed;
      rb = item - slot * nb_routed;
      if (slot >= D) continue;
    } else {
      slot = a.max_slots;
      rb = item - a.max_slots * nb_routed;
    }
    const int nrows = routed ? I : Is;
    const int row0 = rb * kRowsPerItem + warp * kRowsPerWarp;
    float acc[2 * kRowsPerWarp][NT];
#pragma unroll
    for (int r = 0; r < 2 * kRowsPerWarp; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;

    if (routed) {
      const int e = slots.expert[slot];
      const uint8_t* data[2 * kRowsPerWarp];
      const uint8_t* sc[2 * kRowsPerWarp];
      const uint8_t* bi[2 * kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int n = row0 + r;
        RowPtr p1{nullptr, nullptr, nullptr}, p3{nullptr, nullptr, nullptr};
        if (n < nrows) {
          p1 = bank_row(a.d.w1, e, n);
          p3 = bank_row(a.d.w3, e, n);
        }
        data[r] = p1.data; sc[r] = p1.sc; bi[r] = p1.bi;
        data[kRowsPerWarp + r] = p3.data; sc[kRowsPerWarp + r] = p3.sc; bi[kRowsPerWarp + r] = p3.bi;
      }
      if (FMT == DS_FMT_FP4) {
        RowDot<DS_FMT_FP4, 2 * kRowsPerWarp, NT>::run(data, sc, H, xs, H, slots.mask[slot], acc);
      } else {
        const __half* s16[2 * kRowsPerWarp];
        const __half* b16[2 * kRowsPerWarp];
#pragma unroll
        for (int r = 0; r < 2 * kRowsPerWarp; ++r) {
          s16[r] = reinterpret_cast<const __half*>(sc[r]);
          b16[r] = reinterpret_cast<const __half*>(bi[r]);
        }
        RowDotQ3<2 * kRowsPerWarp, NT>::run(data, s16, b16, H, xs, H, xg, slots.mask[slot], acc);
      }
    } else {
      const uint8_t* data[2 * kRowsPerWarp];
      const uint8_t* none[2 * kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int n = row0 + r;
        const bool ok = n < nrows;
        data[r] = ok ? static_cast<const uint8_t*>(a.d.shared_w1) + (size_t)n * H * 2 : nullptr;
        data[kRowsPerWarp + r] = ok ? static_cast<const uint8_t*>(a.d.shared_w3) + (size_t)n * H * 2 : nullptr;
        none[r] = none[kRowsPerWarp + r] = nullptr;
      }
      RowDot<DS_FMT_BF16, 2 * kRowsPerWarp, NT>::run(data, none, H, xs, H, (1u << T) - 1u, acc);
    }

    // reduce and apply the SwiGLU epilogue
#pragma unroll
    for (int r = 0; r < 2 * kRowsPerWarp; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = warp_sum(acc[r][t]);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int n = row0 + r;
        if (n >= nrows) continue;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= T) continue;
          float hv = silu_glu(acc[r][t], acc[kRowsPerWarp + r][t],
                              routed ? a.d.swiglu_limit : 10.0f);
          if (routed) {
            const bool on = (slots.mask[slot] >> t) & 1u;
            hv = on ? (a.d.route_before_down ? hv * slots.gate[slot][t] : hv) : 0.0f;
          }
          a.h[((size_t)slot * T + t) * a.h_stride + n] = hv;
        }
      }
    }
  }
}

// ============================================================== kernel B

template <int FMT, int NT>
__global__ void __launch_bounds__(kThreads, 1) moe_down_kernel(const DecodeArgs a) {
  extern __shared__ float4 smem4[];
  __shared__ Slots slots;
  const int H = a.d.hidden, I = a.d.inter, T = a.tokens;
  const bool has_shared = a.d.shared_w2 != nullptr;
  const int Is = a.d.shared_inter;
  float* hs = reinterpret_cast<float*>(smem4);  // staged h: [g][T][I]

  build_slots(a, slots);
  const int D = slots.count;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRowsPerItem + warp * kRowsPerWarp;

  // how many routed slots fit in shared memory at once
  const size_t slot_bytes = (size_t)T * I * 4 + (FMT == DS_FMT_Q3 ? (size_t)T * (I / 64) * 4 : 0);
  const size_t shared_bytes = has_shared ? (size_t)T * Is * 4 : 0;
  int per_group = (int)((kSmemBudget - shared_bytes) / slot_bytes);
  if (per_group < 1) per_group = 1;

  float routed_acc[kRowsPerWarp][NT];
  float shared_acc[kRowsPerWarp][NT];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) routed_acc[r][t] = shared_acc[r][t] = 0.f;

  for (int g0 = 0; g0 < D || (g0 == 0 && D == 0); g0 += per_group) {
    const int g1 = min(D, g0 + per_group);
    const bool last = g1 >= D;
    // ---- stage h of slots [g0, g1) (and the shared h with the last group)
    __syncthreads();
    for (int s = g0; s < g1; ++s) {
      float* dst = hs + (size_t)(s - g0) * T * I;
      stage_f32(a.h + (size_t)s * T * a.h_stride, T, I, a.h_stride, dst);
    }
    float* xg_base = hs + (size_t)(g1 - g0) * T * I;  // Q3 group sums [g][T][I/64]
    float* hsh = xg_base + (FMT == DS_FMT_Q3 ? (size_t)(g1 - g0) * T * (I / 64) : 0);
    if (last && has_shared) stage_f32(a.h + (size_t)a.max_slots * T * a.h_stride, T, Is, a.h_stride, hsh);
    __syncthreads();
    if (FMT == DS_FMT_Q3) {
      for (int s = g0; s < g1; ++s)
        stage_group_sums(hs + (size_t)(s - g0) * T * I, T, I, xg_base + (size_t)(s - g0) * T * (I / 64));
      __syncthreads();
    }

    for (int s = g0; s < g1; ++s) {
      const int e = slots.expert[s];
      const uint32_t mask = slots.mask[s];
      const float* hslot = hs + (size_t)(s - g0) * T * I;
      const uint8_t* data[kRowsPerWarp];
      const uint8_t* sc[kRowsPerWarp];
      const uint8_t* bi[kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int n = row0 + r;
        RowPtr p{nullptr, nullptr, nullptr};
        if (n < H) p = bank_row(a.d.w2, e, n);
        data[r] = p.data; sc[r] = p.sc; bi[r] = p.bi;
      }
      float acc[kRowsPerWarp][NT];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
      if (FMT == DS_FMT_FP4) {
        RowDot<DS_FMT_FP4, kRowsPerWarp, NT>::run(data, sc, I, hslot, I, mask, acc);
      } else {
        const __half* s16[kRowsPerWarp];
        const __half* b16[kRowsPerWarp];
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          s16[r] = reinterpret_cast<const __half*>(sc[r]);
          b16[r] = reinterpret_cast<const __half*>(bi[r]);
        }
        RowDotQ3<kRowsPerWarp, NT>::run(data, s16, b16, I, hslot, I,
                                         xg_base + (size_t)(s - g0) * T * (I / 64), mask, acc);
      }
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float v = warp_sum(acc[r][t]);
          if ((mask >> t) & 1u) {
            // route_before_down == 0: the gate multiplies the down output
            const float y = a.d.route_before_down ? v : v * slots.gate[s][t];
            routed_acc[r][t] += y;
          }
        }
    }

    if (last && has_shared) {
      const uint8_t* data[kRowsPerWarp];
      const uint8_t* none[kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int n = row0 + r;
        data[r] = n < H ? static_cast<const uint8_t*>(a.d.shared_w2) + (size_t)n * Is * 2 : nullptr;
        none[r] = nullptr;
      }
      RowDot<DS_FMT_BF16, kRowsPerWarp, NT>::run(data, none, Is, hsh, Is, (1u << T) - 1u, shared_acc);
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) shared_acc[r][t] = warp_sum(shared_acc[r][t]);
    }
    if (D == 0) break;
  }

  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int n = row0 + r;
      if (n >= H) continue;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= T) continue;
        float v = routed_acc[r][t];
        if (a.x_f32) {
          if (has_shared) v += shared_acc[r][t];
          static_cast<float*>(a.out)[(size_t)t * H + n] = v;
        } else {
          // the shared expert's output is cast to x.dtype before the add
          if (has_shared) v += __bfloat162float(__float2bfloat16_rn(shared_acc[r][t]));
          static_cast<__nv_bfloat16*>(a.out)[(size_t)t * H + n] = __float2bfloat16_rn(v);
        }
      }
    }
  }
}

// ============================================================== qmm

// out[r, n] = sum_k x[r, k] * W[n, k] for one compressed matrix W (FP4 or Q3),
// f32 accumulate, f32 out.  Block = 8 warps x 2 output rows = 16 rows of W
// (blockIdx.x) for up to 8 rows of x (blockIdx.y), x staged in shared memory
// as swizzled f32 (plus the 64-group sums for Q3).
template <int FMT, int NT>
__global__ void __launch_bounds__(kThreads) qmm_kernel(const DsExpertBank w, const void* x, int x_f32,
                                                        int64_t rows, float* out) {
  extern __shared__ float4 smem4[];
  const int K = w.cols, N = w.rows;
  const int64_t r0 = (int64_t)blockIdx.y * NT;
  const int T = (rows - r0 < (int64_t)NT) ? (int)(rows - r0) : NT;
  float* xs = reinterpret_cast<float*>(smem4);  // [T][K]
  float* xg = xs + (size_t)NT * K;              // [T][K/64] (Q3)
  if (x_f32)
    stage_f32(static_cast<const float*>(x) + r0 * K, T, K, K, xs);
  else
    stage_bf16(static_cast<const __nv_bfloat16*>(x) + r0 * K, T, K, xs);
  __syncthreads();
  if (FMT == DS_FMT_Q3) {
    stage_group_sums(xs, T, K, xg);
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRowsPerItem + warp * kRowsPerWarp;
  const uint32_t tmask = (T >= 32) ? 0xffffffffu : ((1u << T) - 1u);
  float acc[kRowsPerWarp][NT];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
  const uint8_t* data[kRowsPerWarp];
  const uint8_t* sc[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const RowPtr p = bank_row(w, 0, row0 + r);
    data[r] = row0 + r < N ? p.data : nullptr;
    sc[r] = p.sc;
  }
  if (FMT == DS_FMT_FP4) {
    RowDot<DS_FMT_FP4, kRowsPerWarp, NT>::run(data, sc, K, xs, K, tmask, acc);
  } else {
    const __half* scq[kRowsPerWarp];
    const __half* biq[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const RowPtr p = bank_row(w, 0, row0 + r);
      scq[r] = reinterpret_cast<const __half*>(p.sc);
      biq[r] = reinterpret_cast<const __half*>(p.bi);
    }
    RowDotQ3<kRowsPerWarp, NT>::run(data, scq, biq, K, xs, K, xg, tmask, acc);
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float v = warp_sum(acc[r][t]);
      if (lane == 0 && t < T && row0 + r < N) out[(r0 + t) * N + row0 + r] = v;
    }
}

// ============================================================== host side

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int validate_bank(const DsExpertBank& b, int fmt, int E, int N, int K, const char* name) {
  DS_REQUIRE(b.format == fmt, DS_EINVAL, "moe_decode: %s format %d != routed format %d", name, b.format, fmt);
  DS_REQUIRE(b.n_experts == E && b.rows == N && b.cols == K, DS_EINVAL,
             "moe_decode: %s bank is [%d, %d, %d], expected [%d, %d, %d]", name, b.n_experts, b.rows,
             b.cols, E, N, K);
  DS_REQUIRE(b.data && b.scales, DS_EINVAL, "moe_decode: %s bank has null pointers", name);
  if (fmt == DS_FMT_FP4) {
    DS_REQUIRE(K % 32 == 0, DS_EINVAL, "moe_decode: %s K=%d not a multiple of 32", name, K);
    DS_REQUIRE(ds::aligned(b.data, 16), DS_EALIGN, "moe_decode: %s data must be 16-byte aligned", name);
  } else {
    DS_REQUIRE(K % 64 == 0, DS_EINVAL, "moe_decode: %s K=%d not a multiple of 64", name, K);
    DS_REQUIRE(b.biases != nullptr, DS_EINVAL, "moe_decode: %s Q3 bank needs biases", name);
    DS_REQUIRE(ds::aligned(b.data, 8) && ds::aligned(b.scales, 2) && ds::aligned(b.biases, 2),
               DS_EALIGN, "moe_decode: %s Q3 words 8-byte aligned, scales/biases 2-byte", name);
  }
  return DS_OK;
}

int validate(const DsMoeDesc* d, int64_t tokens) {
  DS_REQUIRE(d != nullptr, DS_EINVAL, "moe_decode: null descriptor");
  DS_REQUIRE(tokens >= 1 && tokens <= kMaxTokens, DS_EINVAL, "moe_decode: tokens must be in [1, %d]",
             kMaxTokens);
  DS_REQUIRE(d->top_k >= 1 && tokens * d->top_k <= kMaxEntries, DS_EINVAL,
             "moe_decode: tokens * top_k must be in [1, %d]", kMaxEntries);
  DS_REQUIRE(d->hidden > 0 && d->inter > 0 && d->n_experts > 0, DS_EINVAL, "moe_decode: bad geometry");
  DS_REQUIRE(d->hidden % 64 == 0 && d->inter % 64 == 0, DS_EINVAL,
             "moe_decode: hidden and inter must be multiples of 64");
  const int fmt = d->w1.format;
  DS_REQUIRE(fmt == DS_FMT_FP4 || fmt == DS_FMT_Q3, DS_ENOTSUP, "moe_decode: routed format must be FP4 or Q3");
  int st;
  if ((st = validate_bank(d->w1, fmt, d->n_experts, d->inter, d->hidden, "w1")) != DS_OK) return st;
  if ((st = validate_bank(d->w3, fmt, d->n_experts, d->inter, d->hidden, "w3")) != DS_OK) return st;
  if ((st = validate_bank(d->w2, fmt, d->n_experts, d->hidden, d->inter, "w2")) != DS_OK) return st;
  const bool sh = d->shared_w1 || d->shared_w3 || d->shared_w2;
  if (sh) {
    DS_REQUIRE(d->shared_w1 && d->shared_w3 && d->shared_w2, DS_EINVAL,
               "moe_decode: shared expert needs all of w1, w3, w2");
    DS_REQUIRE(d->shared_inter > 0 && d->shared_inter % 64 == 0, DS_EINVAL,
               "moe_decode: shared_inter must be a positive multiple of 64");
    DS_REQUIRE(ds::aligned(d->shared_w1, 16) && ds::aligned(d->shared_w3, 16) && ds::aligned(d->shared_w2, 16),
               DS_EALIGN, "moe_decode: shared weights must be 16-byte aligned");
  }
  return DS_OK;
}

struct WsLayout {
  size_t err_off, h_off, total;
  int max_slots, h_stride;
};

WsLayout ws_layout(const DsMoeDesc* d, int64_t tokens) {
  WsLayout w;
  w.max_slots = (int)std::min<int64_t>(tokens * d->top_k, d->n_experts);
  const bool sh = d->shared_w1 != nullptr;
  w.h_stride = (int)align_up(std::max(d->inter, sh ? d->shared_inter : 0), 4);
  w.err_off = 0;
  w.h_off = ds::decode::kWsReserved;
  w.total = w.h_off + (size_t)(w.max_slots + 1) * tokens * w.h_stride * sizeof(float);
  w.total = align_up(w.total, 256);
  return w;
}

template <int FMT, int NT>
int launch_decode(const DecodeArgs& a, cudaStream_t st) {
  const int H = a.d.hidden, I = a.d.inter, T = a.tokens;
  const bool sh = a.d.shared_w1 != nullptr;
  // kernel A
  size_t smem_a = (size_t)T * H * 4 + (FMT == DS_FMT_Q3 ? (size_t)T * (H / 64) * 4 : 0);
  DS_REQUIRE(smem_a <= (size_t)kSmemBudget, DS_EINVAL, "moe_decode: tokens * hidden too large for shared memory");
  static thread_local int configured_a = 0, configured_b = 0;
  (void)configured_a;
  (void)configured_b;
  DS_CHECK_CUDA(cudaFuncSetAttribute(moe_gate_up_kernel<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBudget + 16 * 1024));
  DS_CHECK_CUDA(cudaFuncSetAttribute(moe_down_kernel<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBudget + 16 * 1024));
  const int nb_routed = (I + kRowsPerItem - 1) / kRowsPerItem;
  const int nb_shared = sh ? (a.d.shared_inter + kRowsPerItem - 1) / kRowsPerItem : 0;
  const int items = a.max_slots * nb_routed + nb_shared;
  int grid_a = std::min(items, ds::sm_count());
  if (grid_a < 1) grid_a = 1;
  moe_gate_up_kernel<FMT, NT><<<grid_a, kThreads, smem_a, st>>>(a);
  DS_CHECK_LAUNCH("moe_gate_up_kernel");
  // kernel B: shared memory = routed h group + Q3 group sums + shared h
  const size_t slot_bytes = (size_t)T * I * 4 + (FMT == DS_FMT_Q3 ? (size_t)T * (I / 64) * 4 : 0);
  const size_t shared_bytes = sh ? (size_t)T * a.d.shared_inter * 4 : 0;
  DS_REQUIRE(slot_bytes + shared_bytes <= (size_t)kSmemBudget, DS_EINVAL,
             "moe_decode: tokens * inter too large for shared memory");
  int per_group = (int)((kSmemBudget - shared_bytes) / slot_bytes);
  if (per_group < 1) per_group = 1;
  const int groups_max = std::min(per_group, a.max_slots);
  const size_t smem_b = (size_t)groups_max * slot_bytes + shared_bytes;
  const int grid_b = (H + kRowsPerItem - 1) / kRowsPerItem;
  moe_down_kernel<FMT, NT><<<grid_b, kThreads, smem_b, st>>>(a);
  DS_CHECK_LAUNCH("moe_down_kernel");
  return DS_OK;
}

template <int FMT>
int dispatch_tokens(const DecodeArgs& a, cudaStream_t st) {
  if (a.tokens == 1) return launch_decode<FMT, 1>(a, st);
  if (a.tokens == 2) return launch_decode<FMT, 2>(a, st);
  if (a.tokens <= 4) return launch_decode<FMT, 4>(a, st);
  return launch_decode<FMT, 8>(a, st);
}

// Kernel choice of one call, made from the descriptor and the scratch the
// caller provides (workspace_bytes); ds_moe_decode and ds_moe_decode_noalloc
// both come through here, so a given (layer, tokens, scratch size) always runs
// the same kernels:
//   FP4 banks with scale atoms, bf16 x  -> tcgen05 kernels (moe_decode_t5.cu)
//   one token, FP4 banks, bf16 x         -> register-dequant kernel (moe_decode_rd.cu)
//   Q3 banks, bf16 x                    -> dp2a CUDA-core kernels (moe_decode_q3.cu)
//   anything else (f32 x, ...)          -> the generic kernels above
// A path whose scratch does not fit in workspace_bytes is skipped.  (At one
// token the tcgen05 kernels stream config 2's layer faster than the
// register-dequant kernel, measured; the latter serves banks without atoms.)
int dispatch(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (ds::decode::t5_supported(a) && workspace_bytes >= ds::decode::t5_workspace_bytes(a.d, a.tokens))
    return ds::decode::launch_t5(a, workspace, workspace_bytes, s);
  if (ds::decode::rd_supported(a) && workspace_bytes >= ds::decode::rd_workspace_bytes(a.d))
    return ds::decode::launch_rd(a, workspace, workspace_bytes, s);
  if (ds::decode::q3_supported(a) && workspace_bytes >= ds::decode::q3_workspace_bytes(a.d, a.tokens))
    return ds::decode::launch_q3(a, workspace, workspace_bytes, s);
  DS_REQUIRE(!a.d.out_f32 || a.x_f32, DS_ENOTSUP,
             "moe_decode: out_f32 with bf16 x needs FP4 banks (with scale atoms above one token) or Q3 banks");
  return a.d.w1.format == DS_FMT_FP4 ? dispatch_tokens<DS_FMT_FP4>(a, s) : dispatch_tokens<DS_FMT_Q3>(a, s);
}

}  // namespace

extern "C" int ds_moe_decode_workspace_size(const DsMoeDesc* desc, int64_t tokens, size_t* bytes) {
  int st = validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(bytes != nullptr, DS_EINVAL, "moe_decode_workspace_size: null output");
  size_t total = ws_layout(desc, tokens).total;
  if (desc->w1.format == DS_FMT_FP4 && desc->w1.scales_tc && desc->w3.scales_tc && desc->w2.scales_tc &&
      tokens <= ds::decode::kMaxTokens)
    total = std::max(total, ds::decode::t5_workspace_bytes(*desc, (int)tokens));
  if (desc->w1.format == DS_FMT_Q3) total = std::max(total, ds::decode::q3_workspace_bytes(*desc, (int)tokens));
  if (desc->w1.format == DS_FMT_FP4 && tokens == 1) total = std::max(total, ds::decode::rd_workspace_bytes(*desc));
  *bytes = total;
  return DS_OK;
}

namespace {

// Checks shared by ds_moe_decode and ds_moe_decode_route; fills the decode arguments.
int decode_args(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens, const int32_t* topk_ids,
                const float* topk_w, void* out, void* workspace, size_t workspace_bytes, DecodeArgs& a) {
  int st = validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(x && topk_ids && topk_w && out && workspace, DS_EINVAL, "moe_decode: null pointer");
  DS_REQUIRE(x_dtype == DS_BF16 || x_dtype == DS_F32, DS_EINVAL, "moe_decode: x_dtype must be DS_BF16 or DS_F32");
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 4) && ds::aligned(workspace, 256), DS_EALIGN,
             "moe_decode: x 16-byte, out 4-byte and workspace 256-byte aligned");
  const WsLayout w = ws_layout(desc, tokens);
  DS_REQUIRE(workspace_bytes >= w.total, DS_EINVAL, "moe_decode: workspace %zu bytes < required %zu",
             workspace_bytes, w.total);
  a.d = *desc;
  a.x = x;
  a.x_f32 = x_dtype == DS_F32;
  a.tokens = (int)tokens;
  a.ids = topk_ids;
  a.gates = topk_w;
  a.out = out;
  a.h = reinterpret_cast<float*>(static_cast<char*>(workspace) + w.h_off);
  a.max_slots = w.max_slots;
  a.h_stride = w.h_stride;
  a.err = reinterpret_cast<int*>(static_cast<char*>(workspace) + w.err_off);
  return DS_OK;
}

}  // namespace

extern "C" int ds_moe_decode(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens, const int32_t* topk_ids,
                             const float* topk_w, void* out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  DecodeArgs a;
  const int st = decode_args(desc, x, x_dtype, tokens, topk_ids, topk_w, out, workspace, workspace_bytes, a);
  if (st != DS_OK) return st;
  return dispatch(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int ds_moe_decode_route(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                                   const float* logits, const float* route_bias, int route_kind, float route_scale,
                                   int32_t* topk_ids, float* topk_w, void* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  DecodeArgs a;
  int st = decode_args(desc, x, x_dtype, tokens, topk_ids, topk_w, out, workspace, workspace_bytes, a);
  if (st != DS_OK) return st;
  DS_REQUIRE(logits != nullptr, DS_EINVAL, "moe_decode_route: null logits");
  DS_REQUIRE(desc->n_experts <= 1024 && desc->top_k <= 32, DS_EINVAL,
             "moe_decode_route: n_experts <= 1024 and top_k <= 32 (the router's limits)");
  DS_REQUIRE(route_kind == DS_ROUTE_SOFTMAX || route_kind == DS_ROUTE_SQRTSOFTPLUS || route_kind == DS_ROUTE_SCORES,
             DS_EINVAL, "moe_decode_route: unknown route kind %d", route_kind);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ds::decode::t5_supported(a) && workspace_bytes >= ds::decode::t5_workspace_bytes(a.d, a.tokens)) {
    a.logits = logits;                 // the tcgen05 prep kernel routes in its own launch
    a.route_bias = route_bias;
    a.route_kind = route_kind;
    a.route_scale = route_scale;
    return ds::decode::launch_t5(a, workspace, workspace_bytes, s);
  }
  st = ds_route_topk(logits, route_bias, tokens, desc->n_experts, desc->top_k, route_kind, route_scale, topk_ids,
                     topk_w, stream);
  if (st != DS_OK) return st;
  return dispatch(a, workspace, workspace_bytes, s);
}

// ============================================================== qmm host side

namespace {

template <int FMT, int NT>
int launch_qmm(const DsExpertBank& w, const void* x, int x_f32, int64_t rows, float* out, cudaStream_t s) {
  const size_t smem = (size_t)NT * w.cols * 4 + (FMT == DS_FMT_Q3 ? (size_t)NT * (w.cols / 64) * 4 : 0);
  DS_REQUIRE(smem <= (size_t)kSmemBudget, DS_EINVAL, "qmm: K = %d too large (x rows staged in shared memory)",
             w.cols);
  DS_CHECK_CUDA(cudaFuncSetAttribute(qmm_kernel<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBudget + 16 * 1024));
  const dim3 grid((w.rows + kRowsPerItem - 1) / kRowsPerItem, (unsigned)((rows + NT - 1) / NT));
  qmm_kernel<FMT, NT><<<grid, kThreads, smem, s>>>(w, x, x_f32, rows, out);
  DS_CHECK_LAUNCH("qmm_kernel");
  return DS_OK;
}

template <int FMT>
int qmm_rows(const DsExpertBank& w, const void* x, int x_f32, int64_t rows, float* out, cudaStream_t s) {
  if (rows == 1) return launch_qmm<FMT, 1>(w, x, x_f32, rows, out, s);
  if (rows == 2) return launch_qmm<FMT, 2>(w, x, x_f32, rows, out, s);
  if (rows <= 4) return launch_qmm<FMT, 4>(w, x, x_f32, rows, out, s);
  return launch_qmm<FMT, 8>(w, x, x_f32, rows, out, s);
}

}  // namespace

extern "C" int ds_qmm(const DsExpertBank* w, const void* x, int x_dtype, int64_t rows, float* out, void* stream) {
  DS_REQUIRE(w != nullptr, DS_EINVAL, "qmm: null matrix");
  DS_REQUIRE(w->format == DS_FMT_FP4 || w->format == DS_FMT_Q3, DS_ENOTSUP, "qmm: format must be FP4 or Q3");
  DS_REQUIRE(w->n_experts == 1, DS_EINVAL, "qmm: one matrix (n_experts == 1), got %d", w->n_experts);
  DS_REQUIRE(w->rows > 0 && w->cols > 0, DS_EINVAL, "qmm: bad matrix geometry [%d, %d]", w->rows, w->cols);
  DS_REQUIRE(rows >= 0 && rows <= (int64_t)65535 * 8, DS_EINVAL, "qmm: rows must be in [0, %d]", 65535 * 8);
  DS_REQUIRE(x_dtype == DS_F32 || x_dtype == DS_BF16, DS_EINVAL, "qmm: x_dtype must be DS_F32 or DS_BF16");
  DS_REQUIRE(w->data && w->scales && x && out, DS_EINVAL, "qmm: null pointer");
  if (w->format == DS_FMT_FP4) {
    DS_REQUIRE(w->cols % 32 == 0, DS_EINVAL, "qmm: FP4 K = %d not a multiple of 32", w->cols);
    DS_REQUIRE(ds::aligned(w->data, 16), DS_EALIGN, "qmm: FP4 data must be 16-byte aligned");
  } else {
    DS_REQUIRE(w->cols % 64 == 0, DS_EINVAL, "qmm: Q3 K = %d not a multiple of 64", w->cols);
    DS_REQUIRE(w->biases != nullptr, DS_EINVAL, "qmm: Q3 matrix needs biases");
    DS_REQUIRE(ds::aligned(w->data, 8) && ds::aligned(w->scales, 2) && ds::aligned(w->biases, 2), DS_EALIGN,
               "qmm: Q3 words 8-byte aligned, scales/biases 2-byte");
  }
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 4), DS_EALIGN, "qmm: x 16-byte and out 4-byte aligned");
  DS_REQUIRE(w->cols % 4 == 0, DS_EINVAL, "qmm: K must be a multiple of 4");
  if (rows == 0) return DS_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int xf = x_dtype == DS_F32;
  return w->format == DS_FMT_FP4 ? qmm_rows<DS_FMT_FP4>(*w, x, xf, rows, out, s)
                                 : qmm_rows<DS_FMT_Q3>(*w, x, xf, rows, out, s);
}

// ============================================================== no-allocation variant
//
// Some callers cannot hand the library a workspace: a serving loop whose
// device memory is carved up once at start-up by its own pool (and whose pool
// may not be touched from the decode thread), or a host thread that runs
// between stream-ordered allocator phases and must not trigger an
// allocation, implicit or not.  ds_moe_decode_noalloc takes its scratch
// from a file-scope __device__ array instead: the CUDA runtime reserves it
// when the module is loaded, so the call itself allocates no device memory
// (tensor maps live in fixed static tables).

namespace {

// Scratch limit: 8 MiB.  The call runs the kernels ds_moe_decode would run
// with a workspace of this size (dispatch() above): the fastest path whose
// scratch fits.  The generic kernels need 4096 + (slots + 1) * tokens * stride
// * 4 bytes (slots = min(tokens * k, experts), stride = max(inter,
// shared_inter)); config 2's layer (hidden 4096, inter 2048, top-8) fits every
// path at one token.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};

// Device address of the scratch array on the current device, resolved once
// per device (the first call on a device does this setup, which is why that
// first call should come before any stream capture).  Every path keeps its
// error word in the first 4 bytes of its scratch.
int noalloc_scratch(void** out) {
  int dev = 0;
  DS_CHECK_CUDA(cudaGetDevice(&dev));
  DS_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, DS_EINVAL, "moe_decode_noalloc: device %d beyond %d", dev,
             kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    DS_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    DS_REQUIRE(p != nullptr && ds::aligned(p, 256), DS_ECUDA, "moe_decode_noalloc: bad scratch address");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return DS_OK;
}

}  // namespace

extern "C" size_t ds_moe_decode_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

extern "C" int ds_moe_decode_noalloc(const DsMoeDesc* desc, const void* x, int x_dtype, int64_t tokens,
                                     const int32_t* topk_ids, const float* topk_w, void* out, void* stream) {
  int st = validate(desc, tokens);
  if (st != DS_OK) return st;
  DS_REQUIRE(x && topk_ids && topk_w && out, DS_EINVAL, "moe_decode_noalloc: null pointer");
  DS_REQUIRE(x_dtype == DS_BF16 || x_dtype == DS_F32, DS_EINVAL,
             "moe_decode_noalloc: x_dtype must be DS_BF16 or DS_F32");
  DS_REQUIRE(ds::aligned(x, 16) && ds::aligned(out, 4), DS_EALIGN,
             "moe_decode_noalloc: x 16-byte and out 4-byte aligned");
  // The generic kernels are the fallback of every call: their scratch must fit.
  const WsLayout w = ws_layout(desc, tokens);
  DS_REQUIRE(w.total <= kNoAllocScratchBytes, DS_ERANGE,
             "moe_decode_noalloc: this layer needs %zu bytes of scratch, the static limit is %zu "
             "(use ds_moe_decode with a workspace)",
             w.total, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch)) != DS_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The error word and the single-token kernel's control words are the only
  // scratch that must start at zero (every other byte the kernels read is
  // written earlier in the same call); clear them on the stream so that the
  // word reports this call alone and an earlier call that gave up leaves no
  // trace.
  DS_CHECK_CUDA(cudaMemsetAsync(scratch, 0, ds::decode::rd_control_bytes(*desc), s));
  DecodeArgs a;
  a.d = *desc;
  a.x = x;
  a.x_f32 = x_dtype == DS_F32;
  a.tokens = (int)tokens;
  a.ids = topk_ids;
  a.gates = topk_w;
  a.out = out;
  a.h = reinterpret_cast<float*>(static_cast<char*>(scratch) + w.h_off);
  a.max_slots = w.max_slots;
  a.h_stride = w.h_stride;
  a.err = static_cast<int*>(scratch);
  return dispatch(a, scratch, kNoAllocScratchBytes, s);
}

extern "C" int ds_moe_decode_noalloc_status(int32_t* err, void* stream) {
  DS_REQUIRE(err != nullptr, DS_EINVAL, "moe_decode_noalloc_status: null output");
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != DS_OK) return st;
  DS_CHECK_CUDA(cudaMemcpyAsync(err, scratch, sizeof(int32_t), cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return DS_OK;
}
