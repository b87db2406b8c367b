// Routing arithmetic shared by the router kernel (route.cu, one 256-thread
// block per row) and the decode prep kernel that routes inside its own launch
// (moe_decode_t5.cu, one warp per row).  Both forms compute the same keys,
// reduce them in the same order (the 256-thread block's: a warp xor tree per
// warp, then warps 0..7 folded in order) and select with the same warp
// procedure, so their ids and gates are equal bit for bit.
//
// Keys (src/deepseeker/mlx_forward.py:62-81 and the softmax top-k router):
//   softmax       : p = exp(l - max) / sum, key = p, gate = p / sum(chosen p)
//   sqrt-softplus : s = sqrt(softplus(l)), key = s + bias,
//                   gate = s / (sum(chosen s) + 1e-20) * route_scale
//   scores        : s = l, otherwise as sqrt-softplus
// Ties: softmax -> lower id first; the others -> higher id first (the
// reference takes the last top_k of an ascending stable argsort).  NaN keys
// never win; slots beyond the valid keys get id -1 and gate 0.
#pragma once

#include <math.h>
#include <stdint.h>

#include "ds_common.cuh"

namespace ds {
namespace route {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;
constexpr int kRowThreads = 256;                      // threads of the row kernel
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kPerThread = kMaxExperts / kRowThreads; // experts per thread of the row kernel

// Order-preserving map of a float key to u32 (larger key -> larger code);
// -0.0 is folded onto +0.0 (they compare equal) and NaN maps to 0, which no
// valid key takes.
__device__ __forceinline__ uint32_t key_code(float k) {
  if (k != k) return 0u;
  const uint32_t u = __float_as_uint(k + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Value and key of expert e for the score kinds (not softmax).
__device__ __forceinline__ void score_key(float l, int kind, const float* bias, int e, float& val, float& key) {
  // softplus(l) = logaddexp(l, 0) = max(l, 0) + log1p(exp(-|l|))
  const float sc = (kind == DS_ROUTE_SCORES) ? l : sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
  val = sc;
  key = sc + (bias ? bias[e] : 0.0f);
}

// Packed selection word of expert e: key code above, tie-break bits below.
__device__ __forceinline__ uint64_t pack_key(uint32_t code, int e, bool ties_high) {
  const uint32_t tb = ties_high ? (uint32_t)e : (uint32_t)(0xFFFFu - e);
  return code ? (((uint64_t)code << 32) | tb) : 0ull;
}

// Warp selection: lane l holds experts l + 32 j as packed words pk[j] and
// their values vv[j].  Top_k rounds of a two-step warp maximum; lane r < top_k
// gets the r-th chosen expert (descending key) and its gate, other lanes -1.
// The gate divides by the chosen values summed in slot order.
template <int kPer>
__device__ __forceinline__ void select_topk(uint64_t (&pk)[kPer], const float (&vv)[kPer], int top_k, int kind,
                                            float route_scale, bool ties_high, int lane, int& chosen_out,
                                            float& gate_out) {
  int chosen = -1;
  float cval = 0.0f;
  for (int r = 0; r < top_k; ++r) {
    uint64_t best = 0ull;
#pragma unroll
    for (int j = 0; j < kPer; ++j) best = pk[j] > best ? pk[j] : best;
    const uint32_t hi = (uint32_t)(best >> 32);
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
    if (mhi == 0u) break;                                // no valid key left (warp-uniform)
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)best : 0u);
    const int e = ties_high ? (int)mlo : (int)(0xFFFFu - mlo);
    const int jt = (e & 31) == lane ? (e >> 5) : -1;     // this lane's taken key, if any
    float mine = 0.0f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      mine = j == jt ? vv[j] : mine;
      pk[j] = j == jt ? 0ull : pk[j];
    }
    const float v = __shfl_sync(0xffffffffu, mine, e & 31);
    if (lane == r) {
      chosen = e;
      cval = v;
    }
  }
  float total = 0.0f;                                      // chosen values summed in slot order
#pragma unroll 8
  for (int r = 0; r < top_k; ++r) {
    const int c = __shfl_sync(0xffffffffu, chosen, r);
    const float v = __shfl_sync(0xffffffffu, cval, r);
    if (c >= 0) total += v;
  }
  float w = 0.0f;
  if (chosen >= 0) w = (kind == DS_ROUTE_SOFTMAX) ? cval / total : (cval / (total + 1e-20f)) * route_scale;
  chosen_out = chosen;
  gate_out = w;
}

// One row routed by one warp.  Expert e = lane + 32 jj belongs to thread
// (jj % 8) * 32 + lane of the row kernel as its element jj / 8; the softmax
// maximum and sum are formed per such thread in element order, reduced by an
// xor tree per row-kernel warp and folded over those warps in order, as the
// row kernel does.  Lane r < top_k returns the r-th expert and gate.
template <int kPer>
__device__ __forceinline__ void route_row_warp(const float* __restrict__ lg, const float* __restrict__ bias,
                                               int n_experts, int top_k, int kind, float route_scale, int lane,
                                               int& chosen, float& gate) {
  static_assert(kPer >= 1 && kPer <= kMaxExperts / 32, "experts per lane");
  float val[kPer];
  uint64_t pk[kPer];
  const bool ties_high = (kind != DS_ROUTE_SOFTMAX);
#pragma unroll
  for (int jj = 0; jj < kPer; ++jj) {
    const int e = lane + 32 * jj;
    val[jj] = 0.0f;
    pk[jj] = 0ull;
    if (e < n_experts) {
      const float l = lg[e];
      if (kind == DS_ROUTE_SOFTMAX) {
        val[jj] = l;
      } else {
        float key;
        score_key(l, kind, bias, e, val[jj], key);
        pk[jj] = pack_key(key_code(key), e, ties_high);
      }
    }
  }
  if (kind == DS_ROUTE_SOFTMAX) {
    float mx = 0.0f;
#pragma unroll
    for (int vw = 0; vw < kRowWarps; ++vw) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) {
        const int jj = vw + kRowWarps * j;
        if (jj < kPer && lane + 32 * jj < n_experts) m = fmaxf(m, val[jj]);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      mx = vw == 0 ? m : fmaxf(mx, m);
    }
    float sum = 0.0f;
#pragma unroll
    for (int vw = 0; vw < kRowWarps; ++vw) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) {
        const int jj = vw + kRowWarps * j;
        if (jj < kPer && lane + 32 * jj < n_experts) {
          val[jj] = expf(val[jj] - mx);
          s += val[jj];
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) s = s + __shfl_xor_sync(0xffffffffu, s, o);
      sum = vw == 0 ? s : sum + s;
    }
#pragma unroll
    for (int jj = 0; jj < kPer; ++jj) {
      const int e = lane + 32 * jj;
      if (e < n_experts) {
        val[jj] = val[jj] / sum;        // probability: the selection key (ties -> lower id)
        pk[jj] = pack_key(key_code(val[jj]), e, ties_high);
      }
    }
  }
  select_topk<kPer>(pk, val, top_k, kind, route_scale, ties_high, lane, chosen, gate);
}

}  // namespace route
}  // namespace ds
