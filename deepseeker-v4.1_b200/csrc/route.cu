// Router: per token, select top_k experts and their gates.
//
// Selection is k rounds of a warp-wide arg-max over the row's keys
// (n_experts <= 1024, top_k <= 32), so the slot order is descending key.  Tie-breaking follows each reference:
//   softmax       : descending probability, ties -> lower id
//                   (torch.argsort(-p, stable=True) restatement);
//   sqrt-softplus : the reference takes the LAST top_k of an ascending stable
//                   argsort of s + bias (src/deepseeker/mlx_forward.py:75-77),
//                   so among equal keys the HIGHER id is selected first.
#include <math.h>

#include "ds_common.cuh"

namespace {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;

struct KeyIdx {
  float key;
  int idx;
};

// a "beats" b under the tie rule.  NaN keys never win.
__device__ __forceinline__ bool beats(const KeyIdx& a, const KeyIdx& b, bool ties_high) {
  if (a.idx < 0) return false;
  if (b.idx < 0) return true;
  if (a.key > b.key) return true;
  if (a.key < b.key) return false;
  return ties_high ? (a.idx > b.idx) : (a.idx < b.idx);
}

// One warp per row: each lane holds n_experts/32 keys in registers; k rounds
// of a shuffle arg-max pick the experts.  The kernel first lets the next
// kernel on the stream (the MoE layer, launched with programmatic stream
// serialisation) start its prologue; that kernel waits for this one before
// reading the routing.
// kPer = keys per lane (n_experts <= 32 * kPer), a compile-time bound so the
// per-round scans cover only the live keys.
template <int kPer>
__global__ void __launch_bounds__(32)
route_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int n_experts,
                  int top_k, int kind, float route_scale, int32_t* __restrict__ ids,
                  float* __restrict__ weights) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int row = blockIdx.x, lane = threadIdx.x;
  const float* lg = logits + (int64_t)row * n_experts;
  const bool ties_high = (kind != DS_ROUTE_SOFTMAX);
  const float qnan = __uint_as_float(0x7FC00000u);
  float key[kPer], val[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    key[j] = qnan;
    val[j] = 0.0f;
    if (e < n_experts) {
      const float l = lg[e];
      if (kind == DS_ROUTE_SOFTMAX) {
        val[j] = l;
        mx = fmaxf(mx, l);
      } else {
        // softplus(l) = logaddexp(l, 0) = max(l, 0) + log1p(exp(-|l|))
        const float sc = (kind == DS_ROUTE_SCORES) ? l : sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
        val[j] = sc;
        key[j] = sc + (bias ? bias[e] : 0.0f);
      }
    }
  }
  if (kind == DS_ROUTE_SOFTMAX) {
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (lane + 32 * j < n_experts) {
        val[j] = expf(val[j] - mx);
        sum += val[j];
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (lane + 32 * j < n_experts) {
        val[j] = val[j] / sum;  // probability: the selection key (ties -> lower id)
        key[j] = val[j];
      }
    }
  }
  float chosen_val = 0.0f, total = 0.0f;  // lane r keeps slot r
  int chosen_id = -1;
  for (int r = 0; r < top_k; ++r) {
    KeyIdx best{-INFINITY, -1};
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      KeyIdx c{key[j], lane + 32 * j};
      if (c.key == c.key && beats(c, best, ties_high)) best = c;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      KeyIdx other{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
      if (beats(other, best, ties_high)) best = other;
    }
    float v = 0.0f;
    if (best.idx >= 0 && (best.idx & 31) == lane) {
      const int j = best.idx >> 5;
#pragma unroll
      for (int q = 0; q < kPer; ++q)
        if (q == j) {
          v = val[q];
          key[q] = qnan;  // remove
        }
    }
    v = __shfl_sync(0xffffffffu, v, best.idx >= 0 ? (best.idx & 31) : 0);
    if (best.idx >= 0) total += v;
    if (lane == r) {
      chosen_id = best.idx;
      chosen_val = best.idx >= 0 ? v : 0.0f;
    }
  }
  if (lane < top_k) {
    float w = 0.0f;
    if (chosen_id >= 0)
      w = (kind == DS_ROUTE_SOFTMAX) ? chosen_val / total : (chosen_val / (total + 1e-20f)) * route_scale;
    ids[(int64_t)row * top_k + lane] = chosen_id;
    weights[(int64_t)row * top_k + lane] = w;
  }
}

}  // namespace

extern "C" int ds_route_topk(const float* logits, const float* bias, int64_t rows, int n_experts,
                             int top_k, int kind, float route_scale, int32_t* ids, float* weights,
                             void* stream) {
  DS_REQUIRE(rows >= 0, DS_EINVAL, "route_topk: negative rows");
  DS_REQUIRE(n_experts >= 1 && n_experts <= kMaxExperts, DS_EINVAL,
             "route_topk: n_experts must be in [1, %d]", kMaxExperts);
  DS_REQUIRE(top_k >= 1 && top_k <= kMaxTopK && top_k <= n_experts, DS_EINVAL,
             "route_topk: top_k must be in [1, min(%d, n_experts)]", kMaxTopK);
  DS_REQUIRE(kind == DS_ROUTE_SOFTMAX || kind == DS_ROUTE_SQRTSOFTPLUS || kind == DS_ROUTE_SCORES, DS_EINVAL,
             "route_topk: unknown kind %d", kind);
  if (rows == 0) return DS_OK;
  DS_REQUIRE(rows <= 0x7fffffff, DS_EINVAL, "route_topk: too many rows");
  DS_REQUIRE(logits && ids && weights, DS_EINVAL, "route_topk: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = (unsigned)rows;
  const int per = (n_experts + 31) / 32;
  if (per <= 1)
    route_topk_kernel<1><<<g, 32, 0, st>>>(logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 2)
    route_topk_kernel<2><<<g, 32, 0, st>>>(logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 4)
    route_topk_kernel<4><<<g, 32, 0, st>>>(logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 8)
    route_topk_kernel<8><<<g, 32, 0, st>>>(logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 16)
    route_topk_kernel<16><<<g, 32, 0, st>>>(logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else
    route_topk_kernel<32><<<g, 32, 0, st>>>(logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  DS_CHECK_LAUNCH("route_topk_kernel");
  return DS_OK;
}
