// Router: per token, select top_k experts and their gates.
//
// One CTA per row.  Selection is k rounds of a block-wide arg-max over the
// row's keys held in shared memory (n_experts <= 1024, top_k <= 32), so the
// slot order is descending key.  Tie-breaking follows each reference:
//   softmax       : descending probability, ties -> lower id
//                   (torch.argsort(-p, stable=True) restatement);
//   sqrt-softplus : the reference takes the LAST top_k of an ascending stable
//                   argsort of s + bias (src/deepseeker/mlx_forward.py:75-77),
//                   so among equal keys the HIGHER id is selected first.
#include <math.h>

#include "ds_common.cuh"

namespace {

constexpr int kRouteThreads = 256;
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

__global__ void __launch_bounds__(kRouteThreads)
route_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int n_experts,
                  int top_k, int kind, float route_scale, int32_t* __restrict__ ids,
                  float* __restrict__ weights) {
  __shared__ float key[kMaxExperts];
  __shared__ float val[kMaxExperts];   // softmax: exp(l - max); sqrtsoftplus: s
  __shared__ KeyIdx warp_best[kRouteThreads / 32];
  __shared__ float red[kRouteThreads / 32];
  __shared__ int chosen[kMaxTopK];
  __shared__ float total_s;

  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* lg = logits + (int64_t)row * n_experts;
  const bool ties_high = (kind != DS_ROUTE_SOFTMAX);

  // ---- keys
  float local_max = -INFINITY;
  for (int e = tid; e < n_experts; e += kRouteThreads) {
    const float l = lg[e];
    if (kind == DS_ROUTE_SOFTMAX) {
      key[e] = l;
      local_max = fmaxf(local_max, l);
    } else {
      // softplus(l) = logaddexp(l, 0) = max(l, 0) + log1p(exp(-|l|))
      const float s = (kind == DS_ROUTE_SCORES) ? l : sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
      val[e] = s;
      key[e] = s + (bias ? bias[e] : 0.0f);
    }
  }
  if (kind == DS_ROUTE_SOFTMAX) {
    for (int o = 16; o; o >>= 1) local_max = fmaxf(local_max, __shfl_xor_sync(0xffffffffu, local_max, o));
    if (lane == 0) red[warp] = local_max;
    __syncthreads();
    float mx = red[0];
    for (int w = 1; w < kRouteThreads / 32; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float local_sum = 0.0f;
    for (int e = tid; e < n_experts; e += kRouteThreads) {
      const float p = expf(key[e] - mx);
      val[e] = p;
      local_sum += p;
    }
    for (int o = 16; o; o >>= 1) local_sum += __shfl_xor_sync(0xffffffffu, local_sum, o);
    if (lane == 0) red[warp] = local_sum;
    __syncthreads();
    if (tid == 0) {
      float s = 0.0f;
      for (int w = 0; w < kRouteThreads / 32; ++w) s += red[w];
      total_s = s;
    }
    __syncthreads();
    // probabilities become the selection key (ties on p -> lower id)
    for (int e = tid; e < n_experts; e += kRouteThreads) {
      const float p = val[e] / total_s;
      val[e] = p;
      key[e] = p;
    }
  }
  __syncthreads();

  // ---- k rounds of arg-max
  for (int r = 0; r < top_k; ++r) {
    KeyIdx best{-INFINITY, -1};
    for (int e = tid; e < n_experts; e += kRouteThreads) {
      KeyIdx c{key[e], e};
      if (!(c.key == c.key)) continue;  // NaN never selected
      if (beats(c, best, ties_high)) best = c;
    }
    for (int o = 16; o; o >>= 1) {
      KeyIdx other{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
      if (beats(other, best, ties_high)) best = other;
    }
    if (lane == 0) warp_best[warp] = best;
    __syncthreads();
    if (tid == 0) {
      KeyIdx b = warp_best[0];
      for (int w = 1; w < kRouteThreads / 32; ++w)
        if (beats(warp_best[w], b, ties_high)) b = warp_best[w];
      chosen[r] = b.idx;
      if (b.idx >= 0) key[b.idx] = __uint_as_float(0x7FC00000u);  // remove (NaN)
    }
    __syncthreads();
  }

  // ---- gates
  if (tid == 0) {
    float s = 0.0f;
    for (int r = 0; r < top_k; ++r) s += (chosen[r] >= 0) ? val[chosen[r]] : 0.0f;
    for (int r = 0; r < top_k; ++r) {
      const int e = chosen[r];
      float w = 0.0f;
      if (e >= 0) {
        w = (kind == DS_ROUTE_SOFTMAX) ? val[e] / s : (val[e] / (s + 1e-20f)) * route_scale;
      }
      ids[(int64_t)row * top_k + r] = e;
      weights[(int64_t)row * top_k + r] = w;
    }
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
  route_topk_kernel<<<(unsigned)rows, kRouteThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  DS_CHECK_LAUNCH("route_topk_kernel");
  return DS_OK;
}
