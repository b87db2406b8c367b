// Router: per token, select top_k experts and their gates.
//
// One 256-thread block per row: all threads compute the keys (softmax
// probabilities or sqrt-softplus scores + bias); then one warp selects the
// top_k with top_k rounds of a two-step warp maximum (redux.sync) over keys
// packed as (order-preserving key bits, tie-break bits).  Slots come out in
// descending key order; tie-breaking follows each reference:
//   softmax       : descending probability, ties -> lower id
//                   (torch.argsort(-p, stable=True) restatement);
//   sqrt-softplus : the reference takes the LAST top_k of an ascending stable
//                   argsort of s + bias (src/deepseeker/mlx_forward.py:75-77),
//                   so among equal keys the HIGHER id is selected first.
// NaN keys never win; slots beyond the valid keys get id -1 and gate 0.
#include <math.h>

#include "ds_common.cuh"
#include "route.cuh"

namespace {

using ds::route::kMaxExperts;
using ds::route::kMaxTopK;
constexpr int kRouteThreads = ds::route::kRowThreads;

// Block-wide reduction in a fixed order (warp xor tree, then warps 0..7 in
// order), so every thread gets the same value bit for bit.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, w) : v + w;
  }
  __syncthreads();                       // red[] may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kRouteThreads / 32; ++w) r = kMax ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// kPer = keys per lane of the selecting warp (n_experts <= 32 * kPer).  The
// kernel first lets the next kernel on the stream (launched with
// programmatic stream serialisation) start its prologue; that kernel waits
// for this one before reading the routing.
template <int kPer>
__global__ void __launch_bounds__(kRouteThreads)
route_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int n_experts,
                  int top_k, int kind, float route_scale, int32_t* __restrict__ ids,
                  float* __restrict__ weights) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // launched with programmatic stream serialisation: the logits may come from
  // the previous kernel, so wait for it (a no-op after a kernel that did not
  // trigger early)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ uint32_t scode[kMaxExperts];
  __shared__ float sval[kMaxExperts];
  __shared__ float red[kRouteThreads / 32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* lg = logits + (int64_t)row * n_experts;
  const bool ties_high = (kind != DS_ROUTE_SOFTMAX);
  constexpr int kPerThread = ds::route::kPerThread;
  float key[kPerThread], val[kPerThread];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int e = tid + kRouteThreads * j;
    key[j] = __uint_as_float(0x7FC00000u);
    val[j] = 0.0f;
    if (e < n_experts) {
      const float l = lg[e];
      if (kind == DS_ROUTE_SOFTMAX) {
        val[j] = l;
        mx = fmaxf(mx, l);
      } else {
        ds::route::score_key(l, kind, bias, e, val[j], key[j]);
      }
    }
  }
  if (kind == DS_ROUTE_SOFTMAX) {
    mx = block_reduce<true>(mx, red);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j)
      if (tid + kRouteThreads * j < n_experts) {
        val[j] = expf(val[j] - mx);
        sum += val[j];
      }
    sum = block_reduce<false>(sum, red);
#pragma unroll
    for (int j = 0; j < kPerThread; ++j)
      if (tid + kRouteThreads * j < n_experts) {
        val[j] = val[j] / sum;  // probability: the selection key (ties -> lower id)
        key[j] = val[j];
      }
  }
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int e = tid + kRouteThreads * j;
    if (e < n_experts) {
      scode[e] = ds::route::key_code(key[j]);
      sval[e] = val[j];
    }
  }
  __syncthreads();
  if (tid >= 32) return;
  // ---- selection, one warp: lane l holds experts l + 32 j
  const int lane = tid;
  uint64_t pk[kPer];
  float vv[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    pk[j] = e < n_experts ? ds::route::pack_key(scode[e], e, ties_high) : 0ull;
    vv[j] = e < n_experts ? sval[e] : 0.0f;
  }
  int chosen;
  float w;
  ds::route::select_topk<kPer>(pk, vv, top_k, kind, route_scale, ties_high, lane, chosen, w);
  if (lane < top_k) {
    ids[(int64_t)row * top_k + lane] = chosen;
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
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t rc;
  if (per <= 2)
    rc = cudaLaunchKernelEx(&cfg, route_topk_kernel<2>, logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 4)
    rc = cudaLaunchKernelEx(&cfg, route_topk_kernel<4>, logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 8)
    rc = cudaLaunchKernelEx(&cfg, route_topk_kernel<8>, logits, bias, n_experts, top_k, kind, route_scale, ids, weights);
  else if (per <= 16)
    rc = cudaLaunchKernelEx(&cfg, route_topk_kernel<16>, logits, bias, n_experts, top_k, kind, route_scale, ids,
                            weights);
  else
    rc = cudaLaunchKernelEx(&cfg, route_topk_kernel<32>, logits, bias, n_experts, top_k, kind, route_scale, ids,
                            weights);
  DS_CHECK_CUDA(rc);
  DS_CHECK_LAUNCH("route_topk_kernel");
  return DS_OK;
}
