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

namespace {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;
constexpr int kRouteThreads = 256;

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

// Order-preserving map of a float key to u32 (larger key -> larger code);
// -0.0 is folded onto +0.0 (they compare equal) and NaN maps to 0, which no
// valid key takes.
__device__ __forceinline__ uint32_t key_code(float k) {
  if (k != k) return 0u;
  const uint32_t u = __float_as_uint(k + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
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
  __shared__ int sel[kMaxTopK];
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* lg = logits + (int64_t)row * n_experts;
  const bool ties_high = (kind != DS_ROUTE_SOFTMAX);
  constexpr int kPerThread = kMaxExperts / kRouteThreads;
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
        // softplus(l) = logaddexp(l, 0) = max(l, 0) + log1p(exp(-|l|))
        const float sc = (kind == DS_ROUTE_SCORES) ? l : sqrtf(fmaxf(l, 0.0f) + log1pf(expf(-fabsf(l))));
        val[j] = sc;
        key[j] = sc + (bias ? bias[e] : 0.0f);
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
      scode[e] = key_code(key[j]);
      sval[e] = val[j];
    }
  }
  __syncthreads();
  if (tid >= 32) return;
  // ---- selection, one warp: lane l holds experts l + 32 j as packed
  // (key code << 32 | tie bits); tie bits order equal keys by the tie rule
  const int lane = tid;
  uint64_t pk[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    const uint32_t c = e < n_experts ? scode[e] : 0u;
    const uint32_t tb = ties_high ? (uint32_t)e : (uint32_t)(0xFFFFu - e);
    pk[j] = c ? (((uint64_t)c << 32) | tb) : 0ull;
  }
  int chosen = -1;
  for (int r = 0; r < top_k; ++r) {
    uint64_t best = 0ull;
#pragma unroll
    for (int j = 0; j < kPer; ++j) best = pk[j] > best ? pk[j] : best;
    const uint32_t hi = (uint32_t)(best >> 32);
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
    if (mhi == 0u) break;                                  // no valid key left (warp-uniform)
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)best : 0u);
    const int e = ties_high ? (int)mlo : (int)(0xFFFFu - mlo);
    const int jt = (e & 31) == lane ? (e >> 5) : -1;       // this lane's taken key, if any
#pragma unroll
    for (int j = 0; j < kPer; ++j) pk[j] = j == jt ? 0ull : pk[j];
    if (lane == r) chosen = e;
  }
  if (lane < top_k) sel[lane] = chosen;
  __syncwarp();
  if (lane < top_k) {
    float total = 0.0f;                    // chosen values summed in slot order
    for (int r = 0; r < top_k; ++r)
      if (sel[r] >= 0) total += sval[sel[r]];
    float w = 0.0f;
    if (chosen >= 0) {
      const float v = sval[chosen];
      w = (kind == DS_ROUTE_SOFTMAX) ? v / total : (v / (total + 1e-20f)) * route_scale;
    }
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
