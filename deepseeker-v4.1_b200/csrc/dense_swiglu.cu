// Dense-weight SwiGLU expert FFN over explicit (row, expert) pairs: the GPU
// execution behind grouped_swiglu / naive_swiglu when the experts are given as
// dense matrices (src/deepseeker/grouped.py:34-81: gate/up [H, I], down [I, H],
// y = (g * sigmoid(g) * (x up)) down, g = x gate, optional route weight after
// the down projection, scatter-add into the token rows).
//
// Pass 1: one CTA per pair computes y_pair in f32 (x row and h in shared
// memory; weight columns read coalesced across threads).
// Pass 2: every token row sums its pairs in the order the caller lists them
// (CSR: row_ptr[T + 1] into the pair arrays), which fixes the addition order
// of the reference loop it replaces.
#include "ds_common.cuh"

namespace {

__global__ void __launch_bounds__(256) pair_ffn_kernel(const float* __restrict__ x, int T, int E, int H, int I,
                                                       const float* __restrict__ gate, const float* __restrict__ upw,
                                                       const float* __restrict__ down, const int32_t* __restrict__ prow,
                                                       const int32_t* __restrict__ pexp,
                                                       const float* __restrict__ pw, float limit,
                                                       float* __restrict__ y) {
  extern __shared__ float sm[];
  float* xs = sm;       // [H]
  float* hs = sm + H;   // [I]
  const int pr = blockIdx.x;
  const int row = prow[pr], e = pexp[pr];
  if (row < 0 || row >= T || e < 0 || e >= E) {  // guarded: the host validates, this keeps reads in bounds
    for (int j = threadIdx.x; j < H; j += blockDim.x) y[(size_t)pr * H + j] = __int_as_float(0x7FC00000);
    return;
  }
  for (int i = threadIdx.x; i < H; i += blockDim.x) xs[i] = x[(size_t)row * H + i];
  __syncthreads();
  const float* G = gate + (size_t)e * H * I;
  const float* U = upw + (size_t)e * H * I;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    float g = 0.f, u = 0.f;
    for (int k = 0; k < H; ++k) {
      g = fmaf(xs[k], G[(size_t)k * I + i], g);
      u = fmaf(xs[k], U[(size_t)k * I + i], u);
    }
    if (limit > 0.f) {
      g = fminf(g, limit);
      u = fminf(fmaxf(u, -limit), limit);
    }
    hs[i] = (g / (1.0f + expf(-g))) * u;
  }
  __syncthreads();
  const float* D = down + (size_t)e * I * H;
  const float w = pw ? pw[pr] : 1.0f;
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < I; ++i) acc = fmaf(hs[i], D[(size_t)i * H + j], acc);
    y[(size_t)pr * H + j] = acc * w;
  }
}

__global__ void __launch_bounds__(256) row_sum_kernel(const float* __restrict__ y, const int32_t* __restrict__ row_ptr,
                                                      int H, float* __restrict__ out) {
  const int t = blockIdx.x;
  const int b = row_ptr[t], e = row_ptr[t + 1];
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    float acc = 0.f;
    for (int p = b; p < e; ++p) acc += y[(size_t)p * H + j];
    out[(size_t)t * H + j] = acc;
  }
}

}  // namespace

extern "C" int ds_dense_swiglu_workspace_size(int64_t n_pairs, int hidden, size_t* bytes) {
  DS_REQUIRE(n_pairs >= 0 && hidden > 0 && bytes, DS_EINVAL, "dense_swiglu_workspace_size: bad arguments");
  *bytes = (size_t)n_pairs * hidden * sizeof(float);
  return DS_OK;
}

extern "C" int ds_dense_swiglu(const float* x, int64_t tokens, int hidden, int inter, int n_experts,
                               const float* gate, const float* up, const float* down, int64_t n_pairs,
                               const int32_t* pair_row, const int32_t* pair_expert, const float* pair_weight,
                               const int32_t* row_ptr, float swiglu_limit, float* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  DS_REQUIRE(tokens >= 0 && hidden > 0 && inter > 0 && n_experts > 0 && n_pairs >= 0, DS_EINVAL,
             "dense_swiglu: bad shape");
  DS_REQUIRE((size_t)hidden + inter <= 12 * 1024, DS_ENOTSUP, "dense_swiglu: hidden + inter must be <= 12288");
  DS_REQUIRE(tokens == 0 || (x && out && row_ptr), DS_EINVAL, "dense_swiglu: null pointer");
  DS_REQUIRE(n_pairs == 0 || (gate && up && down && pair_row && pair_expert && workspace), DS_EINVAL,
             "dense_swiglu: null pointer");
  DS_REQUIRE(workspace_bytes >= (size_t)n_pairs * hidden * sizeof(float), DS_EINVAL,
             "dense_swiglu: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* y = static_cast<float*>(workspace);
  if (n_pairs > 0) {
    const size_t smem = ((size_t)hidden + inter) * sizeof(float);
    DS_CHECK_CUDA(cudaFuncSetAttribute(pair_ffn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    pair_ffn_kernel<<<(unsigned)n_pairs, 256, smem, s>>>(x, (int)tokens, n_experts, hidden, inter, gate, up, down, pair_row, pair_expert,
                                                         pair_weight, swiglu_limit, y);
    DS_CHECK_LAUNCH("pair_ffn_kernel");
  }
  if (tokens > 0) {
    row_sum_kernel<<<(unsigned)tokens, 256, 0, s>>>(y, row_ptr, hidden, out);
    DS_CHECK_LAUNCH("row_sum_kernel");
  }
  return DS_OK;
}
