// Shared definitions of the decode MoE kernels (moe_decode.cu: kernel
// selection and generic path, moe_decode_rd.cu: single-token register
// dequant, moe_decode_t5.cu: tcgen05, moe_decode_q3.cu: q3 banks).
#pragma once

#include "ds_common.cuh"

namespace ds {
namespace decode {

constexpr int kMaxTokens = 8;

// Bytes [0, kWsReserved) of every decode workspace: the error word at offset
// 0 (written by every path) and, from byte 256, the single-token kernel's
// control words (grid barrier, shared-expert arrival counters), which must be
// zero before a call and are left zero by every call that completes.  No
// path lays any other data out below kWsReserved, so calls of different
// layers and paths can share one workspace.
constexpr size_t kWsReserved = 4096;
constexpr int kMaxEntries = 128;  // tokens * top_k

// Error bits written to the workspace error word.
constexpr int kErrExpertRange = 1;
constexpr int kErrWaitTimeout = 2;

struct DecodeArgs {
  DsMoeDesc d;
  const void* x;      // [T, H] bf16 or f32 (x_f32)
  int x_f32;          // 1: x and out are f32; 0: bf16
  int tokens;
  const int32_t* ids; // [T, k]
  const float* gates; // [T, k]
  void* out;          // [T, H], dtype of x
  float* h;           // [max_slots + 1][T][h_stride] f32
  int max_slots;      // routed slots reserved = min(T*k, E)
  int h_stride;       // max(I, shared_inter), multiple of 4
  int* err;           // device error word
  // tcgen05 and q3 paths only: the shared expert is added to output rows
  // [sh_row0, sh_row1) (expert-parallel ranks add it to their own rows)
  int sh_row0 = 0, sh_row1 = 1 << 30;
  // tcgen05 and q3 paths only: row stride (elements) of shared_w2 when the
  // shared expert is a column slice of a wider one (0: shared_inter), and an
  // f32 [T, H] output that receives the shared expert's sum unrounded
  // instead of adding it to `out` (expert-parallel ranks that each hold a
  // slice)
  int sh_w2_ld = 0;
  float* out_sh = nullptr;
  // tcgen05 path only: route inside the decode (ds_moe_decode_route).  With
  // logits [T, E] set, ids / gates are outputs the prep kernel writes.
  const float* logits = nullptr;
  const float* route_bias = nullptr;
  int route_kind = DS_ROUTE_SOFTMAX;
  float route_scale = 1.0f;
};

// Routed slots of a decode call, built per CTA in shared memory (blockDim >=
// tokens * top_k threads; ends with __syncthreads).
struct Slots {
  int count;
  int expert[kMaxEntries];
  uint32_t mask[kMaxEntries];                 // bit t: token t routed here
  float gate[kMaxEntries][kMaxTokens];
  int ids[kMaxEntries];
  int first[kMaxEntries];
};

// Distinct routed experts in ascending id, with each token's gate taken from
// its first slot holding that expert (src/deepseeker/mlx_forward.py:394-404).
__device__ inline void build_slots(const DecodeArgs& a, Slots& s) {
  const int tid = threadIdx.x;
  const int k = a.d.top_k;
  const int n = a.tokens * k;
  if (tid < kMaxEntries) {
    s.mask[tid] = 0u;
#pragma unroll
    for (int t = 0; t < kMaxTokens; ++t) s.gate[tid][t] = 0.0f;
  }
  if (tid == 0) s.count = 0;
  if (tid < n) {
    int id = a.ids[tid];
    if (id >= a.d.n_experts) {
      atomicOr(a.err, 1);
      id = -1;
    }
    s.ids[tid] = id < 0 ? -1 : id;
  }
  __syncthreads();
  if (tid < n) {
    const int id = s.ids[tid];
    int first = id >= 0;
    for (int j = 0; j < tid && first; ++j) first = (s.ids[j] != id);
    s.first[tid] = first;
  }
  __syncthreads();
  if (tid < n) {
    const int id = s.ids[tid];
    if (id >= 0) {
      int rank = 0;
      for (int j = 0; j < n; ++j) rank += (s.first[j] && s.ids[j] < id);
      if (s.first[tid]) {
        s.expert[rank] = id;
        atomicAdd(&s.count, 1);
      }
      const int t = tid / k;
      int first_in_row = 1;
      for (int j = t * k; j < tid; ++j) first_in_row &= (s.ids[j] != id);
      if (first_in_row) {
        s.gate[rank][t] = a.gates[tid];
        atomicOr(&s.mask[rank], 1u << t);
      }
    }
  }
  __syncthreads();
}


// Single-token register-dequant pipeline (moe_decode_rd.cu): FP4 banks (no
// scale atoms needed), bf16 x, one cooperative kernel per layer.  Its
// workspace holds control words that must be zero before the first call and
// that every completed call leaves zero.
bool rd_supported(const DecodeArgs& a);
size_t rd_workspace_bytes(const DsMoeDesc& d);
size_t rd_control_bytes(const DsMoeDesc& d);  // leading workspace bytes: error word + control words
int launch_rd(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st);

// tcgen05 pipeline for 1..8 tokens (moe_decode_t5.cu): FP4 banks that carry
// prepared scale atoms, bf16 x.  Needs its own workspace size.
bool t5_supported(const DecodeArgs& a);
size_t t5_workspace_bytes(const DsMoeDesc& d, int tokens);
int launch_t5(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st);

// CUDA-core pipeline for q3 routed banks, 1..8 tokens, bf16 x
// (moe_decode_q3.cu).  Needs its own workspace size.
bool q3_supported(const DecodeArgs& a);
size_t q3_workspace_bytes(const DsMoeDesc& d, int tokens);
int launch_q3(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st);

}  // namespace decode
}  // namespace ds
