// Shared definitions of the decode MoE kernels (moe_decode.cu: generic path,
// moe_decode_tc.cu: single-token tensor-core pipeline).
#pragma once

#include "ds_common.cuh"

namespace ds {
namespace decode {

constexpr int kMaxTokens = 8;
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
  // tcgen05 path only: the shared expert is added to output rows
  // [sh_row0, sh_row1) (expert-parallel ranks add it to their own rows)
  int sh_row0 = 0, sh_row1 = 1 << 30;
  // tcgen05 path only: row stride (elements) of shared_w2 when the shared
  // expert is a column slice of a wider one (0: shared_inter), and an f32
  // [T, H] output that receives the shared expert's sum unrounded instead
  // of adding it to `out` (expert-parallel ranks that each hold a slice)
  int sh_w2_ld = 0;
  float* out_sh = nullptr;
};

// Single-token tensor-core pipeline (moe_decode_tc.cu).  Returns true and
// launches when the geometry is supported; false means "use the generic path".
bool tc_supported(const DecodeArgs& a);
int launch_tc(const DecodeArgs& a, cudaStream_t st);
// Same launch, tensor maps encoded on the stack for this call only (no cache,
// so no host heap either).
int launch_tc_uncached(const DecodeArgs& a, cudaStream_t st);

// tcgen05 pipeline for 1..8 tokens (moe_decode_t5.cu): FP4 banks that carry
// prepared scale atoms, bf16 x.  Needs its own workspace size.
bool t5_supported(const DecodeArgs& a);
size_t t5_workspace_bytes(const DsMoeDesc& d, int tokens);
int launch_t5(const DecodeArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st);

}  // namespace decode
}  // namespace ds
