// Pieces shared by the grouped expert FFN over FP4 banks (grouped.cu) and
// over q3 banks (grouped_q3.cu): bounded waits, SwiGLU, the e4m3 piece
// scales of the activation operands, the scale-atom byte layout, the
// combine kernel and tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "ds_common.cuh"
#include "ptx.cuh"

namespace ds {
namespace grouped {

constexpr int kBlock = 16;                    // expert runs are padded to this many rows (MMA N step)
constexpr int kSfAtom = 512;                  // 128 rows x 4 ue8m0 bytes (one 128-wide K chunk)
constexpr uint64_t kWaitNs = 2000000000ull;   // 2 s
constexpr int kErrTimeout = 2;

enum { GATEUP = 0, DOWN = 1 };

// Bounded mbarrier wait that also gives up when another role has aborted.
// Between checks the thread is suspended in try_wait (it resumes when the
// phase completes), so waiting roles leave the issue slots to the warps
// that convert and drain.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
  using namespace ds::ptx;
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      *abort = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

// Warp-uniform version: lane 0 waits, the verdict is broadcast, and every lane
// then observes the completed phase itself (it cannot advance without us).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_or_abort(bar, parity, abort, err) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)ds::ptx::mbar_test_wait(bar, parity);
  return ok != 0;
}

__device__ __forceinline__ float silu_glu(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  return (g / (1.0f + expf(-g))) * u;
}

// ue8m0 byte for piece `pc` of a block whose maximum has f32 exponent field
// `ef`: piece 0 maps the maximum into [128, 256), each later piece is 2^5 finer.
__device__ __forceinline__ int piece_scale(int ef, int pc) { return min(max(ef - 7 - 5 * pc, 1), 253); }
__device__ __forceinline__ float scale_of(int sfb) { return __uint_as_float((uint32_t)sfb << 23); }
__device__ __forceinline__ float inv_scale_of(int sfb) { return __uint_as_float((uint32_t)(254 - sfb) << 23); }

// Offset of (row r, k-block kb of the chunk) inside a 512-byte scale atom.
__device__ __forceinline__ int atom_off(int r, int kb) { return (r & 31) * 16 + (r >> 5) * 4 + kb; }

// out[t] = sum over slots (top-k order) of [w] * y[row of the pair].
// An expert id out of range makes the align step report n_pad = -1 and leave
// the pair positions unwritten: the output is then NaN and error bit 1 is set.
template <typename OutT>
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ pos,
                                                      const float* __restrict__ topk_w, const int32_t* n_pad, int* err,
                                                      int k, int H, int route_after, OutT* __restrict__ out) {
  const int t = blockIdx.x;
  if (*n_pad < 0) {
    if (t == 0 && threadIdx.x == 0) atomicOr(err, 1);
    for (int h = threadIdx.x; h < H; h += blockDim.x) out[(size_t)t * H + h] = (OutT)__int_as_float(0x7FC00000);
    return;
  }
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < k; ++s) {
      const int ps = pos[t * k + s];
      if (ps < 0) continue;
      const float w = route_after ? topk_w[t * k + s] : 1.0f;
      const float4 v = *reinterpret_cast<const float4*>(y + (size_t)ps * H + h);
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    OutT* o = out + (size_t)t * H + h;
    if constexpr (sizeof(OutT) == 4) {
      *reinterpret_cast<float4*>(o) = acc;
    } else {
      __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y), b = __floats2bfloat162_rn(acc.z, acc.w);
      *reinterpret_cast<uint2*>(o) =
          make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    }
  }
}

// Launches the combine kernel for out_dtype (DS_BF16 or DS_F32).
int launch_combine(const float* y, const int32_t* pos, const float* topk_w, const int32_t* n_pad, int* err, int k,
                   int H, int route_after, void* out, int out_dtype, int64_t tokens, cudaStream_t s);

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

// Activation pieces [rows][row_bytes] (UINT8, 128-byte swizzle) viewed as
// {128 B, rows, row_bytes / 128}; a box is 128 B x box_rows.
bool map_pieces(CUtensorMap* m, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows);

inline size_t up(size_t v, size_t a = 1024) { return (v + a - 1) / a * a; }

// q3 banks through the grouped path (grouped_q3.cu).
size_t q3_workspace_bytes(const DsMoeDesc* d, int64_t T);
int q3_validate(const DsMoeDesc* d);
int q3_ffn(const DsMoeDesc* d, const void* x, int64_t tokens, const int32_t* topk_ids, const float* topk_w,
           void* out, int out_dtype, void* workspace, size_t workspace_bytes, cudaStream_t s);

}  // namespace grouped
}  // namespace ds
