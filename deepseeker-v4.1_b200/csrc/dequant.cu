// Standalone dequantisation / quantisation kernels (HBM-bound byte work).
//
//   ds_fp4_dequant        e2m1 + ue8m0 (or f32) scales -> f32 / bf16, bit-exact
//   ds_fp8_block_dequant  e4m3 + 32x32 ue8m0 blocks -> f32
//   ds_q3_dequant         3-bit affine (group 64) -> f32 / bf16
//   ds_q3_quantize        f32 -> 3-bit affine (builder rule)
//   ds_fp4_quantize       f32 -> e2m1 + ue8m0 (builder rule, synthetic weights)
//
// All arithmetic is IEEE round-to-nearest with denormals honoured: this file
// must never be built with --use_fast_math or -ftz=true.
#include "ds_common.cuh"

namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t work, int per_block = kThreads) {
  int64_t b = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)ds::sm_count() * 16;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

template <bool kU8Scale>
__device__ __forceinline__ float load_scale(const void* scales, int64_t i) {
  if (kU8Scale) return ds::u8m0_value(static_cast<const uint8_t*>(scales)[i]);
  return static_cast<const float*>(scales)[i];
}

// Vector path: one 16-byte chunk = 32 codes = exactly one scale block.
template <bool kU8Scale, bool kBf16Out>
__global__ void __launch_bounds__(kThreads)
fp4_dequant_chunks(const uint4* __restrict__ packed, int64_t n_chunks,
                   const void* __restrict__ scales, void* __restrict__ out) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n_chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = __ldg(packed + c);
    const float s = load_scale<kU8Scale>(scales, c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float r[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        r[i * 8 + j] = __fmul_rn(ds::e2m1_value((w[i] >> (4 * j)) & 0xFu), s);
      }
    }
    if (kBf16Out) {
      uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + c * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t p[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          __nv_bfloat162 b2 = __floats2bfloat162_rn(r[q * 8 + 2 * t], r[q * 8 + 2 * t + 1]);
          p[t] = *reinterpret_cast<uint32_t*>(&b2);
        }
        o[q] = make_uint4(p[0], p[1], p[2], p[3]);
      }
    } else {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + c * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
    }
  }
}

// Scalar path: one thread per packed byte (any alignment, any tail).
template <bool kU8Scale, bool kBf16Out>
__global__ void __launch_bounds__(kThreads)
fp4_dequant_bytes(const uint8_t* __restrict__ packed, int64_t first, int64_t n_bytes,
                  const void* __restrict__ scales, void* __restrict__ out) {
  for (int64_t b = first + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < n_bytes;
       b += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t byte = packed[b];
    const float s = load_scale<kU8Scale>(scales, b >> 4);
    const float lo = __fmul_rn(ds::e2m1_value(byte & 0xFu), s);
    const float hi = __fmul_rn(ds::e2m1_value(byte >> 4), s);
    if (kBf16Out) {
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
      o[2 * b] = __float2bfloat16_rn(lo);
      o[2 * b + 1] = __float2bfloat16_rn(hi);
    } else {
      float* o = static_cast<float*>(out);
      o[2 * b] = lo;
      o[2 * b + 1] = hi;
    }
  }
}

template <bool kU8Scale, bool kBf16Out>
int launch_fp4(const uint8_t* packed, int64_t n_bytes, const void* scales, void* out,
               cudaStream_t st) {
  int64_t first = 0;
  const bool vec = ds::aligned(packed, 16) && ds::aligned(out, 16) &&
                   (kU8Scale || ds::aligned(scales, 4));
  if (vec) {
    const int64_t n_chunks = n_bytes / 16;
    if (n_chunks > 0) {
      fp4_dequant_chunks<kU8Scale, kBf16Out><<<grid_for(n_chunks), kThreads, 0, st>>>(
          reinterpret_cast<const uint4*>(packed), n_chunks, scales, out);
      DS_CHECK_LAUNCH("fp4_dequant_chunks");
    }
    first = n_chunks * 16;
  }
  if (first < n_bytes) {
    fp4_dequant_bytes<kU8Scale, kBf16Out><<<grid_for(n_bytes - first), kThreads, 0, st>>>(
        packed, first, n_bytes, scales, out);
    DS_CHECK_LAUNCH("fp4_dequant_bytes");
  }
  return DS_OK;
}

// ---------------------------------------------------------------- FP8 (e4m3)

__device__ __forceinline__ float e4m3_value(uint32_t b) {
  const uint32_t s = (b >> 7) & 1u, e = (b >> 3) & 0xFu, m = b & 7u;
  float v;
  if (e == 0xFu && m == 7u) {
    v = __uint_as_float(0x7FC00000u);
  } else if (e == 0u) {
    v = __fmul_rn((float)m, 0.001953125f);  // m * 2^-9 (exact)
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  }
  return s ? -v : v;
}

__global__ void __launch_bounds__(kThreads)
fp8_block_dequant_kernel(const uint8_t* __restrict__ packed, int64_t rows, int64_t cols,
                         const uint8_t* __restrict__ scales, float* __restrict__ out) {
  const int64_t n = rows * cols;
  const int64_t sc = cols / 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const float s = ds::u8m0_value(scales[(r / 32) * sc + c / 32]);
    out[i] = __fmul_rn(e4m3_value(packed[i]), s);
  }
}

// ---------------------------------------------------------------- 3-bit affine

// Decode code e (0..63) of one group.  Group layout (six u32 words): word w
// in 0..3 holds the low two bits of element 16w+i at bits [2i, 2i+2); word
// 4+h holds bit 2: element 16(2h+v)+j at bit 8v+j and element 16(2h+v)+8+j at
// bit 16+8v+j (v in {0,1}, j < 8).
__device__ __forceinline__ uint32_t q3_code(const uint32_t (&w)[6], int e) {
  const int wi = e >> 4, j = e & 7, upper = (e >> 3) & 1;
  const int lo_shift = upper * 16 + 2 * j;
  const int h = wi >> 1, v = wi & 1;
  const int hi_shift = upper * 16 + 8 * v + j;
  return ((w[wi] >> lo_shift) & 3u) | (((w[4 + h] >> hi_shift) & 1u) << 2);
}

template <bool kBf16Out>
__global__ void __launch_bounds__(kThreads)
q3_dequant_kernel(const uint32_t* __restrict__ words, const __half* __restrict__ scales,
                  const __half* __restrict__ biases, int64_t n_groups, void* __restrict__ out) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n_groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    uint32_t w[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) w[i] = __ldg(words + g * 6 + i);
    const float s = __half2float(scales[g]);
    const float b = __half2float(biases[g]);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      float r[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) r[t] = __fadd_rn(__fmul_rn(s, (float)q3_code(w, q * 4 + t)), b);
      if (kBf16Out) {
        __nv_bfloat162 a = __floats2bfloat162_rn(r[0], r[1]);
        __nv_bfloat162 c = __floats2bfloat162_rn(r[2], r[3]);
        uint2 p = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&c));
        reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + g * 64)[q] = p;
      } else {
        reinterpret_cast<float4*>(static_cast<float*>(out) + g * 64)[q] =
            make_float4(r[0], r[1], r[2], r[3]);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
q3_quantize_kernel(const float* __restrict__ w, int64_t n_groups, uint32_t* __restrict__ words,
                   __half* __restrict__ scales, __half* __restrict__ biases) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < n_groups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const float* src = w + g * 64;
    float mn = src[0], mx = src[0];
    for (int i = 1; i < 64; ++i) {
      mn = fminf(mn, src[i]);
      mx = fmaxf(mx, src[i]);
    }
    const __half s16 = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), 7.0f));
    const __half b16 = __float2half_rn(mn);
    const float s = __half2float(s16), b = __half2float(b16);
    uint32_t out[6] = {0u, 0u, 0u, 0u, 0u, 0u};
    for (int e = 0; e < 64; ++e) {
      uint32_t q = 0u;
      if (s > 0.0f) {
        float t = rintf(__fdiv_rn(__fsub_rn(src[e], b), s));
        t = fminf(fmaxf(t, 0.0f), 7.0f);
        q = (uint32_t)t;
      }
      const int wi = e >> 4, j = e & 7, upper = (e >> 3) & 1;
      out[wi] |= (q & 3u) << (upper * 16 + 2 * j);
      out[4 + (wi >> 1)] |= ((q >> 2) & 1u) << (upper * 16 + 8 * (wi & 1) + j);
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) words[g * 6 + i] = out[i];
    scales[g] = s16;
    biases[g] = b16;
  }
}

// ---------------------------------------------------------------- FP4 quantiser

__global__ void __launch_bounds__(kThreads)
fp4_quantize_kernel(const float* __restrict__ w, int64_t n_blocks, uint8_t* __restrict__ packed,
                    uint8_t* __restrict__ scales) {
  for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < n_blocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const float* src = w + blk * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));
    int e = 0;
    if (amax > 0.0f) {
      const double a = (double)amax;
      e = (int)ceil(log2(a / 6.0));
      // exact fix-up: smallest e with amax <= 6 * 2^e
      while (a > ldexp(6.0, e)) ++e;
      while (a <= ldexp(6.0, e - 1)) --e;
      e = max(-127, min(127, e));
    }
    const double inv = ldexp(1.0, -e);
    uint32_t word[4] = {0u, 0u, 0u, 0u};
    for (int i = 0; i < 32; ++i) {
      const double sc = (double)src[i] * inv;
      const double m = fabs(sc);
      uint32_t code = (m > 0.25) + (m >= 0.75) + (m > 1.25) + (m >= 1.75) + (m > 2.5) +
                      (m >= 3.5) + (m > 5.0);
      if (sc < 0.0 && code > 0u) code |= 8u;
      word[i >> 3] |= code << (4 * (i & 7));
    }
    reinterpret_cast<uint4*>(packed)[blk] = make_uint4(word[0], word[1], word[2], word[3]);
    scales[blk] = (uint8_t)(e + 127);
  }
}

}  // namespace

// ============================================================================

extern "C" int ds_fp4_dequant(const uint8_t* packed, int64_t n_bytes, const void* scales,
                              int scale_kind, int64_t n_scales, void* out, int out_dtype,
                              void* stream) {
  DS_REQUIRE(n_bytes >= 0, DS_EINVAL, "fp4_dequant: negative size");
  const int64_t n = 2 * n_bytes;
  DS_REQUIRE(n_scales == (n + 31) / 32, DS_EINVAL, "scales must cover ceil(n/32) blocks");
  DS_REQUIRE(scale_kind == DS_F32 || scale_kind == DS_U8, DS_EINVAL,
             "fp4_dequant: scale_kind must be DS_F32 or DS_U8");
  DS_REQUIRE(out_dtype == DS_F32 || out_dtype == DS_BF16, DS_EINVAL,
             "fp4_dequant: out_dtype must be DS_F32 or DS_BF16");
  if (n_bytes == 0) return DS_OK;
  DS_REQUIRE(packed && scales && out, DS_EINVAL, "fp4_dequant: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (scale_kind == DS_U8) {
    return out_dtype == DS_BF16 ? launch_fp4<true, true>(packed, n_bytes, scales, out, st)
                                : launch_fp4<true, false>(packed, n_bytes, scales, out, st);
  }
  return out_dtype == DS_BF16 ? launch_fp4<false, true>(packed, n_bytes, scales, out, st)
                              : launch_fp4<false, false>(packed, n_bytes, scales, out, st);
}

extern "C" int ds_fp8_block_dequant(const uint8_t* packed, int64_t rows, int64_t cols,
                                    const uint8_t* scales, float* out, void* stream) {
  DS_REQUIRE(rows >= 0 && cols >= 0 && rows % 32 == 0 && cols % 32 == 0, DS_EINVAL,
             "fp8_block_dequant: rows and cols must be multiples of 32");
  if (rows * cols == 0) return DS_OK;
  DS_REQUIRE(packed && scales && out, DS_EINVAL, "fp8_block_dequant: null pointer");
  fp8_block_dequant_kernel<<<grid_for(rows * cols), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, rows, cols, scales, out);
  DS_CHECK_LAUNCH("fp8_block_dequant_kernel");
  return DS_OK;
}

extern "C" int ds_q3_dequant(const uint32_t* words, const uint16_t* scales, const uint16_t* biases,
                             int64_t rows, int64_t cols, void* out, int out_dtype, void* stream) {
  DS_REQUIRE(rows >= 0 && cols >= 0 && cols % 64 == 0, DS_EINVAL,
             "q3_dequant: cols must be a multiple of the group size 64");
  DS_REQUIRE(out_dtype == DS_F32 || out_dtype == DS_BF16, DS_EINVAL,
             "q3_dequant: out_dtype must be DS_F32 or DS_BF16");
  const int64_t n_groups = rows * (cols / 64);
  if (n_groups == 0) return DS_OK;
  DS_REQUIRE(words && scales && biases && out, DS_EINVAL, "q3_dequant: null pointer");
  DS_REQUIRE(ds::aligned(words, 4) && ds::aligned(scales, 2) && ds::aligned(biases, 2) &&
                 ds::aligned(out, 16),
             DS_EALIGN, "q3_dequant: words 4-byte, scales/biases 2-byte, out 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __half* s = reinterpret_cast<const __half*>(scales);
  const __half* b = reinterpret_cast<const __half*>(biases);
  if (out_dtype == DS_BF16)
    q3_dequant_kernel<true><<<grid_for(n_groups), kThreads, 0, st>>>(words, s, b, n_groups, out);
  else
    q3_dequant_kernel<false><<<grid_for(n_groups), kThreads, 0, st>>>(words, s, b, n_groups, out);
  DS_CHECK_LAUNCH("q3_dequant_kernel");
  return DS_OK;
}

extern "C" int ds_q3_quantize(const float* w, int64_t rows, int64_t cols, uint32_t* words,
                              uint16_t* scales, uint16_t* biases, void* stream) {
  DS_REQUIRE(rows >= 0 && cols >= 0 && cols % 64 == 0, DS_EINVAL,
             "q3_quantize: cols must be a multiple of the group size 64");
  const int64_t n_groups = rows * (cols / 64);
  if (n_groups == 0) return DS_OK;
  DS_REQUIRE(w && words && scales && biases, DS_EINVAL, "q3_quantize: null pointer");
  q3_quantize_kernel<<<grid_for(n_groups), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      w, n_groups, words, reinterpret_cast<__half*>(scales), reinterpret_cast<__half*>(biases));
  DS_CHECK_LAUNCH("q3_quantize_kernel");
  return DS_OK;
}

extern "C" int ds_fp4_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* packed,
                               uint8_t* scales, void* stream) {
  DS_REQUIRE(rows >= 0 && cols >= 0 && cols % 32 == 0, DS_EINVAL,
             "fp4_quantize: cols must be a multiple of the block size 32");
  const int64_t n_blocks = rows * (cols / 32);
  if (n_blocks == 0) return DS_OK;
  DS_REQUIRE(w && packed && scales, DS_EINVAL, "fp4_quantize: null pointer");
  DS_REQUIRE(ds::aligned(packed, 16), DS_EALIGN, "fp4_quantize: packed must be 16-byte aligned");
  fp4_quantize_kernel<<<grid_for(n_blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      w, n_blocks, packed, scales);
  DS_CHECK_LAUNCH("fp4_quantize_kernel");
  return DS_OK;
}
