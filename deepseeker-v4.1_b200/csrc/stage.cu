// Staging of a decode step's inputs and outputs between pinned host memory
// and the device by a kernel instead of the copy engines.
//
// A host-fed decode step moves a few kilobytes each way (x and the router
// logits in, the output rows out).  Issued as copy-engine transfers, every
// such copy costs several microseconds of its own on the step's critical
// path; here one launch copies up to four byte ranges with 16-byte loads and
// stores, reading or writing pinned host memory through its device mapping
// (the address cudaHostGetDevicePointer returns), so the transfer is a few
// PCIe round trips inside one short kernel.
#include <cuda_runtime.h>

#include "deepseeker_b200.h"
#include "ds_common.cuh"

namespace {

constexpr int kMaxRanges = 4;
constexpr int kCopyThreads = 256;

struct Ranges {
  uint4* dst[kMaxRanges];
  const uint4* src[kMaxRanges];
  int64_t words[kMaxRanges];  // 16-byte words per range
};

// blockIdx.y = range; a grid-stride loop over its words.
__global__ void __launch_bounds__(kCopyThreads) copy_ranges_kernel(const __grid_constant__ Ranges r) {
  const int k = blockIdx.y;
  const int64_t n = r.words[k];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    r.dst[k][i] = r.src[k][i];
}

}  // namespace

extern "C" int ds_host_device_pointer(const void* host, void** device) {
  DS_REQUIRE(host != nullptr && device != nullptr, DS_EINVAL, "host_device_pointer: null pointer");
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();   // leave no sticky error behind for the caller
    return ds::set_error(DS_EINVAL, "host_device_pointer: not pinned, mapped host memory (%s)", cudaGetErrorString(e));
  }
  *device = d;
  return DS_OK;
}

extern "C" int ds_copy_ranges(int n, void* const* dst, const void* const* src, const size_t* bytes, void* stream) {
  DS_REQUIRE(n >= 1 && n <= kMaxRanges, DS_EINVAL, "copy_ranges: 1..%d ranges, got %d", kMaxRanges, n);
  DS_REQUIRE(dst && src && bytes, DS_EINVAL, "copy_ranges: null array");
  Ranges r = {};
  int64_t most = 0;
  for (int k = 0; k < n; ++k) {
    DS_REQUIRE(dst[k] && src[k], DS_EINVAL, "copy_ranges: null pointer in range %d", k);
    DS_REQUIRE(ds::aligned(dst[k], 16) && ds::aligned(src[k], 16) && bytes[k] % 16 == 0, DS_EALIGN,
               "copy_ranges: range %d needs 16-byte aligned pointers and a multiple of 16 bytes", k);
    r.dst[k] = static_cast<uint4*>(dst[k]);
    r.src[k] = static_cast<const uint4*>(src[k]);
    r.words[k] = (int64_t)(bytes[k] / 16);
    most = r.words[k] > most ? r.words[k] : most;
  }
  if (most == 0) return DS_OK;
  const int64_t blocks = (most + kCopyThreads - 1) / kCopyThreads;
  const dim3 grid((unsigned)(blocks < 148 ? blocks : 148), (unsigned)n);
  copy_ranges_kernel<<<grid, kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(r);
  DS_CHECK_LAUNCH("copy_ranges_kernel");
  return DS_OK;
}
