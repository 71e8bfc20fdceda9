// Input staging for a decode step: a kernel that copies a few KB (the step's
// query and new K / V rows) from page-locked host memory, read directly over
// the bus through its device mapping, into device memory.  For transfers this
// small the copy engine's fixed cost dominates (about 11 us on B200 for a
// 12 KB row); one thread block reading the host memory finishes in a few us.
#include "kernels.h"

namespace adakv {
namespace {

__global__ void __launch_bounds__(256) stage_kernel(const unsigned char* src, unsigned char* dst,
                                                    size_t bytes) {
  const size_t n16 = bytes / 16;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) d4[i] = s4[i];
  // the tail (bytes % 16) byte by byte
  const size_t t = n16 * 16 + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < bytes) dst[t] = src[t];
}

}  // namespace

cudaError_t launch_stage(const void* src, void* dst, size_t bytes, cudaStream_t st) {
  const size_t n16 = bytes / 16;
  const int blocks = (int)std::min<size_t>(std::max<size_t>((n16 + 255) / 256, 1), 148);
  stage_kernel<<<blocks, 256, 0, st>>>(static_cast<const unsigned char*>(src),
                                       static_cast<unsigned char*>(dst), bytes);
  return cudaGetLastError();
}

}  // namespace adakv
