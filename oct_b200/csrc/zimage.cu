// zimage.cu -- ingress kernels of the Z-Image model-block executors.
//
// The reference's executors take BF16 activations (nr0_bf16_ingress.sdslv:
// the sixteen BF16 bits become the high half of a binary32) and binary16
// weights in the cache layout [in][out] (nr0_fused_qkv.sdslv unpacks each
// half lane straight to f32).  Both widenings are exact; these kernels do
// them on the device, HBM-bound, so uploads move the 2-byte payloads only.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace oct {
namespace {

constexpr int kThreads = 256;

__global__ void widen_bf16_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, uint64_t n) {
  const uint64_t step = static_cast<uint64_t>(gridDim.x) * kThreads;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(kThreads) + threadIdx.x; i < n; i += step)
    dst[i] = __uint_as_float(static_cast<uint32_t>(src[i]) << 16);
}

// [rows][cols] binary16 -> dst[r * ld + col0 + c] fp32.
__global__ void widen_f16_kernel(const uint16_t* __restrict__ src, uint32_t rows, uint32_t cols,
                                 float* __restrict__ dst, uint64_t ld, uint32_t col0) {
  const uint64_t n = static_cast<uint64_t>(rows) * cols;
  const uint64_t step = static_cast<uint64_t>(gridDim.x) * kThreads;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(kThreads) + threadIdx.x; i < n; i += step) {
    const uint64_t r = i / cols, c = i - r * cols;
    dst[r * ld + col0 + c] = __half2float(__ushort_as_half(src[i]));
  }
}

uint32_t grid_for(uint64_t n) {
  const uint64_t b = (n + kThreads - 1) / kThreads;
  return static_cast<uint32_t>(b == 0 ? 1 : (b < 148ull * 16 ? b : 148ull * 16));
}

}  // namespace

cudaError_t widen_bf16(const void* src, float* dst, uint64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  widen_bf16_kernel<<<grid_for(n), kThreads, 0, stream>>>(static_cast<const uint16_t*>(src), dst, n);
  return cudaGetLastError();
}

cudaError_t widen_f16(const void* src, uint32_t rows, uint32_t cols, float* dst, uint64_t ld, uint32_t col0,
                      cudaStream_t stream) {
  const uint64_t n = static_cast<uint64_t>(rows) * cols;
  if (n == 0) return cudaSuccess;
  widen_f16_kernel<<<grid_for(n), kThreads, 0, stream>>>(static_cast<const uint16_t*>(src), rows, cols, dst, ld,
                                                         col0);
  return cudaGetLastError();
}

}  // namespace oct
