// gemma_m1.cu -- the Gemma-4 E2B "M1" boundary operations with BF16 storage rounding.
//
// These are the model-private entry points Oct's Go validation lane binds
// (internal/prometheus/bridge.go:466-515; reactor_api.h:2686-2712):
//
//   projection-activation RMSNorm  fp32 in, output rounded to BF16
//                                   (reactor_api.c:362-368: bf16_roundtrip_output = 1)
//   head RMSNorm                    input and output rounded to BF16 (reactor_api.c:370-395)
//   half-split RoPE                 BF16 product, BF16 sum / difference, half pairing
//                                   (cpuGemma4e2bRope, gemma4e2b_m1_rtx.go:834-861)
//   head RMSNorm -> RoPE            the two above fused, nothing read back in between
//                                   (reactor_api.c:404-505)
//   raw attention scores            q . k * scale, MQA (every query head reads KV head 0),
//                                   no mask, no softmax (cpuGemma4e2bRawScores,
//                                   gemma4e2b_m1_rtx.go:863-883)
//
// Arithmetic follows the reference's own known-answer oracles
// (Marionette/reactor_concept_rmsnorm_tests.cpp:12-70): BF16 rounding is
// round-to-nearest-even on the fp32 bit pattern (float32ToBF16,
// gemma4e2b_m1_rtx.go:1009-1014); the RMSNorm sum of squares is accumulated in
// binary64 and inv = float(1 / sqrt(sum / width + eps)); the normalised value
// is (x * inv) * weight in fp32; score dot products are accumulated in
// binary64 and rounded once.  All inputs reach these kernels already checked
// finite by the host, as the reference checks them.
//
// These are small, HBM-bound element / row operations: one warp per row
// (RMSNorm), one thread per element (RoPE), shared-memory tiles of Q and K
// (scores).  No tensor cores: the score chain's reference arithmetic is a
// binary64 dot product of BF16-exact values.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace oct {
namespace {

constexpr int kThreads = 256;

// Round-to-nearest-even to BF16, returned re-expanded to fp32 (finite inputs).
__device__ __forceinline__ float bf16_round(float v) {
  uint32_t b = __float_as_uint(v);
  b += 0x7fffu + ((b >> 16) & 1u);
  return __uint_as_float(b & 0xffff0000u);
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row: y = round_out((round_in(x) * inv) * w), inv written per row.
template <bool ROUND_IN, bool ROUND_OUT>
__global__ void __launch_bounds__(kThreads) m1_rmsnorm_kernel(const float* __restrict__ in, uint64_t stride,
                                                              const float* __restrict__ w, float* __restrict__ out,
                                                              float* __restrict__ inv_out, uint32_t rows,
                                                              uint32_t width, float eps) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (kThreads / 32);
  for (uint64_t r = blockIdx.x * (kThreads / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const float* x = in + r * stride;
    double ss = 0.0;
    for (uint32_t c = lane; c < width; c += 32) {
      const float v = ROUND_IN ? bf16_round(x[c]) : x[c];
      ss += static_cast<double>(v) * static_cast<double>(v);  // exact square in binary64
    }
    ss = warp_sum(ss);
    const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(width) + static_cast<double>(eps)));
    if (lane == 0 && inv_out != nullptr) inv_out[r] = inv;
    float* y = out + r * width;
    for (uint32_t c = lane; c < width; c += 32) {
      const float v = ROUND_IN ? bf16_round(x[c]) : x[c];
      const float t = __fmul_rn(__fmul_rn(v, inv), __ldg(w + c));
      y[c] = ROUND_OUT ? bf16_round(t) : t;
    }
  }
}

// Half-split RoPE of one element from its row `src` (head_width values):
// bf16(bf16(x[c] cos[f]) -/+ bf16(x[mate] sin[f])), f = c mod (hw / 2).
__device__ __forceinline__ float rope_one(const float* src, const float* cos_row, const float* sin_row, uint32_t c,
                                          uint32_t half) {
  const uint32_t f = c < half ? c : c - half;
  const uint32_t mate = c < half ? c + half : c - half;
  const float first = bf16_round(__fmul_rn(src[c], __ldg(cos_row + f)));
  const float second = bf16_round(__fmul_rn(src[mate], __ldg(sin_row + f)));
  return bf16_round(c < half ? __fsub_rn(first, second) : __fadd_rn(first, second));
}

// One thread per output element of [tokens][heads][hw]; tables are [tokens][hw].
__global__ void __launch_bounds__(kThreads) m1_rope_kernel(const float* __restrict__ src, const float* __restrict__ cs,
                                                           const float* __restrict__ sn, float* __restrict__ out,
                                                           uint32_t heads, uint32_t hw, uint64_t total) {
  const uint64_t step = static_cast<uint64_t>(gridDim.x) * kThreads;
  const uint32_t half = hw / 2;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(kThreads) + threadIdx.x; i < total; i += step) {
    const uint64_t row = i / hw;  // (token, head)
    const uint32_t c = static_cast<uint32_t>(i - row * hw);
    const uint64_t token = row / heads;
    out[i] = rope_one(src + row * hw, cs + token * hw, sn + token * hw, c, half);
  }
}

// One warp per (token, head) row: BF16 head RMSNorm into shared memory, then RoPE
// from it.  Shared memory: hw floats per warp.
__global__ void __launch_bounds__(kThreads) m1_head_rmsnorm_rope_kernel(
    const float* __restrict__ in, const float* __restrict__ w, const float* __restrict__ cs,
    const float* __restrict__ sn, float* __restrict__ out, uint32_t rows, uint32_t heads, uint32_t hw, float eps) {
  extern __shared__ float smem[];
  const uint32_t lane = threadIdx.x & 31u;
  float* y = smem + (threadIdx.x / 32) * hw;
  const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (kThreads / 32);
  const uint32_t half = hw / 2;
  for (uint64_t r = blockIdx.x * (kThreads / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const float* x = in + r * hw;
    double ss = 0.0;
    for (uint32_t c = lane; c < hw; c += 32) {
      const float v = bf16_round(x[c]);
      ss += static_cast<double>(v) * static_cast<double>(v);
    }
    ss = warp_sum(ss);
    const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(hw) + static_cast<double>(eps)));
    for (uint32_t c = lane; c < hw; c += 32)
      y[c] = bf16_round(__fmul_rn(__fmul_rn(bf16_round(x[c]), inv), __ldg(w + c)));
    __syncwarp();
    const uint64_t token = r / heads;
    for (uint32_t c = lane; c < hw; c += 32) out[r * hw + c] = rope_one(y, cs + token * hw, sn + token * hw, c, half);
    __syncwarp();  // y is rewritten by this warp's next row
  }
}

// scores[h][i][j] = float(sum_d double(q[i][h][d]) * double(k[j][d]) * scale).
// One CTA per (16 query rows, 16 keys, head); each thread one (i, j) pair.
constexpr int kScoreTile = 16;
__global__ void __launch_bounds__(kScoreTile* kScoreTile) m1_scores_kernel(const float* __restrict__ q,
                                                                            const float* __restrict__ k,
                                                                            float* __restrict__ scores,
                                                                            uint32_t tokens, uint32_t qheads,
                                                                            uint32_t hw, double scale) {
  extern __shared__ float tile[];  // [16][hw] queries then [16][hw] keys
  float* qs = tile;
  float* ks = tile + kScoreTile * hw;
  const uint32_t h = blockIdx.z;
  const uint32_t i0 = blockIdx.y * kScoreTile, j0 = blockIdx.x * kScoreTile;
  const uint32_t tid = threadIdx.y * kScoreTile + threadIdx.x;
  for (uint32_t e = tid; e < kScoreTile * hw; e += kScoreTile * kScoreTile) {
    const uint32_t r = e / hw, d = e - r * hw;
    qs[e] = (i0 + r < tokens) ? q[(static_cast<uint64_t>(i0 + r) * qheads + h) * hw + d] : 0.f;
    ks[e] = (j0 + r < tokens) ? k[static_cast<uint64_t>(j0 + r) * hw + d] : 0.f;
  }
  __syncthreads();
  const uint32_t i = i0 + threadIdx.y, j = j0 + threadIdx.x;
  if (i >= tokens || j >= tokens) return;
  const float* qr = qs + threadIdx.y * hw;
  const float* kr = ks + threadIdx.x * hw;
  double acc = 0.0;
  for (uint32_t d = 0; d < hw; ++d) acc = fma(static_cast<double>(qr[d]), static_cast<double>(kr[d]), acc);
  scores[(static_cast<uint64_t>(h) * tokens + i) * tokens + j] = static_cast<float>(acc * scale);
}

uint32_t grid_for(uint64_t work, uint64_t per_block) {
  const uint64_t b = (work + per_block - 1) / per_block;
  const uint64_t cap = 148ull * 16;
  return static_cast<uint32_t>(b < cap ? (b == 0 ? 1 : b) : cap);
}

}  // namespace

cudaError_t m1_rmsnorm_bf16(const float* in, uint64_t stride, const float* w, float* out, float* inv_rms,
                            uint32_t rows, uint32_t width, float eps, bool round_in, bool round_out,
                            cudaStream_t stream) {
  if (rows == 0 || width == 0) return cudaSuccess;
  const uint32_t grid = grid_for(rows, kThreads / 32);
  if (round_in && round_out)
    m1_rmsnorm_kernel<true, true><<<grid, kThreads, 0, stream>>>(in, stride, w, out, inv_rms, rows, width, eps);
  else if (round_out)
    m1_rmsnorm_kernel<false, true><<<grid, kThreads, 0, stream>>>(in, stride, w, out, inv_rms, rows, width, eps);
  else if (round_in)
    m1_rmsnorm_kernel<true, false><<<grid, kThreads, 0, stream>>>(in, stride, w, out, inv_rms, rows, width, eps);
  else
    m1_rmsnorm_kernel<false, false><<<grid, kThreads, 0, stream>>>(in, stride, w, out, inv_rms, rows, width, eps);
  return cudaGetLastError();
}

cudaError_t m1_rope_bf16(const float* src, const float* cos_table, const float* sin_table, float* out,
                         uint32_t tokens, uint32_t heads, uint32_t head_width, cudaStream_t stream) {
  const uint64_t total = static_cast<uint64_t>(tokens) * heads * head_width;
  if (total == 0) return cudaSuccess;
  if (head_width % 2) return cudaErrorInvalidValue;
  m1_rope_kernel<<<grid_for(total, kThreads), kThreads, 0, stream>>>(src, cos_table, sin_table, out, heads,
                                                                     head_width, total);
  return cudaGetLastError();
}

cudaError_t m1_head_rmsnorm_rope(const float* in, const float* w, const float* cos_table, const float* sin_table,
                                 float* out, uint32_t tokens, uint32_t heads, uint32_t head_width, float eps,
                                 cudaStream_t stream) {
  const uint64_t rows = static_cast<uint64_t>(tokens) * heads;
  if (rows == 0) return cudaSuccess;
  if (head_width % 2 || head_width > kM1MaxHeadWidth || rows > 0xFFFFFFFFull) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(kThreads / 32) * head_width * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(m1_head_rmsnorm_rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  m1_head_rmsnorm_rope_kernel<<<grid_for(rows, kThreads / 32), kThreads, smem, stream>>>(
      in, w, cos_table, sin_table, out, static_cast<uint32_t>(rows), heads, head_width, eps);
  return cudaGetLastError();
}

cudaError_t m1_raw_scores(const float* q, const float* k, float* scores, uint32_t tokens, uint32_t query_heads,
                          uint32_t head_width, float scale, cudaStream_t stream) {
  if (tokens == 0 || query_heads == 0) return cudaSuccess;
  if (head_width == 0 || head_width > kM1MaxHeadWidth || query_heads > 65535u) return cudaErrorInvalidValue;
  const size_t smem = 2ull * kScoreTile * head_width * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(m1_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  const uint32_t tiles = (tokens + kScoreTile - 1) / kScoreTile;
  m1_scores_kernel<<<dim3(tiles, tiles, query_heads), dim3(kScoreTile, kScoreTile), smem, stream>>>(
      q, k, scores, tokens, query_heads, head_width, static_cast<double>(scale));
  return cudaGetLastError();
}

}  // namespace oct
