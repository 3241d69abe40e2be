// sgemm_fma.cu -- the FP32-FMA control SGEMM on the CUDA cores.
//
// Same contract as the tensor-core kernel: C[m x n] = A[m x k] * B[k x n],
// row-major fp32 with leading dimensions, C overwritten.  Each output is one
// fp32 fused-multiply-add chain over k in ascending order -- the order of Oct's
// CPU oracle `cpuSGEMM` (internal/prometheus/runtime.go:319-331) -- so it is
// the plain-fp32 control the 3xTF32 path is compared with.
//
// Tiling: 128x128 output tile per 256-thread CTA, 8x8 outputs per thread held
// in registers, K staged 8 deep through double-buffered shared memory with a
// register prefetch of the next slab.  Loads of A and B are 128-bit when the
// row stride and base allow it and fall back to predicated scalar loads on the
// ragged edges (zero fill), which is the exact-tail behaviour of the
// reference's `SgemmReg2x2Tile16x16ExactTailFp32` shader
// (shaders/sdslv/production/sgemm/sgemm_reg2x2_tile16x16_exacttail_fp32.sdslv:137-185).
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace oct {
namespace {

constexpr int TM = 128, TN = 128, TK = 8, PAD = 4;

__device__ __forceinline__ void load4(const float* __restrict__ base, uint64_t ld, uint32_t row, uint32_t col,
                                      uint32_t rows, uint32_t cols, bool vec_ok, float (&v)[4]) {
  v[0] = v[1] = v[2] = v[3] = 0.f;
  if (row >= rows) return;
  const float* p = base + row * ld + col;
  if (vec_ok && col + 4 <= cols) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col + j < cols) v[j] = __ldg(p + j);
  }
}

// B_TRANS: B is given as [n][k] row-major and the product is A * B^T.
// blockIdx.z selects the batch entry (element strides stride_a/b/c).
template <bool B_TRANS>
__global__ void __launch_bounds__(256) sgemm_fma_kernel(const float* __restrict__ a, uint64_t lda,
                                                        const float* __restrict__ b, uint64_t ldb,
                                                        float* __restrict__ c, uint64_t ldc, uint32_t m,
                                                        uint32_t n, uint32_t k, uint64_t stride_a,
                                                        uint64_t stride_b, uint64_t stride_c) {
  __shared__ __align__(16) float As[2][TK][TM + PAD];  // A slab, transposed: [k][m]
  __shared__ __align__(16) float Bs[2][TK][TN + PAD];  // B slab: [k][n]
  a += blockIdx.z * stride_a;
  b += blockIdx.z * stride_b;
  c += blockIdx.z * stride_c;

  const uint32_t tid = threadIdx.x;
  const uint32_t tx = tid & 15, ty = tid >> 4;
  const uint32_t m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const bool a_vec = (lda % 4 == 0) && ((reinterpret_cast<uintptr_t>(a) & 15u) == 0);
  const bool b_vec = (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(b) & 15u) == 0);

  // Loader coordinates: A (and B^T) -> row t/2, k offset (t%2)*4; B -> k row t/32, col (t%32)*4.
  const uint32_t a_row = tid >> 1, a_k = (tid & 1) * 4;
  const uint32_t b_k = tid >> 5, b_col = (tid & 31) * 4;
  auto load_b = [&](uint32_t k0, float (&v)[4]) {
    if constexpr (B_TRANS) load4(b, ldb, n0 + a_row, k0 + a_k, n, k, b_vec, v);
    else load4(b, ldb, k0 + b_k, n0 + b_col, k, n, b_vec, v);
  };
  auto store_b = [&](uint32_t buf, const float (&v)[4]) {
    if constexpr (B_TRANS) {
#pragma unroll
      for (int j = 0; j < 4; ++j) Bs[buf][a_k + j][a_row] = v[j];
    } else {
      *reinterpret_cast<float4*>(&Bs[buf][b_k][b_col]) = make_float4(v[0], v[1], v[2], v[3]);
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float ra[4], rb[4];
  const uint32_t num_kt = (k + TK - 1) / TK;
  load4(a, lda, m0 + a_row, a_k, m, k, a_vec, ra);
  load_b(0, rb);
#pragma unroll
  for (int j = 0; j < 4; ++j) As[0][a_k + j][a_row] = ra[j];
  store_b(0, rb);
  __syncthreads();

  for (uint32_t kt = 0; kt < num_kt; ++kt) {
    const uint32_t cur = kt & 1;
    const bool more = kt + 1 < num_kt;
    if (more) {
      const uint32_t k1 = (kt + 1) * TK;
      load4(a, lda, m0 + a_row, k1 + a_k, m, k, a_vec, ra);
      load_b(k1, rb);
    }
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      const uint32_t nxt = cur ^ 1u;
#pragma unroll
      for (int j = 0; j < 4; ++j) As[nxt][a_k + j][a_row] = ra[j];
      store_b(nxt, rb);
    }
    __syncthreads();
  }

  const bool c_vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= m) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = n0 + h * 64 + tx * 4;
      float* dst = c + row * ldc + col;
      if (c_vec && col + 4 <= n) {
        *reinterpret_cast<float4*>(dst) =
            make_float4(acc[i][h * 4], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < n) dst[j] = acc[i][h * 4 + j];
      }
    }
  }
}

}  // namespace

cudaError_t sgemm_fma(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                      uint32_t m, uint32_t n, uint32_t k, cudaStream_t stream, const GemmBatch* batch) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  const GemmBatch one{};
  const GemmBatch& bt = batch != nullptr ? *batch : one;
  if (bt.count == 0) return cudaSuccess;
  const dim3 grid((n + TN - 1) / TN, (m + TM - 1) / TM, bt.count);
  if (grid.y > 65535u || grid.z > 65535u) return cudaErrorInvalidValue;
  if (bt.b_trans)
    sgemm_fma_kernel<true><<<grid, 256, 0, stream>>>(a, lda, b, ldb, c, ldc, m, n, k, bt.stride_a, bt.stride_b,
                                                     bt.stride_c);
  else
    sgemm_fma_kernel<false><<<grid, 256, 0, stream>>>(a, lda, b, ldb, c, ldc, m, n, k, bt.stride_a, bt.stride_b,
                                                      bt.stride_c);
  return cudaGetLastError();
}

}  // namespace oct
