// sgemm_smallm.cu -- fp32 SGEMM for small M (1..16 rows): the shape of Gemma's
// per-token products (the reference's small-M corpus, gemma4e2b_sgemm_corpus_test.go:44-59,
// m in {1, 2, 7, 15, 16} x 256 / 2048 x 1536).
//
// With so few rows the product is bound by reading B once from HBM (4*K*N
// bytes), not by arithmetic: a tensor-core or 128 x 128 FMA tile would spend
// nearly all its work on padding rows.  Each thread owns 4 adjacent columns and
// up to 4 rows (16 accumulators; larger m spreads its rows over CTAs that re-read
// the same B columns from L2), keeps 8 rows of its B columns in flight as
// 16-byte loads, and takes A from shared memory.  K is split over enough CTAs to fill
// the GPU; the last CTA to finish a column tile adds the split partials in
// split order, so the result does not depend on which CTA finishes first.
// Within a split the sum runs over k in increasing order, in fp32 (as Oct's
// cpuSGEMM, runtime.go:319-331).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kernels.h"

namespace oct {
namespace {

constexpr int SM_THREADS = 128;
constexpr int SM_MMAX = 16;  // largest m
constexpr int SM_COLS = SM_THREADS * 4;  // columns per CTA
constexpr int SM_KT = 64;                // k values of A staged per step
constexpr int SM_UNROLL = 8;             // rows of B in flight per thread

// MR = row capacity (m <= MR): fewer rows, fewer accumulators, more CTAs per SM.
template <int MR>
__global__ void __launch_bounds__(SM_THREADS) sgemm_smallm_kernel(
    const float* __restrict__ a, uint64_t lda, const float* __restrict__ b, uint64_t ldb, float* __restrict__ c,
    uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, uint32_t kchunk, float* __restrict__ partial,
    unsigned int* __restrict__ counters) {
  __shared__ __align__(16) float as[MR][SM_KT];
  __shared__ bool last_cta;
  const uint32_t col = blockIdx.x * SM_COLS + threadIdx.x * 4;
  const uint32_t split = blockIdx.y, splits = gridDim.y;
  // row group: this CTA owns rows [row0, row0 + MR) of C (B columns are re-read from L2 by the others)
  const uint32_t row0 = blockIdx.z * MR;
  a += static_cast<uint64_t>(row0) * lda;
  c += static_cast<uint64_t>(row0) * ldc;
  const uint32_t m_all = m;
  m = min(static_cast<uint32_t>(MR), m - row0);
  const uint32_t k0 = split * kchunk, k1 = min(k, k0 + kchunk);
  const bool vec = (ldb % 4 == 0) && ((reinterpret_cast<uintptr_t>(b) & 15u) == 0) && col + 4 <= n;
  float acc[MR][4];
#pragma unroll
  for (int i = 0; i < MR; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  auto load_b = [&](const float* q) -> float4 {
    if (vec) return __ldg(reinterpret_cast<const float4*>(q));
    float4 v;
    v.x = col < n ? __ldg(q) : 0.f;
    v.y = col + 1 < n ? __ldg(q + 1) : 0.f;
    v.z = col + 2 < n ? __ldg(q + 2) : 0.f;
    v.w = col + 3 < n ? __ldg(q + 3) : 0.f;
    return v;
  };
  for (uint32_t kt = k0; kt < k1; kt += SM_KT) {
    const uint32_t kn = min(static_cast<uint32_t>(SM_KT), k1 - kt);
    for (uint32_t i = threadIdx.x; i < MR * SM_KT; i += SM_THREADS) {
      const uint32_t r = i / SM_KT, kk = i % SM_KT;
      as[r][kk] = (r < m && kk < kn) ? a[static_cast<uint64_t>(r) * lda + kt + kk] : 0.f;
    }
    __syncthreads();
    if (col < n) {
      const float* bp = b + static_cast<uint64_t>(kt) * ldb + col;
      uint32_t kk = 0;
      for (; kk + SM_UNROLL <= kn; kk += SM_UNROLL) {
        float4 bv[SM_UNROLL];
#pragma unroll
        for (int u = 0; u < SM_UNROLL; ++u) bv[u] = load_b(bp + static_cast<uint64_t>(kk + u) * ldb);
#pragma unroll
        for (int u = 0; u < SM_UNROLL; ++u)
#pragma unroll
          for (int r = 0; r < MR; ++r) {
            const float av = as[r][kk + u];
            acc[r][0] = fmaf(av, bv[u].x, acc[r][0]);
            acc[r][1] = fmaf(av, bv[u].y, acc[r][1]);
            acc[r][2] = fmaf(av, bv[u].z, acc[r][2]);
            acc[r][3] = fmaf(av, bv[u].w, acc[r][3]);
          }
      }
      for (; kk < kn; ++kk) {
        const float4 bv = load_b(bp + static_cast<uint64_t>(kk) * ldb);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          const float av = as[r][kk];
          acc[r][0] = fmaf(av, bv.x, acc[r][0]);
          acc[r][1] = fmaf(av, bv.y, acc[r][1]);
          acc[r][2] = fmaf(av, bv.z, acc[r][2]);
          acc[r][3] = fmaf(av, bv.w, acc[r][3]);
        }
      }
    }
    __syncthreads();
  }

  // (row loops run over the compile-time capacity so the accumulators stay in registers)
  if (splits == 1) {
    if (col < n)
#pragma unroll
      for (uint32_t r = 0; r < MR; ++r)
        if (r < m)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (col + j < n) c[static_cast<uint64_t>(r) * ldc + col + j] = acc[r][j];
    return;
  }
  // partial[split][r][col], then the last CTA of this column tile reduces in split order
  if (col < n)
#pragma unroll
    for (uint32_t r = 0; r < MR; ++r)
      if (r < m)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < n) partial[(static_cast<uint64_t>(split) * m_all + row0 + r) * n + col + j] = acc[r][j];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(&counters[blockIdx.z * gridDim.x + blockIdx.x], 1u);
    last_cta = (prev == splits - 1);
  }
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  if (col < n)
    for (uint32_t r = 0; r < m; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (col + j >= n) continue;
        float s = 0.f;
        for (uint32_t sp = 0; sp < splits; ++sp)
          s += __ldcg(&partial[(static_cast<uint64_t>(sp) * m_all + row0 + r) * n + col + j]);
        c[static_cast<uint64_t>(r) * ldc + col + j] = s;
      }
  if (threadIdx.x == 0) counters[blockIdx.z * gridDim.x + blockIdx.x] = 0;  // ready for the next launch
}

// Enough CTAs to keep ~8 per SM streaming B, but the split partials (written
// and read once: 8 * splits * m * n bytes) stay near 10 % of B's 4 * k * n.
constexpr uint32_t SM_GROUP = 4;  // rows per CTA when m > 4
uint32_t smallm_groups(uint32_t m) { return m <= SM_GROUP ? 1u : (m + SM_GROUP - 1) / SM_GROUP; }

uint32_t smallm_splits(uint32_t m, uint32_t n, uint32_t k) {
  const uint32_t tiles = (n + SM_COLS - 1) / SM_COLS * smallm_groups(m);
  uint32_t splits = std::max<uint32_t>(1u, (8u * 148u + tiles - 1) / tiles);
  const uint32_t per_split = std::max<uint32_t>(SM_KT, 20u * m);
  splits = std::min<uint32_t>(splits, std::max<uint32_t>(1u, k / per_split));
  return std::min<uint32_t>(splits, 65535u);
}

}  // namespace

bool sgemm_smallm_supported(uint32_t m) { return m >= 1 && m <= static_cast<uint32_t>(SM_MMAX); }

uint64_t sgemm_smallm_scratch_bytes(uint32_t m, uint32_t n, uint32_t k) {
  const uint32_t tiles = (n + SM_COLS - 1) / SM_COLS * smallm_groups(m);
  const uint32_t splits = smallm_splits(m, n, k);
  if (splits == 1) return 0;
  return 1024 + ((static_cast<uint64_t>(tiles) * 4 + 255) & ~uint64_t(255)) +
         static_cast<uint64_t>(splits) * m * n * sizeof(float);
}

cudaError_t sgemm_smallm(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                         uint32_t m, uint32_t n, uint32_t k, void* scratch, cudaStream_t stream) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if (!sgemm_smallm_supported(m)) return cudaErrorInvalidValue;
  const uint32_t col_tiles = (n + SM_COLS - 1) / SM_COLS, groups = smallm_groups(m);
  const uint32_t tiles = col_tiles * groups;  // counters: one per (column tile, row group)
  const uint32_t splits = smallm_splits(m, n, k);
  const uint32_t kchunk = ((k + splits - 1) / splits + SM_KT - 1) / SM_KT * SM_KT;
  const uint32_t used = (k + kchunk - 1) / kchunk;  // splits that own at least one k
  unsigned int* counters = nullptr;
  float* partial = nullptr;
  if (used > 1) {
    if (scratch == nullptr) return cudaErrorInvalidValue;
    counters = static_cast<unsigned int*>(scratch);
    partial = reinterpret_cast<float*>(static_cast<char*>(scratch) +
                                       ((static_cast<uint64_t>(tiles) * 4 + 255) & ~uint64_t(255)));
    const cudaError_t e = cudaMemsetAsync(counters, 0, static_cast<size_t>(tiles) * 4, stream);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid(col_tiles, used, groups);
  if (m <= 1)
    sgemm_smallm_kernel<1><<<grid, SM_THREADS, 0, stream>>>(a, lda, b, ldb, c, ldc, m, n, k, kchunk, partial, counters);
  else if (m <= 2)
    sgemm_smallm_kernel<2><<<grid, SM_THREADS, 0, stream>>>(a, lda, b, ldb, c, ldc, m, n, k, kchunk, partial, counters);
  else
    sgemm_smallm_kernel<SM_GROUP><<<grid, SM_THREADS, 0, stream>>>(a, lda, b, ldb, c, ldc, m, n, k, kchunk, partial,
                                                                   counters);
  return cudaGetLastError();
}

}  // namespace oct
