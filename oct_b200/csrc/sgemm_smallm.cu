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
#include "ptx.cuh"

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

// ------------------------------------------------------------------ bulk-copy-fed variant
// When B's rows can be copied as whole 16-byte-granular segments (ldb and n
// multiples of 4, B 16-byte aligned), one thread streams the CTA's 512-column
// tile of B into a 6-stage shared-memory ring with cp.async.bulk (8 rows = 16 KB
// per stage, five stages in flight), so the loads run ahead of the FMAs, and all
// m <= 16 rows live in one CTA (no row groups re-reading B from L2).  The CTA's
// two halves (warps 0-3, 4-7) take rows 0-3 and 4-7 of each stage, each thread
// four columns; the halves' sums meet in shared memory at the end.  Warps never
// wait for one another inside the K loop: a slot's full barrier (the copies)
// and empty barrier (one arrival per warp) order it, and thread 0 refills a
// slot once all eight warps have released it.  A's rows
// for the CTA's K range are staged once in shared memory and read as float4
// (four k values per load).  Split-K with the same ordered reduction.
constexpr int BK_THREADS = 256;
constexpr int BK_SR = 8;           // B rows per stage (16 KB)
constexpr int BK_STAGES = 6;
constexpr uint32_t BK_KMAX = 256;  // k values per CTA (A staged in shared memory)

template <int MR>
__global__ void __launch_bounds__(BK_THREADS, 2) sgemm_smallm_bulk_kernel(
    const float* __restrict__ a, uint64_t lda, const float* __restrict__ b, uint64_t ldb, float* __restrict__ c,
    uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, uint32_t kchunk, float* __restrict__ partial,
    unsigned int* __restrict__ counters, unsigned int* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);  // [stage][BK_SR][SM_COLS]
  float* as = ring + BK_STAGES * BK_SR * SM_COLS;    // [MR][BK_KMAX]
  uint64_t* bars = reinterpret_cast<uint64_t*>(as + MR * BK_KMAX);  // full[BK_STAGES], empty[BK_STAGES]
  uint64_t* empty = bars + BK_STAGES;
  __shared__ bool last_cta;
  __shared__ int abort_flag;
  const uint32_t tid = threadIdx.x, half = tid / SM_THREADS, lane4 = tid % SM_THREADS;
  const uint32_t col0 = blockIdx.x * SM_COLS;
  const uint32_t cols = min(static_cast<uint32_t>(SM_COLS), n - col0);
  const uint32_t split = blockIdx.y, splits = gridDim.y;
  const uint32_t k0 = split * kchunk, k1 = min(k, k0 + kchunk);
  const uint32_t kn = k1 - k0;
  const uint32_t stages_total = (kn + BK_SR - 1) / BK_SR;
  const uint32_t col = col0 + lane4 * 4;
  if (tid == 0) {
    for (int s = 0; s < BK_STAGES; ++s) {
      mbar_init(&bars[s], 1);
      mbar_init(&empty[s], BK_THREADS / 32);
    }
    abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncthreads();
  auto issue = [&](uint32_t st) {  // stage st -> slot st % BK_STAGES (thread 0)
    const uint32_t slot = st % BK_STAGES;
    const uint32_t r0 = k0 + st * BK_SR, nr = min(static_cast<uint32_t>(BK_SR), k1 - r0);
    float* dst = ring + slot * BK_SR * SM_COLS;
    mbar_arrive_expect_tx(&bars[slot], nr * cols * 4u);
    for (uint32_t i = 0; i < nr; ++i)
      bulk_load(dst + i * SM_COLS, b + static_cast<uint64_t>(r0 + i) * ldb + col0, cols * 4u, &bars[slot]);
  };
  uint32_t issued = min(stages_total, static_cast<uint32_t>(BK_STAGES));  // thread 0's count
  if (tid == 0)
    for (uint32_t st = 0; st < issued; ++st) issue(st);
  // A rows of this CTA's K range -> shared memory (zero past m / kn), while the
  // first copies fly; all of a thread's loads are issued before the first store
  static_assert(BK_KMAX % BK_THREADS == 0, "A staging assumes whole rows per pass");
  {
    constexpr int kPer = MR * BK_KMAX / BK_THREADS;
    float v[kPer];
#pragma unroll
    for (int it = 0; it < kPer; ++it) {
      const uint32_t i = tid + it * BK_THREADS, r = i / BK_KMAX, kk = i % BK_KMAX;
      v[it] = (r < m && kk < kn) ? __ldg(&a[static_cast<uint64_t>(r) * lda + k0 + kk]) : 0.f;
    }
#pragma unroll
    for (int it = 0; it < kPer; ++it) as[tid + it * BK_THREADS] = v[it];
  }
  __syncthreads();
  float acc[MR][4];
#pragma unroll
  for (int i = 0; i < MR; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  bool ok = true;
  for (uint32_t st = 0; st < stages_total; ++st) {
    const uint32_t slot = st % BK_STAGES;
    ok = __all_sync(0xffffffffu, ok && mbar_wait(&bars[slot], (st / BK_STAGES) & 1u, err, kErrWaitRow));
    if (!ok || *reinterpret_cast<volatile int*>(&abort_flag) != 0) {
      ok = false;
      *reinterpret_cast<volatile int*>(&abort_flag) = 1;
      break;
    }
    const uint32_t nr = min(static_cast<uint32_t>(BK_SR), kn - st * BK_SR);
    const uint32_t rb = 4 * half, re = min(nr, rb + 4);  // this half's rows of the stage
    if (col < col0 + cols && rb < re) {
      const float* src = ring + slot * BK_SR * SM_COLS + lane4 * 4;
      if (re - rb == 4) {
        float4 bv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) bv[q] = *reinterpret_cast<const float4*>(src + (rb + q) * SM_COLS);
        const uint32_t kk = st * BK_SR + rb;  // a multiple of 4
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          const float4 av = *reinterpret_cast<const float4*>(&as[r * BK_KMAX + kk]);
          const float a4[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[r][0] = fmaf(a4[q], bv[q].x, acc[r][0]);
            acc[r][1] = fmaf(a4[q], bv[q].y, acc[r][1]);
            acc[r][2] = fmaf(a4[q], bv[q].z, acc[r][2]);
            acc[r][3] = fmaf(a4[q], bv[q].w, acc[r][3]);
          }
        }
      } else {
        for (uint32_t rr = rb; rr < re; ++rr) {  // ragged end of the K range: rows past nr hold stale data
          const float4 bv = *reinterpret_cast<const float4*>(src + rr * SM_COLS);
          const uint32_t kk = st * BK_SR + rr;
#pragma unroll
          for (int r = 0; r < MR; ++r) {
            const float av = as[r * BK_KMAX + kk];
            acc[r][0] = fmaf(av, bv.x, acc[r][0]);
            acc[r][1] = fmaf(av, bv.y, acc[r][1]);
            acc[r][2] = fmaf(av, bv.z, acc[r][2]);
            acc[r][3] = fmaf(av, bv.w, acc[r][3]);
          }
        }
      }
    }
    __syncwarp();
    if ((tid & 31u) == 0) mbar_arrive(&empty[slot]);  // this warp is done with the slot
    if (tid == 0 && st + BK_STAGES < stages_total) {
      // refill once every warp has released the slot (bounded wait)
      if (mbar_wait(&empty[slot], (st / BK_STAGES) & 1u, err, kErrWaitEmpty)) {
        fence_proxy_async_smem();
        issue(st + BK_STAGES);
        issued = st + BK_STAGES + 1;
      } else {
        ok = false;
      }
    }
  }
  if (!__syncthreads_and(ok)) {
    // drain: stages [0, issued) were issued; a slot's phases complete in
    // order, so waiting (bounded) for its newest copy is enough
    if (tid == 0) {
      for (uint32_t s = 0; s < static_cast<uint32_t>(BK_STAGES) && s < issued; ++s) {
        const uint32_t count = (issued - s + BK_STAGES - 1) / BK_STAGES;
        if (!mbar_wait(&bars[s], (count - 1) & 1u, err, kErrWaitDrain)) break;
      }
    }
    return;
  }
  // the halves meet: half 1's sums through the (now idle) ring, added by half 0
  float* meet = ring;  // [MR * 4][SM_THREADS]
  if (half == 1)
#pragma unroll
    for (int r = 0; r < MR; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) meet[(r * 4 + j) * SM_THREADS + lane4] = acc[r][j];
  __syncthreads();
  if (half == 0) {
#pragma unroll
    for (int r = 0; r < MR; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][j] += meet[(r * 4 + j) * SM_THREADS + lane4];
    if (col < n)  // n is a multiple of 4 here: col..col+3 are all in range
#pragma unroll
      for (uint32_t r = 0; r < MR; ++r)
        if (r < m) {
          if (splits == 1) {
#pragma unroll
            for (int j = 0; j < 4; ++j) c[static_cast<uint64_t>(r) * ldc + col + j] = acc[r][j];
          } else {
            *reinterpret_cast<float4*>(&partial[(static_cast<uint64_t>(split) * m + r) * n + col]) =
                make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
          }
        }
  }
  if (splits == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&counters[blockIdx.x], 1u);
    last_cta = (prev == splits - 1);
  }
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  // the last CTA of the tile sums the splits in split order, one (row, column
  // quad) per thread at a time, eight float4 partials in flight
  const uint64_t sstride = static_cast<uint64_t>(m) * n / 4;  // float4s between splits
  for (uint32_t u = tid; u < m * static_cast<uint32_t>(SM_THREADS); u += BK_THREADS) {
    const uint32_t r = u / SM_THREADS, cq = col0 + (u % SM_THREADS) * 4;
    if (cq >= n) continue;
    const float4* p = reinterpret_cast<const float4*>(&partial[static_cast<uint64_t>(r) * n + cq]);
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t sp = 0;
    for (; sp + 8 <= splits; sp += 8) {
      float4 v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = __ldcg(p + (sp + q) * sstride);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        sum.x += v[q].x;
        sum.y += v[q].y;
        sum.z += v[q].z;
        sum.w += v[q].w;
      }
    }
    for (; sp < splits; ++sp) {
      const float4 v = __ldcg(p + sp * sstride);
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
    }
    float* dst = c + static_cast<uint64_t>(r) * ldc + cq;
    dst[0] = sum.x;
    dst[1] = sum.y;
    dst[2] = sum.z;
    dst[3] = sum.w;
  }
  if (tid == 0) counters[blockIdx.x] = 0;
}

bool smallm_bulk_ok(const float* b, uint64_t ldb, uint32_t n) {
  return ldb % 4 == 0 && n % 4 == 0 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0;
}

template <int MR>
constexpr uint32_t smallm_bulk_smem() {
  return (BK_STAGES * BK_SR * SM_COLS + MR * BK_KMAX) * 4u + 2u * BK_STAGES * 8u;
}

// resident CTAs per SM by shared memory (228 KB per SM, 1 KB reserved per CTA)
constexpr uint32_t smallm_bulk_per_sm(uint32_t m) {
  const uint32_t mr = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : m <= 8 ? 8 : 16;
  const uint32_t smem = (BK_STAGES * BK_SR * SM_COLS + mr * BK_KMAX) * 4u + 2u * BK_STAGES * 8u + 1024u;
  return 233472u / smem;
}

// splits for the bulk variant: each CTA covers <= BK_KMAX k values; otherwise as
// many as fill one wave of resident CTAs (148 SMs), so no tail wave runs
// half-empty; a split keeps >= 20 m k values where k allows, which holds the
// partials' traffic near a tenth of B's
uint32_t smallm_bulk_splits(uint32_t m, uint32_t n, uint32_t k) {
  const uint32_t tiles = (n + SM_COLS - 1) / SM_COLS;
  const uint32_t floor_splits = (k + BK_KMAX - 1) / BK_KMAX;
  uint32_t splits = std::max<uint32_t>(floor_splits, 148u * smallm_bulk_per_sm(m) / tiles);
  splits = std::min<uint32_t>(splits, std::max<uint32_t>(floor_splits, k / std::max(16u, 20u * m)));
  return std::min<uint32_t>(std::max<uint32_t>(splits, 1u), 65535u);
}

}  // namespace

bool sgemm_smallm_supported(uint32_t m) { return m >= 1 && m <= static_cast<uint32_t>(SM_MMAX); }

uint64_t sgemm_smallm_scratch_bytes(uint32_t m, uint32_t n, uint32_t k) {
  // enough for either variant (the choice between them depends on pointers)
  const uint32_t tiles = (n + SM_COLS - 1) / SM_COLS * smallm_groups(m);
  const uint32_t splits = std::max(smallm_splits(m, n, k), smallm_bulk_splits(m, n, k));
  if (splits == 1) return 0;
  return 1024 + ((static_cast<uint64_t>(tiles) * 4 + 255) & ~uint64_t(255)) +
         static_cast<uint64_t>(splits) * m * n * sizeof(float);
}

namespace {
template <int MR>
cudaError_t launch_bulk(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc, uint32_t m,
                        uint32_t n, uint32_t k, void* scratch, unsigned int* err, cudaStream_t stream) {
  const uint32_t tiles = (n + SM_COLS - 1) / SM_COLS;
  const uint32_t splits = smallm_bulk_splits(m, n, k);
  const uint32_t kchunk = std::min<uint32_t>(BK_KMAX, ((k + splits - 1) / splits + 3) / 4 * 4);
  const uint32_t used = (k + kchunk - 1) / kchunk;
  unsigned int* counters = nullptr;
  float* partial = nullptr;
  if (used > 1) {
    if (scratch == nullptr) return cudaErrorInvalidValue;
    counters = static_cast<unsigned int*>(scratch);
    partial = reinterpret_cast<float*>(static_cast<char*>(scratch) +
                                       ((static_cast<uint64_t>(tiles) * smallm_groups(m) * 4 + 255) & ~uint64_t(255)));
    const cudaError_t e = cudaMemsetAsync(counters, 0, static_cast<size_t>(tiles) * 4, stream);
    if (e != cudaSuccess) return e;
  }
  constexpr uint32_t smem = smallm_bulk_smem<MR>();
  cudaError_t e = cudaFuncSetAttribute(sgemm_smallm_bulk_kernel<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  sgemm_smallm_bulk_kernel<MR><<<dim3(tiles, used), BK_THREADS, smem, stream>>>(a, lda, b, ldb, c, ldc, m, n, k,
                                                                               kchunk, partial, counters, err);
  return cudaGetLastError();
}
}  // namespace

cudaError_t sgemm_smallm(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                         uint32_t m, uint32_t n, uint32_t k, void* scratch, cudaStream_t stream, unsigned int* err) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if (!sgemm_smallm_supported(m)) return cudaErrorInvalidValue;
  if (err != nullptr && smallm_bulk_ok(b, ldb, n)) {
    if (m <= 1) return launch_bulk<1>(a, lda, b, ldb, c, ldc, m, n, k, scratch, err, stream);
    if (m <= 2) return launch_bulk<2>(a, lda, b, ldb, c, ldc, m, n, k, scratch, err, stream);
    if (m <= 4) return launch_bulk<4>(a, lda, b, ldb, c, ldc, m, n, k, scratch, err, stream);
    if (m <= 8) return launch_bulk<8>(a, lda, b, ldb, c, ldc, m, n, k, scratch, err, stream);
    return launch_bulk<16>(a, lda, b, ldb, c, ldc, m, n, k, scratch, err, stream);
  }
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
