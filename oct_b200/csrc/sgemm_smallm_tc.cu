// sgemm_smallm_tc.cu -- fp32 SGEMM for small M (1..16 rows) on the tcgen05 tensor
// cores, 3xTF32, with the TF32 split done inside the kernel: the shape of Gemma's
// per-token products (the reference's small-M corpus, gemma4e2b_sgemm_corpus_test.go:44-59).
//
// The product is bound by reading B once from HBM.  The CUDA-core kernel
// (sgemm_smallm.cu) spends most of the FP32 pipe on it at m = 16; here the
// multiply-adds go to the tensor core and the SMs only convert B:
//   * the roles are swapped, C^T = B^T A^T: the MMA's M side (128 lanes of TMEM)
//     runs over 128 columns of B and C, its N side (16) over the rows of A and C,
//     so M is padded only in the MMA's N = 16, never in shared memory;
//   * per stage each CTA's TMA reads a raw [32 k][128 n] box of B (N-major, as B
//     lies in memory) and a raw [16 m][32 k] box of A (K-major, swizzled as the
//     MMA reads it) straight from the caller's arrays, zero-filling past m, n, k;
//   * two converter warps per stage slot transpose B into K-major hi / lo tiles
//     (round to nearest tf32, then the remainder, as the split pass does) and
//     split A in place; every element of B is converted exactly once;
//   * one thread issues 3 tcgen05.mma (M = 128, N = 16, K = 8) per 8-deep k step
//     into one of two 16-column TMEM accumulators, restarting every 64 of K; the
//     four epilogue warps add each chunk into fp32 running sums (round to nearest);
//   * K is split over CTAs so the grid fills the GPU; each split writes its
//     partial C into scratch and a second kernel adds the partials in split
//     order, so the result does not depend on timing.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace oct {
namespace {

constexpr uint32_t ST_BK = 32;                       // k per stage (128-byte K-major rows)
constexpr uint32_t ST_NT = 128;                      // columns of B / C per CTA (MMA M)
constexpr uint32_t ST_MN = 16;                       // rows of A / C (MMA N)
constexpr uint32_t ST_S = 4;                         // stages
constexpr uint32_t ST_CONV = 2;                      // converter warps per stage slot
constexpr uint32_t ST_KC = 64;                       // K per TMEM accumulation chunk
constexpr uint32_t ST_BRAW = ST_BK * ST_NT * 4;      // raw B box [32][128]
constexpr uint32_t ST_BT = ST_NT * ST_BK * 4;        // one of B^T hi / lo [128][32]
constexpr uint32_t ST_A = ST_MN * ST_BK * 4;         // one of A hi / lo [16][32]
constexpr uint32_t ST_STAGE = ST_BRAW + 2 * ST_BT + 2 * ST_A;
constexpr uint32_t ST_SMEM = ST_S * ST_STAGE + 1024;
constexpr uint32_t ST_EPI_WARP0 = 2 + ST_S * ST_CONV;  // warps 10..13
constexpr int ST_THREADS = 32 * (ST_EPI_WARP0 + 4);
static_assert(ST_STAGE % 1024 == 0, "stage slots keep the 128-byte swizzle atoms aligned");

__global__ void __launch_bounds__(ST_THREADS, 1)
    sgemm_smallm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                           float* __restrict__ c, uint64_t ldc, float* __restrict__ partial, uint32_t m, uint32_t n,
                           uint32_t k, uint32_t kchunk, unsigned int* __restrict__ err) {
  constexpr uint32_t IDESC = umma_idesc_tf32(ST_NT, ST_MN);
  constexpr uint32_t KBC = ST_KC / ST_BK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t raw_full[ST_S], full_bar[ST_S], empty_bar[ST_S];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t aborted;
  __shared__ uint32_t issued_kb;
  __shared__ uint32_t converted_kb[ST_S * ST_CONV];

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * ST_NT;
  const uint32_t split = blockIdx.y;
  const uint32_t k0 = split * kchunk, k1 = min(k, k0 + kchunk);
  const uint32_t num_kb = (k1 - k0 + ST_BK - 1) / ST_BK;
  const uint32_t num_chunks = (num_kb + KBC - 1) / KBC;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < ST_S; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&full_bar[s], ST_CONV);
      mbar_init(&empty_bar[s], 1);
    }
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(&drain_bar, 1);
    aborted = 0;
    issued_kb = 0;
    for (uint32_t w = 0; w < ST_S * ST_CONV; ++w) converted_kb[w] = w / ST_CONV;  // each warp's next stage
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      for (uint32_t kb = 0; kb < num_kb; ++kb) {
        const uint32_t s = kb % ST_S;
        if (kb >= ST_S && !mbar_wait(&empty_bar[s], ((kb / ST_S) - 1) & 1u, err, kErrWaitEmpty)) {
          atomicExch(&aborted, 1u);
          break;
        }
        if (*(volatile uint32_t*)&aborted != 0u) break;
        uint8_t* st = smem + s * ST_STAGE;
        const int kx = static_cast<int>(k0 + kb * ST_BK);
        mbar_arrive_expect_tx(&raw_full[s], ST_BRAW + ST_A);
        tma_load_2d(st, &tm_b, &raw_full[s], static_cast<int>(n0), kx);           // B [32 k][128 n]
        tma_load_2d(st + ST_BRAW + 2 * ST_BT, &tm_a, &raw_full[s], kx, 0);        // A [16 m][32 k] -> A hi slot
        *(volatile uint32_t*)&issued_kb = kb + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      for (uint32_t kb = 0; kb < num_kb; ++kb) {
        const uint32_t chunk = kb / KBC, in_chunk = kb % KBC, buf = chunk & 1u;
        if (in_chunk == 0 && chunk >= 2) {
          if (!mbar_wait(&acc_empty[buf], ((chunk >> 1) - 1) & 1u, err, kErrWaitAccum)) {
            atomicExch(&aborted, 1u);
            break;
          }
          tc_fence_after();
        }
        const uint32_t s = kb % ST_S;
        if (!mbar_wait(&full_bar[s], (kb / ST_S) & 1u, err, kErrWaitFull)) {
          atomicExch(&aborted, 1u);
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_addr(smem + s * ST_STAGE);
        const uint32_t bt_hi = base + ST_BRAW, bt_lo = bt_hi + ST_BT;
        const uint32_t a_hi = bt_hi + 2 * ST_BT, a_lo = a_hi + ST_A;
        const uint32_t d = tmem + buf * ST_MN;
#pragma unroll
        for (uint32_t kk = 0; kk < ST_BK / 8; ++kk) {
          const uint32_t off = kk * 32;
          const uint64_t dbh = umma_desc_kmajor(bt_hi + off, 128);
          const uint64_t dbl = umma_desc_kmajor(bt_lo + off, 128);
          const uint64_t dah = umma_desc_kmajor(a_hi + off, 128);
          const uint64_t dal = umma_desc_kmajor(a_lo + off, 128);
          umma_tf32(d, dbl, dah, IDESC, (in_chunk | kk) != 0u ? 1u : 0u);
          umma_tf32(d, dbh, dal, IDESC, 1u);
          umma_tf32(d, dbh, dah, IDESC, 1u);
        }
        umma_commit(&empty_bar[s]);
        if (in_chunk == KBC - 1 || kb == num_kb - 1) umma_commit(&acc_full[buf]);
      }
      umma_commit(&drain_bar);
    }
  } else if (warp < ST_EPI_WARP0) {
    // ---------------- converters: warps (2 s + 2, 2 s + 3) own stage slot s and share
    // its granules; a warp only waits for the next phase of its own slot's barrier.
    const uint32_t cw = warp - 2u;
    const uint32_t slot = cw / ST_CONV, half = cw % ST_CONV;
    // Each lane owns whole rows of B^T (columns of B): rows lane + 32 t, t = 2 half, 2 half + 1,
    // all 8 k groups of each; the second warp also splits A (4 granules a lane).
    constexpr uint32_t GROUPS = ST_BK / 4;
    static_assert(ST_CONV == 2 && ST_NT == 128 && ST_A / 16 % 32 == 0, "two warps share 4 x 32 rows and A");
    for (uint32_t kb = slot; kb < num_kb; kb += ST_S) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&raw_full[slot], (kb / ST_S) & 1u, err, kErrWaitFull));
      if (!ok || *(volatile uint32_t*)&aborted != 0u) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      uint8_t* st = smem + slot * ST_STAGE;
      const float* braw = reinterpret_cast<const float*>(st);  // [32][128]
      uint8_t* bthi = st + ST_BRAW;
      uint8_t* btlo = bthi + ST_BT;
      float4* ahi = reinterpret_cast<float4*>(btlo + ST_BT);
      float4* alo = reinterpret_cast<float4*>(btlo + ST_BT + ST_A);
#pragma unroll 1
      for (uint32_t t = 2 * half; t < 2 * half + 2; ++t) {
        const uint32_t r = lane + 32u * t, x = r & 7u;
        const float* src = braw + r;
        float4 v[GROUPS];
#pragma unroll
        for (uint32_t g = 0; g < GROUPS; ++g)
          v[g] = make_float4(src[(4 * g) * ST_NT], src[(4 * g + 1) * ST_NT], src[(4 * g + 2) * ST_NT],
                             src[(4 * g + 3) * ST_NT]);
#pragma unroll
        for (uint32_t g = 0; g < GROUPS; ++g) {
          float4 h, l;
          h.x = to_tf32(v[g].x); h.y = to_tf32(v[g].y); h.z = to_tf32(v[g].z); h.w = to_tf32(v[g].w);
          l.x = to_tf32(v[g].x - h.x); l.y = to_tf32(v[g].y - h.y);
          l.z = to_tf32(v[g].z - h.z); l.w = to_tf32(v[g].w - h.w);
          const uint32_t off = r * 128u + ((g ^ x) << 4);  // 128-byte swizzle
          *reinterpret_cast<float4*>(bthi + off) = h;
          *reinterpret_cast<float4*>(btlo + off) = l;
        }
      }
      if (half == 1) {
        float4 v[ST_A / 16 / 32];
#pragma unroll
        for (uint32_t u = 0; u < ST_A / 16 / 32; ++u) v[u] = ahi[lane + 32 * u];
#pragma unroll
        for (uint32_t u = 0; u < ST_A / 16 / 32; ++u) {
          float4 h, l;
          h.x = to_tf32(v[u].x); h.y = to_tf32(v[u].y); h.z = to_tf32(v[u].z); h.w = to_tf32(v[u].w);
          l.x = to_tf32(v[u].x - h.x); l.y = to_tf32(v[u].y - h.y);
          l.z = to_tf32(v[u].z - h.z); l.w = to_tf32(v[u].w - h.w);
          ahi[lane + 32 * u] = h;
          alo[lane + 32 * u] = l;
        }
      }
      fence_proxy_async_smem();  // the generic-proxy writes, visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full_bar[slot]);
        *(volatile uint32_t*)&converted_kb[cw] = kb + ST_S;
      }
    }
  } else {
    // ---------------- epilogue: lane quarter (warp % 4) of TMEM = 32 columns of C
    const uint32_t q = warp & 3u;
    const uint32_t lane_addr = (q * 32u) << 16;
    float run[ST_MN];
#pragma unroll
    for (uint32_t j = 0; j < ST_MN; ++j) run[j] = 0.f;
    bool ok = true;
    for (uint32_t ch = 0; ch < num_chunks; ++ch) {
      const uint32_t buf = ch & 1u;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (ch >> 1) & 1u, err, kErrWaitAccum));
      if (!ok) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      tc_fence_after();
      uint32_t r[16];
      tmem_ld_32x32b_x16(tmem + lane_addr + buf * ST_MN, r);
      tmem_ld_wait();
#pragma unroll
      for (uint32_t j = 0; j < ST_MN; ++j) run[j] += __uint_as_float(r[j]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    const uint32_t col = n0 + q * 32u + lane;
    if (ok && col < n) {
      float* dst = partial == nullptr ? c + col : partial + static_cast<uint64_t>(split) * m * n + col;
      const uint64_t ld = partial == nullptr ? ldc : n;
#pragma unroll
      for (uint32_t j = 0; j < ST_MN; ++j)
        if (j < m) dst[j * ld] = run[j];
    }
  }

  tc_fence_before();
  __syncthreads();
  // Teardown: the MMA thread's last commit says every MMA finished; a CTA that
  // aborted also waits (bounded) for its TMA copies that no converter consumed.
  if (threadIdx.x == 32) mbar_wait(&drain_bar, 0, err, kErrWaitDrain);
  if (aborted && threadIdx.x == 0) {
    uint32_t done = converted_kb[0];
    for (uint32_t w = 1; w < ST_S * ST_CONV; ++w) done = min(done, converted_kb[w]);
    for (uint32_t kb = done; kb < issued_kb; ++kb)
      if (!mbar_wait(&raw_full[kb % ST_S], (kb / ST_S) & 1u, err, kErrWaitDrain)) break;
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// C[i][j] = sum over splits s, in order, of partial[s][i][j].
__global__ void smallm_tc_reduce_kernel(const float* __restrict__ partial, float* __restrict__ c, uint64_t ldc,
                                        uint32_t m, uint32_t n, uint32_t splits) {
  const uint64_t total = static_cast<uint64_t>(m) * n;
  for (uint64_t e = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    float s = partial[e];
    for (uint32_t sp = 1; sp < splits; ++sp) s += partial[static_cast<uint64_t>(sp) * total + e];
    const uint32_t i = static_cast<uint32_t>(e / n), j = static_cast<uint32_t>(e - static_cast<uint64_t>(i) * n);
    c[static_cast<uint64_t>(i) * ldc + j] = s;
  }
}

bool make_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_x,
              uint32_t box_y, bool swizzle128) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 4};
  const cuuint32_t box[2] = {box_x, box_y};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K splits: enough CTAs for two per SM, each split at least 256 deep.
uint32_t smallm_tc_splits(uint32_t n, uint32_t k, uint32_t* kchunk) {
  const uint32_t tiles = (n + ST_NT - 1) / ST_NT;
  uint32_t splits = std::max<uint32_t>(1, (2 * 148 + tiles - 1) / tiles);
  splits = std::min<uint32_t>(splits, std::max<uint32_t>(1, k / 256));
  uint32_t chunk = (k + splits - 1) / splits;
  chunk = (chunk + ST_KC - 1) / ST_KC * ST_KC;
  *kchunk = chunk;
  return (k + chunk - 1) / chunk;
}

}  // namespace

bool sgemm_smallm_tc_eligible(const float* a, uint64_t lda, const float* b, uint64_t ldb, uint32_t m, uint32_t n,
                              uint32_t k) {
  return m >= 1 && m <= ST_MN && n > 0 && k > 0 && lda % 4 == 0 && ldb % 4 == 0 &&
         (reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0 &&
         lda < (1ull << 37) && ldb < (1ull << 37);
}

uint64_t sgemm_smallm_tc_scratch_bytes(uint32_t m, uint32_t n, uint32_t k) {
  uint32_t chunk = 0;
  const uint32_t splits = smallm_tc_splits(n, k, &chunk);
  return splits > 1 ? static_cast<uint64_t>(splits) * m * n * sizeof(float) : 0;
}

cudaError_t sgemm_smallm_tc(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                            uint32_t m, uint32_t n, uint32_t k, void* scratch, unsigned int* err,
                            cudaStream_t stream) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if (!sgemm_smallm_tc_eligible(a, lda, b, ldb, m, n, k) || err == nullptr) return cudaErrorInvalidValue;
  uint32_t kchunk = 0;
  const uint32_t splits = smallm_tc_splits(n, k, &kchunk);
  float* partial = nullptr;
  if (splits > 1) {
    if (scratch == nullptr) return cudaErrorInvalidValue;
    partial = static_cast<float*>(scratch);
  }
  CUtensorMap m_a, m_b;
  if (!make_map(&m_a, a, k, m, lda, ST_BK, ST_MN, true) || !make_map(&m_b, b, n, k, ldb, ST_NT, ST_BK, false))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(sgemm_smallm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ST_SMEM));
  if (e != cudaSuccess) return e;
  const dim3 grid((n + ST_NT - 1) / ST_NT, splits);
  sgemm_smallm_tc_kernel<<<grid, ST_THREADS, ST_SMEM, stream>>>(m_a, m_b, c, ldc, partial, m, n, k, kchunk, err);
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const uint64_t total = static_cast<uint64_t>(m) * n;
  const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((total + 255) / 256, 148ull * 8));
  smallm_tc_reduce_kernel<<<blocks, 256, 0, stream>>>(partial, c, ldc, m, n, splits);
  return cudaGetLastError();
}

}  // namespace oct
