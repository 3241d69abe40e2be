// sgemm_tc.cu -- fp32 SGEMM on the sm_100a tensor cores with the 3xTF32 split.
//
// C[m x n] = A[m x k] * B[k x n], all row-major fp32, C overwritten.  This is the
// product Oct's `prometheus_reactor_runtime_sgemm` computes
// (internal/prometheus/native/reactor_api.h:2587-2595) and that its CPU oracle
// `cpuSGEMM` restates (internal/prometheus/runtime.go:319-331).
//
// Precision: each operand x is split as x_hi = tf32(x) and x_lo = tf32(x - x_hi)
// (round to nearest), which represents x to about 2^-22 relative.  The product
// is accumulated in fp32 in TMEM as  A_hi*B_hi + A_hi*B_lo + A_lo*B_hi;  the
// dropped A_lo*B_lo term is below fp32 resolution.  The result is as accurate
// as a plain fp32 dot product (tests pin it against an fp64 oracle).
//
// Pipeline:
//   1. split_rows / split_transpose write hi/lo copies of A and of B^T into
//      a zero-padded, K-major scratch layout (M to 128, N to 256, K to 32).
//      Padding removes every ragged edge from the main loop.
//   2. sgemm3x_kernel: one CTA per 128x256 output tile, warp-specialised:
//        warp 0      TMA producer: 4 tiles per stage (A_hi, A_lo, B_hi, B_lo)
//                    into a `STAGES`-deep shared-memory ring, 64/128-B swizzle;
//        warp 1      MMA issuer: one thread issues 3 tcgen05.mma (kind::tf32,
//                    M=128, N=256, K=8) per 8-deep k step into one of two
//                    128x256 fp32 TMEM accumulators (alternating every 64 of
//                    K, see the accumulation note), frees a stage with
//                    tcgen05.commit;
//        warps 2..9  epilogue: drain each K chunk's accumulator from TMEM
//                    (tcgen05.ld) into fp32 register running sums, then store C
//                    with predicated (exact-tail) vector stores.
//   Every wait is bounded (see ptx.cuh); a timeout sets a bit in `err`.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <algorithm>
#include <mutex>

#include "../../include/prometheus_reactor.h"
#include "kernels.h"
#include "ptx.cuh"

namespace oct {
namespace {

constexpr uint32_t BM = 128;
constexpr uint32_t BN = 256;
constexpr uint32_t KPAD = 32;       // K padding granule of the split buffers
constexpr uint32_t GROUP_M = 16;    // tile rasterisation: M tiles per group
constexpr uint32_t TMEM_COLS = 512; // two 256-column fp32 accumulators (2 x BN)
constexpr int NUM_THREADS = 320;  // producer warp, MMA warp, 8 epilogue warps

template <int BK>
struct TileCfg {
  static constexpr uint32_t SWZ = BK * 4;                 // bytes per smem row = swizzle span
  static constexpr uint32_t A_BYTES = BM * BK * 4;
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr uint32_t STAGES = (BK == 16) ? 4 : 2;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
};

__host__ __device__ inline uint32_t round_up(uint32_t x, uint32_t g) { return (x + g - 1) / g * g; }

// ------------------------------------------------------------------ split
// hi = tf32(v), lo = tf32(v - hi); v = 0 outside [rows, cols).
// Each thread produces 4 consecutive padded columns of one row.
// blockIdx.y selects the batch entry: src + src_stride.at(y), outputs + y * rows_p * cols_p.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ src, uint64_t ld,
                                                         uint32_t rows, uint32_t cols,
                                                         float* __restrict__ hi, float* __restrict__ lo,
                                                         uint32_t rows_p, uint32_t cols_p, EntryStride src_stride) {
  src += src_stride.at(blockIdx.y);
  hi += static_cast<uint64_t>(blockIdx.y) * rows_p * cols_p;
  lo += static_cast<uint64_t>(blockIdx.y) * rows_p * cols_p;
  const uint64_t groups_per_row = cols_p / 4;
  const uint64_t total = static_cast<uint64_t>(rows_p) * groups_per_row;
  const bool vec_ok = (ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t r = static_cast<uint32_t>(g / groups_per_row);
    const uint32_t c = static_cast<uint32_t>(g % groups_per_row) * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < rows) {
      const float* p = src + r * ld + c;
      if (vec_ok && c + 4 <= cols) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c + j < cols) v[j] = __ldg(p + j);
      }
    }
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = to_tf32(v[j]);
      l[j] = to_tf32(v[j] - h[j]);
    }
    const uint64_t o = static_cast<uint64_t>(r) * cols_p + c;
    *reinterpret_cast<float4*>(hi + o) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + o) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// B is [k x n] row-major; writes hi/lo of B^T as [n_p x k_p] (K-major), zero padded.
// 32x32 tiles through shared memory keep both the read and the write coalesced.
// blockIdx.z selects the batch entry: b + b_stride.at(z), outputs + z * np * kp.
__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ b, uint64_t ldb,
                                                              uint32_t k, uint32_t n,
                                                              float* __restrict__ hi, float* __restrict__ lo,
                                                              uint32_t kp, uint32_t np, EntryStride b_stride) {
  __shared__ float tile[32][33];
  b += b_stride.at(blockIdx.z);
  hi += static_cast<uint64_t>(blockIdx.z) * np * kp;
  lo += static_cast<uint64_t>(blockIdx.z) * np * kp;
  const uint32_t n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t kk = k0 + ty + 8 * i, nn = n0 + tx;
    tile[ty + 8 * i][tx] = (kk < k && nn < n) ? __ldg(b + kk * ldb + nn) : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t nn = n0 + ty + 8 * i, kk = k0 + tx;
    const float v = tile[tx][ty + 8 * i];
    const float h = to_tf32(v);
    const uint64_t o = static_cast<uint64_t>(nn) * kp + kk;
    hi[o] = h;
    lo[o] = to_tf32(v - h);
  }
}

// ------------------------------------------------------------------ main kernel
// Accumulation precision.  The tensor core adds each MMA's products into the
// TMEM accumulator with round-toward-zero, so a single accumulator over all of
// K collects a biased error that grows like K^1.5 (at K = 512 it is already 4x
// the error of a plain fp32 dot product).  The kernel therefore restarts the
// TMEM accumulation every KC elements of K and adds each chunk's partial sum
// into an fp32 running sum in registers (round-to-nearest).  Two 256-column
// TMEM buffers alternate so the MMA fills one chunk while the epilogue warps
// drain the other.  With KC = 64 the result is more accurate than Oct's own
// sequential fp32 CPU loop at every K tested (512 ... 8192).
constexpr uint32_t KC = 64;                 // K elements per TMEM accumulation chunk
constexpr uint32_t NUM_EPI_WARPS = 8;       // 2 per TMEM lane quarter: 128 columns each

template <int BK>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    sgemm3x_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                   const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                   float* __restrict__ c, uint32_t m, uint32_t n, uint64_t ldc, uint32_t kb_total,
                   uint32_t tiles_m, uint32_t tiles_n, uint32_t entry_rows_a, uint32_t entry_rows_b,
                   EntryStride stride_c, const float* __restrict__ residual, uint64_t ldr,
                   unsigned int* __restrict__ err, const RowScatter scatter, uint32_t kb_split) {
  using Cfg = TileCfg<BK>;
  constexpr uint32_t S = Cfg::STAGES;
  constexpr uint32_t KBC = KC / BK;  // k-blocks per accumulation chunk
  constexpr uint32_t IDESC = umma_idesc_tf32(BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t issued_kb, consumed_kb, aborted;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Batch entry, then grouped rasterisation inside it: GROUP_M tile rows
  // sweep all tile columns together.  Split buffers stack the batch entries
  // along rows (Mp and Np rows each), so a tile never straddles two entries.
  // Split K (kb_split > 0): entry e is the K range [e * kb_split, ...) of one
  // product (the host passes zero entry rows), written to its own slice of C
  // (or, scattering, to its own slot of the owner rank).
  const uint32_t tiles_per_entry = tiles_m * tiles_n;
  const uint32_t entry = blockIdx.x / tiles_per_entry;
  const uint32_t kb0 = kb_split != 0u ? entry * kb_split : 0u;
  const uint32_t num_kb = kb_split != 0u ? min(kb_total - kb0, kb_split) : kb_total;
  const uint32_t num_chunks = (num_kb + KBC - 1) / KBC;
  const uint32_t t = blockIdx.x % tiles_per_entry;
  const uint32_t per_group = GROUP_M * tiles_n;
  const uint32_t first_m = (t / per_group) * GROUP_M;
  const uint32_t group_rows = min(tiles_m - first_m, GROUP_M);
  const uint32_t tile_m = first_m + (t % per_group) % group_rows;
  const uint32_t tile_n = (t % per_group) / group_rows;
  c += stride_c.at(entry);
  if (residual != nullptr) residual += stride_c.at(entry);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], NUM_EPI_WARPS);
    }
    mbar_init(&drain_bar, 1);
    issued_kb = 0;
    consumed_kb = 0;
    aborted = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tensormap(&tm_ahi);
    prefetch_tensormap(&tm_alo);
    prefetch_tensormap(&tm_bhi);
    prefetch_tensormap(&tm_blo);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: the warp runs the loop converged, one elected lane issues
    const int row_a = static_cast<int>(entry * entry_rows_a + tile_m * BM);
    const int row_b = static_cast<int>(entry * entry_rows_b + tile_n * BN);
    uint32_t kb = 0;
    for (; kb < num_kb; ++kb) {
      const uint32_t s = kb % S;
      if (kb >= S) {
        if (!__all_sync(0xffffffffu, mbar_wait(&empty_bar[s], ((kb / S) - 1) & 1u, err, kErrWaitEmpty))) {
          if (lane == 0) atomicExch(&aborted, 1u);
          break;
        }
      }
      if (__any_sync(0xffffffffu, *(volatile uint32_t*)&aborted != 0u)) break;
      uint8_t* st = smem + s * Cfg::STAGE_BYTES;
      const int kx = static_cast<int>((kb0 + kb) * BK);
      if (elect_one()) {
        mbar_arrive_expect_tx(&full_bar[s], Cfg::STAGE_BYTES);
        tma_load_2d(st, &tm_ahi, &full_bar[s], kx, row_a);
        tma_load_2d(st + Cfg::A_BYTES, &tm_alo, &full_bar[s], kx, row_a);
        tma_load_2d(st + 2 * Cfg::A_BYTES, &tm_bhi, &full_bar[s], kx, row_b);
        tma_load_2d(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tm_blo, &full_bar[s], kx, row_b);
      }
      __syncwarp();
    }
    if (lane == 0) issued_kb = kb;
  } else if (warp == 1) {
    // ---------------- MMA issuer: converged warp (descriptors stay warp-uniform), one
    // elected lane issues each tcgen05 instruction
    uint32_t kb = 0;
    for (; kb < num_kb; ++kb) {
      const uint32_t chunk = kb / KBC, in_chunk = kb % KBC;
      const uint32_t buf = chunk & 1u;
      if (in_chunk == 0 && chunk >= 2) {
        // the epilogue must have drained chunk - 2 out of this buffer
        if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], ((chunk >> 1) - 1) & 1u, err, kErrWaitAccum))) {
          if (lane == 0) atomicExch(&aborted, 1u);
          break;
        }
        tc_fence_after();
      }
      const uint32_t s = kb % S;
      if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[s], (kb / S) & 1u, err, kErrWaitFull))) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      const uint32_t base = smem_addr(smem + s * Cfg::STAGE_BYTES);
      const uint32_t a_hi = base, a_lo = base + Cfg::A_BYTES;
      const uint32_t b_hi = base + 2 * Cfg::A_BYTES, b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
      for (uint32_t kk = 0; kk < BK / 8; ++kk) {
        const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K
        const uint64_t dah = umma_desc_kmajor(a_hi + off, Cfg::SWZ);
        const uint64_t dal = umma_desc_kmajor(a_lo + off, Cfg::SWZ);
        const uint64_t dbh = umma_desc_kmajor(b_hi + off, Cfg::SWZ);
        const uint64_t dbl = umma_desc_kmajor(b_lo + off, Cfg::SWZ);
        if (elect_one()) {
          umma_tf32(d_tmem, dal, dbh, IDESC, (in_chunk | kk) != 0u ? 1u : 0u);
          umma_tf32(d_tmem, dah, dbl, IDESC, 1u);
          umma_tf32(d_tmem, dah, dbh, IDESC, 1u);
        }
        __syncwarp();
      }
      if (elect_one()) {
        umma_commit(&empty_bar[s]);  // frees the smem stage when these MMAs finish
        if (in_chunk == KBC - 1 || kb == num_kb - 1) umma_commit(&acc_full[buf]);
      }
      __syncwarp();
    }
    if (lane == 0) consumed_kb = kb;
    if (elect_one()) umma_commit(&drain_bar);  // arrives when every MMA issued above has completed
    __syncwarp();
  } else {
    // ---------------- epilogue: warps 2..9; (warp % 4) owns a TMEM lane quarter,
    // (warp - 2) / 4 selects which 128 of the 256 columns this warp sums.
    const uint32_t q = warp & 3u;
    const uint32_t h = (warp - 2u) >> 2;
    const uint32_t lane_addr = (q * 32u) << 16;
    float run[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) run[j] = 0.f;
    bool ok = true;
    for (uint32_t ch = 0; ch < num_chunks; ++ch) {
      const uint32_t buf = ch & 1u;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (ch >> 1) & 1u, err, kErrWaitAccum));
      if (!ok) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      tc_fence_after();
#pragma unroll
      for (uint32_t g = 0; g < 4; ++g) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * BN + h * 128u + g * 32u, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) run[g * 32 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (scatter.dst != nullptr && num_kb > 0) {
      // Row scatter: stage the 128 x 256 tile in the operand ring (idle once the
      // last accumulator chunk arrived: every MMA and TMA copy has completed), then
      // each warp stores whole rows as 512-byte coalesced segments -- the remote
      // rows cross NVLink in full packets instead of 16-byte pieces.
      constexpr uint32_t LDS = BN + 4;  // padded row stride (floats): conflict-free float4 stores
      float* stage_tile = reinterpret_cast<float*>(smem);
      if (ok) {
        float* srow = stage_tile + (q * 32 + lane) * LDS + h * 128u;
#pragma unroll
        for (int j = 0; j < 128; j += 4)
          *reinterpret_cast<float4*>(srow + j) = make_float4(run[j], run[j + 1], run[j + 2], run[j + 3]);
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight epilogue warps
      if (*(volatile uint32_t*)&aborted == 0u && scatter.bcast > 0u) {
        // Broadcast: each row to every rank, the peers first and this rank last,
        // each warp starting at a different peer so the links fill evenly.
        const uint32_t ew = warp - 2u;
        for (uint32_t lr = ew; lr < BM; lr += 8u) {
          const uint32_t row = tile_m * BM + lr;
          if (row >= m) break;
          const float* srow = stage_tile + lr * LDS;
          for (uint32_t i = 1; i <= scatter.bcast; ++i) {
            const uint32_t rk = (scatter.src_rank + (i == scatter.bcast ? 0u : 1u + (i - 1u + ew) % (scatter.bcast - 1u))) %
                                scatter.bcast;
            float* drow = scatter.dst[rk] + static_cast<uint64_t>(row) * scatter.ld + scatter.col_offset;
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
              const uint32_t cl = half * 128u + lane * 4u;
              const uint32_t col = tile_n * BN + cl;
              if (col + 4 <= n) {
                *reinterpret_cast<float4*>(drow + col) = *reinterpret_cast<const float4*>(srow + cl);
              } else {
                for (uint32_t t = 0; t < 4; ++t)
                  if (col + t < n) drow[col + t] = srow[cl + t];
              }
            }
          }
        }
      } else if (*(volatile uint32_t*)&aborted == 0u) {
        const uint32_t ew = warp - 2u;
        for (uint32_t lr = ew; lr < BM; lr += 8u) {
          const uint32_t row = tile_m * BM + lr;
          if (row >= m) break;
          const uint32_t owner = row / scatter.rows_per_rank;
          const uint32_t slot = scatter.src_rank + (kb_split != 0u ? entry : 0u);
          const uint64_t slot_row =
              static_cast<uint64_t>(slot) * scatter.rows_per_rank + (row - owner * scatter.rows_per_rank);
          float* drow = scatter.dst[owner] + slot_row * scatter.ld;
          const float* srow = stage_tile + lr * LDS;
#pragma unroll
          for (uint32_t half = 0; half < 2; ++half) {
            const uint32_t cl = half * 128u + lane * 4u;  // column within the tile
            const uint32_t col = tile_n * BN + cl;
            if (col + 4 <= n) {
              *reinterpret_cast<float4*>(drow + col) = *reinterpret_cast<const float4*>(srow + cl);
            } else {
              for (uint32_t t = 0; t < 4; ++t)
                if (col + t < n) drow[col + t] = srow[cl + t];
            }
          }
        }
      }
    } else if (ok && num_kb > 0) {
      const uint32_t row = tile_m * BM + q * 32 + lane;
      const uint32_t col0 = tile_n * BN + h * 128u;
      const bool vec_ok = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) &&
                          (residual == nullptr ||
                           ((ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(residual) & 15u) == 0)));
      if (row < m && col0 < n) {
        float* dst = c + static_cast<uint64_t>(row) * ldc + col0;
        // Optional fused residual epilogue: C = R + A * B (R may alias C).
        const float* src = residual != nullptr ? residual + static_cast<uint64_t>(row) * ldr + col0 : nullptr;
        if (vec_ok && col0 + 128 <= n) {
#pragma unroll
          for (int j = 0; j < 128; j += 4) {
            float4 v = make_float4(run[j], run[j + 1], run[j + 2], run[j + 3]);
            if (src != nullptr) {
              const float4 r4 = *reinterpret_cast<const float4*>(src + j);
              v.x += r4.x;
              v.y += r4.y;
              v.z += r4.z;
              v.w += r4.w;
            }
            *reinterpret_cast<float4*>(dst + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 128; ++j)
            if (col0 + j < n) dst[j] = src != nullptr ? src[j] + run[j] : run[j];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Teardown.  The MMA thread waits (bounded) until all its MMAs completed; an
  // aborted CTA also waits for TMA copies still in flight before it exits.
  if (threadIdx.x == 32) mbar_wait(&drain_bar, 0, err, kErrWaitDrain);
  if (aborted && threadIdx.x == 0) {
    for (uint32_t kb = consumed_kb; kb < issued_kb; ++kb)
      if (!mbar_wait(&full_bar[kb % S], (kb / S) & 1u, err, kErrWaitDrain)) break;
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ CTA-pair kernel
// Same product and accumulation scheme on a CTA pair (cluster of 2) that owns a
// 256 x 256 output tile: each CTA stages its own 128 rows of A and 128 of the
// 256 B^T rows, and the leader CTA issues tcgen05.mma.cta_group::2 (M = 256,
// N = 256), which reads the operand halves of both CTAs.  Per CTA a stage is
// 32 KB instead of 48 KB for the same tensor work, so six stages fit, and each
// CTA keeps a 128 x 256 accumulator half in its own TMEM.
//   * both CTAs' TMA loads count their bytes on the leader's `full` barrier;
//   * the leader's commits multicast to both CTAs' `empty` / `acc_full`;
//   * both CTAs' epilogue warps arrive on the leader's `acc_empty` (16 arrivals).
constexpr uint32_t PAIR_BM = 256, PAIR_HALF = 128;

template <int BK>
struct PairCfg {
  static constexpr uint32_t SWZ = BK * 4;
  static constexpr uint32_t A_BYTES = PAIR_HALF * BK * 4;  // this CTA's 128 rows of A
  static constexpr uint32_t B_BYTES = PAIR_HALF * BK * 4;  // this CTA's 128 rows of B^T
  static constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr uint32_t STAGES = (BK == 16) ? 6 : 3;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
};

template <int BK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    sgemm3x_pair_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                        const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                        float* __restrict__ c, uint32_t m, uint32_t n, uint64_t ldc, uint32_t num_kb,
                        uint32_t tiles_m, uint32_t tiles_n, uint32_t entry_rows_a, uint32_t entry_rows_b,
                        EntryStride stride_c, const float* __restrict__ residual, uint64_t ldr,
                        unsigned int* __restrict__ err, const RowScatter scatter) {
  using Cfg = PairCfg<BK>;
  constexpr uint32_t S = Cfg::STAGES;
  constexpr uint32_t KBC = KC / BK;
  constexpr uint32_t IDESC = umma_idesc_tf32(PAIR_BM, BN);
  constexpr uint16_t PAIR_MASK = 0x3;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t aborted;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();  // 0 = leader
  const uint32_t num_chunks = (num_kb + KBC - 1) / KBC;

  const uint32_t pair = blockIdx.x >> 1;
  const uint32_t tiles_per_entry = tiles_m * tiles_n;
  const uint32_t entry = pair / tiles_per_entry;
  const uint32_t t = pair % tiles_per_entry;
  const uint32_t per_group = GROUP_M * tiles_n;
  const uint32_t first_m = (t / per_group) * GROUP_M;
  const uint32_t group_rows = min(tiles_m - first_m, GROUP_M);
  const uint32_t tile_m = first_m + (t % per_group) % group_rows;
  const uint32_t tile_n = (t % per_group) / group_rows;
  c += stride_c.at(entry);
  if (residual != nullptr) residual += stride_c.at(entry);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * NUM_EPI_WARPS);
    }
    mbar_init(&drain_bar, 1);
    aborted = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tensormap(&tm_ahi);
    prefetch_tensormap(&tm_alo);
    prefetch_tensormap(&tm_bhi);
    prefetch_tensormap(&tm_blo);
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      const int row_a = static_cast<int>(entry * entry_rows_a + tile_m * PAIR_BM + rank * PAIR_HALF);
      const int row_b = static_cast<int>(entry * entry_rows_b + tile_n * BN + rank * PAIR_HALF);
      for (uint32_t kb = 0; kb < num_kb; ++kb) {
        const uint32_t s = kb % S;
        if (kb >= S) {
          if (!mbar_wait(&empty_bar[s], ((kb / S) - 1) & 1u, err, kErrWaitEmpty)) {
            atomicExch(&aborted, 1u);
            break;
          }
        }
        uint8_t* st = smem + s * Cfg::STAGE_BYTES;
        const int kx = static_cast<int>(kb * BK);
        if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::STAGE_BYTES);
        tma_load_2d_pair(st, &tm_ahi, &full_bar[s], kx, row_a);
        tma_load_2d_pair(st + Cfg::A_BYTES, &tm_alo, &full_bar[s], kx, row_a);
        tma_load_2d_pair(st + 2 * Cfg::A_BYTES, &tm_bhi, &full_bar[s], kx, row_b);
        tma_load_2d_pair(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tm_blo, &full_bar[s], kx, row_b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader CTA only)
      for (uint32_t kb = 0; kb < num_kb; ++kb) {
        const uint32_t chunk = kb / KBC, in_chunk = kb % KBC;
        const uint32_t buf = chunk & 1u;
        if (in_chunk == 0 && chunk >= 2) {
          if (!mbar_wait(&acc_empty[buf], ((chunk >> 1) - 1) & 1u, err, kErrWaitAccum)) {
            atomicExch(&aborted, 1u);
            break;
          }
          tc_fence_after();
        }
        const uint32_t s = kb % S;
        if (!mbar_wait(&full_bar[s], (kb / S) & 1u, err, kErrWaitFull)) {
          atomicExch(&aborted, 1u);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const uint32_t base = smem_addr(smem + s * Cfg::STAGE_BYTES);
        const uint32_t a_hi = base, a_lo = base + Cfg::A_BYTES;
        const uint32_t b_hi = base + 2 * Cfg::A_BYTES, b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
        for (uint32_t kk = 0; kk < BK / 8; ++kk) {
          const uint32_t off = kk * 32;
          const uint64_t dah = umma_desc_kmajor(a_hi + off, Cfg::SWZ);
          const uint64_t dal = umma_desc_kmajor(a_lo + off, Cfg::SWZ);
          const uint64_t dbh = umma_desc_kmajor(b_hi + off, Cfg::SWZ);
          const uint64_t dbl = umma_desc_kmajor(b_lo + off, Cfg::SWZ);
          umma_tf32_pair(d_tmem, dal, dbh, IDESC, (in_chunk | kk) != 0u ? 1u : 0u);
          umma_tf32_pair(d_tmem, dah, dbl, IDESC, 1u);
          umma_tf32_pair(d_tmem, dah, dbh, IDESC, 1u);
        }
        umma_commit_pair_mc(&empty_bar[s], PAIR_MASK);
        if (in_chunk == KBC - 1 || kb == num_kb - 1) umma_commit_pair_mc(&acc_full[buf], PAIR_MASK);
      }
      umma_commit_pair_mc(&drain_bar, PAIR_MASK);
    }
  } else {
    // ---------------- epilogue: warps 2..9 of both CTAs, each on its own TMEM half
    const uint32_t q = warp & 3u;
    const uint32_t h = (warp - 2u) >> 2;
    const uint32_t lane_addr = (q * 32u) << 16;
    float run[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) run[j] = 0.f;
    bool ok = true;
    for (uint32_t ch = 0; ch < num_chunks; ++ch) {
      const uint32_t buf = ch & 1u;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (ch >> 1) & 1u, err, kErrWaitAccum));
      if (!ok) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      tc_fence_after();
#pragma unroll
      for (uint32_t g = 0; g < 4; ++g) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * BN + h * 128u + g * 32u, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) run[g * 32 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&acc_empty[buf], 0);
    }
    if (scatter.dst != nullptr && num_kb > 0) {
      // Row scatter (owner rows or broadcast, as the single-CTA kernel's): this CTA's 128 x 256
      // half tile is staged in its own operand ring -- idle once the last
      // accumulator chunk arrived, since the leader's final commit covers every
      // pair MMA, and every TMA copy was consumed by one -- then each warp stores
      // whole rows as 512-byte coalesced segments.
      constexpr uint32_t LDS = BN + 4;  // padded row stride (floats): conflict-free float4 stores
      float* stage_tile = reinterpret_cast<float*>(smem);
      if (ok) {
        float* srow = stage_tile + (q * 32 + lane) * LDS + h * 128u;
#pragma unroll
        for (int j = 0; j < 128; j += 4)
          *reinterpret_cast<float4*>(srow + j) = make_float4(run[j], run[j + 1], run[j + 2], run[j + 3]);
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight epilogue warps of this CTA
      if (*(volatile uint32_t*)&aborted == 0u && scatter.bcast > 0u) {
        // Broadcast (the column-parallel product's gather): each row to every rank,
        // the peers first and this rank last, each warp starting at a different peer.
        const uint32_t ew = warp - 2u;
        for (uint32_t lr = ew; lr < PAIR_HALF; lr += 8u) {
          const uint32_t row = tile_m * PAIR_BM + rank * PAIR_HALF + lr;
          if (row >= m) break;
          const float* srow = stage_tile + lr * LDS;
          for (uint32_t i = 1; i <= scatter.bcast; ++i) {
            const uint32_t rk = (scatter.src_rank + (i == scatter.bcast ? 0u : 1u + (i - 1u + ew) % (scatter.bcast - 1u))) %
                                scatter.bcast;
            float* drow = scatter.dst[rk] + static_cast<uint64_t>(row) * scatter.ld + scatter.col_offset;
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
              const uint32_t cl = half * 128u + lane * 4u;
              const uint32_t col = tile_n * BN + cl;
              if (col + 4 <= n) {
                *reinterpret_cast<float4*>(drow + col) = *reinterpret_cast<const float4*>(srow + cl);
              } else {
                for (uint32_t t = 0; t < 4; ++t)
                  if (col + t < n) drow[col + t] = srow[cl + t];
              }
            }
          }
        }
      } else if (*(volatile uint32_t*)&aborted == 0u) {
        const uint32_t ew = warp - 2u;
        for (uint32_t lr = ew; lr < PAIR_HALF; lr += 8u) {
          const uint32_t row = tile_m * PAIR_BM + rank * PAIR_HALF + lr;
          if (row >= m) break;
          const uint32_t owner = row / scatter.rows_per_rank;
          const uint64_t slot_row =
              static_cast<uint64_t>(scatter.src_rank) * scatter.rows_per_rank + (row - owner * scatter.rows_per_rank);
          float* drow = scatter.dst[owner] + slot_row * scatter.ld;
          const float* srow = stage_tile + lr * LDS;
#pragma unroll
          for (uint32_t half = 0; half < 2; ++half) {
            const uint32_t cl = half * 128u + lane * 4u;  // column within the tile
            const uint32_t col = tile_n * BN + cl;
            if (col + 4 <= n) {
              *reinterpret_cast<float4*>(drow + col) = *reinterpret_cast<const float4*>(srow + cl);
            } else {
              for (uint32_t t = 0; t < 4; ++t)
                if (col + t < n) drow[col + t] = srow[cl + t];
            }
          }
        }
      }
    } else if (ok && num_kb > 0) {
      const uint32_t row = tile_m * PAIR_BM + rank * PAIR_HALF + q * 32 + lane;
      const uint32_t col0 = tile_n * BN + h * 128u;
      const bool vec_ok = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) &&
                          (residual == nullptr ||
                           ((ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(residual) & 15u) == 0)));
      if (row < m && col0 < n) {
        float* dst = c + static_cast<uint64_t>(row) * ldc + col0;
        const float* src = residual != nullptr ? residual + static_cast<uint64_t>(row) * ldr + col0 : nullptr;
        if (vec_ok && col0 + 128 <= n) {
#pragma unroll
          for (int j = 0; j < 128; j += 4) {
            float4 v = make_float4(run[j], run[j + 1], run[j + 2], run[j + 3]);
            if (src != nullptr) {
              const float4 r4 = *reinterpret_cast<const float4*>(src + j);
              v.x += r4.x;
              v.y += r4.y;
              v.z += r4.z;
              v.w += r4.w;
            }
            *reinterpret_cast<float4*>(dst + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 128; ++j)
            if (col0 + j < n) dst[j] = src != nullptr ? src[j] + run[j] : run[j];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Teardown: the leader's last commit (multicast) tells both CTAs that every
  // pair MMA finished; then both CTAs meet before the pair frees its TMEM, so
  // no CTA leaves while the leader's MMAs could still read its shared memory.
  if (threadIdx.x == 32) mbar_wait(&drain_bar, 0, err, kErrWaitDrain);
  __syncthreads();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ in-SM split, CTA pair
// The CTA-pair product with the TF32 split done inside the kernel, so no split
// pass runs and HBM carries each operand once, in fp32, straight from the
// caller's row-major A and B:
//   * each CTA's TMA loads its raw A rows [128][BK] (K-major, swizzled as the
//     MMA reads them) into the stage's A_hi slot, and its raw B rows
//     [BK][128] (B is N-major) unswizzled into the stage's B_raw slot, counting
//     the bytes on the CTA's own `raw_full` barrier; the TMA zero-fills every
//     element past m, n or k, so ragged edges need no padding;
//   * one converter warp per stage slot (each CTA), owning its slot's stages, split A
//     in place (A_hi <- tf32(a), A_lo <- tf32(a - A_hi), elementwise: both
//     slots share one layout) and transpose B from B_raw into the K-major
//     swizzled B_hi / B_lo slots, make the writes visible to the tensor core
//     (fence.proxy.async) and arrive on the leader's `full` barrier;
//   * the leader issues the same three tcgen05.mma.cta_group::2 per 8-deep k
//     step as sgemm3x_pair_kernel; accumulation and epilogue are unchanged.
// 16 warps: producer, MMA issuer, six converters, eight epilogue warps.  The
// epilogue's fp32 running sums need ~170 registers a thread, the other roles
// few: warpgroups 0-1 give registers back (setmaxnreg.dec) and 2-3 take them
// (setmaxnreg.inc).  The launcher checks that the launch's register budget
// covers the split, so the increase can always be granted.
constexpr int INSM_THREADS = 512;
constexpr uint32_t INSM_CONV_WARP0 = 2;
constexpr uint32_t INSM_CONV_WARPS = 6;
constexpr uint32_t INSM_EPI_WARP0 = 8;
constexpr uint32_t INSM_REGS_LOW = 80;    // warpgroups 0-1: producer, MMA, converters
constexpr uint32_t INSM_REGS_HIGH = 168;  // warpgroups 2-3: epilogue
static_assert(2 * 128 * INSM_REGS_LOW + 2 * 128 * INSM_REGS_HIGH <= 65536, "register split exceeds the SM file");

template <int BK>
struct InsmCfg {
  static constexpr uint32_t SWZ = BK * 4;
  static constexpr uint32_t A_BYTES = PAIR_HALF * BK * 4;
  static constexpr uint32_t B_BYTES = PAIR_HALF * BK * 4;
  static constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 3 * B_BYTES;  // A hi, A lo, B hi, B lo, B raw
  static constexpr uint32_t STAGES = (BK == 16) ? 5 : 2;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
};

// Byte offset of the 16-byte granule `g` of K-major row `r` in a tile whose
// rows are `swz` bytes long, under the TMA / UMMA swizzle of that span
// (granule index XOR the row bits above the span: 64 B: (r / 2) % 4, 128 B: r % 8).
template <uint32_t SWZ>
__device__ __forceinline__ uint32_t swizzled_offset(uint32_t r, uint32_t g) {
  if constexpr (SWZ == 128u) {
    return r * 128u + ((g ^ (r & 7u)) << 4);
  } else {
    return r * 64u + ((g ^ ((r >> 1) & 3u)) << 4);
  }
}

template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <int BK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(INSM_THREADS, 1)
    sgemm3x_insm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        float* __restrict__ c, uint32_t m, uint32_t n, uint64_t ldc, uint32_t num_kb,
                        uint32_t tiles_m, uint32_t tiles_n, const float* __restrict__ residual, uint64_t ldr,
                        unsigned int* __restrict__ err) {
  using Cfg = InsmCfg<BK>;
  constexpr uint32_t S = Cfg::STAGES;
  constexpr uint32_t KBC = KC / BK;
  constexpr uint32_t IDESC = umma_idesc_tf32(PAIR_BM, BN);
  constexpr uint16_t PAIR_MASK = 0x3;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t raw_full[S];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t aborted;
  __shared__ uint32_t issued_kb;
  __shared__ uint32_t converted_kb[INSM_CONV_WARPS];

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();  // 0 = leader
  const uint32_t num_chunks = (num_kb + KBC - 1) / KBC;

  const uint32_t t = blockIdx.x >> 1;
  const uint32_t per_group = GROUP_M * tiles_n;
  const uint32_t first_m = (t / per_group) * GROUP_M;
  const uint32_t group_rows = min(tiles_m - first_m, GROUP_M);
  const uint32_t tile_m = first_m + (t % per_group) % group_rows;
  const uint32_t tile_n = (t % per_group) / group_rows;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&full_bar[s], 2);  // one converter warp in each CTA
      mbar_init(&empty_bar[s], 1);
    }
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * NUM_EPI_WARPS);
    }
    mbar_init(&drain_bar, 1);
    aborted = 0;
    issued_kb = 0;
    for (uint32_t w = 0; w < INSM_CONV_WARPS; ++w) converted_kb[w] = w < S ? w : 0xFFFFFFFFu;  // next stage
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  // Register split: the same setmaxnreg instruction in every warp of a warpgroup,
  // before the warps branch into their roles.
  if (warp < INSM_EPI_WARP0) {
   setmaxnreg_dec<INSM_REGS_LOW>();
   if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (each CTA, its own barrier)
      const int row_a = static_cast<int>(tile_m * PAIR_BM + rank * PAIR_HALF);
      const int col_b = static_cast<int>(tile_n * BN + rank * PAIR_HALF);
      for (uint32_t kb = 0; kb < num_kb; ++kb) {
        const uint32_t s = kb % S;
        if (kb >= S) {
          if (!mbar_wait(&empty_bar[s], ((kb / S) - 1) & 1u, err, kErrWaitEmpty)) {
            atomicExch(&aborted, 1u);
            break;
          }
        }
        if (*(volatile uint32_t*)&aborted != 0u) break;
        uint8_t* st = smem + s * Cfg::STAGE_BYTES;
        const int kx = static_cast<int>(kb * BK);
        mbar_arrive_expect_tx(&raw_full[s], Cfg::A_BYTES + Cfg::B_BYTES);
        tma_load_2d(st, &tm_a, &raw_full[s], kx, row_a);
        tma_load_2d(st + 2 * Cfg::A_BYTES + 2 * Cfg::B_BYTES, &tm_b, &raw_full[s], col_b, kx);
        *(volatile uint32_t*)&issued_kb = kb + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader CTA only)
      for (uint32_t kb = 0; kb < num_kb; ++kb) {
        const uint32_t chunk = kb / KBC, in_chunk = kb % KBC;
        const uint32_t buf = chunk & 1u;
        if (in_chunk == 0 && chunk >= 2) {
          if (!mbar_wait(&acc_empty[buf], ((chunk >> 1) - 1) & 1u, err, kErrWaitAccum)) {
            atomicExch(&aborted, 1u);
            break;
          }
          tc_fence_after();
        }
        const uint32_t s = kb % S;
        if (!mbar_wait_cluster(&full_bar[s], (kb / S) & 1u, err, kErrWaitFull)) {
          atomicExch(&aborted, 1u);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const uint32_t base = smem_addr(smem + s * Cfg::STAGE_BYTES);
        const uint32_t a_hi = base, a_lo = base + Cfg::A_BYTES;
        const uint32_t b_hi = base + 2 * Cfg::A_BYTES, b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
        for (uint32_t kk = 0; kk < BK / 8; ++kk) {
          const uint32_t off = kk * 32;
          const uint64_t dah = umma_desc_kmajor(a_hi + off, Cfg::SWZ);
          const uint64_t dal = umma_desc_kmajor(a_lo + off, Cfg::SWZ);
          const uint64_t dbh = umma_desc_kmajor(b_hi + off, Cfg::SWZ);
          const uint64_t dbl = umma_desc_kmajor(b_lo + off, Cfg::SWZ);
          umma_tf32_pair(d_tmem, dal, dbh, IDESC, (in_chunk | kk) != 0u ? 1u : 0u);
          umma_tf32_pair(d_tmem, dah, dbl, IDESC, 1u);
          umma_tf32_pair(d_tmem, dah, dbh, IDESC, 1u);
        }
        umma_commit_pair_mc(&empty_bar[s], PAIR_MASK);
        if (in_chunk == KBC - 1 || kb == num_kb - 1) umma_commit_pair_mc(&acc_full[buf], PAIR_MASK);
      }
      umma_commit_pair_mc(&drain_bar, PAIR_MASK);
    }
  } else {
    // ---------------- converters (each CTA): split A in place, transpose + split B.
    // Converter warp w owns stage slot w (one warp per slot, S <= 6): it takes
    // stages kb = w, w + S, ..., so several stages convert at once, each warp's
    // proxy fence covers a whole stage, and a warp only ever waits for the next
    // phase of its own slot's barrier (a parity wait further ahead would pass
    // at once).
    const uint32_t cw = warp - INSM_CONV_WARP0;
    constexpr uint32_t A_ITEMS = Cfg::A_BYTES / 16;          // float4 granules of A
    constexpr uint32_t B_ITEMS = PAIR_HALF * (BK / 4);       // granules of B^T: (row n, k group g)
    static_assert(S <= INSM_CONV_WARPS, "one converter warp per stage slot");
    for (uint32_t kb = cw; cw < S && kb < num_kb; kb += S) {
      const uint32_t s = kb % S;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&raw_full[s], (kb / S) & 1u, err, kErrWaitFull));
      if (!ok || *(volatile uint32_t*)&aborted != 0u) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      uint8_t* st = smem + s * Cfg::STAGE_BYTES;
      float4* ahi = reinterpret_cast<float4*>(st);
      float4* alo = reinterpret_cast<float4*>(st + Cfg::A_BYTES);
      uint8_t* bhi = st + 2 * Cfg::A_BYTES;
      uint8_t* blo = bhi + Cfg::B_BYTES;
      const float* braw = reinterpret_cast<const float*>(blo + Cfg::B_BYTES);  // [BK][128]
      // Batches of 8 granules per lane: all loads of a batch are issued before any
      // store (the compiler cannot tell the staging reads from the operand writes).
      constexpr uint32_t BATCH = 8;
      static_assert((A_ITEMS / 32) % BATCH == 0 && (B_ITEMS / 32) % BATCH == 0, "batches tile the stage");
#pragma unroll 1
      for (uint32_t i0 = 0; i0 < A_ITEMS; i0 += 32 * BATCH) {
        float4 v[BATCH];
#pragma unroll
        for (uint32_t u = 0; u < BATCH; ++u) v[u] = ahi[i0 + lane + 32 * u];
#pragma unroll
        for (uint32_t u = 0; u < BATCH; ++u) {
          float4 h, l;
          h.x = to_tf32(v[u].x); h.y = to_tf32(v[u].y); h.z = to_tf32(v[u].z); h.w = to_tf32(v[u].w);
          l.x = to_tf32(v[u].x - h.x); l.y = to_tf32(v[u].y - h.y);
          l.z = to_tf32(v[u].z - h.z); l.w = to_tf32(v[u].w - h.w);
          ahi[i0 + lane + 32 * u] = h;
          alo[i0 + lane + 32 * u] = l;
        }
      }
#pragma unroll 1
      for (uint32_t j0 = 0; j0 < B_ITEMS; j0 += 32 * BATCH) {
        float4 v[BATCH];
#pragma unroll
        for (uint32_t u = 0; u < BATCH; ++u) {
          const uint32_t j = j0 + lane + 32 * u, r = j & (PAIR_HALF - 1), g = j / PAIR_HALF;
          const float* src = braw + (4u * g) * PAIR_HALF + r;
          v[u] = make_float4(src[0], src[PAIR_HALF], src[2 * PAIR_HALF], src[3 * PAIR_HALF]);
        }
#pragma unroll
        for (uint32_t u = 0; u < BATCH; ++u) {
          const uint32_t j = j0 + lane + 32 * u;
          float4 h, l;
          h.x = to_tf32(v[u].x); h.y = to_tf32(v[u].y); h.z = to_tf32(v[u].z); h.w = to_tf32(v[u].w);
          l.x = to_tf32(v[u].x - h.x); l.y = to_tf32(v[u].y - h.y);
          l.z = to_tf32(v[u].z - h.z); l.w = to_tf32(v[u].w - h.w);
          const uint32_t off = swizzled_offset<Cfg::SWZ>(j & (PAIR_HALF - 1), j / PAIR_HALF);
          *reinterpret_cast<float4*>(bhi + off) = h;
          *reinterpret_cast<float4*>(blo + off) = l;
        }
      }
      fence_proxy_async_smem();  // the generic-proxy writes, visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_cluster(&full_bar[s], 0);
        *(volatile uint32_t*)&converted_kb[cw] = kb + S;  // this warp's next stage
      }
    }
  }
  } else {
    setmaxnreg_inc<INSM_REGS_HIGH>();
    // ---------------- epilogue: warps 8..15 of both CTAs, each on its own TMEM half
    const uint32_t q = warp & 3u;
    const uint32_t h = (warp - INSM_EPI_WARP0) >> 2;
    const uint32_t lane_addr = (q * 32u) << 16;
    float run[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) run[j] = 0.f;
    bool ok = true;
    for (uint32_t ch = 0; ch < num_chunks; ++ch) {
      const uint32_t buf = ch & 1u;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (ch >> 1) & 1u, err, kErrWaitAccum));
      if (!ok) {
        if (lane == 0) atomicExch(&aborted, 1u);
        break;
      }
      tc_fence_after();
#pragma unroll
      for (uint32_t g = 0; g < 4; ++g) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + buf * BN + h * 128u + g * 32u, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) run[g * 32 + j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&acc_empty[buf], 0);
    }
    if (ok && num_kb > 0) {
      const uint32_t row = tile_m * PAIR_BM + rank * PAIR_HALF + q * 32 + lane;
      const uint32_t col0 = tile_n * BN + h * 128u;
      const bool vec_ok = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) &&
                          (residual == nullptr ||
                           ((ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(residual) & 15u) == 0)));
      if (row < m && col0 < n) {
        float* dst = c + static_cast<uint64_t>(row) * ldc + col0;
        const float* src = residual != nullptr ? residual + static_cast<uint64_t>(row) * ldr + col0 : nullptr;
        if (vec_ok && col0 + 128 <= n) {
#pragma unroll
          for (int j = 0; j < 128; j += 4) {
            float4 o = make_float4(run[j], run[j + 1], run[j + 2], run[j + 3]);
            if (src != nullptr) {
              const float4 r4 = *reinterpret_cast<const float4*>(src + j);
              o.x += r4.x;
              o.y += r4.y;
              o.z += r4.z;
              o.w += r4.w;
            }
            *reinterpret_cast<float4*>(dst + j) = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 128; ++j)
            if (col0 + j < n) dst[j] = src != nullptr ? src[j] + run[j] : run[j];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Teardown.  The leader's last commit (multicast) tells both CTAs that every
  // pair MMA finished.  A CTA that aborted first waits (bounded) for its own
  // TMA copies still in flight: those the converters never consumed.
  if (threadIdx.x == 32) mbar_wait(&drain_bar, 0, err, kErrWaitDrain);
  if (aborted && threadIdx.x == 0) {
    uint32_t done = converted_kb[0];  // the first stage no converter finished
    for (uint32_t w = 1; w < INSM_CONV_WARPS; ++w) done = min(done, converted_kb[w]);
    for (uint32_t kb = done; kb < issued_kb; ++kb)
      if (!mbar_wait(&raw_full[kb % S], (kb / S) & 1u, err, kErrWaitDrain)) break;
  }
  __syncthreads();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while the leader's MMAs could still read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
// K-major fp32 operand [rows x kp]; box = [bk x box_rows] with a bk*4-byte swizzle.
bool make_operand_map(CUtensorMap* map, const float* base, uint32_t rows, uint32_t kp, uint32_t bk,
                      uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {kp, rows};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kp) * sizeof(float)};
  const cuuint32_t box[2] = {bk, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle swz = (bk == 32) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BK>
// ksplit > 1 (single products only): K in that many ranges of whole
// accumulation chunks (splitk_ranges), one batch entry each; C then receives
// the ranges' partial products in slices of stride m * ldc (no residual), or,
// scattering, each range goes to its own slot of the owner rank.
cudaError_t launch_main(const float* ahi, const float* alo, const float* bhi, const float* blo, float* c,
                        uint64_t ldc, uint32_t m, uint32_t n, const SplitDims& d, unsigned int* err,
                        cudaStream_t stream, uint32_t batch, EntryStride stride_c, const float* residual = nullptr,
                        uint64_t ldr = 0, const RowScatter* scatter = nullptr, uint32_t ksplit = 1) {
  using Cfg = TileCfg<BK>;
  uint32_t kb_split = 0;
  if (ksplit > 1) {
    if (batch != 1 || residual != nullptr || (scatter != nullptr && scatter->bcast > 0)) return cudaErrorInvalidValue;
    const uint32_t kbc = KC / BK, chunks = (d.kp / BK + kbc - 1) / kbc;
    kb_split = (chunks + ksplit - 1) / ksplit * kbc;
    batch = (d.kp / BK + kb_split - 1) / kb_split;
    stride_c = EntryStride{static_cast<uint64_t>(m) * ldc, 0, 0};
  }
  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  const uint32_t rows_a = d.mp * batch, rows_b = d.np * batch;
  if (!make_operand_map(&m_ahi, ahi, rows_a, d.kp, BK, BM) || !make_operand_map(&m_alo, alo, rows_a, d.kp, BK, BM) ||
      !make_operand_map(&m_bhi, bhi, rows_b, d.kp, BK, BN) || !make_operand_map(&m_blo, blo, rows_b, d.kp, BK, BN))
    return cudaErrorInvalidValue;
  // Set on every launch: the attribute belongs to the current device's context.
  cudaError_t e = cudaFuncSetAttribute(sgemm3x_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg::SMEM_BYTES));
  if (e != cudaSuccess) return e;
  const uint32_t tiles_m = (m + BM - 1) / BM, tiles_n = (n + BN - 1) / BN;
  const uint64_t grid = static_cast<uint64_t>(tiles_m) * tiles_n * batch;
  if (grid > 0x7FFFFFFFull) return cudaErrorInvalidValue;
  RowScatter sc = scatter != nullptr ? *scatter : RowScatter{};
  if (sc.dst != nullptr && ((batch != 1 && kb_split == 0) || (sc.rows_per_rank == 0 && sc.bcast == 0) ||
                            sc.ld % 4 != 0 || ldc % 4 != 0 || sc.col_offset % 4 != 0 ||
                            (sc.bcast > 0 && sc.src_rank >= sc.bcast)))
    return cudaErrorInvalidValue;
  if (sc.dst != nullptr && kb_split != 0) sc.src_rank *= batch;  // range e lands in slot src_rank * ranges + e
  sgemm3x_kernel<BK><<<static_cast<uint32_t>(grid), NUM_THREADS, Cfg::SMEM_BYTES, stream>>>(
      m_ahi, m_alo, m_bhi, m_blo, c, m, n, ldc, d.kp / BK, tiles_m, tiles_n, kb_split ? 0u : d.mp,
      kb_split ? 0u : d.np, stride_c, residual, ldr, err, sc, kb_split);
  return cudaGetLastError();
}

// Row-major fp32 matrix [rows][ld] read in place by TMA: box = [box_x x box_y]
// (x innermost), `swz`-byte swizzle (0 = none).  Elements past cols / rows read as 0.
bool make_inplace_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint64_t ld,
                      uint32_t box_x, uint32_t box_y, uint32_t swz) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 4};
  const cuuint32_t box[2] = {box_x, box_y};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swz == 128u  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swz == 64u ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_NONE;
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// setmaxnreg.inc waits until the registers it asks for are free in the block's
// launch allocation (threads x registers per thread at launch): the kernel runs
// only when that allocation covers the whole split.
template <int BK>
bool insm_register_split_fits() {
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, sgemm3x_insm_kernel<BK>) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return static_cast<uint64_t>(fa.numRegs) * INSM_THREADS >=
         2ull * 128 * INSM_REGS_LOW + 2ull * 128 * INSM_REGS_HIGH;
}

template <int BK>
cudaError_t launch_insm(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                        uint32_t m, uint32_t n, uint32_t k, unsigned int* err, cudaStream_t stream,
                        const float* residual, uint64_t ldr) {
  using Cfg = InsmCfg<BK>;
  CUtensorMap m_a, m_b;
  if (!make_inplace_map(&m_a, a, k, m, lda, BK, PAIR_HALF, Cfg::SWZ) ||
      !make_inplace_map(&m_b, b, n, k, ldb, PAIR_HALF, BK, 0))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(sgemm3x_insm_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg::SMEM_BYTES));
  if (e != cudaSuccess) return e;
  if (!insm_register_split_fits<BK>()) return cudaErrorInvalidConfiguration;
  const uint32_t tiles_m = (m + PAIR_BM - 1) / PAIR_BM, tiles_n = (n + BN - 1) / BN;
  const uint64_t grid = 2ull * tiles_m * tiles_n;
  if (grid > 0x7FFFFFFFull) return cudaErrorInvalidValue;
  const uint32_t num_kb = (k + BK - 1) / BK;
  sgemm3x_insm_kernel<BK><<<static_cast<uint32_t>(grid), INSM_THREADS, Cfg::SMEM_BYTES, stream>>>(
      m_a, m_b, c, m, n, ldc, num_kb, tiles_m, tiles_n, residual, ldr, err);
  return cudaGetLastError();
}

template <int BK>
cudaError_t launch_pair(const float* ahi, const float* alo, const float* bhi, const float* blo, float* c,
                        uint64_t ldc, uint32_t m, uint32_t n, const SplitDims& d, unsigned int* err,
                        cudaStream_t stream, uint32_t batch, EntryStride stride_c, const float* residual = nullptr,
                        uint64_t ldr = 0, const RowScatter* scatter = nullptr) {
  using Cfg = PairCfg<BK>;
  if (d.mp % PAIR_BM != 0) return cudaErrorInvalidValue;
  const RowScatter sc = scatter != nullptr ? *scatter : RowScatter{};
  if (sc.dst != nullptr && (batch != 1 || (sc.rows_per_rank == 0 && sc.bcast == 0) || sc.ld % 4 != 0 ||
                            ldc % 4 != 0 || sc.col_offset % 4 != 0 || (sc.bcast > 0 && sc.src_rank >= sc.bcast) ||
                            residual != nullptr))
    return cudaErrorInvalidValue;
  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  const uint32_t rows_a = d.mp * batch, rows_b = d.np * batch;
  if (!make_operand_map(&m_ahi, ahi, rows_a, d.kp, BK, PAIR_HALF) ||
      !make_operand_map(&m_alo, alo, rows_a, d.kp, BK, PAIR_HALF) ||
      !make_operand_map(&m_bhi, bhi, rows_b, d.kp, BK, PAIR_HALF) ||
      !make_operand_map(&m_blo, blo, rows_b, d.kp, BK, PAIR_HALF))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(sgemm3x_pair_kernel<BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg::SMEM_BYTES));
  if (e != cudaSuccess) return e;
  const uint32_t tiles_m = (m + PAIR_BM - 1) / PAIR_BM, tiles_n = (n + BN - 1) / BN;
  const uint64_t grid = 2ull * tiles_m * tiles_n * batch;
  if (grid > 0x7FFFFFFFull) return cudaErrorInvalidValue;
  sgemm3x_pair_kernel<BK><<<static_cast<uint32_t>(grid), NUM_THREADS, Cfg::SMEM_BYTES, stream>>>(
      m_ahi, m_alo, m_bhi, m_blo, c, m, n, ldc, d.kp / BK, tiles_m, tiles_n, d.mp, d.np, stride_c, residual, ldr,
      err, sc);
  return cudaGetLastError();
}

cudaError_t launch_config(int cfg, const float* ahi, const float* alo, const float* bhi, const float* blo, float* c,
                          uint64_t ldc, uint32_t m, uint32_t n, const SplitDims& d, unsigned int* err,
                          cudaStream_t stream, uint32_t batch, EntryStride stride_c, const float* residual = nullptr,
                          uint64_t ldr = 0, const RowScatter* scatter = nullptr, uint32_t ksplit = 1) {
  // the CTA-pair kernels have no split-K form (their row scatter is checked in launch_pair)
  if (ksplit > 1 && cfg != kTcSingle16 && cfg != kTcSingle32) return cudaErrorInvalidValue;
  switch (cfg) {
    case kTcSingle16: return launch_main<16>(ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, batch, stride_c, residual, ldr, scatter, ksplit);
    case kTcSingle32: return launch_main<32>(ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, batch, stride_c, residual, ldr, scatter, ksplit);
    case kTcPair16: return launch_pair<16>(ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, batch, stride_c, residual, ldr, scatter);
    case kTcPair32: return launch_pair<32>(ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, batch, stride_c, residual, ldr, scatter);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// ------------------------------------------------------------------ pre-split weights
// A weight operand B [k][n] that many products reuse is split once into the
// K-major hi/lo layout; later products only split their activation operand.
uint64_t split_b_elems(uint32_t n, uint32_t k) {
  const SplitDims d = split_dims(1, n, k);
  return static_cast<uint64_t>(d.np) * d.kp;
}

cudaError_t sgemm_tc_split_b(const float* b, uint64_t ldb, uint32_t k, uint32_t n, float* bhi, float* blo,
                             cudaStream_t stream) {
  if (k == 0 || n == 0) return cudaSuccess;
  const SplitDims d = split_dims(1, n, k);
  split_transpose_kernel<<<dim3(d.np / 32, d.kp / 32, 1), 256, 0, stream>>>(b, ldb, k, n, bhi, blo, d.kp, d.np, EntryStride{});
  return cudaGetLastError();
}

uint64_t sgemm_tc_a_scratch_bytes(uint32_t m, uint32_t k) {
  const SplitDims d = split_dims(m, 1, k);
  return 2ull * sizeof(float) * d.mp * d.kp;
}

namespace {

// C = R + (P_0 + P_1 + ... ) over the K ranges' partial products P_j
// (ranges * m * n floats, range-major), in range order; R optional.  Rows step
// by blockIdx.y, columns by the x threads (coalesced; no index division).
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ p, uint32_t ranges, uint32_t m,
                                                            uint32_t n, const float* __restrict__ residual,
                                                            uint64_t ldr, float* __restrict__ c, uint64_t ldc) {
  const uint64_t total = static_cast<uint64_t>(m) * n;
  for (uint32_t row = blockIdx.y; row < m; row += gridDim.y) {
    const float* pr = p + static_cast<uint64_t>(row) * n;
    for (uint32_t col = blockIdx.x * 256u + threadIdx.x; col < n; col += gridDim.x * 256u) {
      float s = pr[col];
      for (uint32_t j = 1; j < ranges; ++j) s += pr[j * total + col];
      if (residual != nullptr) s = residual[static_cast<uint64_t>(row) * ldr + col] + s;
      c[static_cast<uint64_t>(row) * ldc + col] = s;
    }
  }
}

// The product on the prepared split operands, split K or not (see SplitK).
cudaError_t run_split_k(int cfg, const float* ahi, const float* alo, const float* bhi, const float* blo, float* c,
                        uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, const SplitDims& d, unsigned int* err,
                        cudaStream_t stream, const float* residual, uint64_t ldr, const RowScatter* scatter,
                        const SplitK* splitk) {
  const uint32_t ranges = splitk != nullptr ? sgemm_tc_k_ranges(k, splitk->ranges) : 1u;
  if (ranges <= 1)
    return launch_config(cfg, ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, 1, EntryStride{}, residual, ldr,
                         scatter);
  if (scatter != nullptr && scatter->dst != nullptr) {
    if (residual != nullptr) return cudaErrorInvalidValue;
    return launch_config(cfg, ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, 1, EntryStride{}, nullptr, 0,
                         scatter, splitk->ranges);
  }
  if (splitk->partial == nullptr) return cudaErrorInvalidValue;
  cudaError_t e = launch_config(cfg, ahi, alo, bhi, blo, splitk->partial, n, m, n, d, err, stream, 1, EntryStride{},
                                nullptr, 0, nullptr, splitk->ranges);
  if (e != cudaSuccess) return e;
  const uint32_t bx = std::min<uint32_t>((n + 255) / 256, 8u);
  const uint32_t by = std::min<uint32_t>(m, std::max<uint32_t>(1u, 148u * 16u / bx));
  splitk_reduce_kernel<<<dim3(bx, by), 256, 0, stream>>>(splitk->partial, ranges, m, n, residual, ldr, c, ldc);
  return cudaGetLastError();
}

}  // namespace

uint32_t sgemm_tc_k_ranges(uint32_t k, uint32_t ranges) {
  if (ranges <= 1 || k == 0) return 1;
  const uint32_t kp = round_up(k, KPAD), chunks = (kp + KC - 1) / KC;
  const uint32_t per = (chunks + ranges - 1) / ranges;
  return (chunks + per - 1) / per;
}

uint32_t sgemm_tc_pick_k_ranges(uint32_t m, uint32_t n, uint32_t k) {
  constexpr uint32_t kSms = 148;
  const uint64_t tiles = static_cast<uint64_t>((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  if (tiles == 0 || tiles >= kSms || k == 0) return 1;
  const uint32_t chunks = (round_up(k, KPAD) + KC - 1) / KC;
  uint32_t best = 1;
  double best_score = -1.0;
  for (uint32_t s = 1; s <= 8 && (s == 1 || chunks / s >= 2); ++s) {
    const uint64_t ctas = tiles * sgemm_tc_k_ranges(k, s);
    const double fill = static_cast<double>(ctas) / (static_cast<double>((ctas + kSms - 1) / kSms) * kSms);
    const double score = fill - 0.03 * (s - 1);  // each range adds a prologue, an epilogue and partial traffic
    if (score > best_score + 1e-9) {
      best_score = score;
      best = s;
    }
  }
  return best;
}

cudaError_t sgemm_tc_presplit(const float* a, uint64_t lda, const float* bhi, const float* blo, float* c,
                              uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, void* a_scratch, unsigned int* err,
                              cudaStream_t stream, const float* residual, uint64_t ldr, int cfg,
                              const RowScatter* scatter, const SplitK* splitk) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(a_scratch) & 1023u) != 0) return cudaErrorInvalidValue;
  const SplitDims d = split_dims(m, n, k);
  float* ahi = static_cast<float*>(a_scratch);
  float* alo = ahi + static_cast<uint64_t>(d.mp) * d.kp;
  const uint64_t groups = static_cast<uint64_t>(d.mp) * (d.kp / 4);
  const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((groups + 255) / 256, 148ull * 16));
  split_rows_kernel<<<dim3(blocks, 1), 256, 0, stream>>>(a, lda, m, k, ahi, alo, d.mp, d.kp, EntryStride{});
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return run_split_k(cfg, ahi, alo, bhi, blo, c, ldc, m, n, k, d, err, stream, residual, ldr, scatter, splitk);
}

// Both operands already split: A hi/lo in the [Mp][Kp] layout of split_dims
// (written by its producer), B as from sgemm_tc_split_b.
cudaError_t sgemm_tc_presplit_ab(const float* ahi, const float* alo, const float* bhi, const float* blo, float* c,
                                 uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, unsigned int* err,
                                 cudaStream_t stream, const float* residual, uint64_t ldr, int cfg,
                                 const SplitK* splitk) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  const SplitDims d = split_dims(m, n, k);
  return run_split_k(cfg, ahi, alo, bhi, blo, c, ldc, m, n, k, d, err, stream, residual, ldr, nullptr, splitk);
}

// A operand already in the split layout (hi/lo, [count][Mp][Kp], zero padded),
// written by its producer; only B is split here (into b_scratch).
cudaError_t sgemm_tc_presplit_a(const float* ahi, const float* alo, const float* b, uint64_t ldb, float* c,
                                uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, void* b_scratch, unsigned int* err,
                                cudaStream_t stream, const GemmBatch* batch, int cfg) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(b_scratch) & 1023u) != 0) return cudaErrorInvalidValue;
  const GemmBatch one{};
  const GemmBatch& bt = batch != nullptr ? *batch : one;
  if (bt.count == 0) return cudaSuccess;
  if (bt.count > 65535u) return cudaErrorInvalidValue;
  const SplitDims d = split_dims(m, n, k);
  const uint64_t b_elems = static_cast<uint64_t>(d.np) * d.kp * bt.count;
  float* bhi = static_cast<float*>(b_scratch);
  float* blo = bhi + b_elems;
  cudaError_t e;
  if (bt.b_trans) {
    const uint64_t bgroups = static_cast<uint64_t>(d.np) * (d.kp / 4);
    const uint32_t bblocks = static_cast<uint32_t>(std::min<uint64_t>((bgroups + 255) / 256, 148ull * 16));
    split_rows_kernel<<<dim3(bblocks, bt.count), 256, 0, stream>>>(b, ldb, n, k, bhi, blo, d.np, d.kp, bt.sb());
  } else {
    split_transpose_kernel<<<dim3(d.np / 32, d.kp / 32, bt.count), 256, 0, stream>>>(b, ldb, k, n, bhi, blo, d.kp,
                                                                                     d.np, bt.sb());
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_config(cfg, ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, bt.count, bt.sc());
}

// ------------------------------------------------------------------ no-allocation variant
// Scratch for oct_b200_sgemm_device_noalloc: some callers cannot call
// cudaMalloc at all (for example a serving process whose fixed memory plan
// hands all of HBM to its own pool, or code that must not trigger the device
// synchronisation an allocation implies).  For them the TF32 split buffers and
// the kernel status word live in this fixed array instead of in a handle.  It
// is reserved on every GPU that loads the library, until the process exits.
constexpr uint64_t kNoAllocSplitBytes = 64ull << 20;  // hi/lo copies of A and B^T
constexpr uint64_t kNoAllocStatusBytes = 1024;        // status word, then padding to 1 KiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocStatusBytes + kNoAllocSplitBytes + 1024];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_base[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  (The array's name in host code is only a host-side stand-in.)
// The address belongs to the device's primary context, the one the CUDA
// runtime API uses; after a cudaDeviceReset the cached value would be stale,
// which the header documents as a limit of this entry point.
cudaError_t noalloc_base(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_base[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_base[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_base[dev];
  return cudaSuccess;
}
}  // namespace

SplitDims split_dims(uint32_t m, uint32_t n, uint32_t k) {
  // M is padded to the CTA-pair tile (256) so both kernels read one layout.
  return SplitDims{round_up(m, PAIR_BM), round_up(n, BN), round_up(k, KPAD)};
}

uint64_t sgemm_tc_scratch_bytes(uint32_t m, uint32_t n, uint32_t k, uint32_t batch) {
  const SplitDims d = split_dims(m, n, k);
  return 2ull * sizeof(float) * batch *
         (static_cast<uint64_t>(d.mp) * d.kp + static_cast<uint64_t>(d.np) * d.kp);
}

bool sgemm_insm_eligible(const float* a, uint64_t lda, const float* b, uint64_t ldb, uint32_t m, uint32_t n,
                         uint32_t k, const GemmBatch* batch) {
  if (batch != nullptr && (batch->count > 1 || batch->b_trans)) return false;
  static const bool regs_ok = insm_register_split_fits<16>() && insm_register_split_fits<32>();
  return regs_ok && m > 0 && n > 0 && k > 0 && lda % 4 == 0 && ldb % 4 == 0 &&
         (reinterpret_cast<uintptr_t>(a) & 15u) == 0 && (reinterpret_cast<uintptr_t>(b) & 15u) == 0 &&
         lda < (1ull << 37) && ldb < (1ull << 37);
}

cudaError_t sgemm_tc_insm(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                          uint32_t m, uint32_t n, uint32_t k, unsigned int* err, int bk, cudaStream_t stream,
                          const SgemmEvents* events, const float* residual, uint64_t ldr) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if (!sgemm_insm_eligible(a, lda, b, ldb, m, n, k, nullptr)) return cudaErrorInvalidValue;
  if (events != nullptr && events->split_begin != nullptr) cudaEventRecord(events->split_begin, stream);
  if (events != nullptr && events->main_begin != nullptr) cudaEventRecord(events->main_begin, stream);
  const cudaError_t e = bk == kTcInsm32 ? launch_insm<32>(a, lda, b, ldb, c, ldc, m, n, k, err, stream, residual, ldr)
                                        : launch_insm<16>(a, lda, b, ldb, c, ldc, m, n, k, err, stream, residual, ldr);
  if (events != nullptr && events->main_end != nullptr) cudaEventRecord(events->main_end, stream);
  return e;
}

cudaError_t sgemm_tc(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                     uint32_t m, uint32_t n, uint32_t k, void* scratch, unsigned int* err, int bk,
                     cudaStream_t stream, const SgemmEvents* events, const GemmBatch* batch) {
  if (m == 0 || n == 0 || k == 0) return cudaSuccess;
  if (bk == kTcInsm16 || bk == kTcInsm32) {
    if (sgemm_insm_eligible(a, lda, b, ldb, m, n, k, batch))
      return sgemm_tc_insm(a, lda, b, ldb, c, ldc, m, n, k, err, bk, stream, events);
    bk = bk == kTcInsm32 ? kTcPair32 : kTcPair16;  // operands TMA cannot read in place: split pass
  }
  if (bk != kTcSingle16 && bk != kTcSingle32 && bk != kTcPair16 && bk != kTcPair32) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(scratch) & 1023u) != 0) return cudaErrorInvalidValue;
  const GemmBatch one{};
  const GemmBatch& bt = batch != nullptr ? *batch : one;
  if (bt.count == 0) return cudaSuccess;
  if (bt.count > 65535u) return cudaErrorInvalidValue;
  const SplitDims d = split_dims(m, n, k);
  const uint64_t a_elems = static_cast<uint64_t>(d.mp) * d.kp * bt.count;
  const uint64_t b_elems = static_cast<uint64_t>(d.np) * d.kp * bt.count;
  if (a_elems > 0x7FFFFFFFull * 4 || b_elems > 0x7FFFFFFFull * 4) return cudaErrorInvalidValue;
  float* ahi = static_cast<float*>(scratch);
  float* alo = ahi + a_elems;
  float* bhi = alo + a_elems;
  float* blo = bhi + b_elems;

  if (events != nullptr && events->split_begin != nullptr) cudaEventRecord(events->split_begin, stream);
  const uint64_t groups = static_cast<uint64_t>(d.mp) * (d.kp / 4);
  const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((groups + 255) / 256, 148ull * 16));
  split_rows_kernel<<<dim3(blocks, bt.count), 256, 0, stream>>>(a, lda, m, k, ahi, alo, d.mp, d.kp, bt.sa());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (bt.b_trans) {
    // B is [n][k]: already K-major, split it like A.
    const uint64_t bgroups = static_cast<uint64_t>(d.np) * (d.kp / 4);
    const uint32_t bblocks = static_cast<uint32_t>(std::min<uint64_t>((bgroups + 255) / 256, 148ull * 16));
    split_rows_kernel<<<dim3(bblocks, bt.count), 256, 0, stream>>>(b, ldb, n, k, bhi, blo, d.np, d.kp, bt.sb());
  } else {
    split_transpose_kernel<<<dim3(d.np / 32, d.kp / 32, bt.count), 256, 0, stream>>>(b, ldb, k, n, bhi, blo, d.kp,
                                                                                     d.np, bt.sb());
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (events != nullptr && events->main_begin != nullptr) cudaEventRecord(events->main_begin, stream);
  e = launch_config(bk, ahi, alo, bhi, blo, c, ldc, m, n, d, err, stream, bt.count, bt.sc());
  if (events != nullptr && events->main_end != nullptr) cudaEventRecord(events->main_end, stream);
  return e;
}

}  // namespace oct

// C = A * B on device pointers with no allocation of any kind; see the header.
extern "C" int oct_b200_sgemm_device_noalloc(const float* d_a, uint64_t lda, const float* d_b, uint64_t ldb,
                                             float* d_c, uint64_t ldc, uint32_t m, uint32_t n, uint32_t k,
                                             void* stream, int* out_detail_code) {
  using namespace oct;
  auto fail = [&](int rc, int detail) {
    if (out_detail_code != nullptr) *out_detail_code = detail;
    return rc;
  };
  try {
    if (out_detail_code != nullptr) *out_detail_code = 0;
    if (d_a == nullptr || d_b == nullptr || d_c == nullptr || lda < k || ldb < n || ldc < n)
      return fail(PROM_ERROR, OCT_B200_DETAIL_INVALID_ARGUMENT);
    if (m == 0 || n == 0 || k == 0) return PROM_OK;
    if (sgemm_tc_scratch_bytes(m, n, k) > kNoAllocSplitBytes)
      return fail(PROM_ERROR, OCT_B200_DETAIL_NOALLOC_TOO_LARGE);
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10) {
      (void)cudaGetLastError();
      return fail(PROM_ERROR, PROM_DETAIL_CAPABILITY_MISMATCH);
    }
    unsigned char* base = nullptr;
    if (noalloc_base(dev, &base) != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(PROM_ERROR, OCT_B200_DETAIL_CUDA_ERROR);
    }
    unsigned int* status = reinterpret_cast<unsigned int*>(base);
    void* split = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(base) + kNoAllocStatusBytes + 1023) &
                                          ~uintptr_t(1023));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The array keeps the previous call's contents: the status word must start
    // at zero; the split buffers (padding included) are fully rewritten.
    cudaError_t e = cudaMemsetAsync(status, 0, sizeof(unsigned int), s);
    if (e == cudaSuccess) e = sgemm_tc(d_a, lda, d_b, ldb, d_c, ldc, m, n, k, split, status, 16, s);
    unsigned int host_status = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&host_status, status, sizeof(host_status), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail(PROM_ERROR, OCT_B200_DETAIL_CUDA_ERROR);
    }
    if (host_status != 0) return fail(PROM_ERROR, OCT_B200_DETAIL_DEVICE_TIMEOUT);
    return PROM_OK;
  } catch (...) {
    return fail(PROM_INTERNAL_ERROR, OCT_B200_DETAIL_CUDA_ERROR);
  }
}
