// reduce.cu -- fused row reductions and RMSNorm over fp32 rows.
//
// Operations (Oct's reduction ABI, internal/prometheus/native/reactor_api.h:377-381):
//   SUM      out[r] = sum_c x[r, c]
//   MAX      out[r] = max_c x[r, c]
//   SOFTMAX  out[r, c] = exp(x[r, c] - max_r) / sum_c exp(x[r, c] - max_r)
// and RMSNorm  out[r, c] = x[r, c] * (1 / sqrt(mean_c x[r, c]^2 + eps)) * w[c]
// (internal/prometheus/zimage/canonical_contract.go:91-105).
//
// Numerics follow the fp64 CPU reference `prom_reduction_cpu_reference`
// (internal/prometheus/native/reactor_vulkan_fused_reduction.c:996-1036): sums
// (of x, of exp, of x^2) accumulate in double, max is exact, the softmax
// quotient is formed in double and rounded once.  exp itself is CUDA's fp32
// `expf` (a few ulp), well inside the tolerance.
//
// Data movement: rows stream HBM -> shared memory with `cp.async.bulk` (the TMA
// engine's untiled copy) into rings of slots, one mbarrier per slot, so several
// rows are in flight while the current one is reduced out of shared memory.  A
// row is read from HBM exactly once; softmax and RMSNorm take all their passes
// over the shared-memory copy.
//   W <= 2048 : per-warp pipelines -- each warp owns its rows and its ring and
//               reduces with warp shuffles only (no CTA-wide barrier);
//   W <= 8192 : the whole 256-thread CTA owns a row, shuffle + shared reduction
//               (more warps per SM to hide the longer per-row arithmetic).
// Rows whose address or width is not 16-byte granular (or wider than 8192)
// take a plain-load fallback kernel with the same arithmetic.
#include <cuda_runtime.h>

#include <cfloat>
#include <algorithm>
#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace oct {
namespace {

constexpr int THREADS = 256;
constexpr uint32_t SLOT_BUDGET_BYTES = 64 * 1024;  // ring size per CTA
constexpr uint32_t BULK_MAX_WIDTH = 8192;

// Launches a one-wave ring kernel with programmatic stream serialization: it may
// be scheduled while the previous kernel in the stream drains, and it waits
// (griddep_wait) for that kernel to complete before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, uint32_t smem, cudaStream_t stream,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

enum Op : int { kSum = 1, kMax = 2, kSoftmax = 3, kRms = 4 };

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Row-group reduction: TPR == 32 -> warp only; TPR == 256 -> whole CTA.
template <int TPR>
__device__ __forceinline__ double group_sum_d(double v, double* scratch) {
  v = warp_sum_d(v);
  if constexpr (TPR == 32) {
    return v;
  } else {
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[w] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) t += scratch[i];
    return t;
  }
}
template <int TPR>
__device__ __forceinline__ float group_max_f(float v, float* scratch) {
  v = warp_max_f(v);
  if constexpr (TPR == 32) {
    return v;
  } else {
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[w] = v;
    __syncthreads();
    float t = scratch[0];
#pragma unroll
    for (int i = 1; i < THREADS / 32; ++i) t = fmaxf(t, scratch[i]);
    return t;
  }
}

__device__ __forceinline__ void note_nonfinite(float v, uint64_t flat, uint64_t& first) {
  if (!isfinite(v) && flat < first) first = flat;
}

// Per-float4 pieces of the row arithmetic, shared by every kernel so that they
// evaluate (and contract) the same expressions.
__device__ __forceinline__ float max4(float4 x) { return fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w)); }
__device__ __forceinline__ float4 exp4(float4 x, float mx) {
  return make_float4(expf(x.x - mx), expf(x.y - mx), expf(x.z - mx), expf(x.w - mx));
}
__device__ __forceinline__ float hsum4(float4 x) { return (x.x + x.y) + (x.z + x.w); }
__device__ __forceinline__ double sq4(float4 x) {
  // four non-negative squares summed in fp32, accumulated in binary64
  return static_cast<double>((x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w));
}

// Processes one row held in shared memory.  `lane` / TPR index the threads of
// the row group; out_row points at this row's output (softmax / RMSNorm) or
// at out[r] (sum / max).
template <int OP, int TPR>
__device__ __forceinline__ float process_row(float* srow, uint32_t w, uint32_t lane, uint64_t row,
                                            float* __restrict__ out, const float* __restrict__ weight, float eps,
                                            double* dscratch, float* fscratch, uint64_t& first_bad) {
  const uint32_t nv = w / 4;
  float4* v4 = reinterpret_cast<float4*>(srow);
  if constexpr (OP == kSum) {
    // four independent binary64 chains (one per float4 lane), joined at the end:
    // the same exact sums as one chain wherever binary64 holds the sum exactly
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 x = v4[i];
      s0 += static_cast<double>(x.x); s1 += static_cast<double>(x.y);
      s2 += static_cast<double>(x.z); s3 += static_cast<double>(x.w);
      if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) {
        note_nonfinite(x.x, row * w + 4 * i, first_bad); note_nonfinite(x.y, row * w + 4 * i + 1, first_bad);
        note_nonfinite(x.z, row * w + 4 * i + 2, first_bad); note_nonfinite(x.w, row * w + 4 * i + 3, first_bad);
      }
    }
    const double s = group_sum_d<TPR>((s0 + s1) + (s2 + s3), dscratch);
    if (lane == 0) out[row] = static_cast<float>(s);
    return 0.f;
  } else if constexpr (OP == kMax) {
    float mx = -FLT_MAX;
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 x = v4[i];
      mx = fmaxf(mx, max4(x));
      if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) {
        note_nonfinite(x.x, row * w + 4 * i, first_bad); note_nonfinite(x.y, row * w + 4 * i + 1, first_bad);
        note_nonfinite(x.z, row * w + 4 * i + 2, first_bad); note_nonfinite(x.w, row * w + 4 * i + 3, first_bad);
      }
    }
    mx = group_max_f<TPR>(mx, fscratch);
    if (lane == 0) out[row] = mx;
    return 0.f;
  } else if constexpr (OP == kSoftmax) {
    float mx = -FLT_MAX;
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 x = v4[i];
      mx = fmaxf(mx, max4(x));
      if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) {
        note_nonfinite(x.x, row * w + 4 * i, first_bad); note_nonfinite(x.y, row * w + 4 * i + 1, first_bad);
        note_nonfinite(x.z, row * w + 4 * i + 2, first_bad); note_nonfinite(x.w, row * w + 4 * i + 3, first_bad);
      }
    }
    mx = group_max_f<TPR>(mx, fscratch);
    // exp(x - max) in fp32; each float4's four positive terms are summed in
    // fp32 (a few ulp) and the row sum accumulates those partials in binary64.
    double s = 0.0;
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 x = exp4(v4[i], mx);
      s += static_cast<double>(hsum4(x));
      v4[i] = x;  // keep exp(x - max) for the normalising pass
    }
    s = group_sum_d<TPR>(s, dscratch);
    const float inv = static_cast<float>(1.0 / s);  // one rounding; the product adds one more
    float4* o4 = reinterpret_cast<float4*>(out + row * w);
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 e = v4[i];
      __stcs(o4 + i, make_float4(e.x * inv, e.y * inv, e.z * inv, e.w * inv));
    }
    return 0.f;
  } else {  // kRms
    double ss = 0.0;
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 x = v4[i];
      ss += sq4(x);
      if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) {
        note_nonfinite(x.x, row * w + 4 * i, first_bad); note_nonfinite(x.y, row * w + 4 * i + 1, first_bad);
        note_nonfinite(x.z, row * w + 4 * i + 2, first_bad); note_nonfinite(x.w, row * w + 4 * i + 3, first_bad);
      }
    }
    ss = group_sum_d<TPR>(ss, dscratch);
    const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(w) + static_cast<double>(eps)));
    float4* o4 = reinterpret_cast<float4*>(out + row * w);
    const float4* w4 = reinterpret_cast<const float4*>(weight);
    for (uint32_t i = lane; i < nv; i += TPR) {
      const float4 x = v4[i];
      const float4 g = __ldg(w4 + i);
      __stcs(o4 + i, make_float4(x.x * inv * g.x, x.y * inv * g.y, x.z * inv * g.z, x.w * inv * g.w));
    }
    return inv;
  }
}

// Bulk-fed kernel.  TPR threads per row; rows_per_batch = THREADS / TPR.
// Rows are `stride` floats apart; when stride == w a batch is one contiguous copy.
template <int OP, int TPR>
__global__ void __launch_bounds__(THREADS) row_bulk_kernel(const float* __restrict__ in, uint64_t stride,
                                                           float* __restrict__ out, float* __restrict__ inv_rms,
                                                           const float* __restrict__ weight, float eps,
                                                           uint32_t rows, uint32_t w, uint32_t ns,
                                                           unsigned long long* __restrict__ nonfinite,
                                                           unsigned int* __restrict__ err) {
  constexpr uint32_t RPB = THREADS / TPR;  // rows per batch
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);
  __shared__ __align__(8) uint64_t bars[8];
  __shared__ double dscratch[RPB][THREADS / 32];
  __shared__ float fscratch[RPB][THREADS / 32];
  __shared__ uint32_t abort_flag;

  const uint32_t batch_floats = RPB * w;
  const uint32_t num_batches = (rows + RPB - 1) / RPB;
  const bool contiguous = (stride == w);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < ns; ++s) mbar_init(&bars[s], 1);
    abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncthreads();
  // The rows (and the output) may belong to the previous kernel in the stream:
  // wait for it to complete before the first global access.  No early trigger:
  // work after this kernel is released at its completion, as without the
  // launch attribute.
  griddep_wait();

  auto issue = [&](uint32_t batch, uint32_t slot) {
    const uint32_t r0 = batch * RPB;
    const uint32_t nr = min(RPB, rows - r0);
    float* dst = ring + slot * batch_floats;
    mbar_arrive_expect_tx(&bars[slot], nr * w * 4u);
    if (contiguous) {
      bulk_load(dst, in + static_cast<uint64_t>(r0) * w, nr * w * 4u, &bars[slot]);
    } else {
      for (uint32_t i = 0; i < nr; ++i)
        bulk_load(dst + i * w, in + static_cast<uint64_t>(r0 + i) * stride, w * 4u, &bars[slot]);
    }
  };

  // Prologue: fill the ring with this CTA's first `ns` batches.  Thread 0
  // counts copies issued per slot so an aborted CTA can drain them.
  uint32_t issued[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < ns; ++s) {
      const uint32_t b = blockIdx.x + s * gridDim.x;
      if (b >= num_batches) break;
      issue(b, s);
      issued[s] += 1;
    }
  }

  uint64_t first_bad = ~0ull;
  const uint32_t grp = threadIdx.x / TPR, lane = threadIdx.x % TPR;
  for (uint32_t j = 0;; ++j) {
    const uint32_t b = blockIdx.x + j * gridDim.x;
    if (b >= num_batches) break;
    const uint32_t slot = j % ns;
    const bool ok = mbar_wait(&bars[slot], (j / ns) & 1u, err, kErrWaitRow);
    if (!ok) abort_flag = 1;
    __syncthreads();
    if (abort_flag) break;
    const uint32_t r = b * RPB + grp;
    if (r < rows) {
      float* srow = ring + slot * batch_floats + grp * w;
      const float inv = process_row<OP, TPR>(srow, w, lane, r, out, weight, eps, dscratch[grp], fscratch[grp],
                                             first_bad);
      if constexpr (OP == kRms) {
        if (lane == 0 && inv_rms != nullptr) inv_rms[r] = inv;
      }
    }
    __syncthreads();  // every thread is done with this slot
    if (threadIdx.x == 0) {
      const uint32_t nb = blockIdx.x + (j + ns) * gridDim.x;
      if (nb < num_batches) {
        fence_proxy_async_smem();
        issue(nb, slot);
        issued[slot] += 1;
      }
    }
  }
  if (first_bad != ~0ull) atomicMin(nonfinite, static_cast<unsigned long long>(first_bad));
  // On abort, wait (bounded) for the newest copy issued into each slot: a
  // slot's phases complete in order, so that drains everything in flight.
  if (abort_flag && threadIdx.x == 0) {
    for (uint32_t s = 0; s < ns; ++s)
      if (issued[s] > 0 && !mbar_wait(&bars[s], (issued[s] - 1) & 1u, err, kErrWaitDrain)) break;
  }
}

// Per-warp pipelines: every warp streams its own rows HBM -> shared memory,
// one cp.async.bulk per row into a private ring of `ns` row slots with one
// mbarrier each, and reduces a row with warp shuffles only.  No CTA-wide
// barrier sits on the data path, so the warps of a CTA overlap their copies
// and their arithmetic freely.  Used for rows up to 2048 floats.
// A slot holds `rps` consecutive rows (one copy when rows are contiguous), so
// short rows still move in multi-kilobyte transfers.
template <int OP>
__global__ void __launch_bounds__(THREADS) row_warp_kernel(const float* __restrict__ in, uint64_t stride,
                                                           float* __restrict__ out, float* __restrict__ inv_rms,
                                                           const float* __restrict__ weight, float eps,
                                                           uint32_t rows, uint32_t w, uint32_t ns, uint32_t wpc,
                                                           uint32_t rps, unsigned long long* __restrict__ nonfinite,
                                                           unsigned int* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= wpc) return;
  const uint32_t slot_floats = rps * w;
  float* ring = reinterpret_cast<float*>(smem_raw) + static_cast<uint64_t>(warp) * ns * slot_floats;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem_raw + static_cast<uint64_t>(wpc) * ns * slot_floats * 4) + warp * ns;
  if (lane == 0) {
    for (uint32_t s = 0; s < ns; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncwarp();
  griddep_wait();  // as in row_bulk_kernel: the previous kernel completes first
  const uint32_t gw = blockIdx.x * wpc + warp, nw = gridDim.x * wpc;
  const uint32_t units = (rows + rps - 1) / rps;
  const uint32_t row_bytes = w * 4u;
  const bool contiguous = (stride == w);
  // Issue unit u (rows u*rps ...) into `slot` (lane 0 only).
  auto issue = [&](uint32_t u, uint32_t slot) {
    const uint32_t r0 = u * rps;
    const uint32_t nr = min(rps, rows - r0);
    float* dst = ring + slot * slot_floats;
    mbar_arrive_expect_tx(&bars[slot], nr * row_bytes);
    if (contiguous) {
      bulk_load(dst, in + static_cast<uint64_t>(r0) * w, nr * row_bytes, &bars[slot]);
    } else {
      for (uint32_t i = 0; i < nr; ++i)
        bulk_load(dst + i * w, in + static_cast<uint64_t>(r0 + i) * stride, row_bytes, &bars[slot]);
    }
  };
  uint32_t issued[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (lane == 0) {
    for (uint32_t s = 0; s < ns; ++s) {
      const uint64_t u = gw + static_cast<uint64_t>(s) * nw;
      if (u >= units) break;
      issue(static_cast<uint32_t>(u), s);
      issued[s] += 1;
    }
  }
  uint64_t first_bad = ~0ull;
  bool aborted = false;
  for (uint32_t j = 0;; ++j) {
    const uint64_t u = gw + static_cast<uint64_t>(j) * nw;
    if (u >= units) break;
    const uint32_t slot = j % ns;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars[slot], (j / ns) & 1u, err, kErrWaitRow));
    if (!ok) {
      aborted = true;
      break;
    }
    const uint32_t r0 = static_cast<uint32_t>(u) * rps;
    const uint32_t nr = min(rps, rows - r0);
    for (uint32_t i = 0; i < nr; ++i) {
      const uint64_t r = r0 + i;
      const float inv = process_row<OP, 32>(ring + slot * slot_floats + i * w, w, lane, r, out, weight, eps, nullptr,
                                            nullptr, first_bad);
      if constexpr (OP == kRms) {
        if (lane == 0 && inv_rms != nullptr) inv_rms[r] = inv;
      }
    }
    __syncwarp();  // every lane is done reading this slot
    if (lane == 0) {
      const uint64_t nu = gw + static_cast<uint64_t>(j + ns) * nw;
      if (nu < units) {
        fence_proxy_async_smem();
        issue(static_cast<uint32_t>(nu), slot);
        issued[slot] += 1;
      }
    }
  }
  if (first_bad != ~0ull) atomicMin(nonfinite, static_cast<unsigned long long>(first_bad));
  if (aborted && lane == 0) {
    // drain: a slot's phases complete in order, so its newest copy is enough
    for (uint32_t s = 0; s < ns; ++s)
      if (issued[s] > 0 && !mbar_wait(&bars[s], (issued[s] - 1) & 1u, err, kErrWaitDrain)) break;
  }
}

// Rows of w = 128 * NV (NV <= 16): one warp per row, each lane holding NV
// float4 of it in registers.  A warp issues the loads of RPW rows at once
// (NV * RPW >= 8 float4 in flight per lane) straight from global memory; with no
// shared-memory ring up to 8 CTAs (64 warps) fit on an SM, so at 32768 x 256
// every row is requested in the first round of loads.  The arithmetic is
// process_row's for TPR = 32, float4 by float4 in the same order.
template <int OP, int NV>
__global__ void __launch_bounds__(THREADS) row_reg_kernel(const float* __restrict__ in, uint64_t stride,
                                                          float* __restrict__ out, float* __restrict__ inv_rms,
                                                          const float* __restrict__ weight, float eps, uint32_t rows,
                                                          unsigned long long* __restrict__ nonfinite) {
  constexpr uint32_t RPW = NV >= 8 ? 1 : 8 / NV;  // rows per warp
  constexpr uint32_t W = 128 * NV;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warp_id = blockIdx.x * static_cast<uint64_t>(THREADS / 32) + (threadIdx.x >> 5);
  const uint64_t r0 = warp_id * RPW;
  griddep_wait();  // as the ring kernels: the previous kernel completes first
  if (r0 >= rows) return;
  float4 v[RPW][NV];
#pragma unroll
  for (uint32_t j = 0; j < RPW; ++j)
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t)
      v[j][t] = (r0 + j < rows) ? __ldcs(reinterpret_cast<const float4*>(in + (r0 + j) * stride) + lane + 32 * t)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
  uint64_t first_bad = ~0ull;
#pragma unroll
  for (uint32_t j = 0; j < RPW; ++j) {
    const uint64_t row = r0 + j;
    if (row >= rows) break;
    {
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        const float4 x = v[j][t];
        const uint32_t i = lane + 32 * t;
        if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) {
          note_nonfinite(x.x, row * W + 4 * i, first_bad); note_nonfinite(x.y, row * W + 4 * i + 1, first_bad);
          note_nonfinite(x.z, row * W + 4 * i + 2, first_bad); note_nonfinite(x.w, row * W + 4 * i + 3, first_bad);
        }
      }
    }
    if constexpr (OP == kSum) {
      double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        s0 += static_cast<double>(v[j][t].x); s1 += static_cast<double>(v[j][t].y);
        s2 += static_cast<double>(v[j][t].z); s3 += static_cast<double>(v[j][t].w);
      }
      const double s = warp_sum_d((s0 + s1) + (s2 + s3));
      if (lane == 0) out[row] = static_cast<float>(s);
    } else if constexpr (OP == kMax) {
      float mx = -FLT_MAX;
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) mx = fmaxf(mx, max4(v[j][t]));
      mx = warp_max_f(mx);
      if (lane == 0) out[row] = mx;
    } else if constexpr (OP == kSoftmax) {
      float mx = -FLT_MAX;
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) mx = fmaxf(mx, max4(v[j][t]));
      mx = warp_max_f(mx);
      double sum = 0.0;
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        v[j][t] = exp4(v[j][t], mx);
        sum += static_cast<double>(hsum4(v[j][t]));
      }
      sum = warp_sum_d(sum);
      const float inv = static_cast<float>(1.0 / sum);
      float4* o4 = reinterpret_cast<float4*>(out + row * W);
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        const float4 e = v[j][t];
        __stcs(o4 + lane + 32 * t, make_float4(e.x * inv, e.y * inv, e.z * inv, e.w * inv));
      }
    } else {  // kRms
      double ss = 0.0;
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) ss += sq4(v[j][t]);
      ss = warp_sum_d(ss);
      const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(W) + static_cast<double>(eps)));
      float4* o4 = reinterpret_cast<float4*>(out + row * W);
      const float4* w4 = reinterpret_cast<const float4*>(weight);
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        const float4 x = v[j][t];
        const float4 g = __ldg(w4 + lane + 32 * t);
        __stcs(o4 + lane + 32 * t, make_float4(x.x * inv * g.x, x.y * inv * g.y, x.z * inv * g.z, x.w * inv * g.w));
      }
      if (lane == 0 && inv_rms != nullptr) inv_rms[row] = inv;
    }
  }
  if (first_bad != ~0ull) atomicMin(nonfinite, static_cast<unsigned long long>(first_bad));
}

// Rows of 4096: two warps per row, each lane holding 16 float4 of its warp's half;
// the two halves meet in shared memory.  Four rows per CTA.
template <int OP>
__global__ void __launch_bounds__(THREADS) row_reg2_kernel(const float* __restrict__ in, uint64_t stride,
                                                           float* __restrict__ out, float* __restrict__ inv_rms,
                                                           const float* __restrict__ weight, float eps, uint32_t rows,
                                                           unsigned long long* __restrict__ nonfinite) {
  constexpr uint32_t NV = 16, W = 4096, PAIRS = THREADS / 64;
  __shared__ double dsh[PAIRS][2];
  __shared__ float fsh[PAIRS][2];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t pair = warp >> 1, half = warp & 1u;
  const uint64_t row = blockIdx.x * static_cast<uint64_t>(PAIRS) + pair;
  const bool live = row < rows;
  griddep_wait();  // as the ring kernels: the previous kernel completes first
  float4 v[NV];
  const uint32_t q0 = half * 512u + lane;  // float4 index within the row: q0 + 32 t
#pragma unroll
  for (uint32_t t = 0; t < NV; ++t)
    v[t] = live ? __ldcs(reinterpret_cast<const float4*>(in + row * stride) + q0 + 32 * t)
                : make_float4(0.f, 0.f, 0.f, 0.f);
  uint64_t first_bad = ~0ull;
  if (live) {
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t) {
      const float4 x = v[t];
      const uint64_t i = q0 + 32 * t;
      if (!(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w))) {
        note_nonfinite(x.x, row * W + 4 * i, first_bad); note_nonfinite(x.y, row * W + 4 * i + 1, first_bad);
        note_nonfinite(x.z, row * W + 4 * i + 2, first_bad); note_nonfinite(x.w, row * W + 4 * i + 3, first_bad);
      }
    }
  }
  // sum of the two halves' partials, the same in both warps of the pair
  auto pair_sum = [&](double p) -> double {
    p = warp_sum_d(p);
    if (lane == 0) dsh[pair][half] = p;
    __syncthreads();
    const double t = dsh[pair][0] + dsh[pair][1];
    __syncthreads();
    return t;
  };
  auto pair_max = [&](float p) -> float {
    p = warp_max_f(p);
    if (lane == 0) fsh[pair][half] = p;
    __syncthreads();
    const float t = fmaxf(fsh[pair][0], fsh[pair][1]);
    __syncthreads();
    return t;
  };
  if constexpr (OP == kSum) {
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t) {
      s0 += static_cast<double>(v[t].x); s1 += static_cast<double>(v[t].y);
      s2 += static_cast<double>(v[t].z); s3 += static_cast<double>(v[t].w);
    }
    const double s = pair_sum((s0 + s1) + (s2 + s3));
    if (live && half == 0 && lane == 0) out[row] = static_cast<float>(s);
  } else if constexpr (OP == kMax) {
    float mx = -FLT_MAX;
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t) mx = fmaxf(mx, max4(v[t]));
    mx = pair_max(mx);
    if (live && half == 0 && lane == 0) out[row] = mx;
  } else if constexpr (OP == kSoftmax) {
    float mx = -FLT_MAX;
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t) mx = fmaxf(mx, max4(v[t]));
    mx = pair_max(mx);
    double sum = 0.0;
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t) {
      v[t] = exp4(v[t], mx);
      sum += static_cast<double>(hsum4(v[t]));
    }
    sum = pair_sum(sum);
    const float inv = static_cast<float>(1.0 / sum);
    if (live) {
      float4* o4 = reinterpret_cast<float4*>(out + row * W);
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        const float4 e = v[t];
        __stcs(o4 + q0 + 32 * t, make_float4(e.x * inv, e.y * inv, e.z * inv, e.w * inv));
      }
    }
  } else {  // kRms
    double ss = 0.0;
#pragma unroll
    for (uint32_t t = 0; t < NV; ++t) ss += sq4(v[t]);
    ss = pair_sum(ss);
    const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(W) + static_cast<double>(eps)));
    if (live) {
      float4* o4 = reinterpret_cast<float4*>(out + row * W);
      const float4* w4 = reinterpret_cast<const float4*>(weight);
#pragma unroll
      for (uint32_t t = 0; t < NV; ++t) {
        const float4 x = v[t];
        const float4 g = __ldg(w4 + q0 + 32 * t);
        __stcs(o4 + q0 + 32 * t, make_float4(x.x * inv * g.x, x.y * inv * g.y, x.z * inv * g.z, x.w * inv * g.w));
      }
      if (half == 0 && lane == 0 && inv_rms != nullptr) inv_rms[row] = inv;
    }
  }
  if (first_bad != ~0ull) atomicMin(nonfinite, static_cast<unsigned long long>(first_bad));
}

template <int OP>
cudaError_t launch_reg2(const float* in, uint64_t stride, float* out, float* inv_rms, const float* weight, float eps,
                        uint32_t rows, unsigned long long* nonfinite, cudaStream_t stream) {
  const uint64_t grid = (static_cast<uint64_t>(rows) + THREADS / 64 - 1) / (THREADS / 64);
  if (grid > 0x7FFFFFFFull) return cudaErrorInvalidValue;
  return launch_dependent(row_reg2_kernel<OP>, dim3(static_cast<uint32_t>(grid)), dim3(THREADS), 0, stream, in,
                          stride, out, inv_rms, weight, eps, rows, nonfinite);
}

template <int OP, int NV>
cudaError_t launch_reg(const float* in, uint64_t stride, float* out, float* inv_rms, const float* weight, float eps,
                       uint32_t rows, unsigned long long* nonfinite, cudaStream_t stream) {
  constexpr uint32_t rows_per_cta = (THREADS / 32) * (NV >= 8 ? 1 : 8 / NV);
  const uint64_t grid = (static_cast<uint64_t>(rows) + rows_per_cta - 1) / rows_per_cta;
  if (grid > 0x7FFFFFFFull) return cudaErrorInvalidValue;
  return launch_dependent(row_reg_kernel<OP, NV>, dim3(static_cast<uint32_t>(grid)), dim3(THREADS), 0, stream, in,
                          stride, out, inv_rms, weight, eps, rows, nonfinite);
}

template <int OP>
cudaError_t launch_warp(const float* in, uint64_t stride, float* out, float* inv_rms, const float* weight, float eps,
                        uint32_t rows, uint32_t w, unsigned long long* nonfinite, unsigned int* err,
                        cudaStream_t stream) {
  const uint32_t row_bytes = w * 4u;
  uint32_t wpc, ns, rps = 1;
  if (row_bytes <= 2048u) {  // short rows: 8 warps, 4 KB slots of rps rows, 64 KB ring -> 3 CTAs per SM
    // (a deeper 224 KB ring at one CTA per SM measured slower: fewer CTAs to hide the latency)
    wpc = 8;
    rps = 4096u / row_bytes;
    ns = 65536u / (wpc * rps * row_bytes);
    ns = ns < 2 ? 2 : (ns > 8 ? 8 : ns);
  } else if (row_bytes <= 8192u) {  // 8 warps x 3 slots, one CTA per SM
    wpc = 8;
    ns = 3;
  } else {  // up to 16 KB rows: 4 warps x 3 slots
    wpc = 4;
    ns = 3;
  }
  const uint32_t smem = wpc * ns * rps * row_bytes + wpc * ns * 8u;
  auto kern = row_warp_kernel<OP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, wpc * 32, smem);
  if (per_sm < 1) per_sm = 1;
  const uint32_t units = (rows + rps - 1) / rps;
  const uint32_t need = (units + wpc - 1) / wpc;
  const uint32_t cap = static_cast<uint32_t>(sms * per_sm);
  return launch_dependent(kern, dim3(need < cap ? need : cap), dim3(wpc * 32), smem, stream, in, stride, out, inv_rms,
                          weight, eps, rows, w, ns, wpc, rps, nonfinite, err);
}

// Plain-load fallback: one CTA per row, any width / alignment.  Same arithmetic.
template <int OP>
__global__ void __launch_bounds__(THREADS) row_plain_kernel(const float* __restrict__ in, uint64_t stride,
                                                            float* __restrict__ out, float* __restrict__ inv_rms,
                                                            const float* __restrict__ weight, float eps,
                                                            uint32_t rows, uint32_t w,
                                                            unsigned long long* __restrict__ nonfinite) {
  __shared__ double dscr[THREADS / 32];
  __shared__ float fscr[THREADS / 32];
  uint64_t first_bad = ~0ull;
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* x = in + static_cast<uint64_t>(r) * stride;
    if constexpr (OP == kSum) {
      double s = 0.0;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS) {
        const float v = __ldg(x + c);
        s += static_cast<double>(v);
        note_nonfinite(v, static_cast<uint64_t>(r) * w + c, first_bad);
      }
      s = group_sum_d<THREADS>(s, dscr);
      if (threadIdx.x == 0) out[r] = static_cast<float>(s);
    } else if constexpr (OP == kMax) {
      float mx = -FLT_MAX;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS) {
        const float v = __ldg(x + c);
        mx = fmaxf(mx, v);
        note_nonfinite(v, static_cast<uint64_t>(r) * w + c, first_bad);
      }
      mx = group_max_f<THREADS>(mx, fscr);
      if (threadIdx.x == 0) out[r] = mx;
    } else if constexpr (OP == kSoftmax) {
      float mx = -FLT_MAX;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS) {
        const float v = __ldg(x + c);
        mx = fmaxf(mx, v);
        note_nonfinite(v, static_cast<uint64_t>(r) * w + c, first_bad);
      }
      mx = group_max_f<THREADS>(mx, fscr);
      double s = 0.0;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS) s += static_cast<double>(expf(__ldg(x + c) - mx));
      s = group_sum_d<THREADS>(s, dscr);
      const double inv = 1.0 / s;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS)
        out[static_cast<uint64_t>(r) * w + c] = static_cast<float>(static_cast<double>(expf(__ldg(x + c) - mx)) * inv);
    } else {
      double ss = 0.0;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS) {
        const float v = __ldg(x + c);
        ss += static_cast<double>(v) * v;
        note_nonfinite(v, static_cast<uint64_t>(r) * w + c, first_bad);
      }
      ss = group_sum_d<THREADS>(ss, dscr);
      const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(w) + static_cast<double>(eps)));
      if (threadIdx.x == 0 && inv_rms != nullptr) inv_rms[r] = inv;
      for (uint32_t c = threadIdx.x; c < w; c += THREADS)
        out[static_cast<uint64_t>(r) * w + c] = __ldg(x + c) * inv * __ldg(weight + c);
    }
    __syncthreads();
  }
  if (first_bad != ~0ull) atomicMin(nonfinite, static_cast<unsigned long long>(first_bad));
}

template <int OP, int TPR>
cudaError_t launch_bulk(const float* in, uint64_t stride, float* out, float* inv_rms, const float* weight, float eps,
                        uint32_t rows, uint32_t w, unsigned long long* nonfinite, unsigned int* err,
                        cudaStream_t stream) {
  constexpr uint32_t RPB = THREADS / TPR;
  const uint32_t batch_bytes = RPB * w * 4u;
  uint32_t ns = SLOT_BUDGET_BYTES / batch_bytes;
  ns = ns < 2 ? 2 : (ns > 8 ? 8 : ns);
  const uint32_t smem = ns * batch_bytes;
  auto kern = row_bulk_kernel<OP, TPR>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, THREADS, smem);
  if (per_sm < 1) per_sm = 1;
  const uint32_t batches = (rows + RPB - 1) / RPB;
  const uint32_t grid = static_cast<uint32_t>(batches < static_cast<uint32_t>(sms * per_sm) ? batches : sms * per_sm);
  return launch_dependent(kern, dim3(grid), dim3(THREADS), smem, stream, in, stride, out, inv_rms, weight, eps, rows,
                          w, ns, nonfinite, err);
}

template <int OP>
cudaError_t dispatch(const float* in, uint64_t stride, float* out, float* inv_rms, const float* weight, float eps,
                     uint32_t rows, uint32_t w, unsigned long long* nonfinite, unsigned int* err,
                     cudaStream_t stream) {
  if (rows == 0 || w == 0) return cudaSuccess;
  // The bulk path needs 16-byte granular rows for the copies and, for the
  // row-wide outputs (softmax, RMSNorm), 16-byte aligned output and weight.
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool rowwise_out = (OP == kSoftmax || OP == kRms);
  const bool aligned = (w % 4 == 0) && (stride % 4 == 0) && a16(in) && (!rowwise_out || a16(out)) &&
                       (weight == nullptr || a16(weight));
  if (aligned && w == 128) return launch_reg<OP, 1>(in, stride, out, inv_rms, weight, eps, rows, nonfinite, stream);
  if (aligned && w == 256) return launch_reg<OP, 2>(in, stride, out, inv_rms, weight, eps, rows, nonfinite, stream);
  if (aligned && w == 512) return launch_reg<OP, 4>(in, stride, out, inv_rms, weight, eps, rows, nonfinite, stream);
  if (aligned && w == 1024) return launch_reg<OP, 8>(in, stride, out, inv_rms, weight, eps, rows, nonfinite, stream);
  if (aligned && w == 2048) return launch_reg<OP, 16>(in, stride, out, inv_rms, weight, eps, rows, nonfinite, stream);
  if (aligned && w == 4096) return launch_reg2<OP>(in, stride, out, inv_rms, weight, eps, rows, nonfinite, stream);
  if (aligned && w <= 2048) return launch_warp<OP>(in, stride, out, inv_rms, weight, eps, rows, w, nonfinite, err, stream);
  if (aligned && w <= BULK_MAX_WIDTH)
    return launch_bulk<OP, THREADS>(in, stride, out, inv_rms, weight, eps, rows, w, nonfinite, err, stream);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint32_t grid = rows < static_cast<uint32_t>(sms * 8) ? rows : static_cast<uint32_t>(sms * 8);
  row_plain_kernel<OP><<<grid, THREADS, 0, stream>>>(in, stride, out, inv_rms, weight, eps, rows, w, nonfinite);
  return cudaGetLastError();
}

}  // namespace

cudaError_t row_reduce(const float* in, float* out, uint32_t rows, uint32_t width, uint32_t op,
                       unsigned long long* nonfinite, unsigned int* err, cudaStream_t stream) {
  switch (op) {
    case 1: return dispatch<kSum>(in, width, out, nullptr, nullptr, 0.f, rows, width, nonfinite, err, stream);
    case 2: return dispatch<kMax>(in, width, out, nullptr, nullptr, 0.f, rows, width, nonfinite, err, stream);
    case 3: return dispatch<kSoftmax>(in, width, out, nullptr, nullptr, 0.f, rows, width, nonfinite, err, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t rmsnorm(const float* in, uint64_t in_stride, const float* weight, float* out, float* inv_rms,
                    uint32_t rows, uint32_t width, float eps, unsigned long long* nonfinite, unsigned int* err,
                    cudaStream_t stream) {
  return dispatch<kRms>(in, in_stride, out, inv_rms, weight, eps, rows, width, nonfinite, err, stream);
}

// ---------------------------------------------------------------- self-check
// The reduction benchmark entry's correctness check (reactor_vulkan_fused_reduction.c:
// 1122-1206 checks its output against prom_reduction_cpu_reference with
// prom_reduction_compare, :996-1114).  Here both halves run on the device: an
// independent plain kernel, one thread per row walking it in order, recomputes
// the expected values (SUM in binary64, MAX exact, SOFTMAX with binary64 exp and
// denominator), and a compare kernel applies the comparator's tolerances and
// records the smallest failing flat index (softmax row-sum failures are encoded
// after the element range).
namespace {

__global__ void check_expected_kernel(const float* __restrict__ in, float* __restrict__ expected, uint32_t rows,
                                      uint32_t width, uint32_t op) {
  for (uint64_t r = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; r < rows;
       r += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const float* v = in + r * width;
    if (op == kSum) {
      double acc = 0.0;
      for (uint32_t c = 0; c < width; ++c) acc += static_cast<double>(v[c]);
      expected[r] = static_cast<float>(acc);
    } else {
      float mx = v[0];
      for (uint32_t c = 1; c < width; ++c) mx = v[c] > mx ? v[c] : mx;
      if (op == kMax) {
        expected[r] = mx;
      } else {
        double den = 0.0;
        for (uint32_t c = 0; c < width; ++c) den += exp(static_cast<double>(v[c]) - mx);
        for (uint32_t c = 0; c < width; ++c)
          expected[r * width + c] = static_cast<float>(exp(static_cast<double>(v[c]) - mx) / den);
      }
    }
  }
}

__device__ __forceinline__ float rel_floor(float expected, float actual) {
  float den = fabsf(expected);
  if (den < 1.0e-20f) den = 1.0f;
  return fabsf(actual - expected) / den;
}

__global__ void check_compare_kernel(const float* __restrict__ expected, const float* __restrict__ actual,
                                     uint32_t rows, uint32_t width, uint32_t op,
                                     unsigned long long* __restrict__ first_bad) {
  const uint64_t count = op == kSoftmax ? static_cast<uint64_t>(rows) * width : rows;
  const float atol = op == kSoftmax ? 2.0e-5f : (op == kMax ? 0.0f : 2.0e-5f * static_cast<float>(width));
  const float rtol = op == kSoftmax ? 2.0e-4f : (op == kMax ? 0.0f : 2.0e-5f);
  const uint64_t step = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const uint64_t t0 = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  for (uint64_t i = t0; i < count; i += step) {
    const float a = actual[i], e = expected[i];
    if (!isfinite(a) || (fabsf(a - e) > atol && rel_floor(e, a) > rtol)) atomicMin(first_bad, i);
  }
  if (op == kSoftmax) {
    for (uint64_t r = t0; r < rows; r += step) {
      double s = 0.0;
      bool ok = true;
      for (uint32_t c = 0; c < width; ++c) {
        const float v = actual[r * width + c];
        if (!isfinite(v) || v < -2.0e-7f) ok = false;
        s += v;
      }
      if (!ok || fabs(s - 1.0) > 3.0e-4) atomicMin(first_bad, count + r);
    }
  }
}

}  // namespace

cudaError_t reduction_self_check(const float* in, const float* actual, float* expected, uint32_t rows,
                                 uint32_t width, uint32_t op, unsigned long long* first_bad, cudaStream_t stream) {
  if (rows == 0 || width == 0) return cudaSuccess;
  if (op != kSum && op != kMax && op != kSoftmax) return cudaErrorInvalidValue;
  const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>((rows + 127) / 128, 148ull * 8));
  check_expected_kernel<<<grid, 128, 0, stream>>>(in, expected, rows, width, op);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  check_compare_kernel<<<148 * 8, 256, 0, stream>>>(expected, actual, rows, width, op, first_bad);
  return cudaGetLastError();
}

}  // namespace oct
