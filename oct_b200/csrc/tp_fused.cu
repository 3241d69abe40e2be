// tp_fused.cu -- tensor-parallel collectives of the block, done over NVLink
// peer memory instead of NCCL calls.
//
// A row-parallel product (out projection, down / W2) leaves a partial sum on
// every rank.  Its GEMM epilogue (sgemm_tc.cu, RowScatter) already writes each
// output row into the row's owner rank, slot [source rank], so the reduction
// traffic crosses NVLink while the GEMM still computes.  Then:
//   signal  -- each rank publishes "my stores for phase p are done" into every
//              rank's flag array (release, system scope);
//   wait    -- one warp spins (bounded) until every source rank's flag for the
//              phase reached this forward's epoch (acquire, system scope);
//   reduce  -- each rank sums the slots of its own rows in a fixed order,
//              applies the block's residual / norm / modulation, keeps what it
//              needs locally and pushes the finished rows to every rank (an
//              all-gather by stores), followed by another signal / wait.
// This is the Megatron all-reduce split into its reduce-scatter and
// all-gather halves, with the first half fused into the GEMM and the second
// into the norm kernel that consumes it.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace oct {
namespace {

constexpr int TP_NT = 256;
constexpr int TP_VPT = 16;  // width <= 16 * 256

__device__ __forceinline__ double tp_block_sum(double v, double* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int i = 0; i < TP_NT / 32; ++i) t += sh[i];
  return t;
}

__global__ void tp_signal_kernel(uint64_t* const* flags, uint32_t slot, uint32_t world, uint32_t src,
                                 uint64_t epoch) {
  const uint32_t t = threadIdx.x;
  if (t < world) {
    __threadfence_system();  // every store this rank made before this kernel is visible first
    uint64_t* f = flags[t] + static_cast<uint64_t>(slot) * world + src;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(epoch) : "memory");
  }
}

__global__ void tp_wait_kernel(const uint64_t* flags, uint32_t slot, uint32_t world, uint64_t epoch,
                               unsigned int* err, unsigned long long budget_ns) {
  const uint32_t t = threadIdx.x;
  if (t < world) {
    const uint64_t* f = flags + static_cast<uint64_t>(slot) * world + t;
    const unsigned long long start = global_timer_ns();
    while (true) {
      uint64_t v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
      if (v >= epoch) break;
      if (global_timer_ns() - start > budget_ns) {
        atomicOr(err, kErrWaitPeer);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// signal + wait in one launch: lane t publishes to rank t, then waits for rank t.
__global__ void tp_phase_kernel(uint64_t* const* flags_dev, const uint64_t* flags_local, uint32_t slot, uint32_t world,
                                uint32_t src, uint64_t epoch, unsigned int* err, unsigned long long budget_ns) {
  const uint32_t t = threadIdx.x;
  if (t < world) {
    __threadfence_system();
    uint64_t* f = flags_dev[t] + static_cast<uint64_t>(slot) * world + src;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(epoch) : "memory");
    const uint64_t* g = flags_local + static_cast<uint64_t>(slot) * world + t;
    const unsigned long long start = global_timer_ns();
    while (true) {
      uint64_t v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(g) : "memory");
      if (v >= epoch) break;
      if (global_timer_ns() - start > budget_ns) {
        atomicOr(err, kErrWaitPeer);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
}

// One CTA per own row (global row = row0 + r):
//   s = sum_k slots[k][r]                           (fixed order k = 0 .. nslots-1)
//   s = rmsnorm(s) * g1                             (if g1)
//   v = res[row] + gate1[item] * s  or  res + s     (if res; else v = s)
//   keep[row] = v                                   (if keep)
//   u = rmsnorm(v) * g2 * mul2[item] + add2[item]   (if g2; else u = v)
//   push[k][row] = u for every rank k               (peers over NVLink, self locally)
__global__ void __launch_bounds__(TP_NT) tp_reduce_rows_kernel(const TpReduce a) {
  __shared__ double sh[TP_NT / 32];
  for (uint32_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
    const uint64_t row = static_cast<uint64_t>(a.row0) + r;
    const uint64_t mo = (row / a.rows_per_item) * a.mod_stride;
    float v[TP_VPT];
#pragma unroll
    for (int i = 0; i < TP_VPT; ++i) v[i] = 0.f;
    for (uint32_t k = 0; k < a.nslots; ++k) {
      const float* sr = a.slots + k * a.slot_stride + static_cast<uint64_t>(r) * a.ld_slot;
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) {
        const uint32_t c = threadIdx.x + i * TP_NT;
        if (c < a.width) v[i] += sr[c];
      }
    }
    if (a.g1 != nullptr) {
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) ss += static_cast<double>(v[i]) * v[i];
      ss = tp_block_sum(ss, sh);
      const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(a.width) + static_cast<double>(a.eps)));
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) {
        const uint32_t c = threadIdx.x + i * TP_NT;
        if (c < a.width) v[i] = v[i] * inv * a.g1[c];
      }
    }
    if (a.res != nullptr) {
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) {
        const uint32_t c = threadIdx.x + i * TP_NT;
        if (c < a.width) v[i] = a.res[row * a.ld_res + c] + (a.gate1 != nullptr ? a.gate1[mo + c] * v[i] : v[i]);
      }
    }
    if (a.keep != nullptr) {
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) {
        const uint32_t c = threadIdx.x + i * TP_NT;
        if (c < a.width) a.keep[row * a.ld_keep + c] = v[i];
      }
    }
    if (a.g2 != nullptr) {
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) ss += static_cast<double>(v[i]) * v[i];
      ss = tp_block_sum(ss, sh);
      const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(a.width) + static_cast<double>(a.eps)));
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) {
        const uint32_t c = threadIdx.x + i * TP_NT;
        if (c >= a.width) continue;
        float y = v[i] * inv * a.g2[c];
        if (a.mul2 != nullptr) y = y * a.mul2[mo + c];
        if (a.add2 != nullptr) y = y + a.add2[mo + c];
        v[i] = y;
      }
    }
    for (uint32_t k = 0; k < a.npush; ++k) {
      float* dst = a.push[k] + row * a.ld_push;
#pragma unroll
      for (int i = 0; i < TP_VPT; ++i) {
        const uint32_t c = threadIdx.x + i * TP_NT;
        if (c < a.width) dst[c] = v[i];
      }
    }
  }
}

}  // namespace

cudaError_t tp_signal(uint64_t* const* flags_dev, uint32_t slot, uint32_t world, uint32_t src, uint64_t epoch,
                      cudaStream_t stream) {
  if (world == 0 || world > 32) return cudaErrorInvalidValue;
  tp_signal_kernel<<<1, 32, 0, stream>>>(flags_dev, slot, world, src, epoch);
  return cudaGetLastError();
}

cudaError_t tp_wait(const uint64_t* flags_local, uint32_t slot, uint32_t world, uint64_t epoch, unsigned int* err,
                    unsigned long long budget_ns, cudaStream_t stream) {
  if (world == 0 || world > 32) return cudaErrorInvalidValue;
  tp_wait_kernel<<<1, 32, 0, stream>>>(flags_local, slot, world, epoch, err, budget_ns);
  return cudaGetLastError();
}

cudaError_t tp_signal_wait(uint64_t* const* flags_dev, const uint64_t* flags_local, uint32_t slot, uint32_t world,
                           uint32_t src, uint64_t epoch, unsigned int* err, unsigned long long budget_ns,
                           cudaStream_t stream) {
  if (world == 0 || world > 32) return cudaErrorInvalidValue;
  tp_phase_kernel<<<1, 32, 0, stream>>>(flags_dev, flags_local, slot, world, src, epoch, err, budget_ns);
  return cudaGetLastError();
}

cudaError_t tp_reduce_rows(const TpReduce& args, cudaStream_t stream) {
  if (args.width == 0 || args.width > static_cast<uint32_t>(TP_VPT * TP_NT) || args.rows_per_item == 0)
    return cudaErrorInvalidValue;
  if (args.rows == 0) return cudaSuccess;
  const uint32_t grid = args.rows < 148u * 16u ? args.rows : 148u * 16u;
  tp_reduce_rows_kernel<<<grid, TP_NT, 0, stream>>>(args);
  return cudaGetLastError();
}

}  // namespace oct
