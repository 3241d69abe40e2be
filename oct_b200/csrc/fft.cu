// fft.cu -- radix-2 complex FFTs (the reference's prometheus_reactor_runtime_fft64 /
// prometheus_reactor_runtime_fft).
//
// The reference runs a decimation-in-time radix-2 network: one bit-reversal
// pass, then log2(N) butterfly passes of span 2, 4, .., N, each a separate
// dispatch through global memory (shaders/sdslv/production/fft/radix2_fp64.sdslv,
// radix2_bit_reverse.sdslv, radix2_butterfly.sdslv).  A butterfly of pass
// `span` on positions (base + lower, base + lower + span / 2) forms
//   t = w * odd   (tr = wr br - wi bi, ti = wr bi + wi br)
//   outputs even + t and even - t,
// with w = the binary64 host table entry lower * (N / span) (fp64), or
// (cos a, sin a) of the fp32 angle a = -+2 pi lower / span (fp32).
//
// Here the same network runs in at most two kernels, each keeping a tile in
// shared memory across many passes:
//   * fft_local_kernel: gathers a tile of S consecutive bit-reversed positions
//     (S = min(N, 2048) complex doubles / 4096 complex floats = 32 KB) and runs
//     every pass with span <= S on it;
//   * fft_global_kernel (N > S): the data as [N / S rows][S columns]; the
//     passes with span > S pair rows within a column, so a CTA holding all rows
//     of a few columns runs every remaining pass.
// Every butterfly computes exactly the reference's operations in the same
// order (products and sums rounded separately, no fused multiply-add), so the
// fp64 transform equals the reference network bit for bit.  HBM traffic is two
// reads and two writes of the data instead of log2(N) + 1 of each.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace oct {
namespace {

constexpr int kThreads = 256;

template <typename T>
struct Cplx;
template <>
struct Cplx<double> {
  using V = double2;
  static constexpr uint32_t kTile = 2048;  // complex elements per local tile (32 KB)
  static constexpr uint32_t kCols = 8;     // columns per CTA in the global passes (128-byte row segments)
};
template <>
struct Cplx<float> {
  using V = float2;
  static constexpr uint32_t kTile = 4096;
  static constexpr uint32_t kCols = 16;
};

__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }

// Twiddle of pass `span` at offset `lower` (< span / 2) for an n-point transform.
template <typename T>
__device__ __forceinline__ typename Cplx<T>::V twiddle(const double* tw, uint32_t n, uint32_t span, uint32_t lower,
                                                       int inverse);
template <>
__device__ __forceinline__ double2 twiddle<double>(const double* tw, uint32_t n, uint32_t span, uint32_t lower, int) {
  const uint32_t i = lower * (n / span);
  return make_double2(tw[2 * i], tw[2 * i + 1]);
}
template <>
__device__ __forceinline__ float2 twiddle<float>(const double*, uint32_t, uint32_t span, uint32_t lower, int inverse) {
  // radix2_butterfly.sdslv: angle = sign * 2 pi * lower / span in fp32, native cos / sin
  const float sign = inverse ? 1.0f : -1.0f;
  const float angle = __fdiv_rn(__fmul_rn(__fmul_rn(sign, 6.28318530717958647692f), static_cast<float>(lower)),
                                static_cast<float>(span));
  float s, c;
  sincosf(angle, &s, &c);
  return make_float2(c, s);
}

// One butterfly in place: a <- a + w b, b <- a - w b.
template <typename T, typename V>
__device__ __forceinline__ void butterfly(V& a, V& b, V w) {
  const T tr = sub_rn(mul_rn(w.x, b.x), mul_rn(w.y, b.y));
  const T ti = add_rn(mul_rn(w.x, b.y), mul_rn(w.y, b.x));
  const V e = a;
  a.x = add_rn(e.x, tr);
  a.y = add_rn(e.y, ti);
  b.x = sub_rn(e.x, tr);
  b.y = sub_rn(e.y, ti);
}

__device__ __forceinline__ uint32_t reverse_bits(uint32_t v, uint32_t bits) {
  return bits == 0 ? 0u : (__brev(v) >> (32u - bits));
}

// Tile t of batch item blockIdx.y: bit-reversal gather and every pass of span <= S.
template <typename T>
__global__ void __launch_bounds__(kThreads) fft_local_kernel(const typename Cplx<T>::V* __restrict__ in,
                                                             typename Cplx<T>::V* __restrict__ out, uint32_t n,
                                                             uint32_t log2n, uint32_t tile, uint32_t log2tile,
                                                             uint64_t stride, const double* __restrict__ tw,
                                                             int inverse, int normalize) {
  using V = typename Cplx<T>::V;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V* s = reinterpret_cast<V*>(smem_raw);
  const uint64_t base = static_cast<uint64_t>(blockIdx.y) * stride;
  const uint32_t t0 = blockIdx.x * tile;
  for (uint32_t p = threadIdx.x; p < tile; p += kThreads) s[p] = in[base + reverse_bits(t0 + p, log2n)];
  __syncthreads();
  for (uint32_t level = 1; level <= log2tile; ++level) {
    const uint32_t span = 1u << level, half = span >> 1;
    const bool last = normalize && level == log2n;
    for (uint32_t q = threadIdx.x; q < tile / 2; q += kThreads) {
      const uint32_t block = q >> (level - 1), lower = q & (half - 1);
      const uint32_t a = block * span + lower;
      V x = s[a], y = s[a + half];
      butterfly<T>(x, y, twiddle<T>(tw, n, span, lower, inverse));
      if (last) {
        const T scale = static_cast<T>(n);
        x.x = x.x / scale; x.y = x.y / scale;
        y.x = y.x / scale; y.y = y.y / scale;
      }
      s[a] = x;
      s[a + half] = y;
    }
    __syncthreads();
  }
  for (uint32_t p = threadIdx.x; p < tile; p += kThreads) out[base + t0 + p] = s[p];
}

// Passes of span 2S .. N over [rows = N / S][S]: a CTA holds kCols columns of every row.
template <typename T>
__global__ void __launch_bounds__(kThreads) fft_global_kernel(typename Cplx<T>::V* __restrict__ data, uint32_t n,
                                                              uint32_t log2n, uint32_t tile, uint32_t log2tile,
                                                              uint64_t stride, const double* __restrict__ tw,
                                                              int inverse, int normalize) {
  using V = typename Cplx<T>::V;
  constexpr uint32_t C = Cplx<T>::kCols;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V* s = reinterpret_cast<V*>(smem_raw);  // [rows][C]
  const uint32_t rows = n >> log2tile;
  const uint64_t base = static_cast<uint64_t>(blockIdx.y) * stride;
  const uint32_t c0 = blockIdx.x * C;
  for (uint32_t e = threadIdx.x; e < rows * C; e += kThreads) {
    const uint32_t r = e / C, c = e - r * C;
    s[e] = data[base + static_cast<uint64_t>(r) * tile + c0 + c];
  }
  __syncthreads();
  for (uint32_t level = log2tile + 1; level <= log2n; ++level) {
    const uint32_t span = 1u << level, half_rows = 1u << (level - 1 - log2tile);
    const bool last = normalize && level == log2n;
    for (uint32_t q = threadIdx.x; q < rows / 2 * C; q += kThreads) {
      const uint32_t pair = q / C, c = q - pair * C;
      const uint32_t block = pair / half_rows, r_low = pair - block * half_rows;
      const uint32_t ra = block * 2 * half_rows + r_low;
      const uint32_t lower = r_low * tile + c0 + c;  // position within the span's lower half
      V x = s[ra * C + c], y = s[(ra + half_rows) * C + c];
      butterfly<T>(x, y, twiddle<T>(tw, n, span, lower, inverse));
      if (last) {
        const T scale = static_cast<T>(n);
        x.x = x.x / scale; x.y = x.y / scale;
        y.x = y.x / scale; y.y = y.y / scale;
      }
      s[ra * C + c] = x;
      s[(ra + half_rows) * C + c] = y;
    }
    __syncthreads();
  }
  for (uint32_t e = threadIdx.x; e < rows * C; e += kThreads) {
    const uint32_t r = e / C, c = e - r * C;
    data[base + static_cast<uint64_t>(r) * tile + c0 + c] = s[e];
  }
}

uint32_t log2u(uint32_t v) {
  uint32_t b = 0;
  while (v > 1) {
    v >>= 1;
    ++b;
  }
  return b;
}

template <typename T>
cudaError_t fft_run(const void* in, void* out, uint32_t n, uint32_t batch, uint64_t stride, const double* tw,
                    bool inverse, bool normalize, cudaStream_t stream) {
  using V = typename Cplx<T>::V;
  if (n == 0 || (n & (n - 1)) != 0 || n > kFftMaxElements || batch == 0 || batch > 65535u) return cudaErrorInvalidValue;
  const uint32_t log2n = log2u(n);
  const uint32_t tile = n < Cplx<T>::kTile ? n : Cplx<T>::kTile;
  const uint32_t log2tile = log2u(tile);
  const size_t smem_local = static_cast<size_t>(tile) * sizeof(V);
  if (smem_local > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(fft_local_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_local));
    if (e != cudaSuccess) return e;
  }
  fft_local_kernel<T><<<dim3(n / tile, batch), kThreads, smem_local, stream>>>(
      static_cast<const V*>(in), static_cast<V*>(out), n, log2n, tile, log2tile, stride, tw, inverse ? 1 : 0,
      normalize ? 1 : 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n == tile) return e;
  constexpr uint32_t C = Cplx<T>::kCols;
  const size_t smem_global = static_cast<size_t>(n / tile) * C * sizeof(V);
  e = cudaFuncSetAttribute(fft_global_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_global));
  if (e != cudaSuccess) return e;
  fft_global_kernel<T><<<dim3(tile / C, batch), kThreads, smem_global, stream>>>(
      static_cast<V*>(out), n, log2n, tile, log2tile, stride, tw, inverse ? 1 : 0, normalize ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace

cudaError_t fft64(const double* in, double* out, uint32_t n, const double* twiddles, cudaStream_t stream) {
  return fft_run<double>(in, out, n, 1, n, twiddles, false, false, stream);
}

cudaError_t fft32(const float* in, float* out, uint32_t n, uint32_t batch, uint64_t stride_elements, bool inverse,
                  bool normalize, cudaStream_t stream) {
  return fft_run<float>(in, out, n, batch, stride_elements, nullptr, inverse, normalize, stream);
}

}  // namespace oct
