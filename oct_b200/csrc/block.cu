// block.cu -- the transformer block of Oct's Prometheus path, B200-first.
//
// Two block families, both fp32 end to end with every matrix product on the
// tcgen05 3xTF32 tensor-core SGEMM (sgemm_tc.cu):
//
//  * DiT (Z-Image style), following `runCanonicalNoiseRefiner0`
//    (internal/prometheus/zimage/canonical_reference.go:377-479): adaLN from a
//    sinusoidal timestep embedding -> RMSNorm + modulation -> fused QKV ->
//    per-head Q/K RMSNorm -> 3-axis interleaved RoPE -> exact bidirectional
//    attention -> out projection -> RMSNorm -> tanh-gated residual -> FFN norm +
//    modulation -> W1|W3 -> SiLU gate -> W2 -> RMSNorm -> gated residual.
//    The adaLN here is 6 x hidden (adds two shifts) where the reference has 4 x hidden.
//  * Gemma-shaped decoder: RMSNorm -> fused QKV (MQA: every query head uses KV
//    head 0) -> half-split RoPE (`cpuGemma4e2bRope`, gemma4e2b_m1_rtx.go:834-861,
//    without its BF16 storage rounding) -> causal attention with scale
//    1/sqrt(head_dim) (`cpuGemma4e2bRawScores`, :863-883) -> out projection +
//    residual -> RMSNorm -> gate|up -> GeGLU (gelu_tanh) -> down + residual.
//
// Data path per forward (T = batch * seq tokens, all buffers owned by the block):
//   norms, RoPE, softmax and gated activations are one-pass fused kernels; the
//   residual adds of the Gemma block ride in the GEMM epilogue; weights are
//   split to TF32 hi/lo once, at upload.  DiT attention is one fused kernel
//   (attention.cu); the Gemma (causal, head 256) attention materialises the
//   scores of every (item, head) and runs Q K^T and P V as strided-batched
//   tensor-core products.
//   Tensor parallel (tp_world > 1): each rank holds H/tp heads and F/tp FFN
//   columns; the two row-parallel products (out projection, down/W2) produce
//   partial sums that are all-reduced over NCCL on the block's stream.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <utility>
#include <vector>

#include "block.h"
#include "kernels.h"
#include "ptx.cuh"

namespace oct {
namespace {

constexpr int NT = 256;

__device__ __forceinline__ double block_sum_d(double v, double* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += sh[i];
  return t;
}

__device__ __forceinline__ float block_max_f(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = sh[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) t = fmaxf(t, sh[i]);
  return t;
}

// Fused row norm, one CTA per row (width <= 16 * 256):
//   y = x * inv_rms * g                              (CanonicalRMSNorm order)
//   y = y * mul[item] + add[item]                    (optional: adaLN modulation)
//   y = res + gate[item] * y   or   y = res + y      (optional: gated residual)
// `item` = row / rows_per_item indexes the per-batch-item vectors (stride mod_stride).
// With out_lo != null the result is written as its TF32 split (hi to out, lo to out_lo).
constexpr int NORM_VPT = 16;
__global__ void __launch_bounds__(NT) norm_fused_kernel(const float* __restrict__ x, uint64_t ldx,
                                                        const float* __restrict__ g, float eps,
                                                        const float* __restrict__ mul, const float* __restrict__ add,
                                                        const float* __restrict__ res, uint64_t ldres,
                                                        const float* __restrict__ gate, uint64_t mod_stride,
                                                        uint32_t rows_per_item, float* __restrict__ out,
                                                        uint64_t ldo, uint32_t rows, uint32_t width,
                                                        float* __restrict__ out_lo) {
  __shared__ double sh[NT / 32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * ldx;
    float v[NORM_VPT];
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < NORM_VPT; ++i) {
      const uint32_t c = threadIdx.x + i * NT;
      v[i] = c < width ? xr[c] : 0.f;
      ss += static_cast<double>(v[i]) * v[i];
    }
    ss = block_sum_d(ss, sh);
    const float inv = static_cast<float>(1.0 / sqrt(ss / static_cast<double>(width) + static_cast<double>(eps)));
    const uint64_t mo = static_cast<uint64_t>(r / rows_per_item) * mod_stride;
#pragma unroll
    for (int i = 0; i < NORM_VPT; ++i) {
      const uint32_t c = threadIdx.x + i * NT;
      if (c >= width) continue;
      float y = v[i] * inv * g[c];
      if (mul != nullptr) y = y * mul[mo + c];
      if (add != nullptr) y = y + add[mo + c];
      if (res != nullptr) y = res[r * ldres + c] + (gate != nullptr ? gate[mo + c] * y : y);
      if (out_lo != nullptr) {  // write the TF32 split the next product reads as its A operand
        const float h = to_tf32(y);
        out_lo[r * ldo + c] = to_tf32(y - h);
        y = h;
      }
      out[r * ldo + c] = y;
    }
  }
}

// Half-split RoPE in place over `heads` heads of width hd starting at column
// col0 of each row: pairs (i, i + hd/2), table cos/sin[pos][hd/2], pos = row % seq.
__global__ void rope_half_kernel(float* __restrict__ buf, uint64_t ld, uint32_t col0, uint32_t heads, uint32_t hd,
                                 const float* __restrict__ cos_t, const float* __restrict__ sin_t, uint32_t seq,
                                 uint32_t rows) {
  const uint32_t half = hd / 2;
  const uint64_t total = static_cast<uint64_t>(rows) * heads * half;
  for (uint64_t idx = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t i = static_cast<uint32_t>(idx % half);
    const uint64_t rh = idx / half;
    const uint32_t head = static_cast<uint32_t>(rh % heads);
    const uint32_t row = static_cast<uint32_t>(rh / heads);
    float* p = buf + row * ld + col0 + head * hd;
    const uint32_t pos = row % seq;
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    const float a = p[i], b = p[i + half];
    p[i] = a * c - b * s;
    p[i + half] = b * c + a * s;
  }
}

// Per-head RMSNorm (width 128, gain g, eps) then 3-axis interleaved RoPE with
// table cos/sin[pos][64]; one warp per (row, head), 4 channels a lane.
// Covers `heads` heads starting at column col0 (Q then K are two launches).
// Writes in place, or, with hi != null, the TF32 hi/lo split into the
// per-head layout of the fused attention kernel: row (item*heads + head)*seq + pos.
__global__ void qk_norm_rope3_kernel(float* __restrict__ buf, uint64_t ld, uint32_t col0, uint32_t heads,
                                     const float* __restrict__ g, float eps, const float* __restrict__ cos_t,
                                     const float* __restrict__ sin_t, uint32_t seq, uint32_t rows,
                                     float* __restrict__ hi, float* __restrict__ lo) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = static_cast<uint64_t>(rows) * heads;
  for (uint64_t wi = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; wi < warps;
       wi += static_cast<uint64_t>(gridDim.x) * blockDim.x / 32) {
    const uint32_t head = static_cast<uint32_t>(wi % heads);
    const uint32_t row = static_cast<uint32_t>(wi / heads);
    float* p = buf + row * ld + col0 + head * 128 + lane * 4;
    float4 v = *reinterpret_cast<float4*>(p);
    double ss = static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
                static_cast<double>(v.w) * v.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = static_cast<float>(1.0 / sqrt(ss / 128.0 + static_cast<double>(eps)));
    const float4 gg = *reinterpret_cast<const float4*>(g + lane * 4);
    v.x = v.x * inv * gg.x;
    v.y = v.y * inv * gg.y;
    v.z = v.z * inv * gg.z;
    v.w = v.w * inv * gg.w;
    const uint32_t pos = row % seq;
    const uint32_t pair0 = lane * 2;  // global pair index of (v.x, v.y); (v.z, v.w) is pair0 + 1
    const float c0 = cos_t[pos * 64 + pair0], s0 = sin_t[pos * 64 + pair0];
    const float c1 = cos_t[pos * 64 + pair0 + 1], s1 = sin_t[pos * 64 + pair0 + 1];
    float4 o;
    o.x = v.x * c0 - v.y * s0;
    o.y = v.x * s0 + v.y * c0;
    o.z = v.z * c1 - v.w * s1;
    o.w = v.z * s1 + v.w * c1;
    if (hi == nullptr) {
      *reinterpret_cast<float4*>(p) = o;
    } else {
      const uint64_t srow = (static_cast<uint64_t>(row / seq) * heads + head) * seq + pos;
      float4 h, l;
      h.x = to_tf32(o.x);
      h.y = to_tf32(o.y);
      h.z = to_tf32(o.z);
      h.w = to_tf32(o.w);
      l.x = to_tf32(o.x - h.x);
      l.y = to_tf32(o.y - h.y);
      l.z = to_tf32(o.z - h.z);
      l.w = to_tf32(o.w - h.w);
      *reinterpret_cast<float4*>(hi + srow * 128 + lane * 4) = h;
      *reinterpret_cast<float4*>(lo + srow * 128 + lane * 4) = l;
    }
  }
}

// Scaled (optionally causal) softmax of score rows, one CTA per row (row
// width <= 16 * 256).  Row r is query position r % seq; causal rows keep keys
// 0..pos and write exact zeros beyond.  exp(s - max) in fp32, the sum in
// binary64, the quotient rounded once.
// The probabilities go straight into the TF32 split layout the P V product
// reads as its A operand: row r = head h (r / seq) and query i (r % seq) goes
// to row h * mp + i of [heads][mp][kp] hi and lo arrays; columns seq..kp-1
// are written as zeros (rows seq..mp-1 stay zero from allocation).  This
// replaces a separate split pass over the heads * seq * seq probabilities.
__global__ void __launch_bounds__(NT) attn_softmax_split_kernel(const float* __restrict__ s, uint32_t rows,
                                                                uint32_t width, uint32_t seq, float scale, int causal,
                                                                float* __restrict__ phi, float* __restrict__ plo,
                                                                uint32_t mp, uint32_t kp) {
  __shared__ double shd[NT / 32];
  __shared__ float shf[NT / 32];
  for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* row = s + static_cast<uint64_t>(r) * width;
    const uint32_t limit = causal ? (r % seq) + 1 : width;
    float v[NORM_VPT];
    float mx = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < NORM_VPT; ++i) {
      const uint32_t c = threadIdx.x + i * NT;
      v[i] = (c < limit) ? row[c] * scale : -FLT_MAX;
      mx = fmaxf(mx, v[i]);
    }
    mx = block_max_f(mx, shf);
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < NORM_VPT; ++i) {
      const uint32_t c = threadIdx.x + i * NT;
      v[i] = (c < limit) ? expf(v[i] - mx) : 0.f;
      sum += static_cast<double>(v[i]);
    }
    sum = block_sum_d(sum, shd);
    const double inv = 1.0 / sum;
    const uint64_t dst = (static_cast<uint64_t>(r / seq) * mp + (r % seq)) * kp;
#pragma unroll
    for (int i = 0; i < NORM_VPT; ++i) {
      const uint32_t c = threadIdx.x + i * NT;
      if (c < width) {
        const float p = static_cast<float>(static_cast<double>(v[i]) * inv);
        const float h = to_tf32(p);
        phi[dst + c] = h;
        plo[dst + c] = to_tf32(p - h);
      }
    }
    for (uint32_t c = width + threadIdx.x; c < kp; c += NT) {
      phi[dst + c] = 0.f;
      plo[dst + c] = 0.f;
    }
  }
}

// act[r, c] = f(gu[r, c]) * gu[r, F + c]; f = gelu_tanh (GeGLU) or silu (SwiGLU).
// With act_lo != null the product is written as its TF32 split (hi to act, lo to act_lo).
template <bool GELU>
__global__ void gated_act_kernel(const float* __restrict__ gu, float* __restrict__ act, uint32_t rows, uint32_t f,
                                 float* __restrict__ act_lo) {
  const uint64_t total4 = static_cast<uint64_t>(rows) * (f / 4);
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = i / (f / 4), c = (i % (f / 4)) * 4;
    const float4 g = *reinterpret_cast<const float4*>(gu + r * 2 * f + c);
    const float4 u = *reinterpret_cast<const float4*>(gu + r * 2 * f + f + c);
    float gv[4] = {g.x, g.y, g.z, g.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = gv[j];
      if constexpr (GELU) {
        o[j] = 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
      } else {
        o[j] = x / (1.f + expf(-x));
      }
    }
    float4 v = make_float4(o[0] * u.x, o[1] * u.y, o[2] * u.z, o[3] * u.w);
    if (act_lo != nullptr) {
      const float4 h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
      *reinterpret_cast<float4*>(act_lo + r * f + c) =
          make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
      v = h;
    }
    *reinterpret_cast<float4*>(act + r * f + c) = v;
  }
}

// 256-d sinusoidal embedding [cos | sin] of one timestep per batch item.
__global__ void timestep_embed_kernel(const float* __restrict__ t, float* __restrict__ out, uint32_t batch) {
  const uint32_t b = blockIdx.x, i = threadIdx.x;  // 128 threads
  if (b >= batch || i >= 128) return;
  const double f = exp(-log(10000.0) * static_cast<double>(i) / 128.0);
  const double a = static_cast<double>(t[b]) * f;
  out[b * 256 + i] = static_cast<float>(cos(a));
  out[b * 256 + 128 + i] = static_cast<float>(sin(a));
}

// adaLN parts [scale_a, gate_a, scale_m, gate_m, shift_a, shift_m] (each d):
// add the bias, then gate = tanh(gate) and scale = scale + 1 (canonical_reference.go:374-381).
__global__ void ada_prep_kernel(float* __restrict__ ada, const float* __restrict__ bias, uint32_t d, uint32_t batch) {
  const uint64_t total = static_cast<uint64_t>(batch) * 6 * d;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t j = static_cast<uint32_t>(i % (6ull * d));
    const uint32_t part = j / d;
    float v = ada[i] + bias[j];
    if (part == 1 || part == 3) v = tanhf(v);
    if (part == 0 || part == 2) v += 1.f;
    ada[i] = v;
  }
}

// The unmodulated block (a context refiner): scales 1, gates 1, shifts 0, so the
// fused norm / residual kernels compute norm(x) and x + y exactly.
__global__ void ada_identity_kernel(float* __restrict__ ada, uint32_t d, uint32_t batch) {
  const uint64_t total = static_cast<uint64_t>(batch) * 6 * d;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t part = static_cast<uint32_t>(i % (6ull * d)) / d;
    ada[i] = part < 4 ? 1.f : 0.f;
  }
}

uint32_t grid_for(uint64_t work, uint32_t per_block) {
  const uint64_t g = (work + per_block - 1) / per_block;
  return static_cast<uint32_t>(g < 148ull * 32 ? (g == 0 ? 1 : g) : 148ull * 32);
}

}  // namespace

// ---------------------------------------------------------------- NCCL (dlopen)
// The library does not link NCCL: the collective symbols are resolved at the
// first tensor-parallel object creation.
NcclApi& nccl() {
  static NcclApi n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    n.get_id = reinterpret_cast<NcclApi::GetUniqueIdFn>(dlsym(h, "ncclGetUniqueId"));
    n.init_rank = reinterpret_cast<NcclApi::CommInitRankFn>(dlsym(h, "ncclCommInitRank"));
    n.all_reduce = reinterpret_cast<NcclApi::AllReduceFn>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<NcclApi::AllGatherFn>(dlsym(h, "ncclAllGather"));
    n.destroy = reinterpret_cast<NcclApi::CommDestroyFn>(dlsym(h, "ncclCommDestroy"));
    n.error_string = reinterpret_cast<NcclApi::GetErrorStringFn>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_id && n.init_rank && n.all_reduce && n.all_gather && n.destroy;
  });
  return n;
}

namespace {
// Cross-rank waits of the fused tensor-parallel path: generous, since ranks
// may reach a forward at different times, but finite.
constexpr unsigned long long kPeerWaitNs = 10ull * 1000000000ull;
constexpr uint32_t kTpSlots = 5;  // 4 phases of a forward + the teardown barrier

}  // namespace

int nccl_unique_id(NcclUniqueIdBytes* out) {
  NcclApi& n = nccl();
  if (!n.ok) return -1;
  return n.get_id(out->bytes);
}

// ---------------------------------------------------------------- Block
Block::~Block() {
  teardown_peers();
  cudaDeviceSynchronize();  // the caller's last stream may already be gone
  for (void* p : allocs_) cudaFree(p);
  for (void* p : sym_raw_) cudaFree(p);
  if (comm_ != nullptr && nccl().ok) nccl().destroy(comm_);
}

float* Block::alloc(uint64_t floats) {
  void* p = nullptr;
  if (cudaMalloc(&p, floats * sizeof(float) + 1024) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  allocs_.push_back(p);
  return reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// A whole cudaMalloc allocation (offset 0), so that a peer's IPC mapping of it
// addresses the same bytes.
float* Block::sym_alloc(uint64_t floats) {
  void* p = nullptr;
  if (cudaMalloc(&p, floats * sizeof(float)) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  sym_raw_.push_back(p);
  return static_cast<float*>(p);
}

// Collective over the block's communicator (every rank calls it once, from
// init): all-gathers each rank's IPC handles, device UUID and choice; opens the
// peers' buffers.  The fused path is taken only if every rank asked for it and
// every rank runs on a different GPU (ranks sharing a GPU would wait on one
// another from separate launches); otherwise every rank stays on NCCL.
int Block::setup_peers() {
  const BlockDims& d = dims_;
  const uint32_t w = d.tp_world, me = d.tp_rank;
  struct Info {
    cudaIpcMemHandle_t h[4];
    unsigned char uuid[16];
    uint32_t want;
    uint32_t pad[3];
  };
  Info mine;
  std::memset(&mine, 0, sizeof(mine));
  mine.want = (rs_ != nullptr && ysym_ != nullptr && flags_ != nullptr && hbuf_ != nullptr) ? 1u : 0u;
  int dev = 0;
  cudaDeviceProp prop;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return -4;
  std::memcpy(mine.uuid, prop.uuid.bytes, 16);
  if (mine.want) {
    void* bufs[4] = {rs_, hbuf_, ysym_, flags_};
    for (int i = 0; i < 4; ++i)
      if (cudaIpcGetMemHandle(&mine.h[i], bufs[i]) != cudaSuccess) {
        (void)cudaGetLastError();
        mine.want = 0;
      }
  }
  std::vector<Info> all(w);
  unsigned char* dbuf = nullptr;
  if (cudaMalloc(&dbuf, sizeof(Info) * (w + 1)) != cudaSuccess) return -3;
  cudaError_t e = cudaMemcpyAsync(dbuf + sizeof(Info) * w, &mine, sizeof(Info), cudaMemcpyHostToDevice, stream_);
  int nrc = 0;
  if (e == cudaSuccess)
    nrc = nccl().all_gather(dbuf + sizeof(Info) * w, dbuf, sizeof(Info), kNcclInt8, comm_, stream_);
  if (e == cudaSuccess && nrc == 0)
    e = cudaMemcpyAsync(all.data(), dbuf, sizeof(Info) * w, cudaMemcpyDeviceToHost, stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  cudaFree(dbuf);
  if (e != cudaSuccess || nrc != 0) return -5;
  bool fused = true;
  for (uint32_t p = 0; p < w; ++p) {
    fused = fused && all[p].want == 1;
    for (uint32_t q = 0; q < p; ++q)
      if (std::memcmp(all[p].uuid, all[q].uuid, 16) == 0) fused = false;
  }
  if (!fused) return 0;  // NCCL all-reduce path
  std::vector<float*> rs(w), hb(w), yb(w);
  std::vector<uint64_t*> fl(w);
  for (uint32_t p = 0; p < w; ++p) {
    if (p == me) {
      rs[p] = rs_;
      hb[p] = hbuf_;
      yb[p] = ysym_;
      fl[p] = flags_;
      continue;
    }
    void* ptr[4] = {nullptr, nullptr, nullptr, nullptr};
    for (int i = 0; i < 4; ++i) {
      if (cudaIpcOpenMemHandle(&ptr[i], all[p].h[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        std::fprintf(stderr, "oct_b200: cudaIpcOpenMemHandle(rank %u buffer %d) failed\n", p, i);
        (void)cudaGetLastError();
        return -5;
      }
      peer_opened_.push_back(ptr[i]);
    }
    rs[p] = static_cast<float*>(ptr[0]);
    hb[p] = static_cast<float*>(ptr[1]);
    yb[p] = static_cast<float*>(ptr[2]);
    fl[p] = static_cast<uint64_t*>(ptr[3]);
  }
  void* arrays = nullptr;
  if (cudaMalloc(&arrays, 4 * w * sizeof(void*)) != cudaSuccess) return -3;
  allocs_.push_back(arrays);
  rs_peers_ = static_cast<float**>(arrays);
  h_peers_ = rs_peers_ + w;
  y_peers_ = h_peers_ + w;
  flag_peers_ = reinterpret_cast<uint64_t**>(y_peers_ + w);
  e = cudaMemcpyAsync(rs_peers_, rs.data(), w * sizeof(void*), cudaMemcpyHostToDevice, stream_);
  if (e == cudaSuccess) e = cudaMemcpyAsync(h_peers_, hb.data(), w * sizeof(void*), cudaMemcpyHostToDevice, stream_);
  if (e == cudaSuccess) e = cudaMemcpyAsync(y_peers_, yb.data(), w * sizeof(void*), cudaMemcpyHostToDevice, stream_);
  if (e == cudaSuccess) e = cudaMemcpyAsync(flag_peers_, fl.data(), w * sizeof(void*), cudaMemcpyHostToDevice, stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) return -4;
  fused_tp_ = true;
  return 0;
}

// Bounded barrier on the teardown slot (no rank unmaps or frees memory a peer
// may still write), then unmap the peers' buffers.
void Block::teardown_peers() {
  if (fused_tp_) {
    // on the default stream: the caller's last stream may already be destroyed
    cudaDeviceSynchronize();
    const uint64_t ep = epoch_ + 1;
    if (tp_signal(flag_peers_, kTpSlots - 1, dims_.tp_world, dims_.tp_rank, ep, nullptr) == cudaSuccess)
      (void)tp_wait(flags_, kTpSlots - 1, dims_.tp_world, ep, err_, kPeerWaitNs, nullptr);
    cudaDeviceSynchronize();
    fused_tp_ = false;
  }
  for (void* p : peer_opened_) cudaIpcCloseMemHandle(p);
  peer_opened_.clear();
}

// Publish this rank's stores of phase `slot`, then wait until every rank's are published.
cudaError_t Block::tp_phase(uint32_t slot) {
  return tp_signal_wait(flag_peers_, flags_, slot, dims_.tp_world, dims_.tp_rank, epoch_, err_, kPeerWaitNs, stream_);
}

static int block_cfg(uint32_t m, uint32_t n, const RowScatter* scatter);  // below, beside the products

int Block::init(const BlockDims& d, const NcclUniqueIdBytes* id, cudaStream_t stream) {
  dims_ = d;
  stream_ = stream;
  if (d.family != kGemma && d.family != kDit) return -1;
  if (d.hidden == 0 || d.heads == 0 || d.head_dim == 0 || d.ffn == 0 || d.seq_len == 0 || d.max_batch == 0) return -1;
  if (d.hidden > NORM_VPT * NT || d.seq_len > NORM_VPT * NT) return -2;  // fused row kernels' width limit
  if (d.hidden % 4 || d.ffn % 4 || d.head_dim % 8) return -2;
  if (d.family == kDit && (d.head_dim != 128 || d.kv_heads != d.heads || d.grid_w == 0)) return -2;
  if (d.family == kGemma && (d.kv_heads == 0 || d.heads % d.kv_heads)) return -2;
  const uint64_t T = static_cast<uint64_t>(d.max_batch) * d.seq_len;
  const uint32_t qkv_cols = (d.heads + 2 * d.kv_heads) * d.head_dim;
  const uint32_t attn_cols = d.heads * d.head_dim;
  // weights (pre-split hi/lo for the products, raw for gains / biases)
  auto split_alloc = [&](SplitW& w, uint32_t k, uint32_t n) {
    w.k = k;
    w.n = n;
    const uint64_t e = split_b_elems(n, k);
    w.hi = alloc(e);
    w.lo = alloc(e);
    return w.hi != nullptr && w.lo != nullptr;
  };
  bool ok = split_alloc(wqkv_, d.hidden, qkv_cols) && split_alloc(wo_, attn_cols, d.hidden) &&
            split_alloc(wgu_, d.hidden, 2 * d.ffn) && split_alloc(wd_, d.ffn, d.hidden);
  norm1_ = alloc(d.hidden);
  norm2_ = alloc(d.hidden);
  ok = ok && norm1_ && norm2_;
  if (d.family == kDit) {
    ada_w_ = alloc(256ull * 6 * d.hidden);
    ada_b_ = alloc(6ull * d.hidden);
    norm3_ = alloc(d.hidden);
    norm4_ = alloc(d.hidden);
    qn_ = alloc(d.head_dim);
    kn_ = alloc(d.head_dim);
    temb_ = alloc(256ull * d.max_batch);
    ada_ = alloc(6ull * d.hidden * d.max_batch);
    tsteps_ = alloc(d.max_batch);
    ok = ok && ada_w_ && ada_b_ && norm3_ && norm4_ && qn_ && kn_ && temb_ && ada_ && tsteps_;
  }
  // activations and workspaces
  // Fused tensor parallel wants hbuf_ (the all-gather target of the FFN input)
  // in a plain cudaMalloc allocation that peers can map.
  const char* tp_mode = std::getenv("OCT_B200_TP_COLLECTIVE");
  const bool want_fused_tp = d.tp_world > 1 && !(tp_mode != nullptr && std::strcmp(tp_mode, "nccl") == 0);
  // Without the peer-memory path, the producers of the products' A operands (norms,
  // gated activation, fused attention) write them straight in the TF32 split layout:
  // hi into hbuf_ / act_ / attn_, lo into hlo_ / actlo_ / attnlo_, rows padded to the
  // 256-row tile (the tensor maps read Mp rows), K a multiple of 32.
  split_producers_ = !want_fused_tp && d.hidden % 32 == 0 && d.ffn % 32 == 0 && attn_cols % 32 == 0;
  const uint64_t TP_rows = split_producers_ ? (T + 255) / 256 * 256 : T;
  hbuf_ = want_fused_tp ? sym_alloc(T * d.hidden) : alloc(TP_rows * d.hidden);
  if (split_producers_) {
    hlo_ = alloc(TP_rows * d.hidden);
    actlo_ = alloc(TP_rows * d.ffn);
    attnlo_ = alloc(TP_rows * attn_cols);
    ok = ok && hlo_ && actlo_ && attnlo_;
  }
  if (want_fused_tp) {
    const uint64_t rpr = (T + d.tp_world - 1) / d.tp_world;  // rows per rank at max_batch
    rs_ = sym_alloc(rpr * d.tp_world * kMaxScatterRanges * d.hidden);
    ysym_ = sym_alloc(T * d.hidden);
    flags_ = reinterpret_cast<uint64_t*>(sym_alloc(2ull * kTpSlots * d.tp_world));
    if (rs_ == nullptr || ysym_ == nullptr || flags_ == nullptr ||
        cudaMemsetAsync(flags_, 0, 8ull * kTpSlots * d.tp_world, stream_) != cudaSuccess)
      return -3;
  }
  qkv_ = alloc(T * qkv_cols);
  if (d.family == kDit) {
    fused_attn_ = flash_attention_supported(d.head_dim, d.seq_len);
    if (const char* mode = std::getenv("OCT_B200_DIT_ATTENTION"))
      if (std::strcmp(mode, "materialized") == 0) fused_attn_ = false;
  } else {
    fused_attn_ = flash_attention256_supported(d.head_dim, d.seq_len, d.heads, d.kv_heads);
    if (const char* mode = std::getenv("OCT_B200_GEMMA_ATTENTION"))
      if (std::strcmp(mode, "materialized") == 0) fused_attn_ = false;
  }
  if (fused_attn_) {
    // Q, K and V^T in the TF32 hi/lo per-head layouts of the fused kernel, all batch items
    const uint64_t e = T * attn_cols;
    const uint64_t ekv = T * static_cast<uint64_t>(d.kv_heads) * d.head_dim;
    qsplit_ = alloc(2 * e);
    ksplit_ = alloc(2 * ekv);
    vtsplit_ = alloc(2 * ekv);
    ok = ok && qsplit_ && ksplit_ && vtsplit_;
  } else {
    scores_ = alloc(static_cast<uint64_t>(d.max_batch) * d.heads * d.seq_len * d.seq_len);
    ok = ok && scores_;
  }
  attn_ = alloc(TP_rows * attn_cols);
  x1_ = alloc(T * d.hidden);
  proj_ = alloc(T * d.hidden);
  gu_ = alloc(T * 2ull * d.ffn);
  act_ = alloc(TP_rows * d.ffn);
  if (!fused_attn_) {
    // P in the TF32 split layout of the P V product, one batch item at a time
    const SplitDims pd = split_dims(d.seq_len, d.head_dim, d.seq_len);
    p_mp_ = pd.mp;
    p_kp_ = pd.kp;
    const uint64_t pe = static_cast<uint64_t>(d.max_batch) * d.heads * pd.mp * pd.kp;
    psplit_ = alloc(2 * pe);
    if (psplit_ == nullptr || cudaMemsetAsync(psplit_, 0, 2 * pe * sizeof(float), stream_) != cudaSuccess) return -3;
  }
  const uint64_t a_need = std::max({sgemm_tc_a_scratch_bytes(T, d.hidden), sgemm_tc_a_scratch_bytes(T, attn_cols),
                                    sgemm_tc_a_scratch_bytes(T, d.ffn)});
  const SplitDims vd = split_dims(1, d.head_dim, d.seq_len);  // V split of the P V product
  const uint64_t b_need =
      fused_attn_ ? 0
                  : std::max(sgemm_tc_scratch_bytes(d.seq_len, d.seq_len, d.head_dim, d.max_batch * d.heads),
                             static_cast<uint64_t>(2ull * sizeof(float) * d.max_batch * d.heads * vd.np * vd.kp));
  scratch_ = alloc(std::max(a_need, b_need) / sizeof(float) + 1);
  // split-K partials: the largest need of the products at the full token count
  // (shorter batches that would need more take fewer ranges)
  {
    const std::pair<uint32_t, uint32_t> nk[] = {{qkv_cols, d.hidden}, {d.hidden, attn_cols},
                                                {2 * d.ffn, d.hidden}, {d.hidden, d.ffn}};
    uint64_t cap = 0;
    for (const auto& p : nk) {
      const uint32_t n = p.first, kk = p.second;
      if (block_cfg(static_cast<uint32_t>(T), n, nullptr) != kTcSingle16) continue;
      const uint32_t r = sgemm_tc_pick_k_ranges(static_cast<uint32_t>(T), n, kk);
      if (r > 1) cap = std::max(cap, static_cast<uint64_t>(sgemm_tc_k_ranges(kk, r)) * T * n);
    }
    if (cap > 0) {
      splitk_ = alloc(cap);
      splitk_cap_ = splitk_ != nullptr ? cap : 0;
    }
  }
  err_ = reinterpret_cast<unsigned int*>(alloc(4));
  ok = ok && hbuf_ && qkv_ && attn_ && x1_ && proj_ && gu_ && act_ && scratch_ && err_;
  if (!ok) return -3;
  if (cudaMemsetAsync(err_, 0, 16, stream_) != cudaSuccess) return -4;
  if (split_producers_) {  // padding rows of the split operands start (and stay) zero
    const uint64_t rows = (T + 255) / 256 * 256;
    const std::pair<float*, uint64_t> bufs[] = {{hbuf_, d.hidden}, {hlo_, d.hidden}, {act_, d.ffn},
                                                {actlo_, d.ffn},   {attn_, attn_cols}, {attnlo_, attn_cols}};
    for (const auto& b : bufs)
      if (cudaMemsetAsync(b.first, 0, rows * b.second * sizeof(float), stream_) != cudaSuccess) return -4;
  }
  if (build_rope_tables() != 0) return -4;
  if (d.tp_world > 1) {
    if (!nccl().ok || id == nullptr) return -5;
    const int nrc = nccl().init_rank(&comm_, static_cast<int>(d.tp_world), *id, static_cast<int>(d.tp_rank));
    if (nrc != 0) {
      std::fprintf(stderr, "oct_b200: ncclCommInitRank(rank %u of %u) failed: %d (%s)\n", d.tp_rank, d.tp_world, nrc,
                   nccl().error_string != nullptr ? nccl().error_string(nrc) : "?");
      comm_ = nullptr;
      return -5;
    }
    const int prc = setup_peers();
    if (prc != 0) return prc;
  }
  return cudaStreamSynchronize(stream_) == cudaSuccess ? 0 : -4;
}

// RoPE tables, computed on the host exactly as the reference does.
int Block::build_rope_tables() {
  const BlockDims& d = dims_;
  const uint32_t half = d.head_dim / 2;
  std::vector<float> c(static_cast<size_t>(d.seq_len) * half), s(c.size());
  if (d.family == kGemma) {
    // inv_freq_i = base^(-2i/hd), angle = pos * inv_freq_i, evaluated in binary64.
    for (uint32_t p = 0; p < d.seq_len; ++p)
      for (uint32_t i = 0; i < half; ++i) {
        const double ang = static_cast<double>(p) * std::pow(static_cast<double>(d.rope_base),
                                                             -2.0 * static_cast<double>(i) / d.head_dim);
        c[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(ang));
        s[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(ang));
      }
  } else {
    // CanonicalRopeFrequency / CanonicalRopeRotate (canonical_contract.go:66-89): fp32
    // frequency and angle, cos/sin of the fp32 angle in binary64, rounded to fp32.
    static const uint32_t axes[3] = {32, 48, 48};
    for (uint32_t p = 0; p < d.seq_len; ++p) {
      // image tokens: (frame, row, column) of a grid_w-wide grid
      // (CanonicalImageTokenCoordinate, canonical_contract.go:53-64); caption / context
      // tokens: (first frame + p, 0, 0) (contextRope, context_refiner_reference.go:151-174)
      const float coord[3] = {static_cast<float>(d.rope_text ? d.rope_frame + p : d.rope_frame),
                              d.rope_text ? 0.f : static_cast<float>(p / d.grid_w),
                              d.rope_text ? 0.f : static_cast<float>(p % d.grid_w)};
      uint32_t pair = 0;
      for (int a = 0; a < 3; ++a)
        for (uint32_t q = 0; q < axes[a] / 2; ++q, ++pair) {
          const float freq = static_cast<float>(1.0 / std::pow(static_cast<double>(d.rope_base),
                                                               2.0 * static_cast<double>(q) / axes[a]));
          const float ang = coord[a] * freq;
          c[static_cast<size_t>(p) * half + pair] = static_cast<float>(std::cos(static_cast<double>(ang)));
          s[static_cast<size_t>(p) * half + pair] = static_cast<float>(std::sin(static_cast<double>(ang)));
        }
    }
  }
  rope_cos_ = alloc(c.size());
  rope_sin_ = alloc(s.size());
  if (rope_cos_ == nullptr || rope_sin_ == nullptr) return -3;
  if (cudaMemcpy(rope_cos_, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) return -4;
  if (cudaMemcpy(rope_sin_, s.data(), s.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) return -4;
  return 0;
}

int Block::set_weight(uint32_t slot, const float* src, uint64_t count, bool on_device) {
  const BlockDims& d = dims_;
  const uint32_t qkv_cols = (d.heads + 2 * d.kv_heads) * d.head_dim;
  const uint32_t attn_cols = d.heads * d.head_dim;
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  auto raw = [&](float* dst, uint64_t want) -> int {
    if (count != want || dst == nullptr) return -1;
    return cudaMemcpyAsync(dst, src, want * 4, kind, stream_) == cudaSuccess ? 0 : -4;
  };
  auto split = [&](SplitW& w, uint32_t k, uint32_t n) -> int {
    if (count != static_cast<uint64_t>(k) * n) return -1;
    const float* dsrc = src;
    float* staging = nullptr;
    if (!on_device) {
      if (cudaMalloc(&staging, count * 4) != cudaSuccess) return -4;
      if (cudaMemcpyAsync(staging, src, count * 4, cudaMemcpyHostToDevice, stream_) != cudaSuccess) {
        cudaFree(staging);
        return -4;
      }
      dsrc = staging;
    }
    cudaError_t e = sgemm_tc_split_b(dsrc, n, k, n, w.hi, w.lo, stream_);
    if (staging != nullptr) {
      cudaStreamSynchronize(stream_);
      cudaFree(staging);
    }
    return e == cudaSuccess ? 0 : -4;
  };
  int rc;
  if (d.family == kGemma) {
    switch (slot) {
      case kGemmaNorm1: rc = raw(norm1_, d.hidden); break;
      case kGemmaWqkv: rc = split(wqkv_, d.hidden, qkv_cols); break;
      case kGemmaWo: rc = split(wo_, attn_cols, d.hidden); break;
      case kGemmaNorm2: rc = raw(norm2_, d.hidden); break;
      case kGemmaWgu: rc = split(wgu_, d.hidden, 2 * d.ffn); break;
      case kGemmaWd: rc = split(wd_, d.ffn, d.hidden); break;
      default: return -1;
    }
  } else {
    switch (slot) {
      case kDitAdaW: rc = raw(ada_w_, 256ull * 6 * d.hidden); break;
      case kDitAdaB: rc = raw(ada_b_, 6ull * d.hidden); break;
      case kDitAttnNorm1: rc = raw(norm1_, d.hidden); break;
      case kDitWqkv: rc = split(wqkv_, d.hidden, qkv_cols); break;
      case kDitQNorm: rc = raw(qn_, d.head_dim); break;
      case kDitKNorm: rc = raw(kn_, d.head_dim); break;
      case kDitWo: rc = split(wo_, attn_cols, d.hidden); break;
      case kDitAttnNorm2: rc = raw(norm2_, d.hidden); break;
      case kDitFfnNorm1: rc = raw(norm3_, d.hidden); break;
      case kDitW13: rc = split(wgu_, d.hidden, 2 * d.ffn); break;
      case kDitW2: rc = split(wd_, d.ffn, d.hidden); break;
      case kDitFfnNorm2: rc = raw(norm4_, d.hidden); break;
      default: return -1;
    }
  }
  if (rc != 0) return rc;
  return cudaStreamSynchronize(stream_) == cudaSuccess ? 0 : -4;
}

// Products of at least 2048 x 2048 run on the CTA-pair kernel with 32-deep
// stages (faster under the power cap; same MMAs in the same order, so the same
// bits), those whose epilogue scatters rows to the tensor-parallel owners
// included; smaller ones on the single-CTA kernel.
static int block_cfg(uint32_t m, uint32_t n, const RowScatter* /*scatter*/) {
  return (m >= 2048 && n >= 2048) ? kTcPair32 : kTcSingle16;
}

// Single-CTA products under one wave of tiles (the tensor-parallel shards and
// short batches) run split K: a scattering product in up to kMaxScatterRanges
// ranges (its partials land in that many owner slots per rank), the others in
// as many as the partial buffer holds.  The count is fixed per block and
// product, from the block's largest token count, so a sequence's output does
// not depend on the batch it runs in (a product that takes the CTA-pair kernel
// at that count never splits; single and pair give the same bits); every rank
// takes the same decision.
uint32_t Block::k_ranges(uint32_t n, uint32_t k, bool scatter) const {
  const uint32_t tmax = dims_.max_batch * dims_.seq_len;
  if (block_cfg(tmax, n, nullptr) != kTcSingle16) return 1;
  const uint32_t r = sgemm_tc_pick_k_ranges(tmax, n, k);
  if (r <= 1) return 1;
  if (scatter) return std::min(r, kMaxScatterRanges);
  const uint64_t need = static_cast<uint64_t>(sgemm_tc_k_ranges(k, r)) * tmax * n;
  return need <= splitk_cap_ ? r : 1;
}

cudaError_t Block::gemm(const float* a, uint64_t lda, const SplitW& w, float* c, uint64_t ldc, uint32_t m,
                        const float* residual, uint64_t ldr, const RowScatter* scatter, uint32_t* ranges) {
  const int cfg = block_cfg(m, w.n, scatter);
  const bool scatters = scatter != nullptr && scatter->dst != nullptr;
  SplitK sk;
  if (cfg == kTcSingle16) {
    sk.ranges = k_ranges(w.n, w.k, scatters);
    sk.partial = splitk_;
  }
  if (ranges != nullptr) *ranges = sgemm_tc_k_ranges(w.k, sk.ranges);
  return sgemm_tc_presplit(a, lda, w.hi, w.lo, c, ldc, m, w.n, w.k, scratch_, err_, stream_, residual, ldr, cfg,
                           scatter, &sk);
}

cudaError_t Block::gemm_ab(const float* ahi, const float* alo, const SplitW& w, float* c, uint64_t ldc, uint32_t m,
                           const float* residual, uint64_t ldr) {
  const int cfg = block_cfg(m, w.n, nullptr);
  SplitK sk;
  if (cfg == kTcSingle16) {
    sk.ranges = k_ranges(w.n, w.k, false);
    sk.partial = splitk_;
  }
  return sgemm_tc_presplit_ab(ahi, alo, w.hi, w.lo, c, ldc, m, w.n, w.k, err_, stream_, residual, ldr, cfg, &sk);
}

cudaError_t Block::all_reduce(float* buf, uint64_t count) {
  if (dims_.tp_world <= 1) return cudaSuccess;
  return nccl().all_reduce(buf, buf, count, kNcclFloat32, kNcclSum, comm_, stream_) == 0 ? cudaSuccess
                                                                                          : cudaErrorUnknown;
}

// Attention of one batch item: scores = Q K^T per head (batched), softmax, O = P V.
// Materialised attention of every batch item at once: scores = Q K^T for each
// (item, head) entry as one strided-batched product, one softmax launch over all
// score rows, O = P V as one batched product.  Entry e = item * heads + head:
// operands step by head inside an item (stride) and by item (outer).
cudaError_t Block::attention(uint32_t batch, uint64_t ldq, uint32_t k_col, uint32_t v_col, bool shared_kv) {
  const BlockDims& d = dims_;
  const uint64_t S = d.seq_len, hd = d.head_dim;
  const uint32_t entries = batch * d.heads;
  GemmBatch qk;
  qk.count = entries;
  qk.inner = d.heads;
  qk.stride_a = hd;
  qk.outer_a = S * ldq;
  qk.stride_b = shared_kv ? 0 : hd;
  qk.outer_b = S * ldq;
  qk.stride_c = S * S;
  qk.outer_c = static_cast<uint64_t>(d.heads) * S * S;
  qk.b_trans = true;
  cudaError_t e = sgemm_tc(qkv_, ldq, qkv_ + k_col, ldq, scores_, S, S, S, hd, scratch_, err_, 16, stream_, nullptr,
                           &qk);
  if (e != cudaSuccess) return e;
  const uint64_t pe = static_cast<uint64_t>(d.max_batch) * d.heads * p_mp_ * p_kp_;  // one of P hi / P lo
  const uint64_t rows = static_cast<uint64_t>(entries) * S;
  attn_softmax_split_kernel<<<grid_for(rows, 1), NT, 0, stream_>>>(
      scores_, static_cast<uint32_t>(rows), S, S, 1.0f / std::sqrt(static_cast<float>(hd)),
      d.family == kGemma ? 1 : 0, psplit_, psplit_ + pe, p_mp_, p_kp_);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  GemmBatch pv;
  pv.count = entries;
  pv.inner = d.heads;
  pv.stride_b = shared_kv ? 0 : hd;
  pv.outer_b = S * ldq;
  const uint64_t ldo = static_cast<uint64_t>(d.heads) * hd;
  pv.stride_c = hd;
  pv.outer_c = S * ldo;
  return sgemm_tc_presplit_a(psplit_, psplit_ + pe, qkv_ + v_col, ldq, attn_, ldo, S, hd, S, scratch_, err_, stream_,
                             &pv);
}

int Block::forward(const float* x, float* y, uint32_t batch, const float* timesteps_host,
                   const float* temb_device) {
  const BlockDims& d = dims_;
  if (batch == 0 || batch > d.max_batch) return -1;
  const uint32_t T = batch * d.seq_len;
  const uint32_t qkv_cols = (d.heads + 2 * d.kv_heads) * d.head_dim;
  const uint32_t attn_cols = d.heads * d.head_dim;
  const bool lead = d.tp_rank == 0;  // rank that adds the residual into row-parallel partial sums
  cudaError_t e = cudaSuccess;
  auto ok = [&]() { return e == cudaSuccess && (e = cudaGetLastError()) == cudaSuccess; };
  // Fused tensor parallel (peer memory) when every rank owns an equal row share.
  const bool tpf = fused_tp_ && T % d.tp_world == 0;
  const uint32_t rpr = tpf ? T / d.tp_world : 0;
  // producers write the products' A operands already split (hi in the fp32 buffer, lo beside it)
  const bool sp = split_producers_ && !tpf;
  RowScatter sc;
  TpReduce red;
  if (tpf) {
    ++epoch_;  // every rank runs the same forwards, so the epochs agree
    sc.dst = rs_peers_;
    sc.rows_per_rank = rpr;
    sc.src_rank = d.tp_rank;
    sc.ld = d.hidden;
    red.slots = rs_;
    red.nslots = d.tp_world;
    red.slot_stride = static_cast<uint64_t>(rpr) * d.hidden;
    red.ld_slot = d.hidden;
    red.rows = rpr;
    red.row0 = d.tp_rank * rpr;
    red.width = d.hidden;
    red.rows_per_item = d.seq_len;
    red.eps = d.eps;
    red.npush = d.tp_world;
    red.ld_push = d.hidden;
  }
  if (d.family == kGemma) {
    norm_fused_kernel<<<grid_for(T, 1), NT, 0, stream_>>>(x, d.hidden, norm1_, d.eps, nullptr, nullptr, nullptr, 0,
                                                          nullptr, 0, d.seq_len, hbuf_, d.hidden, T, d.hidden,
                                                          sp ? hlo_ : nullptr);
    if (!ok()) return -4;
    e = sp ? gemm_ab(hbuf_, hlo_, wqkv_, qkv_, qkv_cols, T) : gemm(hbuf_, d.hidden, wqkv_, qkv_, qkv_cols, T);
    if (!ok()) return -4;
    const uint64_t rope_work = static_cast<uint64_t>(T) * (d.heads + d.kv_heads) * (d.head_dim / 2);
    rope_half_kernel<<<grid_for(rope_work, NT), NT, 0, stream_>>>(qkv_, qkv_cols, 0, d.heads + d.kv_heads,
                                                                 d.head_dim, rope_cos_, rope_sin_, d.seq_len, T);
    if (!ok()) return -4;
    if (fused_attn_) {
      // Q, K and V^T as TF32 splits in half-head layouts, then one fused causal launch
      const uint64_t se = static_cast<uint64_t>(T) * attn_cols;
      const uint64_t skv = static_cast<uint64_t>(T) * d.kv_heads * d.head_dim;
      const uint32_t halves = d.head_dim / 128;
      e = split_heads(qkv_, qkv_cols, batch, d.heads * halves, d.seq_len, qsplit_, qsplit_ + se, stream_);
      if (ok()) e = split_heads(qkv_ + attn_cols, qkv_cols, batch, d.kv_heads * halves, d.seq_len, ksplit_,
                                ksplit_ + skv, stream_);
      if (ok()) e = split_transpose_heads(qkv_ + attn_cols + static_cast<uint64_t>(d.kv_heads) * d.head_dim, qkv_cols,
                                          batch, d.kv_heads * halves, d.seq_len, vtsplit_, vtsplit_ + skv, stream_);
      if (!ok()) return -4;
      const AttnOperands ops{qsplit_, qsplit_ + se, ksplit_, ksplit_ + skv, vtsplit_, vtsplit_ + skv};
      e = flash_attention256_tf32x3(ops, attn_, attn_cols, batch, d.heads, d.kv_heads, d.seq_len,
                                    1.0f / std::sqrt(static_cast<float>(d.head_dim)), true, err_, stream_,
                                    sp ? attnlo_ : nullptr);
    } else {
      e = attention(batch, qkv_cols, attn_cols, attn_cols + d.kv_heads * d.head_dim, true);
    }
    if (!ok()) return -4;
    if (tpf) {
      // partial O Wo rows -> their owners; owners: x1 = x + sum, h = RMSNorm(x1) -> every rank
      uint32_t ranges = 1;
      e = gemm(attn_, attn_cols, wo_, rs_, d.hidden, T, nullptr, 0, &sc, &ranges);
      if (ok()) e = tp_phase(0);
      if (!ok()) return -4;
      TpReduce r = red;
      r.nslots = d.tp_world * ranges;  // each rank's partials arrive in `ranges` slots
      r.res = x;
      r.ld_res = d.hidden;
      r.keep = x1_;
      r.ld_keep = d.hidden;
      r.g2 = norm2_;
      r.push = h_peers_;
      e = tp_reduce_rows(r, stream_);
      if (ok()) e = tp_phase(1);
      if (!ok()) return -4;
    } else {
      e = (sp && fused_attn_) ? gemm_ab(attn_, attnlo_, wo_, x1_, d.hidden, T, lead ? x : nullptr, d.hidden)
                              : gemm(attn_, attn_cols, wo_, x1_, d.hidden, T, lead ? x : nullptr, d.hidden);  // x1 = x + O Wo
      if (ok()) e = all_reduce(x1_, static_cast<uint64_t>(T) * d.hidden);
      if (!ok()) return -4;
      norm_fused_kernel<<<grid_for(T, 1), NT, 0, stream_>>>(x1_, d.hidden, norm2_, d.eps, nullptr, nullptr, nullptr,
                                                            0, nullptr, 0, d.seq_len, hbuf_, d.hidden, T, d.hidden,
                                                            sp ? hlo_ : nullptr);
      if (!ok()) return -4;
    }
    e = sp ? gemm_ab(hbuf_, hlo_, wgu_, gu_, 2ull * d.ffn, T) : gemm(hbuf_, d.hidden, wgu_, gu_, 2ull * d.ffn, T);
    if (!ok()) return -4;
    gated_act_kernel<true><<<grid_for(static_cast<uint64_t>(T) * d.ffn / 4, NT), NT, 0, stream_>>>(
        gu_, act_, T, d.ffn, sp ? actlo_ : nullptr);
    if (!ok()) return -4;
    if (tpf) {
      // partial act Wd rows -> owners; owners: y = x1 + sum -> every rank
      uint32_t ranges = 1;
      e = gemm(act_, d.ffn, wd_, rs_, d.hidden, T, nullptr, 0, &sc, &ranges);
      if (ok()) e = tp_phase(2);
      if (!ok()) return -4;
      TpReduce r = red;
      r.nslots = d.tp_world * ranges;  // each rank's partials arrive in `ranges` slots
      r.res = x1_;
      r.ld_res = d.hidden;
      r.push = y_peers_;
      e = tp_reduce_rows(r, stream_);
      if (ok()) e = tp_phase(3);
      if (ok()) e = cudaMemcpyAsync(y, ysym_, static_cast<uint64_t>(T) * d.hidden * sizeof(float),
                                    cudaMemcpyDeviceToDevice, stream_);
      return ok() ? 0 : -4;
    }
    e = sp ? gemm_ab(act_, actlo_, wd_, y, d.hidden, T, lead ? x1_ : nullptr, d.hidden)  // y = x1 + act Wd
           : gemm(act_, d.ffn, wd_, y, d.hidden, T, lead ? x1_ : nullptr, d.hidden);
    if (ok()) e = all_reduce(y, static_cast<uint64_t>(T) * d.hidden);
    return ok() ? 0 : -4;
  }
  // ---- DiT
  if (d.unmodulated) {
    ada_identity_kernel<<<grid_for(6ull * d.hidden * batch, NT), NT, 0, stream_>>>(ada_, d.hidden, batch);
    if (!ok()) return -4;
  } else {
    if (temb_device != nullptr) {
      e = cudaMemcpyAsync(temb_, temb_device, 256ull * batch * sizeof(float), cudaMemcpyDeviceToDevice, stream_);
      if (!ok()) return -4;
    } else {
      if (timesteps_host == nullptr) return -1;
      e = cudaMemcpyAsync(tsteps_, timesteps_host, batch * sizeof(float), cudaMemcpyHostToDevice, stream_);
      if (!ok()) return -4;
      timestep_embed_kernel<<<batch, 128, 0, stream_>>>(tsteps_, temb_, batch);
      if (!ok()) return -4;
    }
    e = sgemm_fma(temb_, 256, ada_w_, 6ull * d.hidden, ada_, 6ull * d.hidden, batch, 6 * d.hidden, 256, stream_);
    if (!ok()) return -4;
    ada_prep_kernel<<<grid_for(6ull * d.hidden * batch, NT), NT, 0, stream_>>>(ada_, ada_b_, d.hidden, batch);
    if (!ok()) return -4;
  }
  const uint64_t ms = 6ull * d.hidden;
  float* scale_a = ada_;
  float* gate_a = ada_ + d.hidden;
  float* scale_m = ada_ + 2ull * d.hidden;
  float* gate_m = ada_ + 3ull * d.hidden;
  float* shift_a = ada_ + 4ull * d.hidden;
  float* shift_m = ada_ + 5ull * d.hidden;
  norm_fused_kernel<<<grid_for(T, 1), NT, 0, stream_>>>(x, d.hidden, norm1_, d.eps, scale_a, shift_a, nullptr, 0,
                                                        nullptr, ms, d.seq_len, hbuf_, d.hidden, T, d.hidden,
                                                        sp ? hlo_ : nullptr);
  if (!ok()) return -4;
  e = sp ? gemm_ab(hbuf_, hlo_, wqkv_, qkv_, qkv_cols, T) : gemm(hbuf_, d.hidden, wqkv_, qkv_, qkv_cols, T);
  if (!ok()) return -4;
  const uint64_t qk_warps = static_cast<uint64_t>(T) * d.heads;
  const uint64_t se = static_cast<uint64_t>(T) * attn_cols;  // elements of one split half (this batch)
  qk_norm_rope3_kernel<<<grid_for(qk_warps * 32, NT), NT, 0, stream_>>>(
      qkv_, qkv_cols, 0, d.heads, qn_, 1e-5f, rope_cos_, rope_sin_, d.seq_len, T, fused_attn_ ? qsplit_ : nullptr,
      fused_attn_ ? qsplit_ + se : nullptr);
  if (!ok()) return -4;
  qk_norm_rope3_kernel<<<grid_for(qk_warps * 32, NT), NT, 0, stream_>>>(
      qkv_, qkv_cols, attn_cols, d.heads, kn_, 1e-5f, rope_cos_, rope_sin_, d.seq_len, T,
      fused_attn_ ? ksplit_ : nullptr, fused_attn_ ? ksplit_ + se : nullptr);
  if (!ok()) return -4;
  if (fused_attn_) {
    // one fused launch over every (query tile, head, batch item)
    e = split_transpose_heads(qkv_ + 2ull * attn_cols, qkv_cols, batch, d.heads, d.seq_len, vtsplit_, vtsplit_ + se,
                              stream_);
    if (!ok()) return -4;
    const AttnOperands ops{qsplit_, qsplit_ + se, ksplit_, ksplit_ + se, vtsplit_, vtsplit_ + se};
    e = flash_attention_tf32x3(ops, attn_, attn_cols, batch, d.heads, d.seq_len,
                               1.0f / std::sqrt(static_cast<float>(d.head_dim)), err_, stream_,
                               sp ? attnlo_ : nullptr);
  } else {
    e = attention(batch, qkv_cols, attn_cols, 2 * attn_cols, false);
  }
  if (!ok()) return -4;
  if (tpf) {
    // partial attn Wo rows -> owners; owners: x1 = x + gate_a * RMSNorm(sum),
    // h = RMSNorm(x1) * scale_m + shift_m -> every rank
    uint32_t ranges = 1;
    e = gemm(attn_, attn_cols, wo_, rs_, d.hidden, T, nullptr, 0, &sc, &ranges);
    if (ok()) e = tp_phase(0);
    if (!ok()) return -4;
    TpReduce r = red;
    r.nslots = d.tp_world * ranges;  // each rank's partials arrive in `ranges` slots
    r.mod_stride = ms;
    r.g1 = norm2_;
    r.gate1 = gate_a;
    r.res = x;
    r.ld_res = d.hidden;
    r.keep = x1_;
    r.ld_keep = d.hidden;
    r.g2 = norm3_;
    r.mul2 = scale_m;
    r.add2 = shift_m;
    r.push = h_peers_;
    e = tp_reduce_rows(r, stream_);
    if (ok()) e = tp_phase(1);
    if (!ok()) return -4;
  } else {
    e = (sp && fused_attn_) ? gemm_ab(attn_, attnlo_, wo_, proj_, d.hidden, T)
                            : gemm(attn_, attn_cols, wo_, proj_, d.hidden, T);
    if (ok()) e = all_reduce(proj_, static_cast<uint64_t>(T) * d.hidden);
    if (!ok()) return -4;
    // res = x + gate_a * RMSNorm(proj)
    norm_fused_kernel<<<grid_for(T, 1), NT, 0, stream_>>>(proj_, d.hidden, norm2_, d.eps, nullptr, nullptr, x,
                                                          d.hidden, gate_a, ms, d.seq_len, x1_, d.hidden, T, d.hidden, nullptr);
    if (!ok()) return -4;
    norm_fused_kernel<<<grid_for(T, 1), NT, 0, stream_>>>(x1_, d.hidden, norm3_, d.eps, scale_m, shift_m, nullptr, 0,
                                                          nullptr, ms, d.seq_len, hbuf_, d.hidden, T, d.hidden,
                                                          sp ? hlo_ : nullptr);
    if (!ok()) return -4;
  }
  e = sp ? gemm_ab(hbuf_, hlo_, wgu_, gu_, 2ull * d.ffn, T) : gemm(hbuf_, d.hidden, wgu_, gu_, 2ull * d.ffn, T);
  if (!ok()) return -4;
  gated_act_kernel<false><<<grid_for(static_cast<uint64_t>(T) * d.ffn / 4, NT), NT, 0, stream_>>>(
      gu_, act_, T, d.ffn, sp ? actlo_ : nullptr);
  if (!ok()) return -4;
  if (tpf) {
    // partial act W2 rows -> owners; owners: y = x1 + gate_m * RMSNorm(sum) -> every rank
    uint32_t ranges = 1;
    e = gemm(act_, d.ffn, wd_, rs_, d.hidden, T, nullptr, 0, &sc, &ranges);
    if (ok()) e = tp_phase(2);
    if (!ok()) return -4;
    TpReduce r = red;
    r.nslots = d.tp_world * ranges;  // each rank's partials arrive in `ranges` slots
    r.mod_stride = ms;
    r.g1 = norm4_;
    r.gate1 = gate_m;
    r.res = x1_;
    r.ld_res = d.hidden;
    r.push = y_peers_;
    e = tp_reduce_rows(r, stream_);
    if (ok()) e = tp_phase(3);
    if (ok()) e = cudaMemcpyAsync(y, ysym_, static_cast<uint64_t>(T) * d.hidden * sizeof(float),
                                  cudaMemcpyDeviceToDevice, stream_);
    return ok() ? 0 : -4;
  }
  e = sp ? gemm_ab(act_, actlo_, wd_, proj_, d.hidden, T) : gemm(act_, d.ffn, wd_, proj_, d.hidden, T);
  if (ok()) e = all_reduce(proj_, static_cast<uint64_t>(T) * d.hidden);
  if (!ok()) return -4;
  // y = res + gate_m * RMSNorm(w2 out)
  norm_fused_kernel<<<grid_for(T, 1), NT, 0, stream_>>>(proj_, d.hidden, norm4_, d.eps, nullptr, nullptr, x1_,
                                                        d.hidden, gate_m, ms, d.seq_len, y, d.hidden, T, d.hidden, nullptr);
  return ok() ? 0 : -4;
}

unsigned int Block::read_status() {
  unsigned int v = 0;
  if (cudaMemcpyAsync(&v, err_, 4, cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
      cudaStreamSynchronize(stream_) != cudaSuccess)
    return 0xFFFFFFFFu;
  cudaMemsetAsync(err_, 0, 4, stream_);
  return v;
}

}  // namespace oct
