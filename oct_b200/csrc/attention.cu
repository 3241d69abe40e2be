// attention.cu -- fused exact attention on the sm_100a tensor cores (3xTF32).
//
// O = softmax(Q K^T * scale) V for heads of 128 channels, bidirectional: the
// attention of the Z-Image block (`canonicalAttention`,
// internal/prometheus/zimage/canonical_reference.go:241-289).  The score
// matrix never leaves the SM: per CTA, 128 queries of one head stream over the
// keys in blocks of 32 with the online (running max / running sum) softmax.
//
// Operands are pre-split to TF32 hi/lo like every other product here
// (x = hi + lo, three products hi*hi + hi*lo + lo*hi), laid out per head:
//   Q hi/lo   [items*heads*S][128]   rows = queries  (A of Q K^T, loaded into TMEM)
//   K hi/lo   [items*heads*S][128]   rows = keys     (K-major B of Q K^T)
//   V^T hi/lo [items*heads*128][S]   rows = channels (K-major B of P V)
// Tensor memory (512 columns of 128 lanes; lane = query row of the tile):
//   [0,128) Q hi  [128,256) Q lo       A operands of Q K^T, written once
//   [256,288) S main  [288,320) S corr score block: hi*hi, and hi*lo + lo*hi
//   [320,352) P hi  [352,384) P lo     A operands of P V, written by the softmax warps
//   [384,512) O block                  P V of one key block
// The round-toward-zero TMEM accumulation only ever sums one 128-channel dot
// product (S) or 32 keys (O block); every O block is merged into fp32 running
// sums in registers with round-to-nearest, so the result keeps fp32 accuracy.
//
// Warp roles (320 threads, one CTA per SM): warp 0 TMA producer (K and V^T
// blocks through a 3-stage ring), warp 1 MMA issuer, warps 2-5 softmax
// (S -> P, one query row per thread), warps 6-9 correction (the fp32 output
// sums of the same rows, merged from each P V block; they take each row's
// rescale factor from the softmax warps through shared memory).  Every wait
// is bounded (ptx.cuh); on a timeout the kernel records the error bit, drains
// its MMAs and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace oct {
namespace {

constexpr uint32_t FA_BQ = 128;   // queries per CTA
constexpr uint32_t FA_BKV = 32;   // keys per block
constexpr uint32_t FA_HD = 128;   // channels per head
constexpr uint32_t FA_STAGES = 3;
constexpr uint32_t FA_K_BYTES = FA_BKV * FA_HD * 4;   // 16 KB: one of K hi / K lo
constexpr uint32_t FA_V_BYTES = FA_HD * FA_BKV * 4;   // 16 KB: one of V^T hi / lo
constexpr uint32_t FA_STAGE_BYTES = 2 * FA_K_BYTES + 2 * FA_V_BYTES;
constexpr uint32_t FA_SMEM = FA_STAGES * FA_STAGE_BYTES + 1024;
constexpr int FA_THREADS = 320;
constexpr uint32_t COL_QHI = 0, COL_QLO = 128, COL_SM = 256, COL_SC = 288, COL_PHI = 320, COL_PLO = 352,
                   COL_O = 384;

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::tf32, A K-major in tensor memory.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Named barrier 1: the MMA warp and the eight softmax / correction warps
// (Q hi/lo are in tensor memory).
__device__ __forceinline__ void q_ready_barrier() { asm volatile("bar.sync 1, 288;" ::: "memory"); }

// The running max of a row moves only when a key block's max exceeds it by
// more than FA_TAU (natural-log units): probabilities then stay below e^8 in
// fp32, and the rescale of the output sums is skipped in almost every block.
constexpr float FA_TAU = 8.0f;

__global__ void __launch_bounds__(FA_THREADS, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tm_khi, const __grid_constant__ CUtensorMap tm_klo,
                      const __grid_constant__ CUtensorMap tm_vhi, const __grid_constant__ CUtensorMap tm_vlo,
                      const float* __restrict__ qhi, const float* __restrict__ qlo, float* __restrict__ out,
                      uint64_t ldo, uint32_t heads, uint32_t seq, float scale, unsigned int* __restrict__ err,
                      float* __restrict__ out_lo) {
  constexpr uint32_t IDESC_S = umma_idesc_tf32(FA_BQ, FA_BKV);
  constexpr uint32_t IDESC_O = umma_idesc_tf32(FA_BQ, FA_HD);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t kv_full[FA_STAGES], kv_empty[FA_STAGES];
  __shared__ __align__(8) uint64_t s_full, s_empty, p_full, o_full, o_empty, drain_bar;
  __shared__ __align__(8) uint64_t alpha_full[2], l_ready;
  __shared__ float alpha_sh[2][FA_BQ];  // per-row rescale factor of key block j, slot (j - 1) & 1
  __shared__ float inv_l_sh[FA_BQ];     // per-row 1 / sum of probabilities
  __shared__ uint32_t tmem_slot;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t qtile = blockIdx.x, head = blockIdx.y, item = blockIdx.z;
  const uint32_t nb = seq / FA_BKV;
  const uint64_t slab = static_cast<uint64_t>(item) * heads + head;  // (item, head) index
  const int key_row0 = static_cast<int>(slab * seq);                 // first row in K hi/lo
  const int vt_row0 = static_cast<int>(slab * FA_HD);                // first row in V^T hi/lo

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < FA_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_empty, 4);
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
    mbar_init(&o_empty, 4);
    mbar_init(&drain_bar, 1);
    mbar_init(&alpha_full[0], 4);
    mbar_init(&alpha_full[1], 4);
    mbar_init(&l_ready, 4);
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tensormap(&tm_khi);
    prefetch_tensormap(&tm_klo);
    prefetch_tensormap(&tm_vhi);
    prefetch_tensormap(&tm_vlo);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: K block = 4 boxes of 32 channels x 32 keys (hi, lo); V^T block = 1 box
      for (uint32_t j = 0; j < nb; ++j) {
        const uint32_t st = j % FA_STAGES;
        if (j >= FA_STAGES && !mbar_wait(&kv_empty[st], ((j / FA_STAGES) - 1) & 1u, err, kErrWaitEmpty)) break;
        uint8_t* base = smem + st * FA_STAGE_BYTES;
        mbar_arrive_expect_tx(&kv_full[st], FA_STAGE_BYTES);
        const int krow = key_row0 + static_cast<int>(j * FA_BKV);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          tma_load_2d(base + a * 4096, &tm_khi, &kv_full[st], a * 32, krow);
          tma_load_2d(base + FA_K_BYTES + a * 4096, &tm_klo, &kv_full[st], a * 32, krow);
        }
        tma_load_2d(base + 2 * FA_K_BYTES, &tm_vhi, &kv_full[st], static_cast<int>(j * FA_BKV), vt_row0);
        tma_load_2d(base + 2 * FA_K_BYTES + FA_V_BYTES, &tm_vlo, &kv_full[st], static_cast<int>(j * FA_BKV),
                    vt_row0);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop converged (descriptors stay
    // warp-uniform); one elected lane issues each tcgen05 instruction.
    q_ready_barrier();
    tc_fence_after();
    auto issue_pv = [&](uint32_t jj) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(&p_full, jj & 1u, err, kErrWaitAccum))) return false;
      if (jj >= 1 && !__all_sync(0xffffffffu, mbar_wait(&o_empty, (jj - 1) & 1u, err, kErrWaitAccum))) return false;
      tc_fence_after();
      const uint32_t st = jj % FA_STAGES;
      const uint32_t vbase = smem_addr(smem + st * FA_STAGE_BYTES + 2 * FA_K_BYTES);
#pragma unroll
      for (uint32_t kk = 0; kk < FA_BKV / 8; ++kk) {
        const uint64_t dvh = umma_desc_kmajor(vbase + kk * 32, 128);
        const uint64_t dvl = umma_desc_kmajor(vbase + FA_V_BYTES + kk * 32, 128);
        if (elect_one()) {
          umma_tf32_ts(tmem + COL_O, tmem + COL_PHI + kk * 8, dvl, IDESC_O, kk != 0 ? 1u : 0u);
          umma_tf32_ts(tmem + COL_O, tmem + COL_PLO + kk * 8, dvh, IDESC_O, 1u);
          umma_tf32_ts(tmem + COL_O, tmem + COL_PHI + kk * 8, dvh, IDESC_O, 1u);
        }
        __syncwarp();
      }
      if (elect_one()) {
        umma_commit(&o_full);
        umma_commit(&kv_empty[st]);
      }
      __syncwarp();
      return true;
    };
    bool ok = true;
    for (uint32_t j = 0; j < nb && ok; ++j) {
      const uint32_t st = j % FA_STAGES;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[st], (j / FA_STAGES) & 1u, err, kErrWaitFull))) {
        ok = false;
        break;
      }
      if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(&s_empty, (j - 1) & 1u, err, kErrWaitAccum))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t kbase = smem_addr(smem + st * FA_STAGE_BYTES);
#pragma unroll
      for (uint32_t kk = 0; kk < FA_HD / 8; ++kk) {
        const uint32_t koff = (kk >> 2) * 4096 + (kk & 3) * 32;  // box of 32 channels, 8 channels per step
        const uint64_t dkh = umma_desc_kmajor(kbase + koff, 128);
        const uint64_t dkl = umma_desc_kmajor(kbase + FA_K_BYTES + koff, 128);
        if (elect_one()) {
          umma_tf32_ts(tmem + COL_SM, tmem + COL_QHI + kk * 8, dkh, IDESC_S, kk != 0 ? 1u : 0u);
          umma_tf32_ts(tmem + COL_SC, tmem + COL_QHI + kk * 8, dkl, IDESC_S, kk != 0 ? 1u : 0u);
          umma_tf32_ts(tmem + COL_SC, tmem + COL_QLO + kk * 8, dkh, IDESC_S, 1u);
        }
        __syncwarp();
      }
      if (elect_one()) umma_commit(&s_full);
      __syncwarp();
      if (j >= 1) ok = issue_pv(j - 1);
    }
    if (ok && nb > 0) ok = issue_pv(nb - 1);
    if (elect_one()) umma_commit(&drain_bar);
    __syncwarp();
  } else {
    // warps 2..5: softmax (S -> P); warps 6..9: correction (merge P V blocks into the output sums).
    // Thread = one query row = one TMEM lane; a warp may only touch TMEM lanes 32 * (warp % 4) ...
    const bool softmax = warp < 6;
    const uint32_t quad = warp & 3u;
    const uint32_t row = quad * 32 + lane;
    const uint32_t lane_addr = (quad * 32u) << 16;
    {
      // Q hi (softmax warps) / Q lo (correction warps) -> TMEM, 32 channels at a time
      const uint64_t qrow = slab * seq + static_cast<uint64_t>(qtile) * FA_BQ + row;
      const float* src = (softmax ? qhi : qlo) + qrow * FA_HD;
      const uint32_t col = softmax ? COL_QHI : COL_QLO;
#pragma unroll 1
      for (uint32_t c0 = 0; c0 < FA_HD; c0 += 32) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(src + c0 + i));
          r[i] = __float_as_uint(v.x);
          r[i + 1] = __float_as_uint(v.y);
          r[i + 2] = __float_as_uint(v.z);
          r[i + 3] = __float_as_uint(v.w);
        }
        tmem_st_32x32b_x32(tmem + lane_addr + col + c0, r);
      }
      tmem_st_wait();
    }
    tc_fence_before();
    q_ready_barrier();

    if (softmax) {
      float m_run = -FLT_MAX;
      double l_run = 0.0;
      for (uint32_t j = 0; j < nb; ++j) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full, j & 1u, err, kErrWaitAccum))) break;
        tc_fence_after();
        float p[32];
        {
          uint32_t sm[32], sc[32];
          tmem_ld_32x32b_x32(tmem + lane_addr + COL_SM, sm);
          tmem_ld_32x32b_x32(tmem + lane_addr + COL_SC, sc);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) p[i] = (__uint_as_float(sm[i]) + __uint_as_float(sc[i])) * scale;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty);
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = fmaxf(p[i], p[i + 16]);
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) t[i] = fmaxf(t[i], t[i + w]);
        const float mx = t[0];
        const float m_new = (mx > m_run + FA_TAU) ? mx : m_run;  // the first block always moves it
        const float alpha = (m_new == m_run) ? 1.0f : expf(m_run - m_new);
#pragma unroll
        for (int i = 0; i < 32; ++i) p[i] = expf(p[i] - m_new);
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = p[i] + p[i + 16];
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) t[i] += t[i + w];
        l_run = l_run * static_cast<double>(alpha) + static_cast<double>(t[0]);
        m_run = m_new;
        if (j >= 1) {
          // hand the rescale factor of this block to the correction warps, then
          // wait until P V of the previous block has read the P buffer
          alpha_sh[(j - 1) & 1u][row] = alpha;
          __syncwarp();
          if (lane == 0) mbar_arrive(&alpha_full[(j - 1) & 1u]);
          if (!__all_sync(0xffffffffu, mbar_wait(&o_full, (j - 1) & 1u, err, kErrWaitAccum))) break;
          tc_fence_after();
        }
        {
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float h = to_tf32(p[i]);
            ph[i] = __float_as_uint(h);
            pl[i] = __float_as_uint(to_tf32(p[i] - h));
          }
          tmem_st_32x32b_x32(tmem + lane_addr + COL_PHI, ph);
          tmem_st_32x32b_x32(tmem + lane_addr + COL_PLO, pl);
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full);
      }
      inv_l_sh[row] = static_cast<float>(1.0 / l_run);
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_ready);
    } else {
      float o_run[FA_HD];
#pragma unroll
      for (int i = 0; i < static_cast<int>(FA_HD); ++i) o_run[i] = 0.f;
      bool ok = true;
      for (uint32_t j = 1; j < nb; ++j) {
        // o_run (relative to the previous max) += P_{j-1} V_{j-1}, then * alpha_j
        ok = __all_sync(0xffffffffu, mbar_wait(&alpha_full[(j - 1) & 1u], ((j - 1) >> 1) & 1u, err, kErrWaitAccum) &&
                                         mbar_wait(&o_full, (j - 1) & 1u, err, kErrWaitAccum));
        if (!ok) break;
        tc_fence_after();
        const float alpha = alpha_sh[(j - 1) & 1u][row];
        const bool rescale = __any_sync(0xffffffffu, alpha != 1.0f);
#pragma unroll
        for (uint32_t g = 0; g < FA_HD / 32; ++g) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_addr + COL_O + g * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o_run[g * 32 + i] += __uint_as_float(r[i]);
          if (rescale) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o_run[g * 32 + i] *= alpha;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty);
      }
      if (ok && nb > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&o_full, (nb - 1) & 1u, err, kErrWaitAccum) &&
                                         mbar_wait(&l_ready, 0, err, kErrWaitAccum));
        if (ok) {
          tc_fence_after();
          const float inv = inv_l_sh[row];
          const uint64_t o = (static_cast<uint64_t>(item) * seq + static_cast<uint64_t>(qtile) * FA_BQ + row) * ldo +
                             static_cast<uint64_t>(head) * FA_HD;
          float* dst = out + o;
          float* dst_lo = out_lo != nullptr ? out_lo + o : nullptr;  // TF32 split for the next product
#pragma unroll
          for (uint32_t g = 0; g < FA_HD / 32; ++g) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + COL_O + g * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const int c = static_cast<int>(g * 32) + i;
              float4 v = make_float4((o_run[c] + __uint_as_float(r[i])) * inv,
                                     (o_run[c + 1] + __uint_as_float(r[i + 1])) * inv,
                                     (o_run[c + 2] + __uint_as_float(r[i + 2])) * inv,
                                     (o_run[c + 3] + __uint_as_float(r[i + 3])) * inv);
              if (dst_lo != nullptr) {
                const float4 h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
                *reinterpret_cast<float4*>(dst_lo + c) =
                    make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
                v = h;
              }
              *reinterpret_cast<float4*>(dst + c) = v;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 32) mbar_wait(&drain_bar, 0, err, kErrWaitDrain);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ 256-channel heads, CTA pair
// Gemma's attention: heads of 256 channels, optionally causal, K / V heads shared
// by groups of query heads (MQA: one K / V head).  Q hi/lo of a 256-channel head
// would fill all 512 TMEM columns, so a cluster of two CTAs takes one 128-query
// tile and each CTA works on one 128-channel half of the head: CTA r holds Q
// channels [128 r, 128 r + 128) in its TMEM, streams the same channels of K and
// V^T, and computes a partial score block S_r = Q_r K_r^T (exactly as
// flash_attn_kernel computes a 128-channel head).  The softmax warps of each CTA
// send their partial block to the other CTA through distributed shared memory and
// add the two: S_0 + S_1 in one CTA and S_1 + S_0 in the other are the same fp32
// sums (addition commutes), so both CTAs form the same probabilities, and each
// accumulates the output for its 128 channels.  The operands use the 128-channel
// layouts of flash_attn_kernel with each 256-channel head taken as two half heads
// (half head 2 h + r), which split_heads / split_transpose_heads produce.
// Causal: query position q sees keys 0 .. q; a 128-query tile stops after its
// diagonal key blocks, and the largest tiles start first.
// Shared memory: a 2-slot ring of K blocks (hi, lo) and a 2-slot ring of V^T
// blocks (hi, lo), so a K slot frees as soon as its scores are computed, and a
// double-buffered exchange area that the other CTA writes.  The score exchange
// is software-pipelined: a CTA sends its partial block j + 1 before it works on
// block j, so the partial it needs has normally arrived by the time it looks.
// Exchange layout, group-major: [FA_BKV / 4 groups][128 rows][4 floats], so each 16-byte
// remote store instruction of a warp writes 512 contiguous bytes, and the local 16-byte reads
// of consecutive rows are conflict-free.
constexpr uint32_t FA2_RING = 2;
constexpr uint32_t FA2_K_STAGE = 2 * FA_K_BYTES;  // K hi, K lo of one key block
constexpr uint32_t FA2_V_STAGE = 2 * FA_V_BYTES;  // V^T hi, V^T lo of one key block
constexpr uint32_t FA2_SX_FLOATS = FA_BQ * FA_BKV;
constexpr uint32_t FA2_SX_BYTES = FA2_SX_FLOATS * 4;
constexpr uint32_t FA2_SMEM = FA2_RING * (FA2_K_STAGE + FA2_V_STAGE) + 2 * FA2_SX_BYTES + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(FA_THREADS, 1)
    flash_attn_pair_kernel(const __grid_constant__ CUtensorMap tm_khi, const __grid_constant__ CUtensorMap tm_klo,
                           const __grid_constant__ CUtensorMap tm_vhi, const __grid_constant__ CUtensorMap tm_vlo,
                           const float* __restrict__ qhi, const float* __restrict__ qlo, float* __restrict__ out,
                           uint64_t ldo, uint32_t heads, uint32_t kv_heads, uint32_t seq, float scale,
                           uint32_t causal, unsigned int* __restrict__ err, float* __restrict__ out_lo) {
  constexpr uint32_t IDESC_S = umma_idesc_tf32(FA_BQ, FA_BKV);
  constexpr uint32_t IDESC_O = umma_idesc_tf32(FA_BQ, FA_HD);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kring = smem;
  uint8_t* vring = smem + FA2_RING * FA2_K_STAGE;
  float* sx = reinterpret_cast<float*>(vring + FA2_RING * FA2_V_STAGE);  // [2][8][128][4], written by the peer
  __shared__ __align__(8) uint64_t k_full[FA2_RING], k_empty[FA2_RING], v_full[FA2_RING], v_empty[FA2_RING];
  __shared__ __align__(8) uint64_t s_full, s_empty, p_full, o_full, o_empty, drain_bar;
  __shared__ __align__(8) uint64_t alpha_full[2], l_ready, sx_full[2], sx_empty[2];
  __shared__ float alpha_sh[2][FA_BQ];
  __shared__ float inv_l_sh[FA_BQ];
  __shared__ uint32_t tmem_slot;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank(), peer = rank ^ 1u;
  const uint32_t tiles = seq / FA_BQ;
  const uint32_t qtile = tiles - 1u - (blockIdx.x >> 1);  // largest causal tiles first
  const uint32_t head = blockIdx.y, item = blockIdx.z;
  const uint32_t nb = causal ? (qtile + 1u) * (FA_BQ / FA_BKV) : seq / FA_BKV;
  const uint32_t kv_head = head / (heads / kv_heads);
  const uint64_t qslab = (static_cast<uint64_t>(item) * heads + head) * 2 + rank;       // half head of Q
  const uint64_t kvslab = (static_cast<uint64_t>(item) * kv_heads + kv_head) * 2 + rank;  // half head of K, V
  const int key_row0 = static_cast<int>(kvslab * seq);
  const int vt_row0 = static_cast<int>(kvslab * FA_HD);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < FA2_RING; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_empty, 4);
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
    mbar_init(&o_empty, 4);
    mbar_init(&drain_bar, 1);
    mbar_init(&alpha_full[0], 4);
    mbar_init(&alpha_full[1], 4);
    mbar_init(&l_ready, 4);
    for (uint32_t b = 0; b < 2; ++b) {
      mbar_init(&sx_full[b], 4);   // the peer's softmax warps, after their stores into buffer b
      mbar_init(&sx_empty[b], 4);  // the peer's softmax warps, after reading what this CTA sent into buffer b
    }
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tensormap(&tm_khi);
    prefetch_tensormap(&tm_klo);
    prefetch_tensormap(&tm_vhi);
    prefetch_tensormap(&tm_vlo);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (uint32_t j = 0; j < nb; ++j) {
        const uint32_t st = j % FA2_RING, ph = ((j / FA2_RING) - 1) & 1u;
        if (j >= FA2_RING && !mbar_wait(&k_empty[st], ph, err, kErrWaitEmpty)) break;
        uint8_t* kb = kring + st * FA2_K_STAGE;
        mbar_arrive_expect_tx(&k_full[st], FA2_K_STAGE);
        const int krow = key_row0 + static_cast<int>(j * FA_BKV);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          tma_load_2d(kb + a * 4096, &tm_khi, &k_full[st], a * 32, krow);
          tma_load_2d(kb + FA_K_BYTES + a * 4096, &tm_klo, &k_full[st], a * 32, krow);
        }
        if (j >= FA2_RING && !mbar_wait(&v_empty[st], ph, err, kErrWaitEmpty)) break;
        uint8_t* vb = vring + st * FA2_V_STAGE;
        mbar_arrive_expect_tx(&v_full[st], FA2_V_STAGE);
        tma_load_2d(vb, &tm_vhi, &v_full[st], static_cast<int>(j * FA_BKV), vt_row0);
        tma_load_2d(vb + FA_V_BYTES, &tm_vlo, &v_full[st], static_cast<int>(j * FA_BKV), vt_row0);
      }
    }
  } else if (warp == 1) {
    q_ready_barrier();
    tc_fence_after();
    auto issue_pv = [&](uint32_t jj) -> bool {
      const uint32_t st = jj % FA2_RING;
      if (!__all_sync(0xffffffffu, mbar_wait(&p_full, jj & 1u, err, kErrWaitAccum))) return false;
      if (jj >= 1 && !__all_sync(0xffffffffu, mbar_wait(&o_empty, (jj - 1) & 1u, err, kErrWaitAccum))) return false;
      if (!__all_sync(0xffffffffu, mbar_wait(&v_full[st], (jj / FA2_RING) & 1u, err, kErrWaitFull))) return false;
      tc_fence_after();
      const uint32_t vbase = smem_addr(vring + st * FA2_V_STAGE);
#pragma unroll
      for (uint32_t kk = 0; kk < FA_BKV / 8; ++kk) {
        const uint64_t dvh = umma_desc_kmajor(vbase + kk * 32, 128);
        const uint64_t dvl = umma_desc_kmajor(vbase + FA_V_BYTES + kk * 32, 128);
        if (elect_one()) {
          umma_tf32_ts(tmem + COL_O, tmem + COL_PHI + kk * 8, dvl, IDESC_O, kk != 0 ? 1u : 0u);
          umma_tf32_ts(tmem + COL_O, tmem + COL_PLO + kk * 8, dvh, IDESC_O, 1u);
          umma_tf32_ts(tmem + COL_O, tmem + COL_PHI + kk * 8, dvh, IDESC_O, 1u);
        }
        __syncwarp();
      }
      if (elect_one()) {
        umma_commit(&o_full);
        umma_commit(&v_empty[st]);
      }
      __syncwarp();
      return true;
    };
    // Q K^T of block jj (single TMEM score buffer: the softmax warps have loaded block jj - 1)
    auto issue_s = [&](uint32_t jj) -> bool {
      const uint32_t st = jj % FA2_RING;
      if (!__all_sync(0xffffffffu, mbar_wait(&k_full[st], (jj / FA2_RING) & 1u, err, kErrWaitFull))) return false;
      if (jj >= 1 && !__all_sync(0xffffffffu, mbar_wait(&s_empty, (jj - 1) & 1u, err, kErrWaitAccum))) return false;
      tc_fence_after();
      const uint32_t kbase = smem_addr(kring + st * FA2_K_STAGE);
#pragma unroll
      for (uint32_t kk = 0; kk < FA_HD / 8; ++kk) {
        const uint32_t koff = (kk >> 2) * 4096 + (kk & 3) * 32;
        const uint64_t dkh = umma_desc_kmajor(kbase + koff, 128);
        const uint64_t dkl = umma_desc_kmajor(kbase + FA_K_BYTES + koff, 128);
        if (elect_one()) {
          umma_tf32_ts(tmem + COL_SM, tmem + COL_QHI + kk * 8, dkh, IDESC_S, kk != 0 ? 1u : 0u);
          umma_tf32_ts(tmem + COL_SC, tmem + COL_QHI + kk * 8, dkl, IDESC_S, kk != 0 ? 1u : 0u);
          umma_tf32_ts(tmem + COL_SC, tmem + COL_QLO + kk * 8, dkh, IDESC_S, 1u);
        }
        __syncwarp();
      }
      if (elect_one()) {
        umma_commit(&s_full);
        umma_commit(&k_empty[st]);
      }
      __syncwarp();
      return true;
    };
    // The scores run two blocks ahead of P V: the softmax warps fetch (and send)
    // block j + 1 before they finish block j, so S(j + 2) can start before P(j) exists.
    bool ok = nb > 0 && issue_s(0);
    if (ok && nb > 1) ok = issue_s(1);
    for (uint32_t j = 0; j < nb && ok; ++j) {
      if (j + 2 < nb) ok = issue_s(j + 2);
      if (ok) ok = issue_pv(j);
    }
    if (elect_one()) umma_commit(&drain_bar);
    __syncwarp();
  } else {
    const bool softmax = warp < 6;
    const uint32_t quad = warp & 3u;
    const uint32_t row = quad * 32 + lane;
    const uint32_t lane_addr = (quad * 32u) << 16;
    {
      const uint64_t qrow = qslab * seq + static_cast<uint64_t>(qtile) * FA_BQ + row;
      const float* src = (softmax ? qhi : qlo) + qrow * FA_HD;
      const uint32_t col = softmax ? COL_QHI : COL_QLO;
#pragma unroll 1
      for (uint32_t c0 = 0; c0 < FA_HD; c0 += 32) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(src + c0 + i));
          r[i] = __float_as_uint(v.x);
          r[i + 1] = __float_as_uint(v.y);
          r[i + 2] = __float_as_uint(v.z);
          r[i + 3] = __float_as_uint(v.w);
        }
        tmem_st_32x32b_x32(tmem + lane_addr + col + c0, r);
      }
      tmem_st_wait();
    }
    tc_fence_before();
    q_ready_barrier();

    if (softmax) {
      float m_run = -FLT_MAX;
      double l_run = 0.0;
      const uint32_t qpos = qtile * FA_BQ + row;
      // Load this CTA's partial score block jj from TMEM into `part`, free the TMEM
      // scores for the next product, and send the partial into the peer's buffer jj % 2.
      auto fetch_send = [&](uint32_t jj, float (&part)[32]) -> bool {
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full, jj & 1u, err, kErrWaitAccum))) return false;
        tc_fence_after();
        {
          uint32_t sm[32], sc[32];
          tmem_ld_32x32b_x32(tmem + lane_addr + COL_SM, sm);
          tmem_ld_32x32b_x32(tmem + lane_addr + COL_SC, sc);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) part[i] = __uint_as_float(sm[i]) + __uint_as_float(sc[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty);
        const uint32_t b = jj & 1u;
        // the peer has read what this CTA sent into buffer b two blocks ago
        if (jj >= 2 && !__all_sync(0xffffffffu, mbar_spin_cluster(&sx_empty[b], ((jj >> 1) - 1) & 1u, err,
                                                                   kErrWaitPeer)))
          return false;
        const uint32_t dst = cluster_smem_addr(sx + b * FA2_SX_FLOATS + row * 4, peer);
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          st_cluster_v4(dst + 4u * (i / 4) * FA_BQ * 4, part[i], part[i + 1], part[i + 2], part[i + 3]);
        __syncwarp();  // every lane's stores come before the warp's release below
        if (lane == 0) mbar_arrive_cluster(&sx_full[b], peer);
        return true;
      };
      float pc[32], pn[32];
      bool ok = nb > 0 && fetch_send(0, pc);
      for (uint32_t j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb && !fetch_send(j + 1, pn)) break;
        // the peer's partial of block j (sent one block ahead) completes the scores
        const uint32_t b = j & 1u;
        if (!__all_sync(0xffffffffu, mbar_spin_cluster(&sx_full[b], (j >> 1) & 1u, err, kErrWaitPeer))) break;
        float p[32];
        const float* mine = sx + b * FA2_SX_FLOATS + row * 4;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 q4 = *reinterpret_cast<const float4*>(mine + (i / 4) * FA_BQ * 4);
          p[i] = (pc[i] + q4.x) * scale;
          p[i + 1] = (pc[i + 1] + q4.y) * scale;
          p[i + 2] = (pc[i + 2] + q4.z) * scale;
          p[i + 3] = (pc[i + 3] + q4.w) * scale;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(&sx_empty[b], peer);
#pragma unroll
        for (int i = 0; i < 32; ++i) pc[i] = pn[i];
        if (causal && (j + 1) * FA_BKV > qtile * FA_BQ) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (j * FA_BKV + static_cast<uint32_t>(i) > qpos) p[i] = -INFINITY;
        }
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = fmaxf(p[i], p[i + 16]);
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) t[i] = fmaxf(t[i], t[i + w]);
        const float mx = t[0];
        const float m_new = (mx > m_run + FA_TAU) ? mx : m_run;
        const float alpha = (m_new == m_run) ? 1.0f : expf(m_run - m_new);
#pragma unroll
        for (int i = 0; i < 32; ++i) p[i] = expf(p[i] - m_new);
#pragma unroll
        for (int i = 0; i < 16; ++i) t[i] = p[i] + p[i + 16];
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) t[i] += t[i + w];
        l_run = l_run * static_cast<double>(alpha) + static_cast<double>(t[0]);
        m_run = m_new;
        if (j >= 1) {
          alpha_sh[(j - 1) & 1u][row] = alpha;
          __syncwarp();
          if (lane == 0) mbar_arrive(&alpha_full[(j - 1) & 1u]);
          if (!__all_sync(0xffffffffu, mbar_wait(&o_full, (j - 1) & 1u, err, kErrWaitAccum))) break;
          tc_fence_after();
        }
        {
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float h = to_tf32(p[i]);
            ph[i] = __float_as_uint(h);
            pl[i] = __float_as_uint(to_tf32(p[i] - h));
          }
          tmem_st_32x32b_x32(tmem + lane_addr + COL_PHI, ph);
          tmem_st_32x32b_x32(tmem + lane_addr + COL_PLO, pl);
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full);
      }
      inv_l_sh[row] = static_cast<float>(1.0 / l_run);
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_ready);
    } else {

      float o_run[FA_HD];
#pragma unroll
      for (int i = 0; i < static_cast<int>(FA_HD); ++i) o_run[i] = 0.f;
      bool ok = true;
      for (uint32_t j = 1; j < nb; ++j) {
        ok = __all_sync(0xffffffffu, mbar_wait(&alpha_full[(j - 1) & 1u], ((j - 1) >> 1) & 1u, err, kErrWaitAccum) &&
                                         mbar_wait(&o_full, (j - 1) & 1u, err, kErrWaitAccum));
        if (!ok) break;
        tc_fence_after();
        const float alpha = alpha_sh[(j - 1) & 1u][row];
        const bool rescale = __any_sync(0xffffffffu, alpha != 1.0f);
#pragma unroll
        for (uint32_t g = 0; g < FA_HD / 32; ++g) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_addr + COL_O + g * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o_run[g * 32 + i] += __uint_as_float(r[i]);
          if (rescale) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o_run[g * 32 + i] *= alpha;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty);
      }
      if (ok && nb > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&o_full, (nb - 1) & 1u, err, kErrWaitAccum) &&
                                         mbar_wait(&l_ready, 0, err, kErrWaitAccum));
        if (ok) {
          tc_fence_after();
          const float inv = inv_l_sh[row];
          const uint64_t o = (static_cast<uint64_t>(item) * seq + static_cast<uint64_t>(qtile) * FA_BQ + row) * ldo +
                             (static_cast<uint64_t>(head) * 2 + rank) * FA_HD;
          float* dst = out + o;
          float* dst_lo = out_lo != nullptr ? out_lo + o : nullptr;
#pragma unroll
          for (uint32_t g = 0; g < FA_HD / 32; ++g) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + lane_addr + COL_O + g * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const int c = static_cast<int>(g * 32) + i;
              float4 v = make_float4((o_run[c] + __uint_as_float(r[i])) * inv,
                                     (o_run[c + 1] + __uint_as_float(r[i + 1])) * inv,
                                     (o_run[c + 2] + __uint_as_float(r[i + 2])) * inv,
                                     (o_run[c + 3] + __uint_as_float(r[i + 3])) * inv);
              if (dst_lo != nullptr) {
                const float4 h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
                *reinterpret_cast<float4*>(dst_lo + c) =
                    make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
                v = h;
              }
              *reinterpret_cast<float4*>(dst + c) = v;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 32) mbar_wait(&drain_bar, 0, err, kErrWaitDrain);
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still write its exchange buffer or barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// V [items*S rows][ldv] (head h in columns h*128 ..) -> V^T hi / lo [(item*heads + h)*128 + c][S].
// 32 x 32 tiles through shared memory: reads along channels, writes along positions.
__global__ void split_transpose_heads_kernel(const float* __restrict__ v, uint64_t ldv, uint32_t heads, uint32_t seq,
                                             float* __restrict__ vthi, float* __restrict__ vtlo) {
  __shared__ float tile[32][33];
  const uint32_t pos0 = blockIdx.x * 32;
  const uint32_t col0 = blockIdx.y * 32;  // column within the item's heads*128 V columns
  const uint32_t item = blockIdx.z;
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
#pragma unroll
  for (uint32_t r = ty; r < 32; r += 8)
    tile[r][tx] = v[(static_cast<uint64_t>(item) * seq + pos0 + r) * ldv + col0 + tx];
  __syncthreads();
#pragma unroll
  for (uint32_t r = ty; r < 32; r += 8) {
    const uint32_t col = col0 + r;  // = head * 128 + channel
    const float x = tile[tx][r];
    const float h = to_tf32(x);
    const uint64_t o = (static_cast<uint64_t>(item) * heads * FA_HD + col) * seq + pos0 + tx;
    vthi[o] = h;
    vtlo[o] = to_tf32(x - h);
  }
}

// X [items*S rows][ldx] (head h in columns h*128 ..) -> hi / lo [(item*heads + h)*S + pos][128];
// one thread per 4 channels.
__global__ void split_heads_kernel(const float* __restrict__ x, uint64_t ldx, uint32_t heads, uint32_t seq,
                                   uint64_t quads, float* __restrict__ hi, float* __restrict__ lo) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < quads;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t c4 = static_cast<uint32_t>(i % (heads * FA_HD / 4));  // float4 within the token's heads*128
    const uint64_t tok = i / (heads * FA_HD / 4);
    const uint32_t h = c4 / (FA_HD / 4), c = (c4 % (FA_HD / 4)) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + tok * ldx + c4 * 4);
    const uint64_t item = tok / seq, pos = tok % seq;
    const uint64_t o = ((item * heads + h) * seq + pos) * FA_HD + c;
    float4 a, b;
    a.x = to_tf32(v.x);
    a.y = to_tf32(v.y);
    a.z = to_tf32(v.z);
    a.w = to_tf32(v.w);
    b.x = to_tf32(v.x - a.x);
    b.y = to_tf32(v.y - a.y);
    b.z = to_tf32(v.z - a.z);
    b.w = to_tf32(v.w - a.w);
    *reinterpret_cast<float4*>(hi + o) = a;
    *reinterpret_cast<float4*>(lo + o) = b;
  }
}

// Row-major fp32 [rows][cols] with a box of 32 columns (128 bytes, 128-byte swizzle) x box_rows.
bool make_attn_map(CUtensorMap* map, const float* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * sizeof(float)};
  const cuuint32_t box[2] = {32, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool flash_attention256_supported(uint32_t head_dim, uint32_t seq, uint32_t heads, uint32_t kv_heads) {
  return head_dim == 2 * FA_HD && seq >= FA_BQ && seq % FA_BQ == 0 && kv_heads > 0 && heads % kv_heads == 0;
}

cudaError_t flash_attention256_tf32x3(const AttnOperands& in, float* out, uint64_t ldo, uint32_t items, uint32_t heads,
                                      uint32_t kv_heads, uint32_t seq, float scale, bool causal, unsigned int* err,
                                      cudaStream_t stream, float* out_lo) {
  if (!flash_attention256_supported(2 * FA_HD, seq, heads, kv_heads) || items == 0 || heads == 0)
    return cudaErrorInvalidValue;
  const uint64_t kv_slabs = static_cast<uint64_t>(items) * kv_heads * 2;
  if (kv_slabs * seq > 0x7FFFFFFFull || static_cast<uint64_t>(items) * heads * 2 * seq > 0x7FFFFFFFull)
    return cudaErrorInvalidValue;
  CUtensorMap m_khi, m_klo, m_vhi, m_vlo;
  if (!make_attn_map(&m_khi, in.khi, kv_slabs * seq, FA_HD, FA_BKV) ||
      !make_attn_map(&m_klo, in.klo, kv_slabs * seq, FA_HD, FA_BKV) ||
      !make_attn_map(&m_vhi, in.vthi, kv_slabs * FA_HD, seq, FA_HD) ||
      !make_attn_map(&m_vlo, in.vtlo, kv_slabs * FA_HD, seq, FA_HD))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(flash_attn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(FA2_SMEM));
  if (e != cudaSuccess) return e;
  const dim3 grid(2 * (seq / FA_BQ), heads, items);
  flash_attn_pair_kernel<<<grid, FA_THREADS, FA2_SMEM, stream>>>(m_khi, m_klo, m_vhi, m_vlo, in.qhi, in.qlo, out, ldo,
                                                                 heads, kv_heads, seq, scale, causal ? 1u : 0u, err,
                                                                 out_lo);
  return cudaGetLastError();
}

bool flash_attention_supported(uint32_t head_dim, uint32_t seq) {
  return head_dim == FA_HD && seq >= FA_BQ && seq % FA_BQ == 0;
}

cudaError_t split_transpose_heads(const float* v, uint64_t ldv, uint32_t items, uint32_t heads, uint32_t seq,
                                  float* vthi, float* vtlo, cudaStream_t stream) {
  if (seq % 32 != 0 || items == 0 || heads == 0) return cudaErrorInvalidValue;
  const dim3 grid(seq / 32, heads * FA_HD / 32, items);
  split_transpose_heads_kernel<<<grid, 256, 0, stream>>>(v, ldv, heads, seq, vthi, vtlo);
  return cudaGetLastError();
}

cudaError_t split_heads(const float* x, uint64_t ldx, uint32_t items, uint32_t heads, uint32_t seq, float* hi,
                        float* lo, cudaStream_t stream) {
  if (items == 0 || heads == 0 || seq == 0 || ldx % 4 != 0) return cudaErrorInvalidValue;
  const uint64_t quads = static_cast<uint64_t>(items) * seq * heads * (FA_HD / 4);
  const uint64_t blocks = std::min<uint64_t>((quads + 255) / 256, 148ull * 16);
  split_heads_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, ldx, heads, seq, quads, hi, lo);
  return cudaGetLastError();
}

cudaError_t flash_attention_tf32x3(const AttnOperands& in, float* out, uint64_t ldo, uint32_t items, uint32_t heads,
                                   uint32_t seq, float scale, unsigned int* err, cudaStream_t stream, float* out_lo) {
  if (!flash_attention_supported(FA_HD, seq) || items == 0 || heads == 0) return cudaErrorInvalidValue;
  const uint64_t slabs = static_cast<uint64_t>(items) * heads;
  if (slabs * seq > 0x7FFFFFFFull) return cudaErrorInvalidValue;  // TMA row coordinates are int32
  CUtensorMap m_khi, m_klo, m_vhi, m_vlo;
  if (!make_attn_map(&m_khi, in.khi, slabs * seq, FA_HD, FA_BKV) ||
      !make_attn_map(&m_klo, in.klo, slabs * seq, FA_HD, FA_BKV) ||
      !make_attn_map(&m_vhi, in.vthi, slabs * FA_HD, seq, FA_HD) ||
      !make_attn_map(&m_vlo, in.vtlo, slabs * FA_HD, seq, FA_HD))
    return cudaErrorInvalidValue;
  cudaError_t e =
      cudaFuncSetAttribute(flash_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(FA_SMEM));
  if (e != cudaSuccess) return e;
  const dim3 grid(seq / FA_BQ, heads, items);
  flash_attn_kernel<<<grid, FA_THREADS, FA_SMEM, stream>>>(m_khi, m_klo, m_vhi, m_vlo, in.qhi, in.qlo, out, ldo, heads,
                                                           seq, scale, err, out_lo);
  return cudaGetLastError();
}

}  // namespace oct
