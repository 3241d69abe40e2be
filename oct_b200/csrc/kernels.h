// kernels.h -- host-side launchers for the CUDA kernels, used by the C-ABI layer.
// Every launcher enqueues on `stream` and returns a cudaError_t for the launch;
// kernel-side wait timeouts land in the `err` device word.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace oct {

// ---------------------------------------------------------------- SGEMM
// Padded extents of the split-TF32 operand buffers for an (m, n, k) product.
struct SplitDims {
  uint32_t mp, np, kp;  // m rounded to the M tile, n to the N tile, k to 32
};
SplitDims split_dims(uint32_t m, uint32_t n, uint32_t k);

// Bytes of scratch needed by sgemm_tc for (m, n, k): hi/lo copies of A and of
// B^T, per batch entry, times `batch`.
uint64_t sgemm_tc_scratch_bytes(uint32_t m, uint32_t n, uint32_t k, uint32_t batch = 1);

// Strided batch of independent products C_i = A_i * op(B_i), i < count, with
// X_i = X + i * stride_x (element strides; a stride of 0 shares the operand).
// b_trans: B is given as [n][k] row-major and op(B) = B^T (the "NT" product).
// Element offset of batch entry e: e * stride, or, with inner > 0, a two-level
// index (e / inner) * outer + (e % inner) * stride (e.g. entry = item * heads + head).
struct EntryStride {
  uint64_t stride = 0;
  uint32_t inner = 0;
  uint64_t outer = 0;
  __host__ __device__ uint64_t at(uint32_t e) const {
    return inner != 0 ? static_cast<uint64_t>(e / inner) * outer + static_cast<uint64_t>(e % inner) * stride
                      : static_cast<uint64_t>(e) * stride;
  }
};

struct GemmBatch {
  uint32_t count = 1;
  uint64_t stride_a = 0, stride_b = 0, stride_c = 0;
  bool b_trans = false;
  // optional second level: entry e = (e / inner, e % inner); outer_* step the first index
  uint32_t inner = 0;
  uint64_t outer_a = 0, outer_b = 0, outer_c = 0;
  EntryStride sa() const { return EntryStride{stride_a, inner, outer_a}; }
  EntryStride sb() const { return EntryStride{stride_b, inner, outer_b}; }
  EntryStride sc() const { return EntryStride{stride_c, inner, outer_c}; }
};

// Tensor-core kernel configurations: one CTA per 128 x 256 tile, or a CTA pair
// (cta_group::2) per 256 x 256 tile; 16 or 32 K elements per pipeline stage.
enum TcConfig : int {
  kTcSingle16 = 16, kTcSingle32 = 32, kTcPair16 = 216, kTcPair32 = 232,
  kTcInsm16 = 316, kTcInsm32 = 332,  // CTA pair, TF32 split inside the kernel (no split pass)
};

// 3xTF32 tensor-core SGEMM.  `scratch` must hold sgemm_tc_scratch_bytes and be
// 1024-byte aligned.  bk is a TcConfig.
// Optional events (may be null) are recorded on `stream` before the split
// pass, before the main kernel and after it, for per-kernel timing.
struct SgemmEvents {
  cudaEvent_t split_begin = nullptr, main_begin = nullptr, main_end = nullptr;
};
cudaError_t sgemm_tc(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                     uint32_t m, uint32_t n, uint32_t k, void* scratch, unsigned int* err, int bk,
                     cudaStream_t stream, const SgemmEvents* events = nullptr, const GemmBatch* batch = nullptr);
// The in-SM split kernel reads A and B in place with TMA: single products whose
// bases are 16-byte aligned and whose leading dimensions are multiples of 4.
// It needs no scratch; C = R + A * B when `residual` is given.
bool sgemm_insm_eligible(const float* a, uint64_t lda, const float* b, uint64_t ldb, uint32_t m, uint32_t n,
                         uint32_t k, const GemmBatch* batch);
cudaError_t sgemm_tc_insm(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                          uint32_t m, uint32_t n, uint32_t k, unsigned int* err, int bk, cudaStream_t stream,
                          const SgemmEvents* events = nullptr, const float* residual = nullptr, uint64_t ldr = 0);

// Pre-split weights: sgemm_tc_split_b writes the hi/lo K-major layout of a
// [k][n] operand (split_b_elems floats each); sgemm_tc_presplit then computes
// C = R + A * B (R = residual, optional, may alias C) splitting only A into
// a_scratch (sgemm_tc_a_scratch_bytes, 1024-byte aligned).
uint64_t split_b_elems(uint32_t n, uint32_t k);
cudaError_t sgemm_tc_split_b(const float* b, uint64_t ldb, uint32_t k, uint32_t n, float* bhi, float* blo,
                             cudaStream_t stream);
uint64_t sgemm_tc_a_scratch_bytes(uint32_t m, uint32_t k);
// Row scatter epilogue (single-CTA configurations): output row r goes to rank
// owner = r / rows_per_rank, into dst[owner] at row
// src_rank * rows_per_rank + (r - owner * rows_per_rank), leading dimension ld.
// `dst` is a device array of one base pointer per rank (peers' memory included).
// Broadcast form (bcast = world > 0; rows_per_rank unused): every output row r
// goes to every rank k, into dst[k] at row r, columns col_offset.. -- the
// column-parallel product's all-gather done by the epilogue's stores.
struct RowScatter {
  float* const* dst = nullptr;
  uint32_t rows_per_rank = 0;
  uint32_t src_rank = 0;
  uint64_t ld = 0;
  uint32_t bcast = 0;
  uint64_t col_offset = 0;
};
// Split K for products that fill less than one wave of SMs (single-CTA
// configurations only): K in `ranges` ranges of whole 64-deep accumulation
// chunks (sgemm_tc_k_ranges gives how many run), one CTA per (tile, range).
// Without a row scatter the ranges' partial products go to `partial`
// (ranges * m * n floats) and a second kernel sums them in range order into
// C = R + sum; with one, range j goes to slot src_rank * ranges + j of the
// owner rank, whose reduction sums the slots in order.
struct SplitK {
  uint32_t ranges = 1;
  float* partial = nullptr;
};
uint32_t sgemm_tc_k_ranges(uint32_t k, uint32_t ranges);
// The range count for an (m, n, k) product on the single-CTA kernel: 1 when
// its 128 x 256 tiles fill a wave, else the count (<= 8, each range >= 128 of
// K) whose CTAs fill the waves they start best.
uint32_t sgemm_tc_pick_k_ranges(uint32_t m, uint32_t n, uint32_t k);
cudaError_t sgemm_tc_presplit(const float* a, uint64_t lda, const float* bhi, const float* blo, float* c,
                              uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, void* a_scratch, unsigned int* err,
                              cudaStream_t stream, const float* residual = nullptr, uint64_t ldr = 0,
                              int cfg = kTcSingle16, const RowScatter* scatter = nullptr,
                              const SplitK* splitk = nullptr);

// A and B both already split: A hi/lo rows of length Kp (split_dims), written by
// the kernel that produced A; C = R + A * B as in sgemm_tc_presplit.
cudaError_t sgemm_tc_presplit_ab(const float* ahi, const float* alo, const float* bhi, const float* blo, float* c,
                                 uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, unsigned int* err,
                                 cudaStream_t stream, const float* residual = nullptr, uint64_t ldr = 0,
                                 int cfg = kTcSingle16, const SplitK* splitk = nullptr);

// A already split by its producer (hi/lo in the [count][Mp][Kp] layout of
// split_dims, zero padded); B is split into b_scratch.  Strided batch as GemmBatch.
cudaError_t sgemm_tc_presplit_a(const float* ahi, const float* alo, const float* b, uint64_t ldb, float* c,
                                uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, void* b_scratch, unsigned int* err,
                                cudaStream_t stream, const GemmBatch* batch, int cfg = kTcSingle16);

// Plain FP32-FMA SGEMM on the CUDA cores (control variant); no scratch.
cudaError_t sgemm_fma(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                      uint32_t m, uint32_t n, uint32_t k, cudaStream_t stream, const GemmBatch* batch = nullptr);

// cuTensorMapEncodeTiled through the runtime's driver entry point (null if absent).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// ---------------------------------------------------------------- fused attention
// Exact bidirectional attention over heads of 128 channels, one fused
// tensor-core kernel (attention.cu).  Operands are TF32 hi/lo splits:
//   q/k hi, lo: [items*heads*seq][128] (row (item*heads + h)*seq + position)
//   vt hi, lo:  [items*heads*128][seq] (V transposed per head)
// out[(item*seq + position) * ldo + h*128 + c].  seq must be a multiple of 128.
struct AttnOperands {
  const float *qhi, *qlo, *khi, *klo, *vthi, *vtlo;
};
bool flash_attention_supported(uint32_t head_dim, uint32_t seq);
// With out_lo != null the output is written as its TF32 split: hi to out, lo to out_lo.
cudaError_t flash_attention_tf32x3(const AttnOperands& in, float* out, uint64_t ldo, uint32_t items, uint32_t heads,
                                   uint32_t seq, float scale, unsigned int* err, cudaStream_t stream,
                                   float* out_lo = nullptr);
// Heads of 256 channels (Gemma), causal or not, K / V heads shared by groups of
// heads / kv_heads query heads: one CTA pair per 128-query tile, each CTA on one
// 128-channel half.  Operands in the layouts above with every 256-channel head
// taken as two half heads: q hi/lo from split_heads over 2 * heads half heads,
// k hi/lo and vt hi/lo over 2 * kv_heads; out[(item*seq + position) * ldo + h*256 + c].
bool flash_attention256_supported(uint32_t head_dim, uint32_t seq, uint32_t heads, uint32_t kv_heads);
cudaError_t flash_attention256_tf32x3(const AttnOperands& in, float* out, uint64_t ldo, uint32_t items, uint32_t heads,
                                      uint32_t kv_heads, uint32_t seq, float scale, bool causal, unsigned int* err,
                                      cudaStream_t stream, float* out_lo = nullptr);
// V columns of `heads` heads ([items*seq][ldv], head h at columns h*128..) ->
// the vt hi/lo layout above.
// Q or K columns of `heads` heads ([items*seq][ldx]) -> the q/k hi/lo layout above.
cudaError_t split_heads(const float* x, uint64_t ldx, uint32_t items, uint32_t heads, uint32_t seq, float* hi,
                        float* lo, cudaStream_t stream);
cudaError_t split_transpose_heads(const float* v, uint64_t ldv, uint32_t items, uint32_t heads, uint32_t seq,
                                  float* vthi, float* vtlo, cudaStream_t stream);

// ---------------------------------------------------------------- tensor parallel over peer memory
// (tp_fused.cu).  Flags are [slot][world] u64 epochs in each rank's memory.
// signal: rank `src` stores `epoch` into flags_dev[k][slot][src] of every rank k
// (release, system scope).  wait: until flags_local[slot][s] >= epoch for every
// source s (acquire), at most budget_ns, else kErrWaitPeer in *err.
cudaError_t tp_signal(uint64_t* const* flags_dev, uint32_t slot, uint32_t world, uint32_t src, uint64_t epoch,
                      cudaStream_t stream);
cudaError_t tp_wait(const uint64_t* flags_local, uint32_t slot, uint32_t world, uint64_t epoch, unsigned int* err,
                    unsigned long long budget_ns, cudaStream_t stream);
// signal, then wait, in one launch
cudaError_t tp_signal_wait(uint64_t* const* flags_dev, const uint64_t* flags_local, uint32_t slot, uint32_t world,
                           uint32_t src, uint64_t epoch, unsigned int* err, unsigned long long budget_ns,
                           cudaStream_t stream);
// Reduce the row-scatter slots of this rank's rows, then residual / norm /
// modulation, then push the rows to every rank (see tp_fused.cu).
struct TpReduce {
  const float* slots = nullptr;  // [nslots][rows][ld_slot]
  uint32_t nslots = 0;
  uint64_t slot_stride = 0, ld_slot = 0;
  uint32_t rows = 0, row0 = 0, width = 0, rows_per_item = 1;
  uint64_t mod_stride = 0;
  float eps = 1e-6f;
  const float* g1 = nullptr;
  const float* gate1 = nullptr;
  const float* res = nullptr;
  uint64_t ld_res = 0;
  float* keep = nullptr;
  uint64_t ld_keep = 0;
  const float* g2 = nullptr;
  const float* mul2 = nullptr;
  const float* add2 = nullptr;
  float* const* push = nullptr;  // device array of npush row-major [*][ld_push] buffers
  uint32_t npush = 0;
  uint64_t ld_push = 0;
};
cudaError_t tp_reduce_rows(const TpReduce& args, cudaStream_t stream);

// Small-M fp32 SGEMM (1 <= m <= 16): HBM-bound on B, CUDA-core FMA, split-K with
// an ordered reduction of the partials (sgemm_smallm.cu).  `scratch` must hold
// sgemm_smallm_scratch_bytes (may be 0 bytes: then it may be null).
bool sgemm_smallm_supported(uint32_t m);
uint64_t sgemm_smallm_scratch_bytes(uint32_t m, uint32_t n, uint32_t k);
// With `err` (the kernel status word) and B rows copyable in 16-byte units, the
// bulk-copy-fed variant runs; otherwise the register-streaming one.
cudaError_t sgemm_smallm(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                         uint32_t m, uint32_t n, uint32_t k, void* scratch, cudaStream_t stream,
                         unsigned int* err = nullptr);

// Small-M fp32 SGEMM (1 <= m <= 16) on the tcgen05 tensor cores with the TF32
// split inside the kernel (sgemm_smallm_tc.cu): A and B read in place by TMA
// (16-byte aligned, leading dimensions multiples of 4), split-K partials in
// `scratch` (sgemm_smallm_tc_scratch_bytes, may be 0) added in split order.
bool sgemm_smallm_tc_eligible(const float* a, uint64_t lda, const float* b, uint64_t ldb, uint32_t m, uint32_t n,
                              uint32_t k);
uint64_t sgemm_smallm_tc_scratch_bytes(uint32_t m, uint32_t n, uint32_t k);
cudaError_t sgemm_smallm_tc(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                            uint32_t m, uint32_t n, uint32_t k, void* scratch, unsigned int* err,
                            cudaStream_t stream);

// ---------------------------------------------------------------- reductions
// op: 1 = row sum, 2 = row max, 3 = stable softmax.  `nonfinite` (device
// u64, preset to UINT64_MAX by the caller) receives the smallest flat index of
// a NaN/Inf input element, if any.
cudaError_t row_reduce(const float* in, float* out, uint32_t rows, uint32_t width, uint32_t op,
                       unsigned long long* nonfinite, unsigned int* err, cudaStream_t stream);

// RMSNorm: out = in * inv_rms * weight, inv_rms = 1/sqrt(mean(in^2)+eps).
// in_stride is the element distance between consecutive input rows.
cudaError_t rmsnorm(const float* in, uint64_t in_stride, const float* weight, float* out, float* inv_rms,
                    uint32_t rows, uint32_t width, float eps, unsigned long long* nonfinite, unsigned int* err,
                    cudaStream_t stream);

// Correctness check of a reduction's output on the device: `expected` (row count,
// or rows * width for softmax, floats) receives an independent recomputation and
// `first_bad` (preset to UINT64_MAX) the smallest failing flat index under the
// reference comparator's tolerances; softmax row-sum failures are reported as
// rows * width + row.
cudaError_t reduction_self_check(const float* in, const float* actual, float* expected, uint32_t rows,
                                 uint32_t width, uint32_t op, unsigned long long* first_bad, cudaStream_t stream);

// ---------------------------------------------------------------- Z-Image ingress (zimage.cu)
// BF16 values (the high half of a binary32) and binary16 values widened exactly
// to fp32; widen_f16 writes a [rows][cols] source at column col0 of a dst with
// leading dimension ld.
cudaError_t widen_bf16(const void* src, float* dst, uint64_t n, cudaStream_t stream);
cudaError_t widen_f16(const void* src, uint32_t rows, uint32_t cols, float* dst, uint64_t ld, uint32_t col0,
                      cudaStream_t stream);

// ---------------------------------------------------------------- FFT (fft.cu)
// Radix-2 decimation-in-time complex transforms of n = 2^k <= kFftMaxElements
// points, interleaved (re, im) pairs; `in` and `out` must not overlap.
// fft64: forward, one transform, binary64, host twiddle table of n doubles
// (cos, sin of -2 pi i / n for i < n / 2).  fft32: `batch` transforms
// stride_elements apart, twiddles computed per pass in fp32; inverse uses +2 pi,
// normalize divides the inverse by n.
constexpr uint32_t kFftMaxElements = 1u << 20;
cudaError_t fft64(const double* in, double* out, uint32_t n, const double* twiddles, cudaStream_t stream);
cudaError_t fft32(const float* in, float* out, uint32_t n, uint32_t batch, uint64_t stride_elements, bool inverse,
                  bool normalize, cudaStream_t stream);

// ---------------------------------------------------------------- Gemma M1 boundary (gemma_m1.cu)
// BF16 storage rounding as the reference's M1 entry points apply it; inputs
// must already be checked finite.  Head widths are even and <= kM1MaxHeadWidth.
constexpr uint32_t kM1MaxHeadWidth = 1024;
// y = round_out((round_in(x) * inv) * w) per row, inv = float(1/sqrt(sum x^2 / width + eps))
// with the sum of squares in binary64.
cudaError_t m1_rmsnorm_bf16(const float* in, uint64_t stride, const float* w, float* out, float* inv_rms,
                            uint32_t rows, uint32_t width, float eps, bool round_in, bool round_out,
                            cudaStream_t stream);
// Half-split RoPE of [tokens][heads][head_width] with [tokens][head_width] tables
// (only each row's first head_width / 2 entries are read), BF16 products and sums.
cudaError_t m1_rope_bf16(const float* src, const float* cos_table, const float* sin_table, float* out,
                         uint32_t tokens, uint32_t heads, uint32_t head_width, cudaStream_t stream);
// The BF16 head RMSNorm of every (token, head) row followed by the RoPE above.
cudaError_t m1_head_rmsnorm_rope(const float* in, const float* w, const float* cos_table, const float* sin_table,
                                 float* out, uint32_t tokens, uint32_t heads, uint32_t head_width, float eps,
                                 cudaStream_t stream);
// scores[h][i][j] = float(sum_d q[i][h][d] k[j][d] * scale) in binary64; k is [tokens][head_width]
// (one KV head shared by every query head).
cudaError_t m1_raw_scores(const float* q, const float* k, float* scores, uint32_t tokens, uint32_t query_heads,
                          uint32_t head_width, float scale, cudaStream_t stream);

}  // namespace oct
