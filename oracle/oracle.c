/*
 * oracle.c -- CPU restatement of Oct's own CPU arithmetic for the Prometheus
 * fp32 compute path.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke
 * check and the benchmark's CPU-baseline leg use it as the checker; the
 * product library never links, loads or calls it.
 *
 * Oct's CPU paths are Go (no Go toolchain is available here) and plain C inside
 * its Vulkan reactor (which cannot build without Vulkan and the external
 * Concept headers), so each function below restates one reference function,
 * cited file:line, in the same loop order and the same precision.  Build with
 * -ffp-contract=off so fp32 `sum += a*b` rounds the product and the sum
 * separately, exactly as Go on amd64 does.
 *
 * Pinning: tests/test_oracle_pins.py checks these functions against known
 * answers derived by exact rational arithmetic from the reference's own test
 * matrices (runtime.go:242-249 deterministicMatrix, Marionette
 * reactor_concept_sgemm_tests.cpp:14-19 Matrix, reactor_reduction_tests.cpp:
 * 77-114 deterministic_input and its extreme / constant / heterogeneous rows)
 * and against the committed fixtures in tests/golden/.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <pthread.h>
#include <string.h>
#include <unistd.h>

#define ORACLE_API __attribute__((visibility("default")))

/* ------------------------------------------------------- row-parallel helper
   Rows are independent in every function here, so the multi-threaded forms
   split [begin, end) into `threads` contiguous ranges; results are identical
   to the serial form. */
typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end);
typedef struct {
  range_fn fn;
  void* ctx;
  int64_t begin, end;
} range_job;

static void* range_main(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}

static void parallel_rows(int threads, int64_t begin, int64_t end, range_fn fn, void* ctx) {
  enum { MAXT = 256 };
  if (threads < 1) threads = 1;
  if (threads > MAXT) threads = MAXT;
  if (end - begin < threads) threads = (int)(end - begin > 0 ? end - begin : 1);
  if (threads == 1) {
    fn(ctx, begin, end);
    return;
  }
  pthread_t tid[MAXT];
  range_job job[MAXT];
  int started[MAXT];
  const int64_t span = end - begin;
  for (int t = 0; t < threads; ++t) {
    job[t].fn = fn;
    job[t].ctx = ctx;
    job[t].begin = begin + span * t / threads;
    job[t].end = begin + span * (t + 1) / threads;
    started[t] = pthread_create(&tid[t], NULL, range_main, &job[t]) == 0;
    if (!started[t]) range_main(&job[t]);
  }
  for (int t = 0; t < threads; ++t)
    if (started[t]) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------ SGEMM */

/* cpuSGEMM (internal/prometheus/runtime.go:319-331): serial i-j-k, fp32
   accumulator, left-to-right over k.  Rows [row0, row0 + nrows) only, so a
   bounded sample of a large product can be timed or checked. */
ORACLE_API void oracle_cpu_sgemm_f32_rows(int64_t m, int64_t n, int64_t k, const float* a, const float* b, float* c,
                                          int64_t row0, int64_t nrows) {
  (void)m;
  for (int64_t row = row0; row < row0 + nrows; ++row) {
    for (int64_t col = 0; col < n; ++col) {
      float sum = 0.0f;
      for (int64_t kk = 0; kk < k; ++kk) sum += a[row * k + kk] * b[kk * n + col];
      c[(row - row0) * n + col] = sum;
    }
  }
}

ORACLE_API void oracle_cpu_sgemm_f32(int64_t m, int64_t n, int64_t k, const float* a, const float* b, float* c) {
  oracle_cpu_sgemm_f32_rows(m, n, k, a, b, c, 0, m);
}

/* The same fp32 i-j-k arithmetic with rows spread over `threads` POSIX
   threads: the all-core CPU baseline (results identical to the serial form). */
typedef struct {
  int64_t m, n, k, row0;
  const float* a;
  const float* b;
  float* c;
} sgemm_f32_ctx;

static void sgemm_f32_range(void* p, int64_t begin, int64_t end) {
  const sgemm_f32_ctx* x = (const sgemm_f32_ctx*)p;
  oracle_cpu_sgemm_f32_rows(x->m, x->n, x->k, x->a, x->b, x->c + (begin - x->row0) * x->n, begin, end - begin);
}

ORACLE_API void oracle_cpu_sgemm_f32_mt(int64_t m, int64_t n, int64_t k, const float* a, const float* b, float* c,
                                        int64_t row0, int64_t nrows, int threads) {
  sgemm_f32_ctx x = {m, n, k, row0, a, b, c};
  parallel_rows(threads, row0, row0 + nrows, sgemm_f32_range, &x);
}

/* __octMatMulMM[float64] (internal/build/emit_go_runtime.go:168-200): the
   compiled Oct CPU `@` -- serial i-j-k with a float64 accumulator. */
ORACLE_API void oracle_oct_matmul_f64_rows(int64_t m, int64_t n, int64_t k, const double* a, const double* b,
                                           double* c, int64_t row0, int64_t nrows) {
  (void)m;
  for (int64_t r = row0; r < row0 + nrows; ++r) {
    for (int64_t col = 0; col < n; ++col) {
      double acc = 0.0;
      for (int64_t kk = 0; kk < k; ++kk) acc += a[r * k + kk] * b[kk * n + col];
      c[(r - row0) * n + col] = acc;
    }
  }
}

/* Binary64 accumulation of an fp32 product, as the native SGEMM test's
   CheckProduct (internal/prometheus/native/Marionette/reactor_concept_sgemm_tests.cpp:21-27):
   expected += double(a) * b.  Rows [row0, row0 + nrows). */
typedef struct {
  int64_t n, k, row0;
  const float* a;
  const float* b;
  double* c;
} sgemm_f64_ctx;

static void sgemm_f64_range(void* p, int64_t begin, int64_t end) {
  const sgemm_f64_ctx* x = (const sgemm_f64_ctx*)p;
  for (int64_t row = begin; row < end; ++row) {
    double* out = x->c + (row - x->row0) * x->n;
    for (int64_t col = 0; col < x->n; ++col) out[col] = 0.0;
    for (int64_t kk = 0; kk < x->k; ++kk) {
      const double av = (double)x->a[row * x->k + kk];
      const float* brow = x->b + kk * x->n;
      for (int64_t col = 0; col < x->n; ++col) out[col] += av * (double)brow[col];
    }
  }
}

ORACLE_API void oracle_sgemm_f64_rows(int64_t m, int64_t n, int64_t k, const float* a, const float* b, double* c,
                                      int64_t row0, int64_t nrows, int threads) {
  (void)m;
  sgemm_f64_ctx x = {n, k, row0, a, b, c};
  parallel_rows(threads, row0, row0 + nrows, sgemm_f64_range, &x);
}

/* compareAgainstOracle (internal/prometheus/runtime.go:339-383): an element
   fails when it is non-finite, or when BOTH its absolute and relative error
   exceed the tolerances (relative error is 0 when expected == 0). */
typedef struct OracleCorrectness {
  int32_t pass;
  int32_t failing_count;
  int64_t first_failing_index;
  double max_abs_error;
  double max_rel_error;
  float first_expected;
  float first_actual;
} OracleCorrectness;

ORACLE_API void oracle_compare_against_oracle(const float* expected, const float* actual, int64_t count,
                                              double abs_tol, double rel_tol, OracleCorrectness* res) {
  memset(res, 0, sizeof(*res));
  res->pass = 1;
  res->first_failing_index = -1;
  for (int64_t i = 0; i < count; ++i) {
    const float e = expected[i], a = actual[i];
    if (!isfinite(e) || !isfinite(a)) {
      if (res->first_failing_index < 0) {
        res->first_failing_index = i;
        res->first_expected = e;
        res->first_actual = a;
      }
      res->failing_count++;
      res->pass = 0;
      continue;
    }
    const double abs_err = fabs((double)(e - a));
    const double rel_err = e != 0.0f ? abs_err / fabs((double)e) : 0.0;
    if (abs_err > res->max_abs_error) res->max_abs_error = abs_err;
    if (rel_err > res->max_rel_error) res->max_rel_error = rel_err;
    if (abs_err > abs_tol && rel_err > rel_tol) {
      if (res->first_failing_index < 0) {
        res->first_failing_index = i;
        res->first_expected = e;
        res->first_actual = a;
      }
      res->failing_count++;
      res->pass = 0;
    }
  }
}

/* ------------------------------------------------------------- reductions */
enum { OP_SUM = 1, OP_MAX = 2, OP_SOFTMAX = 3 };

/* prom_find_nonfinite (reactor_vulkan_fused_reduction.c:859-868): index of
   the first NaN/Inf, or -1. */
ORACLE_API int64_t oracle_find_nonfinite(const float* x, int64_t count) {
  for (int64_t i = 0; i < count; ++i)
    if (!isfinite(x[i])) return i;
  return -1;
}

/* prom_reduction_cpu_reference (reactor_vulkan_fused_reduction.c:996-1036):
   SUM accumulates in double and rounds once; MAX is exact; SOFTMAX subtracts
   the fp32 row max, sums exp() in double and divides in double.  Returns 0
   on success, -6814 on non-finite input (the reference's detail code). */
typedef struct {
  int64_t width;
  int op;
  const float* in;
  float* out;
} reduce_ctx;

static void reduce_range(void* p, int64_t begin, int64_t end) {
  const reduce_ctx* x = (const reduce_ctx*)p;
  const int64_t width = x->width;
  const int op = x->op;
  float* out = x->out;
  for (int64_t row = begin; row < end; ++row) {
    const float* v = x->in + row * width;
    if (op == OP_SUM) {
      double acc = 0.0;
      for (int64_t c = 0; c < width; ++c) acc += (double)v[c];
      out[row] = (float)acc;
    } else if (op == OP_MAX) {
      float mx = v[0];
      for (int64_t c = 1; c < width; ++c)
        if (v[c] > mx) mx = v[c];
      out[row] = mx;
    } else {
      float mx = v[0];
      double den = 0.0;
      for (int64_t c = 1; c < width; ++c)
        if (v[c] > mx) mx = v[c];
      for (int64_t c = 0; c < width; ++c) den += exp((double)v[c] - mx);
      for (int64_t c = 0; c < width; ++c) out[row * width + c] = (float)(exp((double)v[c] - mx) / den);
    }
  }
}

ORACLE_API int oracle_reduction_cpu_reference(int64_t rows, int64_t width, int op, const float* in, float* out,
                                              int threads) {
  if (oracle_find_nonfinite(in, rows * width) >= 0) return -6814;
  reduce_ctx x = {width, op, in, out};
  parallel_rows(threads, 0, rows, reduce_range, &x);
  return 0;
}

/* prom_reduction_compare (reactor_vulkan_fused_reduction.c:1038-1114).
   Tolerances: SUM abs 2e-5*W or rel 2e-5; MAX exact; SOFTMAX abs 2e-5 or rel
   2e-4, every value >= -2e-7 and each row summing to 1 within 3e-4.
   Relative error divides by |expected| floored at 1 below 1e-20.
   Returns 0 on pass, 1 on the first mismatch (reported in *mm). */
typedef struct OracleMismatch {
  int64_t row;
  int64_t column;
  float expected;
  float actual;
  float abs_error;
  float rel_error;
} OracleMismatch;

static float rel_err_floor(float expected, float actual) {
  float den = fabsf(expected);
  if (den < 1.0e-20f) den = 1.0f;
  return fabsf(actual - expected) / den;
}

ORACLE_API int oracle_reduction_compare(int64_t rows, int64_t width, int op, const float* expected,
                                        const float* actual, OracleMismatch* mm) {
  const int64_t count = op == OP_SOFTMAX ? rows * width : rows;
  const float atol = op == OP_SOFTMAX ? 2.0e-5f : (op == OP_MAX ? 0.0f : 2.0e-5f * (float)width);
  const float rtol = op == OP_SOFTMAX ? 2.0e-4f : (op == OP_MAX ? 0.0f : 2.0e-5f);
  for (int64_t i = 0; i < count; ++i) {
    const float ae = fabsf(actual[i] - expected[i]);
    const float re = rel_err_floor(expected[i], actual[i]);
    if (!isfinite(actual[i]) || (ae > atol && re > rtol)) {
      if (mm != NULL) {
        mm->row = op == OP_SOFTMAX ? i / width : i;
        mm->column = op == OP_SOFTMAX ? i % width : -1;
        mm->expected = expected[i];
        mm->actual = actual[i];
        mm->abs_error = ae;
        mm->rel_error = re;
      }
      return 1;
    }
  }
  if (op == OP_SOFTMAX) {
    for (int64_t r = 0; r < rows; ++r) {
      double s = 0.0;
      for (int64_t c = 0; c < width; ++c) {
        const float v = actual[r * width + c];
        if (!isfinite(v) || v < -2.0e-7f) {
          if (mm != NULL) {
            mm->row = r;
            mm->column = c;
            mm->expected = 0.0f;
            mm->actual = v;
            mm->abs_error = fabsf(v);
            mm->rel_error = fabsf(v);
          }
          return 1;
        }
        s += v;
      }
      if (fabs(s - 1.0) > 3.0e-4) {
        if (mm != NULL) {
          mm->row = r;
          mm->column = -1;
          mm->expected = 1.0f;
          mm->actual = (float)s;
          mm->abs_error = (float)fabs(s - 1.0);
          mm->rel_error = mm->abs_error;
        }
        return 1;
      }
    }
  }
  return 0;
}

/* ---------------------------------------------------------------- RMSNorm */

/* cpuHeadRMSNorm (internal/prometheus/gemma4e2b_m1_rtx.go:811-832) and
   CanonicalRMSNorm (internal/prometheus/zimage/canonical_contract.go:91-105),
   per row: fp32 left-to-right sum of squares, m = sum/W + eps in fp32, then
     head form (form 0):      scale = float32(1.0 / sqrt(float64(m)))
     canonical form (form 1): scale = float32(1) / float32(sqrt(float64(m)))
   (the canonical form rounds the square root to fp32 and divides in fp32),
   and out = x * scale * weight in fp32, left to right. */
typedef struct {
  int64_t width, stride;
  const float* in;
  const float* weight;
  float eps;
  double eps64;
  float* out;
  float* inv;
  double* out64;
  double* inv64;
  int form;
} rms_ctx;

static void rms_f32_range(void* p, int64_t begin, int64_t end) {
  const rms_ctx* q = (const rms_ctx*)p;
  const int64_t width = q->width;
  for (int64_t r = begin; r < end; ++r) {
    const float* x = q->in + r * q->stride;
    float sum = 0.0f;
    for (int64_t c = 0; c < width; ++c) sum += x[c] * x[c];
    const float m = sum / (float)width + q->eps;
    const float scale = q->form == 1 ? 1.0f / (float)sqrt((double)m) : (float)(1.0 / sqrt((double)m));
    if (q->inv != NULL) q->inv[r] = scale;
    for (int64_t c = 0; c < width; ++c) q->out[r * width + c] = x[c] * scale * q->weight[c];
  }
}

ORACLE_API void oracle_rmsnorm_f32(int64_t rows, int64_t width, int64_t stride, const float* in, const float* weight,
                                   float eps, float* out, float* inv_rms, int threads, int form) {
  rms_ctx q = {width, stride, in, weight, eps, 0.0, out, inv_rms, NULL, NULL, form};
  parallel_rows(threads, 0, rows, rms_f32_range, &q);
}

/* The same formula evaluated in binary64 throughout (the fp64 oracle). */
static void rms_f64_range(void* p, int64_t begin, int64_t end) {
  const rms_ctx* q = (const rms_ctx*)p;
  const int64_t width = q->width;
  for (int64_t r = begin; r < end; ++r) {
    const float* x = q->in + r * q->stride;
    double sum = 0.0;
    for (int64_t c = 0; c < width; ++c) sum += (double)x[c] * (double)x[c];
    const double scale = 1.0 / sqrt(sum / (double)width + q->eps64);
    if (q->inv64 != NULL) q->inv64[r] = scale;
    for (int64_t c = 0; c < width; ++c) q->out64[r * width + c] = (double)x[c] * scale * (double)q->weight[c];
  }
}

ORACLE_API void oracle_rmsnorm_f64(int64_t rows, int64_t width, int64_t stride, const float* in, const float* weight,
                                   double eps, double* out, double* inv_rms, int threads) {
  rms_ctx q = {width, stride, in, weight, 0.0f, eps, NULL, NULL, out, inv_rms, 0};
  parallel_rows(threads, 0, rows, rms_f64_range, &q);
}

/* ---------------------------------------------------------------- Gemma M1 BF16 boundary */

/* float32ToBF16 then bf16ToFloat32 (internal/prometheus/gemma4e2b_m1_rtx.go:1005-1014):
   round to nearest even on the fp32 bit pattern, re-expanded to fp32. */
static float bf16_round(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  b += 0x7fffu + ((b >> 16) & 1u);
  b &= 0xffff0000u;
  float r;
  memcpy(&r, &b, 4);
  return r;
}

ORACLE_API void oracle_bf16_round(int64_t n, const float* in, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_round(in[i]);
}

/* The reference's own RMSNorm oracle with optional BF16 rounding of input and
   output (internal/prometheus/native/Marionette/reactor_concept_rmsnorm_tests.cpp:17-35,
   the arithmetic of the M46 family, reactor_api.c:250-395): binary64 sum of
   squares, inv = float(1 / sqrt(sum / width + eps)) in binary64, value =
   (x * inv) * weight in fp32, then the optional output rounding. */
ORACLE_API void oracle_m1_rmsnorm(int64_t rows, int64_t width, int64_t stride, const float* in, const float* weight,
                                  float eps, int round_in, int round_out, float* out, float* inv_rms) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = in + r * stride;
    double sum = 0.0;
    for (int64_t c = 0; c < width; ++c) {
      const double v = round_in ? bf16_round(x[c]) : x[c];
      sum += v * v;
    }
    const float inv = (float)(1.0 / sqrt(sum / (double)width + (double)eps));
    if (inv_rms != NULL) inv_rms[r] = inv;
    for (int64_t c = 0; c < width; ++c) {
      const float v = round_in ? bf16_round(x[c]) : x[c];
      const float t = v * inv * weight[c];
      out[r * width + c] = round_out ? bf16_round(t) : t;
    }
  }
}

/* cpuGemma4e2bRope (internal/prometheus/gemma4e2b_m1_rtx.go:834-861): for row
   (token, head) and component c, f = c mod hw/2, mate = the other half's c;
   first = bf16(x[c] * cos[token][f]), second = bf16(x[mate] * sin[token][f]),
   out = bf16(first - second) for the first half, bf16(first + second) for the
   second.  Tables are [token][hw]; only their first hw/2 entries are read. */
ORACLE_API void oracle_m1_rope(int64_t tokens, int64_t heads, int64_t hw, const float* src, const float* cos_t,
                               const float* sin_t, float* out) {
  const int64_t half = hw / 2;
  for (int64_t t = 0; t < tokens; ++t)
    for (int64_t h = 0; h < heads; ++h) {
      const int64_t base = (t * heads + h) * hw;
      for (int64_t c = 0; c < hw; ++c) {
        const int64_t f = c % half;
        const int64_t mate = c >= half ? base + f : base + f + half;
        const float first = bf16_round(src[base + c] * cos_t[t * hw + f]);
        const float second = bf16_round(src[mate] * sin_t[t * hw + f]);
        out[base + c] = bf16_round(c >= half ? first + second : first - second);
      }
    }
}

/* Raw pre-mask scores from positioned Q [tokens][qheads][hw] and K [tokens][hw]
   (every query head reads KV head 0, cpuGemma4e2bRawScores,
   gemma4e2b_m1_rtx.go:863-883), out [qheads][tokens][tokens].  form 0 is the
   reference test's independent chain: binary64 dot, times scale, rounded once
   (Marionette/reactor_concept_rmsnorm_tests.cpp:157-162); form 1 is the Go
   loop itself: fp32 accumulation left to right, then * scale in fp32. */
ORACLE_API void oracle_m1_scores(int64_t tokens, int64_t qheads, int64_t hw, const float* q, const float* k,
                                 double scale, int form, float* out) {
  for (int64_t h = 0; h < qheads; ++h)
    for (int64_t i = 0; i < tokens; ++i)
      for (int64_t j = 0; j < tokens; ++j) {
        const float* qr = q + (i * qheads + h) * hw;
        const float* kr = k + j * hw;
        float* dst = out + (h * tokens + i) * tokens + j;
        if (form == 1) {
          float acc = 0.0f;
          for (int64_t d = 0; d < hw; ++d) acc += qr[d] * kr[d];
          *dst = acc * (float)scale;
        } else {
          double acc = 0.0;
          for (int64_t d = 0; d < hw; ++d) acc += (double)qr[d] * (double)kr[d];
          *dst = (float)(acc * scale);
        }
      }
}

/* ---------------------------------------------------------------- FFT */

/* The reference's binary64 FFT (prometheus_reactor_runtime_fft64): twiddles
   computed on the host in binary64, table[2i] = cos(-2 pi i / n),
   table[2i+1] = sin(..) for i < n/2 (internal/prometheus/native/
   reactor_concept_fft.cpp:51-58); one bit-reversal pass and log2(n) radix-2
   butterfly passes through ping-pong buffers, each output formed as
   a +- (wr br - wi bi, wr bi + wi br) with the twiddle lower * (n / span)
   (shaders/sdslv/production/fft/radix2_fp64.sdslv).  `twiddles` receives the n-double table. */
ORACLE_API void oracle_fft64(int64_t n, const double* in, double* out, double* twiddles) {
  const double pi = 3.14159265358979323846264338327950288;
  double* tw = twiddles; /* n doubles */
  for (int64_t i = 0; i < n / 2; ++i) {
    const double angle = -2.0 * pi * (double)i / (double)n;
    tw[2 * i] = cos(angle);
    tw[2 * i + 1] = sin(angle);
  }
  int bits = 0;
  while ((1ll << bits) < n) ++bits;
  double* src = (double*)malloc(sizeof(double) * 2 * (size_t)n);
  double* dst = (double*)malloc(sizeof(double) * 2 * (size_t)n);
  if (src == NULL || dst == NULL) {
    free(src);
    free(dst);
    return;
  }
  for (int64_t i = 0; i < n; ++i) {
    int64_t r = 0, v = i;
    for (int k = 0; k < bits; ++k) {
      r = (r << 1) | (v & 1);
      v >>= 1;
    }
    src[2 * r] = in[2 * i];
    src[2 * r + 1] = in[2 * i + 1];
  }
  for (int64_t half = 1; half < n; half *= 2) {
    const int64_t span = 2 * half;
    for (int64_t index = 0; index < n; ++index) {
      const int64_t lane = index % span, lower = lane % half;
      const int64_t base = index - lane + lower, other = base + half;
      const int64_t t = lower * (n / span);
      const double wr = tw[2 * t], wi = tw[2 * t + 1];
      const double ar = src[2 * base], ai = src[2 * base + 1], br = src[2 * other], bi = src[2 * other + 1];
      const double tr = wr * br - wi * bi, ti = wr * bi + wi * br;
      dst[2 * index] = lane < half ? ar + tr : ar - tr;
      dst[2 * index + 1] = lane < half ? ai + ti : ai - ti;
    }
    double* sw = src;
    src = dst;
    dst = sw;
  }
  for (int64_t i = 0; i < 2 * n; ++i) out[i] = src[i];
  free(src);
  free(dst);
}

/* The fp32 transform of prometheus_reactor_runtime_fft with the shader's per-pass
   angle sign * 2 pi * lower / span in fp32 and libm cosf / sinf for its native
   cos / sin (radix2_butterfly.sdslv); inverse normalisation divides by n in
   the last pass.  `batch` transforms `stride` complex elements apart. */
ORACLE_API void oracle_fft32(int64_t n, int64_t batch, int64_t stride, int inverse, int normalize, const float* in,
                             float* out) {
  int bits = 0;
  while ((1ll << bits) < n) ++bits;
  float* src = (float*)malloc(sizeof(float) * 2 * (size_t)n);
  float* dst = (float*)malloc(sizeof(float) * 2 * (size_t)n);
  if (src == NULL || dst == NULL) {
    free(src);
    free(dst);
    return;
  }
  for (int64_t bt = 0; bt < batch; ++bt) {
    const float* x = in + 2 * bt * stride;
    for (int64_t i = 0; i < n; ++i) {
      int64_t r = 0, v = i;
      for (int k = 0; k < bits; ++k) {
        r = (r << 1) | (v & 1);
        v >>= 1;
      }
      src[2 * r] = x[2 * i];
      src[2 * r + 1] = x[2 * i + 1];
    }
    for (int64_t half = 1; half < n; half *= 2) {
      const int64_t span = 2 * half;
      const int last = normalize && span == n;
      for (int64_t index = 0; index < n; ++index) {
        const int64_t lane = index % span, lower = lane % half;
        const int64_t base = index - lane + lower, other = base + half;
        const float sign = inverse ? 1.0f : -1.0f;
        const float angle = sign * 6.28318530717958647692f * (float)lower / (float)span;
        const float wr = cosf(angle), wi = sinf(angle);
        const float br = src[2 * other], bi = src[2 * other + 1];
        const float tr = wr * br - wi * bi, ti = wr * bi + wi * br;
        float re = lane < half ? src[2 * base] + tr : src[2 * base] - tr;
        float im = lane < half ? src[2 * base + 1] + ti : src[2 * base + 1] - ti;
        if (last) {
          re = re / (float)n;
          im = im / (float)n;
        }
        dst[2 * index] = re;
        dst[2 * index + 1] = im;
      }
      float* sw = src;
      src = dst;
      dst = sw;
    }
    for (int64_t i = 0; i < 2 * n; ++i) out[2 * bt * stride + i] = src[i];
  }
  free(src);
  free(dst);
}

ORACLE_API int oracle_max_threads(void) {
  const long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}
