// fft_api.cpp -- the FFT entry points of the C ABI (fft.cu does the transforms).
//
// Validation order, detail codes, stages and the diagnostics record follow
// internal/prometheus/native/reactor_vulkan_fft.c:26-128 and
// reactor_concept_fft.cpp:38-116.  The binary64 twiddle table is computed on the
// host once per size, exactly as the reference computes it
// (angle = -2 pi i / N in binary64, cos and sin, reactor_concept_fft.cpp:51-58),
// and uploaded; the transform itself runs on the device only.
#include <cmath>
#include <cstring>
#include <vector>

#include "runtime.h"

namespace {

using namespace oct::rt;

constexpr uint32_t kForward = 1, kInverse = 2;         // PROM_FFT_DIRECTION_* (reactor_vulkan_fft.c:7-8)
constexpr uint32_t kRolePing = 2, kRolePong = 3;       // buffer roles of the plan (:16-19)
constexpr uint32_t kTwiddleNativeSinCos = 2;           // PROM_FFT_TWIDDLE_MODE_NATIVE_SIN_COS (:12)
constexpr double kPi = 3.14159265358979323846264338327950288;

PrometheusFftDiagnostics default_diag() {
  PrometheusFftDiagnostics d{};
  d.struct_size = sizeof(d);
  d.api_declared = 1;
  d.last_failure_detail = PROM_FFT_DETAIL_UNAVAILABLE;
  d.last_validation_status = PROM_FFT_PATH_STATUS_UNAVAILABLE;
  d.executed_path_id = PROM_FFT_PATH_UNAVAILABLE;
  return d;
}

PrometheusFftDiagnostics& diag_of(Runtime* rt) {
  if (!rt->fft_diag_init) {
    rt->fft_diag = default_diag();
    rt->fft_diag_init = true;
  }
  return rt->fft_diag;
}

bool pow2(uint32_t v) { return v != 0 && (v & (v - 1)) == 0; }
uint32_t log2u(uint32_t v) {
  uint32_t b = 0;
  while (v > 1) {
    v >>= 1;
    ++b;
  }
  return b;
}

// prom_fft_validate_request (reactor_vulkan_fft.c:59-86): 0 or a detail code.
int validate(const PrometheusFftRequest* r, uint32_t* direction, uint64_t* physical) {
  if (r == nullptr || r->struct_size < sizeof(*r)) return PROM_FFT_DETAIL_INVALID_REQUEST;
  if (r->input == nullptr) return PROM_FFT_DETAIL_NULL_INPUT;
  if (r->output == nullptr) return PROM_FFT_DETAIL_NULL_OUTPUT;
  if (r->element_count == 0) return PROM_FFT_DETAIL_ZERO_ELEMENT_COUNT;
  if (!pow2(r->element_count)) return PROM_FFT_DETAIL_NON_POWER_OF_TWO;
  if (r->element_count > oct::kFftMaxElements) return PROM_FFT_DETAIL_UNSUPPORTED_SIZE;
  if (r->batch_count == 0) return PROM_FFT_DETAIL_ZERO_BATCH_COUNT;
  if ((r->flags & PROM_FFT_FLAG_FORWARD) && (r->flags & PROM_FFT_FLAG_INVERSE))
    return PROM_FFT_DETAIL_INVALID_DIRECTION_FLAGS;
  if ((r->flags & PROM_FFT_FLAG_INVERSE_NORMALIZE) && !(r->flags & PROM_FFT_FLAG_INVERSE))
    return PROM_FFT_DETAIL_INVERSE_NORMALIZE_REQUIRES_INVERSE;
  if (r->stride_elements != 0 && r->stride_elements < r->element_count) return PROM_FFT_DETAIL_INVALID_STRIDE;
  if (r->stride_elements != 0 && r->batch_count > UINT32_MAX / r->stride_elements) return PROM_FFT_DETAIL_SIZE_OVERFLOW;
  const uint32_t stride = r->stride_elements == 0 ? r->element_count : r->stride_elements;
  const uint64_t elems = static_cast<uint64_t>(r->batch_count - 1) * stride + r->element_count;
  if (elems == 0 || elems * sizeof(PrometheusComplex32) > UINT32_MAX) return PROM_FFT_DETAIL_SIZE_OVERFLOW;
  if (static_cast<uint64_t>(r->element_count) * r->batch_count > 65535ull * 256ull) return PROM_FFT_DETAIL_UNSUPPORTED_SIZE;
  *direction = (r->flags & PROM_FFT_FLAG_INVERSE) ? kInverse : kForward;
  *physical = elems;
  return 0;
}

// The radix-2 plan's bookkeeping (reactor_vulkan_fft.c:88-101) into the diagnostics.
void apply_plan(PrometheusFftDiagnostics& d, uint32_t n, uint32_t direction) {
  const uint32_t passes = log2u(n);
  d.plan_valid = 1;
  d.plan_element_count = n;
  d.plan_log2_element_count = passes;
  d.plan_pass_count = passes;
  d.ping_pong_swap_count = passes;
  // passes alternate ping -> pong -> ping ...; the last destination holds the output
  d.final_output_role = passes == 0 ? kRolePing : (passes % 2 == 1 ? kRolePong : kRolePing);
  d.plan_first_span = passes > 0 ? 2 : 0;
  d.plan_last_span = passes > 0 ? n : 0;
  d.plan_radix_mask = passes > 0 ? (1u << 2) : 0;
  d.plan_bit_reversal_required = n > 1 ? 1 : 0;
  d.plan_first_source_role = passes > 0 ? kRolePing : 1;
  d.plan_first_destination_role = passes > 0 ? kRolePong : kRolePing;
  d.plan_direction = direction;
  d.plan_twiddle_mode = kTwiddleNativeSinCos;
}

cudaError_t stage_fft(Runtime* rt, DevBuf& b, uint64_t bytes, int slot) {
  if (b.raw != nullptr && bytes <= b.cap) {
    ++rt->fft_reuse[slot];
    return cudaSuccess;
  }
  ++rt->fft_grow[slot];
  return b.ensure(bytes, rt->stream);
}

void set(uint32_t* stage, int* detail, uint32_t s, int d) {
  if (stage != nullptr) *stage = s;
  if (detail != nullptr) *detail = d;
}

// Host-side fault injection (PROM_TESTCFG_*), as the reference's FFT tests drive it
// (Marionette/reactor_fft64_tests.cpp:59-76): the output is never written.
int injected(const Runtime* rt, uint32_t* stage) {
  if (rt->test_flags & PROM_TESTCFG_FAIL_BUFFER_ALLOC) {
    *stage = PROM_STAGE_INIT;
    return PROM_FFT_DETAIL_ALLOCATION_FAILED;
  }
  if (rt->test_flags & PROM_TESTCFG_FAIL_UPLOAD) {
    *stage = PROM_STAGE_TRANSFER_IN;
    return PROM_FFT_DETAIL_UPLOAD_FAILED;
  }
  if (rt->test_flags & PROM_TESTCFG_FAIL_DISPATCH) {
    *stage = PROM_STAGE_SUBMIT;
    return PROM_FFT_DETAIL_DISPATCH_FAILED;
  }
  if (rt->test_flags & PROM_TESTCFG_FAIL_DOWNLOAD) {
    *stage = PROM_STAGE_TRANSFER_OUT;
    return PROM_FFT_DETAIL_READBACK_FAILED;
  }
  return 0;
}

}  // namespace

extern "C" {

int prometheus_reactor_runtime_fft64(void* handle, const double* input, double* output, uint32_t count,
                                     uint32_t* stage, int* detail) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      set(stage, detail, PROM_STAGE_INIT, PROM_INVALID_HANDLE);
      return PROM_INVALID_HANDLE;
    }
    if (input == nullptr || output == nullptr || !pow2(count) || count > oct::kFftMaxElements) {
      set(stage, detail, PROM_STAGE_INIT, PROM_FFT_DETAIL_INVALID_REQUEST);
      return PROM_ERROR;
    }
    if (!rt->available) {
      set(stage, detail, PROM_STAGE_INIT, PROM_FFT_DETAIL_VULKAN_UNAVAILABLE);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    uint32_t fstage = PROM_STAGE_INIT;
    const int inj = injected(rt, &fstage);
    if (inj != 0) {
      set(stage, detail, fstage, inj);
      return PROM_ERROR;
    }
    const uint64_t bytes = 16ull * count;
    if (stage_fft(rt, rt->fft_in, bytes, 0) != cudaSuccess || stage_fft(rt, rt->fft_out, bytes, 1) != cudaSuccess ||
        stage_fft(rt, rt->fft_tw, 8ull * count, 2) != cudaSuccess) {
      (void)cudaGetLastError();
      set(stage, detail, PROM_STAGE_INIT, PROM_FFT_DETAIL_ALLOCATION_FAILED);
      return PROM_ERROR;
    }
    double* din = static_cast<double*>(rt->fft_in.aligned());
    double* dout = static_cast<double*>(rt->fft_out.aligned());
    double* dtw = static_cast<double*>(rt->fft_tw.aligned());
    cudaError_t e = cudaSuccess;
    if (rt->fft_tw_count != count) {
      std::vector<double> table(count);
      for (uint32_t i = 0; i < count / 2; ++i) {
        const double angle = -2.0 * kPi * i / count;
        table[2 * i] = std::cos(angle);
        table[2 * i + 1] = std::sin(angle);
      }
      e = cudaMemcpyAsync(dtw, table.data(), 8ull * count, cudaMemcpyHostToDevice, rt->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);  // `table` is pageable and local
      rt->fft_tw_count = e == cudaSuccess ? count : 0;
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(din, input, bytes, cudaMemcpyHostToDevice, rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      set(stage, detail, PROM_STAGE_TRANSFER_IN, PROM_FFT_DETAIL_UPLOAD_FAILED);
      return PROM_ERROR;
    }
    e = oct::fft64(din, dout, count, dtw, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      set(stage, detail, PROM_STAGE_SUBMIT, PROM_FFT_DETAIL_DISPATCH_FAILED);
      return PROM_ERROR;
    }
    e = cudaMemcpyAsync(output, dout, bytes, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      set(stage, detail, PROM_STAGE_TRANSFER_OUT, PROM_FFT_DETAIL_READBACK_FAILED);
      return PROM_ERROR;
    }
    set(stage, detail, PROM_STAGE_TRANSFER_OUT, 0);
    return PROM_OK;
  } catch (...) {
    set(stage, detail, PROM_STAGE_INIT, PROM_FFT_DETAIL_ALLOCATION_FAILED);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_fft(void* handle, const PrometheusFftRequest* r, uint32_t* out_stage,
                                   int* out_detail_code) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      set(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_INVALID_HANDLE);
      return PROM_INVALID_HANDLE;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    PrometheusFftDiagnostics& d = diag_of(rt);
    d = default_diag();
    d.ping_arena_grow_count = rt->fft_grow[0];  // the arena counters are cumulative
    d.ping_arena_reuse_count = rt->fft_reuse[0];
    d.pong_arena_grow_count = rt->fft_grow[1];
    d.pong_arena_reuse_count = rt->fft_reuse[1];
    if (r != nullptr) {
      d.last_element_count = r->element_count;
      d.last_batch_count = r->batch_count;
      d.last_stride_elements = r->stride_elements;
      d.last_flags = r->flags;
      d.last_effective_stride_elements = r->stride_elements == 0 ? r->element_count : r->stride_elements;
    }
    uint32_t direction = kForward;
    uint64_t physical = 0;
    const int v = validate(r, &direction, &physical);
    if (v != 0) {
      d.last_direction = direction;
      d.last_failure_detail = v;
      set(out_stage, out_detail_code, PROM_STAGE_INIT, v);
      return PROM_ERROR;
    }
    apply_plan(d, r->element_count, direction);
    d.last_direction = direction;
    d.requested_path_id = PROM_FFT_PATH_VULKAN_RADIX2_RESERVED;
    d.requested_radix = 2;
    if (!rt->available) {
      d.last_failure_detail = PROM_FFT_DETAIL_VULKAN_UNAVAILABLE;
      set(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_FFT_DETAIL_VULKAN_UNAVAILABLE);
      return PROM_ERROR;
    }
    d.capability_reported = d.production_enabled = d.benchmark_enabled = 1;
    d.last_validation_status = PROM_FFT_PATH_STATUS_BENCHMARK_ENABLED;
    auto fail = [&](uint32_t s, int det) {
      (void)cudaGetLastError();
      d.executed_path_id = PROM_FFT_PATH_UNAVAILABLE;
      d.last_failure_detail = det;
      set(out_stage, out_detail_code, s, det);
      return PROM_ERROR;
    };
    uint32_t fstage = PROM_STAGE_INIT;
    const int inj = injected(rt, &fstage);
    if (inj != 0) return fail(fstage, inj);
    const uint32_t n = r->element_count, batch = r->batch_count;
    const uint64_t stride = r->stride_elements == 0 ? n : r->stride_elements;
    const uint64_t bytes = physical * sizeof(PrometheusComplex32);
    if (stage_fft(rt, rt->fft_in, bytes, 0) != cudaSuccess || stage_fft(rt, rt->fft_out, bytes, 1) != cudaSuccess)
      return fail(PROM_STAGE_INIT, PROM_FFT_DETAIL_ALLOCATION_FAILED);
    float* din = static_cast<float*>(rt->fft_in.aligned());
    float* dout = static_cast<float*>(rt->fft_out.aligned());
    if (cudaMemcpyAsync(din, r->input, bytes, cudaMemcpyHostToDevice, rt->stream) != cudaSuccess)
      return fail(PROM_STAGE_TRANSFER_IN, PROM_FFT_DETAIL_UPLOAD_FAILED);
    cudaError_t e = oct::fft32(din, dout, n, batch, stride, direction == kInverse,
                               (r->flags & PROM_FFT_FLAG_INVERSE_NORMALIZE) != 0, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) return fail(PROM_STAGE_SUBMIT, PROM_FFT_DETAIL_DISPATCH_FAILED);
    // each batch's n outputs only; the caller's elements between batches stay as they are
    e = cudaMemcpy2DAsync(r->output, stride * sizeof(PrometheusComplex32), dout, stride * sizeof(PrometheusComplex32),
                          n * sizeof(PrometheusComplex32), batch, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) return fail(PROM_STAGE_TRANSFER_OUT, PROM_FFT_DETAIL_READBACK_FAILED);
    d.executed_path_id = PROM_FFT_PATH_VULKAN_RADIX2_RESERVED;
    d.executed_radix = 2;
    d.last_failure_detail = 0;
    d.ping_arena_grow_count = rt->fft_grow[0];
    d.ping_arena_reuse_count = rt->fft_reuse[0];
    d.pong_arena_grow_count = rt->fft_grow[1];
    d.pong_arena_reuse_count = rt->fft_reuse[1];
    set(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, 0);
    return PROM_OK;
  } catch (...) {
    set(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_FFT_DETAIL_ALLOCATION_FAILED);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_fft_benchmark_variant(void* handle, const PrometheusFftRequest* request,
                                                     uint32_t requested_variant, uint32_t* out_stage,
                                                     int* out_detail_code) {
  if (requested_variant != PROM_FFT_BENCHMARK_VARIANT_RADIX2) {
    set(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_FFT_DETAIL_PLAN_DISPATCH_DISAGREEMENT);
    return PROM_ERROR;
  }
  return prometheus_reactor_runtime_fft(handle, request, out_stage, out_detail_code);
}

int prometheus_reactor_runtime_fft_diagnostics_sized(void* handle, PrometheusFftDiagnostics* out_diag,
                                                     uint32_t out_size) {
  try {
    if (out_diag == nullptr || out_size == 0) return PROM_ERROR;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    const PrometheusFftDiagnostics& d = diag_of(rt);
    if (out_size > sizeof(d)) out_size = sizeof(d);
    std::memset(out_diag, 0, out_size);
    std::memcpy(out_diag, &d, out_size);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_fft_diagnostics(void* handle, PrometheusFftDiagnostics* out_diag) {
  return prometheus_reactor_runtime_fft_diagnostics_sized(handle, out_diag, sizeof(PrometheusFftDiagnostics));
}

}  // extern "C"
