// diagnostics_api.cpp -- the reduction diagnostics / benchmark entries and the
// async SGEMM diagnostics of the C ABI.
//
//   prometheus_reactor_runtime_reduction_diagnostics  reactor_concept_reduction.cpp:96-110
//   prometheus_reactor_runtime_reduction_benchmark    reactor_vulkan_fused_reduction.c:1122-1206
//   prometheus_reactor_runtime_sgemm_async_diagnostics reactor_sgemm.cpp:6371-6412
//
// Counters keep the reference's field meanings with their CUDA counterparts: a
// handle serialises its reductions on one stream (one physical slot that is
// never quarantined), a "command record" is one prepared launch sequence and a
// "queue submit" one enqueued reduction kernel.  The benchmark's correctness
// check runs on the device (oct::reduction_self_check): an independent
// recomputation and the reference comparator's tolerances.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "runtime.h"

namespace {

using namespace oct::rt;

}  // namespace

extern "C" {

int prometheus_reactor_runtime_reduction_diagnostics(void* handle, PrometheusReductionDiagnostics* out) {
  if (out == nullptr) return PROM_ERROR;
  try {
    std::memset(out, 0, sizeof(*out));
    out->struct_size = sizeof(*out);
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    const ReductionStats& st = rt->red_stats;
    out->configured_ring_depth = st.ring_depth;
    out->physical_slot_count = 1;
    out->validation_enabled = 0;
    out->validation_error_count = 0;
    if (!st.initialized) return PROM_OK;
    out->initialized = 1;
    out->production_enabled = 1;
    out->next_logical_request_id = rt->next_request_id;
    out->total_requests = st.total;
    out->successful_requests = st.success;
    out->logical_failure_count = st.failures;
    out->physical_recycle_count = st.total;
    out->reap_count = st.total;
    out->pipeline_create_count = 1;
    out->command_record_count = st.command_records;
    out->queue_submit_count = st.submits;
    out->buffer_allocation_count = st.allocations;
    out->buffer_reuse_count = st.reuses;
    out->temporary_capacity_bytes = rt->rin.cap + rt->rout.cap;
    out->last_replay_id = st.last_replay;
    out->last_gpu_duration_ns = st.last_gpu_ns;
    out->last_end_to_end_ns = st.last_e2e_ns;
    out->last_stage_count = st.last_stage_count;
    out->last_physical_slot_id = 0;
    out->last_physical_slot_generation = st.slot_generation;
    out->last_detail_code = st.last_detail;
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_reduction_benchmark(void* handle, const PrometheusReductionBenchmarkRequest* request,
                                                   PrometheusReductionBenchmarkResult* out_result) {
  if (out_result == nullptr) return PROM_ERROR;
  PrometheusReductionBenchmarkResult& out = *out_result;
  try {
    std::memset(&out, 0, sizeof(out));
    out.struct_size = sizeof(out);
    out.first_mismatch_row = UINT32_MAX;
    out.first_mismatch_column = UINT32_MAX;
    if (request == nullptr || request->struct_size < sizeof(*request) || request->measured_iterations == 0 ||
        request->measured_iterations > 10000u) {
      out.detail_code = PROM_REDUCTION_DETAIL_INVALID_REQUEST;
      return PROM_ERROR;
    }
    PrometheusReductionRequest exec = request->reduction;
    PrometheusReductionExecutionResult res{};
    for (uint32_t i = 0; i < request->warmup_iterations; ++i) {
      if (prometheus_reactor_runtime_reduction(handle, &exec, &res) != PROM_OK) {
        out.detail_code = res.detail_code;
        return PROM_ERROR;
      }
    }
    std::vector<uint64_t> gpu(request->measured_iterations), e2e(request->measured_iterations);
    for (uint32_t i = 0; i < request->measured_iterations; ++i) {
      if (prometheus_reactor_runtime_reduction(handle, &exec, &res) != PROM_OK) {
        out.detail_code = res.detail_code;
        return PROM_ERROR;
      }
      gpu[i] = res.gpu_duration_ns;
      e2e[i] = res.end_to_end_ns;
      out.completed_iterations += 1;
    }
    // The executions validated the request; check the caller's last output on the device.
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      out.detail_code = PROM_REDUCTION_DETAIL_RUNTIME_UNAVAILABLE;
      return PROM_INVALID_HANDLE;
    }
    const uint32_t rows = exec.row_count, width = exec.elements_per_row, op = exec.operation;
    const uint64_t total = static_cast<uint64_t>(rows) * width;
    const uint64_t out_count = op == PROM_REDUCTION_OPERATION_SOFTMAX ? total : rows;
    {
      std::lock_guard<std::mutex> lock(rt->mu);
      if (rt->rin.ensure(total * 4, rt->stream) != cudaSuccess ||
          rt->rout.ensure(2 * out_count * 4, rt->stream) != cudaSuccess) {
        out.detail_code = PROM_REDUCTION_DETAIL_RESOURCE_CREATE_FAILED;
        return PROM_ERROR;
      }
      float* din = static_cast<float*>(rt->rin.aligned());
      float* dact = static_cast<float*>(rt->rout.aligned());
      float* dexp = dact + out_count;
      cudaError_t e = reset_words(rt);
      if (e == cudaSuccess) e = cudaMemcpyAsync(din, exec.input, total * 4, cudaMemcpyHostToDevice, rt->stream);
      if (e == cudaSuccess) e = cudaMemcpyAsync(dact, exec.output, out_count * 4, cudaMemcpyHostToDevice, rt->stream);
      if (e == cudaSuccess)
        e = oct::reduction_self_check(din, dact, dexp, rows, width, op, rt->nonfinite_word(), rt->stream);
      Words w;
      if (e != cudaSuccess || read_words(rt, &w) != cudaSuccess) {
        (void)cudaGetLastError();
        out.detail_code = PROM_REDUCTION_DETAIL_COMPLETION_UNCERTAIN;
        return PROM_ERROR;
      }
      if (w.nonfinite != ~0ull) {
        const float* actual = static_cast<const float*>(exec.output);
        if (w.nonfinite < out_count) {
          const uint64_t i = w.nonfinite;
          float expected = 0.f;
          if (cudaMemcpy(&expected, dexp + i, 4, cudaMemcpyDeviceToHost) != cudaSuccess) (void)cudaGetLastError();
          out.first_mismatch_row = static_cast<uint32_t>(op == PROM_REDUCTION_OPERATION_SOFTMAX ? i / width : i);
          out.first_mismatch_column =
              op == PROM_REDUCTION_OPERATION_SOFTMAX ? static_cast<uint32_t>(i % width) : UINT32_MAX;
          out.first_expected = expected;
          out.first_actual = actual[i];
          out.first_absolute_error = std::fabs(actual[i] - expected);
          const float den = std::fabs(expected) < 1.0e-20f ? 1.0f : std::fabs(expected);
          out.first_relative_error = out.first_absolute_error / den;
        } else {  // a softmax row whose values do not sum to one
          const uint64_t r = w.nonfinite - out_count;
          out.first_mismatch_row = static_cast<uint32_t>(r);
          out.first_expected = 1.0f;
          out.first_actual = std::nanf("");
        }
        out.detail_code = PROM_REDUCTION_DETAIL_READBACK_FAILED;
        return PROM_ERROR;
      }
    }
    out.correctness_passed = 1;
    std::sort(gpu.begin(), gpu.end());
    std::sort(e2e.begin(), e2e.end());
    const size_t n = gpu.size();
    out.gpu_min_ns = gpu.front();
    out.gpu_median_ns = gpu[n / 2];
    out.gpu_max_ns = gpu.back();
    out.end_to_end_min_ns = e2e.front();
    out.end_to_end_median_ns = e2e[n / 2];
    out.end_to_end_max_ns = e2e.back();
    out.stage_count = res.plan.stage_count;
    out.temporary_bytes = res.plan.temporary_bytes;
    out.replay_id = res.plan.replay_id;
    out.validation_passed = 1;  // no validation layer exists to report errors
    out.detail_code = 0;
    return PROM_OK;
  } catch (...) {
    out.detail_code = PROM_REDUCTION_DETAIL_RESOURCE_CREATE_FAILED;
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_sgemm_async_diagnostics(void* handle, PrometheusSgemmAsyncDiagnostics* out) {
  if (out == nullptr) return PROM_ERROR;
  try {
    std::memset(out, 0, sizeof(*out));
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    const AsyncStats& st = rt->async_stats;
    out->task_capacity = kAsyncSlots;
    out->queue_full_count = st.queue_full;
    out->stale_id_rejection_count = st.stale_ids;
    out->max_in_flight = st.max_in_flight;
    out->reap_poll_count = st.polls;
    out->reap_success_count = st.reaped;
    for (int i = 0; i < kAsyncSlots; ++i) {
      const AsyncTask& t = rt->tasks[i];
      PrometheusSgemmAsyncTaskDiagnostics& d = out->tasks[i];
      if (!t.active) continue;
      out->active_task_count += 1;
      if (t.state == PROM_ASYNC_STATE_SUBMITTED) out->submitted_count += 1;
      if (t.state == PROM_ASYNC_STATE_READY) out->ready_count += 1;
      if (t.state == PROM_ASYNC_STATE_FAILED) out->failed_count += 1;
      if (t.state == PROM_ASYNC_STATE_CONSUMED) out->consumed_count += 1;
      if (t.abandoned) out->abandoned_count += 1;
      d.task_id = t.id;
      d.generation = t.generation;
      d.lifecycle_state = t.state;
      d.physical_slot_id = static_cast<uint32_t>(i);
      d.physical_slot_generation = t.generation;
      d.submission_sequence = t.sequence;
      d.timing_valid = t.timed ? 1u : 0u;
      d.gpu_duration_ns = t.gpu_ns;
      d.failure_detail = t.state == PROM_ASYNC_STATE_FAILED ? t.final_detail : 0;
      d.failure_class = t.state == PROM_ASYNC_STATE_FAILED ? 1u : 0u;
      d.abandoned = t.abandoned ? 1u : 0u;
      d.physical_slot_state = t.state;
      const bool done = t.state == PROM_ASYNC_STATE_READY || t.state == PROM_ASYNC_STATE_FAILED ||
                        t.state == PROM_ASYNC_STATE_CONSUMED;
      d.physical_completion_confirmed = done ? 1u : 0u;
      d.reap_pending = t.state == PROM_ASYNC_STATE_SUBMITTED ? 1u : 0u;
      d.reap_completed = done ? 1u : 0u;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

}  // extern "C"
