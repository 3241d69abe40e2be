// reactor_api.cpp -- the C ABI of libprometheus_reactor.so (ABI v1) over CUDA.
//
// This file is the drop-in boundary: the symbols, argument meanings, status /
// stage / detail conventions and validation order of Oct's Prometheus reactor
// (internal/prometheus/native/reactor_api.h, reactor_api.c, reactor_sgemm.cpp,
// reactor_concept_reduction.cpp, reactor_vulkan_fused_reduction.c), with the
// Vulkan runtime underneath replaced by one CUDA stream per handle and the
// kernels in sgemm_tc.cu, sgemm_fma.cu and reduce.cu.
//
// There is no CPU fallback anywhere: a handle without a usable sm_100 device
// reports available=0 from probe and every compute call fails with a detail
// code.  No C++ exception crosses the boundary (each entry point catches).
#include "../../include/prometheus_reactor.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "block.h"
#include "kernels.h"
#include "runtime.h"

namespace oct {
namespace rt {

std::mutex g_registry_mu;
std::unordered_set<Runtime*>* g_registry = new std::unordered_set<Runtime*>();

Runtime* lookup(void* handle) {
  if (handle == nullptr) return nullptr;
  std::lock_guard<std::mutex> lock(g_registry_mu);
  Runtime* rt = static_cast<Runtime*>(handle);
  if (g_registry->count(rt) == 0 || rt->magic != kMagic) return nullptr;
  return rt;
}

void register_runtime(Runtime* rt) {
  std::lock_guard<std::mutex> lock(g_registry_mu);
  g_registry->insert(rt);
}

void unregister_runtime(Runtime* rt) {
  std::lock_guard<std::mutex> lock(g_registry_mu);
  g_registry->erase(rt);
}

}  // namespace rt
}  // namespace oct

namespace {

using namespace oct::rt;


// The next set of per-launch timing events (created on first use); null on failure.
const oct::SgemmEvents* next_timing_events(Runtime* rt) {
  if (rt->timing_used == rt->timing_events.size()) {
    oct::SgemmEvents fresh;
    if (cudaEventCreate(&fresh.split_begin) != cudaSuccess || cudaEventCreate(&fresh.main_begin) != cudaSuccess ||
        cudaEventCreate(&fresh.main_end) != cudaSuccess)
      return nullptr;
    rt->timing_events.push_back(fresh);
  }
  return &rt->timing_events[rt->timing_used++];
}

// ---------------------------------------------------------------- SGEMM core
// Enqueues C = A * B for device pointers; chooses the kernel.
bool known_variant(uint32_t v) {
  return v == OCT_B200_SGEMM_AUTO || v == OCT_B200_SGEMM_TC3XTF32 || v == OCT_B200_SGEMM_FMA ||
         v == OCT_B200_SGEMM_SMALLM || v == OCT_B200_SGEMM_SMALLM_TC ||
         v == OCT_B200_SGEMM_TC_BK16 || v == OCT_B200_SGEMM_TC_BK32 || v == OCT_B200_SGEMM_TC_PAIR16 ||
         v == OCT_B200_SGEMM_TC_PAIR32 || v == OCT_B200_SGEMM_TC_INSM16 || v == OCT_B200_SGEMM_TC_INSM32;
}

// The kernel a variant id runs for (m, n, k): AUTO picks the small-M kernel for
// m <= 16 (the product reads B once from HBM and has almost no arithmetic per
// byte), the FMA control for other tiny products (they do not fill one 128x256
// tensor-core tile usefully), the CTA-pair kernel with 32-deep stages for
// products of at least 2048 x 2048 (in a sustained loop at the 1 kW power cap
// it finishes an 8192^3 step ~10 % sooner than the single-CTA kernel), else the
// single-CTA 3xTF32 kernel.  Every tensor-core variant issues the same MMAs in
// the same order, so the choice changes no bits of C.
uint32_t resolve_variant(uint32_t variant, uint32_t m, uint32_t n, uint32_t k) {
  if (variant != OCT_B200_SGEMM_AUTO) return variant;
  if (oct::sgemm_smallm_supported(m)) return OCT_B200_SGEMM_SMALLM;
  const double work = static_cast<double>(m) * n * k;
  if (work < 4.0e6) return OCT_B200_SGEMM_FMA;
  return (m >= 2048 && n >= 2048) ? OCT_B200_SGEMM_TC_PAIR32 : OCT_B200_SGEMM_TC3XTF32;
}

}  // namespace

// `scratch` (default: the handle's) holds the TF32 split operands; calls that
// run concurrently on different streams need different scratch buffers.
int oct::rt::enqueue_sgemm(Runtime* rt, const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c,
                           uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, uint32_t variant, cudaStream_t stream,
                           const oct::GemmBatch* batch, DevBuf* scratch) {
  variant = resolve_variant(variant, m, n, k);
  if (scratch == nullptr) scratch = &rt->scratch;
  // the small-M kernels have no batched or B^T form: those take the FMA control
  if ((variant == OCT_B200_SGEMM_SMALLM || variant == OCT_B200_SGEMM_SMALLM_TC) && batch != nullptr &&
      (batch->count > 1 || batch->b_trans))
    variant = OCT_B200_SGEMM_FMA;
  cudaError_t e;
  if (variant == OCT_B200_SGEMM_SMALLM_TC) {
    if (!oct::sgemm_smallm_supported(m)) return OCT_B200_DETAIL_UNSUPPORTED_SHAPE;
    if (oct::sgemm_smallm_tc_eligible(a, lda, b, ldb, m, n, k)) {
      const uint64_t need = oct::sgemm_smallm_tc_scratch_bytes(m, n, k);
      if (need != 0 && scratch->ensure(need, stream) != cudaSuccess) return OCT_B200_DETAIL_OUT_OF_MEMORY;
      e = oct::sgemm_smallm_tc(a, lda, b, ldb, c, ldc, m, n, k, need != 0 ? scratch->aligned() : nullptr,
                               rt->err_word(), stream);
      return e == cudaSuccess ? 0 : OCT_B200_DETAIL_CUDA_ERROR;
    }
    variant = OCT_B200_SGEMM_SMALLM;  // operands TMA cannot read in place
  }
  if (variant == OCT_B200_SGEMM_SMALLM) {
    if (!oct::sgemm_smallm_supported(m)) return OCT_B200_DETAIL_UNSUPPORTED_SHAPE;
    const uint64_t need = oct::sgemm_smallm_scratch_bytes(m, n, k);
    if (need != 0 && scratch->ensure(need, stream) != cudaSuccess) return OCT_B200_DETAIL_OUT_OF_MEMORY;
    e = oct::sgemm_smallm(a, lda, b, ldb, c, ldc, m, n, k, need != 0 ? scratch->aligned() : nullptr, stream,
                          rt->err_word());
  } else if (variant == OCT_B200_SGEMM_FMA) {
    e = oct::sgemm_fma(a, lda, b, ldb, c, ldc, m, n, k, stream, batch);
  } else if (variant == OCT_B200_SGEMM_TC3XTF32 || variant == OCT_B200_SGEMM_TC_BK16 ||
             variant == OCT_B200_SGEMM_TC_BK32 || variant == OCT_B200_SGEMM_TC_PAIR16 ||
             variant == OCT_B200_SGEMM_TC_PAIR32 || variant == OCT_B200_SGEMM_TC_INSM16 ||
             variant == OCT_B200_SGEMM_TC_INSM32) {
    const int bk = variant == OCT_B200_SGEMM_TC3XTF32 ? oct::kTcSingle16 : static_cast<int>(variant);
    const bool insm = (bk == oct::kTcInsm16 || bk == oct::kTcInsm32) &&
                      oct::sgemm_insm_eligible(a, lda, b, ldb, m, n, k, batch);
    if (!insm) {  // the in-SM split kernel needs no split scratch
      const uint64_t need = oct::sgemm_tc_scratch_bytes(m, n, k, batch != nullptr ? batch->count : 1u);
      e = scratch->ensure(need, stream);
      if (e != cudaSuccess) return OCT_B200_DETAIL_OUT_OF_MEMORY;
    }
    const oct::SgemmEvents* ev = nullptr;
    if (rt->timing && (ev = next_timing_events(rt)) == nullptr) return OCT_B200_DETAIL_CUDA_ERROR;
    e = oct::sgemm_tc(a, lda, b, ldb, c, ldc, m, n, k, insm ? nullptr : scratch->aligned(), rt->err_word(), bk,
                      stream, ev, batch);
  } else {
    return OCT_B200_DETAIL_BAD_VARIANT;
  }
  return e == cudaSuccess ? 0 : OCT_B200_DETAIL_CUDA_ERROR;
}

namespace {

Runtime* create_runtime(const PrometheusReactorConfig* cfg, int* status) {
  Runtime* rt = new (std::nothrow) Runtime();
  if (rt == nullptr) {
    *status = PROM_INTERNAL_ERROR;
    return nullptr;
  }
  if (cfg != nullptr) {
    const uint32_t sz = cfg->struct_size;
    if (sz >= offsetof(PrometheusReactorConfig, test_flags) + sizeof(uint32_t)) rt->test_flags = cfg->test_flags;
    if (sz >= offsetof(PrometheusReactorConfig, async_test_flags) + sizeof(uint32_t))
      rt->async_test_flags = cfg->async_test_flags;
    if (sz >= offsetof(PrometheusReactorConfig, reduction_test_flags) + sizeof(uint32_t))
      rt->reduction_test_flags = cfg->reduction_test_flags;
    if (sz >= offsetof(PrometheusReactorConfig, reduction_ring_depth) + sizeof(uint32_t))
      rt->red_stats.ring_depth = cfg->reduction_ring_depth;
  }
  if (rt->test_flags & PROM_TESTCFG_FAIL_DEVICE_CREATE) {
    // Injected on the host: the handle exists but reports no device.
    rt->reason = PROM_REASON_VULKAN_UNAVAILABLE;
    *status = PROM_OK;
    return rt;
  }
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    (void)cudaGetLastError();
    rt->reason = PROM_REASON_VULKAN_UNAVAILABLE;
    *status = PROM_OK;
    return rt;
  }
  cudaGetDevice(&rt->device);
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, rt->device) != cudaSuccess || prop.major != 10) {
    rt->reason = PROM_REASON_VULKAN_UNAVAILABLE;
    *status = PROM_OK;
    return rt;
  }
  if (cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&rt->ev0) != cudaSuccess || cudaEventCreate(&rt->ev1) != cudaSuccess ||
      rt->words.ensure(16, rt->stream) != cudaSuccess || reset_words(rt) != cudaSuccess ||
      cudaStreamSynchronize(rt->stream) != cudaSuccess) {
    rt->reason = PROM_REASON_VULKAN_UNAVAILABLE;
    *status = PROM_OK;
    return rt;
  }
  rt->available = true;
  *status = PROM_OK;
  return rt;
}

void destroy_runtime(Runtime* rt) {
  if (rt->stream != nullptr) cudaStreamSynchronize(rt->stream);
  for (auto& kv : rt->blocks) delete kv.second;
  rt->blocks.clear();
  for (auto& kv : rt->tp_sgemms) delete kv.second;
  rt->tp_sgemms.clear();
  destroy_model_block(rt);
  for (auto& ev : rt->timing_events) {
    cudaEventSynchronize(ev.main_end);
    cudaEventDestroy(ev.split_begin);
    cudaEventDestroy(ev.main_begin);
    cudaEventDestroy(ev.main_end);
  }
  for (auto& t : rt->tasks) {
    if (t.begin != nullptr) cudaEventDestroy(t.begin);
    if (t.done != nullptr) cudaEventDestroy(t.done);
    t.a.release();
    t.b.release();
    t.c.release();
  }
  for (DevBuf* b : {&rt->scratch, &rt->da, &rt->db, &rt->dc, &rt->rin, &rt->rout, &rt->rw, &rt->rinv, &rt->words,
                    &rt->batch_c, &rt->m1_cos, &rt->m1_sin, &rt->m1_q, &rt->m1_k, &rt->m1_scores, &rt->fft_in,
                    &rt->fft_out, &rt->fft_tw})
    b->release();
  for (cudaStream_t* st : {&rt->copy_in, &rt->copy_out})
    if (*st != nullptr) {
      cudaStreamSynchronize(*st);
      cudaStreamDestroy(*st);
      *st = nullptr;
    }
  for (cudaEvent_t ev : rt->pipe_events) cudaEventDestroy(ev);
  rt->pipe_events.clear();
  for (uint32_t w = 0; w < kBatchWorkers; ++w) {
    if (rt->batch_streams[w] != nullptr) {
      cudaStreamSynchronize(rt->batch_streams[w]);
      cudaStreamDestroy(rt->batch_streams[w]);
    }
    rt->batch_scratch[w].release();
    rt->batch_a[w].release();
    rt->batch_b[w].release();
  }
  if (rt->ev0 != nullptr) cudaEventDestroy(rt->ev0);
  if (rt->ev1 != nullptr) cudaEventDestroy(rt->ev1);
  if (rt->stream != nullptr) cudaStreamDestroy(rt->stream);
  rt->magic = 0;
  delete rt;
}

// ---------------------------------------------------------------- reductions
struct ReductionShape {
  uint32_t rows, width, operation, finalization, flags;
  uint64_t input_count, output_count;
};

// Admission rules of reactors/PrometheusReduction.concept:66-88 with the row
// and total ceilings widened (the detail codes are unchanged).
int validate_shape(const ReductionShape& s) {
  if (s.rows == 0) return PROM_REDUCTION_DETAIL_ZERO_ROW_COUNT;
  if (s.width == 0) return PROM_REDUCTION_DETAIL_ZERO_ROW_WIDTH;
  if (s.rows > OCT_B200_REDUCTION_MAX_ROWS) return PROM_REDUCTION_DETAIL_ROW_LIMIT;
  if (s.width > PROM_REDUCTION_MAX_ELEMENTS_PER_ROW) return PROM_REDUCTION_DETAIL_WIDTH_LIMIT;
  const uint64_t total = static_cast<uint64_t>(s.rows) * s.width;
  if (total > OCT_B200_REDUCTION_MAX_TOTAL_ELEMENTS) return PROM_REDUCTION_DETAIL_ELEMENT_LIMIT;
  if (s.operation != PROM_REDUCTION_OPERATION_SUM && s.operation != PROM_REDUCTION_OPERATION_MAX &&
      s.operation != PROM_REDUCTION_OPERATION_SOFTMAX)
    return PROM_REDUCTION_DETAIL_UNSUPPORTED_OPERATION;
  uint64_t output = s.rows;
  if (s.operation == PROM_REDUCTION_OPERATION_SOFTMAX) {
    if (s.finalization != PROM_REDUCTION_FINALIZATION_STABLE_SOFTMAX) return PROM_REDUCTION_DETAIL_INVALID_FINALIZATION;
    output = total;
  } else if (s.finalization != PROM_REDUCTION_FINALIZATION_NONE) {
    return PROM_REDUCTION_DETAIL_INVALID_FINALIZATION;
  }
  if (s.flags > 2u || (s.operation != PROM_REDUCTION_OPERATION_SOFTMAX && s.flags != 0u))
    return PROM_REDUCTION_DETAIL_UNSUPPORTED_STRATEGY;
  if (s.flags == PROM_REDUCTION_FLAG_FORCE_FUSED && s.width > PROM_REDUCTION_FORCE_FUSED_MAX_ELEMENTS_PER_ROW)
    return PROM_REDUCTION_DETAIL_UNSUPPORTED_STRATEGY;
  if (s.input_count != total) return PROM_REDUCTION_DETAIL_INPUT_SIZE_MISMATCH;
  if (s.output_count != output) return PROM_REDUCTION_DETAIL_OUTPUT_SIZE_MISMATCH;
  return 0;
}

ReductionShape shape_of(const PrometheusReductionRequest* r) {
  return ReductionShape{r->row_count, r->elements_per_row, r->operation, r->finalization, r->flags,
                        r->input_element_count, r->output_element_count};
}

uint64_t fnv_u32(uint64_t h, uint32_t v) {
  for (uint32_t i = 0; i < 4; ++i) {
    h ^= static_cast<uint64_t>((v >> (i * 8u)) & 0xFFu);
    h *= 1099511628211ull;
  }
  return h;
}

// The logical schedule Oct's planner emits (reactors/PrometheusReduction.concept:
// 96-164, serialised as reactor_vulkan_fused_reduction.c:101-148).  The CUDA
// path executes every schedule as ONE fused kernel with a single HBM pass; the
// plan is still reported so plan-level callers and replay ids stay compatible.
void build_plan(const ReductionShape& s, PrometheusReductionPlan* p) {
  static const uint32_t shader_of[8] = {0,
                                        PROM_REDUCTION_SHADER_ROW_SUM,
                                        PROM_REDUCTION_SHADER_ROW_MAX,
                                        PROM_REDUCTION_SHADER_SOFTMAX_EXP_SUM,
                                        PROM_REDUCTION_SHADER_SOFTMAX_NORMALIZE,
                                        PROM_REDUCTION_SHADER_SOFTMAX_FUSED,
                                        PROM_REDUCTION_SHADER_ROW_SUM_PACKED_SHORT,
                                        PROM_REDUCTION_SHADER_SOFTMAX_PACKED_SHORT};
  std::memset(p, 0, sizeof(*p));
  p->struct_size = sizeof(*p);
  p->operation = s.operation;
  p->row_count = s.rows;
  p->elements_per_row = s.width;
  p->local_size = PROM_REDUCTION_LOCAL_SIZE;
  p->elements_per_partial = PROM_REDUCTION_ELEMENTS_PER_PARTIAL;
  p->temporary_alignment_bytes = sizeof(float);
  const uint32_t partials = (s.width + PROM_REDUCTION_ELEMENTS_PER_PARTIAL - 1) / PROM_REDUCTION_ELEMENTS_PER_PARTIAL;
  p->partial_count = partials;
  p->strategy = PROM_REDUCTION_STRATEGY_COMPOSED;
  const uint64_t row_bytes = static_cast<uint64_t>(s.rows) * 4u;
  const uint64_t partial_bytes = partials > 1 ? row_bytes * partials : 0;

  auto append = [&](uint32_t role, uint64_t groups, uint32_t width, uint32_t out_partials, uint32_t temp_role,
                    uint64_t temp_bytes) {
    PrometheusReductionStageDispatch& st = p->stages[p->stage_count++];
    st.stage_role = role;
    st.shader_id = shader_of[role];
    st.implementation_id = 1000u + role;
    st.groups_x = static_cast<uint32_t>(std::min<uint64_t>(groups, UINT32_MAX));
    st.groups_y = 1;
    st.groups_z = 1;
    st.input_elements_per_row = width;
    st.output_partials_per_row = out_partials;
    st.temporary_role = temp_role;
    st.temporary_bytes_written = temp_bytes;
  };
  // A row reduction is one partial pass plus, with >1 partial, a finishing pass.
  auto reduce = [&](uint32_t partial_role, uint32_t final_role, uint32_t destination, uint64_t dest_bytes) {
    uint32_t first_dest = destination;
    uint64_t first_bytes = dest_bytes;
    if (partials > 1) {
      first_dest = PROM_REDUCTION_TEMPORARY_PARTIALS;
      first_bytes = row_bytes * partials;
    }
    append(partial_role, static_cast<uint64_t>(s.rows) * partials, s.width, partials, first_dest, first_bytes);
    if (partials > 1) append(final_role, s.rows, partials, 1, destination, dest_bytes);
  };

  bool packed;
  if (s.operation == PROM_REDUCTION_OPERATION_SOFTMAX)
    packed = s.flags == 0 && s.width <= PROM_REDUCTION_PACKED_SHORT_WIDTH_MAX;
  else if (s.operation != PROM_REDUCTION_OPERATION_SUM)
    packed = false;
  else
    packed = (s.width <= 96u && s.rows >= PROM_REDUCTION_PACKED_SHORT_SUM_MIN_ROWS) ||
             (s.width <= PROM_REDUCTION_PACKED_SHORT_WIDTH_MAX && s.rows >= PROM_REDUCTION_PACKED_SHORT_SUM_WIDE_MIN_ROWS);

  if (packed) {
    p->strategy = PROM_REDUCTION_STRATEGY_PACKED_SHORT_ROWS;
    append(s.operation == PROM_REDUCTION_OPERATION_SOFTMAX ? 7u : 6u,
           (s.rows + PROM_REDUCTION_PACKED_SHORT_ROWS_PER_GROUP - 1) / PROM_REDUCTION_PACKED_SHORT_ROWS_PER_GROUP,
           s.width, 1, 0, 0);
  } else if (s.operation != PROM_REDUCTION_OPERATION_SOFTMAX) {
    reduce(s.operation, s.operation, PROM_REDUCTION_TEMPORARY_NONE, 0);
    p->temporary_bytes = partial_bytes;
  } else if (s.flags != PROM_REDUCTION_FLAG_FORCE_COMPOSED &&
             (s.flags == PROM_REDUCTION_FLAG_FORCE_FUSED || s.width <= PROM_REDUCTION_ELEMENTS_PER_PARTIAL)) {
    p->strategy = PROM_REDUCTION_STRATEGY_FUSED_SINGLE_WORKGROUP;
    append(5u, s.rows, s.width, 1, 0, 0);
  } else {
    reduce(2u, 2u, PROM_REDUCTION_TEMPORARY_ROW_MAX, row_bytes);
    reduce(3u, 1u, PROM_REDUCTION_TEMPORARY_ROW_SUM, row_bytes);
    const uint64_t total = static_cast<uint64_t>(s.rows) * s.width;
    append(4u, (total + PROM_REDUCTION_LOCAL_SIZE - 1) / PROM_REDUCTION_LOCAL_SIZE, s.width, 1, 0, 0);
    p->temporary_bytes = partial_bytes + 2u * row_bytes;
  }

  uint64_t h = 1469598103934665603ull;
  h = fnv_u32(h, p->operation);
  h = fnv_u32(h, p->row_count);
  h = fnv_u32(h, p->elements_per_row);
  h = fnv_u32(h, p->strategy);
  h = fnv_u32(h, p->partial_count);
  h = fnv_u32(h, p->stage_count);
  for (uint32_t i = 0; i < p->stage_count; ++i) {
    const PrometheusReductionStageDispatch& st = p->stages[i];
    h = fnv_u32(h, st.stage_role);
    h = fnv_u32(h, st.shader_id);
    h = fnv_u32(h, st.implementation_id);
    h = fnv_u32(h, st.groups_x);
    h = fnv_u32(h, st.input_elements_per_row);
    h = fnv_u32(h, st.output_partials_per_row);
    h = fnv_u32(h, st.temporary_role);
    h = fnv_u32(h, static_cast<uint32_t>(st.temporary_bytes_written));
    h = fnv_u32(h, static_cast<uint32_t>(st.temporary_bytes_written >> 32u));
  }
  p->replay_id = h;
}

// Runs one reduction over host buffers; fills stage/detail/timing.
// Records one executed reduction request in the handle's counters.
void note_reduction(Runtime* rt, int rc, int32_t detail, uint32_t stage_count, uint64_t replay, uint64_t gpu_ns,
                    uint64_t e2e_ns) {
  ReductionStats& st = rt->red_stats;
  st.initialized = true;
  ++st.total;
  ++st.slot_generation;
  if (rc == PROM_OK) {
    ++st.success;
  } else {
    ++st.failures;
  }
  st.last_detail = detail;
  st.last_stage_count = stage_count;
  st.last_replay = replay;
  st.last_gpu_ns = gpu_ns;
  st.last_e2e_ns = e2e_ns;
}

int run_reduction_host(Runtime* rt, const float* in, float* out, uint32_t rows, uint32_t width, uint32_t op,
                       uint32_t* stage, int32_t* detail, uint64_t* gpu_ns, uint32_t* gpu_valid,
                       uint64_t* first_nonfinite) {
  const uint64_t total = static_cast<uint64_t>(rows) * width;
  const uint64_t out_count = (op == PROM_REDUCTION_OPERATION_SOFTMAX) ? total : rows;
  if (rt->reduction_test_flags & PROM_REDUCTION_TESTCFG_FAIL_COMMAND_RECORD) {
    *stage = PROM_STAGE_SUBMIT;
    *detail = PROM_REDUCTION_DETAIL_COMMAND_RECORD_FAILED;
    return PROM_ERROR;
  }
  ++rt->red_stats.command_records;
  {
    const bool grow_in = rt->rin.raw == nullptr || total * 4 > rt->rin.cap;
    const bool grow_out = rt->rout.raw == nullptr || out_count * 4 > rt->rout.cap;
    rt->red_stats.allocations += static_cast<uint64_t>(grow_in) + static_cast<uint64_t>(grow_out);
    rt->red_stats.reuses += static_cast<uint64_t>(!grow_in) + static_cast<uint64_t>(!grow_out);
  }
  if (rt->rin.ensure(total * 4, rt->stream) != cudaSuccess || rt->rout.ensure(out_count * 4, rt->stream) != cudaSuccess) {
    *stage = PROM_STAGE_INIT;
    *detail = PROM_REDUCTION_DETAIL_RESOURCE_CREATE_FAILED;
    return PROM_ERROR;
  }
  float* din = static_cast<float*>(rt->rin.aligned());
  float* dout = static_cast<float*>(rt->rout.aligned());
  cudaError_t e = reset_words(rt);
  if (e == cudaSuccess) e = cudaMemcpyAsync(din, in, total * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e != cudaSuccess) {
    *stage = PROM_STAGE_TRANSFER_IN;
    *detail = PROM_REDUCTION_DETAIL_QUEUE_SUBMIT_FAILED;
    return PROM_ERROR;
  }
  if (rt->reduction_test_flags & PROM_REDUCTION_TESTCFG_FAIL_QUEUE_SUBMIT) {
    cudaStreamSynchronize(rt->stream);
    *stage = PROM_STAGE_SUBMIT;
    *detail = PROM_REDUCTION_DETAIL_QUEUE_SUBMIT_FAILED;
    return PROM_ERROR;
  }
  cudaEventRecord(rt->ev0, rt->stream);
  e = oct::row_reduce(din, dout, rows, width, op, rt->nonfinite_word(), rt->err_word(), rt->stream);
  if (e == cudaSuccess) ++rt->red_stats.submits;
  cudaEventRecord(rt->ev1, rt->stream);
  Words w;
  if (e != cudaSuccess || read_words(rt, &w) != cudaSuccess ||
      (rt->reduction_test_flags & PROM_REDUCTION_TESTCFG_FAIL_COMPLETION_OBSERVATION) || w.err != 0) {
    (void)cudaGetLastError();
    *stage = PROM_STAGE_SUBMIT;
    *detail = PROM_REDUCTION_DETAIL_COMPLETION_UNCERTAIN;
    return PROM_ERROR;
  }
  if (w.nonfinite != ~0ull) {
    *first_nonfinite = w.nonfinite;
    *stage = PROM_STAGE_TRANSFER_IN;
    *detail = PROM_REDUCTION_DETAIL_NONFINITE_INPUT;
    return PROM_ERROR;  // output untouched: nothing was copied back
  }
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, rt->ev0, rt->ev1) == cudaSuccess) {
    *gpu_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
    *gpu_valid = 1;
  }
  e = cudaMemcpyAsync(out, dout, out_count * 4, cudaMemcpyDeviceToHost, rt->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
  if (e != cudaSuccess) {
    *stage = PROM_STAGE_TRANSFER_OUT;
    *detail = PROM_REDUCTION_DETAIL_READBACK_FAILED;
    return PROM_ERROR;
  }
  *stage = PROM_STAGE_NONE;
  *detail = 0;
  return PROM_OK;
}

bool finite_f(float v) { return std::isfinite(v); }

}  // namespace

namespace {
AsyncTask* find_task(Runtime* rt, int id) {
  for (auto& t : rt->tasks)
    if (t.active && t.id == id) return &t;
  return nullptr;
}
// Non-blocking completion check of a submitted task.
void poll_task(Runtime* rt, AsyncTask* t) {
  if (t->state != PROM_ASYNC_STATE_SUBMITTED) return;
  ++rt->async_stats.polls;
  if (rt->test_flags & PROM_TESTCFG_FAIL_ASYNC_POLL) {
    t->state = PROM_ASYNC_STATE_FAILED;
    t->final_detail = PROM_DETAIL_INJECTED_ASYNC_POLL_FAILURE;
    t->final_stage = PROM_STAGE_SUBMIT;
    ++rt->async_stats.failed;
    return;
  }
  const cudaError_t q = cudaEventQuery(t->done);
  if (q == cudaErrorNotReady) return;
  ++rt->async_stats.reaped;
  if (q != cudaSuccess) {
    (void)cudaGetLastError();
    t->state = PROM_ASYNC_STATE_FAILED;
    t->final_detail = PROM_DETAIL_ASYNC_FAILED;
    ++rt->async_stats.failed;
    return;
  }
  Words w;
  if (read_words(rt, &w) != cudaSuccess || w.err != 0) {
    t->state = PROM_ASYNC_STATE_FAILED;
    t->final_detail = OCT_B200_DETAIL_DEVICE_TIMEOUT;
    ++rt->async_stats.failed;
    return;
  }
  float ms = 0.f;
  if (t->begin != nullptr && cudaEventElapsedTime(&ms, t->begin, t->done) == cudaSuccess) {
    t->timed = true;
    t->gpu_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
  }
  t->state = PROM_ASYNC_STATE_READY;
  t->final_stage = PROM_STAGE_TRANSFER_OUT;
  ++rt->async_stats.ready;
}
uint32_t outstanding(Runtime* rt) {
  uint32_t c = 0;
  for (auto& t : rt->tasks)
    if (t.active && t.state != PROM_ASYNC_STATE_CONSUMED) ++c;
  return c;
}
}  // namespace


// =========================================================================== ABI
extern "C" {

uint32_t prometheus_reactor_abi_version(void) { return PROM_REACTOR_ABI_V1; }

int prometheus_reactor_runtime_create(void* config, void** out_handle) {
  try {
    if (out_handle == nullptr) return PROM_ERROR;
    *out_handle = nullptr;
    const PrometheusReactorConfig* cfg = static_cast<const PrometheusReactorConfig*>(config);
    if (cfg != nullptr && cfg->struct_size < offsetof(PrometheusReactorConfig, test_flags) + sizeof(uint32_t))
      return PROM_ERROR;
    int status = PROM_OK;
    Runtime* rt = create_runtime(cfg, &status);
    if (rt == nullptr) return status;
    {
      std::lock_guard<std::mutex> lock(g_registry_mu);
      g_registry->insert(rt);
    }
    *out_handle = rt;
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_destroy(void* handle) {
  try {
    Runtime* rt = nullptr;
    {
      std::lock_guard<std::mutex> lock(g_registry_mu);
      Runtime* cand = static_cast<Runtime*>(handle);
      if (handle == nullptr || g_registry->count(cand) == 0) return PROM_INVALID_HANDLE;
      g_registry->erase(cand);
      rt = cand;
    }
    {
      std::lock_guard<std::mutex> lock(rt->mu);  // callers must be quiescent; this only orders teardown
    }
    destroy_runtime(rt);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_probe(void* handle, PrometheusCaps* out_caps) {
  if (out_caps == nullptr) return PROM_ERROR;
  std::memset(out_caps, 0, sizeof(*out_caps));
  Runtime* rt = lookup(handle);
  if (rt == nullptr) return PROM_INVALID_HANDLE;
  out_caps->available = rt->available ? 1u : 0u;
  out_caps->backend_type = rt->available ? PROM_BACKEND_VULKAN : PROM_BACKEND_UNKNOWN;
  out_caps->reason_code = rt->available ? PROM_REASON_NONE : rt->reason;
  return PROM_OK;
}

int prometheus_runtime_create(void* config, void** out_handle) {
  return prometheus_reactor_runtime_create(config, out_handle);
}
int prometheus_runtime_destroy(void* handle) { return prometheus_reactor_runtime_destroy(handle); }
int prometheus_runtime_probe(void* handle, PrometheusCaps* out_caps) {
  return prometheus_reactor_runtime_probe(handle, out_caps);
}

// Validation order and codes follow reactor_sgemm.cpp:4149-4176.
namespace {
// Host-injected failure flags that the one-shot path reports stage by stage.
constexpr uint32_t kTestFlagsWithHostInjection =
    PROM_TESTCFG_FAIL_BUFFER_ALLOC | PROM_TESTCFG_FAIL_UPLOAD | PROM_TESTCFG_FAIL_DISPATCH | PROM_TESTCFG_FAIL_DOWNLOAD;

// Large host-buffer products: transfers and tensor work overlap inside the one
// call.  B goes up first and is split once; A goes up in row chunks on a copy
// stream, each chunk's product starts as soon as its rows landed, and each C
// chunk goes down on a second copy stream as soon as it is computed.  Every C
// element is computed exactly as in the one-shot path (same kernel, same K
// order), so the result is bit-identical.  With pinned caller buffers all
// three engines run concurrently; with pageable ones the host thread stages
// one copy at a time while the GPU keeps computing.
int sgemm_host_pipelined(Runtime* rt, const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                         float* da, float* db, float* dc, int cfg, uint32_t* out_stage, int* out_detail_code) {
  cudaStream_t cs = rt->stream;
  if (rt->copy_in == nullptr && cudaStreamCreateWithFlags(&rt->copy_in, cudaStreamNonBlocking) != cudaSuccess) {
    rt->copy_in = nullptr;
    set_status(out_stage, out_detail_code, PROM_STAGE_INIT, OCT_B200_DETAIL_CUDA_ERROR);
    return PROM_ERROR;
  }
  if (rt->copy_out == nullptr && cudaStreamCreateWithFlags(&rt->copy_out, cudaStreamNonBlocking) != cudaSuccess) {
    rt->copy_out = nullptr;
    set_status(out_stage, out_detail_code, PROM_STAGE_INIT, OCT_B200_DETAIL_CUDA_ERROR);
    return PROM_ERROR;
  }
  // ~16 row chunks of at least 256 rows (the tile-pair height): the last chunk's
  // product and download are the part of the step that no upload hides
  const uint32_t rows = std::max<uint32_t>(256u, ((m + 15u) / 16u + 255u) / 256u * 256u);
  const uint32_t nchunks = (m + rows - 1) / rows;
  const uint32_t nev = 2 * nchunks + 1;
  while (rt->pipe_events.size() < nev) {
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, OCT_B200_DETAIL_CUDA_ERROR);
      return PROM_ERROR;
    }
    rt->pipe_events.push_back(ev);
  }
  const uint64_t b_elems = oct::split_b_elems(n, k);
  const uint64_t b_bytes = (2 * b_elems * sizeof(float) + 1023) & ~uint64_t(1023);
  if (rt->scratch.ensure(b_bytes + oct::sgemm_tc_a_scratch_bytes(rows, k) + 1024, cs) != cudaSuccess) {
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_OUT_OF_MEMORY);
    return PROM_ERROR;
  }
  float* bhi = static_cast<float*>(rt->scratch.aligned());
  float* blo = bhi + b_elems;
  void* a_scratch = static_cast<char*>(rt->scratch.aligned()) + b_bytes;
  cudaEvent_t ev_b = rt->pipe_events[0];
  auto ev_a = [&](uint32_t i) { return rt->pipe_events[1 + i]; };
  auto ev_g = [&](uint32_t i) { return rt->pipe_events[1 + nchunks + i]; };
  const uint64_t b_n = static_cast<uint64_t>(k) * n;
  uint32_t fail_stage = PROM_STAGE_NONE;
  int fail_detail = 0;
  auto fail = [&](uint32_t stage, int detail) {
    if (fail_stage == PROM_STAGE_NONE) {
      fail_stage = stage;
      fail_detail = detail;
    }
  };
  cudaError_t e = reset_words(rt);
  if (e == cudaSuccess) e = cudaMemcpyAsync(db, b, b_n * 4, cudaMemcpyHostToDevice, rt->copy_in);
  if (e == cudaSuccess) e = cudaEventRecord(ev_b, rt->copy_in);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, ev_b, 0);
  if (e == cudaSuccess) e = oct::sgemm_tc_split_b(db, n, k, n, bhi, blo, cs);
  if (e != cudaSuccess) fail(PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_CUDA_ERROR);
  for (uint32_t i = 0; i < nchunks && fail_stage == PROM_STAGE_NONE; ++i) {
    const uint32_t r0 = i * rows, rc = std::min(rows, m - r0);
    const uint64_t a_off = static_cast<uint64_t>(r0) * k, c_off = static_cast<uint64_t>(r0) * n;
    e = cudaMemcpyAsync(da + a_off, a + a_off, static_cast<uint64_t>(rc) * k * 4, cudaMemcpyHostToDevice,
                        rt->copy_in);
    if (e == cudaSuccess) e = cudaEventRecord(ev_a(i), rt->copy_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, ev_a(i), 0);
    if (e != cudaSuccess) {
      fail(PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_CUDA_ERROR);
      break;
    }
    e = oct::sgemm_tc_presplit(da + a_off, k, bhi, blo, dc + c_off, n, rc, n, k, a_scratch, rt->err_word(), cs,
                               nullptr, 0, cfg);
    if (e == cudaSuccess) e = cudaEventRecord(ev_g(i), cs);
    if (e != cudaSuccess) {
      fail(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
      break;
    }
    if (i >= 1) {  // the previous chunk's result goes down while this one computes
      const uint32_t p0 = (i - 1) * rows, pc = std::min(rows, m - p0);
      const uint64_t p_off = static_cast<uint64_t>(p0) * n;
      e = cudaStreamWaitEvent(rt->copy_out, ev_g(i - 1), 0);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(c + p_off, dc + p_off, static_cast<uint64_t>(pc) * n * 4, cudaMemcpyDeviceToHost,
                            rt->copy_out);
      if (e != cudaSuccess) fail(PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
    }
  }
  if (fail_stage == PROM_STAGE_NONE) {
    const uint32_t p0 = (nchunks - 1) * rows, pc = m - p0;
    const uint64_t p_off = static_cast<uint64_t>(p0) * n;
    e = cudaStreamWaitEvent(rt->copy_out, ev_g(nchunks - 1), 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(c + p_off, dc + p_off, static_cast<uint64_t>(pc) * n * 4, cudaMemcpyDeviceToHost,
                          rt->copy_out);
    if (e != cudaSuccess) fail(PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
  }
  // drain every stream, failed or not
  const cudaError_t s_in = cudaStreamSynchronize(rt->copy_in);
  const cudaError_t s_cs = cudaStreamSynchronize(cs);
  const cudaError_t s_out = cudaStreamSynchronize(rt->copy_out);
  if (s_in != cudaSuccess) fail(PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_CUDA_ERROR);
  if (s_cs != cudaSuccess) fail(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
  if (s_out != cudaSuccess) fail(PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
  Words w;
  if (fail_stage == PROM_STAGE_NONE && (read_words(rt, &w) != cudaSuccess || w.err != 0))
    fail(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_DEVICE_TIMEOUT);
  if (fail_stage != PROM_STAGE_NONE) {
    set_status(out_stage, out_detail_code, fail_stage, fail_detail);
    return PROM_ERROR;
  }
  set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, PROM_DETAIL_PATH_DIRECT);
  return PROM_OK;
}

// The host-buffer SGEMM behind prometheus_reactor_runtime_sgemm and
// ..._sgemm_benchmark_variant (`requested` = an OCT_B200_SGEMM_* id).
int sgemm_host(void* handle, const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
               uint32_t requested, uint32_t* out_stage, int* out_detail_code) {
  try {
    set_status(out_stage, out_detail_code, PROM_STAGE_NONE, 0);
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_INVALID_HANDLE);
      return PROM_INVALID_HANDLE;
    }
    if (a == nullptr || b == nullptr || c == nullptr) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, PROM_ERROR);
      return PROM_ERROR;
    }
    if (m == 0 || n == 0 || k == 0) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_ERROR);
      return PROM_ERROR;
    }
    if (!known_variant(requested)) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, OCT_B200_DETAIL_BAD_VARIANT);
      return PROM_ERROR;
    }
    if (!rt->available) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_DETAIL_CAPABILITY_MISMATCH);
      return PROM_ERROR;
    }
    uint64_t a_n, b_n, c_n;
    if (!checked_mul(m, k, &a_n) || !checked_mul(k, n, &b_n) || !checked_mul(m, n, &c_n) ||
        a_n > (UINT64_MAX / 8) || b_n > (UINT64_MAX / 8) || c_n > (UINT64_MAX / 8)) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, PROM_DETAIL_SIZE_OVERFLOW);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, 0);
    if ((rt->test_flags & PROM_TESTCFG_FAIL_BUFFER_ALLOC) || rt->da.ensure(a_n * 4, rt->stream) != cudaSuccess ||
        rt->db.ensure(b_n * 4, rt->stream) != cudaSuccess || rt->dc.ensure(c_n * 4, rt->stream) != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_OUT_OF_MEMORY);
      return PROM_ERROR;
    }
    if (rt->test_flags & PROM_TESTCFG_FAIL_UPLOAD) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, PROM_DETAIL_INJECTED_UPLOAD_FAILURE);
      return PROM_ERROR;
    }
    float* da = static_cast<float*>(rt->da.aligned());
    float* db = static_cast<float*>(rt->db.aligned());
    float* dc = static_cast<float*>(rt->dc.aligned());
    const uint32_t variant = (rt->test_flags & PROM_TESTCFG_FORCE_STRICT_FP32) ? OCT_B200_SGEMM_FMA : requested;
    const uint32_t exec = resolve_variant(variant, m, n, k);
    if ((exec == OCT_B200_SGEMM_TC3XTF32 || exec == OCT_B200_SGEMM_TC_BK16 || exec == OCT_B200_SGEMM_TC_PAIR32) &&
        m >= 1024 && static_cast<double>(m) * n * k >= 1.0e9 && (rt->test_flags & kTestFlagsWithHostInjection) == 0) {
      const int cfg = exec == OCT_B200_SGEMM_TC_PAIR32 ? oct::kTcPair32 : oct::kTcSingle16;
      const int pd = sgemm_host_pipelined(rt, a, b, c, m, n, k, da, db, dc, cfg, out_stage, out_detail_code);
      return pd;
    }
    cudaError_t e = reset_words(rt);
    if (e == cudaSuccess) e = cudaMemcpyAsync(da, a, a_n * 4, cudaMemcpyHostToDevice, rt->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(db, b, b_n * 4, cudaMemcpyHostToDevice, rt->stream);
    if (e != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_CUDA_ERROR);
      return PROM_ERROR;
    }
    if (rt->test_flags & PROM_TESTCFG_FAIL_DISPATCH) {
      cudaStreamSynchronize(rt->stream);
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_DETAIL_INJECTED_DISPATCH_FAILURE);
      return PROM_ERROR;
    }
    const int d = enqueue_sgemm(rt, da, k, db, n, dc, n, m, n, k, variant, rt->stream);
    if (d != 0) {
      cudaStreamSynchronize(rt->stream);
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, d);
      return PROM_ERROR;
    }
    if (rt->test_flags & PROM_TESTCFG_FAIL_DOWNLOAD) {
      cudaStreamSynchronize(rt->stream);
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, PROM_DETAIL_INJECTED_DOWNLOAD_FAILURE);
      return PROM_ERROR;
    }
    Words w;
    if (read_words(rt, &w) != cudaSuccess) {
      (void)cudaGetLastError();
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
      return PROM_ERROR;
    }
    if (w.err != 0) {
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, OCT_B200_DETAIL_DEVICE_TIMEOUT);
      return PROM_ERROR;
    }
    e = cudaMemcpyAsync(c, dc, c_n * 4, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
      return PROM_ERROR;
    }
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, PROM_DETAIL_PATH_DIRECT);
    return PROM_OK;
  } catch (...) {
    set_status(out_stage, out_detail_code, PROM_STAGE_INIT, OCT_B200_DETAIL_CUDA_ERROR);
    return PROM_INTERNAL_ERROR;
  }
}
}  // namespace

int prometheus_reactor_runtime_sgemm(void* handle, const float* a, const float* b, float* c, uint32_t m, uint32_t n,
                                     uint32_t k, uint32_t* out_stage, int* out_detail_code) {
  return sgemm_host(handle, a, b, c, m, n, k, OCT_B200_SGEMM_AUTO, out_stage, out_detail_code);
}

int prometheus_reactor_runtime_sgemm_benchmark_variant(void* handle, const float* a, const float* b, float* c,
                                                       uint32_t m, uint32_t n, uint32_t k, uint32_t requested_variant,
                                                       uint32_t* out_stage, int* out_detail_code) {
  return sgemm_host(handle, a, b, c, m, n, k, requested_variant, out_stage, out_detail_code);
}

namespace {
uint64_t wall_ns() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}

// Nearest-rank percentile with the index rounded up (reactor_sgemm.cpp:5357-5367).
uint64_t percentile_ns(std::vector<uint64_t> v, uint32_t num, uint32_t den) {
  if (v.empty() || den == 0) return 0;
  std::sort(v.begin(), v.end());
  const uint64_t scaled = (static_cast<uint64_t>(v.size() - 1) * num + (den - 1)) / den;
  return v[std::min<uint64_t>(scaled, v.size() - 1)];
}

// CUDA events bracketing one resident product (or one group of them).
struct EventPair {
  cudaEvent_t begin = nullptr, end = nullptr;
  bool make() { return cudaEventCreate(&begin) == cudaSuccess && cudaEventCreate(&end) == cudaSuccess; }
  void destroy() {
    if (begin != nullptr) cudaEventDestroy(begin);
    if (end != nullptr) cudaEventDestroy(end);
    begin = end = nullptr;
  }
  uint64_t elapsed_ns() const {
    float ms = 0.f;
    return cudaEventElapsedTime(&ms, begin, end) == cudaSuccess ? static_cast<uint64_t>(ms * 1.0e6) : 0;
  }
};
}  // namespace

// Resident benchmark (reactor_sgemm.cpp:5629-5978): validation order and result
// fields follow the reference; the reference's Vulkan command-buffer counters
// count CUDA enqueues and stream waits here.
int prometheus_reactor_runtime_sgemm_resident_benchmark(void* handle,
                                                        const PrometheusSgemmResidentBenchmarkRequest* request,
                                                        PrometheusSgemmResidentBenchmarkResult* out) {
  if (out == nullptr) return PROM_ERROR;
  std::memset(out, 0, sizeof(*out));
  out->struct_size = static_cast<uint32_t>(sizeof(*out));
  std::vector<EventPair> evs;
  auto cleanup = [&]() {
    for (auto& e : evs) e.destroy();
  };
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      out->setup_stage = PROM_STAGE_INIT;
      out->setup_detail_code = PROM_INVALID_HANDLE;
      return PROM_INVALID_HANDLE;
    }
    out->resident_mode_available = rt->available ? 1u : 0u;
    const PrometheusSgemmResidentBenchmarkRequest* r = request;
    if (r == nullptr || r->a == nullptr || r->b == nullptr || r->m == 0 || r->n == 0 || r->k == 0 ||
        ((r->flags & PROM_SGEMM_RESIDENT_FLAG_VALIDATE_READBACK) != 0 && r->c == nullptr)) {
      out->setup_stage = PROM_STAGE_TRANSFER_IN;
      out->setup_detail_code = PROM_ERROR;
      return PROM_ERROR;
    }
    if (!rt->available) {
      out->setup_stage = PROM_STAGE_INIT;
      out->setup_detail_code = PROM_DETAIL_CAPABILITY_MISMATCH;
      return PROM_ERROR;
    }
    const uint32_t m = r->m, n = r->n, k = r->k;
    uint64_t a_n, b_n, c_n;
    if (!checked_mul(m, k, &a_n) || !checked_mul(k, n, &b_n) || !checked_mul(m, n, &c_n) ||
        a_n > (UINT64_MAX / 8) || b_n > (UINT64_MAX / 8) || c_n > (UINT64_MAX / 8)) {
      out->setup_stage = PROM_STAGE_TRANSFER_IN;
      out->setup_detail_code = PROM_DETAIL_SIZE_OVERFLOW;
      return PROM_ERROR;
    }
    const bool explicit_variant = r->mode == PROM_SGEMM_RESIDENT_MODE_EXPLICIT_VARIANT;
    const uint32_t requested = explicit_variant ? r->requested_variant : OCT_B200_SGEMM_AUTO;
    if (!known_variant(requested)) {
      out->setup_stage = PROM_STAGE_INIT;
      out->setup_detail_code = OCT_B200_DETAIL_BAD_VARIANT;
      return PROM_ERROR;
    }
    const uint32_t iterations = r->iterations == 0 ? 1u : r->iterations;
    const uint32_t warmup = r->warmup_iterations;
    const uint32_t depth = r->diagnostic_batch_depth == 0 ? 1u : r->diagnostic_batch_depth;
    std::lock_guard<std::mutex> lock(rt->mu);
    cudaStream_t st = rt->stream;

    // ---- setup: upload once, one product
    const uint64_t t_setup0 = wall_ns();
    if (rt->da.ensure(a_n * 4, st) != cudaSuccess || rt->db.ensure(b_n * 4, st) != cudaSuccess ||
        rt->dc.ensure(c_n * 4, st) != cudaSuccess) {
      out->setup_stage = PROM_STAGE_TRANSFER_IN;
      out->setup_detail_code = OCT_B200_DETAIL_OUT_OF_MEMORY;
      return PROM_ERROR;
    }
    float* da = static_cast<float*>(rt->da.aligned());
    float* db = static_cast<float*>(rt->db.aligned());
    float* dc = static_cast<float*>(rt->dc.aligned());
    const uint64_t t_up0 = wall_ns();
    cudaError_t e = reset_words(rt);
    if (e == cudaSuccess) e = cudaMemcpyAsync(da, r->a, a_n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(db, r->b, b_n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    out->upload_once_wall_ns = wall_ns() - t_up0;
    if (e != cudaSuccess) {
      out->setup_stage = PROM_STAGE_TRANSFER_IN;
      out->setup_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    int d = enqueue_sgemm(rt, da, k, db, n, dc, n, m, n, k, requested, st);
    Words w;
    if (d == 0 && (read_words(rt, &w) != cudaSuccess || w.err != 0)) d = OCT_B200_DETAIL_DEVICE_TIMEOUT;
    out->setup_wall_ns = wall_ns() - t_setup0;
    if (d != 0) {
      out->setup_stage = PROM_STAGE_SUBMIT;
      out->setup_detail_code = d;
      return PROM_ERROR;
    }
    out->setup_stage = PROM_STAGE_TRANSFER_OUT;
    out->setup_detail_code = PROM_DETAIL_PATH_DIRECT;
    out->resident_mode_used = 1u;
    out->requested_variant = explicit_variant ? r->requested_variant : 0u;
    out->production_selected_variant = resolve_variant(OCT_B200_SGEMM_AUTO, m, n, k);
    out->executed_variant = resolve_variant(requested, m, n, k);
    out->executed_compute_mode =
        (out->executed_variant == OCT_B200_SGEMM_FMA || out->executed_variant == OCT_B200_SGEMM_SMALLM) ? 2u : 1u;

    auto fail_final = [&](uint32_t stage, int detail) {
      cudaStreamSynchronize(st);
      cleanup();
      out->final_stage = stage;
      out->final_detail_code = detail;
      return PROM_ERROR;
    };
    auto product = [&]() { return enqueue_sgemm(rt, da, k, db, n, dc, n, m, n, k, requested, st); };
    std::vector<uint64_t> kernel, submit, wait, query;

    if ((r->flags & PROM_SGEMM_RESIDENT_FLAG_M29_SUBMISSION_RING) != 0) {
      // ---- ring: up to `ring` products in flight, each bracketed by its own events
      const uint32_t ring = r->diagnostic_batch_depth == 0 ? 2u : r->diagnostic_batch_depth;
      if (ring < 1 || ring > 4) return fail_final(PROM_STAGE_SUBMIT, PROM_ERROR);
      evs.resize(ring);
      for (auto& ev : evs)
        if (!ev.make()) return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
      uint32_t slot_busy[4] = {0, 0, 0, 0};
      auto run_ring = [&](uint32_t count, bool record) -> int {
        uint32_t outstanding = 0, next_slot = 0;
        for (uint32_t i = 0; i < count; ++i) {
          const uint32_t sl = next_slot;
          next_slot = (next_slot + 1) % ring;
          if (slot_busy[sl]) {  // the ring is full: harvest the oldest slot first
            out->ring_full_count += 1;
            out->ring_poll_count += 1;
            if (cudaEventQuery(evs[sl].end) == cudaErrorNotReady) {
              out->ring_forced_wait_count += 1;
              if (cudaEventSynchronize(evs[sl].end) != cudaSuccess) return OCT_B200_DETAIL_CUDA_ERROR;
            }
            if (record) kernel.push_back(evs[sl].elapsed_ns());
            out->ring_query_harvest_count += 1;
            out->ring_slot_recycle_count += 1;
            slot_busy[sl] = 0;
            outstanding -= 1;
          }
          if (cudaEventRecord(evs[sl].begin, st) != cudaSuccess) return OCT_B200_DETAIL_CUDA_ERROR;
          const int pd = product();
          if (pd != 0) return pd;
          if (cudaEventRecord(evs[sl].end, st) != cudaSuccess) return OCT_B200_DETAIL_CUDA_ERROR;
          slot_busy[sl] = 1;
          outstanding += 1;
          out->max_in_flight_depth = std::max(out->max_in_flight_depth, outstanding);
        }
        for (uint32_t i = 0; i < ring; ++i) {  // drain in submission order
          const uint32_t sl = (next_slot + i) % ring;
          if (!slot_busy[sl]) continue;
          out->ring_poll_count += 1;
          if (cudaEventSynchronize(evs[sl].end) != cudaSuccess) return OCT_B200_DETAIL_CUDA_ERROR;
          if (record) kernel.push_back(evs[sl].elapsed_ns());
          out->ring_query_harvest_count += 1;
          slot_busy[sl] = 0;
        }
        return 0;
      };
      if (warmup != 0 && (d = run_ring(warmup, false)) != 0) return fail_final(PROM_STAGE_SUBMIT, d);
      const uint64_t t0 = wall_ns();
      d = run_ring(iterations, true);
      const uint64_t t1 = wall_ns();
      if (d != 0) return fail_final(PROM_STAGE_SUBMIT, d);
      out->iterations = iterations;
      out->total_loop_wall_ns = t1 - t0;
      out->diagnostic_batch_depth = ring;
      out->queue_submissions = iterations;
      out->fence_waits = static_cast<uint32_t>(out->ring_forced_wait_count);
      out->command_buffer_recordings = iterations;
      out->command_buffer_resets = iterations;
      out->descriptor_updates = iterations;
      out->configured_ring_depth = ring;
      out->physical_slot_count = 4;
      for (uint32_t i = 0; i < 4; ++i) out->ring_final_slot_state[i] = slot_busy[i];
    } else {
      // ---- serial: each iteration enqueues `depth` products and waits once
      evs.resize(1);
      if (!evs[0].make()) return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
      for (uint32_t i = 0; i < warmup; ++i) {
        for (uint32_t j = 0; j < depth; ++j)
          if ((d = product()) != 0) return fail_final(PROM_STAGE_SUBMIT, d);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
      }
      const uint64_t t0 = wall_ns();
      for (uint32_t i = 0; i < iterations; ++i) {
        const uint64_t s0 = wall_ns();
        if (cudaEventRecord(evs[0].begin, st) != cudaSuccess)
          return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
        for (uint32_t j = 0; j < depth; ++j)
          if ((d = product()) != 0) return fail_final(PROM_STAGE_SUBMIT, d);
        if (cudaEventRecord(evs[0].end, st) != cudaSuccess)
          return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
        const uint64_t s1 = wall_ns();
        if (cudaEventSynchronize(evs[0].end) != cudaSuccess)
          return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_CUDA_ERROR);
        const uint64_t s2 = wall_ns();
        kernel.push_back(evs[0].elapsed_ns());
        const uint64_t s3 = wall_ns();
        submit.push_back(s1 - s0);
        wait.push_back(s2 - s1);
        query.push_back(s3 - s2);
      }
      const uint64_t t1 = wall_ns();
      out->iterations = iterations * depth;
      out->total_loop_wall_ns = t1 - t0;
      out->dispatch_submit_wall_ns_median = percentile_ns(submit, 50, 100);
      out->sync_wait_wall_ns_median = percentile_ns(wait, 50, 100);
      out->query_result_wall_ns_median = percentile_ns(query, 50, 100);
      out->diagnostic_batch_depth = depth;
      out->queue_submissions = iterations;
      out->fence_waits = iterations;
      out->command_buffer_recordings = iterations;
      out->command_buffer_resets = iterations;
      out->descriptor_updates = iterations;
    }
    if (read_words(rt, &w) != cudaSuccess || w.err != 0) return fail_final(PROM_STAGE_SUBMIT, OCT_B200_DETAIL_DEVICE_TIMEOUT);
    out->gpu_timestamp_valid = 1u;
    for (uint64_t x : kernel)
      if (x == 0) out->gpu_timestamp_valid = 0u;
    if (kernel.empty()) out->gpu_timestamp_valid = 0u;
    if (out->gpu_timestamp_valid) {
      out->kernel_min_ns = percentile_ns(kernel, 0, 100);
      out->kernel_median_ns = percentile_ns(kernel, 50, 100);
      out->kernel_p95_ns = percentile_ns(kernel, 95, 100);
      out->gpu_timing_failure_reason = PROM_SGEMM_GPU_TIMING_FAILURE_NONE;
    }
    if ((r->flags & PROM_SGEMM_RESIDENT_FLAG_VALIDATE_READBACK) != 0) {
      const uint64_t t0 = wall_ns();
      e = cudaMemcpyAsync(r->c, dc, c_n * 4, cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess) e = cudaStreamSynchronize(st);
      out->readback_once_wall_ns = wall_ns() - t0;
      out->validation_wall_ns = out->readback_once_wall_ns;
      if (e != cudaSuccess) return fail_final(PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
    }
    cleanup();
    out->final_stage = PROM_STAGE_SUBMIT;
    out->final_detail_code = PROM_DETAIL_PATH_STAGED_UPLOAD_TILED;
    return PROM_OK;
  } catch (...) {
    cleanup();
    out->final_stage = PROM_STAGE_CLEANUP;
    out->final_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
    return PROM_INTERNAL_ERROR;
  }
}

// Batch (reactor_sgemm.cpp:5984-6009; reactor_batch.c:89-180, 244-520): the
// flag mask, plan validation (u32 element counts, as the reference's plan) and
// ordered commit follow the reference; the execution is one CUDA stream per
// worker with its own staging and split scratch.
int prometheus_reactor_runtime_sgemm_batch(void* handle, const PrometheusSgemmBatchEntry* entries,
                                           uint32_t entry_count, uint32_t flags, uint32_t* out_stage,
                                           int* out_detail_code) {
  try {
    set_status(out_stage, out_detail_code, PROM_STAGE_NONE, 0);
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_INVALID_HANDLE);
      return PROM_INVALID_HANDLE;
    }
    if ((flags & ~(0xFFu | PROM_BATCH_FLAG_PARTITION_CONTIGUOUS)) != 0) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_DETAIL_BATCH_UNSUPPORTED_OPTION);
      return PROM_ERROR;
    }
    if (!rt->available) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_DETAIL_BATCH_EXECUTION_FAILED);
      return PROM_ERROR;
    }
    if (entries == nullptr || entry_count == 0) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_ERROR);
      return PROM_ERROR;
    }
    auto fits_u32 = [](uint32_t x, uint32_t y) { return static_cast<uint64_t>(x) * y <= 0xFFFFFFFFull; };
    for (uint32_t i = 0; i < entry_count; ++i) {
      const PrometheusSgemmBatchEntry& en = entries[i];
      if (en.a == nullptr || en.b == nullptr || en.c == nullptr || en.m == 0 || en.n == 0 || en.k == 0 ||
          !fits_u32(en.m, en.k) || !fits_u32(en.k, en.n) || !fits_u32(en.m, en.n)) {
        set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_DETAIL_BATCH_PLAN_INVALID);
        return PROM_ERROR;
      }
    }
    uint32_t workers = (flags & 0xFFu) == 0 ? 1u : (flags & 0xFFu);
    workers = std::min(workers, std::min(kBatchWorkers, entry_count));
    const bool contiguous = (flags & PROM_BATCH_FLAG_PARTITION_CONTIGUOUS) != 0;
    std::lock_guard<std::mutex> lock(rt->mu);
    // every entry's C stays on the device until all entries have succeeded
    std::vector<uint64_t> c_off(entry_count);
    uint64_t c_total = 0;
    for (uint32_t i = 0; i < entry_count; ++i) {
      c_off[i] = c_total;
      c_total += (static_cast<uint64_t>(entries[i].m) * entries[i].n * 4 + 255) & ~uint64_t(255);
    }
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, 0);
    if (rt->batch_c.ensure(c_total, rt->stream) != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_OUT_OF_MEMORY);
      return PROM_ERROR;
    }
    for (uint32_t w = 0; w < workers; ++w)
      if (rt->batch_streams[w] == nullptr &&
          cudaStreamCreateWithFlags(&rt->batch_streams[w], cudaStreamNonBlocking) != cudaSuccess) {
        rt->batch_streams[w] = nullptr;
        set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_DETAIL_BATCH_EXECUTION_FAILED);
        return PROM_ERROR;
      }
    if (reset_words(rt) != cudaSuccess || cudaStreamSynchronize(rt->stream) != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_DETAIL_BATCH_EXECUTION_FAILED);
      return PROM_ERROR;
    }
    char* cbase = static_cast<char*>(rt->batch_c.aligned());
    uint32_t fail_stage = PROM_STAGE_NONE;
    int fail_detail = 0;
    for (uint32_t i = 0; i < entry_count && fail_stage == PROM_STAGE_NONE; ++i) {
      const PrometheusSgemmBatchEntry& en = entries[i];
      const uint32_t w = contiguous ? static_cast<uint32_t>(static_cast<uint64_t>(i) * workers / entry_count)
                                    : i % workers;
      cudaStream_t s = rt->batch_streams[w];
      const uint64_t a_n = static_cast<uint64_t>(en.m) * en.k, b_n = static_cast<uint64_t>(en.k) * en.n;
      // a worker's staging is reused by its next entry only after this one's product (same stream)
      if (rt->batch_a[w].ensure(a_n * 4, s) != cudaSuccess || rt->batch_b[w].ensure(b_n * 4, s) != cudaSuccess) {
        fail_stage = PROM_STAGE_TRANSFER_IN;
        fail_detail = OCT_B200_DETAIL_OUT_OF_MEMORY;
        break;
      }
      float* da = static_cast<float*>(rt->batch_a[w].aligned());
      float* db = static_cast<float*>(rt->batch_b[w].aligned());
      float* dc = reinterpret_cast<float*>(cbase + c_off[i]);
      if (cudaMemcpyAsync(da, en.a, a_n * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
          cudaMemcpyAsync(db, en.b, b_n * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        fail_stage = PROM_STAGE_TRANSFER_IN;
        fail_detail = OCT_B200_DETAIL_CUDA_ERROR;
        break;
      }
      const int d = enqueue_sgemm(rt, da, en.k, db, en.n, dc, en.n, en.m, en.n, en.k, OCT_B200_SGEMM_AUTO, s, nullptr,
                                  &rt->batch_scratch[w]);
      if (d != 0) {
        fail_stage = PROM_STAGE_SUBMIT;
        fail_detail = d == OCT_B200_DETAIL_OUT_OF_MEMORY ? d : PROM_DETAIL_BATCH_EXECUTION_FAILED;
      }
    }
    for (uint32_t w = 0; w < workers; ++w)  // drain every worker, failed or not
      if (cudaStreamSynchronize(rt->batch_streams[w]) != cudaSuccess && fail_stage == PROM_STAGE_NONE) {
        fail_stage = PROM_STAGE_SUBMIT;
        fail_detail = PROM_DETAIL_BATCH_EXECUTION_FAILED;
      }
    Words wd;
    if (fail_stage == PROM_STAGE_NONE && (read_words(rt, &wd) != cudaSuccess || wd.err != 0)) {
      fail_stage = PROM_STAGE_SUBMIT;
      fail_detail = OCT_B200_DETAIL_DEVICE_TIMEOUT;
    }
    if (fail_stage != PROM_STAGE_NONE) {
      set_status(out_stage, out_detail_code, fail_stage, fail_detail == 0 ? PROM_ERROR : fail_detail);
      return PROM_ERROR;
    }
    // ordered commit: every output, in entry order, only now
    for (uint32_t i = 0; i < entry_count; ++i) {
      const uint64_t c_n = static_cast<uint64_t>(entries[i].m) * entries[i].n;
      if (cudaMemcpy(entries[i].c, cbase + c_off[i], c_n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
        return PROM_ERROR;
      }
    }
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, 0);
    return PROM_OK;
  } catch (...) {
    set_status(out_stage, out_detail_code, PROM_STAGE_INIT, OCT_B200_DETAIL_CUDA_ERROR);
    return PROM_INTERNAL_ERROR;
  }
}

// ---------------------------------------------------------------- async SGEMM
// Lifecycle and codes follow reactor_sgemm.cpp:6298-6500: submit copies the
// inputs into task-owned device memory and enqueues; query polls a CUDA event;
// consume copies the result into the caller's buffer (length-checked); abandon
// releases a finished task.  Capacity is four tasks.
int prometheus_reactor_runtime_sgemm_submit_async(void* handle, const float* a, const float* b, uint32_t m,
                                                  uint32_t n, uint32_t k, int* out_task_id, uint32_t* out_stage,
                                                  int* out_detail_code) {
  try {
    if (out_task_id == nullptr) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_ERROR);
      return PROM_ERROR;
    }
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_INVALID_HANDLE);
      return PROM_INVALID_HANDLE;
    }
    uint64_t a_n, b_n, c_n;
    if (!rt->available || a == nullptr || b == nullptr || m == 0 || n == 0 || k == 0 || !checked_mul(m, k, &a_n) ||
        !checked_mul(k, n, &b_n) || !checked_mul(m, n, &c_n) || c_n > UINT32_MAX) {
      // c_len in consume is a uint32_t element count, so C must fit it.
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_ERROR);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    AsyncTask* task = nullptr;
    for (auto& t : rt->tasks)
      if (!t.active) {
        task = &t;
        break;
      }
    if (task == nullptr) {
      ++rt->async_stats.queue_full;
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_DETAIL_ASYNC_QUEUE_FULL);
      return PROM_ERROR;
    }
    if ((task->begin == nullptr && cudaEventCreate(&task->begin) != cudaSuccess) ||
        (task->done == nullptr && cudaEventCreate(&task->done) != cudaSuccess)) {
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_DETAIL_ASYNC_SUBMIT_REJECTED);
      return PROM_ERROR;
    }
    if (task->a.ensure(a_n * 4, rt->stream) != cudaSuccess || task->b.ensure(b_n * 4, rt->stream) != cudaSuccess ||
        task->c.ensure(c_n * 4, rt->stream) != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_IN, OCT_B200_DETAIL_OUT_OF_MEMORY);
      return PROM_ERROR;
    }
    float* da = static_cast<float*>(task->a.aligned());
    float* db = static_cast<float*>(task->b.aligned());
    float* dc = static_cast<float*>(task->c.aligned());
    cudaError_t e = reset_words(rt);
    if (e == cudaSuccess) e = cudaMemcpyAsync(da, a, a_n * 4, cudaMemcpyHostToDevice, rt->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(db, b, b_n * 4, cudaMemcpyHostToDevice, rt->stream);
    // The caller may free a / b as soon as submit returns: wait for the copies.
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    const uint32_t variant =
        (rt->test_flags & PROM_TESTCFG_FORCE_STRICT_FP32) ? OCT_B200_SGEMM_FMA : OCT_B200_SGEMM_AUTO;
    if (e == cudaSuccess) e = cudaEventRecord(task->begin, rt->stream);
    int d = (e == cudaSuccess) ? enqueue_sgemm(rt, da, k, db, n, dc, n, m, n, k, variant, rt->stream) : -1;
    if (d == 0) e = cudaEventRecord(task->done, rt->stream);
    if (e != cudaSuccess || d != 0) {
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_ERROR);
      return PROM_ERROR;
    }
    task->active = true;
    task->id = rt->next_task_id++;
    if (rt->next_task_id <= 0) rt->next_task_id = 1;
    task->state = PROM_ASYNC_STATE_SUBMITTED;
    task->m = m;
    task->n = n;
    task->k = k;
    task->final_detail = PROM_DETAIL_PATH_DIRECT;
    task->final_stage = PROM_STAGE_SUBMIT;
    task->generation += 1;
    task->sequence = ++rt->async_stats.sequence;
    task->abandoned = false;
    task->timed = false;
    task->gpu_ns = 0;
    ++rt->async_stats.submitted;
    {
      uint32_t in_flight = 0;
      for (auto& t : rt->tasks)
        if (t.active && t.state == PROM_ASYNC_STATE_SUBMITTED) ++in_flight;
      rt->async_stats.max_in_flight = std::max(rt->async_stats.max_in_flight, in_flight);
    }
    *out_task_id = task->id;
    set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, 0);
    return PROM_OK;
  } catch (...) {
    set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_ERROR);
    return PROM_INTERNAL_ERROR;
  }
}


int prometheus_reactor_runtime_sgemm_query_async(void* handle, int task_id, PrometheusAsyncStatus* out_status) {
  try {
    if (out_status == nullptr) return PROM_ERROR;
    std::memset(out_status, 0, sizeof(*out_status));
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    AsyncTask* t = find_task(rt, task_id);
    if (t == nullptr) {
      out_status->lifecycle_state = PROM_ASYNC_STATE_IDLE;
      out_status->detail_code = PROM_DETAIL_ASYNC_NO_TASK;
      return PROM_ERROR;
    }
    poll_task(rt, t);
    out_status->lifecycle_state = t->state;
    out_status->stage = t->final_stage == 0 ? PROM_STAGE_SUBMIT : t->final_stage;
    out_status->detail_code = t->state == PROM_ASYNC_STATE_SUBMITTED ? PROM_DETAIL_ASYNC_NOT_READY : t->final_detail;
    out_status->ready = t->state == PROM_ASYNC_STATE_READY;
    out_status->failed = t->state == PROM_ASYNC_STATE_FAILED;
    out_status->consumed = t->state == PROM_ASYNC_STATE_CONSUMED;
    out_status->outstanding_tasks = outstanding(rt);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_sgemm_consume_async(void* handle, int task_id, float* c, uint32_t c_len,
                                                   uint32_t* out_stage, int* out_detail_code) {
  try {
    set_status(out_stage, out_detail_code, PROM_STAGE_NONE, 0);
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      set_status(out_stage, out_detail_code, PROM_STAGE_INIT, PROM_INVALID_HANDLE);
      return PROM_INVALID_HANDLE;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    AsyncTask* t = find_task(rt, task_id);
    if (t == nullptr) {
      ++rt->async_stats.stale_ids;
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_DETAIL_ASYNC_INVALID_TASK);
      return PROM_ERROR;
    }
    poll_task(rt, t);
    if (t->state == PROM_ASYNC_STATE_SUBMITTED) {
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT, PROM_DETAIL_ASYNC_NOT_READY);
      return PROM_ERROR;
    }
    if (t->state == PROM_ASYNC_STATE_FAILED) {
      set_status(out_stage, out_detail_code, PROM_STAGE_SUBMIT,
                 t->final_detail != 0 ? t->final_detail : PROM_DETAIL_ASYNC_FAILED);
      return PROM_ERROR;
    }
    if (t->state == PROM_ASYNC_STATE_CONSUMED) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, PROM_DETAIL_ASYNC_ALREADY_CONSUMED);
      return PROM_ERROR;
    }
    const uint64_t need = static_cast<uint64_t>(t->m) * t->n;
    if (c == nullptr || c_len < need) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, PROM_ERROR);
      return PROM_ERROR;
    }
    cudaError_t e = cudaMemcpyAsync(c, t->c.aligned(), need * 4, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
      return PROM_ERROR;
    }
    t->state = PROM_ASYNC_STATE_CONSUMED;
    ++rt->async_stats.consumed;
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, t->final_detail);
    return PROM_OK;
  } catch (...) {
    set_status(out_stage, out_detail_code, PROM_STAGE_TRANSFER_OUT, OCT_B200_DETAIL_CUDA_ERROR);
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_sgemm_abandon_async(void* handle, int task_id) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    AsyncTask* t = find_task(rt, task_id);
    if (t == nullptr) {
      ++rt->async_stats.stale_ids;
      return PROM_ERROR;
    }
    poll_task(rt, t);
    if (t->state == PROM_ASYNC_STATE_SUBMITTED) return PROM_ERROR;  // unconsumed work still in flight
    if (t->state != PROM_ASYNC_STATE_CONSUMED) ++rt->async_stats.abandoned;
    t->abandoned = t->state != PROM_ASYNC_STATE_CONSUMED;
    t->active = false;
    t->state = PROM_ASYNC_STATE_IDLE;
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

// ---------------------------------------------------------------- reductions
int prometheus_reactor_reduction_plan(const PrometheusReductionRequest* request, PrometheusReductionPlan* out_plan) {
  try {
    if (out_plan == nullptr) return PROM_ERROR;
    std::memset(out_plan, 0, sizeof(*out_plan));
    out_plan->struct_size = sizeof(*out_plan);
    if (request == nullptr || request->struct_size < sizeof(*request)) return PROM_ERROR;
    if (validate_shape(shape_of(request)) != 0) return PROM_ERROR;
    build_plan(shape_of(request), out_plan);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

// Validation order follows reactor_concept_reduction.cpp:55-100.
int prometheus_reactor_runtime_reduction(void* handle, const PrometheusReductionRequest* request,
                                         PrometheusReductionExecutionResult* out_result) {
  PrometheusReductionExecutionResult local{};
  PrometheusReductionExecutionResult& out = out_result != nullptr ? *out_result : local;
  try {
    const auto t0 = Clock::now();
    std::memset(&out, 0, sizeof(out));
    out.struct_size = sizeof(out);
    out.physical_slot_id = UINT32_MAX;
    out.first_nonfinite_index = UINT64_MAX;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) {
      out.stage = PROM_STAGE_INIT;
      out.detail_code = PROM_REDUCTION_DETAIL_RUNTIME_UNAVAILABLE;
      return PROM_INVALID_HANDLE;
    }
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_REDUCTION_DETAIL_INVALID_REQUEST;
    if (request == nullptr || request->struct_size < sizeof(*request)) return PROM_ERROR;
    if (request->input == nullptr) {
      out.detail_code = PROM_REDUCTION_DETAIL_NULL_INPUT;
      return PROM_ERROR;
    }
    if (request->output == nullptr) {
      out.detail_code = PROM_REDUCTION_DETAIL_NULL_OUTPUT;
      return PROM_ERROR;
    }
    const ReductionShape s = shape_of(request);
    const int v = validate_shape(s);
    if (v != 0) {
      out.detail_code = v;
      return PROM_ERROR;
    }
    build_plan(s, &out.plan);
    if (!rt->available) {
      out.detail_code = PROM_REDUCTION_DETAIL_RUNTIME_UNAVAILABLE;
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    out.logical_request_id = rt->next_request_id++;
    out.physical_slot_id = 0;
    out.physical_slot_recyclable = 1;
    uint32_t stage = 0;
    int32_t detail = 0;
    const int rc = run_reduction_host(rt, request->input, request->output, s.rows, s.width, s.operation, &stage,
                                      &detail, &out.gpu_duration_ns, &out.gpu_timestamp_valid,
                                      &out.first_nonfinite_index);
    out.stage = stage;
    out.detail_code = detail;
    out.end_to_end_ns = ns_since(t0);
    out.physical_slot_generation = rt->red_stats.slot_generation;
    note_reduction(rt, rc, detail, out.plan.stage_count, out.plan.replay_id, out.gpu_duration_ns, out.end_to_end_ns);
    return rc;
  } catch (...) {
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_REDUCTION_DETAIL_RESOURCE_CREATE_FAILED;
    return PROM_ERROR;
  }
}

// Validation order and codes follow reactor_vulkan_fused_reduction.c:892-994.
// The row / total ceilings are widened to the library's reduction envelope.
int prometheus_reactor_runtime_row_wise_softmax(void* handle, const PrometheusRowWiseSoftmaxRequest* request,
                                                PrometheusRowWiseSoftmaxResult* out_result) {
  PrometheusRowWiseSoftmaxResult local{};
  PrometheusRowWiseSoftmaxResult& out = out_result != nullptr ? *out_result : local;
  try {
    const auto t0 = Clock::now();
    std::memset(&out, 0, sizeof(out));
    out.struct_size = sizeof(out);
    out.first_nonfinite_index = UINT64_MAX;
    auto fail = [&](uint32_t stage, int32_t detail, int rc) {
      out.stage = stage;
      out.detail_code = detail;
      out.output_written = 0;
      return rc;
    };
    if (request == nullptr || request->struct_size < sizeof(*request))
      return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_INVALID_REQUEST, PROM_ERROR);
    const uint64_t total = static_cast<uint64_t>(request->row_count) * request->elements_per_row;
    if (request->input_element_count != total || request->output_element_count != total)
      return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_COUNT_MISMATCH, PROM_ERROR);
    if (total == 0) {
      out.stage = PROM_STAGE_NONE;
      out.detail_code = 0;
      return PROM_OK;
    }
    if (request->input == nullptr) return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_NULL_INPUT, PROM_ERROR);
    if (request->output == nullptr) return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_NULL_OUTPUT, PROM_ERROR);
    if (request->row_count > OCT_B200_REDUCTION_MAX_ROWS)
      return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_ROW_LIMIT, PROM_ERROR);
    if (request->elements_per_row > PROM_ROW_WISE_SOFTMAX_MAX_ELEMENTS_PER_ROW)
      return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_WIDTH_LIMIT, PROM_ERROR);
    if (total > OCT_B200_REDUCTION_MAX_TOTAL_ELEMENTS)
      return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_ELEMENT_LIMIT, PROM_ERROR);
    {
      const uintptr_t ib = reinterpret_cast<uintptr_t>(request->input);
      const uintptr_t ob = reinterpret_cast<uintptr_t>(request->output);
      const uint64_t bytes = total * sizeof(float);
      if (ib != ob && ib < ob + bytes && ob < ib + bytes)
        return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_PARTIAL_ALIAS, PROM_ERROR);
    }
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_RUNTIME_UNAVAILABLE, PROM_INVALID_HANDLE);
    if (!rt->available) return fail(PROM_STAGE_INIT, PROM_SOFTMAX_DETAIL_RUNTIME_UNAVAILABLE, PROM_ERROR);
    std::lock_guard<std::mutex> lock(rt->mu);
    uint32_t stage = 0;
    int32_t detail = 0;
    const int rc = run_reduction_host(rt, request->input, request->output, request->row_count,
                                      request->elements_per_row, PROM_REDUCTION_OPERATION_SOFTMAX, &stage, &detail,
                                      &out.gpu_duration_ns, &out.gpu_timestamp_valid, &out.first_nonfinite_index);
    out.end_to_end_ns = ns_since(t0);
    note_reduction(rt, rc, detail, 1, 0, out.gpu_duration_ns, out.end_to_end_ns);
    if (rc != PROM_OK) {
      const int32_t d = detail == PROM_REDUCTION_DETAIL_NONFINITE_INPUT ? PROM_SOFTMAX_DETAIL_NONFINITE_INPUT : detail;
      return fail(stage, d, rc);
    }
    out.stage = PROM_STAGE_NONE;
    out.detail_code = 0;
    out.physical_dispatch_count = 1;
    out.physical_submission_count = 1;
    out.output_written = 1;
    return PROM_OK;
  } catch (...) {
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_SOFTMAX_DETAIL_RUNTIME_UNAVAILABLE;
    return PROM_ERROR;
  }
}


// ---------------------------------------------------------------- device extensions
int oct_b200_sgemm_device_ld(void* handle, const float* d_a, uint64_t lda, const float* d_b, uint64_t ldb, float* d_c,
                             uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, uint32_t variant, void* stream,
                             int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (d_a == nullptr || d_b == nullptr || d_c == nullptr || lda < k || ldb < n || ldc < n) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_INVALID_ARGUMENT;
      return PROM_ERROR;
    }
    if (!rt->available) {
      if (out_detail_code) *out_detail_code = PROM_DETAIL_CAPABILITY_MISMATCH;
      return PROM_ERROR;
    }
    if (m == 0 || n == 0 || k == 0) return PROM_OK;
    std::lock_guard<std::mutex> lock(rt->mu);
    cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL is the CUDA default stream
    const int d = enqueue_sgemm(rt, d_a, lda, d_b, ldb, d_c, ldc, m, n, k, variant, s);
    if (d != 0) {
      if (out_detail_code) *out_detail_code = d;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_sgemm_batched_device(void* handle, const float* d_a, uint64_t lda, uint64_t stride_a, const float* d_b,
                                  uint64_t ldb, uint64_t stride_b, uint32_t b_trans, float* d_c, uint64_t ldc,
                                  uint64_t stride_c, uint32_t batch, uint32_t m, uint32_t n, uint32_t k,
                                  uint32_t variant, void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    const uint64_t need_ldb = b_trans ? k : n;
    if (d_a == nullptr || d_b == nullptr || d_c == nullptr || lda < k || ldb < need_ldb || ldc < n ||
        batch > 65535u) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_INVALID_ARGUMENT;
      return PROM_ERROR;
    }
    if (!rt->available) {
      if (out_detail_code) *out_detail_code = PROM_DETAIL_CAPABILITY_MISMATCH;
      return PROM_ERROR;
    }
    if (m == 0 || n == 0 || k == 0 || batch == 0) return PROM_OK;
    std::lock_guard<std::mutex> lock(rt->mu);
    oct::GemmBatch bt;
    bt.count = batch;
    bt.stride_a = stride_a;
    bt.stride_b = stride_b;
    bt.stride_c = stride_c;
    bt.b_trans = b_trans != 0;
    const int d = enqueue_sgemm(rt, d_a, lda, d_b, ldb, d_c, ldc, m, n, k, variant, static_cast<cudaStream_t>(stream),
                                &bt);
    if (d != 0) {
      if (out_detail_code) *out_detail_code = d;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_sgemm_device(void* handle, const float* d_a, const float* d_b, float* d_c, uint32_t m, uint32_t n,
                          uint32_t k, uint32_t variant, void* stream, int* out_detail_code) {
  return oct_b200_sgemm_device_ld(handle, d_a, k, d_b, n, d_c, n, m, n, k, variant, stream, out_detail_code);
}

int oct_b200_reduction_device(void* handle, const float* d_in, float* d_out, uint32_t rows, uint32_t width,
                              uint32_t operation, void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (d_in == nullptr || d_out == nullptr || operation < 1 || operation > 3) {
      if (out_detail_code) *out_detail_code = PROM_REDUCTION_DETAIL_INVALID_REQUEST;
      return PROM_ERROR;
    }
    if (!rt->available) {
      if (out_detail_code) *out_detail_code = PROM_REDUCTION_DETAIL_RUNTIME_UNAVAILABLE;
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL is the CUDA default stream
    const cudaError_t e = oct::row_reduce(d_in, d_out, rows, width, operation, rt->nonfinite_word(), rt->err_word(), s);
    if (e != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_attention_device(void* handle, const float* d_q, const float* d_k, const float* d_v, float* d_out,
                              uint32_t items, uint32_t seq, uint32_t heads, uint32_t head_dim, float scale,
                              void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (d_q == nullptr || d_k == nullptr || d_v == nullptr || d_out == nullptr || !finite_f(scale)) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_INVALID_ARGUMENT;
      return PROM_ERROR;
    }
    if (items == 0 || heads == 0 || seq == 0) return PROM_OK;
    if (!oct::flash_attention_supported(head_dim, seq) || items > 65535u || heads > 65535u) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_UNSUPPORTED_SHAPE;
      return PROM_ERROR;
    }
    for (const float* p : {d_q, d_k, d_v, static_cast<const float*>(d_out)})
      if (reinterpret_cast<uintptr_t>(p) % 16 != 0) {
        if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_UNALIGNED;
        return PROM_ERROR;
      }
    if (!rt->available) {
      if (out_detail_code) *out_detail_code = PROM_DETAIL_CAPABILITY_MISMATCH;
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL is the CUDA default stream
    const uint64_t ld = static_cast<uint64_t>(heads) * head_dim;
    const uint64_t e = static_cast<uint64_t>(items) * seq * ld;  // elements of one split half
    const uint64_t half_bytes = (e * sizeof(float) + 1023) & ~uint64_t(1023);
    if (rt->scratch.ensure(6 * half_bytes, s) != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_OUT_OF_MEMORY;
      return PROM_ERROR;
    }
    auto part = [&](int i) { return reinterpret_cast<float*>(static_cast<char*>(rt->scratch.aligned()) + i * half_bytes); };
    const oct::SgemmEvents* ev = nullptr;
    if (rt->timing && (ev = next_timing_events(rt)) == nullptr) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    cudaError_t err = ev ? cudaEventRecord(ev->split_begin, s) : cudaSuccess;
    if (err == cudaSuccess) err = oct::split_heads(d_q, ld, items, heads, seq, part(0), part(1), s);
    if (err == cudaSuccess) err = oct::split_heads(d_k, ld, items, heads, seq, part(2), part(3), s);
    if (err == cudaSuccess) err = oct::split_transpose_heads(d_v, ld, items, heads, seq, part(4), part(5), s);
    if (err == cudaSuccess && ev) err = cudaEventRecord(ev->main_begin, s);
    if (err == cudaSuccess) {
      const oct::AttnOperands ops{part(0), part(1), part(2), part(3), part(4), part(5)};
      err = oct::flash_attention_tf32x3(ops, d_out, ld, items, heads, seq, scale, rt->err_word(), s);
    }
    if (err == cudaSuccess && ev) err = cudaEventRecord(ev->main_end, s);
    if (err != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_selftest_wait_timeout(void* handle, uint64_t budget_ns, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (budget_ns < 1000000ull || budget_ns > 1000000000ull) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_INVALID_ARGUMENT;
      return PROM_ERROR;
    }
    if (!rt->available) {
      if (out_detail_code) *out_detail_code = PROM_DETAIL_CAPABILITY_MISMATCH;
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    DevBuf flag;  // one u64 epoch that no rank ever sets
    cudaError_t e = flag.ensure(64, rt->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(flag.aligned(), 0, 8, rt->stream);
    if (e == cudaSuccess) e = reset_words(rt);
    if (e == cudaSuccess)
      e = oct::tp_wait(static_cast<const uint64_t*>(flag.aligned()), 0, 1, 1, rt->err_word(), budget_ns, rt->stream);
    Words w;
    if (e == cudaSuccess) e = read_words(rt, &w);
    // the observed bit is reported here and cleared: the handle carries no stale status
    if (e == cudaSuccess) e = reset_words(rt);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    flag.release();
    if (e != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    if (w.err != 0) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_DEVICE_TIMEOUT;
      return PROM_ERROR;
    }
    return PROM_OK;  // the wait did not give up: the self-test failed to observe a timeout
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_rmsnorm_device(void* handle, const float* d_in, const float* d_weight, float* d_out, float* d_inv_rms,
                            uint32_t rows, uint32_t width, float epsilon, void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (d_in == nullptr || d_weight == nullptr || d_out == nullptr || !finite_f(epsilon) || epsilon <= 0.f) {
      if (out_detail_code) *out_detail_code = PROM_M46_DETAIL_INVALID_REQUEST;
      return PROM_ERROR;
    }
    if (!rt->available) {
      if (out_detail_code) *out_detail_code = PROM_M46_DETAIL_RESOURCE;
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL is the CUDA default stream
    const cudaError_t e = oct::rmsnorm(d_in, width, d_weight, d_out, d_inv_rms, rows, width, epsilon,
                                       rt->nonfinite_word(), rt->err_word(), s);
    if (e != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_sync_status(void* handle, void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (!rt->available) return PROM_ERROR;
    std::lock_guard<std::mutex> lock(rt->mu);
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    Words w;
    if (read_words(rt, &w) != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    if (reset_words(rt) != cudaSuccess || cudaStreamSynchronize(rt->stream) != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_CUDA_ERROR;
      return PROM_ERROR;
    }
    if (w.err != 0) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_DEVICE_TIMEOUT;
      return PROM_ERROR;
    }
    if (w.nonfinite != ~0ull) {
      if (out_detail_code) *out_detail_code = PROM_REDUCTION_DETAIL_NONFINITE_INPUT;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_set_kernel_timing(void* handle, int enable) {
  Runtime* rt = lookup(handle);
  if (rt == nullptr) return PROM_INVALID_HANDLE;
  std::lock_guard<std::mutex> lock(rt->mu);
  rt->timing = enable != 0;
  rt->timing_used = 0;
  return PROM_OK;
}

int oct_b200_read_kernel_timing(void* handle, double* split_ms_total, double* main_ms_total, uint32_t* launches) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    double split = 0.0, main = 0.0;
    for (size_t i = 0; i < rt->timing_used; ++i) {
      const oct::SgemmEvents& ev = rt->timing_events[i];
      if (cudaEventSynchronize(ev.main_end) != cudaSuccess) return PROM_ERROR;
      float a = 0.f, b = 0.f;
      if (cudaEventElapsedTime(&a, ev.split_begin, ev.main_begin) != cudaSuccess ||
          cudaEventElapsedTime(&b, ev.main_begin, ev.main_end) != cudaSuccess)
        return PROM_ERROR;
      split += a;
      main += b;
    }
    if (split_ms_total) *split_ms_total = split;
    if (main_ms_total) *main_ms_total = main;
    if (launches) *launches = static_cast<uint32_t>(rt->timing_used);
    rt->timing_used = 0;
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_nccl_unique_id(uint8_t* out_128_bytes) {
  if (out_128_bytes == nullptr) return PROM_ERROR;
  oct::NcclUniqueIdBytes id{};
  if (oct::nccl_unique_id(&id) != 0) return PROM_ERROR;
  std::memcpy(out_128_bytes, id.bytes, 128);
  return PROM_OK;
}

int oct_b200_block_create(void* handle, const OctB200BlockConfig* cfg, uint64_t* out_block_id, int* out_detail_code) {
  auto fail = [&](int rc, int detail) {
    if (out_detail_code) *out_detail_code = detail;
    return rc;
  };
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (cfg == nullptr || out_block_id == nullptr || cfg->struct_size < sizeof(OctB200BlockConfig))
      return fail(PROM_ERROR, OCT_B200_DETAIL_BLOCK_INVALID);
    if (!rt->available) return fail(PROM_ERROR, PROM_DETAIL_CAPABILITY_MISMATCH);
    oct::BlockDims d;
    d.family = cfg->family;
    d.hidden = cfg->hidden;
    d.heads = cfg->heads;
    d.kv_heads = cfg->kv_heads;
    d.head_dim = cfg->head_dim;
    d.ffn = cfg->ffn;
    d.seq_len = cfg->seq_len;
    d.max_batch = cfg->max_batch;
    d.eps = cfg->eps;
    d.rope_base = cfg->rope_base;
    d.grid_w = cfg->grid_w;
    d.rope_frame = cfg->rope_frame;
    d.tp_rank = cfg->tp_rank;
    d.tp_world = cfg->tp_world == 0 ? 1 : cfg->tp_world;
    if (d.family == oct::kGemma && d.kv_heads != 1) return fail(PROM_ERROR, OCT_B200_DETAIL_BLOCK_INVALID);
    if (d.tp_rank >= d.tp_world) return fail(PROM_ERROR, OCT_B200_DETAIL_BLOCK_INVALID);
    oct::NcclUniqueIdBytes id{};
    std::memcpy(id.bytes, cfg->nccl_id, 128);
    std::lock_guard<std::mutex> lock(rt->mu);
    oct::Block* b = new (std::nothrow) oct::Block();
    if (b == nullptr) return fail(PROM_ERROR, OCT_B200_DETAIL_BLOCK_ALLOC);
    const int rc = b->init(d, &id, rt->stream);
    if (rc != 0) {
      delete b;
      return fail(PROM_ERROR, rc == -3 ? OCT_B200_DETAIL_BLOCK_ALLOC
                                       : (rc == -5 ? OCT_B200_DETAIL_BLOCK_NCCL : OCT_B200_DETAIL_BLOCK_INVALID));
    }
    const uint64_t id_out = rt->next_block++;
    rt->blocks[id_out] = b;
    *out_block_id = id_out;
    return PROM_OK;
  } catch (...) {
    return fail(PROM_INTERNAL_ERROR, OCT_B200_DETAIL_BLOCK_ALLOC);
  }
}

int oct_b200_block_set_weight(void* handle, uint64_t block_id, uint32_t slot, const float* data,
                              uint64_t element_count, uint32_t data_on_device) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->blocks.find(block_id);
    if (it == rt->blocks.end() || data == nullptr) return PROM_ERROR;
    it->second->set_stream(rt->stream);
    return it->second->set_weight(slot, data, element_count, data_on_device != 0) == 0 ? PROM_OK : PROM_ERROR;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_block_forward_device(void* handle, uint64_t block_id, const float* d_x, float* d_y, uint32_t batch,
                                  const float* timesteps, void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->blocks.find(block_id);
    if (it == rt->blocks.end()) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_BLOCK_NOT_FOUND;
      return PROM_ERROR;
    }
    if (d_x == nullptr || d_y == nullptr) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_BLOCK_INVALID;
      return PROM_ERROR;
    }
    oct::Block* b = it->second;
    b->set_stream(static_cast<cudaStream_t>(stream));
    const int rc = b->forward(d_x, d_y, batch, timesteps);
    if (rc != 0) {
      if (out_detail_code) *out_detail_code = rc == -1 ? OCT_B200_DETAIL_BLOCK_INVALID : OCT_B200_DETAIL_BLOCK_EXEC;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_block_forward(void* handle, uint64_t block_id, const float* x, float* y, uint32_t batch,
                           const float* timesteps, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->blocks.find(block_id);
    if (it == rt->blocks.end()) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_BLOCK_NOT_FOUND;
      return PROM_ERROR;
    }
    if (x == nullptr || y == nullptr) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_BLOCK_INVALID;
      return PROM_ERROR;
    }
    oct::Block* b = it->second;
    const oct::BlockDims& d = b->dims();
    if (batch == 0 || batch > d.max_batch) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_BLOCK_INVALID;
      return PROM_ERROR;
    }
    const uint64_t bytes = static_cast<uint64_t>(batch) * d.seq_len * d.hidden * sizeof(float);
    if (rt->rin.ensure(bytes, rt->stream) != cudaSuccess || rt->rout.ensure(bytes, rt->stream) != cudaSuccess) {
      if (out_detail_code) *out_detail_code = OCT_B200_DETAIL_OUT_OF_MEMORY;
      return PROM_ERROR;
    }
    float* dx = static_cast<float*>(rt->rin.aligned());
    float* dy = static_cast<float*>(rt->rout.aligned());
    b->set_stream(rt->stream);
    cudaError_t e = cudaMemcpyAsync(dx, x, bytes, cudaMemcpyHostToDevice, rt->stream);
    int rc = e == cudaSuccess ? b->forward(dx, dy, batch, timesteps) : -4;
    if (rc == 0) e = cudaMemcpyAsync(y, dy, bytes, cudaMemcpyDeviceToHost, rt->stream);
    if (rc == 0 && e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (rc == 0 && e == cudaSuccess && b->read_status() != 0) rc = -4;
    if (rc != 0 || e != cudaSuccess) {
      (void)cudaGetLastError();
      if (out_detail_code) *out_detail_code = rc == -1 ? OCT_B200_DETAIL_BLOCK_INVALID : OCT_B200_DETAIL_BLOCK_EXEC;
      return PROM_ERROR;
    }
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_block_destroy(void* handle, uint64_t block_id) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->blocks.find(block_id);
    if (it == rt->blocks.end()) return PROM_ERROR;
    delete it->second;
    rt->blocks.erase(it);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

const char* oct_b200_build_info(void) {
  return "oct_b200 prometheus reactor (ABI v1) sm_100a: tcgen05 3xTF32 SGEMM, FP32-FMA SGEMM, bulk-fed reductions";
}

}  // extern "C"
