// gemma_m1_api.cpp -- the Gemma-4 E2B M1 entry points of the C ABI.
//
// The reference family (internal/prometheus/native/reactor_api.c:250-586 and
// reactor_concept_rmsnorm.cpp:38-212) is five model-private operations that
// share one committed RMSNorm weight per handle:
//
//   input RMSNorm, projection-activation RMSNorm (BF16 output), head RMSNorm
//   (BF16 input and output), half-split RoPE, head RMSNorm -> RoPE, and the raw
//   attention-score chain built from two of the latter.
//
// This file keeps the reference's request / result structs, validation order
// and detail codes:
//   * request fields first (PROM_M46_DETAIL_INVALID_REQUEST at stage INIT),
//   * then the handle (PROM_INVALID_HANDLE),
//   * then the weight preparation: width, finiteness (NONFINITE_INPUT), and a
//     weight generation that must exceed the one the handle last committed
//     (STALE_WEIGHT_GENERATION; the generation is committed before execution,
//     as the reference's prepare step does),
//   * then the execution envelope and the input's finiteness,
//   * then one device pass, and a finiteness check of what was read back (READBACK).
// Hashes use the reference's two FNV-1a serialisations: 4 bytes per float for
// weights and the RoPE boundary (reactor_concept_rmsnorm.cpp:42-49), each
// float's bits widened to 8 bytes for RMSNorm inputs / outputs and scores
// (prom_num_hash_float_bits, reactor_vulkan_common.c:398-418).
//
// Widened ceilings (recorded as ABI widenings): tokens, heads and head width up
// to OCT_B200_M1_MAX_*, RMSNorm rows / widths up to the reduction envelope.
#include <cmath>
#include <cstring>

#include "runtime.h"

namespace {

using namespace oct::rt;

constexpr uint64_t kFnvOffset = 1469598103934665603ull;
constexpr uint64_t kFnvPrime = 1099511628211ull;
constexpr uint32_t kMaxRmsWidth = 1u << 20;

uint64_t hash_u32_bits(const float* v, uint64_t n) {
  uint64_t h = kFnvOffset;
  for (uint64_t i = 0; i < n; ++i) {
    uint32_t bits;
    std::memcpy(&bits, v + i, 4);
    for (unsigned b = 0; b < 4; ++b) {
      h ^= static_cast<uint8_t>(bits >> (8 * b));
      h *= kFnvPrime;
    }
  }
  return h;
}

uint64_t hash_u64_bits(const float* v, uint64_t n) {
  if (v == nullptr && n != 0) return 0;
  uint64_t h = kFnvOffset;
  for (uint64_t i = 0; i < n; ++i) {
    uint32_t bits;
    std::memcpy(&bits, v + i, 4);
    const uint64_t wide = bits;
    for (unsigned b = 0; b < 8; ++b) {
      h ^= (wide >> (8 * b)) & 0xffu;
      h *= kFnvPrime;
    }
  }
  return h;
}

bool all_finite(const float* v, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i)
    if (!std::isfinite(v[i])) return false;
  return true;
}

struct StageCounts {
  uint64_t alloc = 0, reuse = 0;
};

cudaError_t stage(DevBuf& b, uint64_t bytes, cudaStream_t s, StageCounts& c) {
  if (b.raw != nullptr && bytes <= b.cap) {
    ++c.reuse;
    return cudaSuccess;
  }
  ++c.alloc;
  return b.ensure(bytes == 0 ? 4 : bytes, s);
}

bool m1_geometry(uint32_t tokens, uint32_t heads, uint32_t head_width) {
  return tokens != 0 && tokens <= OCT_B200_M1_MAX_TOKENS && heads != 0 && heads <= OCT_B200_M1_MAX_HEADS &&
         head_width >= 2 && head_width <= OCT_B200_M1_MAX_HEAD_WIDTH && head_width % 2 == 0;
}

// The weight preparation of every M46-family entry (reactor_concept_rmsnorm.cpp:85-108):
// 0 or a detail code; on success the generation is committed to the handle.
int prepare_weight(Runtime* rt, const float* w, uint64_t count, uint32_t width, uint64_t generation,
                   uint64_t* hash, uint64_t* observed, uint64_t* requested) {
  if (w == nullptr || width == 0 || width > kMaxRmsWidth || generation == 0 || count != width)
    return PROM_M46_DETAIL_INVALID_REQUEST;
  if (!all_finite(w, count)) return PROM_M46_DETAIL_NONFINITE_INPUT;
  *hash = hash_u32_bits(w, count);
  if (!rt->available) return PROM_M46_DETAIL_RESOURCE;
  *observed = rt->m46_weight_generation;
  *requested = generation;
  if (generation <= rt->m46_weight_generation) return PROM_M46_DETAIL_STALE_WEIGHT_GENERATION;
  rt->m46_weight_generation = generation;
  return 0;
}

// Body of the three RMSNorm entries (reactor_api.c:250-395).
int m46_rmsnorm(void* handle, const PrometheusGemma4E2BM1InputRmsNormRequest* r,
                PrometheusGemma4E2BM1InputRmsNormResult* out_result, bool round_in, bool round_out, bool head) {
  if (out_result == nullptr) return PROM_ERROR;
  PrometheusGemma4E2BM1InputRmsNormResult& out = *out_result;
  const auto t0 = Clock::now();
  std::memset(&out, 0, sizeof(out));
  out.struct_size = sizeof(out);
  out.stage = PROM_STAGE_INIT;
  out.detail_code = PROM_M46_DETAIL_INVALID_REQUEST;
  if (head) {
    // reactor_api.c:378-392 (the 120-row and 256-wide ceilings widened)
    if (r == nullptr || r->struct_size < sizeof(*r) || r->input == nullptr || r->weight == nullptr ||
        r->output == nullptr || r->inv_rms_output == nullptr || r->tokens == 0 ||
        r->tokens > OCT_B200_REDUCTION_MAX_ROWS || r->model_width == 0 || r->model_width > kMaxRmsWidth ||
        r->input_row_stride != r->model_width ||
        r->input_element_count != static_cast<uint64_t>(r->tokens) * r->model_width ||
        r->weight_element_count != r->model_width ||
        r->output_element_count != static_cast<uint64_t>(r->tokens) * r->model_width ||
        r->inv_rms_output_element_count != r->tokens || r->epsilon != 0.000001f)
      return PROM_ERROR;
  }
  if (r == nullptr || r->struct_size < sizeof(*r) || r->input == nullptr || r->weight == nullptr ||
      r->output == nullptr || r->inv_rms_output == nullptr || r->tokens == 0 || r->model_width == 0 ||
      r->input_row_stride < r->model_width || r->input_generation == 0 || r->weight_generation == 0 ||
      r->exact_source_hash == 0)
    return PROM_ERROR;
  Runtime* rt = lookup(handle);
  if (rt == nullptr) return PROM_INVALID_HANDLE;
  std::lock_guard<std::mutex> lock(rt->mu);
  uint64_t observed = 0, requested = 0;
  int d = prepare_weight(rt, r->weight, r->weight_element_count, r->model_width, r->weight_generation,
                         &out.weight_hash, &observed, &requested);
  if (d != 0) {
    out.detail_code = d;
    return PROM_ERROR;
  }
  // execution envelope (reactor_concept_rmsnorm.cpp:50-70, ceilings widened)
  uint64_t storage = 0, logical = 0;
  if (!checked_mul(r->tokens, r->input_row_stride, &storage) || !checked_mul(r->tokens, r->model_width, &logical) ||
      r->tokens > OCT_B200_REDUCTION_MAX_ROWS || r->model_width > kMaxRmsWidth ||
      storage != r->input_element_count || storage > (1ull << 36) || logical > OCT_B200_REDUCTION_MAX_TOTAL_ELEMENTS ||
      !std::isfinite(r->epsilon) || r->epsilon <= 0.f || r->output_element_count != logical ||
      r->inv_rms_output_element_count != r->tokens)
    return PROM_ERROR;
  out.input_hash = hash_u64_bits(r->input, storage);
  if (!all_finite(r->input, storage)) {
    out.detail_code = PROM_M46_DETAIL_NONFINITE_INPUT;
    return PROM_ERROR;
  }
  // one device pass
  StageCounts sc;
  if (stage(rt->rin, storage * 4, rt->stream, sc) != cudaSuccess ||
      stage(rt->rw, static_cast<uint64_t>(r->model_width) * 4, rt->stream, sc) != cudaSuccess ||
      stage(rt->rout, logical * 4, rt->stream, sc) != cudaSuccess ||
      stage(rt->rinv, static_cast<uint64_t>(r->tokens) * 4, rt->stream, sc) != cudaSuccess) {
    out.detail_code = PROM_M46_DETAIL_RESOURCE;
    return PROM_ERROR;
  }
  rt->m46_allocations += sc.alloc;
  float* din = static_cast<float*>(rt->rin.aligned());
  float* dw = static_cast<float*>(rt->rw.aligned());
  float* dout = static_cast<float*>(rt->rout.aligned());
  float* dinv = static_cast<float*>(rt->rinv.aligned());
  cudaError_t e = reset_words(rt);
  if (e == cudaSuccess) e = cudaMemcpyAsync(din, r->input, storage * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dw, r->weight, static_cast<uint64_t>(r->model_width) * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    out.stage = PROM_STAGE_TRANSFER_IN;
    out.detail_code = PROM_M46_DETAIL_SUBMIT;
    return PROM_ERROR;
  }
  cudaEventRecord(rt->ev0, rt->stream);
  if (round_in || round_out)
    e = oct::m1_rmsnorm_bf16(din, r->input_row_stride, dw, dout, dinv, r->tokens, r->model_width, r->epsilon,
                             round_in, round_out, rt->stream);
  else
    e = oct::rmsnorm(din, r->input_row_stride, dw, dout, dinv, r->tokens, r->model_width, r->epsilon,
                     rt->nonfinite_word(), rt->err_word(), rt->stream);
  cudaEventRecord(rt->ev1, rt->stream);
  Words w;
  if (e != cudaSuccess || read_words(rt, &w) != cudaSuccess || w.err != 0 ||
      (rt->reduction_test_flags & PROM_REDUCTION_TESTCFG_FAIL_COMPLETION_OBSERVATION)) {
    (void)cudaGetLastError();
    out.stage = PROM_STAGE_SUBMIT;
    out.detail_code = PROM_M46_DETAIL_COMPLETION_UNCERTAIN;
    return PROM_ERROR;  // nothing read back: the caller's output stays untouched
  }
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, rt->ev0, rt->ev1) == cudaSuccess)
    out.apply_gpu_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
  e = cudaMemcpyAsync(r->output, dout, logical * 4, cudaMemcpyDeviceToHost, rt->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(r->inv_rms_output, dinv, static_cast<uint64_t>(r->tokens) * 4, cudaMemcpyDeviceToHost,
                        rt->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    out.stage = PROM_STAGE_TRANSFER_OUT;
    out.detail_code = PROM_M46_DETAIL_READBACK;
    return PROM_ERROR;
  }
  if (!all_finite(r->output, logical) || !all_finite(r->inv_rms_output, r->tokens)) {
    out.detail_code = PROM_M46_DETAIL_READBACK;
    return PROM_ERROR;
  }
  out.output_hash = hash_u64_bits(r->output, logical);
  out.inv_rms_hash = hash_u64_bits(r->inv_rms_output, r->tokens);
  out.stage = PROM_STAGE_NONE;
  out.detail_code = 0;
  out.output_written = 1;
  out.matched_input = 1;
  out.submit_count = 1;
  out.final_readback_count = 1;
  out.no_product_intermediate_readback_change = 1;
  out.retained_bytes = rt->rin.cap + rt->rw.cap + rt->rout.cap + rt->rinv.cap;
  out.buffer_allocation_count = rt->m46_allocations;
  out.buffer_reuse_count = sc.reuse;
  out.pipeline_create_count = 1;
  out.end_to_end_ns = ns_since(t0);
  return PROM_OK;
}

enum Slot : uint32_t { kSlotQuery = 0, kSlotKey = 1, kSlotScore = 2 };

// Head RMSNorm -> RoPE (reactor_api.c:404-505) with rt->mu held and the
// handle already validated.  The positioned rows land in the handle's `slot`
// (Q or K) and, with a non-null output, are read back.
int head_rope_locked(Runtime* rt, const PrometheusGemma4E2BM1HeadRmsNormRopeRequest* r,
                     PrometheusGemma4E2BM1HeadRmsNormRopeResult& out, Slot slot, StageCounts& sc) {
  const uint64_t rows = static_cast<uint64_t>(r->tokens) * r->heads;
  const uint64_t elems = rows * r->head_width;
  const uint64_t table = static_cast<uint64_t>(r->tokens) * r->head_width;
  int d = prepare_weight(rt, r->weight, r->weight_element_count, r->head_width, r->weight_generation,
                         &out.weight_hash, &out.observed_weight_generation, &out.requested_weight_generation);
  if (d != 0) {
    out.detail_code = d;
    return PROM_ERROR;
  }
  out.input_hash = hash_u64_bits(r->input, elems);
  if (!all_finite(r->input, elems) || !all_finite(r->cosine, table) || !all_finite(r->sine, table)) {
    out.detail_code = PROM_M46_DETAIL_NONFINITE_INPUT;
    return PROM_ERROR;
  }
  DevBuf& dst = slot == kSlotKey ? rt->m1_k : rt->m1_q;
  if (stage(rt->rin, elems * 4, rt->stream, sc) != cudaSuccess ||
      stage(rt->rw, static_cast<uint64_t>(r->head_width) * 4, rt->stream, sc) != cudaSuccess ||
      stage(rt->m1_cos, table * 4, rt->stream, sc) != cudaSuccess ||
      stage(rt->m1_sin, table * 4, rt->stream, sc) != cudaSuccess ||
      stage(dst, elems * 4, rt->stream, sc) != cudaSuccess) {
    out.detail_code = PROM_M46_DETAIL_RESOURCE;
    return PROM_ERROR;
  }
  float* din = static_cast<float*>(rt->rin.aligned());
  float* dw = static_cast<float*>(rt->rw.aligned());
  float* dcos = static_cast<float*>(rt->m1_cos.aligned());
  float* dsin = static_cast<float*>(rt->m1_sin.aligned());
  float* dout = static_cast<float*>(dst.aligned());
  cudaError_t e = cudaMemcpyAsync(din, r->input, elems * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dw, r->weight, static_cast<uint64_t>(r->head_width) * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dcos, r->cosine, table * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dsin, r->sine, table * 4, cudaMemcpyHostToDevice, rt->stream);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    out.stage = PROM_STAGE_TRANSFER_IN;
    out.detail_code = PROM_M46_DETAIL_SUBMIT;
    return PROM_ERROR;
  }
  e = oct::m1_head_rmsnorm_rope(din, dw, dcos, dsin, dout, r->tokens, r->heads, r->head_width, r->epsilon,
                                rt->stream);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    out.stage = PROM_STAGE_SUBMIT;
    out.detail_code = PROM_M46_DETAIL_COMMAND;
    return PROM_ERROR;
  }
  ++rt->m1_slot_generation[slot];
  if (r->output != nullptr) {
    e = cudaMemcpyAsync(r->output, dout, elems * 4, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_TRANSFER_OUT;
      out.detail_code = PROM_M46_DETAIL_READBACK;
      return PROM_ERROR;
    }
    if (!all_finite(r->output, elems)) {
      out.detail_code = PROM_M46_DETAIL_READBACK;
      return PROM_ERROR;
    }
    out.output_hash = hash_u64_bits(r->output, elems);
    out.output_written = 1;
  } else {
    if (cudaStreamSynchronize(rt->stream) != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_SUBMIT;
      out.detail_code = PROM_M46_DETAIL_COMPLETION_UNCERTAIN;
      return PROM_ERROR;
    }
    out.output_hash = 1;
  }
  out.stage = PROM_STAGE_NONE;
  out.detail_code = 0;
  out.dispatch_count = 1;
  out.resident_source_bound = 1;
  out.normalized_readback_count = 0;
  out.source_byte_range = elems * 4;
  out.destination_byte_range = elems * 4;
  out.buffer_allocation_count = sc.alloc;
  out.buffer_reuse_count = sc.reuse;
  out.pipeline_create_count = 1;
  return PROM_OK;
}

// Request checks of the head RMSNorm -> RoPE entry (reactor_api.c:418-441), ceilings widened.
bool head_rope_request_ok(const PrometheusGemma4E2BM1HeadRmsNormRopeRequest* r) {
  if (r == nullptr || r->struct_size < sizeof(*r) || r->input == nullptr || r->weight == nullptr ||
      r->cosine == nullptr || r->sine == nullptr || (r->output == nullptr && r->output_element_count != 0) ||
      !m1_geometry(r->tokens, r->heads, r->head_width) || r->epsilon != 0.000001f || r->input_generation == 0 ||
      r->weight_generation == 0 || r->table_generation == 0 || r->exact_source_hash == 0)
    return false;
  const uint64_t rows = static_cast<uint64_t>(r->tokens) * r->heads;
  return r->input_element_count == rows * r->head_width && r->weight_element_count == r->head_width &&
         r->cosine_element_count == static_cast<uint64_t>(r->tokens) * r->head_width &&
         r->sine_element_count == static_cast<uint64_t>(r->tokens) * r->head_width &&
         (r->output == nullptr || r->output_element_count == r->input_element_count);
}

}  // namespace

extern "C" {

int prometheus_reactor_runtime_gemma4e2b_m1_input_rmsnorm(void* handle,
                                                          const PrometheusGemma4E2BM1InputRmsNormRequest* request,
                                                          PrometheusGemma4E2BM1InputRmsNormResult* out_result) {
  try {
    return m46_rmsnorm(handle, request, out_result, false, false, false);
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_gemma4e2b_m1_projection_activation_rmsnorm(
    void* handle, const PrometheusGemma4E2BM1InputRmsNormRequest* request,
    PrometheusGemma4E2BM1InputRmsNormResult* out_result) {
  try {
    return m46_rmsnorm(handle, request, out_result, false, true, false);
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm(void* handle,
                                                         const PrometheusGemma4E2BM1HeadRmsNormRequest* request,
                                                         PrometheusGemma4E2BM1HeadRmsNormResult* out_result) {
  try {
    return m46_rmsnorm(handle, request, out_result, true, true, true);
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

// reactor_concept_rmsnorm.cpp:157-189 (geometry widened).
int prometheus_reactor_runtime_gemma4e2b_m1_rope(void* handle, const PrometheusGemma4E2BM1RopeRequest* r,
                                                 PrometheusGemma4E2BM1RopeResult* out_result) {
  if (out_result == nullptr) return PROM_ERROR;
  PrometheusGemma4E2BM1RopeResult& out = *out_result;
  try {
    std::memset(&out, 0, sizeof(out));
    out.struct_size = sizeof(out);
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_M46_DETAIL_INVALID_REQUEST;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (r == nullptr || r->struct_size < sizeof(*r) || r->source == nullptr || r->cosine == nullptr ||
        r->sine == nullptr || r->output == nullptr || r->source == r->output || r->cosine == r->output ||
        r->sine == r->output || r->cosine == r->sine || !m1_geometry(r->tokens, r->heads, r->head_width) ||
        r->source_generation == 0 || r->table_generation == 0)
      return PROM_ERROR;
    const uint64_t elems = static_cast<uint64_t>(r->tokens) * r->heads * r->head_width;
    const uint64_t table = static_cast<uint64_t>(r->tokens) * r->head_width;
    if (r->source_element_count != elems || r->output_element_count != elems || r->cosine_element_count != table ||
        r->sine_element_count != table)
      return PROM_ERROR;
    if (!all_finite(r->source, elems) || !all_finite(r->cosine, table) || !all_finite(r->sine, table)) {
      out.detail_code = PROM_M46_DETAIL_NONFINITE_INPUT;
      return PROM_ERROR;
    }
    out.source_hash = hash_u32_bits(r->source, elems);
    out.cosine_hash = hash_u32_bits(r->cosine, table);
    out.sine_hash = hash_u32_bits(r->sine, table);
    if (!rt->available) {
      out.detail_code = PROM_M46_DETAIL_RESOURCE;
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    StageCounts sc;
    if (stage(rt->rin, elems * 4, rt->stream, sc) != cudaSuccess ||
        stage(rt->m1_cos, table * 4, rt->stream, sc) != cudaSuccess ||
        stage(rt->m1_sin, table * 4, rt->stream, sc) != cudaSuccess ||
        stage(rt->rout, elems * 4, rt->stream, sc) != cudaSuccess) {
      out.detail_code = PROM_M46_DETAIL_RESOURCE;
      return PROM_ERROR;
    }
    out.stage = PROM_STAGE_NONE;
    out.detail_code = 0;
    float* din = static_cast<float*>(rt->rin.aligned());
    float* dcos = static_cast<float*>(rt->m1_cos.aligned());
    float* dsin = static_cast<float*>(rt->m1_sin.aligned());
    float* dout = static_cast<float*>(rt->rout.aligned());
    cudaError_t e = cudaMemcpyAsync(din, r->source, elems * 4, cudaMemcpyHostToDevice, rt->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dcos, r->cosine, table * 4, cudaMemcpyHostToDevice, rt->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dsin, r->sine, table * 4, cudaMemcpyHostToDevice, rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_TRANSFER_IN;
      out.detail_code = PROM_M46_DETAIL_SUBMIT;
      return PROM_ERROR;
    }
    e = oct::m1_rope_bf16(din, dcos, dsin, dout, r->tokens, r->heads, r->head_width, rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_SUBMIT;
      out.detail_code = PROM_M46_DETAIL_COMMAND;
      return PROM_ERROR;
    }
    e = cudaMemcpyAsync(r->output, dout, elems * 4, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_TRANSFER_OUT;
      out.detail_code = PROM_M46_DETAIL_COMPLETION_UNCERTAIN;
      return PROM_ERROR;
    }
    out.output_written = 1;
    out.dispatch_count = 1;
    out.output_hash = hash_u32_bits(r->output, elems);
    out.buffer_allocation_count = sc.alloc;
    out.buffer_reuse_count = sc.reuse;
    out.pipeline_create_count = 1;
    return PROM_OK;
  } catch (...) {
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_M46_DETAIL_RESOURCE;
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_gemma4e2b_m1_head_rmsnorm_rope(void* handle,
                                                              const PrometheusGemma4E2BM1HeadRmsNormRopeRequest* r,
                                                              PrometheusGemma4E2BM1HeadRmsNormRopeResult* out_result) {
  if (out_result == nullptr) return PROM_ERROR;
  PrometheusGemma4E2BM1HeadRmsNormRopeResult& out = *out_result;
  try {
    std::memset(&out, 0, sizeof(out));
    out.struct_size = sizeof(out);
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_M46_DETAIL_INVALID_REQUEST;
    if (!head_rope_request_ok(r)) return PROM_ERROR;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    StageCounts sc;
    // one KV head is the K slot, any other head count the Q slot
    return head_rope_locked(rt, r, out, r->heads == 1 ? kSlotKey : kSlotQuery, sc);
  } catch (...) {
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_M46_DETAIL_RESOURCE;
    return PROM_ERROR;
  }
}

// reactor_api.c:507-586: both positional preparations in the requested order,
// then the scores from the two resident slots; only the scores are read back.
int prometheus_reactor_runtime_gemma4e2b_m1_attention_scores(void* handle,
                                                             const PrometheusGemma4E2BM1AttentionScoresRequest* r,
                                                             PrometheusGemma4E2BM1AttentionScoresResult* out_result) {
  if (out_result == nullptr) return PROM_ERROR;
  PrometheusGemma4E2BM1AttentionScoresResult& out = *out_result;
  try {
    std::memset(&out, 0, sizeof(out));
    out.struct_size = sizeof(out);
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_M46_DETAIL_INVALID_REQUEST;
    uint64_t qe = 0, ke = 0, se = 0;
    if (r == nullptr || r->struct_size < sizeof(*r) || r->query_input == nullptr || r->key_input == nullptr ||
        r->query_weight == nullptr || r->key_weight == nullptr || r->cosine == nullptr || r->sine == nullptr ||
        r->scores == nullptr || !m1_geometry(r->tokens, r->query_heads, r->head_width) || r->key_heads != 1 ||
        r->epsilon != 0.000001f || !std::isfinite(r->scale) || r->scale <= 0.f || r->preparation_order > 1 ||
        r->query_input_generation == 0 || r->key_input_generation == 0 || r->query_weight_generation == 0 ||
        r->key_weight_generation == 0 || r->table_generation == 0 || r->query_exact_source_hash == 0 ||
        r->key_exact_source_hash == 0 || !checked_mul(r->tokens, r->query_heads, &qe) ||
        !checked_mul(qe, r->head_width, &qe) || !checked_mul(r->tokens, r->key_heads, &ke) ||
        !checked_mul(ke, r->head_width, &ke) || !checked_mul(r->query_heads, r->tokens, &se) ||
        !checked_mul(se, r->tokens, &se) || r->query_input_element_count != qe || r->key_input_element_count != ke ||
        r->query_weight_element_count != r->head_width || r->key_weight_element_count != r->head_width ||
        r->cosine_element_count != static_cast<uint64_t>(r->tokens) * r->head_width ||
        r->sine_element_count != static_cast<uint64_t>(r->tokens) * r->head_width || r->score_element_count != se)
      return PROM_ERROR;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_ERROR;  // the first preparation's INVALID_HANDLE becomes PROM_ERROR
    std::lock_guard<std::mutex> lock(rt->mu);
    PrometheusGemma4E2BM1HeadRmsNormRopeRequest pos{};
    pos.struct_size = sizeof(pos);
    pos.cosine = r->cosine;
    pos.sine = r->sine;
    pos.cosine_element_count = r->cosine_element_count;
    pos.sine_element_count = r->sine_element_count;
    pos.tokens = r->tokens;
    pos.head_width = r->head_width;
    pos.epsilon = r->epsilon;
    pos.table_generation = r->table_generation;
    StageCounts sc;
    for (uint32_t i = 0; i < 2; ++i) {
      const bool key = r->preparation_order == 0 ? i == 1 : i == 0;
      pos.input = key ? r->key_input : r->query_input;
      pos.weight = key ? r->key_weight : r->query_weight;
      pos.input_element_count = key ? ke : qe;
      pos.weight_element_count = r->head_width;
      pos.heads = key ? r->key_heads : r->query_heads;
      pos.input_generation = key ? r->key_input_generation : r->query_input_generation;
      pos.weight_generation = key ? r->key_weight_generation : r->query_weight_generation;
      pos.exact_source_hash = key ? r->key_exact_source_hash : r->query_exact_source_hash;
      PrometheusGemma4E2BM1HeadRmsNormRopeResult pr{};
      pr.stage = PROM_STAGE_INIT;
      pr.detail_code = PROM_M46_DETAIL_INVALID_REQUEST;
      if (head_rope_locked(rt, &pos, pr, key ? kSlotKey : kSlotQuery, sc) != PROM_OK) {
        out.stage = pr.stage;
        out.detail_code = pr.detail_code;
        out.observed_weight_generation = pr.observed_weight_generation;
        out.requested_weight_generation = pr.requested_weight_generation;
        return PROM_ERROR;
      }
      out.observed_weight_generation = pr.observed_weight_generation;
      out.requested_weight_generation = pr.requested_weight_generation;
      out.positional_dispatch_count = i + 1;
    }
    out.stage = PROM_STAGE_NONE;
    if (stage(rt->m1_scores, se * 4, rt->stream, sc) != cudaSuccess) {
      out.detail_code = PROM_M46_DETAIL_RESOURCE;
      return PROM_ERROR;
    }
    float* dq = static_cast<float*>(rt->m1_q.aligned());
    float* dk = static_cast<float*>(rt->m1_k.aligned());
    float* ds = static_cast<float*>(rt->m1_scores.aligned());
    cudaError_t e = oct::m1_raw_scores(dq, dk, ds, r->tokens, r->query_heads, r->head_width, r->scale, rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_SUBMIT;
      out.detail_code = PROM_M46_DETAIL_COMMAND;
      return PROM_ERROR;
    }
    out.score_dispatch_count = 1;
    ++rt->m1_slot_generation[kSlotScore];
    e = cudaMemcpyAsync(r->scores, ds, se * 4, cudaMemcpyDeviceToHost, rt->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      out.stage = PROM_STAGE_TRANSFER_OUT;
      out.detail_code = PROM_M46_DETAIL_COMPLETION_UNCERTAIN;
      return PROM_ERROR;
    }
    out.detail_code = 0;
    out.score_written = 1;
    out.score_readback_count = 1;
    out.host_detour_count = 0;
    out.query_slot_id = 1;
    out.key_slot_id = 2;
    out.score_slot_id = 3;
    out.query_slot_generation = rt->m1_slot_generation[kSlotQuery];
    out.key_slot_generation = rt->m1_slot_generation[kSlotKey];
    out.score_slot_generation = rt->m1_slot_generation[kSlotScore];
    out.query_byte_range = qe * 4;
    out.key_byte_range = ke * 4;
    out.score_byte_range = se * 4;
    out.score_hash = hash_u64_bits(r->scores, se);
    out.buffer_allocation_count = sc.alloc;
    out.buffer_reuse_count = sc.reuse;
    out.pipeline_create_count = 1;
    out.positional_dispatch_count = 2;
    return PROM_OK;
  } catch (...) {
    out.stage = PROM_STAGE_INIT;
    out.detail_code = PROM_M46_DETAIL_RESOURCE;
    return PROM_ERROR;
  }
}

}  // extern "C"
