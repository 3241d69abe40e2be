// zimage_api.cpp -- the Z-Image model-block executors of the C ABI.
//
// The reference owns one closed model block per runtime
// (internal/prometheus/native/reactor_vulkan_model_block.c:1603-1780) and drives
// it through fixed programs of Vulkan pipelines.  Here the block is the
// library's DiT block (block.cu: tcgen05 3xTF32 products, fused attention,
// fused norm / modulation / gated residual kernels) configured at the Z-Image
// Turbo dimensions:
//
//   noise refiner    1024 image tokens of 3840, 30 heads of 128, SwiGLU 10240,
//                    adaLN 256 -> 4 x 3840 (scale / gate for attention and MLP,
//                    no shift), RMSNorm eps 1e-5, RoPE axes (32, 48, 48) theta
//                    256 on the 32-wide image grid at frame 33
//                    (runCanonicalNoiseRefiner0, zimage/canonical_reference.go:315-480;
//                    CanonicalImageFrame(15), canonical_contract.go:44-51)
//   context refiner  32 caption tokens, the same block unmodulated, token t at
//                    RoPE coordinate (t + 1, 0, 0)
//                    (runCanonicalContextRefiner, zimage/context_refiner_reference.go:229-299)
//
// Validation order, detail codes, the weight manifest (binary16, [in][out],
// lexical order) and the generation rules of the resident chain follow the
// reference; the staged audit programs (M1B / M1C / M1D captures, static
// audits) are not provided.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>

#include "runtime.h"

namespace oct {
namespace rt {

// Shader ids of the create request (reactor_vulkan_model_block.c:31-40).
constexpr uint32_t kShaderResidentIdentity = 23, kShaderNoiseRefiner = 24, kShaderContextRefiner = 25,
                   kShaderMainTransformer = 40;
constexpr uint32_t kTokens = 1024, kContextTokens = 32, kWidth = 3840, kHeads = 30, kHeadDim = 128, kFfn = 10240,
                   kTimestep = 256, kAdaParts = 4;
constexpr uint64_t kImageBf16Bytes = 2ull * kTokens * kWidth;
constexpr uint64_t kContextF32Bytes = 4ull * kContextTokens * kWidth;
// Cache-manifest byte counts (reactor_vulkan_model_block.c:160-183).
constexpr uint64_t kNoiseWeightBytes[13] = {30720ull,    7864320ull,  256ull,      29491200ull, 256ull,
                                            88473600ull, 7680ull,     7680ull,     78643200ull, 78643200ull,
                                            78643200ull, 7680ull,     7680ull};
constexpr uint64_t kContextWeightBytes[11] = {256ull,      29491200ull, 256ull,      88473600ull,
                                              7680ull,     7680ull,     78643200ull, 78643200ull,
                                              78643200ull, 7680ull,     7680ull};

struct ModelBlockState {
  uint64_t id = 0;
  uint32_t family = 0, parameter_set = 0, shader_id = 0, weight_count = 0, step_count = 0;
  uint32_t steps[PROM_MODEL_BLOCK_MAX_STEPS] = {};
  uint64_t aggregate = 0, contract = 0, weight_identity = 0, portfolio = 0, precision = 0, route = 0;
  uint64_t ceiling = 0, ext_in = 0, ext_out = 0, audit_bytes = 0;
  PrometheusModelBlockWeightDeclaration weights[PROM_MODEL_BLOCK_MAX_WEIGHTS] = {};
  bool weights_uploaded = false, output_valid = false, audit_valid = false;
  uint32_t binding_state = 0;
  uint64_t binding_generation = 0, output_generation = 0, resident_input_generation = 0;
  uint64_t plan_identity = 0, replay_identity = 0;
  uint64_t execution_count = 0, weight_upload_count = 0, last_execution_ns = 0, submits = 0;
  uint64_t gpu_compute_ns = 0, gpu_ingress_ns = 0, gpu_readback_ns = 0, staging_ns = 0;
  uint64_t cold_allocations = 0;
  int32_t last_detail = 0;
  std::unique_ptr<oct::Block> block;     // the refiners
  DevBuf raw_weights;                    // family 0: the uploaded payloads, held as given
  DevBuf staging16;                      // 2-byte payload staging (activations and weights)
  DevBuf x, pinned, y, audit, temb, wstage;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  ~ModelBlockState() {
    for (DevBuf* b : {&raw_weights, &staging16, &x, &pinned, &y, &audit, &temb, &wstage}) b->release();
    if (e0 != nullptr) cudaEventDestroy(e0);
    if (e1 != nullptr) cudaEventDestroy(e1);
  }
  bool refiner() const {
    return family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO || family == PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO;
  }
  uint32_t tokens() const { return family == PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO ? kContextTokens : kTokens; }
};

void destroy_model_block(Runtime* rt) {
  delete rt->model_block;
  rt->model_block = nullptr;
}

}  // namespace rt
}  // namespace oct

namespace {

using namespace oct::rt;

uint64_t fnv_u64(uint64_t h, uint64_t v) {
  for (unsigned b = 0; b < 8; ++b) {
    h ^= (v >> (8 * b)) & 0xffu;
    h *= 1099511628211ull;
  }
  return h;
}

bool add_bytes(uint64_t* total, uint64_t v) {
  if (v > UINT64_MAX - *total) return false;
  *total += v;
  return true;
}

uint64_t held_bytes(const ModelBlockState* b) {
  uint64_t n = 0;
  for (const DevBuf* d : {&b->raw_weights, &b->staging16, &b->x, &b->pinned, &b->y, &b->audit, &b->temb, &b->wstage})
    n += d->cap;
  return n;
}

// prom_model_block_fill_evidence (reactor_vulkan_model_block.c:259-370) over this block.
void fill_evidence(const ModelBlockState* b, int32_t detail, PrometheusModelBlockEvidence* out) {
  if (out == nullptr) return;
  std::memset(out, 0, sizeof(*out));
  out->struct_size = sizeof(*out);
  out->detail_code = detail;
  if (b == nullptr) return;
  uint64_t declared = 0;
  for (uint32_t i = 0; i < b->weight_count; ++i) declared += b->weights[i].byte_count;
  out->created = 1;
  out->weights_uploaded = b->weights_uploaded ? 1u : 0u;
  out->output_valid = b->output_valid ? 1u : 0u;
  out->audit_valid = b->audit_valid ? 1u : 0u;
  out->fixed_step_count = b->step_count;
  out->weight_count = b->weight_count;
  // The refiners hold their weights widened and split for the tensor cores inside
  // the DiT block; family 0 holds the payloads as given.
  out->persistent_bytes = b->block ? declared * 4 : b->raw_weights.cap;
  out->reusable_bytes = held_bytes(b) - b->raw_weights.cap - b->audit.cap;
  out->audit_bytes = b->audit.cap;
  out->external_bytes = b->ext_in + b->ext_out;
  out->total_committed_bytes = out->persistent_bytes + out->reusable_bytes + out->audit_bytes;
  out->peak_plan_bytes = out->total_committed_bytes;
  out->cold_buffer_allocation_count = b->cold_allocations;
  out->pipeline_create_count = b->block ? 12 : 1;
  out->weight_upload_count = b->weight_upload_count;
  out->execution_count = b->execution_count;
  out->last_execution_ns = b->last_execution_ns;
  out->execution_plan_identity = b->plan_identity;
  out->replay_identity = b->replay_identity;
  out->assembly_family = b->family;
  out->parameter_set = b->parameter_set;
  out->binding_state = b->binding_state;
  out->parameter_set_aggregate_identity = b->aggregate;
  out->binding_generation = b->binding_generation;
  out->output_generation = b->output_generation;
  out->descriptor_generation = b->binding_generation;
  out->gpu_total_ns = b->gpu_compute_ns + b->gpu_ingress_ns + b->gpu_readback_ns;
  out->gpu_compute_ns = b->gpu_compute_ns;
  out->gpu_ingress_transfer_ns = b->gpu_ingress_ns;
  out->gpu_readback_ns = b->gpu_readback_ns;
  out->last_staging_memcpy_ns = b->staging_ns;
}

void mark_failure(ModelBlockState* b, int32_t detail) {
  if (b == nullptr) return;
  b->output_valid = false;
  b->audit_valid = false;
  b->last_detail = detail;
}

bool steps_exact(const PrometheusModelBlockCreateRequest* r) {
  if (r->step_count != PROM_MODEL_BLOCK_MAX_STEPS) return false;
  for (uint32_t i = 0; i < PROM_MODEL_BLOCK_MAX_STEPS; ++i)
    if (r->steps[i] != i + 1) return false;  // bind pipeline .. output copy (reactor_vulkan_model_block.c:170-178)
  return true;
}

// prom_model_block_validate_create_request (reactor_vulkan_model_block.c:393-477).
bool create_request_ok(const PrometheusModelBlockCreateRequest* r) {
  if (r == nullptr || r->struct_size != sizeof(*r) || r->model_contract_identity == 0 || r->weight_identity == 0 ||
      r->shader_portfolio_identity == 0 || r->precision_policy_identity == 0 || r->capability_route_identity == 0 ||
      r->memory_ceiling_bytes == 0 ||
      (r->shader_id != kShaderResidentIdentity && r->shader_id != kShaderNoiseRefiner &&
       r->shader_id != kShaderContextRefiner && r->shader_id != kShaderMainTransformer) ||
      r->weight_count == 0 || r->weight_count > PROM_MODEL_BLOCK_MAX_WEIGHTS || r->audit_bytes == 0 ||
      r->external_input_bytes % 4 || r->external_output_bytes % 4 || r->audit_bytes % 4 || !steps_exact(r))
    return false;
  if (r->shader_id != kShaderMainTransformer && r->external_input_bytes == 0) return false;
  if (r->shader_id == kShaderResidentIdentity && r->external_output_bytes == 0) return false;
  const uint64_t nr_aggregate[2] = {OCT_B200_ZIMAGE_NOISE_REFINER0_AGGREGATE, OCT_B200_ZIMAGE_NOISE_REFINER1_AGGREGATE};
  const uint64_t cr_aggregate[2] = {OCT_B200_ZIMAGE_CONTEXT_REFINER0_AGGREGATE,
                                    OCT_B200_ZIMAGE_CONTEXT_REFINER1_AGGREGATE};
  if (r->assembly_family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO &&
      ((r->parameter_set != PROM_NOISE_REFINER_PARAMETER_SET_0 && r->parameter_set != PROM_NOISE_REFINER_PARAMETER_SET_1) ||
       r->parameter_set_aggregate_identity != nr_aggregate[r->parameter_set - 1] ||
       r->shader_id != kShaderNoiseRefiner))
    return false;
  if (r->assembly_family == PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO &&
      ((r->parameter_set != PROM_CONTEXT_REFINER_PARAMETER_SET_0 &&
        r->parameter_set != PROM_CONTEXT_REFINER_PARAMETER_SET_1) ||
       r->parameter_set_aggregate_identity != cr_aggregate[r->parameter_set - 1] ||
       r->shader_id != kShaderContextRefiner))
    return false;
  // The 30-layer main transformer and its compiled-model sessions are not provided.
  if (r->assembly_family == PROM_MAIN_TRANSFORMER_FAMILY_Z_IMAGE_TURBO || r->shader_id == kShaderMainTransformer)
    return false;
  if (r->assembly_family != 0 && r->assembly_family != PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO &&
      r->assembly_family != PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO)
    return false;
  if (r->assembly_family == 0 && (r->parameter_set != 0 || r->parameter_set_aggregate_identity != 0)) return false;
  // shader 24 is the noise refiner's closed program; shader 25 only the context refiner's
  if (r->shader_id == kShaderNoiseRefiner &&
      (r->assembly_family != PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO || r->weight_count != 13 ||
       r->external_input_bytes != kImageBf16Bytes || r->external_output_bytes != 0 ||
       r->audit_bytes > OCT_B200_ZIMAGE_AUDIT_ARENA_BYTES))
    return false;
  if (r->shader_id == kShaderContextRefiner &&
      (r->assembly_family != PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO || r->weight_count != 11 ||
       r->external_input_bytes != kContextF32Bytes || r->external_output_bytes != 0 ||
       r->audit_bytes > OCT_B200_ZIMAGE_AUDIT_ARENA_BYTES))
    return false;
  uint64_t weight_total = 0, total = 0;
  for (uint32_t i = 0; i < r->weight_count; ++i) {
    const PrometheusModelBlockWeightDeclaration& w = r->weights[i];
    if (w.content_identity == 0 || w.layout_identity == 0 || w.byte_count == 0 || !add_bytes(&weight_total, w.byte_count))
      return false;
    if (r->shader_id == kShaderNoiseRefiner && w.byte_count != kNoiseWeightBytes[i]) return false;
    if (r->shader_id == kShaderContextRefiner && w.byte_count != kContextWeightBytes[i]) return false;
  }
  if (r->shader_id == kShaderNoiseRefiner)
    return add_bytes(&(total = weight_total), 128ull << 20) && total <= r->memory_ceiling_bytes;
  if (r->shader_id == kShaderContextRefiner)
    return add_bytes(&(total = weight_total), 16ull << 20) && total <= r->memory_ceiling_bytes;
  return add_bytes(&total, weight_total) && add_bytes(&total, r->external_input_bytes) &&
         add_bytes(&total, r->external_input_bytes) && add_bytes(&total, r->external_output_bytes) &&
         add_bytes(&total, r->external_output_bytes) && add_bytes(&total, r->audit_bytes) &&
         add_bytes(&total, r->audit_bytes) && add_bytes(&total, weight_total) && total <= r->memory_ceiling_bytes;
}

uint64_t plan_identity(const ModelBlockState* b) {
  uint64_t h = 1469598103934665603ull;
  for (uint64_t v : {b->contract, uint64_t(b->family), uint64_t(b->parameter_set), b->aggregate, b->weight_identity,
                     b->portfolio, b->precision, b->route, uint64_t(b->shader_id), b->ext_in, b->ext_out,
                     b->audit_bytes})
    h = fnv_u64(h, v);
  for (uint32_t i = 0; i < b->weight_count; ++i) {
    h = fnv_u64(h, b->weights[i].content_identity);
    h = fnv_u64(h, b->weights[i].layout_identity);
    h = fnv_u64(h, b->weights[i].byte_count);
  }
  for (uint32_t i = 0; i < b->step_count; ++i) h = fnv_u64(h, b->steps[i]);
  return h;
}

cudaError_t stage_counted(ModelBlockState* b, DevBuf& buf, uint64_t bytes, cudaStream_t s) {
  if (buf.raw != nullptr && bytes <= buf.cap) return cudaSuccess;
  ++b->cold_allocations;
  return buf.ensure(bytes, s);
}

// One refiner weight set into the DiT block: binary16 payloads (lexical order)
// widened on the device into the block's slots.  The noise refiner's 4 x 3840
// adaLN projection fills the first four parts of the block's 6 x 3840 (the
// shift parts stay zero); W1 and W3 become the block's [3840][2 x 10240] W13.
int load_refiner_weights(Runtime* rt, ModelBlockState* b, const PrometheusModelBlockWeightUpload* up) {
  oct::Block& blk = *b->block;
  cudaStream_t s = rt->stream;
  const bool noise = b->family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO;
  const uint32_t base = noise ? 2 : 0;  // the context package has no adaLN tensors
  uint64_t max16 = 0;
  for (uint32_t i = 0; i < b->weight_count; ++i) max16 = std::max(max16, up[i].byte_count);
  const uint64_t stage_floats = 2ull * kWidth * kFfn;  // the largest slot: W13
  if (stage_counted(b, b->staging16, max16, s) != cudaSuccess ||
      stage_counted(b, b->wstage, stage_floats * 4, s) != cudaSuccess)
    return PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED;
  void* d16 = b->staging16.aligned();
  float* w = static_cast<float*>(b->wstage.aligned());
  const auto t0 = Clock::now();
  auto upload16 = [&](uint32_t i) {
    return cudaMemcpyAsync(d16, up[i].bytes, up[i].byte_count, cudaMemcpyHostToDevice, s) == cudaSuccess;
  };
  // widen binding i ([rows][cols]) into the staging matrix at column col0 of width ld
  auto widen = [&](uint32_t i, uint32_t rows, uint32_t cols, uint64_t ld, uint32_t col0) {
    return upload16(i) && oct::widen_f16(d16, rows, cols, w, ld, col0, s) == cudaSuccess;
  };
  auto set = [&](uint32_t slot, uint64_t count) {
    return blk.set_weight(slot, w, count, true) == 0;  // synchronises the stream
  };
  bool ok = true;
  if (noise) {
    const uint64_t parts6 = 6ull * kWidth;
    ok = ok && cudaMemsetAsync(w, 0, parts6 * 4, s) == cudaSuccess && widen(0, 1, kAdaParts * kWidth, parts6, 0) &&
         set(oct::kDitAdaB, parts6);
    ok = ok && cudaMemsetAsync(w, 0, kTimestep * parts6 * 4, s) == cudaSuccess &&
         widen(1, kTimestep, kAdaParts * kWidth, parts6, 0) && set(oct::kDitAdaW, kTimestep * parts6);
  }
  ok = ok && widen(base + 0, 1, kHeadDim, kHeadDim, 0) && set(oct::kDitKNorm, kHeadDim);
  ok = ok && widen(base + 1, kWidth, kWidth, kWidth, 0) && set(oct::kDitWo, 1ull * kWidth * kWidth);
  ok = ok && widen(base + 2, 1, kHeadDim, kHeadDim, 0) && set(oct::kDitQNorm, kHeadDim);
  ok = ok && widen(base + 3, kWidth, 3 * kWidth, 3 * kWidth, 0) && set(oct::kDitWqkv, 3ull * kWidth * kWidth);
  ok = ok && widen(base + 4, 1, kWidth, kWidth, 0) && set(oct::kDitAttnNorm1, kWidth);
  ok = ok && widen(base + 5, 1, kWidth, kWidth, 0) && set(oct::kDitAttnNorm2, kWidth);
  ok = ok && widen(base + 6, kWidth, kFfn, 2 * kFfn, 0) && cudaStreamSynchronize(s) == cudaSuccess &&
       widen(base + 8, kWidth, kFfn, 2 * kFfn, kFfn) && set(oct::kDitW13, 2ull * kWidth * kFfn);
  ok = ok && widen(base + 7, kFfn, kWidth, kWidth, 0) && set(oct::kDitW2, 1ull * kFfn * kWidth);
  ok = ok && widen(base + 9, 1, kWidth, kWidth, 0) && set(oct::kDitFfnNorm1, kWidth);
  ok = ok && widen(base + 10, 1, kWidth, kWidth, 0) && set(oct::kDitFfnNorm2, kWidth);
  ok = ok && cudaStreamSynchronize(s) == cudaSuccess;
  b->staging_ns = ns_since(t0);
  if (!ok) {
    (void)cudaGetLastError();
    return PROM_MODEL_BLOCK_DETAIL_UPLOAD_FAILED;
  }
  b->weight_upload_count += b->weight_count;
  return 0;
}

// Validates a weight payload set against the declarations (binding order, bytes, identities).
bool uploads_match(const ModelBlockState* b, const PrometheusModelBlockWeightUpload* up, uint32_t count) {
  if (up == nullptr || count != b->weight_count) return false;
  for (uint32_t i = 0; i < count; ++i)
    if (up[i].binding_index != i || up[i].bytes == nullptr || up[i].byte_count != b->weights[i].byte_count ||
        up[i].content_identity != b->weights[i].content_identity ||
        up[i].layout_identity != b->weights[i].layout_identity)
      return false;
  return true;
}

ModelBlockState* find_block(Runtime* rt, uint64_t id) {
  ModelBlockState* b = rt->model_block;
  return b != nullptr && b->id == id ? b : nullptr;
}

// Runs the refiner on b->x (or the pinned predecessor) into b->y; timestep
// embedding in b->temb for the noise refiner.
int run_refiner(Runtime* rt, ModelBlockState* b, const float* input) {
  cudaEventRecord(b->e0, rt->stream);
  b->block->set_stream(rt->stream);
  const bool noise = b->family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO;
  const int rc = b->block->forward(input, static_cast<float*>(b->y.aligned()), 1, nullptr,
                                   noise ? static_cast<const float*>(b->temb.aligned()) : nullptr);
  cudaEventRecord(b->e1, rt->stream);
  if (rc != 0 || cudaStreamSynchronize(rt->stream) != cudaSuccess || b->block->read_status() != 0) {
    (void)cudaGetLastError();
    return PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN;
  }
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, b->e0, b->e1) == cudaSuccess)
    b->gpu_compute_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
  ++b->submits;
  return 0;
}

int create_locked(Runtime* rt, const PrometheusModelBlockCreateRequest* r, uint64_t* out_id,
                  PrometheusModelBlockEvidence* ev) {
  if (rt->model_block != nullptr) {
    fill_evidence(rt->model_block, PROM_MODEL_BLOCK_DETAIL_ALREADY_CREATED, ev);
    return PROM_ERROR;
  }
  if (!rt->available) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED, ev);
    return PROM_ERROR;
  }
  std::unique_ptr<ModelBlockState> b(new ModelBlockState());
  b->family = r->assembly_family;
  b->parameter_set = r->parameter_set;
  b->aggregate = r->parameter_set_aggregate_identity;
  b->contract = r->model_contract_identity;
  b->weight_identity = r->weight_identity;
  b->portfolio = r->shader_portfolio_identity;
  b->precision = r->precision_policy_identity;
  b->route = r->capability_route_identity;
  b->ceiling = r->memory_ceiling_bytes;
  b->ext_in = r->external_input_bytes;
  b->ext_out = r->external_output_bytes;
  b->audit_bytes = r->audit_bytes;
  b->shader_id = r->shader_id;
  b->weight_count = r->weight_count;
  b->step_count = r->step_count;
  std::memcpy(b->steps, r->steps, sizeof(b->steps));
  std::memcpy(b->weights, r->weights, sizeof(b->weights));
  if (cudaEventCreate(&b->e0) != cudaSuccess || cudaEventCreate(&b->e1) != cudaSuccess) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED, ev);
    return PROM_ERROR;
  }
  cudaStream_t s = rt->stream;
  if (b->refiner()) {
    oct::BlockDims d;
    d.family = oct::kDit;
    d.hidden = kWidth;
    d.heads = d.kv_heads = kHeads;
    d.head_dim = kHeadDim;
    d.ffn = kFfn;
    d.seq_len = b->tokens();
    d.max_batch = 1;
    d.eps = 1e-5f;  // canonicalNormRows (canonical_reference.go:177-190)
    d.rope_base = 256.f;
    d.grid_w = 32;
    const bool context = b->family == PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO;
    d.rope_frame = context ? 1 : 33;
    d.rope_text = context ? 1 : 0;
    d.unmodulated = context ? 1 : 0;
    b->block.reset(new (std::nothrow) oct::Block());
    const uint64_t act = 4ull * b->tokens() * kWidth;
    if (!b->block || b->block->init(d, nullptr, s) != 0 || stage_counted(b.get(), b->x, act, s) != cudaSuccess ||
        stage_counted(b.get(), b->pinned, act, s) != cudaSuccess ||
        stage_counted(b.get(), b->y, act, s) != cudaSuccess ||
        stage_counted(b.get(), b->temb, 4ull * kTimestep, s) != cudaSuccess ||
        stage_counted(b.get(), b->staging16, context ? act : kImageBf16Bytes, s) != cudaSuccess) {
      (void)cudaGetLastError();
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED, ev);
      return PROM_ERROR;
    }
  } else {
    uint64_t total = 0;
    for (uint32_t i = 0; i < b->weight_count; ++i) total += b->weights[i].byte_count;
    if (stage_counted(b.get(), b->raw_weights, total, s) != cudaSuccess ||
        stage_counted(b.get(), b->x, b->ext_in, s) != cudaSuccess ||
        stage_counted(b.get(), b->y, b->ext_out, s) != cudaSuccess ||
        stage_counted(b.get(), b->audit, b->audit_bytes, s) != cudaSuccess) {
      (void)cudaGetLastError();
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED, ev);
      return PROM_ERROR;
    }
  }
  b->id = rt->next_model_block_id++;
  b->plan_identity = plan_identity(b.get());
  *out_id = b->id;
  rt->model_block = b.release();
  fill_evidence(rt->model_block, 0, ev);
  return PROM_OK;
}

int upload_locked(Runtime* rt, ModelBlockState* b, const PrometheusModelBlockWeightUpload* up, uint32_t count,
                  PrometheusModelBlockEvidence* ev) {
  if (b->weights_uploaded || count != b->weight_count || (rt->test_flags & PROM_TESTCFG_FAIL_UPLOAD)) {
    mark_failure(b, (rt->test_flags & PROM_TESTCFG_FAIL_UPLOAD) ? PROM_MODEL_BLOCK_DETAIL_UPLOAD_FAILED
                                                                : PROM_MODEL_BLOCK_DETAIL_WEIGHT_MISMATCH);
    fill_evidence(b, b->last_detail, ev);
    return PROM_ERROR;
  }
  if (!uploads_match(b, up, count)) {
    mark_failure(b, PROM_MODEL_BLOCK_DETAIL_WEIGHT_MISMATCH);
    fill_evidence(b, b->last_detail, ev);
    return PROM_ERROR;
  }
  int d = 0;
  if (b->block) {
    d = load_refiner_weights(rt, b, up);
  } else {
    uint64_t off = 0;
    for (uint32_t i = 0; i < count && d == 0; ++i) {
      if (cudaMemcpyAsync(static_cast<char*>(b->raw_weights.aligned()) + off, up[i].bytes, up[i].byte_count,
                          cudaMemcpyHostToDevice, rt->stream) != cudaSuccess)
        d = PROM_MODEL_BLOCK_DETAIL_UPLOAD_FAILED;
      off += up[i].byte_count;
    }
    if (d == 0 && cudaStreamSynchronize(rt->stream) != cudaSuccess) d = PROM_MODEL_BLOCK_DETAIL_UPLOAD_FAILED;
    if (d == 0) b->weight_upload_count += count;
  }
  if (d != 0) {
    (void)cudaGetLastError();
    mark_failure(b, d);
    fill_evidence(b, d, ev);
    return PROM_ERROR;
  }
  b->weights_uploaded = true;
  b->binding_state = PROM_NOISE_REFINER_BINDING_BOUND;
  ++b->binding_generation;
  b->output_valid = b->audit_valid = false;
  b->resident_input_generation = 0;
  b->replay_identity = 0;
  b->last_detail = 0;
  fill_evidence(b, 0, ev);
  return PROM_OK;
}

// The closed resident-chain executes of both refiners: external ingress (BF16
// image + timestep, or FP32 context) or the resident predecessor output.
int refiner_execute(Runtime* rt, ModelBlockState* b, uint32_t family, uint32_t required_set, const void* input,
                    const void* timestep, uint64_t input_generation, uint64_t input_identity,
                    uint64_t output_identity, bool resident, PrometheusModelBlockEvidence* ev) {
  const bool first_resident = resident && b->resident_input_generation == 0;
  if (b->family != family || b->parameter_set != required_set || !b->weights_uploaded ||
      b->binding_state != PROM_NOISE_REFINER_BINDING_BOUND ||
      (resident && (input_generation == 0 || (first_resident ? input_generation != b->output_generation
                                                             : input_generation != b->resident_input_generation)))) {
    // the external noise-refiner ingress reports a parameter-set mismatch and leaves
    // the block as it was (reactor_vulkan_model_block.c:2223-2228); the resident and
    // context executes mark the output stale (:3321-3330, 2541-2549)
    if (!resident && family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO) {
      fill_evidence(b, PROM_MODEL_BLOCK_DETAIL_PARAMETER_SET_MISMATCH, ev);
      return PROM_ERROR;
    }
    mark_failure(b, PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT);
    fill_evidence(b, PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT, ev);
    return PROM_ERROR;
  }
  const auto t0 = Clock::now();
  b->output_valid = b->audit_valid = false;
  cudaStream_t s = rt->stream;
  const uint64_t act = static_cast<uint64_t>(b->tokens()) * kWidth;
  float* x = static_cast<float*>(b->x.aligned());
  float* pinned = static_cast<float*>(b->pinned.aligned());
  cudaError_t e = cudaSuccess;
  const float* in = x;
  if (!resident) {
    b->resident_input_generation = 0;  // an external ingress starts a new chain
    cudaEventRecord(b->e0, s);
    if (family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO) {
      e = cudaMemcpyAsync(b->staging16.aligned(), input, act * 2, cudaMemcpyHostToDevice, s);
      if (e == cudaSuccess) e = oct::widen_bf16(b->staging16.aligned(), x, act, s);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(b->staging16.aligned(), timestep, 2ull * kTimestep, cudaMemcpyHostToDevice, s);
      if (e == cudaSuccess) e = oct::widen_bf16(b->staging16.aligned(), static_cast<float*>(b->temb.aligned()), kTimestep, s);
    } else {
      e = cudaMemcpyAsync(x, input, act * 4, cudaMemcpyHostToDevice, s);
    }
    cudaEventRecord(b->e1, s);
    float ms = 0.f;
    if (e == cudaSuccess && cudaStreamSynchronize(s) == cudaSuccess &&
        cudaEventElapsedTime(&ms, b->e0, b->e1) == cudaSuccess)
      b->gpu_ingress_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
  } else {
    // the predecessor's output becomes this chain's pinned input
    if (first_resident)
      e = cudaMemcpyAsync(pinned, b->y.aligned(), act * 4, cudaMemcpyDeviceToDevice, s);
    in = pinned;
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    mark_failure(b, PROM_MODEL_BLOCK_DETAIL_INGRESS_DISPATCH_FAILED);
    fill_evidence(b, b->last_detail, ev);
    return PROM_ERROR;
  }
  const int d = run_refiner(rt, b, in);
  if (d != 0) {
    mark_failure(b, d);
    fill_evidence(b, d, ev);
    return PROM_ERROR;
  }
  b->output_valid = true;
  b->output_generation += 1;
  if (first_resident) b->resident_input_generation = input_generation;
  b->execution_count += family == PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO ? 3 : 1;
  b->last_execution_ns = ns_since(t0);
  b->replay_identity = fnv_u64(fnv_u64(b->plan_identity, resident ? input_generation : input_identity),
                               output_identity);
  b->replay_identity = fnv_u64(b->replay_identity, b->aggregate);
  b->last_detail = 0;
  fill_evidence(b, 0, ev);
  return PROM_OK;
}

int audit_final(Runtime* rt, ModelBlockState* b, uint32_t family, const PrometheusNoiseRefinerFinalAuditRequest* r,
                PrometheusModelBlockEvidence* ev) {
  const uint64_t act = static_cast<uint64_t>(b->tokens()) * kWidth;
  if (b->family != family || !b->output_valid || b->output_generation != r->required_output_generation ||
      r->output_element_capacity < act) {
    const int32_t d = r->output_element_capacity < act ? PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST
                                                      : PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT;
    if (d == PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT) mark_failure(b, d);
    fill_evidence(d == PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT ? b : nullptr, d, ev);
    return PROM_ERROR;
  }
  cudaEventRecord(b->e0, rt->stream);
  cudaError_t e = cudaMemcpyAsync(r->output, b->y.aligned(), act * 4, cudaMemcpyDeviceToHost, rt->stream);
  cudaEventRecord(b->e1, rt->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    mark_failure(b, PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED);
    fill_evidence(b, b->last_detail, ev);
    return PROM_ERROR;
  }
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, b->e0, b->e1) == cudaSuccess)
    b->gpu_readback_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
  b->audit_valid = true;
  b->replay_identity = fnv_u64(b->replay_identity, r->output_identity);
  b->last_detail = 0;
  fill_evidence(b, 0, ev);
  return PROM_OK;
}

// The closed create of the context refiner from the lock's descriptor
// (reactor_vulkan_model_block.c:2305-2367): block 0 only, then its 11 uploads.
const uint64_t* context_descriptor(uint64_t lock, uint32_t local_id, uint32_t* parameter_set) {
  static const uint64_t aggregates[2] = {OCT_B200_ZIMAGE_CONTEXT_REFINER0_AGGREGATE,
                                         OCT_B200_ZIMAGE_CONTEXT_REFINER1_AGGREGATE};
  if (lock != OCT_B200_ZIMAGE_TURBO_LOCK_ID || local_id > 1) return nullptr;
  *parameter_set = local_id == 0 ? PROM_CONTEXT_REFINER_PARAMETER_SET_0 : PROM_CONTEXT_REFINER_PARAMETER_SET_1;
  return &aggregates[local_id];
}

int rebind_locked(Runtime* rt, ModelBlockState* b, uint32_t family, uint32_t from_set, uint32_t to_set,
                  uint64_t aggregate, const PrometheusModelBlockWeightUpload* up, uint32_t count,
                  PrometheusModelBlockEvidence* ev) {
  if (b->family != family || b->parameter_set != from_set || !b->weights_uploaded) {
    fill_evidence(b, PROM_MODEL_BLOCK_DETAIL_REBIND_FAILED, ev);
    return PROM_ERROR;
  }
  const uint64_t* sizes = family == PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO ? kContextWeightBytes : kNoiseWeightBytes;
  for (uint32_t i = 0; i < count; ++i)
    if (up[i].binding_index != i || up[i].bytes == nullptr || up[i].content_identity == 0 ||
        up[i].layout_identity == 0 || up[i].byte_count != sizes[i]) {
      fill_evidence(b, PROM_MODEL_BLOCK_DETAIL_WEIGHT_MISMATCH, ev);
      return PROM_ERROR;
    }
  const int d = load_refiner_weights(rt, b, up);
  if (d != 0) {
    mark_failure(b, d);
    fill_evidence(b, d, ev);
    return PROM_ERROR;
  }
  for (uint32_t i = 0; i < count; ++i) {
    b->weights[i].content_identity = up[i].content_identity;
    b->weights[i].layout_identity = up[i].layout_identity;
  }
  ++b->binding_generation;
  b->output_valid = b->audit_valid = false;  // the resident output stays, as the chain's next input
  b->resident_input_generation = 0;
  b->replay_identity = 0;
  b->parameter_set = to_set;
  b->aggregate = aggregate;
  b->last_detail = 0;
  fill_evidence(b, 0, ev);
  return PROM_OK;
}

}  // namespace

extern "C" {

int prometheus_reactor_runtime_model_block_create(void* handle, const PrometheusModelBlockCreateRequest* request,
                                                  uint64_t* out_block_id, PrometheusModelBlockEvidence* out_evidence) {
  try {
    if (out_block_id != nullptr) *out_block_id = 0;
    Runtime* rt = lookup(handle);
    if (!create_request_ok(request) || out_block_id == nullptr || rt == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    return create_locked(rt, request, out_block_id, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_model_block_upload_weights(void* handle, uint64_t block_id,
                                                          const PrometheusModelBlockWeightUpload* uploads,
                                                          uint32_t upload_count,
                                                          PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || uploads == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return upload_locked(rt, b, uploads, upload_count, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_UPLOAD_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

// reactor_vulkan_model_block.c:1884-1953: the identity block over host buffers.
int prometheus_reactor_runtime_model_block_execute(void* handle, uint64_t block_id,
                                                   const PrometheusModelBlockExecuteRequest* r,
                                                   PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->struct_size != sizeof(*r) || r->input == nullptr ||
        r->output == nullptr || r->input_identity == 0 || r->audit_enabled > 1 || r->element_count == 0 ||
        r->element_count > UINT64_MAX / 4) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    const uint64_t bytes = r->element_count * 4;
    if (!b->weights_uploaded || b->refiner() || bytes != b->ext_in || bytes != b->ext_out ||
        r->element_count > 4194304u) {
      mark_failure(b, PROM_MODEL_BLOCK_DETAIL_STALE_OUTPUT);
      fill_evidence(b, b->last_detail, out_evidence);
      return PROM_ERROR;
    }
    if (r->audit_enabled != 0 && (r->audit_output == nullptr || r->audit_element_capacity * 4 < b->audit_bytes)) {
      mark_failure(b, PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED);
      fill_evidence(b, b->last_detail, out_evidence);
      return PROM_ERROR;
    }
    const auto t0 = Clock::now();
    b->output_valid = b->audit_valid = false;
    cudaStream_t s = rt->stream;
    const uint64_t audit_elems = b->audit_bytes / 4;
    const uint64_t copied = std::min<uint64_t>(audit_elems, r->element_count);
    cudaEventRecord(b->e0, s);
    cudaError_t e = cudaMemcpyAsync(b->x.aligned(), r->input, bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b->y.aligned(), b->x.aligned(), bytes, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess && r->audit_enabled != 0) {
      e = cudaMemsetAsync(b->audit.aligned(), 0, b->audit_bytes, s);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(b->audit.aligned(), b->x.aligned(), copied * 4, cudaMemcpyDeviceToDevice, s);
    }
    cudaEventRecord(b->e1, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess || (rt->test_flags & PROM_TESTCFG_FAIL_DOWNLOAD)) {
      (void)cudaGetLastError();
      mark_failure(b, e != cudaSuccess ? PROM_MODEL_BLOCK_DETAIL_QUEUE_SUBMIT_FAILED : PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED);
      fill_evidence(b, b->last_detail, out_evidence);
      return PROM_ERROR;
    }
    e = cudaMemcpyAsync(r->output, b->y.aligned(), bytes, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && r->audit_enabled != 0)
      e = cudaMemcpyAsync(r->audit_output, b->audit.aligned(), b->audit_bytes, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      mark_failure(b, PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED);
      fill_evidence(b, b->last_detail, out_evidence);
      return PROM_ERROR;
    }
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, b->e0, b->e1) == cudaSuccess)
      b->gpu_compute_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1.0e6);
    b->output_valid = true;
    b->audit_valid = r->audit_enabled != 0;
    b->execution_count += 1;
    b->last_execution_ns = ns_since(t0);
    b->replay_identity = fnv_u64(fnv_u64(b->plan_identity, r->input_identity), r->audit_enabled);
    b->last_detail = 0;
    fill_evidence(b, 0, out_evidence);
    return PROM_OK;
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN, out_evidence);
    return PROM_ERROR;
  }
}

}  // extern "C"

namespace {

// reactor_vulkan_model_block.c:2204-2226: request checks of the external executes.
bool noise_request_ok(const PrometheusNoiseRefiner0ExecuteRequest* r) {
  return r != nullptr && r->struct_size == sizeof(*r) && r->model_input_bf16 != nullptr &&
         r->timestep_bf16 != nullptr && r->model_input_bytes == kImageBf16Bytes &&
         r->timestep_bytes == 2ull * kTimestep && r->input_identity != 0 && r->timestep_identity != 0 &&
         r->output_identity != 0 && r->audit_enabled == 0;
}

int noise_execute(void* handle, uint64_t block_id, const PrometheusNoiseRefiner0ExecuteRequest* r, uint32_t set,
                  PrometheusModelBlockEvidence* ev) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || !noise_request_ok(r)) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, ev);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = rt->model_block;
    if (b == nullptr || b->id != block_id) {
      fill_evidence(b, PROM_MODEL_BLOCK_DETAIL_PARAMETER_SET_MISMATCH, ev);
      return PROM_ERROR;
    }
    return refiner_execute(rt, b, PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO, set, r->model_input_bf16,
                           r->timestep_bf16, 0, r->input_identity, r->output_identity, false, ev);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN, ev);
    return PROM_ERROR;
  }
}

}  // namespace

extern "C" {

int prometheus_reactor_runtime_noise_refiner0_execute(void* handle, uint64_t block_id,
                                                      const PrometheusNoiseRefiner0ExecuteRequest* request,
                                                      PrometheusModelBlockEvidence* out_evidence) {
  return noise_execute(handle, block_id, request, PROM_NOISE_REFINER_PARAMETER_SET_0, out_evidence);
}

int prometheus_reactor_runtime_noise_refiner1_execute(void* handle, uint64_t block_id,
                                                      const PrometheusNoiseRefiner1ExecuteRequest* request,
                                                      PrometheusModelBlockEvidence* out_evidence) {
  return noise_execute(handle, block_id, request, PROM_NOISE_REFINER_PARAMETER_SET_1, out_evidence);
}

// reactor_vulkan_model_block.c:1831-1882.
int prometheus_reactor_runtime_noise_refiner_rebind(void* handle, uint64_t block_id,
                                                    const PrometheusNoiseRefinerRebindRequest* r,
                                                    PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->struct_size != sizeof(*r) || r->uploads == nullptr ||
        r->upload_count != PROM_MODEL_BLOCK_MAX_WEIGHTS || r->lock_identity != OCT_B200_ZIMAGE_TURBO_LOCK_ID ||
        r->model_local_block_id != 1) {  // only block 1's descriptor is a rebind target
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return rebind_locked(rt, b, PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO, PROM_NOISE_REFINER_PARAMETER_SET_0,
                         PROM_NOISE_REFINER_PARAMETER_SET_1, OCT_B200_ZIMAGE_NOISE_REFINER1_AGGREGATE, r->uploads,
                         r->upload_count, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_REBIND_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

// reactor_vulkan_model_block.c:3274-3396 (audit captures not provided).
int prometheus_reactor_runtime_noise_refiner_execute_resident(void* handle, uint64_t block_id,
                                                              const PrometheusNoiseRefinerResidentExecuteRequest* r,
                                                              PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->struct_size != sizeof(*r) || r->input_generation == 0 ||
        r->output_identity == 0 || r->audit_enabled > 1 ||
        (r->audit_enabled == 0 && (r->audit_family != PROM_NOISE_REFINER_AUDIT_NONE || r->audit_stage != 0 ||
                                   r->audit_output != nullptr || r->audit_element_capacity != 0)) ||
        (r->audit_enabled != 0 && (r->audit_family < PROM_NOISE_REFINER_AUDIT_M1B ||
                                   r->audit_family > PROM_NOISE_REFINER_AUDIT_M1D || r->audit_output == nullptr))) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    if (r->audit_enabled != 0) {  // the staged captures are not provided by this library
      mark_failure(b, PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED);
      fill_evidence(b, b->last_detail, out_evidence);
      return PROM_ERROR;
    }
    return refiner_execute(rt, b, PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO, PROM_NOISE_REFINER_PARAMETER_SET_1,
                           nullptr, nullptr, r->input_generation, 0, r->output_identity, true, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_noise_refiner_audit_final(void* handle, uint64_t block_id,
                                                         const PrometheusNoiseRefinerFinalAuditRequest* r,
                                                         PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->struct_size != sizeof(*r) || r->output == nullptr ||
        r->output_identity == 0 || r->required_output_generation == 0 ||
        r->output_element_capacity < static_cast<uint64_t>(kTokens) * kWidth) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return audit_final(rt, b, PROM_NOISE_REFINER_FAMILY_Z_IMAGE_TURBO, r, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_context_refiner_create(void* handle, const PrometheusContextRefinerCreateRequest* r,
                                                      uint64_t* out_block_id,
                                                      PrometheusModelBlockEvidence* out_evidence) {
  try {
    if (out_block_id != nullptr) *out_block_id = 0;
    Runtime* rt = lookup(handle);
    uint32_t set = 0;
    const uint64_t* aggregate = r == nullptr ? nullptr : context_descriptor(r->lock_identity, r->model_local_block_id, &set);
    if (rt == nullptr || r == nullptr || out_block_id == nullptr || r->struct_size != sizeof(*r) ||
        r->uploads == nullptr || r->upload_count != 11 || aggregate == nullptr ||
        set != PROM_CONTEXT_REFINER_PARAMETER_SET_0) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    PrometheusModelBlockCreateRequest closed{};
    closed.struct_size = sizeof(closed);
    closed.assembly_family = PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO;
    closed.parameter_set = set;
    closed.parameter_set_aggregate_identity = *aggregate;
    closed.model_contract_identity = OCT_B200_ZIMAGE_TURBO_LOCK_ID;
    closed.weight_identity = *aggregate;
    closed.shader_portfolio_identity = OCT_B200_ZIMAGE_TURBO_LOCK_ID;
    closed.precision_policy_identity = OCT_B200_ZIMAGE_TURBO_LOCK_ID;
    closed.capability_route_identity = OCT_B200_ZIMAGE_TURBO_LOCK_ID;
    closed.memory_ceiling_bytes = OCT_B200_ZIMAGE_CONTEXT_MEMORY_PLAN_BYTES;
    closed.external_input_bytes = kContextF32Bytes;
    closed.audit_bytes = OCT_B200_ZIMAGE_AUDIT_ARENA_BYTES;
    closed.shader_id = kShaderContextRefiner;
    closed.weight_count = 11;
    closed.step_count = PROM_MODEL_BLOCK_MAX_STEPS;
    for (uint32_t i = 0; i < PROM_MODEL_BLOCK_MAX_STEPS; ++i) closed.steps[i] = i + 1;
    for (uint32_t i = 0; i < 11; ++i) {
      closed.weights[i].content_identity = r->uploads[i].content_identity;
      closed.weights[i].layout_identity = r->uploads[i].layout_identity;
      closed.weights[i].byte_count = r->uploads[i].byte_count;
    }
    if (!create_request_ok(&closed)) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    uint64_t id = 0;
    if (create_locked(rt, &closed, &id, out_evidence) != PROM_OK) return PROM_ERROR;
    if (upload_locked(rt, rt->model_block, r->uploads, r->upload_count, out_evidence) != PROM_OK) {
      // the facade create is atomic: no unbound owner stays behind
      destroy_model_block(rt);
      return PROM_ERROR;
    }
    *out_block_id = id;
    return PROM_OK;
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_RESOURCE_CREATE_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_context_refiner_rebind(void* handle, uint64_t block_id,
                                                      const PrometheusContextRefinerRebindRequest* r,
                                                      PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    uint32_t set = 0;
    const uint64_t* aggregate = r == nullptr ? nullptr : context_descriptor(r->lock_identity, r->model_local_block_id, &set);
    if (rt == nullptr || r == nullptr || r->uploads == nullptr || r->struct_size != sizeof(*r) ||
        r->upload_count != 11 || aggregate == nullptr || set != PROM_CONTEXT_REFINER_PARAMETER_SET_1) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return rebind_locked(rt, b, PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO, PROM_CONTEXT_REFINER_PARAMETER_SET_0,
                         PROM_CONTEXT_REFINER_PARAMETER_SET_1, *aggregate, r->uploads, r->upload_count, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_REBIND_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_context_refiner0_execute(void* handle, uint64_t block_id,
                                                        const PrometheusContextRefiner0ExecuteRequest* r,
                                                        PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->struct_size != sizeof(*r) || r->output_identity == 0 ||
        r->audit_enabled != 0 || r->context_input == nullptr || r->input_identity == 0 ||
        r->context_input_bytes != kContextF32Bytes) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return refiner_execute(rt, b, PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO, PROM_CONTEXT_REFINER_PARAMETER_SET_0,
                           r->context_input, nullptr, 0, r->input_identity, r->output_identity, false, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_context_refiner_execute_resident(
    void* handle, uint64_t block_id, const PrometheusContextRefinerResidentExecuteRequest* r,
    PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->struct_size != sizeof(*r) || r->output_identity == 0 ||
        r->audit_enabled != 0) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return refiner_execute(rt, b, PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO, PROM_CONTEXT_REFINER_PARAMETER_SET_1,
                           nullptr, nullptr, r->input_generation, 0, r->output_identity, true, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_COMPLETION_UNCERTAIN, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_context_refiner_audit_final(void* handle, uint64_t block_id,
                                                           const PrometheusContextRefinerFinalAuditRequest* r,
                                                           PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr || r == nullptr || r->output == nullptr || r->struct_size != sizeof(*r) ||
        r->output_identity == 0 || r->required_output_generation == 0 ||
        r->output_element_capacity < static_cast<uint64_t>(kContextTokens) * kWidth) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_INVALID_REQUEST, out_evidence);
      return PROM_ERROR;
    }
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    return audit_final(rt, b, PROM_CONTEXT_REFINER_FAMILY_Z_IMAGE_TURBO, r, out_evidence);
  } catch (...) {
    fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_AUDIT_FAILED, out_evidence);
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_model_block_get_evidence(void* handle, uint64_t block_id,
                                                        PrometheusModelBlockEvidence* out_evidence) {
  try {
    Runtime* rt = lookup(handle);
    if (out_evidence == nullptr || rt == nullptr) return PROM_ERROR;
    std::lock_guard<std::mutex> lock(rt->mu);
    ModelBlockState* b = find_block(rt, block_id);
    if (b == nullptr) {
      fill_evidence(nullptr, PROM_MODEL_BLOCK_DETAIL_NOT_FOUND, out_evidence);
      return PROM_ERROR;
    }
    fill_evidence(b, b->last_detail, out_evidence);
    return PROM_OK;
  } catch (...) {
    return PROM_ERROR;
  }
}

int prometheus_reactor_runtime_model_block_destroy(void* handle, uint64_t block_id) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_ERROR;
    std::lock_guard<std::mutex> lock(rt->mu);
    if (find_block(rt, block_id) == nullptr) return PROM_ERROR;
    if (rt->stream != nullptr) cudaStreamSynchronize(rt->stream);
    destroy_model_block(rt);
    return PROM_OK;
  } catch (...) {
    return PROM_ERROR;
  }
}

}  // extern "C"
