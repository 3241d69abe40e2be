// tp_sgemm_api.cpp -- the column-parallel SGEMM entry points of the C ABI
// (tp_sgemm.cu does the work).  The reference drives one device per handle
// (prometheus_reactor_runtime_sgemm, internal/prometheus/native/reactor_api.h:2587-2595);
// these entries are its multi-GPU form, one process and one handle per GPU,
// with the objects owned by the handle like the transformer blocks.
#include "runtime.h"

using namespace oct::rt;

namespace {

int fail(int* detail, int rc, int code) {
  if (detail) *detail = code;
  return rc;
}

}  // namespace

extern "C" {

int oct_b200_tp_sgemm_create(void* handle, const OctB200TpSgemmConfig* cfg, uint64_t* out_id, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (cfg == nullptr || out_id == nullptr || cfg->struct_size < sizeof(OctB200TpSgemmConfig))
      return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_TP_INVALID);
    if (!rt->available) return fail(out_detail_code, PROM_ERROR, PROM_DETAIL_CAPABILITY_MISMATCH);
    oct::TpSgemmDims d;
    d.rank = cfg->rank;
    d.world = cfg->world == 0 ? 1 : cfg->world;
    d.max_m = cfg->max_m;
    d.max_n = cfg->max_n;
    d.collective = cfg->collective;
    if (d.rank >= d.world || d.world > 64 || d.max_m == 0 || d.max_n == 0 || d.max_n % (4 * d.world) != 0 ||
        d.collective > OCT_B200_TP_COLLECTIVE_NCCL)
      return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_TP_INVALID);
    oct::NcclUniqueIdBytes id{};
    std::memcpy(id.bytes, cfg->nccl_id, 128);
    std::lock_guard<std::mutex> lock(rt->mu);
    oct::TpSgemm* t = new (std::nothrow) oct::TpSgemm();
    if (t == nullptr) return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_TP_ALLOC);
    const int rc = t->init(d, id, rt->stream);
    if (rc != 0) {
      delete t;
      return fail(out_detail_code, PROM_ERROR,
                  rc == -3 ? OCT_B200_DETAIL_TP_ALLOC
                           : (rc == -5 ? OCT_B200_DETAIL_TP_NCCL
                                       : (rc == -1 ? OCT_B200_DETAIL_TP_INVALID : OCT_B200_DETAIL_CUDA_ERROR)));
    }
    const uint64_t id_out = rt->next_tp_sgemm++;
    rt->tp_sgemms[id_out] = t;
    *out_id = id_out;
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_sgemm_tp_device(void* handle, uint64_t id, const float* d_a, uint64_t lda, const float* d_b_shard,
                             uint64_t ldb, float* d_c, uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, void* stream,
                             float** out_result, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->tp_sgemms.find(id);
    if (it == rt->tp_sgemms.end()) return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_TP_NOT_FOUND);
    const int rc = it->second->run(d_a, lda, d_b_shard, ldb, d_c, ldc, m, n, k, static_cast<cudaStream_t>(stream),
                                   out_result);
    if (rc != 0)
      return fail(out_detail_code, PROM_ERROR,
                  rc == -1 ? OCT_B200_DETAIL_INVALID_ARGUMENT
                           : (rc == -3 ? OCT_B200_DETAIL_OUT_OF_MEMORY : OCT_B200_DETAIL_TP_EXEC));
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_tp_sgemm_sync(void* handle, uint64_t id, void* stream, int* out_detail_code) {
  try {
    if (out_detail_code) *out_detail_code = 0;
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->tp_sgemms.find(id);
    if (it == rt->tp_sgemms.end()) return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_TP_NOT_FOUND);
    unsigned int flags = 0;
    if (it->second->status(static_cast<cudaStream_t>(stream), &flags) != 0)
      return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_CUDA_ERROR);
    if (flags != 0) return fail(out_detail_code, PROM_ERROR, OCT_B200_DETAIL_DEVICE_TIMEOUT);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_tp_sgemm_collective(void* handle, uint64_t id, uint32_t* out_collective) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    if (out_collective == nullptr) return PROM_ERROR;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->tp_sgemms.find(id);
    if (it == rt->tp_sgemms.end()) return PROM_ERROR;
    const oct::TpSgemm* t = it->second;
    *out_collective = t->dims().world == 1 ? OCT_B200_TP_COLLECTIVE_AUTO
                                           : (t->peer_stores() ? OCT_B200_TP_COLLECTIVE_PEER
                                                               : OCT_B200_TP_COLLECTIVE_NCCL);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

int oct_b200_tp_sgemm_destroy(void* handle, uint64_t id) {
  try {
    Runtime* rt = lookup(handle);
    if (rt == nullptr) return PROM_INVALID_HANDLE;
    std::lock_guard<std::mutex> lock(rt->mu);
    auto it = rt->tp_sgemms.find(id);
    if (it == rt->tp_sgemms.end()) return PROM_ERROR;
    delete it->second;
    rt->tp_sgemms.erase(it);
    return PROM_OK;
  } catch (...) {
    return PROM_INTERNAL_ERROR;
  }
}

}  // extern "C"
