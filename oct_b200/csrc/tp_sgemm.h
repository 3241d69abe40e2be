// tp_sgemm.h -- the column-parallel SGEMM object behind the oct_b200_tp_sgemm_* entry points.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "block.h"
#include "kernels.h"

namespace oct {

enum : uint32_t { kTpCollectiveAuto = 0, kTpCollectivePeer = 1, kTpCollectiveNccl = 2 };

struct TpSgemmDims {
  uint32_t rank = 0, world = 1;
  uint32_t max_m = 0, max_n = 0;  // largest m and full n of any call
  uint32_t collective = kTpCollectiveAuto;
};

// C = A * B with B column-sharded over `world` ranks (one process per GPU):
// rank r holds A (m x k, the same on every rank) and B[:, r n/w .. (r+1) n/w),
// computes its column block of C and every rank ends with all of C, row-major.
//   peer stores: the GEMM epilogue writes each finished tile into every rank's
//     output buffer (NVLink stores while the other tiles still compute), then
//     one signal / bounded wait on flags in peer memory;
//   NCCL: the GEMM writes this rank's slab of [world][m][n/w], ncclAllGather
//     fills the others, a repack kernel makes row-major C.
class TpSgemm {
 public:
  TpSgemm() = default;
  ~TpSgemm();
  TpSgemm(const TpSgemm&) = delete;
  TpSgemm& operator=(const TpSgemm&) = delete;

  // Collective over the ranks (every rank calls it): joins the NCCL
  // communicator named by `id`, allocates the output buffers, exchanges IPC
  // handles.  0 on success; -1 bad dims, -3 allocation, -5 NCCL / peer setup.
  int init(const TpSgemmDims& d, const NcclUniqueIdBytes& id, cudaStream_t stream);
  // Enqueue one product on `stream`.  c (optional, ld ldc >= n) receives C;
  // *result (optional) the library's copy (ld n), valid until this rank's
  // next call.  0, -1 bad arguments, -3 allocation, -4 CUDA / NCCL error.
  int run(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc, uint32_t m,
          uint32_t n, uint32_t k, cudaStream_t stream, float** result);
  // Waits for `stream`, returns and clears the kernel status word.
  int status(cudaStream_t stream, unsigned int* out);
  bool peer_stores() const { return fused_; }
  const TpSgemmDims& dims() const { return dims_; }

 private:
  int setup_peers(cudaStream_t stream);
  void teardown_peers();
  cudaError_t ensure(void** buf, uint64_t* cap, uint64_t bytes);

  TpSgemmDims dims_;
  void* comm_ = nullptr;
  bool fused_ = false;
  uint64_t epoch_ = 0;
  float* out_[2] = {nullptr, nullptr};  // whole cudaMalloc allocations (peers map them)
  uint64_t* flags_ = nullptr;           // [2 slots][world] epochs: 0 products, 1 teardown
  float* gather_ = nullptr;             // NCCL path: [world][max_m][max_n / world]
  float** out_peers_ = nullptr;         // device arrays [2][world]
  uint64_t** flag_peers_ = nullptr;     // device array [world]
  unsigned int* err_ = nullptr;
  void* bsplit_ = nullptr;              // B shard hi / lo (split_b_elems each)
  uint64_t bsplit_cap_ = 0;
  void* asplit_ = nullptr;              // A hi / lo (sgemm_tc_a_scratch_bytes), 1024-byte aligned
  uint64_t asplit_cap_ = 0;
  std::vector<void*> peer_opened_;
};

}  // namespace oct
