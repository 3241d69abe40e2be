// block.h -- the transformer block object behind the oct_b200_block_* entry points.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "kernels.h"

namespace oct {

enum : uint32_t { kGemma = 1, kDit = 2 };

// Weight slots (the order of the block's forward pass).
enum : uint32_t {
  kGemmaNorm1 = 0, kGemmaWqkv = 1, kGemmaWo = 2, kGemmaNorm2 = 3, kGemmaWgu = 4, kGemmaWd = 5,
};
enum : uint32_t {
  kDitAdaW = 0, kDitAdaB = 1, kDitAttnNorm1 = 2, kDitWqkv = 3, kDitQNorm = 4, kDitKNorm = 5, kDitWo = 6,
  kDitAttnNorm2 = 7, kDitFfnNorm1 = 8, kDitW13 = 9, kDitW2 = 10, kDitFfnNorm2 = 11,
};

struct BlockDims {
  uint32_t family = 0;
  uint32_t hidden = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0;  // heads / ffn: this rank's share
  uint32_t seq_len = 0, max_batch = 0;
  float eps = 1e-6f, rope_base = 10000.f;
  uint32_t grid_w = 0, rope_frame = 0;
  uint32_t tp_rank = 0, tp_world = 1;
  // DiT variants of the Z-Image executors: rope_text places token p at
  // (rope_frame + p, 0, 0) (caption / context tokens) instead of the image grid;
  // unmodulated runs the block with scale 1, gate 1 and no shift (no adaLN).
  uint32_t rope_text = 0, unmodulated = 0;
};

struct NcclUniqueIdBytes {
  char bytes[128];
};

// ncclGetUniqueId through the dlopen'ed NCCL; 0 on success.
int nccl_unique_id(NcclUniqueIdBytes* out);

// The NCCL entry points the library uses, resolved once by dlopen (ok is false
// when no NCCL library can be loaded).
struct NcclApi {
  typedef int (*GetUniqueIdFn)(void* id);
  typedef int (*CommInitRankFn)(void** comm, int nranks, NcclUniqueIdBytes id, int rank);
  typedef int (*AllReduceFn)(const void* send, void* recv, size_t count, int dtype, int op, void* comm,
                             cudaStream_t stream);
  typedef int (*AllGatherFn)(const void* send, void* recv, size_t count, int dtype, void* comm, cudaStream_t stream);
  typedef int (*CommDestroyFn)(void* comm);
  typedef const char* (*GetErrorStringFn)(int result);
  bool ok = false;
  GetUniqueIdFn get_id = nullptr;
  CommInitRankFn init_rank = nullptr;
  AllReduceFn all_reduce = nullptr;
  AllGatherFn all_gather = nullptr;
  CommDestroyFn destroy = nullptr;
  GetErrorStringFn error_string = nullptr;
};
NcclApi& nccl();
constexpr int kNcclFloat32 = 7;  // ncclFloat32
constexpr int kNcclSum = 0;      // ncclSum
constexpr int kNcclInt8 = 0;     // ncclInt8 (bytes)

class Block {
 public:
  Block() = default;
  ~Block();
  Block(const Block&) = delete;
  Block& operator=(const Block&) = delete;

  // Allocates weights and workspaces for max_batch sequences; with
  // tp_world > 1 also joins the NCCL communicator named by `id`.
  int init(const BlockDims& d, const NcclUniqueIdBytes* id, cudaStream_t stream);
  int set_weight(uint32_t slot, const float* src, uint64_t count, bool on_device);
  // y = block(x) for `batch` sequences of seq_len tokens (x, y: [batch*seq][hidden]).
  // DiT: one timestep per item (host array, embedded sinusoidally on the device),
  // or, with temb_device, the items' 256-d embeddings already on the device.
  int forward(const float* x, float* y, uint32_t batch, const float* timesteps_host,
              const float* temb_device = nullptr);
  void set_stream(cudaStream_t s) { stream_ = s; }
  cudaStream_t stream() const { return stream_; }
  unsigned int read_status();
  const BlockDims& dims() const { return dims_; }
  bool fused_attention() const { return fused_attn_; }

 private:
  struct SplitW {
    float* hi = nullptr;
    float* lo = nullptr;
    uint32_t k = 0, n = 0;
  };
  float* alloc(uint64_t floats);
  int build_rope_tables();
  // `ranges`: the K ranges the product ran in (a scattering product fills that
  // many slots per rank at the owner)
  cudaError_t gemm(const float* a, uint64_t lda, const SplitW& w, float* c, uint64_t ldc, uint32_t m,
                   const float* residual = nullptr, uint64_t ldr = 0, const RowScatter* scatter = nullptr,
                   uint32_t* ranges = nullptr);
  // split-K range count of this block's (n, k) product on the single-CTA kernel
  uint32_t k_ranges(uint32_t n, uint32_t k, bool scatter) const;
  // C = R + A * W with A already split by its producer (hi, lo rows of length w.k)
  cudaError_t gemm_ab(const float* ahi, const float* alo, const SplitW& w, float* c, uint64_t ldc, uint32_t m,
                      const float* residual = nullptr, uint64_t ldr = 0);
  cudaError_t attention(uint32_t batch, uint64_t ldq, uint32_t k_col, uint32_t v_col, bool shared_kv);
  cudaError_t all_reduce(float* buf, uint64_t count);
  // tensor parallel over peer memory (tp_fused.cu)
  float* sym_alloc(uint64_t floats);
  int setup_peers();
  void teardown_peers();
  cudaError_t tp_phase(uint32_t slot);  // signal this rank's stores of `slot`, wait for every rank's
  int forward_tp_fused(const float* x, float* y, uint32_t batch);

  BlockDims dims_;
  cudaStream_t stream_ = nullptr;
  void* comm_ = nullptr;
  std::vector<void*> allocs_;
  SplitW wqkv_, wo_, wgu_, wd_;
  float *norm1_ = nullptr, *norm2_ = nullptr, *norm3_ = nullptr, *norm4_ = nullptr;
  float *qn_ = nullptr, *kn_ = nullptr, *ada_w_ = nullptr, *ada_b_ = nullptr;
  float *temb_ = nullptr, *ada_ = nullptr, *tsteps_ = nullptr;
  float *rope_cos_ = nullptr, *rope_sin_ = nullptr;
  float *hbuf_ = nullptr, *qkv_ = nullptr, *scores_ = nullptr, *attn_ = nullptr, *x1_ = nullptr, *proj_ = nullptr;
  float *gu_ = nullptr, *act_ = nullptr, *scratch_ = nullptr;
  float* psplit_ = nullptr;  // attention probabilities, TF32 hi then lo, [max_batch*heads][p_mp_][p_kp_]
  uint32_t p_mp_ = 0, p_kp_ = 0;
  // producers write the products' A operands pre-split (hi in hbuf_ / act_ / attn_)
  bool split_producers_ = false;
  float *hlo_ = nullptr, *actlo_ = nullptr, *attnlo_ = nullptr;
  // fused attention (DiT, head_dim 128): Q, K, V^T split to TF32 hi/lo per head
  bool fused_attn_ = false;
  float *qsplit_ = nullptr, *ksplit_ = nullptr, *vtsplit_ = nullptr;
  unsigned int* err_ = nullptr;
  // split-K partial products of the products under one wave (splitk_cap_ floats)
  float* splitk_ = nullptr;
  uint64_t splitk_cap_ = 0;
  static constexpr uint32_t kMaxScatterRanges = 4;  // K ranges of a scattering product (owner slots per rank)
  // Fused tensor parallel: the row-parallel products scatter their partial rows
  // into the owner rank's `rs_` slots; owners reduce and push finished rows into
  // every rank's `hbuf_` / `ysym_`.  Flags: [5 slots][world] u64 epochs.
  bool fused_tp_ = false;
  uint64_t epoch_ = 0;
  float *rs_ = nullptr, *ysym_ = nullptr;
  uint64_t* flags_ = nullptr;
  std::vector<void*> sym_raw_;      // this rank's symmetric allocations
  std::vector<void*> peer_opened_;  // peers' allocations mapped into this process
  float** rs_peers_ = nullptr;      // device arrays of one pointer per rank
  float** h_peers_ = nullptr;
  float** y_peers_ = nullptr;
  uint64_t** flag_peers_ = nullptr;
};

}  // namespace oct
