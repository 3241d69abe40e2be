// runtime.h -- the handle behind the C ABI (one CUDA stream per handle) and the
// helpers every entry-point file of libprometheus_reactor.so shares.
#pragma once

#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/prometheus_reactor.h"
#include "block.h"
#include "kernels.h"
#include "tp_sgemm.h"

namespace oct {
namespace rt {

using Clock = std::chrono::steady_clock;
constexpr uint32_t kMagic = 0x0C7B2000u;
constexpr int kAsyncSlots = 4;  // task capacity, as the reference (reactor_api.h:2030 tasks[4])
constexpr uint32_t kBatchWorkers = 8;  // PROM_SGEMM_BATCH_MAX_LOGICAL_WIDTH (reactor_batch.c:56)

inline uint64_t ns_since(Clock::time_point t0) {
  return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(Clock::now() - t0).count());
}

inline void set_status(uint32_t* stage, int* detail, uint32_t s, int d) {
  if (stage != nullptr) *stage = s;
  if (detail != nullptr) *detail = d;
}

// A growable device allocation.  Growth synchronises the owning stream first
// so no kernel in flight still references the old block.
struct DevBuf {
  void* raw = nullptr;
  uint64_t cap = 0;
  void* aligned() const { return reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023)); }
  cudaError_t ensure(uint64_t bytes, cudaStream_t s) {
    if (bytes <= cap && raw != nullptr) return cudaSuccess;
    // Kernels on any stream may still read the old block (device entry points
    // accept caller streams), so growth waits for the whole device.
    (void)s;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    if (raw != nullptr) cudaFree(raw);
    raw = nullptr;
    cap = 0;
    const uint64_t want = bytes + (bytes >> 3);  // 12.5% headroom against regrowth
    e = cudaMalloc(&raw, want + 1024);
    if (e != cudaSuccess) {
      raw = nullptr;
      (void)cudaGetLastError();
      return e;
    }
    cap = want;
    return cudaSuccess;
  }
  void release() {
    if (raw != nullptr) cudaFree(raw);
    raw = nullptr;
    cap = 0;
  }
};

struct AsyncTask {
  bool active = false;
  int id = 0;
  uint32_t state = PROM_ASYNC_STATE_IDLE;
  uint32_t m = 0, n = 0, k = 0;
  int final_detail = 0;
  uint32_t final_stage = 0;
  cudaEvent_t begin = nullptr, done = nullptr;  // bracket the task's work on the handle's stream
  DevBuf a, b, c;
  // diagnostics (prometheus_reactor_runtime_sgemm_async_diagnostics)
  uint32_t generation = 0;       // submissions through this slot
  uint64_t sequence = 0;         // handle-wide submission sequence number
  bool abandoned = false;
  bool timed = false;
  uint64_t gpu_ns = 0;
};

// Lifecycle counters of the async queue.
struct AsyncStats {
  uint64_t submitted = 0, ready = 0, failed = 0, consumed = 0, abandoned = 0;
  uint64_t queue_full = 0, stale_ids = 0, polls = 0, reaped = 0, sequence = 0;
  uint32_t max_in_flight = 0;
};

// Counters of the reduction executor (prometheus_reactor_runtime_reduction_diagnostics).
struct ReductionStats {
  bool initialized = false;
  uint32_t ring_depth = 0;  // as configured (Go passes 3); one CUDA stream serves every request
  uint64_t total = 0, success = 0, failures = 0, command_records = 0, submits = 0;
  uint64_t allocations = 0, reuses = 0;
  uint64_t last_replay = 0, last_gpu_ns = 0, last_e2e_ns = 0;
  uint32_t last_stage_count = 0, slot_generation = 0;
  int32_t last_detail = 0;
};

struct Runtime {
  uint32_t magic = kMagic;
  std::mutex mu;
  int device = 0;
  bool available = false;
  uint32_t reason = PROM_REASON_NONE;
  uint32_t test_flags = 0, async_test_flags = 0, reduction_test_flags = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  DevBuf scratch;               // split-TF32 operand buffers
  DevBuf da, db, dc;            // staging for host-pointer SGEMM
  DevBuf rin, rout, rw, rinv;   // staging for reductions / RMSNorm
  DevBuf words;                 // [0] kernel error bits (u32), [8] first non-finite index (u64)
  AsyncTask tasks[kAsyncSlots];
  int next_task_id = 1;
  AsyncStats async_stats;
  ReductionStats red_stats;
  // Optional per-launch kernel timing of the tensor-core SGEMM (events on the
  // launch stream): split pass and main kernel, summed on read.
  bool timing = false;
  std::vector<oct::SgemmEvents> timing_events;
  size_t timing_used = 0;
  // Pipelined host SGEMM: upload and download streams, chunk events.
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  std::vector<cudaEvent_t> pipe_events;
  // SGEMM batch workers: one stream, split scratch and A/B staging each.
  cudaStream_t batch_streams[kBatchWorkers] = {};
  DevBuf batch_scratch[kBatchWorkers], batch_a[kBatchWorkers], batch_b[kBatchWorkers];
  DevBuf batch_c;  // every entry's C, until the whole batch has succeeded
  // Transformer blocks created on this handle.
  std::unordered_map<uint64_t, oct::Block*> blocks;
  uint64_t next_block = 1;
  // Column-parallel SGEMM objects (tp_sgemm_api.cpp).
  std::unordered_map<uint64_t, oct::TpSgemm*> tp_sgemms;
  uint64_t next_tp_sgemm = 1;
  uint64_t next_request_id = 1;
  // Gemma M1 boundary (gemma_m1_api.cpp): the generation of the handle's one
  // committed RMSNorm weight, and device staging for the positional tables and
  // the resident positioned Q / K rows and scores.
  uint64_t m46_weight_generation = 0;
  uint64_t m46_allocations = 0;   // staging (re)allocations made by the RMSNorm entries
  DevBuf m1_cos, m1_sin, m1_q, m1_k, m1_scores;
  uint32_t m1_slot_generation[3] = {0, 0, 0};  // writes of the Q, K and score slots
  // FFT (fft_api.cpp): device staging, the binary64 twiddle table of the last
  // size, and the diagnostics record of the last request.
  DevBuf fft_in, fft_out, fft_tw;
  uint32_t fft_tw_count = 0;
  uint64_t fft_grow[3] = {0, 0, 0}, fft_reuse[3] = {0, 0, 0};  // ping (in), pong (out), twiddles
  PrometheusFftDiagnostics fft_diag = {};
  bool fft_diag_init = false;
  // The handle's one Z-Image model block (zimage_api.cpp), or null.
  struct ModelBlockState* model_block = nullptr;
  uint64_t next_model_block_id = 1;

  unsigned int* err_word() { return static_cast<unsigned int*>(words.aligned()); }
  unsigned long long* nonfinite_word() {
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(words.aligned()) + 8);
  }
};


struct ModelBlockState;
// Releases the handle's model block (zimage_api.cpp); the handle's stream is idle.
void destroy_model_block(Runtime* rt);

// The live handle behind `handle`, or null when it is not one (locked registry).
Runtime* lookup(void* handle);
// Registers / unregisters a handle in that registry.
void register_runtime(Runtime* rt);
void unregister_runtime(Runtime* rt);

// Resets the kernel status words on the stream (async).
inline cudaError_t reset_words(Runtime* rt) {
  cudaError_t e = cudaMemsetAsync(rt->err_word(), 0, 8, rt->stream);
  if (e != cudaSuccess) return e;
  return cudaMemsetAsync(rt->nonfinite_word(), 0xFF, 8, rt->stream);
}

struct Words {
  unsigned int err = 0;
  unsigned long long nonfinite = ~0ull;
};

inline cudaError_t read_words(Runtime* rt, Words* w) {
  unsigned char host[16];
  cudaError_t e = cudaMemcpyAsync(host, rt->words.aligned(), 16, cudaMemcpyDeviceToHost, rt->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
  if (e != cudaSuccess) return e;
  std::memcpy(&w->err, host, 4);
  std::memcpy(&w->nonfinite, host + 8, 8);
  return cudaSuccess;
}

inline bool checked_mul(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

// Enqueues C = A * B for device pointers and chooses the kernel (reactor_api.cpp).
// `scratch` (default: the handle's) holds the TF32 split operands; calls that
// run concurrently on different streams need different scratch buffers.
int enqueue_sgemm(Runtime* rt, const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc,
                  uint32_t m, uint32_t n, uint32_t k, uint32_t variant, cudaStream_t stream,
                  const GemmBatch* batch = nullptr, DevBuf* scratch = nullptr);

}  // namespace rt
}  // namespace oct
