// tp_sgemm.cu -- column-parallel SGEMM over tensor-parallel ranks with the
// result gathered on every rank (the library-level form of the multi-GPU
// SGEMM; the reference runs one device per handle and has no counterpart).
//
// Per call, on each rank:
//   1. split this rank's B shard [k][n/w] into the TF32 hi / lo K-major layout;
//   2. the 3xTF32 tcgen05 GEMM (sgemm_tc.cu) of A [m][k] by the shard;
//   3a. peer stores: its epilogue stores every finished 128 x 256 tile into
//       the output buffer of every rank at columns r n/w.. (the peers over
//       NVLink, plain st.global, no TMA or bulk copy touches peer memory), so
//       the all-gather overlaps the tiles still being computed; then one
//       signal + bounded wait (tp_fused.cu) publishes "my columns are written";
//   3b. NCCL: the GEMM writes this rank's slab of [w][m][n/w], an in-place
//       ncclAllGather fills the others, repack_kernel makes row-major C.
// Output buffers alternate between calls: a rank can only start writing into
// buffer e % 2 of call e + 2 after every rank signalled call e + 1, which each
// rank's stream issues after it consumed call e's result.
#include "tp_sgemm.h"

#include <algorithm>
#include <cstdio>
#include <cstring>

namespace oct {
namespace {

constexpr unsigned long long kTpWaitNs = 10ull * 1000000000ull;  // bounded cross-rank wait

// gather [w][m][nr] -> dst [m][ldd] (row-major), float4 granules.
__global__ void repack_kernel(const float4* __restrict__ gather, float* __restrict__ dst, uint64_t ldd, uint32_t m,
                              uint32_t nr, uint32_t w, int vec) {
  const uint32_t q = nr / 4;  // granules per slab row
  const uint64_t total = static_cast<uint64_t>(w) * m * q;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t row_all = i / q;  // slab * m + row
    const uint32_t g = static_cast<uint32_t>(i - row_all * q);
    const uint32_t slab = static_cast<uint32_t>(row_all / m);
    const uint32_t row = static_cast<uint32_t>(row_all - static_cast<uint64_t>(slab) * m);
    float* p = dst + row * ldd + static_cast<uint64_t>(slab) * nr + 4ull * g;
    const float4 v = gather[i];
    if (vec) {
      *reinterpret_cast<float4*>(p) = v;
    } else {
      p[0] = v.x;
      p[1] = v.y;
      p[2] = v.z;
      p[3] = v.w;
    }
  }
}

}  // namespace

TpSgemm::~TpSgemm() {
  teardown_peers();
  cudaDeviceSynchronize();
  for (float* p : out_) cudaFree(p);
  cudaFree(flags_);
  cudaFree(gather_);
  cudaFree(out_peers_);
  cudaFree(err_);
  cudaFree(bsplit_);
  cudaFree(asplit_);
  if (comm_ != nullptr && nccl().ok) nccl().destroy(comm_);
}

cudaError_t TpSgemm::ensure(void** buf, uint64_t* cap, uint64_t bytes) {
  if (*buf != nullptr && *cap >= bytes) return cudaSuccess;
  cudaError_t e = cudaDeviceSynchronize();  // earlier calls on any stream may still read it
  if (e != cudaSuccess) return e;
  cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  e = cudaMalloc(buf, bytes + 1024);
  if (e != cudaSuccess) {
    *buf = nullptr;
    (void)cudaGetLastError();
    return e;
  }
  *cap = bytes;
  return cudaSuccess;
}

int TpSgemm::init(const TpSgemmDims& d, const NcclUniqueIdBytes& id, cudaStream_t stream) {
  if (d.world == 0 || d.world > 64 || d.rank >= d.world || d.max_m == 0 || d.max_n == 0 ||
      d.max_n % (4 * d.world) != 0 || d.collective > kTpCollectiveNccl)
    return -1;
  dims_ = d;
  const uint64_t out_bytes = static_cast<uint64_t>(d.max_m) * d.max_n * sizeof(float);
  for (float*& p : out_)
    if (cudaMalloc(&p, out_bytes) != cudaSuccess) {
      (void)cudaGetLastError();
      return -3;
    }
  if (cudaMalloc(&flags_, 2ull * d.world * sizeof(uint64_t)) != cudaSuccess ||
      cudaMalloc(&err_, 16) != cudaSuccess) {
    (void)cudaGetLastError();
    return -3;
  }
  if (cudaMemsetAsync(flags_, 0, 2ull * d.world * sizeof(uint64_t), stream) != cudaSuccess ||
      cudaMemsetAsync(err_, 0, 16, stream) != cudaSuccess)
    return -4;
  if (d.world > 1) {
    if (!nccl().ok) return -5;
    const int nrc = nccl().init_rank(&comm_, static_cast<int>(d.world), id, static_cast<int>(d.rank));
    if (nrc != 0) {
      std::fprintf(stderr, "oct_b200: tp sgemm ncclCommInitRank(rank %u of %u) failed: %d (%s)\n", d.rank, d.world,
                   nrc, nccl().error_string != nullptr ? nccl().error_string(nrc) : "?");
      comm_ = nullptr;
      return -5;
    }
    const int prc = setup_peers(stream);
    if (prc != 0) return prc;
    if (!fused_) {
      if (cudaMalloc(&gather_, out_bytes) != cudaSuccess) {
        (void)cudaGetLastError();
        return -3;
      }
    }
  }
  return cudaStreamSynchronize(stream) == cudaSuccess ? 0 : -4;
}

// Collective (every rank, from init): all-gather each rank's IPC handles, GPU
// UUID and choice of collective over NCCL; open the peers' buffers when every
// rank can take the peer-store path (each on its own GPU, none forcing NCCL).
int TpSgemm::setup_peers(cudaStream_t stream) {
  const uint32_t w = dims_.world, me = dims_.rank;
  struct Info {
    cudaIpcMemHandle_t h[3];
    unsigned char uuid[16];
    uint32_t want;
    uint32_t pad[3];
  };
  Info mine;
  std::memset(&mine, 0, sizeof(mine));
  mine.want = dims_.collective == kTpCollectiveNccl ? 0u : 1u;
  int dev = 0;
  cudaDeviceProp prop;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return -4;
  std::memcpy(mine.uuid, prop.uuid.bytes, 16);
  if (mine.want) {
    void* bufs[3] = {out_[0], out_[1], flags_};
    for (int i = 0; i < 3; ++i)
      if (cudaIpcGetMemHandle(&mine.h[i], bufs[i]) != cudaSuccess) {
        (void)cudaGetLastError();
        mine.want = 0;
      }
  }
  std::vector<Info> all(w);
  unsigned char* dbuf = nullptr;
  if (cudaMalloc(&dbuf, sizeof(Info) * (w + 1)) != cudaSuccess) return -3;
  cudaError_t e = cudaMemcpyAsync(dbuf + sizeof(Info) * w, &mine, sizeof(Info), cudaMemcpyHostToDevice, stream);
  int nrc = 0;
  if (e == cudaSuccess) nrc = nccl().all_gather(dbuf + sizeof(Info) * w, dbuf, sizeof(Info), kNcclInt8, comm_, stream);
  if (e == cudaSuccess && nrc == 0) e = cudaMemcpyAsync(all.data(), dbuf, sizeof(Info) * w, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(dbuf);
  if (e != cudaSuccess || nrc != 0) return -5;
  bool fused = true;
  for (uint32_t p = 0; p < w; ++p) {
    fused = fused && all[p].want == 1;
    for (uint32_t q = 0; q < p; ++q)
      if (std::memcmp(all[p].uuid, all[q].uuid, 16) == 0) fused = false;
  }
  if (!fused) return dims_.collective == kTpCollectivePeer ? -5 : 0;
  std::vector<float*> ptrs(2ull * w);
  std::vector<uint64_t*> fl(w);
  for (uint32_t p = 0; p < w; ++p) {
    if (p == me) {
      ptrs[p] = out_[0];
      ptrs[w + p] = out_[1];
      fl[p] = flags_;
      continue;
    }
    void* ptr[3] = {nullptr, nullptr, nullptr};
    for (int i = 0; i < 3; ++i) {
      if (cudaIpcOpenMemHandle(&ptr[i], all[p].h[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        std::fprintf(stderr, "oct_b200: tp sgemm cudaIpcOpenMemHandle(rank %u buffer %d) failed\n", p, i);
        (void)cudaGetLastError();
        return -5;
      }
      peer_opened_.push_back(ptr[i]);
    }
    ptrs[p] = static_cast<float*>(ptr[0]);
    ptrs[w + p] = static_cast<float*>(ptr[1]);
    fl[p] = static_cast<uint64_t*>(ptr[2]);
  }
  if (cudaMalloc(&out_peers_, 3ull * w * sizeof(void*)) != cudaSuccess) return -3;
  flag_peers_ = reinterpret_cast<uint64_t**>(out_peers_ + 2ull * w);
  e = cudaMemcpyAsync(out_peers_, ptrs.data(), 2ull * w * sizeof(void*), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(flag_peers_, fl.data(), w * sizeof(void*), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return -4;
  fused_ = true;
  return 0;
}

// Bounded barrier on the teardown slot (no rank unmaps or frees a buffer that a
// peer may still write), then unmap the peers' buffers.
void TpSgemm::teardown_peers() {
  if (fused_) {
    cudaDeviceSynchronize();
    const uint64_t ep = epoch_ + 1;
    if (tp_signal(flag_peers_, 1, dims_.world, dims_.rank, ep, nullptr) == cudaSuccess)
      (void)tp_wait(flags_, 1, dims_.world, ep, err_, kTpWaitNs, nullptr);
    cudaDeviceSynchronize();
    fused_ = false;
  }
  for (void* p : peer_opened_) cudaIpcCloseMemHandle(p);
  peer_opened_.clear();
}

int TpSgemm::run(const float* a, uint64_t lda, const float* b, uint64_t ldb, float* c, uint64_t ldc, uint32_t m,
                 uint32_t n, uint32_t k, cudaStream_t stream, float** result) {
  const TpSgemmDims& d = dims_;
  if (a == nullptr || b == nullptr || (c == nullptr && result == nullptr) || m == 0 || n == 0 || k == 0 ||
      m > d.max_m || n > d.max_n || n % (4 * d.world) != 0)
    return -1;
  const uint32_t nr = n / d.world;
  if (lda < k || ldb < nr || (c != nullptr && ldc < n)) return -1;
  const uint64_t belems = split_b_elems(nr, k);
  if (ensure(&bsplit_, &bsplit_cap_, 2ull * belems * sizeof(float)) != cudaSuccess ||
      ensure(&asplit_, &asplit_cap_, sgemm_tc_a_scratch_bytes(m, k)) != cudaSuccess)
    return -3;
  float* bhi = static_cast<float*>(bsplit_);
  float* blo = bhi + belems;
  void* ascratch = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(asplit_) + 1023) & ~uintptr_t(1023));
  ++epoch_;  // every rank issues the same calls, so the epochs agree
  const uint32_t buf = static_cast<uint32_t>(epoch_ & 1u);
  float* out = out_[buf];
  cudaError_t e = sgemm_tc_split_b(b, ldb, k, nr, bhi, blo, stream);
  if (e != cudaSuccess) return -4;
  // the rank's block on the CTA-pair kernel with 32-deep stages from 2048 x 2048 up
  // (as the one-GPU product's AUTO; same bits as the single-CTA kernel)
  const int cfg = (m >= 2048 && nr >= 2048) ? kTcPair32 : kTcSingle16;
  if (d.world == 1) {
    float* dst = c != nullptr ? c : out;
    const uint64_t ldd = c != nullptr ? ldc : n;
    e = sgemm_tc_presplit(a, lda, bhi, blo, dst, ldd, m, n, k, ascratch, err_, stream, nullptr, 0, cfg);
    if (e != cudaSuccess) return -4;
    if (c != nullptr && result != nullptr) {
      e = cudaMemcpy2DAsync(out, n * sizeof(float), c, ldc * sizeof(float), n * sizeof(float), m,
                            cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return -4;
    }
  } else if (fused_) {
    RowScatter sc;
    sc.dst = out_peers_ + static_cast<uint64_t>(buf) * d.world;
    sc.src_rank = d.rank;
    sc.ld = n;
    sc.bcast = d.world;
    sc.col_offset = static_cast<uint64_t>(d.rank) * nr;
    e = sgemm_tc_presplit(a, lda, bhi, blo, out, n, m, nr, k, ascratch, err_, stream, nullptr, 0, cfg, &sc);
    if (e != cudaSuccess) return -4;
    e = tp_signal_wait(flag_peers_, flags_, 0, d.world, d.rank, epoch_, err_, kTpWaitNs, stream);
    if (e != cudaSuccess) return -4;
    if (c != nullptr) {
      e = cudaMemcpy2DAsync(c, ldc * sizeof(float), out, n * sizeof(float), n * sizeof(float), m,
                            cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return -4;
    }
  } else {
    const uint64_t slab = static_cast<uint64_t>(m) * nr;
    float* mine = gather_ + d.rank * slab;
    e = sgemm_tc_presplit(a, lda, bhi, blo, mine, nr, m, nr, k, ascratch, err_, stream, nullptr, 0, cfg);
    if (e != cudaSuccess) return -4;
    if (nccl().all_gather(mine, gather_, slab, kNcclFloat32, comm_, stream) != 0) return -4;
    const uint64_t granules = slab * d.world / 4;
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>((granules + 255) / 256, 148ull * 16));
    const bool both = c != nullptr && result != nullptr;
    float* dst = c != nullptr ? c : out;
    const uint64_t ldd = c != nullptr ? ldc : n;
    const int vec = ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0 && ldd % 4 == 0) ? 1 : 0;
    repack_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float4*>(gather_), dst, ldd, m, nr, d.world, vec);
    if (both)
      repack_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float4*>(gather_), out, n, m, nr, d.world, 1);
    if (cudaGetLastError() != cudaSuccess) return -4;
  }
  if (result != nullptr) *result = out;
  return 0;
}

int TpSgemm::status(cudaStream_t stream, unsigned int* out) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, err_, sizeof(v), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && v != 0) e = cudaMemsetAsync(err_, 0, sizeof(unsigned int), stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  *out = v;
  return e == cudaSuccess ? 0 : -4;
}

}  // namespace oct
