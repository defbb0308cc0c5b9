// kv_copy.cu — byte-moving kernels of the cache path: page scatter/gather,
// batched copy jobs (prefix-cache snapshot/restore, copy-on-write of shared
// tail pages) and conv-ring reordering.  All bit copies with 128-bit accesses.
#include "common.cuh"
#include "kernels.h"

namespace qc {
namespace {

constexpr int HD = 256;
constexpr int PAGE = 64;

// One warp per (position, kv-head) row of 512 B; 4 warps per block cover the
// 4 kv-heads of a position.
__global__ void __launch_bounds__(128) kv_scatter_kernel(uint16_t* k_pool, uint16_t* v_pool,
                                                         const int32_t* page_row, int32_t pos0,
                                                         const uint16_t* k, const uint16_t* v,
                                                         int32_t max_pages, int* err) {
  const int i = blockIdx.x, kvh = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = pos0 + i;
  const int pid = page_row[p / PAGE];
  if (pid < 0 || pid >= max_pages) {
    if (lane == 0) record_error(err, QC_ERR_BOUNDS);
    return;
  }
  const int64_t dst = (((int64_t)pid * 4 + kvh) * PAGE + (p % PAGE)) * HD + lane * 8;
  const int64_t src = ((int64_t)i * 4 + kvh) * HD + lane * 8;
  *reinterpret_cast<uint4*>(k_pool + dst) = *reinterpret_cast<const uint4*>(k + src);
  *reinterpret_cast<uint4*>(v_pool + dst) = *reinterpret_cast<const uint4*>(v + src);
}

__global__ void __launch_bounds__(128) kv_gather_kernel(const uint16_t* k_pool,
                                                        const uint16_t* v_pool,
                                                        const int32_t* page_row, int32_t pos0,
                                                        uint16_t* k, uint16_t* v,
                                                        int32_t max_pages, int* err) {
  const int i = blockIdx.x, kvh = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = pos0 + i;
  const int pid = page_row[p / PAGE];
  if (pid < 0 || pid >= max_pages) {
    if (lane == 0) record_error(err, QC_ERR_BOUNDS);
    return;
  }
  const int64_t src = (((int64_t)pid * 4 + kvh) * PAGE + (p % PAGE)) * HD + lane * 8;
  const int64_t dst = ((int64_t)i * 4 + kvh) * HD + lane * 8;
  *reinterpret_cast<uint4*>(k + dst) = *reinterpret_cast<const uint4*>(k_pool + src);
  *reinterpret_cast<uint4*>(v + dst) = *reinterpret_cast<const uint4*>(v_pool + src);
}

// Batched copy jobs; chunk c belongs to the job j with chunk_start[j] <= c <
// chunk_start[j + 1].  One thread per CTA drives the bulk-copy engine.  The
// CTA's chunks (a contiguous range) stream global -> shared memory
// (cp.async.bulk, completing on an mbarrier) -> global (cp.async.bulk store,
// bulk groups) through a BULK_STAGES-deep ring of `chunk`-byte buffers, so
// BULK_STAGES loads are in flight per SM with no per-byte instructions.
#ifndef QC_BULK_STAGES
#define QC_BULK_STAGES 2
#endif
#ifndef QC_BULK_CTAS
#define QC_BULK_CTAS 4
#endif

constexpr int BULK_STAGES = QC_BULK_STAGES;

__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

__global__ void __launch_bounds__(32) copy_jobs_bulk_kernel(const CopyJob* jobs, int32_t n_jobs,
                                                            const int64_t* chunk_start,
                                                            int64_t n_chunks, int32_t chunk,
                                                            int* err) {
  extern __shared__ __align__(128) unsigned char stage[];
  __shared__ __align__(8) uint64_t full[BULK_STAGES];
  if (threadIdx.x != 0) return;
  for (int i = 0; i < BULK_STAGES; ++i) mbar_init(&full[i], 1);
  fence_mbar_init();
  // contiguous chunk range of this CTA; a job cursor that only moves forward
  const int64_t per = (n_chunks + gridDim.x - 1) / gridDim.x;
  const int64_t c_begin = blockIdx.x * per;
  const int64_t K = max((int64_t)0, min(n_chunks, c_begin + per) - c_begin);
  int lo = 0, hi = n_jobs - 1;  // job of the first chunk
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_start[mid] <= c_begin) lo = mid; else hi = mid - 1;
  }
  int cur = lo;
  CopyJob jb = jobs[cur];
  int64_t next_start = chunk_start[cur + 1];
  auto resolve = [&](int64_t k, const char*& src, char*& dst, uint32_t& bytes) {
    const int64_t c = c_begin + k;  // called with non-decreasing k
    while (c >= next_start) {
      ++cur;
      jb = jobs[cur];
      next_start = chunk_start[cur + 1];
    }
    const int64_t off = (c - chunk_start[cur]) * chunk;
    bytes = static_cast<uint32_t>(min((int64_t)chunk, jb.bytes - off));
    src = static_cast<const char*>(jb.src) + off;
    dst = static_cast<char*>(jb.dst) + off;
  };
  char* dst_of[BULK_STAGES];
  uint32_t bytes_of[BULK_STAGES];
  auto load = [&](int64_t k) {
    const char* src;
    const int s = static_cast<int>(k % BULK_STAGES);
    resolve(k, src, dst_of[s], bytes_of[s]);
    mbar_arrive_expect_tx(&full[s], bytes_of[s]);
    bulk_g2s(stage + (size_t)s * chunk, src, bytes_of[s], &full[s]);
  };
  for (int64_t k = 0; k < K && k < BULK_STAGES; ++k) load(k);
  for (int64_t k = 0; k < K; ++k) {
    const int s = static_cast<int>(k % BULK_STAGES);
    if (!mbar_wait(&full[s], static_cast<uint32_t>((k / BULK_STAGES) & 1), err)) break;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    bulk_s2g(dst_of[s], stage + (size_t)s * chunk, bytes_of[s]);
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    if (k + BULK_STAGES < K) {
      // the store just issued must have read its buffer before the refill
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      load(k + BULK_STAGES);
    }
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ring [4][8192] (slot = position & 3) <-> history [3][8192] oldest first, for
// a sequence whose next token is at position pos.
__global__ void ring_to_hist_kernel(const uint16_t* ring, int32_t pos, uint16_t* hist) {
  const int j = blockIdx.y, c = blockIdx.x * blockDim.x + threadIdx.x;
  const int slot = (pos - 3 + j) & 3;
  hist[j * 8192 + c] = ring[slot * 8192 + c];
}
__global__ void hist_to_ring_kernel(const uint16_t* hist, int32_t pos, uint16_t* ring) {
  const int j = blockIdx.y, c = blockIdx.x * blockDim.x + threadIdx.x;
  const int slot = (pos - 3 + j) & 3;
  ring[slot * 8192 + c] = hist[j * 8192 + c];
}

}  // namespace

cudaError_t launch_kv_scatter(uint16_t* k_pool, uint16_t* v_pool, const int32_t* page_row,
                              int32_t pos0, int32_t n, const uint16_t* k, const uint16_t* v,
                              int32_t max_pages, int* err, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  kv_scatter_kernel<<<n, 128, 0, s>>>(k_pool, v_pool, page_row, pos0, k, v, max_pages, err);
  return cudaGetLastError();
}

cudaError_t launch_kv_gather(const uint16_t* k_pool, const uint16_t* v_pool,
                             const int32_t* page_row, int32_t pos0, int32_t n, uint16_t* k,
                             uint16_t* v, int32_t max_pages, int* err, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  kv_gather_kernel<<<n, 128, 0, s>>>(k_pool, v_pool, page_row, pos0, k, v, max_pages, err);
  return cudaGetLastError();
}

cudaError_t launch_copy_jobs(const CopyJob* jobs_dev, int32_t n_jobs, const int64_t* chunk_start_dev,
                             int64_t n_chunks, int32_t chunk, int* err, cudaStream_t s) {
  if (n_jobs <= 0 || n_chunks <= 0) return cudaSuccess;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = (size_t)BULK_STAGES * chunk;
  static PerDeviceOnce configured;
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(copy_jobs_bulk_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  const int64_t grid = std::min<int64_t>(n_chunks, (int64_t)nsm * QC_BULK_CTAS);
  copy_jobs_bulk_kernel<<<static_cast<unsigned>(grid), 32, smem, s>>>(
      jobs_dev, n_jobs, chunk_start_dev, n_chunks, chunk, err);
  return cudaGetLastError();
}

cudaError_t launch_ring_to_hist(const uint16_t* ring, int32_t pos, uint16_t* hist, cudaStream_t s) {
  ring_to_hist_kernel<<<dim3(8192 / 256, 3), 256, 0, s>>>(ring, pos, hist);
  return cudaGetLastError();
}
cudaError_t launch_hist_to_ring(const uint16_t* hist, int32_t pos, uint16_t* ring, cudaStream_t s) {
  hist_to_ring_kernel<<<dim3(8192 / 256, 3), 256, 0, s>>>(hist, pos, ring);
  return cudaGetLastError();
}

}  // namespace qc
