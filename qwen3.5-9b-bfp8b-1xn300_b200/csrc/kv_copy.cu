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

// Grid-stride over chunks; chunk c belongs to the job j with
// chunk_start[j] <= c < chunk_start[j + 1].  Each thread moves 4 x 16 B per
// iteration with all four loads issued before the stores.
__global__ void __launch_bounds__(256) copy_jobs_kernel(const CopyJob* jobs, int32_t n_jobs,
                                                        const int64_t* chunk_start,
                                                        int64_t n_chunks, int32_t chunk) {
  for (int64_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    int lo = 0, hi = n_jobs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (chunk_start[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const CopyJob jb = jobs[lo];
    const int64_t off = (c - chunk_start[lo]) * chunk;
    const int64_t bytes = min((int64_t)chunk, jb.bytes - off);
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const char*>(jb.src) + off);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(jb.dst) + off);
    const int n16 = static_cast<int>(bytes >> 4);
    int k = threadIdx.x;
    for (; k + 3 * 256 < n16; k += 4 * 256) {
      const uint4 a0 = __ldcs(src + k);
      const uint4 a1 = __ldcs(src + k + 256);
      const uint4 a2 = __ldcs(src + k + 512);
      const uint4 a3 = __ldcs(src + k + 768);
      __stcs(dst + k, a0);
      __stcs(dst + k + 256, a1);
      __stcs(dst + k + 512, a2);
      __stcs(dst + k + 768, a3);
    }
    for (; k < n16; k += 256) __stcs(dst + k, __ldcs(src + k));
  }
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
                             int64_t n_chunks, int32_t chunk, cudaStream_t s) {
  if (n_jobs <= 0 || n_chunks <= 0) return cudaSuccess;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = std::min<int64_t>(n_chunks, (int64_t)nsm * 8);
  copy_jobs_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(jobs_dev, n_jobs, chunk_start_dev,
                                                              n_chunks, chunk);
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
