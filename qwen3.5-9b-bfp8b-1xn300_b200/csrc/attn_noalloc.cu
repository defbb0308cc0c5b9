// attn_noalloc.cu — qc_attn_decode_noalloc: the paged attention decode for
// callers that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits — an engine that
// hands out all device memory from its own arena and forbids allocation after
// start-up, a plugin called inside another framework's memory pool, or a
// deployment that caps the process at a fixed footprint.  Such a caller owns
// the KV pool, the page table, the small weights and the RoPE table already;
// what the attention kernel additionally needs is scratch memory for the
// per-CTA split-K records and the per-step descriptor.  Here that scratch is
// a file-scope __device__ array of fixed size, so the call allocates nothing.
//
// Limits and rules:
//   - at most QC_NOALLOC_MAX_BATCH sequences per call, at most
//     QC_NOALLOC_MAX_CTAS SMs on the device (larger requests are rejected);
//   - the array is ~1.9 MB and stays resident on every GPU that loads the
//     library until the process exits;
//   - every call on a device shares the one array, which keeps the previous
//     call's contents: calls whose kernels overlap on the GPU (two streams, two
//     host threads) race and give wrong results — serialise them;
//   - the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture;
//   - the step descriptor reaches the device as a kernel parameter (a small
//     kernel stores it into the array), so a call copies nothing from host
//     memory and does not wait for earlier work on the stream;
//   - the kernels' error word also lives in the array: it collects
//     QC_ERR_BOUNDS / QC_ERR_TIMEOUT from every call on the device until
//     qc_attn_noalloc_check reads and clears it.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <cudaTypedefs.h>

#include "../../include/qcache.h"
#include "kernels.h"

namespace {

constexpr int MAX_BATCH = QC_NOALLOC_MAX_BATCH;
constexpr int MAX_CTAS = QC_NOALLOC_MAX_CTAS;
constexpr int MAX_SLOTS = 4 * MAX_BATCH + MAX_CTAS;  // partial records
constexpr int DESC_WORDS = 5 * MAX_BATCH + 4;
constexpr int MAX_DEVICES = 64;

// Layout (in floats / int32 words): part_o [MAX_SLOTS][4][256] | part_m
// [MAX_SLOTS][4] | part_l [MAX_SLOTS][4] | descriptor (int32) | error word.
constexpr size_t O_OFF = 0;
constexpr size_t M_OFF = O_OFF + (size_t)MAX_SLOTS * 4 * 256;
constexpr size_t L_OFF = M_OFF + (size_t)MAX_SLOTS * 4;
constexpr size_t D_OFF = L_OFF + (size_t)MAX_SLOTS * 4;
constexpr size_t E_OFF = D_OFF + DESC_WORDS;
constexpr size_t SCRATCH_WORDS = E_OFF + 4;

static __device__ __align__(256) float g_noalloc_scratch[SCRATCH_WORDS];

struct DeviceSetup {
  std::once_flag once;
  int rc = QC_OK;            // outcome of the one-time setup
  char msg[160] = {};
  float* scratch = nullptr;  // device address of g_noalloc_scratch
  int nsm = 0;
};
DeviceSetup g_setup[MAX_DEVICES];
std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// The step descriptor, passed by value to the kernel that stores it.
struct Desc {
  int32_t w[DESC_WORDS];
};

__global__ void noalloc_store_desc_kernel(const Desc d, int32_t words, int32_t* dst) {
  for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = d.w[i];
}

int err(int code, const char* fmt, ...) {
  char buf[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  qc::set_thread_error(buf);
  return code;
}

}  // namespace

extern "C" int qc_attn_decode_noalloc(const uint16_t* proj_dev, uint16_t* k_pool_dev,
                                      uint16_t* v_pool_dev, int32_t max_pages,
                                      const int32_t* page_table_dev, int32_t pt_stride,
                                      const int32_t* pos, int32_t n, const float* q_norm_dev,
                                      const float* k_norm_dev, const float* rope_cos_dev,
                                      const float* rope_sin_dev, uint16_t* out_dev,
                                      qc_stream stream) {
  if (!proj_dev || !k_pool_dev || !v_pool_dev || !page_table_dev || !pos || !q_norm_dev ||
      !k_norm_dev || !rope_cos_dev || !rope_sin_dev || !out_dev)
    return err(QC_ERR_ARG, "qc_attn_decode_noalloc: null pointer argument");
  if (n < 1 || n > MAX_BATCH)
    return err(QC_ERR_ARG, "qc_attn_decode_noalloc: batch of %d sequences, limit is %d", n,
               MAX_BATCH);
  if (max_pages < 1 || pt_stride < 1)
    return err(QC_ERR_ARG, "qc_attn_decode_noalloc: max_pages %d, pt_stride %d", max_pages,
               pt_stride);
  for (int32_t i = 0; i < n; ++i)
    if (pos[i] < 0 || pos[i] / QC_PAGE >= pt_stride)
      return err(QC_ERR_ARG, "qc_attn_decode_noalloc: position %d of sequence %d needs page "
                 "%d, page-table rows hold %d", pos[i], i, pos[i] / QC_PAGE, pt_stride);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return err(QC_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= MAX_DEVICES) return err(QC_ERR_ARG, "device %d out of range", dev);

  // once per device, with that device current
  DeviceSetup& su = g_setup[dev];
  std::call_once(su.once, [&su, dev] {
    cudaError_t e2 = cudaGetSymbolAddress((void**)&su.scratch, g_noalloc_scratch);
    if (e2 == cudaSuccess) e2 = cudaDeviceGetAttribute(&su.nsm, cudaDevAttrMultiProcessorCount, dev);
    if (e2 != cudaSuccess) {
      su.rc = QC_ERR_CUDA;
      snprintf(su.msg, sizeof(su.msg), "qc_attn_decode_noalloc setup: %s", cudaGetErrorString(e2));
      return;
    }
    std::call_once(g_encode_once, [] {
      cudaDriverEntryPointQueryResult qres;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&g_encode, cudaEnableDefault,
                                  &qres) != cudaSuccess ||
          qres != cudaDriverEntryPointSuccess)
        g_encode = nullptr;
    });
    if (!g_encode) {
      su.rc = QC_ERR_CUDA;
      snprintf(su.msg, sizeof(su.msg), "cuTensorMapEncodeTiled unavailable");
    }
  });
  if (su.rc != QC_OK) return err(su.rc, "%s", su.msg);
  if (su.nsm > MAX_CTAS)
    return err(QC_ERR_ARG, "qc_attn_decode_noalloc: %d SMs, limit is %d", su.nsm, MAX_CTAS);

  // descriptor: slots (= page-table rows 0..n-1) | pos | seg | page0 | append | total, per
  Desc dd;
  int32_t* d = dd.w;
  d[2 * n] = 0;
  for (int32_t i = 0; i < n; ++i) {
    d[i] = i;
    d[n + i] = pos[i];
    d[2 * n + 1 + i] = d[2 * n + i] + 4 * (pos[i] / QC_PAGE + 1);
    d[3 * n + 1 + i] = 0;
    d[4 * n + 1 + i] = 1;
  }
  const int32_t total = d[3 * n];
  const int32_t per = (total + su.nsm - 1) / su.nsm;
  d[5 * n + 1] = total;
  d[5 * n + 2] = per;
  int32_t* desc = reinterpret_cast<int32_t*>(su.scratch + D_OFF);
  cudaStream_t st = (cudaStream_t)stream;
  noalloc_store_desc_kernel<<<1, 128, 0, st>>>(dd, 5 * n + 3, desc);
  e = cudaGetLastError();
  if (e != cudaSuccess) return err(QC_ERR_CUDA, "descriptor store: %s", cudaGetErrorString(e));

  // tensor maps over the caller's pools (host-side encoding, no allocation)
  CUtensorMap tmk, tmv;
  const cuuint64_t dims[2] = {(cuuint64_t)QC_HEAD_DIM,
                              (cuuint64_t)max_pages * QC_N_HEAD_KV * QC_PAGE};
  const cuuint64_t strides[1] = {(cuuint64_t)QC_HEAD_DIM * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)qc::KV_BOX_ROWS};
  const cuuint32_t estr[2] = {1, 1};
  for (int kv = 0; kv < 2; ++kv) {
    CUresult r = g_encode(kv ? &tmv : &tmk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                          kv ? (void*)v_pool_dev : (void*)k_pool_dev, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return err(QC_ERR_ARG, "tensor map over the KV pool rejected (pools 16-byte aligned?)");
  }

  qc::AttnArgs a{};
  a.proj = proj_dev;
  a.k_pool = k_pool_dev;
  a.v_pool = v_pool_dev;
  a.page_table = page_table_dev;
  a.pt_stride = pt_stride;
  a.max_pages = max_pages;
  a.slots = desc;
  a.pos = desc + n;
  a.seg = desc + 2 * n;
  a.page0 = desc + 3 * n + 1;
  a.append = desc + 4 * n + 1;
  a.q_norm = q_norm_dev;
  a.k_norm = k_norm_dev;
  a.rope_cos = rope_cos_dev;
  a.rope_sin = rope_sin_dev;
  a.part_o = su.scratch + O_OFF;
  a.part_m = su.scratch + M_OFF;
  a.part_l = su.scratch + L_OFF;
  a.split = desc + 5 * n + 1;
  a.per_hint = per;
  a.n = n;
  a.grid = su.nsm;
  a.err = reinterpret_cast<int*>(su.scratch + E_OFF);
  qc::CombineArgs cb{};
  cb.proj = proj_dev;
  cb.out = out_dev;
  cb.seg = a.seg;
  cb.part_m = a.part_m;
  cb.part_l = a.part_l;
  cb.part_o = a.part_o;
  cb.split = a.split;
  cb.n = n;
  e = qc::launch_attn_decode(a, cb, tmk, tmv, st);
  if (e != cudaSuccess) return err(QC_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return QC_OK;
}

extern "C" int qc_attn_noalloc_check(qc_stream stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return err(QC_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= MAX_DEVICES) return err(QC_ERR_ARG, "device %d out of range", dev);
  DeviceSetup& su = g_setup[dev];
  // no call has run on this device yet (the setup records its outcome first)
  if (!su.scratch) return su.rc != QC_OK ? err(su.rc, "%s", su.msg) : QC_OK;
  e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return err(QC_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
  int* word = reinterpret_cast<int*>(su.scratch + E_OFF);
  int code = 0;
  e = cudaMemcpy(&code, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && code) e = cudaMemset(word, 0, sizeof(int));
  if (e != cudaSuccess) return err(QC_ERR_CUDA, "error word: %s", cudaGetErrorString(e));
  if (code)
    return err(code, "qc_attn_decode_noalloc: the device reported %s",
               code == QC_ERR_BOUNDS ? "a page id out of range (that tile was skipped)"
               : code == QC_ERR_TIMEOUT ? "a wait timeout" : "an error");
  return QC_OK;
}
