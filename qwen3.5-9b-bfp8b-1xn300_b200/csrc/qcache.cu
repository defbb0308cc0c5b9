// qcache.cu — host side of the cache path: the context behind include/qcache.h.
//
// Owns the device pools (paged bf16 KV, DeltaNet state, conv rings, prefix
// snapshots), the host page allocator with refcounts, the per-sequence page
// tables and token histories, and the hashed prefix table.  Every device
// operation is a kernel or copy enqueued on the caller's stream; there is no
// host fallback for any computation.
//
// Reference correspondence (src/engine.cpp): the globals g_k_cache/g_v_cache,
// g_ssm_state, g_conv_state, g_cached_tokens (79-97) become per-sequence
// device state here; reset_state (4164-4176) is qc_seq_reset; the prefix rule
// of generate() (4058-4080) is qc_seq_match_prefix.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/qcache.h"
#include "kernels.h"

using qc::CopyJob;

namespace {

constexpr int HD = QC_HEAD_DIM;
constexpr int PAGE = QC_PAGE;
constexpr int64_t PAGE_ELEMS = (int64_t)QC_N_HEAD_KV * PAGE * HD;       // per layer, K or V
constexpr int64_t RING_ELEMS = 4LL * QC_CONV_CH;                        // [4][8192]
constexpr int64_t HIST_ELEMS = 3LL * QC_CONV_CH;                        // [3][8192]
#ifndef QC_COPY_CHUNK_KB
#define QC_COPY_CHUNK_KB 24
#endif
constexpr int COPY_CHUNK = QC_COPY_CHUNK_KB * 1024;  // bulk-copy ring buffer size
constexpr int STAGING_SLOTS = 4;

struct Seq {
  bool live = false;
  int32_t len = 0;
  std::vector<int32_t> pages;
  std::vector<int32_t> tokens;
  bool dirty = false;  // page-table row differs from the device copy
};

struct Entry {
  bool live = false;
  int32_t P = 0;
  std::vector<int32_t> tokens;
  std::vector<int32_t> pages;  // full pages shared, tail page owned
  int32_t snap = -1;
  uint64_t key = 0;            // chain hash after the last full page
};

}  // namespace

struct qc_ctx {
  qc_config cfg{};
  int device = QC_DEVICE_NONE;
  bool host_only = true;
  int nsm = 148;
  std::string err;
  int32_t pt_stride = 0;  // page-table row capacity (pages per sequence)

  // device pools
  uint16_t* k_pool = nullptr;   // [n_attn][max_pages][4][64][256]
  uint16_t* v_pool = nullptr;
  float* state = nullptr;       // [max_seqs][n_gdn][32][128][128]
  uint16_t* ring = nullptr;     // [max_seqs][n_gdn][4][8192]
  float* snap_state = nullptr;  // [max_snapshots][n_gdn][32][128][128]
  uint16_t* snap_hist = nullptr;// [max_snapshots][n_gdn][3][8192]
  float* q_norm = nullptr;      // [n_attn][256]
  float* k_norm = nullptr;
  float* ssm_a = nullptr;       // [n_gdn][32]
  float* dt_bias = nullptr;     // [n_gdn][32]
  float* ssm_norm = nullptr;    // [n_gdn][128]
  float* conv_w = nullptr;      // [n_gdn][4][8192]
  float* rope_cos = nullptr;    // [max_ctx][32]
  float* rope_sin = nullptr;
  int32_t* page_table = nullptr;// [max_seqs][pt_stride]
  int32_t* desc = nullptr;      // batch: slots | pos | seg | page0 | append
  int32_t* desc_part = nullptr; // same layout, one sequence, for qc_attn_partial
  // split-K over devices through peer memory (qc_p2p_*)
  int32_t p2p_world = 0, p2p_rank = -1;
  char* mbox = nullptr;         // this rank's mailbox (records, then counters)
  char* peer_mbox[QC_P2P_MAX_RANKS] = {};  // every rank's mailbox, self included
  bool p2p_poisoned = false;    // a merge wait expired: refuse until qc_p2p_reset
  float* part_m = nullptr;
  float* part_l = nullptr;
  float* part_o = nullptr;
  int32_t part_slots = 0;
  CopyJob* jobs = nullptr;
  int64_t* chunk_start = nullptr;
  int32_t job_cap = 0;
  int* dev_err = nullptr;       // error words [EK_COUNT][err_layers], see err_site
  int32_t err_layers = 1;
  int32_t ref_math = 0;         // QC_FLAG_REFERENCE_MATH
  std::vector<uint8_t> gdn_ran; // DeltaNet layers already run in the open decode step
  std::vector<uint8_t> attn_ran;// attention layers already run in the open decode step
  uint16_t* pf_q = nullptr;     // prefill: q tile [4][128][256] bf16
  float* pf_rec = nullptr;      // prefill: records [4][pf_split][128][260] f32
  float* pf_conv = nullptr;     // prefill: conv outputs [32][8192] f32
  int32_t pf_split = 0;
  int32_t p_per = 0;            // split over devices: page-heads per CTA of the open range
  std::vector<CUtensorMap> tm_k, tm_v;  // per attention layer, for the TMA tile loads

  // pinned staging ring for host -> device uploads
  char* stage[STAGING_SLOTS] = {};
  cudaEvent_t stage_ev[STAGING_SLOTS] = {};
  size_t stage_cap = 0;
  int stage_next = 0;

  // host bookkeeping
  std::vector<Seq> seqs;
  std::vector<int32_t> page_ref;
  std::vector<int32_t> free_pages;
  std::vector<int32_t> h_page_table;
  std::vector<Entry> entries;
  std::unordered_map<uint64_t, std::vector<int32_t>> index;
  std::vector<int32_t> free_snaps;

  // current decode batch
  bool in_step = false;
  std::vector<int32_t> b_seq, b_pos, b_seg, b_tok;
  bool b_has_tok = false;
  int32_t b_total = 0, b_per = 0, b_grid = 0;
  int64_t last_restore_bytes = 0;
  // open prefill chunk
  bool in_prefill = false;
  int32_t p_seq = -1, p_pos0 = 0, p_n = 0;
  std::vector<int32_t> p_tok;
};

namespace {

// Device error words: one per launch site (kernel kind x layer).  A kernel
// records QC_ERR_TIMEOUT / QC_ERR_BOUNDS into its site's word, so that
// qc_check_device can say which kernel of which layer failed, as the
// reference's hang breadcrumbs name the layer and operation of a stuck device
// call (src/engine.cpp:99-101, 4182-4185).
enum ErrKind {
  EK_ATTN_DECODE, EK_ATTN_MERGE, EK_GDN_DECODE, EK_ATTN_PREFILL, EK_KV_COPY, EK_COPY_JOBS,
  EK_COUNT
};
const char* const kErrKindName[EK_COUNT] = {
    "attention decode (attn_partial_kernel)", "peer-record merge (attn_merge_mailbox_kernel)",
    "DeltaNet decode (gdn_decode_kernel)", "attention prefill (attn_prefill_tc_kernel)",
    "KV scatter/gather (kv_scatter_kernel / kv_gather_kernel)",
    "batched copy (copy_jobs_bulk_kernel)"};

int* err_site(qc_ctx* c, int kind, int layer) {
  return c->dev_err + (int64_t)kind * c->err_layers + layer;
}

int fail(qc_ctx* c, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return code;
}

#define QC_CUDA(c, call)                                                              \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return fail((c), QC_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_),  \
                  __FILE__, __LINE__);                                                \
  } while (0)

#define QC_NEED_DEVICE(c) \
  do {                    \
    if ((c)->host_only) return fail((c), QC_ERR_NODEVICE, "host-only context: no device work"); \
  } while (0)

bool valid_seq(const qc_ctx* c, int32_t s) {
  return s >= 0 && s < (int32_t)c->seqs.size() && c->seqs[s].live;
}

// ---- page allocator
int32_t page_alloc(qc_ctx* c) {
  if (c->free_pages.empty()) return -1;
  const int32_t p = c->free_pages.back();
  c->free_pages.pop_back();
  c->page_ref[p] = 1;
  return p;
}
void page_decref(qc_ctx* c, int32_t p) {
  if (--c->page_ref[p] == 0) c->free_pages.push_back(p);
}

void set_row(qc_ctx* c, int32_t s) {
  Seq& q = c->seqs[s];
  int32_t* row = &c->h_page_table[(size_t)s * c->pt_stride];
  std::fill(row, row + c->pt_stride, -1);
  std::copy(q.pages.begin(), q.pages.end(), row);
  q.dirty = true;
}

// ---- pinned staging
// Returns a pinned buffer whose previous upload has completed.
int stage_acquire(qc_ctx* c, size_t bytes, char** out, int* idx) {
  if (bytes > c->stage_cap)
    return fail(c, QC_ERR_ARG, "upload of %zu bytes exceeds staging capacity %zu", bytes,
                c->stage_cap);
  const int i = c->stage_next;
  c->stage_next = (i + 1) % STAGING_SLOTS;
  QC_CUDA(c, cudaEventSynchronize(c->stage_ev[i]));
  *out = c->stage[i];
  *idx = i;
  return QC_OK;
}
int stage_release(qc_ctx* c, int i, cudaStream_t s) {
  QC_CUDA(c, cudaEventRecord(c->stage_ev[i], s));
  return QC_OK;
}

// Upload every dirty page-table row.
int sync_rows(qc_ctx* c, cudaStream_t s) {
  // the dirty rows go up as one copy of the span that holds them when it fits
  // the staging buffer (a batched restore dirties one row per request), else
  // row by row
  int64_t lo = -1, hi = -1;
  for (size_t i = 0; i < c->seqs.size(); ++i)
    if (c->seqs[i].live && c->seqs[i].dirty) {
      if (lo < 0) lo = (int64_t)i;
      hi = (int64_t)i;
    }
  if (lo < 0) return QC_OK;
  const size_t row_bytes = (size_t)c->pt_stride * sizeof(int32_t);
  const size_t span = (size_t)(hi - lo + 1) * row_bytes;
  if (span <= c->stage_cap) {
    char* buf = nullptr;
    int si = 0;
    if (int rc0 = stage_acquire(c, span, &buf, &si)) return rc0;
    std::memcpy(buf, &c->h_page_table[lo * c->pt_stride], span);
    QC_CUDA(c, cudaMemcpyAsync(c->page_table + lo * c->pt_stride, buf, span,
                               cudaMemcpyHostToDevice, s));
    if (int rc = stage_release(c, si, s)) return rc;
    for (int64_t i = lo; i <= hi; ++i) c->seqs[i].dirty = false;
    return QC_OK;
  }
  for (size_t i = 0; i < c->seqs.size(); ++i) {
    Seq& q = c->seqs[i];
    if (!q.live || !q.dirty) continue;
    char* buf = nullptr;
    int si = 0;
    if (int rc0 = stage_acquire(c, row_bytes, &buf, &si)) return rc0;
    std::memcpy(buf, &c->h_page_table[i * c->pt_stride], row_bytes);
    QC_CUDA(c, cudaMemcpyAsync(c->page_table + i * c->pt_stride, buf, row_bytes,
                               cudaMemcpyHostToDevice, s));
    int rc = stage_release(c, si, s);
    if (rc) return rc;
    q.dirty = false;
  }
  return QC_OK;
}

// Run a list of copy jobs on the device (one launch).
int run_jobs(qc_ctx* c, const std::vector<CopyJob>& jobs, cudaStream_t s, int64_t* bytes_out) {
  if (jobs.empty()) return QC_OK;
  if ((int32_t)jobs.size() > c->job_cap)
    return fail(c, QC_ERR_ARG, "%zu copy jobs exceed capacity %d", jobs.size(), c->job_cap);
  std::vector<int64_t> starts(jobs.size() + 1, 0);
  int64_t total = 0;
  for (size_t j = 0; j < jobs.size(); ++j) {
    starts[j + 1] = starts[j] + (jobs[j].bytes + COPY_CHUNK - 1) / COPY_CHUNK;
    total += jobs[j].bytes;
  }
  const size_t jb = jobs.size() * sizeof(CopyJob), sb = starts.size() * sizeof(int64_t);
  char* buf = nullptr;
  int si = 0;
  if (int rc0 = stage_acquire(c, jb + sb, &buf, &si)) return rc0;
  std::memcpy(buf, jobs.data(), jb);
  std::memcpy(buf + jb, starts.data(), sb);
  QC_CUDA(c, cudaMemcpyAsync(c->jobs, buf, jb, cudaMemcpyHostToDevice, s));
  QC_CUDA(c, cudaMemcpyAsync(c->chunk_start, buf + jb, sb, cudaMemcpyHostToDevice, s));
  int rc = stage_release(c, si, s);
  if (rc) return rc;
  QC_CUDA(c, qc::launch_copy_jobs(c->jobs, (int32_t)jobs.size(), c->chunk_start, starts.back(),
                                  COPY_CHUNK, err_site(c, EK_COPY_JOBS, 0), s));
  if (bytes_out) *bytes_out += 2 * total;
  return QC_OK;
}

// Copy jobs duplicating page src into page dst for every attention layer.
void page_copy_jobs(const qc_ctx* c, int32_t src, int32_t dst, std::vector<CopyJob>& jobs) {
  const int64_t bytes = PAGE_ELEMS * 2;
  for (int l = 0; l < c->cfg.n_attn_layers; ++l) {
    const int64_t base = (int64_t)l * c->cfg.max_pages * PAGE_ELEMS;
    jobs.push_back({c->k_pool + base + src * PAGE_ELEMS, c->k_pool + base + dst * PAGE_ELEMS, bytes});
    jobs.push_back({c->v_pool + base + src * PAGE_ELEMS, c->v_pool + base + dst * PAGE_ELEMS, bytes});
  }
}

float* slot_state(const qc_ctx* c, int32_t s, int layer) {
  return c->state + ((int64_t)s * c->cfg.n_gdn_layers + layer) * QC_GDN_STATE;
}
uint16_t* slot_ring(const qc_ctx* c, int32_t s, int layer) {
  return c->ring + ((int64_t)s * c->cfg.n_gdn_layers + layer) * RING_ELEMS;
}
float* snap_state_ptr(const qc_ctx* c, int32_t snap) {
  return c->snap_state + (int64_t)snap * c->cfg.n_gdn_layers * QC_GDN_STATE;
}
uint16_t* snap_hist_ptr(const qc_ctx* c, int32_t snap, int layer) {
  return c->snap_hist + ((int64_t)snap * c->cfg.n_gdn_layers + layer) * HIST_ELEMS;
}

// ---- prefix hashing: 64-bit mix of the previous hash and a page of tokens.
constexpr uint64_t HASH_SEED = 0x9e3779b97f4a7c15ull;
uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}
uint64_t page_hash(uint64_t prev, const int32_t* t) {
  uint64_t h = mix64(prev ^ 0x51afd7ed558ccd6dull);
  for (int i = 0; i < PAGE; ++i) h = mix64(h ^ (uint32_t)t[i]) + (uint64_t)i;
  return h;
}

int free_seq_pages(qc_ctx* c, int32_t s) {
  Seq& q = c->seqs[s];
  for (int32_t p : q.pages) page_decref(c, p);
  q.pages.clear();
  set_row(c, s);
  return QC_OK;
}

}  // namespace

extern "C" {

// Message of a failed qc_create (which returns no context) on this thread.
static thread_local std::string g_create_err;

const char* qc_last_error(const qc_ctx* ctx) { return ctx ? ctx->err.c_str() : g_create_err.c_str(); }

}  // extern "C"

void qc::set_thread_error(const char* msg) { g_create_err = msg; }

extern "C" {

int qc_create(const qc_config* cfg, int device, qc_ctx** out) {
  if (!cfg || !out) return QC_ERR_ARG;
  *out = nullptr;
  if (cfg->n_attn_layers < 0 || cfg->n_gdn_layers < 0 ||
      cfg->n_attn_layers + cfg->n_gdn_layers <= 0 || cfg->max_seqs <= 0 ||
      cfg->max_pages <= 0 || cfg->max_ctx <= 0 || cfg->max_batch <= 0 ||
      cfg->max_snapshots < 0 || cfg->max_batch > cfg->max_seqs ||
      (cfg->flags & ~QC_FLAG_REFERENCE_MATH) != 0)
    return QC_ERR_ARG;
  qc_ctx* c = new qc_ctx();
  c->cfg = *cfg;
  c->device = device;
  c->ref_math = (cfg->flags & QC_FLAG_REFERENCE_MATH) ? 1 : 0;
  c->host_only = true;  // becomes false once the device pools exist
  c->pt_stride = (cfg->max_ctx + PAGE - 1) / PAGE + 1;
  c->seqs.resize(cfg->max_seqs);
  c->page_ref.assign(cfg->max_pages, 0);
  for (int32_t p = cfg->max_pages - 1; p >= 0; --p) c->free_pages.push_back(p);
  c->h_page_table.assign((size_t)cfg->max_seqs * c->pt_stride, -1);
  c->entries.reserve(64);
  for (int32_t s = cfg->max_snapshots - 1; s >= 0; --s) c->free_snaps.push_back(s);
  if (device == QC_DEVICE_NONE) {
    *out = c;
    return QC_OK;
  }

  // On failure the partial context is released and the message kept for
  // qc_last_error(NULL).
  auto cuda_fail = [&](cudaError_t e, const char* what) {
    char buf[256];
    snprintf(buf, sizeof(buf), "qc_create: %s: %s", what, cudaGetErrorString(e));
    g_create_err = buf;
    c->host_only = false;
    qc_destroy(c);
    return e == cudaErrorMemoryAllocation ? QC_ERR_OOM : QC_ERR_CUDA;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaDeviceGetAttribute(&c->nsm, cudaDevAttrMultiProcessorCount, device);
  const int na = cfg->n_attn_layers, ng = cfg->n_gdn_layers;
  const int64_t pool = (int64_t)std::max(na, 1) * cfg->max_pages * PAGE_ELEMS;
  c->part_slots = 4 * cfg->max_batch + c->nsm + 8;
  c->pf_split = (c->nsm + 3) / 4;
  c->job_cap = cfg->max_batch * (1 + 3 * std::max(ng, 1) + 2 * na) + 64;
  c->err_layers = std::max({na, ng, 1});
  struct A { void** p; size_t bytes; const char* what; };
  const A allocs[] = {
      {(void**)&c->k_pool, (size_t)pool * 2, "k_pool"},
      {(void**)&c->v_pool, (size_t)pool * 2, "v_pool"},
      {(void**)&c->state, (size_t)cfg->max_seqs * std::max(ng, 1) * QC_GDN_STATE * 4, "state"},
      {(void**)&c->ring, (size_t)cfg->max_seqs * std::max(ng, 1) * RING_ELEMS * 2, "ring"},
      {(void**)&c->snap_state, (size_t)std::max(cfg->max_snapshots, 1) * std::max(ng, 1) * QC_GDN_STATE * 4, "snap_state"},
      {(void**)&c->snap_hist, (size_t)std::max(cfg->max_snapshots, 1) * std::max(ng, 1) * HIST_ELEMS * 2, "snap_hist"},
      {(void**)&c->q_norm, (size_t)std::max(na, 1) * HD * 4, "q_norm"},
      {(void**)&c->k_norm, (size_t)std::max(na, 1) * HD * 4, "k_norm"},
      {(void**)&c->ssm_a, (size_t)std::max(ng, 1) * 32 * 4, "ssm_a"},
      {(void**)&c->dt_bias, (size_t)std::max(ng, 1) * 32 * 4, "dt_bias"},
      {(void**)&c->ssm_norm, (size_t)std::max(ng, 1) * 128 * 4, "ssm_norm"},
      {(void**)&c->conv_w, (size_t)std::max(ng, 1) * 4 * QC_CONV_CH * 4, "conv_w"},
      {(void**)&c->rope_cos, (size_t)cfg->max_ctx * 32 * 4, "rope_cos"},
      {(void**)&c->rope_sin, (size_t)cfg->max_ctx * 32 * 4, "rope_sin"},
      {(void**)&c->page_table, (size_t)cfg->max_seqs * c->pt_stride * 4, "page_table"},
      {(void**)&c->desc, (size_t)(5 * cfg->max_batch + 8) * 4, "desc"},
      {(void**)&c->desc_part, 16 * 4, "desc_part"},  // see qc_decode_begin
      {(void**)&c->part_m, (size_t)c->part_slots * 4 * 4, "part_m"},
      {(void**)&c->part_l, (size_t)c->part_slots * 4 * 4, "part_l"},
      {(void**)&c->part_o, (size_t)c->part_slots * 4 * HD * 4, "part_o"},
      {(void**)&c->jobs, (size_t)c->job_cap * sizeof(CopyJob), "jobs"},
      {(void**)&c->chunk_start, (size_t)(c->job_cap + 1) * 8, "chunk_start"},
      {(void**)&c->dev_err, (size_t)EK_COUNT * c->err_layers * 4, "dev_err"},
      {(void**)&c->pf_q, (size_t)4 * 4 * QC_PREFILL_CHUNK * HD * 2, "prefill q"},
      {(void**)&c->pf_conv, (size_t)QC_PREFILL_CHUNK * QC_CONV_CH * 4, "prefill conv"},
      {(void**)&c->pf_rec, (size_t)4 * c->pf_split * 4 * QC_PREFILL_CHUNK * (HD + 4) * 4,
       "prefill records"},
  };
  for (const A& a : allocs) {
    e = cudaMalloc(a.p, a.bytes);
    if (e != cudaSuccess) return cuda_fail(e, a.what);
  }
  // zeroed pools: rows past a page's valid length may enter a tensor-core
  // product multiplied by zero, so they must never hold NaN bit patterns
  if ((e = cudaMemset(c->k_pool, 0, (size_t)pool * 2)) ||
      (e = cudaMemset(c->v_pool, 0, (size_t)pool * 2)))
    return cuda_fail(e, "cudaMemset");
  // zeroed state so that a fresh sequence equals reset_state()
  if ((e = cudaMemset(c->state, 0, (size_t)cfg->max_seqs * std::max(ng, 1) * QC_GDN_STATE * 4)) ||
      (e = cudaMemset(c->ring, 0, (size_t)cfg->max_seqs * std::max(ng, 1) * RING_ELEMS * 2)) ||
      (e = cudaMemset(c->page_table, 0xff, (size_t)cfg->max_seqs * c->pt_stride * 4)) ||
      (e = cudaMemset(c->dev_err, 0, (size_t)EK_COUNT * c->err_layers * 4)))
    return cuda_fail(e, "cudaMemset");

  // RoPE table, the formula of precompute_rope (src/engine.cpp:2408-2420)
  {
    std::vector<float> cs((size_t)cfg->max_ctx * 32), sn((size_t)cfg->max_ctx * 32);
    float freq[32];
    for (int p = 0; p < 32; ++p) freq[p] = 1.0f / powf(10000000.0f, 2.0f * p / QC_ROPE_DIM);
    for (int pos = 0; pos < cfg->max_ctx; ++pos)
      for (int p = 0; p < 32; ++p) {
        const float theta = pos * freq[p];
        cs[(size_t)pos * 32 + p] = cosf(theta);
        sn[(size_t)pos * 32 + p] = sinf(theta);
      }
    if ((e = cudaMemcpy(c->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice)) ||
        (e = cudaMemcpy(c->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice)))
      return cuda_fail(e, "rope upload");
  }
  // TMA tensor maps over each layer's K and V pool: [rows][256] bf16 with
  // rows = max_pages * 4 kv-heads * 64 positions, KV_BOX_ROWS x 64 boxes, 128 B swizzle
  {
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    cudaDriverEntryPointQueryResult qres;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&encode, cudaEnableDefault, &qres);
    if (e != cudaSuccess || !encode || qres != cudaDriverEntryPointSuccess)
      return cuda_fail(e != cudaSuccess ? e : cudaErrorNotSupported, "cuTensorMapEncodeTiled");
    c->tm_k.resize(na);
    c->tm_v.resize(na);
    const cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)cfg->max_pages * QC_N_HEAD_KV * PAGE};
    const cuuint64_t strides[1] = {(cuuint64_t)HD * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)qc::KV_BOX_ROWS};
    const cuuint32_t estr[2] = {1, 1};
    for (int l = 0; l < na; ++l)
      for (int kv = 0; kv < 2; ++kv) {
        uint16_t* base = (kv ? c->v_pool : c->k_pool) + (int64_t)l * cfg->max_pages * PAGE_ELEMS;
        CUresult r = encode(kv ? &c->tm_v[l] : &c->tm_k[l], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                            base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return cuda_fail(cudaErrorInvalidValue, "tensor map encode");
      }
  }
  c->stage_cap = std::max<size_t>((size_t)(5 * cfg->max_batch + 8) * 4 +
                                      (size_t)c->pt_stride * 4,
                                  (size_t)c->job_cap * (sizeof(CopyJob) + 8) + 8);
  for (int i = 0; i < STAGING_SLOTS; ++i) {
    if ((e = cudaMallocHost((void**)&c->stage[i], c->stage_cap)) ||
        (e = cudaEventCreateWithFlags(&c->stage_ev[i], cudaEventDisableTiming)))
      return cuda_fail(e, "staging");
  }
  c->host_only = false;
  *out = c;
  return QC_OK;
}

void qc_destroy(qc_ctx* c) {
  if (!c) return;
  if (!c->host_only) {
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < c->p2p_world; ++r)
      if (r != c->p2p_rank && c->peer_mbox[r]) cudaIpcCloseMemHandle(c->peer_mbox[r]);
    if (c->mbox) cudaFree(c->mbox);
    void* ptrs[] = {c->k_pool, c->v_pool, c->state, c->ring, c->snap_state, c->snap_hist,
                    c->q_norm, c->k_norm, c->ssm_a, c->dt_bias, c->ssm_norm, c->conv_w,
                    c->rope_cos, c->rope_sin, c->page_table, c->desc, c->desc_part, c->pf_q, c->pf_rec, c->pf_conv,
                    c->part_m, c->part_l,
                    c->part_o, c->jobs, c->chunk_start, c->dev_err};
    for (void* p : ptrs)
      if (p) cudaFree(p);
    for (int i = 0; i < STAGING_SLOTS; ++i) {
      if (c->stage[i]) cudaFreeHost(c->stage[i]);
      if (c->stage_ev[i]) cudaEventDestroy(c->stage_ev[i]);
    }
  }
  delete c;
}

int qc_check_device(qc_ctx* c, qc_stream stream) {
  if (!c) return QC_ERR_ARG;
  QC_NEED_DEVICE(c);
  QC_CUDA(c, cudaStreamSynchronize((cudaStream_t)stream));
  const size_t nw = (size_t)EK_COUNT * c->err_layers;
  std::vector<int> words(nw);
  QC_CUDA(c, cudaMemcpy(words.data(), c->dev_err, nw * 4, cudaMemcpyDeviceToHost));
  int code = 0, sites = 0;
  std::string where;
  for (size_t i = 0; i < nw; ++i) {
    if (!words[i]) continue;
    if (!code) {
      code = words[i];
      char buf[256];
      snprintf(buf, sizeof(buf), "%s, layer %d", kErrKindName[i / c->err_layers],
               (int)(i % c->err_layers));
      where = buf;
    }
    ++sites;
  }
  if (!code) return QC_OK;
  QC_CUDA(c, cudaMemset(c->dev_err, 0, nw * 4));
  for (int l = 0; l < c->err_layers; ++l)
    if (words[(size_t)EK_ATTN_MERGE * c->err_layers + l] == QC_ERR_TIMEOUT) c->p2p_poisoned = true;
  return fail(c, code, "device reported %s in %s%s", code == QC_ERR_TIMEOUT ? "a wait timeout"
              : code == QC_ERR_BOUNDS ? "an index out of bounds" : "an error",
              where.c_str(), sites > 1 ? " (and other launch sites)" : "");
}

int qc_set_attn_params(qc_ctx* c, int layer, const float* q_norm, const float* k_norm) {
  if (!c || !q_norm || !k_norm) return QC_ERR_ARG;
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  QC_NEED_DEVICE(c);
  QC_CUDA(c, cudaMemcpy(c->q_norm + layer * HD, q_norm, HD * 4, cudaMemcpyHostToDevice));
  QC_CUDA(c, cudaMemcpy(c->k_norm + layer * HD, k_norm, HD * 4, cudaMemcpyHostToDevice));
  return QC_OK;
}

int qc_set_gdn_params(qc_ctx* c, int layer, const float* ssm_a, const float* dt_bias,
                      const float* ssm_norm, const float* conv_w) {
  if (!c || !ssm_a || !dt_bias || !ssm_norm || !conv_w) return QC_ERR_ARG;
  if (layer < 0 || layer >= c->cfg.n_gdn_layers) return fail(c, QC_ERR_ARG, "gdn layer %d", layer);
  QC_NEED_DEVICE(c);
  QC_CUDA(c, cudaMemcpy(c->ssm_a + layer * 32, ssm_a, 32 * 4, cudaMemcpyHostToDevice));
  QC_CUDA(c, cudaMemcpy(c->dt_bias + layer * 32, dt_bias, 32 * 4, cudaMemcpyHostToDevice));
  QC_CUDA(c, cudaMemcpy(c->ssm_norm + layer * 128, ssm_norm, 128 * 4, cudaMemcpyHostToDevice));
  QC_CUDA(c, cudaMemcpy(c->conv_w + (int64_t)layer * 4 * QC_CONV_CH, conv_w, 4 * QC_CONV_CH * 4,
                        cudaMemcpyHostToDevice));
  return QC_OK;
}

// ----------------------------------------------------------------- sequences

int qc_seq_alloc(qc_ctx* c, int32_t* seq) {
  if (!c || !seq) return QC_ERR_ARG;
  for (int32_t s = 0; s < (int32_t)c->seqs.size(); ++s) {
    if (!c->seqs[s].live) {
      c->seqs[s] = Seq();
      c->seqs[s].live = true;
      set_row(c, s);
      *seq = s;
      return QC_OK;
    }
  }
  return fail(c, QC_ERR_OOM, "no free sequence slot (max_seqs %d)", c->cfg.max_seqs);
}

int qc_seq_reset(qc_ctx* c, int32_t s, qc_stream stream) {
  if (!c) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (c->in_step || c->in_prefill) return fail(c, QC_ERR_ARG, "reset inside an open step");
  free_seq_pages(c, s);
  c->seqs[s].len = 0;
  c->seqs[s].tokens.clear();
  if (!c->host_only) {
    const int ng = c->cfg.n_gdn_layers;
    if (ng > 0) {
      cudaStream_t st = (cudaStream_t)stream;
      QC_CUDA(c, cudaMemsetAsync(slot_state(c, s, 0), 0, (size_t)ng * QC_GDN_STATE * 4, st));
      QC_CUDA(c, cudaMemsetAsync(slot_ring(c, s, 0), 0, (size_t)ng * RING_ELEMS * 2, st));
    }
  }
  return QC_OK;
}

int qc_seq_free(qc_ctx* c, int32_t s) {
  if (!c) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (c->in_step || c->in_prefill) return fail(c, QC_ERR_ARG, "free inside an open step");
  free_seq_pages(c, s);
  c->seqs[s] = Seq();
  return QC_OK;
}

int qc_seq_len(const qc_ctx* c, int32_t s, int32_t* len) {
  if (!c || !len || !valid_seq(c, s)) return QC_ERR_ARG;
  *len = c->seqs[s].len;
  return QC_OK;
}

int qc_seq_pages(const qc_ctx* c, int32_t s, int32_t* pages, int32_t cap, int32_t* n_pages) {
  if (!c || !n_pages || !valid_seq(c, s)) return QC_ERR_ARG;
  const Seq& q = c->seqs[s];
  *n_pages = (int32_t)q.pages.size();
  if (pages)
    for (int32_t i = 0; i < std::min(cap, *n_pages); ++i) pages[i] = q.pages[i];
  return QC_OK;
}

int qc_seq_reserve(qc_ctx* c, int32_t s, int32_t new_len) {
  if (!c) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (c->in_step || c->in_prefill) return fail(c, QC_ERR_ARG, "reserve inside an open step");
  Seq& q = c->seqs[s];
  if (new_len < q.len || new_len > c->cfg.max_ctx)
    return fail(c, QC_ERR_ARG, "reserve %d: length %d, max_ctx %d", new_len, q.len, c->cfg.max_ctx);
  const int32_t need = (new_len + PAGE - 1) / PAGE;
  const size_t before = q.pages.size();
  while ((int32_t)q.pages.size() < need) {
    const int32_t p = page_alloc(c);
    if (p < 0) {
      while (q.pages.size() > before) {
        page_decref(c, q.pages.back());
        q.pages.pop_back();
      }
      return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
    }
    q.pages.push_back(p);
  }
  q.len = new_len;
  set_row(c, s);
  return QC_OK;
}

static int kv_check(qc_ctx* c, int32_t s, int layer, int32_t pos0, int32_t n, bool writing) {
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  const Seq& q = c->seqs[s];
  if (pos0 < 0 || n < 0 || (int64_t)pos0 + n > (int64_t)q.pages.size() * PAGE)
    return fail(c, QC_ERR_ARG, "positions [%d, %d) not backed (%zu pages)", pos0, pos0 + n,
                q.pages.size());
  if (writing)
    for (int32_t pg = pos0 / PAGE; n > 0 && pg <= (pos0 + n - 1) / PAGE; ++pg)
      if (c->page_ref[q.pages[pg]] > 1)
        return fail(c, QC_ERR_ARG, "page %d of sequence %d is shared (prefix cache)", pg, s);
  return QC_OK;
}

int qc_kv_write(qc_ctx* c, int32_t s, int layer, int32_t pos0, int32_t n, const uint16_t* k,
                const uint16_t* v, qc_stream stream) {
  if (!c || !k || !v) return QC_ERR_ARG;
  int rc = kv_check(c, s, layer, pos0, n, true);
  if (rc) return rc;
  QC_NEED_DEVICE(c);
  cudaStream_t st = (cudaStream_t)stream;
  if ((rc = sync_rows(c, st))) return rc;
  const int64_t base = (int64_t)layer * c->cfg.max_pages * PAGE_ELEMS;
  // a write inside an open step: this layer's attention call of the step must
  // not read its pool before this copy completes (see AttnArgs::early)
  if (c->in_step) c->attn_ran[layer] = 1;
  QC_CUDA(c, qc::launch_kv_scatter(c->k_pool + base, c->v_pool + base,
                                   c->page_table + (int64_t)s * c->pt_stride, pos0, n, k, v,
                                   c->cfg.max_pages, err_site(c, EK_KV_COPY, layer), st));
  return QC_OK;
}

int qc_kv_read(qc_ctx* c, int32_t s, int layer, int32_t pos0, int32_t n, uint16_t* k,
               uint16_t* v, qc_stream stream) {
  if (!c || !k || !v) return QC_ERR_ARG;
  int rc = kv_check(c, s, layer, pos0, n, false);
  if (rc) return rc;
  QC_NEED_DEVICE(c);
  cudaStream_t st = (cudaStream_t)stream;
  if ((rc = sync_rows(c, st))) return rc;
  const int64_t base = (int64_t)layer * c->cfg.max_pages * PAGE_ELEMS;
  QC_CUDA(c, qc::launch_kv_gather(c->k_pool + base, c->v_pool + base,
                                  c->page_table + (int64_t)s * c->pt_stride, pos0, n, k, v,
                                  c->cfg.max_pages, err_site(c, EK_KV_COPY, layer), st));
  return QC_OK;
}

int qc_gdn_state_write(qc_ctx* c, int32_t s, int layer, const float* state,
                       const uint16_t* conv, qc_stream stream) {
  if (!c || !state || !conv) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (layer < 0 || layer >= c->cfg.n_gdn_layers) return fail(c, QC_ERR_ARG, "gdn layer %d", layer);
  QC_NEED_DEVICE(c);
  cudaStream_t st = (cudaStream_t)stream;
  // a write inside an open step: this layer's DeltaNet call of the step must
  // not read the state before the write completes (see GdnArgs::early)
  if (c->in_step) c->gdn_ran[layer] = 1;
  QC_CUDA(c, cudaMemcpyAsync(slot_state(c, s, layer), state, (size_t)QC_GDN_STATE * 4,
                             cudaMemcpyDeviceToDevice, st));
  QC_CUDA(c, qc::launch_hist_to_ring(conv, c->seqs[s].len, slot_ring(c, s, layer), st));
  return QC_OK;
}

int qc_gdn_state_read(qc_ctx* c, int32_t s, int layer, float* state, uint16_t* conv,
                      qc_stream stream) {
  if (!c || !state || !conv) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (layer < 0 || layer >= c->cfg.n_gdn_layers) return fail(c, QC_ERR_ARG, "gdn layer %d", layer);
  QC_NEED_DEVICE(c);
  cudaStream_t st = (cudaStream_t)stream;
  QC_CUDA(c, cudaMemcpyAsync(state, slot_state(c, s, layer), (size_t)QC_GDN_STATE * 4,
                             cudaMemcpyDeviceToDevice, st));
  QC_CUDA(c, qc::launch_ring_to_hist(slot_ring(c, s, layer), c->seqs[s].len, conv, st));
  return QC_OK;
}

// --------------------------------------------------------------- decode step

int qc_decode_begin(qc_ctx* c, const int32_t* seq_ids, int32_t n, const int32_t* tokens,
                    qc_stream stream) {
  qc::TraceRange trace_("qc_decode_begin");
  if (!c || !seq_ids) return QC_ERR_ARG;
  if (c->in_step) return fail(c, QC_ERR_ARG, "decode step already open");
  if (c->in_prefill) return fail(c, QC_ERR_ARG, "prefill chunk open");
  if (n <= 0 || n > c->cfg.max_batch)
    return fail(c, QC_ERR_ARG, "batch of %d (max_batch %d)", n, c->cfg.max_batch);
  cudaStream_t st = (cudaStream_t)stream;
  std::vector<CopyJob> cow;
  std::vector<char> seen(c->seqs.size(), 0);
  for (int32_t i = 0; i < n; ++i) {
    const int32_t s = seq_ids[i];
    if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
    if (seen[s]) return fail(c, QC_ERR_ARG, "sequence %d twice in one batch", s);
    seen[s] = 1;
    if (c->seqs[s].len >= c->cfg.max_ctx)
      return fail(c, QC_ERR_ARG, "sequence %d is full (max_ctx %d)", s, c->cfg.max_ctx);
  }
  {
    // pages this step takes (a fresh page at a page boundary, a private copy
    // of a shared tail page), counted before anything changes so that an
    // exhausted pool leaves every sequence as it was
    std::unordered_map<int32_t, int32_t> refs;  // tail page -> sharers left
    size_t need = 0;
    for (int32_t i = 0; i < n; ++i) {
      const Seq& q = c->seqs[seq_ids[i]];
      const int32_t pi = q.len / PAGE;
      if (pi == (int32_t)q.pages.size()) {
        ++need;
        continue;
      }
      auto it = refs.emplace(q.pages[pi], c->page_ref[q.pages[pi]]).first;
      if (it->second > 1) {
        ++need;
        --it->second;
      }
    }
    if (need > c->free_pages.size())
      return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
  }
  for (int32_t i = 0; i < n; ++i) {
    Seq& q = c->seqs[seq_ids[i]];
    const int32_t pi = q.len / PAGE;
    if (pi == (int32_t)q.pages.size()) {
      const int32_t p = page_alloc(c);
      if (p < 0) return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
      q.pages.push_back(p);
      set_row(c, seq_ids[i]);
    } else if (c->page_ref[q.pages[pi]] > 1) {  // shared tail page: copy on write
      const int32_t p = page_alloc(c);
      if (p < 0) return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
      if (!c->host_only) page_copy_jobs(c, q.pages[pi], p, cow);
      page_decref(c, q.pages[pi]);
      q.pages[pi] = p;
      set_row(c, seq_ids[i]);
    }
  }
  c->b_seq.assign(seq_ids, seq_ids + n);
  c->b_pos.resize(n);
  c->b_seg.assign(n + 1, 0);
  for (int32_t i = 0; i < n; ++i) {
    const Seq& q = c->seqs[seq_ids[i]];
    c->b_pos[i] = q.len;
    c->b_seg[i + 1] = c->b_seg[i] + 4 * (q.len / PAGE + 1);
  }
  c->b_has_tok = tokens != nullptr;
  if (tokens) c->b_tok.assign(tokens, tokens + n);
  // split-K sizes live in the device descriptor, so that a captured graph of
  // the layer calls stays valid as the contexts grow; the grid is the SM count
  c->b_total = c->b_seg[n];
  c->b_grid = c->nsm;
  c->b_per = (c->b_total + c->b_grid - 1) / c->b_grid;
  if (!c->host_only) {
    int rc = run_jobs(c, cow, st, nullptr);
    if (rc) return rc;
    if ((rc = sync_rows(c, st))) return rc;
    const size_t words = 5 * (size_t)n + 3;
    char* buf = nullptr;
    int si = 0;
    if ((rc = stage_acquire(c, words * 4, &buf, &si))) return rc;
    int32_t* d = reinterpret_cast<int32_t*>(buf);
    // layout: slots[n] | pos[n] | seg[n+1] | page0[n] | append[n] | total, per
    for (int32_t i = 0; i < n; ++i) {
      d[i] = seq_ids[i];
      d[n + i] = c->b_pos[i];
      d[3 * n + 1 + i] = 0;
      d[4 * n + 1 + i] = 1;
    }
    for (int32_t i = 0; i <= n; ++i) d[2 * n + i] = c->b_seg[i];
    d[5 * n + 1] = c->b_total;
    d[5 * n + 2] = c->b_per;
    QC_CUDA(c, cudaMemcpyAsync(c->desc, buf, words * 4, cudaMemcpyHostToDevice, st));
    if ((rc = stage_release(c, si, st))) return rc;
  }
  c->in_step = true;
  c->gdn_ran.assign(std::max(c->cfg.n_gdn_layers, 1), 0);
  c->attn_ran.assign(std::max(c->cfg.n_attn_layers, 1), 0);
  return QC_OK;
}

int qc_attn_decode(qc_ctx* c, int layer, const uint16_t* proj, uint16_t* out, qc_stream stream) {
  qc::TraceRange trace_("qc_attn_decode");
  if (!c || !proj || !out) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  QC_NEED_DEVICE(c);
  const int32_t n = (int32_t)c->b_seq.size();
  const int64_t base = (int64_t)layer * c->cfg.max_pages * PAGE_ELEMS;
  qc::AttnArgs a{};
  a.proj = proj;
  a.k_pool = c->k_pool + base;
  a.v_pool = c->v_pool + base;
  a.page_table = c->page_table;
  a.pt_stride = c->pt_stride;
  a.max_pages = c->cfg.max_pages;
  a.slots = c->desc;
  a.pos = c->desc + n;
  a.seg = c->desc + 2 * n;
  a.page0 = c->desc + 3 * n + 1;
  a.append = c->desc + 4 * n + 1;
  a.q_norm = c->q_norm + layer * HD;
  a.k_norm = c->k_norm + layer * HD;
  a.rope_cos = c->rope_cos;
  a.rope_sin = c->rope_sin;
  a.part_m = c->part_m;
  a.part_l = c->part_l;
  a.part_o = c->part_o;
  a.split = c->desc + 5 * n + 1;
  a.per_hint = c->b_per;
  a.n = n;
  a.grid = c->b_grid;
  a.err = err_site(c, EK_ATTN_DECODE, layer);
  // K/V streams before the previous kernel completes only if this layer's
  // pool has not been written in this step (its own call appends)
  a.early = c->attn_ran[layer] ? 0 : 1;
  c->attn_ran[layer] = 1;
  qc::CombineArgs cb{};
  cb.ref_math = c->ref_math;
  cb.proj = proj;
  cb.out = out;
  cb.seg = a.seg;
  cb.part_m = c->part_m;
  cb.part_l = c->part_l;
  cb.part_o = c->part_o;
  cb.split = a.split;
  cb.n = n;
  QC_CUDA(c, qc::launch_attn_decode(a, cb, c->tm_k[layer], c->tm_v[layer], (cudaStream_t)stream));
  return QC_OK;
}

int qc_gdn_decode(qc_ctx* c, int layer, const uint16_t* proj, uint16_t* out, qc_stream stream) {
  qc::TraceRange trace_("qc_gdn_decode");
  if (!c || !proj || !out) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  if (layer < 0 || layer >= c->cfg.n_gdn_layers) return fail(c, QC_ERR_ARG, "gdn layer %d", layer);
  QC_NEED_DEVICE(c);
  const int32_t n = (int32_t)c->b_seq.size();
  qc::GdnArgs g{};
  g.ref_math = c->ref_math;
  g.proj = proj;
  g.out = out;
  g.state = slot_state(c, 0, layer);
  g.ring = slot_ring(c, 0, layer);
  g.state_stride = (int64_t)c->cfg.n_gdn_layers * QC_GDN_STATE;
  g.ring_stride = (int64_t)c->cfg.n_gdn_layers * RING_ELEMS;
  g.conv_w = c->conv_w + (int64_t)layer * 4 * QC_CONV_CH;
  g.ssm_a = c->ssm_a + layer * 32;
  g.dt_bias = c->dt_bias + layer * 32;
  g.ssm_norm = c->ssm_norm + layer * 128;
  g.slots = c->desc;
  g.pos = c->desc + n;
  g.n = n;
  g.err = err_site(c, EK_GDN_DECODE, layer);
  // the kernel may read this layer's state before the previous kernel on the
  // stream completes only if no kernel of this step has written it yet
  g.early = c->gdn_ran[layer] ? 0 : 1;
  c->gdn_ran[layer] = 1;
  QC_CUDA(c, qc::launch_gdn_decode(g, (cudaStream_t)stream));
  return QC_OK;
}

int qc_decode_end(qc_ctx* c) {
  if (!c) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  for (size_t i = 0; i < c->b_seq.size(); ++i) {
    Seq& q = c->seqs[c->b_seq[i]];
    if (c->b_has_tok && q.tokens.size() == (size_t)q.len) q.tokens.push_back(c->b_tok[i]);
    q.len += 1;
  }
  c->in_step = false;
  return QC_OK;
}

int qc_decode_abort(qc_ctx* c) {
  if (!c) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  c->in_step = false;
  return QC_OK;
}

// ------------------------------------------------------------------ prefill

int qc_prefill_begin(qc_ctx* c, int32_t s, int32_t n, const int32_t* tokens, qc_stream stream) {
  if (!c) return QC_ERR_ARG;
  if (c->in_step || c->in_prefill) return fail(c, QC_ERR_ARG, "a step is already open");
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (n < 1 || n > QC_PREFILL_CHUNK)
    return fail(c, QC_ERR_ARG, "prefill of %d tokens (1..%d)", n, QC_PREFILL_CHUNK);
  Seq& q = c->seqs[s];
  if (q.len + n > c->cfg.max_ctx)
    return fail(c, QC_ERR_ARG, "sequence %d: %d + %d tokens exceed max_ctx %d", s, q.len, n,
                c->cfg.max_ctx);
  std::vector<CopyJob> cow;
  const int32_t first = q.len / PAGE, last = (q.len + n - 1) / PAGE;
  const bool shared_tail = first < (int32_t)q.pages.size() && c->page_ref[q.pages[first]] > 1;
  // checked before anything changes: an exhausted pool leaves the sequence
  // as it was
  const size_t need = (shared_tail ? 1 : 0) +
                      (size_t)std::max<int32_t>(0, last + 1 - (int32_t)q.pages.size());
  if (need > c->free_pages.size())
    return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
  if (shared_tail) {
    const int32_t p = page_alloc(c);
    if (p < 0) return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
    if (!c->host_only) page_copy_jobs(c, q.pages[first], p, cow);
    page_decref(c, q.pages[first]);
    q.pages[first] = p;
  }
  const size_t before = q.pages.size();
  while ((int32_t)q.pages.size() <= last) {
    const int32_t p = page_alloc(c);
    if (p < 0) {
      while (q.pages.size() > before) {
        page_decref(c, q.pages.back());
        q.pages.pop_back();
      }
      return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
    }
    q.pages.push_back(p);
  }
  set_row(c, s);
  if (!c->host_only) {
    cudaStream_t st = (cudaStream_t)stream;
    int rc = run_jobs(c, cow, st, nullptr);
    if (rc) return rc;
    if ((rc = sync_rows(c, st))) return rc;
  }
  c->in_prefill = true;
  c->p_seq = s;
  c->p_pos0 = q.len;
  c->p_n = n;
  c->p_tok.clear();
  if (tokens) c->p_tok.assign(tokens, tokens + n);
  return QC_OK;
}

int qc_attn_prefill(qc_ctx* c, int layer, const uint16_t* proj, uint16_t* out, qc_stream stream) {
  qc::TraceRange trace_("qc_attn_prefill");
  if (!c || !proj || !out) return QC_ERR_ARG;
  if (!c->in_prefill) return fail(c, QC_ERR_ARG, "no open prefill chunk");
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  QC_NEED_DEVICE(c);
  const int64_t base = (int64_t)layer * c->cfg.max_pages * PAGE_ELEMS;
  qc::AttnPrefillArgs a{};
  a.ref_math = c->ref_math;
  a.proj = proj;
  a.out = out;
  a.k_pool = c->k_pool + base;
  a.v_pool = c->v_pool + base;
  a.page_row = c->page_table + (int64_t)c->p_seq * c->pt_stride;
  a.max_pages = c->cfg.max_pages;
  a.q_norm = c->q_norm + layer * HD;
  a.k_norm = c->k_norm + layer * HD;
  a.rope_cos = c->rope_cos;
  a.rope_sin = c->rope_sin;
  a.q_buf = c->pf_q;
  a.rec = c->pf_rec;
  a.pos0 = c->p_pos0;
  a.T = c->p_n;
  const int32_t n_pages = (c->p_pos0 + c->p_n + PAGE - 1) / PAGE;
  // at least 4 pages per CTA: each CTA's fixed cost (tensor-memory setup, the
  // 64 KiB q tile, a 133 KB record) must be spread over several tiles
  a.n_split = std::max(1, std::min(c->pf_split, n_pages / 4));
  a.err = err_site(c, EK_ATTN_PREFILL, layer);
  QC_CUDA(c, qc::launch_attn_prefill(a, c->tm_k[layer], c->tm_v[layer], (cudaStream_t)stream));
  return QC_OK;
}

int qc_gdn_prefill(qc_ctx* c, int layer, const uint16_t* proj, uint16_t* out, qc_stream stream) {
  qc::TraceRange trace_("qc_gdn_prefill");
  if (!c || !proj || !out) return QC_ERR_ARG;
  if (!c->in_prefill) return fail(c, QC_ERR_ARG, "no open prefill chunk");
  if (layer < 0 || layer >= c->cfg.n_gdn_layers) return fail(c, QC_ERR_ARG, "gdn layer %d", layer);
  QC_NEED_DEVICE(c);
  qc::GdnPrefillArgs g{};
  g.ref_math = c->ref_math;
  g.proj = proj;
  g.out = out;
  g.state = slot_state(c, c->p_seq, layer);
  g.ring = slot_ring(c, c->p_seq, layer);
  g.conv_w = c->conv_w + (int64_t)layer * 4 * QC_CONV_CH;
  g.ssm_a = c->ssm_a + layer * 32;
  g.dt_bias = c->dt_bias + layer * 32;
  g.ssm_norm = c->ssm_norm + layer * 128;
  g.conv_out = c->pf_conv;
  g.pos0 = c->p_pos0;
  g.T = c->p_n;
  QC_CUDA(c, qc::launch_gdn_prefill(g, (cudaStream_t)stream));
  return QC_OK;
}

int qc_prefill_end(qc_ctx* c) {
  if (!c) return QC_ERR_ARG;
  if (!c->in_prefill) return fail(c, QC_ERR_ARG, "no open prefill chunk");
  Seq& q = c->seqs[c->p_seq];
  if (!c->p_tok.empty() && q.tokens.size() == (size_t)q.len)
    q.tokens.insert(q.tokens.end(), c->p_tok.begin(), c->p_tok.end());
  q.len += c->p_n;
  c->in_prefill = false;
  return QC_OK;
}

// ------------------------------------------------------------- prefix cache

int qc_seq_match_prefix(qc_ctx* c, int32_t s, const int32_t* tokens, int32_t n,
                        int32_t* prefix_len, qc_stream stream) {
  qc::TraceRange trace_("qc_seq_match_prefix");
  if (!c || (!tokens && n > 0) || !prefix_len) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  const Seq& q = c->seqs[s];
  // An unknown history (state stood up without tokens) never matches.
  const bool known = q.tokens.size() == (size_t)q.len;
  const int32_t cache_len = q.len;
  int32_t prefix = 0;
  if (known) {
    const int32_t check = std::min(cache_len, n);
    while (prefix < check && tokens[prefix] == q.tokens[prefix]) ++prefix;
  }
  if (prefix < cache_len || prefix >= n) {  // diverged, or nothing left to prefill
    const bool empty = cache_len == 0;
    prefix = 0;
    if (!empty) {
      int rc = qc_seq_reset(c, s, stream);
      if (rc) return rc;
    }
  }
  *prefix_len = prefix;
  return QC_OK;
}

int qc_prefix_page_hashes(const int32_t* tokens, int32_t n, uint64_t* hashes) {
  if ((!tokens && n > 0) || !hashes || n < 0) return QC_ERR_ARG;
  uint64_t h = HASH_SEED;
  for (int32_t i = 0; i < n / PAGE; ++i) {
    h = page_hash(h, tokens + (int64_t)i * PAGE);
    hashes[i] = h;
  }
  return QC_OK;
}

int qc_prefix_insert(qc_ctx* c, int32_t s, const int32_t* tokens, int32_t n, int32_t* entry,
                     qc_stream stream) {
  qc::TraceRange trace_("qc_prefix_insert");
  if (!c || !tokens || !entry || n <= 0) return QC_ERR_ARG;
  if (!valid_seq(c, s)) return fail(c, QC_ERR_ARG, "sequence %d is not live", s);
  if (c->in_step || c->in_prefill) return fail(c, QC_ERR_ARG, "insert inside an open step");
  Seq& q = c->seqs[s];
  if (q.len != n) return fail(c, QC_ERR_ARG, "sequence length %d != %d tokens", q.len, n);
  if (q.tokens.size() == (size_t)n && !std::equal(tokens, tokens + n, q.tokens.begin()))
    return fail(c, QC_ERR_ARG, "tokens differ from the sequence history");
  if (c->free_snaps.empty()) return fail(c, QC_ERR_OOM, "no free snapshot slot");
  const int32_t full = n / PAGE;
  int32_t tail = -1;
  if (n % PAGE) {
    tail = page_alloc(c);
    if (tail < 0) return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
  }
  Entry e;
  e.live = true;
  e.P = n;
  e.tokens.assign(tokens, tokens + n);
  for (int32_t i = 0; i < full; ++i) {
    e.pages.push_back(q.pages[i]);
    c->page_ref[q.pages[i]] += 1;
  }
  if (tail >= 0) e.pages.push_back(tail);
  e.snap = c->free_snaps.back();
  c->free_snaps.pop_back();
  uint64_t h = HASH_SEED;
  for (int32_t i = 0; i < full; ++i) h = page_hash(h, tokens + (int64_t)i * PAGE);
  e.key = h;
  if (!c->host_only) {
    std::vector<CopyJob> jobs;
    const int ng = c->cfg.n_gdn_layers;
    if (ng > 0) {
      jobs.push_back({slot_state(c, s, 0), snap_state_ptr(c, e.snap), (int64_t)ng * QC_GDN_STATE * 4});
      for (int l = 0; l < ng; ++l)
        for (int j = 0; j < 3; ++j)
          jobs.push_back({slot_ring(c, s, l) + (int64_t)((n - 3 + j) & 3) * QC_CONV_CH,
                          snap_hist_ptr(c, e.snap, l) + (int64_t)j * QC_CONV_CH,
                          (int64_t)QC_CONV_CH * 2});
    }
    if (tail >= 0) page_copy_jobs(c, q.pages[full], tail, jobs);
    int rc = run_jobs(c, jobs, (cudaStream_t)stream, nullptr);
    if (rc) {  // give back what the entry took: page references, tail, slot
      for (int32_t p : e.pages) page_decref(c, p);
      c->free_snaps.push_back(e.snap);
      return rc;
    }
  }
  int32_t id = -1;
  for (int32_t i = 0; i < (int32_t)c->entries.size(); ++i)
    if (!c->entries[i].live) { id = i; break; }
  if (id < 0) {
    id = (int32_t)c->entries.size();
    c->entries.emplace_back();
  }
  c->index[e.key].push_back(id);
  c->entries[id] = std::move(e);
  *entry = id;
  return QC_OK;
}

int qc_prefix_lookup(qc_ctx* c, const int32_t* tokens, int32_t n, int32_t* matched,
                     int32_t* entry) {
  qc::TraceRange trace_("qc_prefix_lookup");
  if (!c || (!tokens && n > 0) || !matched || !entry) return QC_ERR_ARG;
  *matched = 0;
  *entry = -1;
  if (n <= 1) return QC_OK;
  const int32_t m = n / PAGE;
  std::vector<uint64_t> h(m + 1);
  h[0] = HASH_SEED;
  for (int32_t i = 0; i < m; ++i) h[i + 1] = page_hash(h[i], tokens + (int64_t)i * PAGE);
  for (int32_t j = m; j >= 0; --j) {
    auto it = c->index.find(h[j]);
    if (it == c->index.end()) continue;
    int32_t best = -1, best_p = 0;
    for (int32_t id : it->second) {
      const Entry& e = c->entries[id];
      if (!e.live || e.P / PAGE != j || e.P >= n || e.P <= best_p) continue;
      if (!std::equal(e.tokens.begin(), e.tokens.end(), tokens)) continue;  // verify ids
      best = id;
      best_p = e.P;
    }
    if (best >= 0) {
      *matched = best_p;
      *entry = best;
      return QC_OK;
    }
  }
  return QC_OK;
}

int qc_prefix_restore(qc_ctx* c, const int32_t* entries, const int32_t* seqs, int32_t n,
                      qc_stream stream) {
  qc::TraceRange trace_("qc_prefix_restore");
  if (!c || !entries || !seqs || n < 0) return QC_ERR_ARG;
  if (c->in_step || c->in_prefill) return fail(c, QC_ERR_ARG, "restore inside an open step");
  for (int32_t i = 0; i < n; ++i) {
    if (entries[i] < 0 || entries[i] >= (int32_t)c->entries.size() || !c->entries[entries[i]].live)
      return fail(c, QC_ERR_ARG, "entry %d is not live", entries[i]);
    if (!valid_seq(c, seqs[i])) return fail(c, QC_ERR_ARG, "sequence %d is not live", seqs[i]);
    if (c->seqs[seqs[i]].len != 0 || !c->seqs[seqs[i]].pages.empty())
      return fail(c, QC_ERR_ARG, "sequence %d is not empty (reset it first)", seqs[i]);
    for (int32_t k = 0; k < i; ++k)
      if (seqs[k] == seqs[i]) return fail(c, QC_ERR_ARG, "sequence %d restored twice", seqs[i]);
  }
  int32_t tails = 0;
  for (int32_t i = 0; i < n; ++i) tails += (c->entries[entries[i]].P % PAGE) ? 1 : 0;
  if (tails > (int32_t)c->free_pages.size())
    return fail(c, QC_ERR_OOM, "KV page pool exhausted (%d pages)", c->cfg.max_pages);
  std::vector<CopyJob> jobs;
  const int ng = c->cfg.n_gdn_layers;
  for (int32_t i = 0; i < n; ++i) {
    const Entry& e = c->entries[entries[i]];
    Seq& q = c->seqs[seqs[i]];
    const int32_t full = e.P / PAGE;
    for (int32_t k = 0; k < full; ++k) {  // page-list gather: share the full pages
      q.pages.push_back(e.pages[k]);
      c->page_ref[e.pages[k]] += 1;
    }
    if (e.P % PAGE) {  // tail page: copy on write
      const int32_t p = page_alloc(c);
      if (!c->host_only) page_copy_jobs(c, e.pages[full], p, jobs);
      q.pages.push_back(p);
    }
    q.len = e.P;
    q.tokens = e.tokens;
    set_row(c, seqs[i]);
    if (!c->host_only && ng > 0) {
      jobs.push_back({snap_state_ptr(c, e.snap), slot_state(c, seqs[i], 0),
                      (int64_t)ng * QC_GDN_STATE * 4});
      for (int l = 0; l < ng; ++l)
        for (int j = 0; j < 3; ++j)
          jobs.push_back({snap_hist_ptr(c, e.snap, l) + (int64_t)j * QC_CONV_CH,
                          slot_ring(c, seqs[i], l) + (int64_t)((e.P - 3 + j) & 3) * QC_CONV_CH,
                          (int64_t)QC_CONV_CH * 2});
    }
  }
  c->last_restore_bytes = 0;
  if (!c->host_only) {
    cudaStream_t st = (cudaStream_t)stream;
    int rc = run_jobs(c, jobs, st, &c->last_restore_bytes);
    if (rc) {  // the copies never ran: the sequences go back to empty
      for (int32_t i = 0; i < n; ++i) {
        Seq& q = c->seqs[seqs[i]];
        for (int32_t p : q.pages) page_decref(c, p);
        q.pages.clear();
        q.len = 0;
        q.tokens.clear();
        set_row(c, seqs[i]);
      }
      return rc;
    }
    if ((rc = sync_rows(c, st))) return rc;
    // the page-table rows are part of the restore traffic
    c->last_restore_bytes += 2LL * n * c->pt_stride * 4;
  }
  return QC_OK;
}

int qc_prefix_release(qc_ctx* c, int32_t id) {
  if (!c) return QC_ERR_ARG;
  if (id < 0 || id >= (int32_t)c->entries.size() || !c->entries[id].live)
    return fail(c, QC_ERR_ARG, "entry %d is not live", id);
  Entry& e = c->entries[id];
  for (int32_t p : e.pages) page_decref(c, p);
  auto& v = c->index[e.key];
  v.erase(std::remove(v.begin(), v.end(), id), v.end());
  if (v.empty()) c->index.erase(e.key);
  c->free_snaps.push_back(e.snap);
  e = Entry();
  return QC_OK;
}

int qc_prefix_last_restore_bytes(const qc_ctx* c, int64_t* bytes) {
  if (!c || !bytes) return QC_ERR_ARG;
  *bytes = c->last_restore_bytes;
  return QC_OK;
}

// ------------------------------------------------- split-K across devices

int qc_attn_partial_range(qc_ctx* c, int32_t page_begin, int32_t page_end, int32_t append,
                          qc_stream stream) {
  if (!c) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  if (c->b_seq.size() != 1) return fail(c, QC_ERR_ARG, "split-K needs a batch of 1");
  QC_NEED_DEVICE(c);
  const int32_t s = c->b_seq[0], pos = c->b_pos[0];
  const Seq& q = c->seqs[s];
  if (page_begin < 0 || page_end < page_begin || page_end > (int32_t)q.pages.size())
    return fail(c, QC_ERR_ARG, "page range [%d, %d) outside the %zu mapped pages", page_begin,
                page_end, q.pages.size());
  const int32_t pos_page = pos / PAGE;
  if (append && (pos_page < page_begin || pos_page >= page_end))
    return fail(c, QC_ERR_ARG, "append requested but page %d of position %d is outside [%d, %d)",
                pos_page, pos, page_begin, page_end);
  if (!append && page_end > pos_page + (pos % PAGE ? 1 : 0))
    return fail(c, QC_ERR_ARG, "range [%d, %d) reaches past the cached positions (< %d)",
                page_begin, page_end, pos);
  cudaStream_t st = (cudaStream_t)stream;
  int rc = sync_rows(c, st);
  if (rc) return rc;
  const int32_t total = 4 * (page_end - page_begin);
  const int32_t per = std::max(1, (total + c->nsm - 1) / c->nsm);
  c->p_per = per;
  // one-sequence descriptor: slot | pos | seg[2] | page0 | append | total, per
  int32_t d[8] = {s, pos, 0, total, page_begin, append ? 1 : 0, total, per};
  char* buf = nullptr;
  int si = 0;
  if ((rc = stage_acquire(c, sizeof(d), &buf, &si))) return rc;
  std::memcpy(buf, d, sizeof(d));
  QC_CUDA(c, cudaMemcpyAsync(c->desc_part, buf, sizeof(d), cudaMemcpyHostToDevice, st));
  return stage_release(c, si, st);
}

int qc_attn_partial(qc_ctx* c, int layer, const uint16_t* proj, float* partial,
                    qc_stream stream) {
  qc::TraceRange trace_("qc_attn_partial");
  if (!c || !proj || !partial) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  if (c->b_seq.size() != 1) return fail(c, QC_ERR_ARG, "split-K needs a batch of 1");
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  QC_NEED_DEVICE(c);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t base = (int64_t)layer * c->cfg.max_pages * PAGE_ELEMS;
  qc::AttnArgs a{};
  a.proj = proj;
  a.k_pool = c->k_pool + base;
  a.v_pool = c->v_pool + base;
  a.page_table = c->page_table;
  a.pt_stride = c->pt_stride;
  a.max_pages = c->cfg.max_pages;
  a.slots = c->desc_part;
  a.pos = c->desc_part + 1;
  a.seg = c->desc_part + 2;
  a.page0 = c->desc_part + 4;
  a.append = c->desc_part + 5;
  a.split = c->desc_part + 6;
  a.per_hint = c->p_per;
  a.q_norm = c->q_norm + layer * HD;
  a.k_norm = c->k_norm + layer * HD;
  a.rope_cos = c->rope_cos;
  a.rope_sin = c->rope_sin;
  a.part_m = c->part_m;
  a.part_l = c->part_l;
  a.part_o = c->part_o;
  a.n = 1;
  a.grid = c->nsm;
  a.err = err_site(c, EK_ATTN_DECODE, layer);
  // K/V streams before the previous kernel completes only if this layer's
  // pool has not been written in this step (its own call appends)
  a.early = c->attn_ran[layer] ? 0 : 1;
  c->attn_ran[layer] = 1;
  qc::CombineArgs cb{};
  cb.ref_math = c->ref_math;
  cb.proj = proj;
  cb.out = nullptr;
  cb.seg = a.seg;
  cb.part_m = c->part_m;
  cb.part_l = c->part_l;
  cb.part_o = c->part_o;
  cb.split = a.split;
  cb.n = 1;
  cb.record = partial;
  QC_CUDA(c, qc::launch_attn_decode(a, cb, c->tm_k[layer], c->tm_v[layer], st));
  return QC_OK;
}

int qc_attn_combine(qc_ctx* c, const float* partials, int32_t n_parts, const uint16_t* proj,
                    uint16_t* out, qc_stream stream) {
  qc::TraceRange trace_("qc_attn_combine");
  if (!c || !partials || !proj || !out || n_parts <= 0) return QC_ERR_ARG;
  QC_NEED_DEVICE(c);
  QC_CUDA(c, qc::launch_attn_merge_records(partials, n_parts, proj, out, c->ref_math,
                                                  (cudaStream_t)stream));
  return QC_OK;
}


// Mailbox layout: records [2][n_attn_layers][world][16][258] f32, then
// counters [n_attn_layers][world] u32 (written by every rank), then this
// rank's own done[n_attn_layers] and consumed[n_attn_layers] u32.
static size_t mbox_rec_bytes(const qc_ctx* c, int world) {
  return (size_t)2 * c->cfg.n_attn_layers * world * 16 * 258 * sizeof(float);
}
// records, then counters [n_layers][world], done [n_layers], consumed
// [n_layers], and one poison word (set by a merge whose wait expired)
static size_t mbox_bytes(const qc_ctx* c, int world) {
  return mbox_rec_bytes(c, world) +
         ((size_t)c->cfg.n_attn_layers * (world + 2) + 1) * sizeof(uint32_t);
}

int qc_p2p_create(qc_ctx* c, int32_t world, int32_t rank, void* handle_out) {
  if (!c || !handle_out || world < 2 || world > QC_P2P_MAX_RANKS || rank < 0 || rank >= world)
    return c ? fail(c, QC_ERR_ARG, "qc_p2p_create: world %d rank %d", world, rank) : QC_ERR_ARG;
  QC_NEED_DEVICE(c);
  if (c->mbox) return fail(c, QC_ERR_ARG, "qc_p2p_create: mailbox already created");
  cudaSetDevice(c->device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, mbox_bytes(c, world));
  if (e != cudaSuccess) return fail(c, QC_ERR_OOM, "qc_p2p_create: %s", cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  if ((e = cudaMemset(p, 0, mbox_bytes(c, world))) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess ||
      (e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
    cudaFree(p);  // nothing half-made stays behind: the call may be retried
    return fail(c, QC_ERR_CUDA, "qc_p2p_create: %s", cudaGetErrorString(e));
  }
  c->mbox = static_cast<char*>(p);
  std::memcpy(handle_out, &h, sizeof(h));
  c->p2p_world = world;
  c->p2p_rank = rank;
  c->peer_mbox[rank] = c->mbox;
  return QC_OK;
}

int qc_p2p_open(qc_ctx* c, int32_t peer, const void* handle) {
  if (!c || !handle) return QC_ERR_ARG;
  QC_NEED_DEVICE(c);
  if (!c->mbox) return fail(c, QC_ERR_ARG, "qc_p2p_open: call qc_p2p_create first");
  if (peer < 0 || peer >= c->p2p_world || peer == c->p2p_rank)
    return fail(c, QC_ERR_ARG, "qc_p2p_open: peer %d", peer);
  if (c->peer_mbox[peer]) return fail(c, QC_ERR_ARG, "qc_p2p_open: peer %d already open", peer);
  cudaSetDevice(c->device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  QC_CUDA(c, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  c->peer_mbox[peer] = static_cast<char*>(p);
  return QC_OK;
}

static uint32_t* mbox_done(qc_ctx* c);

int qc_p2p_reset(qc_ctx* c, qc_stream stream) {
  qc::TraceRange trace_("qc_p2p_reset");
  if (!c) return QC_ERR_ARG;
  QC_NEED_DEVICE(c);
  if (!c->mbox) return fail(c, QC_ERR_ARG, "qc_p2p_reset: no peer mailbox (qc_p2p_create)");
  if (c->in_step) return fail(c, QC_ERR_ARG, "qc_p2p_reset: a decode step is open");
  cudaSetDevice(c->device);
  QC_CUDA(c, cudaStreamSynchronize((cudaStream_t)stream));
  // counters, done, consumed and the poison word; the records need no
  // clearing (a step's records are read only once its counters are complete)
  const size_t off = mbox_rec_bytes(c, c->p2p_world);
  QC_CUDA(c, cudaMemsetAsync(c->mbox + off, 0, mbox_bytes(c, c->p2p_world) - off,
                             (cudaStream_t)stream));
  QC_CUDA(c, cudaStreamSynchronize((cudaStream_t)stream));
  c->p2p_poisoned = false;
  return QC_OK;
}

static uint32_t* mbox_done(qc_ctx* c) {
  return reinterpret_cast<uint32_t*>(c->mbox + mbox_rec_bytes(c, c->p2p_world)) +
         (size_t)c->cfg.n_attn_layers * c->p2p_world;
}

static int p2p_ready(qc_ctx* c) {
  if (!c->mbox) return fail(c, QC_ERR_ARG, "no peer mailbox (qc_p2p_create)");
  if (c->p2p_poisoned)
    return fail(c, QC_ERR_ARG, "a peer-record wait expired: the mailbox step counts are out of "
                               "step until every rank has called qc_p2p_reset");
  for (int r = 0; r < c->p2p_world; ++r)
    if (!c->peer_mbox[r]) return fail(c, QC_ERR_ARG, "peer %d not opened (qc_p2p_open)", r);
  return QC_OK;
}

int qc_attn_partial_p2p(qc_ctx* c, int layer, const uint16_t* proj, qc_stream stream) {
  qc::TraceRange trace_("qc_attn_partial_p2p");
  if (!c || !proj) return QC_ERR_ARG;
  if (!c->in_step) return fail(c, QC_ERR_ARG, "no open decode step");
  if (c->b_seq.size() != 1) return fail(c, QC_ERR_ARG, "split-K needs a batch of 1");
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  QC_NEED_DEVICE(c);
  int rc = p2p_ready(c);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t base = (int64_t)layer * c->cfg.max_pages * PAGE_ELEMS;
  qc::AttnArgs a{};
  a.proj = proj;
  a.k_pool = c->k_pool + base;
  a.v_pool = c->v_pool + base;
  a.page_table = c->page_table;
  a.pt_stride = c->pt_stride;
  a.max_pages = c->cfg.max_pages;
  a.slots = c->desc_part;
  a.pos = c->desc_part + 1;
  a.seg = c->desc_part + 2;
  a.page0 = c->desc_part + 4;
  a.append = c->desc_part + 5;
  a.split = c->desc_part + 6;
  a.per_hint = c->p_per;
  a.q_norm = c->q_norm + layer * HD;
  a.k_norm = c->k_norm + layer * HD;
  a.rope_cos = c->rope_cos;
  a.rope_sin = c->rope_sin;
  a.part_m = c->part_m;
  a.part_l = c->part_l;
  a.part_o = c->part_o;
  a.n = 1;
  a.grid = c->nsm;
  a.err = err_site(c, EK_ATTN_DECODE, layer);
  // K/V streams before the previous kernel completes only if this layer's
  // pool has not been written in this step (its own call appends)
  a.early = c->attn_ran[layer] ? 0 : 1;
  c->attn_ran[layer] = 1;
  qc::CombineArgs cb{};
  cb.ref_math = c->ref_math;
  cb.proj = proj;
  cb.seg = a.seg;
  cb.part_m = c->part_m;
  cb.part_l = c->part_l;
  cb.part_o = c->part_o;
  cb.split = a.split;
  cb.n = 1;
  cb.world = c->p2p_world;
  cb.rank = c->p2p_rank;
  cb.layer = layer;
  cb.n_layers = c->cfg.n_attn_layers;
  for (int r = 0; r < c->p2p_world; ++r) {
    cb.mbox_rec[r] = reinterpret_cast<float*>(c->peer_mbox[r]);
    cb.mbox_cnt[r] = reinterpret_cast<uint32_t*>(c->peer_mbox[r] + mbox_rec_bytes(c, c->p2p_world));
  }
  cb.done = mbox_done(c);
  QC_CUDA(c, qc::launch_attn_decode(a, cb, c->tm_k[layer], c->tm_v[layer], st));
  return QC_OK;
}

int qc_attn_combine_p2p(qc_ctx* c, int layer, const uint16_t* proj, uint16_t* out,
                        qc_stream stream) {
  qc::TraceRange trace_("qc_attn_combine_p2p");
  if (!c || !proj || !out) return QC_ERR_ARG;
  if (layer < 0 || layer >= c->cfg.n_attn_layers) return fail(c, QC_ERR_ARG, "attn layer %d", layer);
  QC_NEED_DEVICE(c);
  int rc = p2p_ready(c);
  if (rc) return rc;
  qc::MailboxMergeArgs m{};
  m.ref_math = c->ref_math;
  m.rec = reinterpret_cast<const float*>(c->mbox);
  m.cnt = reinterpret_cast<const uint32_t*>(c->mbox + mbox_rec_bytes(c, c->p2p_world));
  m.done = mbox_done(c);
  m.consumed = mbox_done(c) + c->cfg.n_attn_layers;
  m.poison = mbox_done(c) + 2 * c->cfg.n_attn_layers;
  m.world = c->p2p_world;
  m.layer = layer;
  m.n_layers = c->cfg.n_attn_layers;
  m.proj = proj;
  m.out = out;
  m.err = err_site(c, EK_ATTN_MERGE, layer);
  QC_CUDA(c, qc::launch_attn_merge_mailbox(m, (cudaStream_t)stream));
  return QC_OK;
}
}  // extern "C"
