// kernels.h — launch interface between the host context (qcache.cu) and the
// device kernels.  Plain structs of device pointers and sizes.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include <nvtx3/nvToolsExt.h>

namespace qc {

// NVTX range around one C-ABI call (named in a profiler's timeline; a no-op
// when no tool is attached).
struct TraceRange {
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

// Which devices (ordinals below 64) have run a one-time setup, such as raising
// a kernel's dynamic shared-memory limit.  Safe to query from the host threads
// of several contexts at once; a device at or above 64 always reports "not
// done", so its setup simply repeats.
class PerDeviceOnce {
 public:
  bool done(int dev) const {
    return dev >= 0 && dev < 64 && ((bits_.load(std::memory_order_acquire) >> dev) & 1u);
  }
  void mark(int dev) {
    if (dev >= 0 && dev < 64) bits_.fetch_or(uint64_t(1) << dev, std::memory_order_release);
  }

 private:
  std::atomic<uint64_t> bits_{0};
};

// Rows of one TMA box of the K/V tensor maps (64 rows x 64 bf16 = 8 KiB,
// 128-byte swizzle); the decode and prefill tile loads and the map encoders
// agree on it.
constexpr int KV_BOX_ROWS = 64;


// Gated-DeltaNet decode step (gdn_decode.cu).
struct GdnArgs {
  const uint16_t* proj;      // [n][12352] bf16
  uint16_t* out;             // [n][4096] bf16
  float* state;              // this layer's state of slot 0; slot s at + s * state_stride
  uint16_t* ring;            // this layer's conv ring [4][8192] bf16 of slot 0
  int64_t state_stride;      // floats between slots
  int64_t ring_stride;       // elements between slots
  const float* conv_w;       // [4][8192]
  const float* ssm_a;        // [32]
  const float* dt_bias;      // [32]
  const float* ssm_norm;     // [128]
  const int32_t* slots;      // [n]
  const int32_t* pos;        // [n]
  int32_t n;
  int32_t ref_math;          // 1: the reference's fast-math activations (common.cuh)
  int32_t early;             // 1: no kernel of the open step writes this layer's state
  int* err;
};
cudaError_t launch_gdn_decode(const GdnArgs& a, cudaStream_t s);

// Split-K paged attention (attn_decode.cu).
struct AttnArgs {
  const uint16_t* proj;      // [n][10240] bf16
  uint16_t* k_pool;          // this layer: [max_pages][4][64][256] bf16
  uint16_t* v_pool;
  const int32_t* page_table; // [max_seqs][pt_stride]
  int32_t pt_stride;
  int32_t max_pages;
  const int32_t* slots;      // [n]
  const int32_t* pos;        // [n]  position of the new token
  const int32_t* seg;        // [n + 1] prefix sums of page-heads (4 * pages processed)
  const int32_t* page0;      // [n]  first page processed (0 for a full decode)
  const int32_t* append;     // [n]  1: this call appends the new token and attends to it
  const float* q_norm;       // [256]
  const float* k_norm;       // [256]
  const float* rope_cos;     // [max_ctx][32]
  const float* rope_sin;
  float* part_m;             // [slots][4] (log2 domain)
  float* part_l;             // [slots][4]
  float* part_o;             // [slots][4][256]
  const int32_t* split;      // [2] page-heads in the batch, page-heads per CTA
  int32_t n;
  int32_t grid;              // CTAs (the SM count; CTAs past the work exit)
  int32_t early;             // 1: no kernel of the open step writes this layer's K/V pool,
                             //    the page table or the descriptor before this launch
  int32_t per_hint;          // page-heads per CTA as the host last computed them (0: not
                             //    known); picks the kernel, not the split
  int* err;
};
// Combine the partials of each (sequence, kv-head) pair, apply the gate and
// store bf16 (attn_decode.cu).
struct CombineArgs {
  const uint16_t* proj;
  uint16_t* out;             // [n][4096]
  const int32_t* seg;
  const float* part_m;
  const float* part_l;
  const float* part_o;
  const int32_t* split;
  int32_t n;
  int32_t ref_math;          // 1: the reference's fast-math gate (common.cuh)
  // when non-null: write the merged record (m, l, o unnormalised) of sequence
  // 0 as [16 heads][2 + 256] instead of the gated bf16 output
  float* record;
  // when world > 0 (split over devices through peer memory): write the record
  // into slot [step & 1][layer][rank] of every rank's mailbox instead, then
  // add 1 to counter [layer][rank] of every rank (system scope); step =
  // this rank's done[layer] + 1
  int32_t world, rank, layer, n_layers;
  float* mbox_rec[QC_P2P_MAX_RANKS];       // each rank's record area (peer pointers)
  uint32_t* mbox_cnt[QC_P2P_MAX_RANKS];    // each rank's counters
  const uint32_t* done;                    // this rank's merged steps per layer
};
// tmk / tmv: 2D tensor maps over this layer's K / V pool viewed as
// [max_pages * 4 * 64 rows][256 bf16], box KV_BOX_ROWS rows x 64 columns,
// 128 B swizzle.
cudaError_t launch_attn_decode(const AttnArgs& a, const CombineArgs& c, const CUtensorMap& tmk,
                               const CUtensorMap& tmv, cudaStream_t s);
int attn_smem_bytes();
// Merge n_parts records [n_parts][16][258] (m, l, o) into the gated bf16
// output [4096] of one sequence (attn_decode.cu).
cudaError_t launch_attn_merge_records(const float* records, int32_t n_parts, const uint16_t* proj,
                                      uint16_t* out, int ref_math, cudaStream_t s);
// The same merge from this rank's mailbox, after waiting (bounded) until every
// rank's counter [layer][r] has reached 16 * (done[layer] + 1); the last CTA
// to finish advances done[layer].
struct MailboxMergeArgs {
  const float* rec;        // this rank's record area [2][n_layers][world][16][258]
  const uint32_t* cnt;     // this rank's counters [n_layers][world]
  uint32_t* done;          // [n_layers] steps merged
  uint32_t* consumed;      // [n_layers] CTAs finished, for advancing done
  uint32_t* poison;        // set by a wait that gave up; later merges refuse until reset
  int32_t world, layer, n_layers;
  const uint16_t* proj;
  uint16_t* out;
  int32_t ref_math;
  int* err;
};
cudaError_t launch_attn_merge_mailbox(const MailboxMergeArgs& m, cudaStream_t s);

// Message returned by qc_last_error(NULL) on this thread (qcache.cu).
void set_thread_error(const char* msg);

// Chunked prefill of T <= QC_PREFILL_CHUNK tokens of one sequence (prefill.cu).
struct GdnPrefillArgs {
  const uint16_t* proj;      // [T][12352] bf16
  uint16_t* out;             // [T][4096] bf16
  float* state;              // this sequence's state of this layer [32][128][128]
  uint16_t* ring;            // this sequence's conv ring of this layer [4][8192]
  const float* conv_w;
  const float* ssm_a;
  const float* dt_bias;
  const float* ssm_norm;
  float* conv_out;           // scratch [T][8192] f32: conv + SiLU outputs of the chunk
  int32_t pos0;              // position of the chunk's first token
  int32_t T;
  int32_t ref_math;
};
cudaError_t launch_gdn_prefill(const GdnPrefillArgs& a, cudaStream_t s);

struct AttnPrefillArgs {
  const uint16_t* proj;      // [T][10240] bf16
  uint16_t* out;             // [T][4096] bf16
  uint16_t* k_pool;          // this layer
  uint16_t* v_pool;
  const int32_t* page_row;   // this sequence's page-table row
  int32_t max_pages;
  const float* q_norm;
  const float* k_norm;
  const float* rope_cos;
  const float* rope_sin;
  uint16_t* q_buf;           // scratch [4 kv-heads][128 rows][256] bf16, row = head * 32 + t
  float* rec;                // scratch [4][n_split][128 rows][260] f32 (m, l, pad, o)
  int32_t pos0;
  int32_t T;
  int32_t n_split;           // CTAs per kv-head
  int32_t ref_math;
  int* err;
};
cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, const CUtensorMap& tmk,
                                const CUtensorMap& tmv, cudaStream_t s);
int attn_prefill_smem_bytes();

// Copies (kv_copy.cu).
// Scatter / gather of positions [pos0, pos0 + n) of one sequence between a
// contiguous [n][4][256] array and the paged pool of one layer.
cudaError_t launch_kv_scatter(uint16_t* k_pool, uint16_t* v_pool, const int32_t* page_row,
                              int32_t pos0, int32_t n, const uint16_t* k, const uint16_t* v,
                              int32_t max_pages, int* err, cudaStream_t s);
cudaError_t launch_kv_gather(const uint16_t* k_pool, const uint16_t* v_pool,
                             const int32_t* page_row, int32_t pos0, int32_t n, uint16_t* k,
                             uint16_t* v, int32_t max_pages, int* err, cudaStream_t s);
// Generic batched copy: n_jobs jobs of (src, dst, bytes), bytes and both
// addresses multiples of 16; jobs split into chunks of `chunk` bytes.
struct CopyJob {
  const void* src;
  void* dst;
  int64_t bytes;
};
// Chunks run through the bulk-copy engine: addresses and sizes multiples of 16.
cudaError_t launch_copy_jobs(const CopyJob* jobs_dev, int32_t n_jobs, const int64_t* chunk_start_dev,
                             int64_t n_chunks, int32_t chunk, int* err, cudaStream_t s);
// Conv ring <-> oldest-first [3][8192] history of one layer of one sequence.
cudaError_t launch_ring_to_hist(const uint16_t* ring, int32_t pos, uint16_t* hist, cudaStream_t s);
cudaError_t launch_hist_to_ring(const uint16_t* hist, int32_t pos, uint16_t* ring, cudaStream_t s);

// BFP8_B GEMV (bfp8.cu).  Rows m < split go to y0[b * ld0 + m], the others to
// y1[b * ld1 + m - split]; mode 1 adds into y0/y1 with the reference's resadd
// rounding.  batch <= bfp8_gemv_columns() per launch; with S > 1 k-chunks a
// merge kernel follows the GEMV on the stream.
struct Bfp8GemvArgs {
  const uint8_t* w;
  const uint16_t* x;
  uint16_t* y0;
  uint16_t* y1;
  int64_t ld0, ld1;
  int32_t split;
  int32_t mode;
  float* partial;   // [S][columns][M] f32 split-K partial sums
  int* err;
  int32_t M, K, Mt, Kt, ku, S, n_units, batch;
};
cudaError_t bfp8_prepare_device();
cudaError_t launch_bfp8_gemv(const Bfp8GemvArgs& a, int grid, cudaStream_t s);
cudaError_t launch_bfp8_pack(const uint16_t* w, int32_t M, int32_t K, uint8_t* out, cudaStream_t s);
cudaError_t launch_bfp8_transcode(uint8_t* tiles, int64_t n_tiles, int to_device, cudaStream_t s);
int bfp8_gemv_columns();
int bfp8_gemv_warps_per_cta();
int bfp8_gemv_ctas_per_sm(int batch);

// Token sampling (sample.cu): one cluster of CTAs per row of logits.
struct SampleArgs {
  const uint16_t* logits;  // [batch][ld] bf16
  int64_t ld;
  int32_t vocab, batch, slice;
  float temperature, top_p;
  const double* uniform;   // [batch] in [0, 1)
  int32_t* tokens;         // [batch]
};
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t s);
size_t sample_smem_bytes();

}  // namespace qc
