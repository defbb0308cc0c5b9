/*
 * qcache.h — C ABI of the B200 (sm_100a) per-token cache path of the
 * Qwen3.5-9B hybrid stack (24 Gated-DeltaNet layers + 8 full-attention
 * layers).
 *
 * In the reference engine this path is inline host C++ inside
 * forward_decode()/forward_prefill() and generate() (src/engine.cpp), with
 * file-scope globals for the caches.  This header is the thin boundary that
 * replaces those blocks: the engine keeps its public API (src/engine.h:69-90)
 * and calls these functions where it used to run the host math.
 *
 * Conventions (mirroring the reference's, src/engine.cpp:79-97, 4164-4176):
 *   - every call returns an int status (QC_OK == 0); nothing throws, nothing
 *     exits; qc_last_error() returns a message for the last failure;
 *   - one context per GPU, externally synchronised (the reference serialises
 *     inference behind one mutex, src/server.cpp:20,125);
 *   - tensors named *_dev are device pointers owned by the caller; all device
 *     work is enqueued on the caller's stream (a cudaStream_t passed as void*);
 *   - the context owns the KV page pool, the DeltaNet state, the conv rings,
 *     the prefix snapshots and the page tables;
 *   - bf16 values travel as uint16_t bit patterns; f32 -> bf16 conversions done
 *     by this library round to nearest even.
 */
#ifndef QCACHE_H
#define QCACHE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fixed model shapes (src/model_config.h:15-33, src/engine.cpp:2383-2393) ---- */
#define QC_N_HEAD        16
#define QC_N_HEAD_KV     4
#define QC_HEAD_DIM      256
#define QC_ROPE_DIM      64
#define QC_ATTN_Q_DIM    (QC_N_HEAD * QC_HEAD_DIM * 2)         /* 8192: [16][q 256 | gate 256] */
#define QC_ATTN_PROJ     (QC_ATTN_Q_DIM + 2 * QC_N_HEAD_KV * QC_HEAD_DIM) /* 10240 */
#define QC_ATTN_OUT      (QC_N_HEAD * QC_HEAD_DIM)             /* 4096 */
#define QC_GDN_K_HEADS   16
#define QC_GDN_V_HEADS   32
#define QC_GDN_HEAD      128
#define QC_CONV_CH       8192                                  /* q 2048 | k 2048 | v 4096 */
#define QC_CONV_TAPS     4
#define QC_GDN_PROJ      12352                                 /* conv 8192 | z 4096 | alpha 32 | beta 32 */
#define QC_GDN_OUT       4096
#define QC_GDN_STATE     (QC_GDN_V_HEADS * QC_GDN_HEAD * QC_GDN_HEAD) /* floats per layer per sequence */
#define QC_PAGE          64                                    /* tokens per KV page */
#define QC_PREFILL_CHUNK 32                                    /* tokens per prefill call */

/* ---- status codes ---- */
#define QC_OK            0
#define QC_ERR_ARG       1   /* bad argument / state (message in qc_last_error) */
#define QC_ERR_OOM       2   /* page pool, sequence slots or snapshot slots exhausted */
#define QC_ERR_CUDA      3   /* a CUDA runtime call failed */
#define QC_ERR_TIMEOUT   4   /* a bounded device wait expired (kernel returned early) */
#define QC_ERR_BOUNDS    5   /* a device-side index check failed (access skipped) */
#define QC_ERR_NODEVICE  6   /* device work requested on a host-only context */

/* qc_create(device = QC_DEVICE_NONE) makes a host-only context: page
 * allocation, sequence bookkeeping and the prefix table work, every call that
 * would touch the GPU returns QC_ERR_NODEVICE.  It exists to test the host
 * logic on machines without a GPU; it computes nothing. */
#define QC_DEVICE_NONE   (-1)
#define QC_P2P_MAX_RANKS 8

typedef struct qc_ctx qc_ctx;
typedef void* qc_stream;   /* cudaStream_t */

typedef struct qc_config {
  int32_t n_attn_layers;   /* full-attention layers (8) */
  int32_t n_gdn_layers;    /* Gated-DeltaNet layers (24) */
  int32_t max_seqs;        /* live sequence slots */
  int32_t max_pages;       /* physical KV pages (QC_PAGE tokens each, all attention layers) */
  int32_t max_ctx;         /* positions per sequence; size of the RoPE table */
  int32_t max_batch;       /* sequences per decode step */
  int32_t max_snapshots;   /* DeltaNet/conv snapshot slots of the prefix cache */
  int32_t flags;           /* QC_FLAG_* bits, 0 for the defaults */
} qc_config;

/* Activation math.  By default (flags 0) the kernels compute the exact
 * functions (expf; sigmoid 1/(1+exp(-x)); SiLU x*sigmoid(x)).  With
 * QC_FLAG_REFERENCE_MATH they compute what the reference computes, with
 * Schraudolph's fast exp (src/engine.cpp:2349-2376) in the softplus of the
 * decay, the beta and output-gate sigmoids and every SiLU (conv output, z
 * gate), so outputs follow the reference engine's own results (within f32
 * reordering) instead of the exact functions, which differ from them by up
 * to a few percent.  Either way the cost is the same. */
#define QC_FLAG_REFERENCE_MATH 1

/* ---------------------------------------------------------------- context */

/* Replaces the cache allocations of load_model_and_tokenizer
 * (src/engine.cpp:3835-3843) and precompute_rope (src/engine.cpp:2408-2420,
 * called at src/engine.cpp:3850-3853). */
int qc_create(const qc_config* cfg, int device, qc_ctx** out);
void qc_destroy(qc_ctx* ctx);
const char* qc_last_error(const qc_ctx* ctx);
/* Reads and clears the device error words written by kernels (QC_ERR_TIMEOUT /
 * QC_ERR_BOUNDS); synchronises the given stream first.  There is one word per
 * launch site (kernel kind x layer), so qc_last_error names the kernel and the
 * layer that failed first, as the reference's hang breadcrumbs name the layer
 * and operation of a stuck call (src/engine.cpp:99-101, 4182-4185). */
int qc_check_device(qc_ctx* ctx, qc_stream stream);

/* Per-layer small weights, host pointers, copied to the device.
 * Attention: q_norm, k_norm [256] (cache_small_weights, src/engine.cpp:1819-1821).
 * DeltaNet: ssm_a [32] (already negative, = -exp(A_log)), dt_bias [32],
 * ssm_norm [128], conv_w [4][8192] tap-major (the transposed layout built by
 * src/gguf_loader.cpp:389-396). */
int qc_set_attn_params(qc_ctx* ctx, int attn_layer, const float* q_norm, const float* k_norm);
int qc_set_gdn_params(qc_ctx* ctx, int gdn_layer, const float* ssm_a, const float* dt_bias,
                      const float* ssm_norm, const float* conv_w);

/* -------------------------------------------------------------- sequences */

int qc_seq_alloc(qc_ctx* ctx, int32_t* seq);
int qc_seq_free(qc_ctx* ctx, int32_t seq);
/* reset_state() for one sequence (src/engine.cpp:4164-4176): zero the DeltaNet
 * state and conv ring, release the KV pages, forget the cached tokens. */
int qc_seq_reset(qc_ctx* ctx, int32_t seq, qc_stream stream);
int qc_seq_len(const qc_ctx* ctx, int32_t seq, int32_t* len);
/* Number of KV pages mapped by the sequence and their physical ids. */
int qc_seq_pages(const qc_ctx* ctx, int32_t seq, int32_t* pages, int32_t cap, int32_t* n_pages);

/* Back positions [0, new_len) with pages and set the length (no data written).
 * Used to stand up an existing context before writing it with qc_kv_write. */
int qc_seq_reserve(qc_ctx* ctx, int32_t seq, int32_t new_len);
/* Scatter n positions starting at pos0 from a contiguous [n][4][256] bf16
 * device array into the sequence's pages of one attention layer (and the
 * gather that reads them back).  Bit copies. */
int qc_kv_write(qc_ctx* ctx, int32_t seq, int attn_layer, int32_t pos0, int32_t n,
                const uint16_t* k_dev, const uint16_t* v_dev, qc_stream stream);
int qc_kv_read(qc_ctx* ctx, int32_t seq, int attn_layer, int32_t pos0, int32_t n,
               uint16_t* k_dev, uint16_t* v_dev, qc_stream stream);
/* DeltaNet recurrent state [32][128][128] f32 and conv history [3][8192] bf16
 * (oldest token first, the layout of g_conv_state, src/engine.cpp:92-94,
 * 3215-3233) of one layer of one sequence, device pointers. */
int qc_gdn_state_write(qc_ctx* ctx, int32_t seq, int gdn_layer, const float* state_dev,
                       const uint16_t* conv_dev, qc_stream stream);
int qc_gdn_state_read(qc_ctx* ctx, int32_t seq, int gdn_layer, float* state_dev,
                      uint16_t* conv_dev, qc_stream stream);

/* ----------------------------------------------------------- decode step */

/* Start one decode token for n sequences (n <= max_batch): each sequence's
 * token goes to position len(seq) (g_pos in the reference); a page is mapped
 * when the position opens one.  tokens (host, may be NULL) are recorded in the
 * sequences' token history (g_cached_tokens.push_back, src/engine.cpp:4151). */
int qc_decode_begin(qc_ctx* ctx, const int32_t* seq_ids, int32_t n, const int32_t* tokens,
                    qc_stream stream);
/* Full-attention layer for the batch (src/engine.cpp:3485-3564):
 * proj_dev [n][10240] bf16 -> out_dev [n][4096] bf16.  Fused per-head Q/K
 * RMSNorm, partial RoPE, bf16 KV append, split-K GQA flash-decode, sigmoid
 * output gate. */
int qc_attn_decode(qc_ctx* ctx, int attn_layer, const uint16_t* proj_dev, uint16_t* out_dev,
                   qc_stream stream);
/* Gated-DeltaNet layer for the batch (src/engine.cpp:3204-3327):
 * proj_dev [n][12352] bf16 -> out_dev [n][4096] bf16.  Causal conv ring +
 * SiLU, L2-normalised q/k, decay/beta, delta-rule state update, gated RMSNorm. */
int qc_gdn_decode(qc_ctx* ctx, int gdn_layer, const uint16_t* proj_dev, uint16_t* out_dev,
                  qc_stream stream);
/* Commit the token: len(seq) += 1 for every sequence of the batch (g_pos++,
 * src/engine.cpp:4150). */
int qc_decode_end(qc_ctx* ctx);
/* Close the open step without committing the token (lengths and token
 * histories unchanged; a page mapped for the position stays mapped).  Used
 * after capturing the layer calls of a step into a CUDA graph, and to abandon
 * a step after an error.  The layer calls read the step's positions and split
 * sizes from device memory written by qc_decode_begin, so a captured graph of
 * them replays correctly after every later qc_decode_begin for the same
 * sequence list.  Layer kernels of a step read their own layer's KV pool and
 * DeltaNet state while the previous kernel on the stream is still draining
 * (programmatic dependent launch) when nothing of the step has written them
 * yet; a write through qc_kv_write / qc_gdn_state_write inside an open step
 * turns that off for the layer.  A captured graph keeps the choice made at
 * capture, so do not replay it with such a write between qc_decode_begin and
 * the replay. */
int qc_decode_abort(qc_ctx* ctx);

/* ------------------------------------------------------------------ prefill */

/* Chunked prefill of n <= QC_PREFILL_CHUNK tokens of ONE sequence, positions
 * len(seq) .. len(seq) + n - 1 — the function the reference computes token by
 * token in forward_prefill (src/engine.cpp:2602-2722, 2843-2929).  Same
 * protocol as a decode step: qc_prefill_begin, then every layer, then
 * qc_prefill_end (commits len += n and records tokens, which may be NULL).
 *   qc_attn_prefill: proj_dev [n][10240] -> out_dev [n][4096]; appends the n
 *     K/V rows (same bytes as n decode appends) and attends causally.
 *   qc_gdn_prefill:  proj_dev [n][12352] -> out_dev [n][4096]; the state is
 *     read and written once for the chunk.
 * A prefill and a decode step cannot be open at the same time. */
int qc_prefill_begin(qc_ctx* ctx, int32_t seq, int32_t n, const int32_t* tokens,
                     qc_stream stream);
int qc_attn_prefill(qc_ctx* ctx, int attn_layer, const uint16_t* proj_dev, uint16_t* out_dev,
                    qc_stream stream);
int qc_gdn_prefill(qc_ctx* ctx, int gdn_layer, const uint16_t* proj_dev, uint16_t* out_dev,
                   qc_stream stream);
int qc_prefill_end(qc_ctx* ctx);

/* ----------------------------------------------------------- prefix cache */

/* The reference's single-sequence prefix rule (src/engine.cpp:4058-4080):
 * longest common prefix of tokens against the sequence's recorded history;
 * if the history diverges, or the whole prompt is already cached, the
 * sequence is reset and *prefix_len = 0.  Afterwards the caller prefills
 * tokens[*prefix_len:]. */
int qc_seq_match_prefix(qc_ctx* ctx, int32_t seq, const int32_t* tokens, int32_t n,
                        int32_t* prefix_len, qc_stream stream);

/* Hashed prefix cache (no reference counterpart: the reference keeps one
 * token vector, src/engine.cpp:96-97).  An entry holds a token prefix of
 * length P, the KV pages that cover it (full pages shared by refcount, the
 * partial tail page copied) and a DeltaNet/conv snapshot taken at P.
 *
 * insert: snapshot sequence `seq` (its length must equal n and its history
 *         must equal tokens) as a new entry.
 * lookup: longest entry whose tokens are a prefix of tokens[0:n] with P < n
 *         (at least one token is left to prefill, as in the reference);
 *         *entry = -1 and *matched = 0 on a miss.  Host only.
 * restore: for i < n, give seqs[i] (freshly reset) the state of entries[i]:
 *         page-table gather, tail-page copy-on-write, snapshot restore; one
 *         batched launch.  Afterwards len(seqs[i]) = P(entries[i]).
 * release: drop an entry (pages are freed when no sequence maps them). */
int qc_prefix_insert(qc_ctx* ctx, int32_t seq, const int32_t* tokens, int32_t n, int32_t* entry,
                     qc_stream stream);
int qc_prefix_lookup(qc_ctx* ctx, const int32_t* tokens, int32_t n, int32_t* matched,
                     int32_t* entry);
int qc_prefix_restore(qc_ctx* ctx, const int32_t* entries, const int32_t* seqs, int32_t n,
                      qc_stream stream);
int qc_prefix_release(qc_ctx* ctx, int32_t entry);
/* Bytes the last qc_prefix_restore call moved on the device (read + write). */
int qc_prefix_last_restore_bytes(const qc_ctx* ctx, int64_t* bytes);
/* Chained page hash h_i = H(h_{i-1}, tokens[64i:64i+64]) for the n/64 full
 * pages of tokens (pure host function). */
int qc_prefix_page_hashes(const int32_t* tokens, int32_t n, uint64_t* hashes);

/* --------------------------------------------- split-K across GPUs (long ctx) */

/* Long-context decode of one sequence split over devices by KV position.
 * Each device's context maps the whole sequence and holds the KV of its page
 * range.  After qc_decode_begin (batch of one sequence):
 *   qc_attn_partial_range: this device attends pages [page_begin, page_end);
 *     append != 0 on the device whose range holds the new position (it
 *     appends the token and attends to it).  Uploads the step's descriptor.
 *   qc_attn_partial: per layer, writes the range's record partial_dev
 *     [16][2 + 256] f32: per q-head m (max of score * log2 e), l (sum of
 *     2^(s - m)) and o[256] (unnormalised).  Reads the range from device
 *     memory, so a CUDA graph of the per-layer calls replays for every step.
 *   qc_attn_combine: merges n_parts records [n_parts][16][258] (all-gathered
 *     from the devices, e.g. over NCCL) and applies the sigmoid gate:
 *     out_dev [4096] bf16, as qc_attn_decode would produce. */
int qc_attn_partial_range(qc_ctx* ctx, int32_t page_begin, int32_t page_end, int32_t append,
                          qc_stream stream);
int qc_attn_partial(qc_ctx* ctx, int attn_layer, const uint16_t* proj_dev, float* partial_dev,
                    qc_stream stream);
int qc_attn_combine(qc_ctx* ctx, const float* partials_dev, int32_t n_parts,
                    const uint16_t* proj_dev, uint16_t* out_dev, qc_stream stream);

/* The same split with the records exchanged through peer memory over NVLink
 * instead of a collective library (one process per GPU, all on one node):
 *   qc_p2p_create: allocates this rank's mailbox (records of every layer and
 *     rank, double-buffered by step, plus arrival counters) and writes its
 *     CUDA IPC handle (QC_P2P_HANDLE_BYTES) to handle_out; the caller ships
 *     the handles between its processes (any transport);
 *   qc_p2p_open: maps peer rank `peer`'s mailbox from its handle (every rank
 *     other than this one, once);
 *   qc_attn_partial_p2p: like qc_attn_partial, but the kernel that merges the
 *     range's record stores it into every rank's mailbox (peer stores over
 *     NVLink) and then bumps every rank's counter for (layer, this rank);
 *   qc_attn_combine_p2p: waits on the device until all ranks' records of the
 *     step have arrived (bounded: after 1 s the error word reports
 *     QC_ERR_TIMEOUT, see qc_check_device, and the output is not written),
 *     then merges them as qc_attn_combine does.
 * Every rank must run the same steps and layers (qc_attn_partial_range opens
 * a step).  Destroy the contexts only after all ranks have finished their
 * last step.
 * Failure: when a rank's records do not arrive within 1 s (a rank that died,
 * stalled or skipped a layer), the merge gives up, qc_check_device reports
 * QC_ERR_TIMEOUT naming the layer, and the mailbox is poisoned: the ranks'
 * step counts no longer agree, so every later qc_attn_combine_p2p on this
 * rank writes no output and reports QC_ERR_TIMEOUT again, and after
 * qc_check_device has seen the timeout, qc_attn_partial_p2p and
 * qc_attn_combine_p2p return QC_ERR_ARG.  To recover, every surviving rank
 * closes its step (qc_decode_abort), synchronises its stream, meets the
 * others at a host barrier, calls qc_p2p_reset (zeroes its own counters, step
 * counts and poison word), and meets them at a second barrier before the
 * next step.  A rank that is gone must be replaced, or the mailboxes
 * recreated with the new world size.
 */
#define QC_P2P_HANDLE_BYTES 64
int qc_p2p_create(qc_ctx* ctx, int32_t world, int32_t rank, void* handle_out);
int qc_p2p_open(qc_ctx* ctx, int32_t peer, const void* handle);
int qc_attn_partial_p2p(qc_ctx* ctx, int attn_layer, const uint16_t* proj_dev, qc_stream stream);
int qc_attn_combine_p2p(qc_ctx* ctx, int attn_layer, const uint16_t* proj_dev, uint16_t* out_dev,
                        qc_stream stream);
/* Clears this rank's mailbox counters, step counts and poison word (see
 * "Failure" above); synchronises the stream.  No decode step may be open. */
int qc_p2p_reset(qc_ctx* ctx, qc_stream stream);

/* ------------------------------------------- decode without device allocation */

/* No counterpart in the reference.  For callers that may not allocate device
 * memory (an engine that owns all GPU memory in its own arena, a plugin
 * running inside another framework's pool, a process capped at a fixed
 * footprint): one full-attention decode step like qc_attn_decode, but with no
 * context and no allocation.  The caller passes everything that persists:
 *   k_pool_dev, v_pool_dev [max_pages][4][64][256] bf16 (one layer);
 *   page_table_dev [n][pt_stride] int32, row i mapping sequence i's pages;
 *   pos (host) [n]: position of each sequence's new token, whose K/V are
 *     appended into its page; q_norm_dev, k_norm_dev [256] f32;
 *   rope_cos_dev, rope_sin_dev [>= max(pos) + 1][32] f32, the table of
 *     precompute_rope (src/engine.cpp:2408-2420);
 *   proj_dev [n][10240] and out_dev [n][4096] bf16.
 * The kernels' scratch (split-K partial records, step descriptor) is one
 * fixed array of about 1.9 MB compiled into the library, resident on every GPU
 * that loads it until exit.  Limits: n <= QC_NOALLOC_MAX_BATCH and at most
 * QC_NOALLOC_MAX_CTAS SMs; larger requests return QC_ERR_ARG.  All calls on a
 * device share that array: calls that overlap on the GPU race, so serialise
 * them.  The first call on each device looks up the array's address with that
 * device current; make it before any stream capture.  The step descriptor
 * travels as a kernel parameter, so the call reads no host memory
 * asynchronously and does not wait for earlier work on the stream.  On
 * failure qc_last_error(NULL) describes the error. */
#define QC_NOALLOC_MAX_BATCH 64
#define QC_NOALLOC_MAX_CTAS  192
int qc_attn_decode_noalloc(const uint16_t* proj_dev, uint16_t* k_pool_dev, uint16_t* v_pool_dev,
                           int32_t max_pages, const int32_t* page_table_dev, int32_t pt_stride,
                           const int32_t* pos, int32_t n, const float* q_norm_dev,
                           const float* k_norm_dev, const float* rope_cos_dev,
                           const float* rope_sin_dev, uint16_t* out_dev, qc_stream stream);
/* Errors the kernels of qc_attn_decode_noalloc found on the current device
 * (a page-table entry outside [0, max_pages): QC_ERR_BOUNDS, that tile was
 * skipped and the output is wrong; an expired wait: QC_ERR_TIMEOUT), collected
 * over every call since the last check.  Synchronises the stream, returns the
 * code (message in qc_last_error(NULL)) and clears it.  Allocates nothing. */
int qc_attn_noalloc_check(qc_stream stream);

/* Which decode-attention kernel later launches use (no counterpart in the
 * reference, whose attention is one host loop): QC_ATTN_KERNEL_AUTO, the
 * default, takes the tcgen05 kernel when each CTA streams at most 60
 * page-heads and the mma.sync kernel otherwise; the other two force one.
 * Both compute the same records (within f32 summation order).  Process-wide,
 * for tests and tuning; a captured graph keeps the kernel it was captured
 * with.  Returns the previous mode, or -QC_ERR_ARG for an unknown mode. */
#define QC_ATTN_KERNEL_AUTO 0
#define QC_ATTN_KERNEL_MMA  1
#define QC_ATTN_KERNEL_TC   2
int qc_attn_select_kernel(int mode);

#ifdef __cplusplus
}
#endif

#endif /* QCACHE_H */
