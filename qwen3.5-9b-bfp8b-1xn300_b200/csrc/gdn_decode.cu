// gdn_decode.cu — one Gated-DeltaNet decode step, fused in a single
// memory-bound pass (src/engine.cpp:3204-3327).
//
// Small batches (at most 8 sequences): R CTAs per (sequence, v-head) — R = 4
// for one or two sequences (a cluster), R = 1 (one 512-thread CTA per head)
// from 3 to 8 — so that enough SMs stream.  CTA r owns state rows
// [r*128/R, (r+1)*128/R) of the head (rows are independent in the delta rule,
// src/engine.cpp:3284-3305).  The CTA
//   1. loads every small input of its prologue first (conv taps, conv
//      weights, projection row, per-head parameters): a timeline of the
//      kernel (globaltimer stamps per CTA, batch 8) showed these loads
//      waiting ~5 us behind the multi-megabyte state copies when those were
//      issued first, and ~2 us when issued before them;
//   2. then copies its state slice into shared memory in 16-row chunks
//      (bulk copies, one mbarrier each);
//   3. runs the causal conv (width 4) + SiLU for the 128 q and 128 k channels
//      of k-head vh % 16 and its own v channels, appends the new input to the
//      conv ring, L2-normalises q and k, computes decay and beta;
//   4. per row, as soon as its chunk has landed: decay, s·k, delta, rank-1
//      update, s·q — one float4 per lane, warp-shuffle dot products — and
//      stores the row straight back to HBM with 128-bit stores;
//   5. gated RMSNorm over the head's 128 outputs (for R > 1 the CTAs of the
//      cluster exchange their partial sums of squares through distributed
//      shared memory with plain stores), then bf16 outputs.
// Programmatic dependent launch: nothing the previous kernel on the stream
// can have written is read before griddepcontrol.wait, except what no kernel
// of the open decode step writes before this one (the host's a.early: the
// step descriptor, this layer's ring, weights and state), so those loads and
// the state copies overlap the previous kernel's tail.  Measured (us per
// token and layer, batch 1 / 4 / 8): 2-CTA clusters with one 32 KiB copy
// issued first 6.67 / 2.23 / 1.47; prologue loads first 4.78 / 1.73 / 1.20;
// one CTA per head from 3 sequences 1.65 / 1.15; early loads under the
// dependent launch 4.42 / 1.54 / 1.10; early state copies 4.53 / - / 1.06.
// Large batches use the persistent producer/consumer kernel further down,
// without the dependent launch (it measured slower there: 0.770 -> 0.814 at
// batch 64).
// HBM traffic per (sequence, layer): state 2 MiB read + 2 MiB written, conv
// ring 3 x 16 KiB read + 16 KiB written, projection row 24.7 KB, output 8 KB.
//
// Conv ring: the history of the last three inputs lives in a 4-slot ring,
// slot = position & 3.  The token at position t reads slots (t-3)&3, (t-2)&3,
// (t-1)&3 (taps 0..2, oldest first) and writes its input to slot t&3, which
// no CTA of this step reads, so the CTAs that share a k-head never race.  The
// ring holds bf16: every value it stores is a projection output, which is
// bf16 (the reference widens bf16 GEMV outputs, src/engine.cpp:1732-1753).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace qc {
namespace {

constexpr int HK = 128;              // k-dim per head
constexpr int CONV = 8192;           // conv channels
constexpr int Z_OFF = 8192;          // z offset in the projection row
constexpr int A_OFF = 12288;         // alpha offset
constexpr int B_OFF = 12320;         // beta offset
constexpr float EPS = 1e-6f;
constexpr float SSM_SCALE = 1.0f / 11.3137f;  // src/engine.cpp:3249

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#ifndef QC_GDN_MINB
#define QC_GDN_MINB(T) (1024 / (T) > 0 ? 1024 / (T) : 1)
#endif
#ifndef QC_GDN_PDL_SMALL
#define QC_GDN_PDL_SMALL 1
#endif
#ifndef QC_GDN_EARLY_TMA
#define QC_GDN_EARLY_TMA 1
#endif
#ifndef QC_GDN_PDL_LARGE
#define QC_GDN_PDL_LARGE 0
#endif

// R CTAs (a cluster when R > 1) per (sequence, v-head), T threads each.
template <int R, int T>
__global__ void __launch_bounds__(T, QC_GDN_MINB(T)) gdn_decode_kernel(const GdnArgs a) {
  constexpr int RB = HK / R;     // state rows per CTA
  constexpr int NW = T / 32;     // warps
  constexpr int RPW = RB / NW;   // rows per warp
  constexpr int QKPT = (2 * HK + T - 1) / T;    // q/k channels per thread (some idle)
  constexpr int CR = RB < 16 ? RB : 16;         // rows per state chunk
  constexpr int NCH = RB / CR;
  static_assert(RPW >= 1 && RPW <= 32 && RB % NW == 0 && RB <= T &&
                (RPW <= CR ? CR % RPW == 0 : RPW % CR == 0), "row split");
  extern __shared__ __align__(128) float s_state[];  // [RB][128]
  __shared__ __align__(16) float s_q[HK];
  __shared__ __align__(16) float s_k[HK];
  __shared__ float s_v[RB];
  __shared__ float s_o[RB];
  __shared__ float s_red[2 * NW];
  __shared__ float s_ssq[R];
  __shared__ __align__(8) uint64_t s_bar[NCH];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y;
  const int vh = blockIdx.x / R;
  const int r = blockIdx.x % R;  // == rank in the cluster (cluster dims (R,1,1))
  const int kh = vh & 15;        // kh = vh % 16 (src/engine.cpp:3254)
  if (tid == 0) {
    for (int c = 0; c < NCH; ++c) mbar_init(&s_bar[c], 1);
    fence_mbar_init();
  }
  // Loads of what the previous kernel on the stream cannot have written (the
  // step descriptor, this layer's conv ring and weights: no kernel of the open
  // step writes them before this one, a.early) are issued before
  // griddepcontrol.wait; the projection row after it.
  if (!a.early) griddep_wait();
  const int slot = a.slots[b];
  const int pos = a.pos[b];
  float* st = a.state + slot * a.state_stride + (int64_t)vh * HK * HK + (int64_t)r * RB * HK;
  uint16_t* ring = a.ring + slot * a.ring_stride;
  const uint16_t* x = a.proj + (int64_t)b * 12352;
  const int t0 = (pos - 3) & 3, t1 = (pos - 2) & 3, t2 = (pos - 1) & 3, tw = pos & 3;
  const float* w = a.conv_w;

  // ---- every small input is loaded first: these loads are on the critical
  // path, the state copy is not (it lands while the prologue computes), and
  // loads issued after a multi-megabyte bulk transfer queue behind it.
  // Thread j owns q/k channels i = j + m*T (q for i < 128, k after) and, for
  // j < RB, v channel / state row j of this CTA.
  float qk_w[QKPT][4], qk_h[QKPT][4];
  int qk_c[QKPT];
  uint16_t qk_x[QKPT];
#pragma unroll
  for (int m = 0; m < QKPT; ++m) {
    const int i = min(tid + m * T, 2 * HK - 1);  // idle threads repeat the last channel
    const int c = (i < HK) ? kh * HK + i : 2048 + kh * HK + (i - HK);
    qk_c[m] = c;
    qk_h[m][0] = bf2f(ring[t0 * CONV + c]);
    qk_h[m][1] = bf2f(ring[t1 * CONV + c]);
    qk_h[m][2] = bf2f(ring[t2 * CONV + c]);
#pragma unroll
    for (int t = 0; t < 4; ++t) qk_w[m][t] = w[t * CONV + c];
  }
  const bool has_row = tid < RB;
  const int cv = 4096 + vh * HK + r * RB + (has_row ? tid : 0);
  float v_w[4], v_h[4], zf = 0.0f, nrm = 0.0f;
  uint16_t v_x = 0;
  if (has_row) {
    v_h[0] = bf2f(ring[t0 * CONV + cv]);
    v_h[1] = bf2f(ring[t1 * CONV + cv]);
    v_h[2] = bf2f(ring[t2 * CONV + cv]);
#pragma unroll
    for (int t = 0; t < 4; ++t) v_w[t] = w[t * CONV + cv];
    nrm = a.ssm_norm[r * RB + tid];
  }
  const float dtb = a.dt_bias[vh], ssa = a.ssm_a[vh];
#if QC_GDN_EARLY_TMA
  if (a.early) {
    __syncthreads();
    if (tid == 0) {
      for (int c = 0; c < NCH; ++c) {
        mbar_arrive_expect_tx(&s_bar[c], CR * HK * 4);
        bulk_g2s(s_state + c * CR * HK, st + c * CR * HK, CR * HK * 4, &s_bar[c]);
      }
    }
  }
#endif
  if (a.early) griddep_wait();
  griddep_launch();
#pragma unroll
  for (int m = 0; m < QKPT; ++m) {
    qk_x[m] = x[qk_c[m]];
    qk_h[m][3] = bf2f(qk_x[m]);
  }
  if (has_row) {
    v_x = x[cv];
    v_h[3] = bf2f(v_x);
    zf = bf2f(x[Z_OFF + vh * HK + r * RB + tid]);
  }
  const float a_raw = bf2f(x[A_OFF + vh]), b_raw = bf2f(x[B_OFF + vh]);
  __syncthreads();  // every warp has issued its loads (and the barriers are initialised)
#if QC_GDN_EARLY_TMA
  if (tid == 0 && !a.early) {
#else
  if (tid == 0) {
#endif
    for (int c = 0; c < NCH; ++c) {
      mbar_arrive_expect_tx(&s_bar[c], CR * HK * 4);
      bulk_g2s(s_state + c * CR * HK, st + c * CR * HK, CR * HK * 4, &s_bar[c]);
    }
  }
  // Split cluster barrier, first half: announces that this CTA runs, so that
  // peers may write its shared memory after their matching wait.  Relaxed:
  // no memory ordering is needed here, and its latency hides behind the conv.
  if constexpr (R > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // ---- conv1d + SiLU (src/engine.cpp:3204-3234), ring append
  float sq = 0.0f, sk = 0.0f;
#pragma unroll
  for (int m = 0; m < QKPT; ++m) {
    const int i = tid + m * T;
    if (i >= 2 * HK) break;
    float y = qk_h[m][0] * qk_w[m][0];
    y = fmaf(qk_h[m][1], qk_w[m][1], y);
    y = fmaf(qk_h[m][2], qk_w[m][2], y);
    y = fmaf(qk_h[m][3], qk_w[m][3], y);
    y = act_silu(y, a.ref_math);
    if (i < HK) { s_q[i] = y; sq = fmaf(y, y, sq); }
    else { s_k[i - HK] = y; sk = fmaf(y, y, sk); }
    // one CTA of one v-head writes each q/k channel of the ring
    if (vh < 16 && (i & (HK - 1)) / RB == r) ring[tw * CONV + qk_c[m]] = qk_x[m];
  }
  if (has_row) {
    float y = v_h[0] * v_w[0];
    y = fmaf(v_h[1], v_w[1], y);
    y = fmaf(v_h[2], v_w[2], y);
    y = fmaf(v_h[3], v_w[3], y);
    s_v[tid] = act_silu(y, a.ref_math);
    ring[tw * CONV + cv] = v_x;
  }

  // ---- L2 normalisation of q and k (src/engine.cpp:3261-3275)
  sq = warp_sum(sq);
  sk = warp_sum(sk);
  if (lane == 0) {
    s_red[warp] = sq;
    s_red[NW + warp] = sk;
  }
  __syncthreads();
  float tq = 0.0f, tk = 0.0f;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    tq += s_red[i];
    tk += s_red[NW + i];
  }
  const float qs = 1.0f / sqrtf(tq + EPS), ks = 1.0f / sqrtf(tk + EPS);

  // ---- decay and beta (src/engine.cpp:3277-3281)
  const float biased = a_raw + dtb;
  const float sp = (biased > 20.0f) ? biased : logf(1.0f + softplus_exp(biased, a.ref_math));
  const float decay = expf(sp * ssa);
  const float beta = gate_sigmoid(b_raw, a.ref_math);

  // ---- delta rule (src/engine.cpp:3284-3305), rows of this warp, as soon as
  // the chunk holding them has landed
  float ssq_w = 0.0f;
  const int row0 = warp * RPW;
  bool ok = true;
  for (int c = row0 / CR; ok && c * CR < row0 + RPW; ++c) ok = mbar_wait(&s_bar[c], 0, a.err);
  if (ok) {
    float4 k4 = reinterpret_cast<const float4*>(s_k)[lane];
    float4 q4 = reinterpret_cast<const float4*>(s_q)[lane];
    k4.x *= ks; k4.y *= ks; k4.z *= ks; k4.w *= ks;
    q4.x *= qs; q4.y *= qs; q4.z *= qs; q4.w *= qs;
    const float4* srow = reinterpret_cast<const float4*>(s_state);
    float4* grow = reinterpret_cast<float4*>(st);
    constexpr int G = RPW < 4 ? RPW : 4;  // rows in flight per warp (register budget)
#pragma unroll 1
    for (int g0 = 0; g0 < RPW; g0 += G) {
      float4 rr[G];
      float skr[G];
#pragma unroll
      for (int i = 0; i < G; ++i) {
        float4 v = srow[(row0 + g0 + i) * 32 + lane];
        v.x *= decay; v.y *= decay; v.z *= decay; v.w *= decay;
        rr[i] = v;
        float d = v.x * k4.x;
        d = fmaf(v.y, k4.y, d);
        d = fmaf(v.z, k4.z, d);
        d = fmaf(v.w, k4.w, d);
        skr[i] = d;
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
        for (int i = 0; i < G; ++i) skr[i] += __shfl_xor_sync(FULL_MASK, skr[i], m);
      float o[G];
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const int row = row0 + g0 + i;
        const float dd = beta * (s_v[row] - skr[i]);
        float4 v = rr[i];
        v.x = fmaf(k4.x, dd, v.x);
        v.y = fmaf(k4.y, dd, v.y);
        v.z = fmaf(k4.z, dd, v.z);
        v.w = fmaf(k4.w, dd, v.w);
        __stcs(grow + row * 32 + lane, v);  // coalesced 512 B per row, streamed
        float d = v.x * q4.x;
        d = fmaf(v.y, q4.y, d);
        d = fmaf(v.z, q4.z, d);
        d = fmaf(v.w, q4.w, d);
        o[i] = d;
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
        for (int i = 0; i < G; ++i) o[i] += __shfl_xor_sync(FULL_MASK, o[i], m);
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const float ov = o[i] * SSM_SCALE;
        if (lane == i) s_o[row0 + g0 + i] = ov;
        ssq_w = fmaf(ov, ov, ssq_w);
      }
    }
  }
  ok = __syncthreads_and(ok);  // s_red reuse
  if (lane == 0) s_red[warp] = ssq_w;
  __syncthreads();
  float part = 0.0f;
#pragma unroll
  for (int i = 0; i < NW; ++i) part += s_red[i];

  // ---- gated RMSNorm over the head's 128 outputs (src/engine.cpp:3307-3322)
  float tot = part;
  if constexpr (R > 1) {
    // every CTA pushes its partial sum of squares into slot r of each peer's
    // s_ssq (distributed shared memory, plain stores), then one cluster
    // barrier (release/acquire) publishes them; nobody reads remote memory
    // after the barrier, so CTAs may exit right after it
    cg::cluster_group cluster = cg::this_cluster();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every peer has started
    if (tid < R) *cluster.map_shared_rank(&s_ssq[r], tid) = part;
    cluster.sync();
    tot = 0.0f;
#pragma unroll
    for (int q = 0; q < R; ++q) tot += s_ssq[q];
  }
  if (!ok) return;
  const float rms = 1.0f / sqrtf(tot / 128.0f + EPS);
  if (has_row) {
    const float y = (s_o[tid] * rms) * nrm * act_silu(zf, a.ref_math);
    a.out[(int64_t)b * 4096 + vh * HK + r * RB + tid] = f2bf(y);
  }
}

// Persistent variant for large batches: every CTA walks work items (one
// (sequence, v-head) each) with stride gridDim.x.  The last warp streams the
// state of its items in 16-row chunks (8 KiB bulk copies) through a 4-deep
// ring, running ahead across item boundaries, so HBM stays busy while the
// consumer warps run the conv prologue, the delta rule and the gated RMSNorm
// of the current head.  Shape, from measurement at batch 64 (fraction of the
// measured copy bandwidth): 8 consumer warps, 6 CTAs/SM, 3 stages 0.81 — the
// 32-register cap of that occupancy spilled; 4 consumer warps (4 rows per warp
// and chunk, 71 registers), 5 CTAs/SM, 4 stages 0.855.  Neither giving every
// CTA the same number of items (the last third of the CTAs otherwise gets one
// item more), nor 7 CTAs/SM with 2 stages, nor 32-row chunks did better.
#ifndef QC_GDN_CHUNK
#define QC_GDN_CHUNK 16
#endif
constexpr int PCHUNK = QC_GDN_CHUNK;       // rows per chunk

#ifndef QC_GDN_STAGES
#define QC_GDN_STAGES 4
#endif
#ifndef QC_GDN_CTAS
#define QC_GDN_CTAS 5
#endif
constexpr int PSTAGES = QC_GDN_STAGES;
#ifndef QC_GDN_WARPS
#define QC_GDN_WARPS 4
#endif
constexpr int PCONSUMERS = QC_GDN_WARPS;
constexpr int PTHREADS = (PCONSUMERS + 1) * 32;
constexpr int PRPW = PCHUNK / PCONSUMERS;  // rows per consumer warp per chunk
static_assert(PCHUNK % PCONSUMERS == 0 && PRPW <= 32, "chunk split");

struct PSmem {
  float st[PSTAGES][PCHUNK * HK];
  float q[HK];
  float k[HK];
  float v[HK];
  float z[HK];
  float o[HK];
  float red[3 * PCONSUMERS];  // q norm | k norm | output sum of squares
  uint64_t full[PSTAGES];
  uint64_t empty[PSTAGES];
  // the next item's prologue inputs, fetched with cp.async while the current
  // item streams: channel i < 384 is q (i < 128), k, then v of the head
  __align__(16) float w[4][3 * HK];     // conv taps
  __align__(16) uint16_t hist[3][3 * HK];  // conv ring, oldest tap first
  __align__(16) uint16_t x[4 * HK];     // new inputs of the channels, then z
  uint32_t ab[2];                        // words holding alpha and beta
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

// Issues (does not wait for) the copies of item u's prologue inputs into
// sm.w / sm.hist / sm.x / sm.ab; every 16-byte run is 16-byte aligned when
// proj, the ring and the conv weights are (checked at launch).
__device__ __forceinline__ void prefetch_item(PSmem& sm, const GdnArgs& a, int u, int tid) {
  constexpr int NT = PCONSUMERS * 32;
  const int b = u >> 5, vh = u & 31, kh = vh & 15;
  const int pos = a.pos[b];
  const uint16_t* ring = a.ring + a.slots[b] * a.ring_stride;
  const uint16_t* x = a.proj + (int64_t)b * 12352;
  // run r (0..2) of 128 channels: q, k, v; run 3 of x is z
  auto chan0 = [&](int r) { return r == 0 ? kh * HK : r == 1 ? 2048 + kh * HK : 4096 + vh * HK; };
  // 16-byte pieces: w 4 taps x 3 runs x 32, ring 3 taps x 3 runs x 16, x 4 runs x 16
  constexpr int NW = 4 * 3 * 32, NH = 3 * 3 * 16, NX = 4 * 16;
  for (int k = tid; k < NW + NH + NX; k += NT) {
    if (k < NW) {
      const int tap = k / 96, r = (k / 32) % 3, e = k % 32;
      cp_async16(&sm.w[tap][r * HK + 4 * e], a.conv_w + tap * CONV + chan0(r) + 4 * e);
    } else if (k < NW + NH) {
      const int kk = k - NW, tap = kk / 48, r = (kk / 16) % 3, e = kk % 16;
      const int slot = (pos - 3 + tap) & 3;
      cp_async16(&sm.hist[tap][r * HK + 8 * e], ring + slot * CONV + chan0(r) + 8 * e);
    } else {
      const int kk = k - NW - NH, r = kk / 16, e = kk % 16;
      const int c0 = r < 3 ? chan0(r) : Z_OFF + vh * HK;
      cp_async16(&sm.x[r * HK + 8 * e], x + c0 + 8 * e);
    }
  }
  if (tid < 2) {
    const int off = (tid == 0 ? A_OFF : B_OFF) + vh;  // the bf16 is half of this word
    cp_async4(&sm.ab[tid], x + (off & ~1));
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void pconsumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(PCONSUMERS * 32) : "memory");
}

template <bool PRE>
__global__ void __launch_bounds__(PTHREADS, QC_GDN_CTAS) gdn_decode_persistent(const GdnArgs a) {
  extern __shared__ __align__(128) unsigned char praw[];
  PSmem& sm = *reinterpret_cast<PSmem*>(praw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = a.n * 32;
  if (tid == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], PCONSUMERS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == PCONSUMERS) {  // ------------------------------------ producer
    griddep_wait();
    if (lane != 0) return;
    int i = 0;
    for (int u = blockIdx.x; u < n_items; u += gridDim.x) {
      const int b = u >> 5, vh = u & 31;
      const float* src = a.state + a.slots[b] * a.state_stride + (int64_t)vh * HK * HK;
      for (int j = 0; j < HK / PCHUNK; ++j, ++i) {
        const int s = i % PSTAGES;
        if (i >= PSTAGES && !mbar_wait(&sm.empty[s], ((i / PSTAGES) - 1) & 1, a.err)) return;
        mbar_arrive_expect_tx(&sm.full[s], PCHUNK * HK * 4);
        bulk_g2s(sm.st[s], src + j * PCHUNK * HK, PCHUNK * HK * 4, &sm.full[s]);
      }
    }
    return;
  }

  // ----------------------------------------------------------------- consumers
  griddep_wait();
  griddep_launch();
  bool aborted = false;
  int i = 0;
  const float* w = a.conv_w;
  if (PRE && blockIdx.x < n_items) prefetch_item(sm, a, blockIdx.x, tid);
  for (int u = blockIdx.x; u < n_items; u += gridDim.x) {
    const int b = u >> 5, vh = u & 31, kh = vh & 15;
    const int slot = a.slots[b], pos = a.pos[b];
    uint16_t* ring = a.ring + slot * a.ring_stride;
    const uint16_t* x = a.proj + (int64_t)b * 12352;
    float* st = a.state + slot * a.state_stride + (int64_t)vh * HK * HK;
    const int t0 = (pos - 3) & 3, t1 = (pos - 2) & 3, t2 = (pos - 1) & 3, tw = pos & 3;
    // channel c of the head, local index li (q 0..127, k 128..255, v 256..383)
    auto conv1 = [&](int c, int li) -> float {
      float y;
      if (PRE) {
        y = bf2f(sm.hist[0][li]) * sm.w[0][li];
        y = fmaf(bf2f(sm.hist[1][li]), sm.w[1][li], y);
        y = fmaf(bf2f(sm.hist[2][li]), sm.w[2][li], y);
        y = fmaf(bf2f(sm.x[li]), sm.w[3][li], y);
      } else {
        y = bf2f(ring[t0 * CONV + c]) * w[c];
        y = fmaf(bf2f(ring[t1 * CONV + c]), w[CONV + c], y);
        y = fmaf(bf2f(ring[t2 * CONV + c]), w[2 * CONV + c], y);
        y = fmaf(bf2f(x[c]), w[3 * CONV + c], y);
      }
      return act_silu(y, a.ref_math);
    };
    if (PRE) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      pconsumer_sync();
    }
    // ---- prologue: conv + SiLU of the head's q, k and v channels
    constexpr int NT = PCONSUMERS * 32;
    float sq = 0.0f, sk = 0.0f;
    for (int t = tid; t < 2 * HK; t += NT) {
      const int c = (t < HK) ? kh * HK + t : 2048 + kh * HK + (t - HK);
      const float y = conv1(c, t);
      if (vh < 16) ring[tw * CONV + c] = PRE ? sm.x[t] : x[c];
      if (t < HK) { sm.q[t] = y; sq = fmaf(y, y, sq); }
      else { sm.k[t - HK] = y; sk = fmaf(y, y, sk); }
    }
    for (int t = tid; t < HK; t += NT) {
      const int cv = 4096 + vh * HK + t;
      sm.v[t] = conv1(cv, 2 * HK + t);
      ring[tw * CONV + cv] = PRE ? sm.x[2 * HK + t] : x[cv];
      sm.z[t] = bf2f(PRE ? sm.x[3 * HK + t] : x[Z_OFF + vh * HK + t]);
    }
    uint16_t a_raw, b_raw;
    if (PRE) {
      a_raw = uint16_t(sm.ab[0] >> (((A_OFF + vh) & 1) * 16));
      b_raw = uint16_t(sm.ab[1] >> (((B_OFF + vh) & 1) * 16));
    } else {
      a_raw = x[A_OFF + vh];
      b_raw = x[B_OFF + vh];
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      sm.red[warp] = sq;
      sm.red[PCONSUMERS + warp] = sk;
    }
    pconsumer_sync();
    // every read of the prefetch buffer is done: fetch the next item's inputs
    if (PRE && u + (int)gridDim.x < n_items) prefetch_item(sm, a, u + gridDim.x, tid);
    float tq = 0.0f, tk = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < PCONSUMERS; ++w2) {
      tq += sm.red[w2];
      tk += sm.red[PCONSUMERS + w2];
    }
    const float qs = 1.0f / sqrtf(tq + EPS), ks = 1.0f / sqrtf(tk + EPS);
    const float biased = bf2f(a_raw) + a.dt_bias[vh];
    const float sp = (biased > 20.0f) ? biased : logf(1.0f + softplus_exp(biased, a.ref_math));
    const float decay = expf(sp * a.ssm_a[vh]);
    const float beta = gate_sigmoid(bf2f(b_raw), a.ref_math);
    float4 k4 = reinterpret_cast<const float4*>(sm.k)[lane];
    float4 q4 = reinterpret_cast<const float4*>(sm.q)[lane];
    k4.x *= ks; k4.y *= ks; k4.z *= ks; k4.w *= ks;
    q4.x *= qs; q4.y *= qs; q4.z *= qs; q4.w *= qs;

    // ---- delta rule over the 4 chunks: warp w owns rows 4w..4w+3 of a chunk
    float ssq = 0.0f;
    for (int j = 0; j < HK / PCHUNK; ++j, ++i) {
      const int s = i % PSTAGES;
      if (!aborted && !mbar_wait(&sm.full[s], (i / PSTAGES) & 1, a.err)) aborted = true;
      if (aborted) continue;
      const float4* srow = reinterpret_cast<const float4*>(sm.st[s]);
      float4 rr[PRPW];
      float skr[PRPW];
#pragma unroll
      for (int r = 0; r < PRPW; ++r) {
        float4 v = srow[(warp * PRPW + r) * 32 + lane];
        v.x *= decay; v.y *= decay; v.z *= decay; v.w *= decay;
        rr[r] = v;
        float d = v.x * k4.x;
        d = fmaf(v.y, k4.y, d);
        d = fmaf(v.z, k4.z, d);
        d = fmaf(v.w, k4.w, d);
        skr[r] = d;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);  // stage free: rows are in registers
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
        for (int r = 0; r < PRPW; ++r) skr[r] += __shfl_xor_sync(FULL_MASK, skr[r], m);
      float o[PRPW];
      float4* grow = reinterpret_cast<float4*>(st + j * PCHUNK * HK);
#pragma unroll
      for (int r = 0; r < PRPW; ++r) {
        const int row = warp * PRPW + r;
        const float dd = beta * (sm.v[j * PCHUNK + row] - skr[r]);
        float4 v = rr[r];
        v.x = fmaf(k4.x, dd, v.x);
        v.y = fmaf(k4.y, dd, v.y);
        v.z = fmaf(k4.z, dd, v.z);
        v.w = fmaf(k4.w, dd, v.w);
        __stcs(grow + row * 32 + lane, v);
        float d = v.x * q4.x;
        d = fmaf(v.y, q4.y, d);
        d = fmaf(v.z, q4.z, d);
        d = fmaf(v.w, q4.w, d);
        o[r] = d;
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
        for (int r = 0; r < PRPW; ++r) o[r] += __shfl_xor_sync(FULL_MASK, o[r], m);
#pragma unroll
      for (int r = 0; r < PRPW; ++r) {
        const float ov = o[r] * SSM_SCALE;
        if (lane == r) sm.o[j * PCHUNK + warp * PRPW + r] = ov;
        ssq = fmaf(ov, ov, ssq);
      }
    }
    // ---- gated RMSNorm (src/engine.cpp:3307-3322)
    if (lane == 0) sm.red[2 * PCONSUMERS + warp] = ssq;
    pconsumer_sync();
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < PCONSUMERS; ++q) tot += sm.red[2 * PCONSUMERS + q];
    const float rms = 1.0f / sqrtf(tot / 128.0f + EPS);
    for (int t = tid; !aborted && t < HK; t += NT) {
      const float yy = (sm.o[t] * rms) * a.ssm_norm[t] * act_silu(sm.z[t], a.ref_math);
      a.out[(int64_t)b * 4096 + vh * HK + t] = f2bf(yy);
    }
    pconsumer_sync();  // sm.q/k/v/z/o/red are rewritten by the next item
  }
}

cudaError_t launch_persistent(const GdnArgs& a, cudaStream_t s) {
  static PerDeviceOnce configured;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(gdn_decode_persistent<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(PSmem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gdn_decode_persistent<false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PSmem));
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  const int items = a.n * 32;
  const int grid = items < QC_GDN_CTAS * nsm ? items : QC_GDN_CTAS * nsm;
  // the prologue prefetch copies 16-byte runs: proj rows (24704 B apart),
  // ring slots and conv weights must start on 16-byte boundaries
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.proj) | reinterpret_cast<uintptr_t>(a.ring) |
                         reinterpret_cast<uintptr_t>(a.conv_w)) & 15) == 0 &&
                       (a.ring_stride * 2) % 16 == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(PTHREADS, 1, 1);
  cfg.dynamicSmemBytes = sizeof(PSmem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = QC_GDN_PDL_LARGE;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return aligned ? cudaLaunchKernelEx(&cfg, gdn_decode_persistent<true>, a)
                 : cudaLaunchKernelEx(&cfg, gdn_decode_persistent<false>, a);
}

template <int R, int T>
cudaError_t launch_r(const GdnArgs& a, cudaStream_t s) {
  constexpr int smem = (HK / R) * HK * 4;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(gdn_decode_kernel<R, T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(32 * R, a.n, 1);
  cfg.blockDim = dim3(T, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = QC_GDN_PDL_SMALL;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = R;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = R > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gdn_decode_kernel<R, T>, a);
}

}  // namespace

cudaError_t launch_gdn_decode(const GdnArgs& a, cudaStream_t s) {
  if (a.n <= 0) return cudaSuccess;
  // Small batches split each head over a cluster of 8 CTAs to fill the 148
  // SMs; large batches give each (sequence, head) one CTA streaming the whole
  // 64 KiB state slice.
  // Measured on B200 (us/token/layer, batch 1 / 4 / 8): clusters of 4 CTAs
  // x 256 threads 6.5 / 2.2 / 1.8; clusters of 2 x 256 6.8 / 2.07 / 1.39;
  // persistent 9.6 / 2.5 / 1.37 and best from 16 up.
#ifndef QC_GDN_R_SMALL
#define QC_GDN_R_SMALL 1
#endif
#ifndef QC_GDN_T_SMALL
#define QC_GDN_T_SMALL 512
#endif
#ifndef QC_GDN_CLUSTER_MAX
#define QC_GDN_CLUSTER_MAX 8
#endif
#ifndef QC_GDN_R_TINY
#define QC_GDN_R_TINY 4
#endif
#ifndef QC_GDN_T_TINY
#define QC_GDN_T_TINY 256
#endif
  if (a.n <= 2) return launch_r<QC_GDN_R_TINY, QC_GDN_T_TINY>(a, s);
  if (a.n <= QC_GDN_CLUSTER_MAX) return launch_r<QC_GDN_R_SMALL, QC_GDN_T_SMALL>(a, s);
  return launch_persistent(a, s);
}

}  // namespace qc
