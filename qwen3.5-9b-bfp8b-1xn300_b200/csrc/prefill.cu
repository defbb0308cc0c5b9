// prefill.cu — chunked prefill of T <= QC_PREFILL_CHUNK tokens of one
// sequence.  The reference prefills token by token with the decode math
// (src/engine.cpp:2602-2722 DeltaNet, :2843-2929 attention); these kernels
// compute the same function for a whole chunk per launch.
//
// DeltaNet (gdn_prefill_kernel): a cluster of 8 CTAs per v-head, CTA r owning
// 16 of the head's 128 state rows.  Phase A computes, for every token of the
// chunk in parallel, the causal conv + SiLU of the head's q and k channels and
// of the CTA's v channels (history from the conv ring, then the chunk's own
// inputs), the L2 norms, decay and beta.  Phase B keeps the CTA's rows of the
// fp32 state in registers (one row per half-warp, two float4 per lane) and
// runs the delta rule token after token — the state is read from and written
// to HBM once per chunk instead of once per token.  Phase C applies
// the gated RMSNorm per token.
//
// The conv of all channels runs first in gdn_prefill_conv_kernel, which also
// advances the conv ring.
//
// Attention: prefill_qk_kernel normalises and rotates the chunk's q (to a
// bf16 scratch tile) and k, and appends K/V into the pages (the decode
// append's exact recipe).  attn_prefill_kernel then runs, per kv-head and
// page range, a flash-attention pass over the pages with the 128 query rows
// of the group (4 heads x 32 tokens): 8 consumer warps of 16 rows each,
// S = Q.K^T and O += P.V on the tensor cores (mma.sync m16n8k16, bf16 in,
// fp32 accumulate) straight from the swizzled TMA tiles, P reused from the S
// accumulators as the A operand, causal mask inside the chunk; it writes one
// (m, l, o) record per row.  prefill_combine_kernel merges the page ranges and
// applies the output gate.  Q enters the MMAs rounded to bf16 (decode keeps
// a bf16 residual as well); the error this adds is ~1e-3 relative.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace qc {
namespace {

constexpr int HK = 128;
constexpr int CONV = 8192;
constexpr float EPS = 1e-6f;
constexpr float SSM_SCALE = 1.0f / 11.3137f;  // src/engine.cpp:3249
constexpr int TMAX = QC_PREFILL_CHUNK;
constexpr int HD = 256;
constexpr int PAGE = 64;
constexpr int ROWS = 4 * TMAX;                // query rows per kv-head: 4 heads x 32 tokens
constexpr int PSTAGES = 2;
constexpr int BOX_ROWS = KV_BOX_ROWS;
constexpr int BOX_BYTES = BOX_ROWS * 128;
constexpr float SCALE_LOG2 = 0.0625f * 1.4426950408889634f;
constexpr int REC = HD + 4;                   // record: m, l, 2 pad, o[256] (16 B aligned)

constexpr int GR = 8;            // CTAs per v-head (a cluster)
constexpr int GRB = HK / GR;     // state rows per CTA
constexpr int GRPW = GRB / 8;    // rows per warp

struct GdnPrefillSmem {
  float q[TMAX][HK];
  float k[TMAX][HK];
  float v[TMAX][GRB];
  float o[TMAX][GRB];
  float decay[TMAX];
  float beta[TMAX];
  float kq[TMAX];                // k_t . q_t of the normalised vectors
  float ssq[GR][TMAX];          // per-token partial sums of squares, slot per CTA
};

// Cluster of GR CTAs per v-head; CTA r owns state rows [r*GRB, (r+1)*GRB).
__global__ void __launch_bounds__(256, 1) gdn_prefill_kernel(const GdnPrefillArgs a) {
  extern __shared__ __align__(16) unsigned char raw[];
  GdnPrefillSmem& sm = *reinterpret_cast<GdnPrefillSmem*>(raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int vh = blockIdx.x / GR, r = static_cast<int>(cluster.block_rank());
  const int kh = vh & 15;  // kh = vh % 16 (src/engine.cpp:3254)
  const int T = a.T;
  // first half of a split cluster barrier: peers may write our shared memory
  // after their matching wait
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // ---- phase A: the chunk's conv outputs of the head's q and k channels and
  // of this CTA's v channels (computed once per chunk by the conv kernel)
  // per token: 32 float4 of q, 32 of k, 4 of this CTA's v; all of a thread's
  // loads are issued before any is stored
  constexpr int NV4 = 2 * HK / 4 + GRB / 4;  // 68
  constexpr int NLD = (TMAX * NV4 + 255) / 256;
  {
    float4 buf[NLD];
#pragma unroll
    for (int u = 0; u < NLD; ++u) {
      const int idx = tid + 256 * u;
      buf[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (idx < T * NV4) {
        const int t = idx / NV4, e = idx % NV4;
        const int c = (e < 32) ? kh * HK + 4 * e
                    : (e < 64) ? 2048 + kh * HK + 4 * (e - 32)
                               : 4096 + vh * HK + r * GRB + 4 * (e - 64);
        buf[u] = *reinterpret_cast<const float4*>(a.conv_out + (int64_t)t * CONV + c);
      }
    }
#pragma unroll
    for (int u = 0; u < NLD; ++u) {
      const int idx = tid + 256 * u;
      if (idx < T * NV4) {
        const int t = idx / NV4, e = idx % NV4;
        float* dst = (e < 32) ? &sm.q[t][4 * e] : (e < 64) ? &sm.k[t][4 * (e - 32)] : &sm.v[t][4 * (e - 64)];
        *reinterpret_cast<float4*>(dst) = buf[u];
      }
    }
  }
  if (tid < T) {  // decay and beta (src/engine.cpp:3277-3281)
    const uint16_t* x = a.proj + (int64_t)tid * 12352;
    const float biased = bf2f(x[12288 + vh]) + a.dt_bias[vh];
    const float sp = (biased > 20.0f) ? biased : logf(1.0f + softplus_exp(biased, a.ref_math));
    sm.decay[tid] = expf(sp * a.ssm_a[vh]);
    sm.beta[tid] = gate_sigmoid(bf2f(x[12320 + vh]), a.ref_math);
  }
  __syncthreads();
  // L2 normalisation of q and k per token (src/engine.cpp:3261-3275)
  for (int t = warp; t < T; t += 8) {
    float4 q4 = reinterpret_cast<float4*>(sm.q[t])[lane];
    float4 k4 = reinterpret_cast<float4*>(sm.k[t])[lane];
    const float sq = warp_sum(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
    const float sk = warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w);
    const float qs = 1.0f / sqrtf(sq + EPS), ks = 1.0f / sqrtf(sk + EPS);
    q4.x *= qs; q4.y *= qs; q4.z *= qs; q4.w *= qs;
    k4.x *= ks; k4.y *= ks; k4.z *= ks; k4.w *= ks;
    reinterpret_cast<float4*>(sm.q[t])[lane] = q4;
    reinterpret_cast<float4*>(sm.k[t])[lane] = k4;
    const float kq = warp_sum(q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w);
    if (lane == 0) sm.kq[t] = kq;
  }
  __syncthreads();

  // ---- phase B: delta rule token by token, this warp's rows in registers:
  // half-warp h owns local row row0 + h, lane j of the half holds dims
  // 4j..4j+3 and 64+4j..64+4j+3, so each row's dot products reduce over 16
  // lanes (4 butterfly levels for both sums, 8 shuffles per token)
  static_assert(GRPW == 2, "one row per half-warp");
  const int hw = lane >> 4, j = lane & 15;
  const int row = warp * GRPW + hw;  // local row
  float* st = a.state + (int64_t)vh * HK * HK + (int64_t)r * GRB * HK;
  float4* srow = reinterpret_cast<float4*>(st) + row * 32;
  float4 S0 = srow[j], S1 = srow[j + 16];
  // Per token both dot products read the state before the token: with
  // sk = decay (S.k), d = beta (v - sk) and S' = decay S + d k^T, the
  // output is S'.q = decay (S.q) + d (k.q) — one reduction tree per token
  // instead of two in sequence.
  for (int t = 0; t < T; ++t) {
    const float4 ka = reinterpret_cast<const float4*>(sm.k[t])[j];
    const float4 kb = reinterpret_cast<const float4*>(sm.k[t])[j + 16];
    const float4 qa = reinterpret_cast<const float4*>(sm.q[t])[j];
    const float4 qb = reinterpret_cast<const float4*>(sm.q[t])[j + 16];
    const float dec = sm.decay[t], bt = sm.beta[t], kq = sm.kq[t], vv = sm.v[t][row];
    float sk = S0.x * ka.x, sk2 = S1.x * kb.x, sq = S0.x * qa.x, sq2 = S1.x * qb.x;
    sk = fmaf(S0.y, ka.y, sk);  sk2 = fmaf(S1.y, kb.y, sk2);
    sq = fmaf(S0.y, qa.y, sq);  sq2 = fmaf(S1.y, qb.y, sq2);
    sk = fmaf(S0.z, ka.z, sk);  sk2 = fmaf(S1.z, kb.z, sk2);
    sq = fmaf(S0.z, qa.z, sq);  sq2 = fmaf(S1.z, qb.z, sq2);
    sk = fmaf(S0.w, ka.w, sk);  sk2 = fmaf(S1.w, kb.w, sk2);
    sq = fmaf(S0.w, qa.w, sq);  sq2 = fmaf(S1.w, qb.w, sq2);
    sk += sk2;
    sq += sq2;
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) {
      sk += __shfl_xor_sync(FULL_MASK, sk, m);
      sq += __shfl_xor_sync(FULL_MASK, sq, m);
    }
    const float dd = bt * (vv - dec * sk);
    S0.x = fmaf(ka.x, dd, S0.x * dec);
    S0.y = fmaf(ka.y, dd, S0.y * dec);
    S0.z = fmaf(ka.z, dd, S0.z * dec);
    S0.w = fmaf(ka.w, dd, S0.w * dec);
    S1.x = fmaf(kb.x, dd, S1.x * dec);
    S1.y = fmaf(kb.y, dd, S1.y * dec);
    S1.z = fmaf(kb.z, dd, S1.z * dec);
    S1.w = fmaf(kb.w, dd, S1.w * dec);
    if (j == 0) sm.o[t][row] = fmaf(dd, kq, dec * sq) * SSM_SCALE;
  }
  srow[j] = S0;
  srow[j + 16] = S1;
  __syncthreads();

  // ---- phase C: gated RMSNorm per token (src/engine.cpp:3307-3322); the
  // per-token partial sums of squares of the cluster's CTAs meet in every
  // CTA's shared memory (plain remote stores), then one cluster barrier
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // peers have started
  for (int t = warp; t < T; t += 8) {
    float x = (lane < GRB) ? sm.o[t][lane] : 0.0f;
    const float ss = warp_sum(x * x);
    if (lane < GR) *cluster.map_shared_rank(&sm.ssq[r][t], lane) = ss;
  }
  cluster.sync();
#pragma unroll 2
  for (int idx = tid; idx < T * GRB; idx += 256) {
    const int t = idx / GRB, d = idx % GRB;
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < GR; ++q) tot += sm.ssq[q][t];
    const float rms = 1.0f / sqrtf(tot / 128.0f + EPS);
    const int dd = r * GRB + d;
    const float z = bf2f(a.proj[(int64_t)t * 12352 + 8192 + vh * HK + dd]);
    const float y = (sm.o[t][d] * rms) * a.ssm_norm[dd] * act_silu(z, a.ref_math);
    a.out[(int64_t)t * 4096 + vh * HK + dd] = f2bf(y);
  }
}

// Conv + SiLU of every channel for every token of the chunk
// (src/engine.cpp:3204-3234) into conv_out [T][8192] f32.  A CTA covers 32
// channels x 4 groups of 8 tokens; a group's history is the conv ring (first
// group) or the chunk's own earlier inputs.  After a CTA barrier — every read
// of the ring for these channels happens inside this CTA — the threads owning
// the chunk's last 4 tokens advance the ring (slot = position & 3).
constexpr int CONV_CH = 32;
constexpr int CONV_TG = 8;
__global__ void __launch_bounds__(128) gdn_prefill_conv_kernel(const GdnPrefillArgs a) {
  const int cl = threadIdx.x & 31, tg = threadIdx.x >> 5;
  const int c = blockIdx.x * CONV_CH + cl;
  const int pos0 = a.pos0, T = a.T, t0 = tg * CONV_TG;
  const float w0 = a.conv_w[c], w1 = a.conv_w[CONV + c], w2 = a.conv_w[2 * CONV + c],
              w3 = a.conv_w[3 * CONV + c];
  // history h[j] = input at chunk-relative token t0 - 3 + j
  float h[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = t0 - 3 + j;
    h[j] = (t < 0) ? bf2f(a.ring[((pos0 + t) & 3) * CONV + c])
                   : (t < T ? bf2f(a.proj[(int64_t)t * 12352 + c]) : 0.0f);
  }
  uint16_t xb[CONV_TG];
#pragma unroll
  for (int j = 0; j < CONV_TG; ++j)
    xb[j] = (t0 + j < T) ? a.proj[(int64_t)(t0 + j) * 12352 + c] : uint16_t(0);
#pragma unroll
  for (int j = 0; j < CONV_TG; ++j) {
    if (t0 + j >= T) break;
    const float x = bf2f(xb[j]);
    float y = h[0] * w0;
    y = fmaf(h[1], w1, y);
    y = fmaf(h[2], w2, y);
    y = fmaf(x, w3, y);
    a.conv_out[(int64_t)(t0 + j) * CONV + c] = act_silu(y, a.ref_math);
    h[0] = h[1];
    h[1] = h[2];
    h[2] = x;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < CONV_TG; ++j) {
    const int t = t0 + j;
    if (t < T && t >= T - 4) a.ring[((pos0 + t) & 3) * CONV + c] = xb[j];
  }
}

// ------------------------------------------------------------- attention

// q, k norm + RoPE and the K/V append for every token of the chunk: warp w < 16
// handles q-head w, warps 16-19 kv-head w - 16 (K) and its V row.
__global__ void __launch_bounds__(640) prefill_qk_kernel(const AttnPrefillArgs a) {
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = a.pos0 + t;
  const float* cs = a.rope_cos + (int64_t)pos * 32;
  const float* sn = a.rope_sin + (int64_t)pos * 32;
  const uint16_t* prow = a.proj + (int64_t)t * 10240;
  if (warp < 16) {
    float x[8];
    unpack8(*reinterpret_cast<const uint4*>(prow + warp * 2 * HD + lane * 8), x);
    norm_rope_lane(x, a.q_norm, cs, sn, lane);
    uint4 w;
    w.x = uint32_t(f2bf(x[0])) | (uint32_t(f2bf(x[1])) << 16);
    w.y = uint32_t(f2bf(x[2])) | (uint32_t(f2bf(x[3])) << 16);
    w.z = uint32_t(f2bf(x[4])) | (uint32_t(f2bf(x[5])) << 16);
    w.w = uint32_t(f2bf(x[6])) | (uint32_t(f2bf(x[7])) << 16);
    const int kvh = warp >> 2, row = (warp & 3) * TMAX + t;
    *reinterpret_cast<uint4*>(a.q_buf + ((int64_t)kvh * ROWS + row) * HD + lane * 8) = w;
    return;
  }
  const int kvh = warp - 16;
  const int pid = a.page_row[pos / PAGE];
  if (pid < 0 || pid >= a.max_pages) {
    if (lane == 0) record_error(a.err, QC_ERR_BOUNDS);
    return;
  }
  const int64_t off = (((int64_t)pid * 4 + kvh) * PAGE + (pos % PAGE)) * HD + lane * 8;
  float x[8];
  unpack8(*reinterpret_cast<const uint4*>(prow + 8192 + kvh * HD + lane * 8), x);
  norm_rope_lane(x, a.k_norm, cs, sn, lane);
  uint4 w;
  w.x = uint32_t(f2bf(x[0])) | (uint32_t(f2bf(x[1])) << 16);
  w.y = uint32_t(f2bf(x[2])) | (uint32_t(f2bf(x[3])) << 16);
  w.z = uint32_t(f2bf(x[4])) | (uint32_t(f2bf(x[5])) << 16);
  w.w = uint32_t(f2bf(x[6])) | (uint32_t(f2bf(x[7])) << 16);
  *reinterpret_cast<uint4*>(a.k_pool + off) = w;
  *reinterpret_cast<uint4*>(a.v_pool + off) =
      *reinterpret_cast<const uint4*>(prow + 9216 + kvh * HD + lane * 8);
}

// byte offset of (row, dim) in a swizzled tile of `rows` rows
__device__ __forceinline__ uint32_t pswz(int row, int dim, int rows) {
  return (uint32_t)((dim >> 6) * (rows * 128) + row * 128 + ((((dim & 63) >> 3) ^ (row & 7)) << 4));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y,
                                      uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------- tcgen05 flash pass

// warps 0-3: softmax (one query row per thread); warp 4 issues the MMAs,
// warp 5 the TMA loads
constexpr int TC_MMA_WARP = 4, TC_TMA_WARP = 5;
constexpr int TC_THREADS = 6 * 32;
constexpr uint32_t TMEM_COLS = 512;            // S x 2 (64 each) + O (256)
constexpr float RESCALE_THRESHOLD = 8.0f;      // log2 units: rescale O only past 2^8

struct __align__(1024) TcSmem {
  uint16_t q[ROWS * HD];            // [col block 4][row 128][128 B], swizzled
  uint16_t k[PSTAGES][PAGE * HD];   // [col block 4][pos 64][128 B]
  uint16_t v[PSTAGES][PAGE * HD];
  uint16_t p[2][ROWS * PAGE];       // double-buffered [row 128][128 B], swizzled
  uint64_t full[PSTAGES], empty[PSTAGES];
  // per tile parity b: s_* for the S buffers, p_full[b] (P written), o_done[b]
  // (P . V done); parity waits then never face a barrier two phases ahead
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2];
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(TC_THREADS, 1)
    attn_prefill_tc_kernel(const AttnPrefillArgs a, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ unsigned char raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                          ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y, split = blockIdx.x;
  const int end = a.pos0 + a.T;
  const int n_pages = (end + PAGE - 1) / PAGE;
  const int per = (n_pages + a.n_split - 1) / a.n_split;
  const int pg0 = split * per, pg1 = min(n_pages, pg0 + per);
  const int nt = max(0, pg1 - pg0);
  float* rec = a.rec + ((int64_t)kvh * a.n_split + split) * ROWS * REC;

  if (tid == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.s_free[b], 1);
    }
    mbar_init(&sm.p_full[0], 1);
    mbar_init(&sm.p_full[1], 1);
    mbar_init(&sm.o_done[0], 1);
    mbar_init(&sm.o_done[1], 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == TC_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // q tile of this kv-head, swizzled; rows of tokens beyond the chunk are zero.
  // Loads are batched 8 deep so their L2 latencies overlap.
  {
    constexpr int N16 = ROWS * (HD / 8);   // 16-byte chunks
    for (int i0 = tid; i0 < N16; i0 += 8 * TC_THREADS) {
      uint4 w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k * TC_THREADS, row = i / (HD / 8), ch = i % (HD / 8);
        w[k] = (i < N16 && (row % TMAX) < a.T)
                   ? *reinterpret_cast<const uint4*>(a.q_buf + ((int64_t)kvh * ROWS + row) * HD + ch * 8)
                   : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k * TC_THREADS, row = i / (HD / 8), ch = i % (HD / 8);
        if (i < N16)
          *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(sm.q) + pswz(row, ch * 8, ROWS)) = w[k];
      }
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_s[2] = {tmem, tmem + 64}, t_o = tmem + 128;

  if (warp == TC_TMA_WARP) {  // --------------------------------- producer
    if (lane == 0) {
      for (int i = 0; i < nt && !sm.abort; ++i) {
        const int s = i % PSTAGES, pg = pg0 + i;
        if (i >= PSTAGES && !mbar_wait(&sm.empty[s], ((i / PSTAGES) - 1) & 1, a.err)) {
          sm.abort = 1;
          break;
        }
        const int pid = a.page_row[pg];
        const int rows = min(PAGE, end - pg * PAGE);
        // all 64 rows of a valid page (one box per 64 rows); the softmax
        // warps zero the rows past `rows` before P.V reads them
        const int nbox = (pid >= 0 && pid < a.max_pages) ? PAGE / BOX_ROWS : 0;
        if (nbox == 0) record_error(a.err, QC_ERR_BOUNDS);
        (void)rows;
        mbar_arrive_expect_tx(&sm.full[s], uint32_t(nbox * 4 * BOX_BYTES * 2));
        const int row0 = (pid * 4 + kvh) * PAGE;
        for (int rb = 0; rb < nbox; ++rb)
          for (int cb = 0; cb < 4; ++cb) {
            const int off = (cb * PAGE * 128 + rb * BOX_BYTES) / 2;
            tma2d(&sm.k[s][off], &tmk, cb * 64, row0 + rb * BOX_ROWS, &sm.full[s]);
            tma2d(&sm.v[s][off], &tmv, cb * 64, row0 + rb * BOX_ROWS, &sm.full[s]);
          }
      }
    }
  } else if (warp == TC_MMA_WARP) {  // ------------------------- MMA issuer
    if (lane == 0) {
      // S = Q . K^T: M 128, N 64, K-major A and B
      const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) |
                            ((uint32_t(ROWS) >> 4) << 24);
      // O += P . V: M 128, N 256, A K-major, B (V [pos][dim]) MN-major
      const uint32_t id_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((256u >> 3) << 17) |
                            ((uint32_t(ROWS) >> 4) << 24);
      const uint32_t q_addr = smem_u32(sm.q);
      // S(i) = Q . K(i)^T into TMEM buffer i & 1
      auto issue_qk = [&](int i) -> bool {
        const int s = i % PSTAGES, b = i & 1;
        if (!mbar_wait(&sm.full[s], (i / PSTAGES) & 1, a.err)) return false;
        if (i >= 2 && !mbar_wait(&sm.s_free[b], ((i >> 1) - 1) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[s]);
        for (int cb = 0; cb < 4; ++cb)
          for (int ks = 0; ks < 4; ++ks)
            umma(t_s[b], umma_desc(q_addr + cb * ROWS * 128 + ks * 32, 16, 1024),
                 umma_desc(k_addr + cb * PAGE * 128 + ks * 32, 16, 1024), id_s, (cb | ks) != 0);
        umma_commit(&sm.s_full[b]);
        return true;
      };
      bool ok = nt == 0 || issue_qk(0);
      for (int i = 0; i < nt && ok; ++i) {
        // the next tile's scores run while the softmax works on this one
        if (i + 1 < nt && !(ok = issue_qk(i + 1))) break;
        if (!mbar_wait(&sm.p_full[i & 1], (i >> 1) & 1, a.err)) break;   // softmax wrote P(i)
        tc_fence_after();
        const int s = i % PSTAGES;
        const uint32_t v_addr = smem_u32(sm.v[s]), p_addr = smem_u32(sm.p[i & 1]);
        for (int kk = 0; kk < 4; ++kk)
          umma(t_o, umma_desc(p_addr + kk * 32, 16, 1024),
               umma_desc(v_addr + kk * 2048, PAGE * 128, 1024), id_o, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&sm.o_done[i & 1]);
        umma_commit(&sm.empty[s]);
      }
    }
  } else {  // ------------------------------------ softmax: thread = row
    const int row = warp * 32 + lane, tok = row % TMAX;
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    float m_ref = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int i = 0; i < nt && ok; ++i) {
      const int b = i & 1, pg = pg0 + i;
      const int rows = min(PAGE, end - pg * PAGE);
      ok = mbar_wait(&sm.s_full[b], (i >> 1) & 1, a.err);
      if (!ok) break;
      tc_fence_after();
      float sv[64];
      float (&s0)[32] = *reinterpret_cast<float(*)[32]>(&sv[0]);
      float (&s1)[32] = *reinterpret_cast<float(*)[32]>(&sv[32]);
      tmem_ld32(t_s[b] + lane_off, s0);
      tmem_ld32(t_s[b] + lane_off + 32, s1);
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (row == 0) mbar_arrive(&sm.s_free[b]);
      // rows of the page past its valid length hold whatever an earlier
      // sequence left in a reused page (possibly not finite): P is zero there,
      // but 0 * Inf would still reach O, so zero those V rows before P.V reads
      // them.  The tile landed (S(i) was computed from it); the proxy fence
      // before p_full orders these stores before the tensor-core read.  A row
      // is 128 B in each of the four 64-column boxes of the stage.
      if (rows < PAGE) {
        unsigned char* vs = reinterpret_cast<unsigned char*>(sm.v[i % PSTAGES]);
        for (int k = row; k < (PAGE - rows) * 32; k += 128) {
          const int r = rows + k / 32, cb = (k % 32) / 8, c16 = k % 8;
          *reinterpret_cast<uint4*>(vs + cb * PAGE * 128 + r * 128 + c16 * 16) =
              make_uint4(0, 0, 0, 0);
        }
      }
      // mask (position exists; causal inside the chunk) and scale
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const int kp = pg * PAGE + j;
        const bool valid = j < rows && kp <= a.pos0 + tok && tok < a.T;
        sv[j] = valid ? sv[j] * SCALE_LOG2 : -INFINITY;
        mt = fmaxf(mt, sv[j]);
      }
      // P buffer i & 1 was read by P . V of tile i - 2; O is complete up to
      // tile i - 1 only after that product, which a rescale must wait for.
      // Each o_done barrier completes once per tile of its parity, and the
      // phase waited for is always the newest it can have completed (P(i)
      // is not written yet), so parity waits are unambiguous.
      const bool rescale =
          mt > m_ref + RESCALE_THRESHOLD || (m_ref == -INFINITY && mt != -INFINITY);
      if (i >= 2) ok = mbar_wait(&sm.o_done[i & 1], ((i - 2) >> 1) & 1, a.err);
      if (ok && rescale && i >= 1) ok = mbar_wait(&sm.o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err);
      if (!ok) break;
      tc_fence_after();
      if (rescale) {
        const float f = (m_ref == -INFINITY) ? 0.0f : exp2f(m_ref - mt);
        if (i > 0) {
#pragma unroll 1
          for (int c = 0; c < 256; c += 32) {
            float ov[32];
            tmem_ld32(t_o + lane_off + c, ov);
#pragma unroll
            for (int j = 0; j < 32; ++j) ov[j] *= f;
            tmem_st32(t_o + lane_off + c, ov);
          }
        }
        l *= f;
        m_ref = mt;
      }
      // P = 2^(s - m_ref) in bf16, row-major 128 B per row, swizzled
      unsigned char* prow = reinterpret_cast<unsigned char*>(sm.p[i & 1]);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x = sv[ch * 8 + e];
          pv[e] = (x == -INFINITY) ? 0.0f : exp2f(x - m_ref);
          l += pv[e];
        }
        uint4 w;
        w.x = pack2(pv[0], pv[1]);
        w.y = pack2(pv[2], pv[3]);
        w.z = pack2(pv[4], pv[5]);
        w.w = pack2(pv[6], pv[7]);
        *reinterpret_cast<uint4*>(prow + row * 128 + ((ch ^ (row & 7)) << 4)) = w;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (row == 0) mbar_arrive(&sm.p_full[i & 1]);
    }
    // ---- record of this row: m (log2 domain), l, o unnormalised
    for (int k = max(0, nt - 2); k < nt && ok; ++k) ok = mbar_wait(&sm.o_done[k & 1], (k >> 1) & 1, a.err);
    float* r = rec + (int64_t)row * REC;
    if (ok && nt > 0) {
      tc_fence_after();
      r[0] = m_ref;
      r[1] = l;
#pragma unroll 1
      for (int c = 0; c < 256; c += 32) {
        float ov[32];
        tmem_ld32(t_o + lane_off + c, ov);
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(r + 4 + c + j) = make_float4(ov[j], ov[j + 1], ov[j + 2], ov[j + 3]);
      }
    } else {
      r[0] = -INFINITY;
      r[1] = 0.0f;
      for (int c = 0; c < 256; c += 4) *reinterpret_cast<float4*>(r + 4 + c) = make_float4(0, 0, 0, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TC_MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// Merge the page ranges of each row and apply the gate: block per (kv-head,
// row), thread per dimension.
__global__ void __launch_bounds__(256) prefill_combine_kernel(const AttnPrefillArgs a) {
  const int kvh = blockIdx.y, row = blockIdx.x, d = threadIdx.x;
  const int t = row % TMAX, hh = row / TMAX;
  if (t >= a.T) return;
  float M = -INFINITY;
  for (int sp = 0; sp < a.n_split; ++sp)
    M = fmaxf(M, a.rec[(((int64_t)kvh * a.n_split + sp) * ROWS + row) * REC]);
  float L = 0.0f, O = 0.0f;
  for (int sp = 0; sp < a.n_split; ++sp) {
    const float* r = a.rec + (((int64_t)kvh * a.n_split + sp) * ROWS + row) * REC;
    const float f = (r[0] == -INFINITY) ? 0.0f : exp2f(r[0] - M);
    L = fmaf(f, r[1], L);
    O = fmaf(f, r[4 + d], O);
  }
  const int h = kvh * 4 + hh;
  const float gt = bf2f(a.proj[(int64_t)t * 10240 + h * 2 * HD + HD + d]);
  a.out[(int64_t)t * 4096 + h * HD + d] = f2bf((O / L) * gate_sigmoid(gt, a.ref_math));
}

}  // namespace

cudaError_t launch_gdn_prefill(const GdnPrefillArgs& a, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(gdn_prefill_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(GdnPrefillSmem));
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  gdn_prefill_conv_kernel<<<CONV / CONV_CH, 32 * (TMAX / CONV_TG), 0, s>>>(a);
  cudaError_t e0 = cudaGetLastError();
  if (e0 != cudaSuccess) return e0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(32 * GR, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = sizeof(GdnPrefillSmem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = GR;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gdn_prefill_kernel, a);
}

}  // namespace qc

namespace qc {

int attn_prefill_smem_bytes() { return (int)sizeof(TcSmem) + 1024; }

cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, const CUtensorMap& tmk,
                                const CUtensorMap& tmv, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn_prefill_smem_bytes());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  prefill_qk_kernel<<<a.T, 640, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_prefill_tc_kernel<<<dim3(a.n_split, 4), TC_THREADS, attn_prefill_smem_bytes(), s>>>(a, tmk, tmv);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  prefill_combine_kernel<<<dim3(ROWS, 4), 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace qc
