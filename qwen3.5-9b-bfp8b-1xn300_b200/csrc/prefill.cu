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
// fp32 state in registers (2 rows per warp, one float4 per lane and row) and
// runs the delta rule token after token — the state is read from and written
// to HBM once per chunk instead of once per token.  Phase C applies
// the gated RMSNorm per token.  The conv ring is advanced by a separate
// launch after all heads have read it (gdn_prefill_ring_kernel).
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
constexpr int PCONS = ROWS / 16;              // consumer warps, 16 rows each
constexpr int PTHREADS = (PCONS + 1) * 32;
constexpr int BOX_ROWS = 16;
constexpr int BOX_BYTES = BOX_ROWS * 128;
constexpr float SCALE_LOG2 = 0.0625f * 1.4426950408889634f;

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
  const int T = a.T, pos0 = a.pos0;
  const float* w = a.conv_w;
  // first half of a split cluster barrier: peers may write our shared memory
  // after their matching wait
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // ---- phase A: conv + SiLU of q, k (all 128 channels) and of this CTA's v
  // channels, every token of the chunk (src/engine.cpp:3204-3234)
  constexpr int NCH = 2 * HK + GRB;
  for (int idx = tid; idx < T * NCH; idx += 256) {
    const int t = idx / NCH, ch = idx % NCH;
    const int c = (ch < HK) ? kh * HK + ch
                : (ch < 2 * HK) ? 2048 + kh * HK + (ch - HK)
                                : 4096 + vh * HK + r * GRB + (ch - 2 * HK);
    float xs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = pos0 + t - 3 + j;  // tap j reads position p
      xs[j] = (p >= pos0) ? bf2f(a.proj[(int64_t)(p - pos0) * 12352 + c])
                          : bf2f(a.ring[(p & 3) * CONV + c]);
    }
    float y = xs[0] * w[c];
    y = fmaf(xs[1], w[CONV + c], y);
    y = fmaf(xs[2], w[2 * CONV + c], y);
    y = fmaf(xs[3], w[3 * CONV + c], y);
    y = silu_exact(y);
    if (ch < HK) sm.q[t][ch] = y;
    else if (ch < 2 * HK) sm.k[t][ch - HK] = y;
    else sm.v[t][ch - 2 * HK] = y;
  }
  if (tid < T) {  // decay and beta (src/engine.cpp:3277-3281)
    const uint16_t* x = a.proj + (int64_t)tid * 12352;
    const float biased = bf2f(x[12288 + vh]) + a.dt_bias[vh];
    const float sp = (biased > 20.0f) ? biased : logf(1.0f + expf(biased));
    sm.decay[tid] = expf(sp * a.ssm_a[vh]);
    sm.beta[tid] = sigmoid_exact(bf2f(x[12320 + vh]));
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
  }
  __syncthreads();

  // ---- phase B: delta rule token by token, this warp's rows in registers
  const int row0 = warp * GRPW;  // local row
  float* st = a.state + (int64_t)vh * HK * HK + (int64_t)r * GRB * HK;
  float4 S[GRPW];
#pragma unroll
  for (int i = 0; i < GRPW; ++i) S[i] = reinterpret_cast<const float4*>(st)[(row0 + i) * 32 + lane];
  for (int t = 0; t < T; ++t) {
    const float4 k4 = reinterpret_cast<const float4*>(sm.k[t])[lane];
    const float4 q4 = reinterpret_cast<const float4*>(sm.q[t])[lane];
    const float dec = sm.decay[t], bt = sm.beta[t];
    float sk[GRPW];
#pragma unroll
    for (int i = 0; i < GRPW; ++i) {
      S[i].x *= dec; S[i].y *= dec; S[i].z *= dec; S[i].w *= dec;
      float d = S[i].x * k4.x;
      d = fmaf(S[i].y, k4.y, d);
      d = fmaf(S[i].z, k4.z, d);
      d = fmaf(S[i].w, k4.w, d);
      sk[i] = d;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
      for (int i = 0; i < GRPW; ++i) sk[i] += __shfl_xor_sync(FULL_MASK, sk[i], m);
    float o[GRPW];
#pragma unroll
    for (int i = 0; i < GRPW; ++i) {
      const float dd = bt * (sm.v[t][row0 + i] - sk[i]);
      S[i].x = fmaf(k4.x, dd, S[i].x);
      S[i].y = fmaf(k4.y, dd, S[i].y);
      S[i].z = fmaf(k4.z, dd, S[i].z);
      S[i].w = fmaf(k4.w, dd, S[i].w);
      float d = S[i].x * q4.x;
      d = fmaf(S[i].y, q4.y, d);
      d = fmaf(S[i].z, q4.z, d);
      d = fmaf(S[i].w, q4.w, d);
      o[i] = d;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
      for (int i = 0; i < GRPW; ++i) o[i] += __shfl_xor_sync(FULL_MASK, o[i], m);
    if (lane < GRPW) {
      float ov = o[0];
#pragma unroll
      for (int i = 1; i < GRPW; ++i) ov = (lane == i) ? o[i] : ov;
      sm.o[t][row0 + lane] = ov * SSM_SCALE;
    }
  }
#pragma unroll
  for (int i = 0; i < GRPW; ++i) reinterpret_cast<float4*>(st)[(row0 + i) * 32 + lane] = S[i];
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
  for (int idx = tid; idx < T * GRB; idx += 256) {
    const int t = idx / GRB, d = idx % GRB;
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < GR; ++q) tot += sm.ssq[q][t];
    const float rms = 1.0f / sqrtf(tot / 128.0f + EPS);
    const int dd = r * GRB + d;
    const float z = bf2f(a.proj[(int64_t)t * 12352 + 8192 + vh * HK + dd]);
    const float y = (sm.o[t][d] * rms) * a.ssm_norm[dd] * silu_exact(z);
    a.out[(int64_t)t * 4096 + vh * HK + dd] = f2bf(y);
  }
}

// Advance the conv ring past the chunk: positions max(pos0, pos0 + T - 4) ..
// pos0 + T - 1 land in slots position & 3 (the four most recent inputs).
__global__ void gdn_prefill_ring_kernel(const GdnPrefillArgs a) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= CONV) return;
  const int first = max(0, a.T - 4);
  for (int t = first; t < a.T; ++t)
    a.ring[((a.pos0 + t) & 3) * CONV + c] = a.proj[(int64_t)t * 12352 + c];
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

struct __align__(1024) PrefillSmem {
  uint16_t k[PSTAGES][PAGE * HD];   // swizzled tiles, as in decode
  uint16_t v[PSTAGES][PAGE * HD];
  uint16_t q[ROWS * HD];            // swizzled: [col block 4][row 128][128 B]
  uint64_t full[PSTAGES];
  uint64_t empty[PSTAGES];
};

// byte offset of (row, dim) in a swizzled tile of `rows` rows
__device__ __forceinline__ uint32_t pswz(int row, int dim, int rows) {
  return (uint32_t)((dim >> 6) * (rows * 128) + row * 128 + ((((dim & 63) >> 3) ^ (row & 7)) << 4));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
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

__global__ void __launch_bounds__(PTHREADS, 1)
    attn_prefill_kernel(const AttnPrefillArgs a, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ unsigned char raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                                    ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y, split = blockIdx.x;
  const int end = a.pos0 + a.T;                     // positions [0, end) exist
  const int n_pages = (end + PAGE - 1) / PAGE;
  const int per = (n_pages + a.n_split - 1) / a.n_split;
  const int pg0 = split * per, pg1 = min(n_pages, pg0 + per);
  float* rec = a.rec + ((int64_t)kvh * a.n_split + split) * ROWS * (HD + 2);

  if (tid == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], PCONS);
    }
    fence_mbar_init();
  }
  // q tile of this kv-head into shared memory, swizzled; rows of tokens
  // beyond the chunk are zero
  for (int i = tid; i < ROWS * (HD / 8); i += PTHREADS) {
    const int row = i / (HD / 8), ch = i % (HD / 8);
    uint4 w = make_uint4(0, 0, 0, 0);
    if ((row % TMAX) < a.T)
      w = *reinterpret_cast<const uint4*>(a.q_buf + ((int64_t)kvh * ROWS + row) * HD + ch * 8);
    *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(sm.q) + pswz(row, ch * 8, ROWS)) = w;
  }
  __syncthreads();

  if (warp == PCONS) {  // ---------------------------------------- producer
    if (lane != 0) return;
    for (int pg = pg0, i = 0; pg < pg1; ++pg, ++i) {
      const int s = i % PSTAGES;
      if (i >= PSTAGES && !mbar_wait(&sm.empty[s], ((i / PSTAGES) - 1) & 1, a.err)) return;
      const int pid = a.page_row[pg];
      const int rows = min(PAGE, end - pg * PAGE);
      const int nbox = (pid >= 0 && pid < a.max_pages) ? (rows + BOX_ROWS - 1) / BOX_ROWS : 0;
      if (nbox == 0) record_error(a.err, QC_ERR_BOUNDS);
      mbar_arrive_expect_tx(&sm.full[s], uint32_t(nbox * 4 * BOX_BYTES * 2));
      const int row0 = (pid * 4 + kvh) * PAGE;
      for (int rb = 0; rb < nbox; ++rb)
        for (int cb = 0; cb < 4; ++cb) {
          const int off = (cb * PAGE * 128 + rb * BOX_BYTES) / 2;
          tma2d(&sm.k[s][off], &tmk, cb * 64, row0 + rb * BOX_ROWS, &sm.full[s]);
          tma2d(&sm.v[s][off], &tmv, cb * 64, row0 + rb * BOX_ROWS, &sm.full[s]);
        }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int g = lane >> 2, t4 = lane & 3;
  const int r0 = warp * 16;                 // rows r0..r0+15 = head (r0 / 32), tokens
  const int tok_a = (r0 % TMAX) + g;        // token of accumulator rows g (c0, c1)
  const int tok_b = tok_a + 8;              // and g + 8 (c2, c3)
  float o[32][4];
#pragma unroll
  for (int n = 0; n < 32; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
  bool aborted = false;
  const uint32_t qbase = smem_u32(sm.q);
  for (int pg = pg0, i = 0; pg < pg1; ++pg, ++i) {
    const int s = i % PSTAGES;
    if (!aborted && !mbar_wait(&sm.full[s], (i / PSTAGES) & 1, a.err)) aborted = true;
    if (aborted) continue;
    const uint32_t kb = smem_u32(sm.k[s]), vb = smem_u32(sm.v[s]);
    const int rows = min(PAGE, end - pg * PAGE);
    // ---- S[16 rows x 64 pos] = Q . K^T
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      uint32_t af[4];
      ldsm4(qbase + pswz(r0 + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * j + (lane >> 4) * 8, ROWS),
            af);
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // n-tiles 2np, 2np + 1
        uint32_t bf[4];
        ldsm4(kb + pswz(16 * np + (lane & 7) + (lane >> 4) * 8, 16 * j + ((lane >> 3) & 1) * 8,
                        PAGE),
              bf);
        mma16816(sc[2 * np], af, bf[0], bf[1]);
        mma16816(sc[2 * np + 1], af, bf[2], bf[3]);
      }
    }
    // ---- mask (position exists, causal inside the chunk) and online softmax
    const int base = pg * PAGE;
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kp = base + n * 8 + 2 * t4 + e, col = n * 8 + 2 * t4 + e;
        const bool va = col < rows && kp <= a.pos0 + tok_a && tok_a < a.T;
        const bool vb2 = col < rows && kp <= a.pos0 + tok_b && tok_b < a.T;
        sc[n][e] = va ? sc[n][e] * SCALE_LOG2 : -INFINITY;
        sc[n][2 + e] = vb2 ? sc[n][2 + e] * SCALE_LOG2 : -INFINITY;
        mx_a = fmaxf(mx_a, sc[n][e]);
        mx_b = fmaxf(mx_b, sc[n][2 + e]);
      }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(FULL_MASK, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(FULL_MASK, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(FULL_MASK, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(FULL_MASK, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float c_a = (mn_a == -INFINITY) ? 1.0f : exp2f(m_a - mn_a);
    const float c_b = (mn_b == -INFINITY) ? 1.0f : exp2f(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    float ps_a = 0.0f, ps_b = 0.0f;
    uint32_t pa[4][4];  // A fragments of P for the 4 k-steps of 16 positions
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = (sc[n][0] == -INFINITY) ? 0.0f : exp2f(sc[n][0] - mn_a);
      const float p1 = (sc[n][1] == -INFINITY) ? 0.0f : exp2f(sc[n][1] - mn_a);
      const float p2 = (sc[n][2] == -INFINITY) ? 0.0f : exp2f(sc[n][2] - mn_b);
      const float p3 = (sc[n][3] == -INFINITY) ? 0.0f : exp2f(sc[n][3] - mn_b);
      ps_a += p0 + p1;
      ps_b += p2 + p3;
      // k-step n/2: a0/a1 from the even n-tile, a2/a3 from the odd one
      pa[n >> 1][(n & 1) * 2 + 0] = pack2(p0, p1);
      pa[n >> 1][(n & 1) * 2 + 1] = pack2(p2, p3);
    }
    l_a = fmaf(l_a, c_a, ps_a);
    l_b = fmaf(l_b, c_b, ps_b);
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      o[n][0] *= c_a; o[n][1] *= c_a;
      o[n][2] *= c_b; o[n][3] *= c_b;
    }
    // ---- O[16 x 256] += P[16 x 64] . V[64 x 256]
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 16; ++dp) {  // n-tiles 2dp, 2dp + 1 (dims 16dp..16dp+15)
        uint32_t bf[4];
        ldsm4t(vb + pswz(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, 16 * dp + (lane >> 4) * 8,
                         PAGE),
               bf);
        mma16816(o[2 * dp], pa[kk], bf[0], bf[1]);
        mma16816(o[2 * dp + 1], pa[kk], bf[2], bf[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }
  // ---- records: m (log2 domain), l, o unnormalised, per row
  l_a += __shfl_xor_sync(FULL_MASK, l_a, 1);
  l_a += __shfl_xor_sync(FULL_MASK, l_a, 2);
  l_b += __shfl_xor_sync(FULL_MASK, l_b, 1);
  l_b += __shfl_xor_sync(FULL_MASK, l_b, 2);
  float* ra = rec + (int64_t)(r0 + g) * (HD + 2);
  float* rb = rec + (int64_t)(r0 + g + 8) * (HD + 2);
  if (t4 == 0) {
    ra[0] = m_a; ra[1] = l_a;
    rb[0] = m_b; rb[1] = l_b;
  }
#pragma unroll
  for (int n = 0; n < 32; ++n) {
    const int d = n * 8 + 2 * t4;
    ra[2 + d] = o[n][0];
    ra[3 + d] = o[n][1];
    rb[2 + d] = o[n][2];
    rb[3 + d] = o[n][3];
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
    M = fmaxf(M, a.rec[(((int64_t)kvh * a.n_split + sp) * ROWS + row) * (HD + 2)]);
  float L = 0.0f, O = 0.0f;
  for (int sp = 0; sp < a.n_split; ++sp) {
    const float* r = a.rec + (((int64_t)kvh * a.n_split + sp) * ROWS + row) * (HD + 2);
    const float f = (r[0] == -INFINITY) ? 0.0f : exp2f(r[0] - M);
    L = fmaf(f, r[1], L);
    O = fmaf(f, r[2 + d], O);
  }
  const int h = kvh * 4 + hh;
  const float gt = bf2f(a.proj[(int64_t)t * 10240 + h * 2 * HD + HD + d]);
  a.out[(int64_t)t * 4096 + h * HD + d] = f2bf((O / L) * sigmoid_exact(gt));
}

}  // namespace

cudaError_t launch_gdn_prefill(const GdnPrefillArgs& a, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(gdn_prefill_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(GdnPrefillSmem));
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, gdn_prefill_kernel, a);
  if (e != cudaSuccess) return e;
  gdn_prefill_ring_kernel<<<CONV / 256, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace qc

namespace qc {

int attn_prefill_smem_bytes() { return (int)sizeof(PrefillSmem) + 1024; }

cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, const CUtensorMap& tmk,
                                const CUtensorMap& tmv, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn_prefill_smem_bytes());
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  prefill_qk_kernel<<<a.T, 640, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_prefill_kernel<<<dim3(a.n_split, 4), PTHREADS, attn_prefill_smem_bytes(), s>>>(a, tmk, tmv);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  prefill_combine_kernel<<<dim3(ROWS, 4), 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace qc
