// gdn_decode.cu — one Gated-DeltaNet decode step, fused in a single
// memory-bound pass (src/engine.cpp:3204-3327).
//
// Work split: a cluster of R CTAs per (sequence, v-head); CTA r of the cluster
// owns state rows [r*128/R, (r+1)*128/R) of that head (rows are independent in
// the delta rule, src/engine.cpp:3284-3305).  The CTA
//   1. starts one bulk copy (TMA, cp.async.bulk) of its 128/R x 512 B state
//      slice into shared memory;
//   2. meanwhile runs the causal conv (width 4) + SiLU for the 128 q and 128 k
//      channels of k-head vh % 16 and its own v channels, and appends the new
//      input to the conv ring;
//   3. L2-normalises q and k, computes decay and beta;
//   4. per row: decay, s·k, delta, rank-1 update, s·q — one float4 per lane,
//      warp-shuffle dot products — and stores the row straight back to HBM
//      with 128-bit stores;
//   5. gated RMSNorm over the head's 128 outputs: the CTAs of the cluster
//      exchange their partial sums of squares through distributed shared
//      memory (no multicast), then each CTA writes its outputs as bf16.
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

template <int R>
__global__ void __launch_bounds__(128) gdn_decode_kernel(const GdnArgs a) {
  constexpr int RB = HK / R;   // state rows per CTA
  constexpr int RPW = RB / 4;  // rows per warp
  __shared__ __align__(128) float s_state[RB * HK];
  __shared__ __align__(16) float s_q[HK];
  __shared__ __align__(16) float s_k[HK];
  __shared__ float s_v[RB];
  __shared__ float s_z[RB];
  __shared__ float s_o[RB];
  __shared__ float s_red[8];
  __shared__ float s_ssq;
  __shared__ __align__(8) uint64_t s_bar;

  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.y;
  const int vh = blockIdx.x / R;
  const int r = static_cast<int>(cluster.block_rank());
  const int kh = vh & 15;  // kh = vh % 16 (src/engine.cpp:3254)
  const int slot = a.slots[b];
  const int pos = a.pos[b];
  float* st = a.state + slot * a.state_stride + (int64_t)vh * HK * HK + (int64_t)r * RB * HK;
  uint16_t* ring = a.ring + slot * a.ring_stride;
  const uint16_t* x = a.proj + (int64_t)b * 12352;

  if (tid == 0) {
    mbar_init(&s_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&s_bar, RB * HK * 4);
    bulk_g2s(s_state, st, RB * HK * 4, &s_bar);
  }

  // ---- conv1d + SiLU (src/engine.cpp:3204-3234), ring append
  const int t0 = (pos - 3) & 3, t1 = (pos - 2) & 3, t2 = (pos - 1) & 3, tw = pos & 3;
  const float* w = a.conv_w;
  auto conv1 = [&](int c) -> float {
    float y = bf2f(ring[t0 * CONV + c]) * w[c];
    y = fmaf(bf2f(ring[t1 * CONV + c]), w[CONV + c], y);
    y = fmaf(bf2f(ring[t2 * CONV + c]), w[2 * CONV + c], y);
    y = fmaf(bf2f(x[c]), w[3 * CONV + c], y);
    return silu_exact(y);
  };
  const int cq = kh * HK + tid;
  const int ck = 2048 + kh * HK + tid;
  const float qv = conv1(cq);
  const float kv = conv1(ck);
  if (vh < 16 && tid / RB == r) {  // one CTA of one v-head writes each q/k channel
    ring[tw * CONV + cq] = x[cq];
    ring[tw * CONV + ck] = x[ck];
  }
  if (tid < RB) {
    const int cv = 4096 + vh * HK + r * RB + tid;
    s_v[tid] = conv1(cv);
    ring[tw * CONV + cv] = x[cv];
    s_z[tid] = bf2f(x[Z_OFF + vh * HK + r * RB + tid]);
  }

  // ---- L2 normalisation of q and k (src/engine.cpp:3261-3275)
  {
    const float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
    if (lane == 0) {
      s_red[warp] = sq;
      s_red[4 + warp] = sk;
    }
    __syncthreads();
    const float tq = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
    const float tk = (s_red[4] + s_red[5]) + (s_red[6] + s_red[7]);
    s_q[tid] = qv * (1.0f / sqrtf(tq + EPS));
    s_k[tid] = kv * (1.0f / sqrtf(tk + EPS));
  }

  // ---- decay and beta (src/engine.cpp:3277-3281)
  const float biased = bf2f(x[A_OFF + vh]) + a.dt_bias[vh];
  const float sp = (biased > 20.0f) ? biased : logf(1.0f + expf(biased));
  const float decay = expf(sp * a.ssm_a[vh]);
  const float beta = sigmoid_exact(bf2f(x[B_OFF + vh]));
  __syncthreads();  // s_q, s_k, s_v ready

  const bool ok = mbar_wait(&s_bar, 0, a.err);

  // ---- delta rule (src/engine.cpp:3284-3305), rows of this warp
  float ssq_w = 0.0f;
  if (ok) {
    const float4 k4 = reinterpret_cast<const float4*>(s_k)[lane];
    const float4 q4 = reinterpret_cast<const float4*>(s_q)[lane];
    const float4* srow = reinterpret_cast<const float4*>(s_state);
    float4 rr[RPW];
    float sk[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      float4 v = srow[(warp * RPW + i) * 32 + lane];
      v.x *= decay; v.y *= decay; v.z *= decay; v.w *= decay;
      rr[i] = v;
      float d = v.x * k4.x;
      d = fmaf(v.y, k4.y, d);
      d = fmaf(v.z, k4.z, d);
      d = fmaf(v.w, k4.w, d);
      sk[i] = d;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
      for (int i = 0; i < RPW; ++i) sk[i] += __shfl_xor_sync(FULL_MASK, sk[i], m);
    float o[RPW];
    float4* grow = reinterpret_cast<float4*>(st);
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int row = warp * RPW + i;
      const float dd = beta * (s_v[row] - sk[i]);
      float4 v = rr[i];
      v.x = fmaf(k4.x, dd, v.x);
      v.y = fmaf(k4.y, dd, v.y);
      v.z = fmaf(k4.z, dd, v.z);
      v.w = fmaf(k4.w, dd, v.w);
      grow[row * 32 + lane] = v;  // coalesced 512 B per row
      float d = v.x * q4.x;
      d = fmaf(v.y, q4.y, d);
      d = fmaf(v.z, q4.z, d);
      d = fmaf(v.w, q4.w, d);
      o[i] = d;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
      for (int i = 0; i < RPW; ++i) o[i] += __shfl_xor_sync(FULL_MASK, o[i], m);
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const float ov = o[i] * SSM_SCALE;
      if (lane == i) s_o[warp * RPW + i] = ov;
      ssq_w = fmaf(ov, ov, ssq_w);
    }
  }
  if (lane == 0) s_red[warp] = ssq_w;
  __syncthreads();
  if (tid == 0) s_ssq = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);

  // ---- gated RMSNorm over the head's 128 outputs (src/engine.cpp:3307-3322)
  cluster.sync();
  float tot = 0.0f;
#pragma unroll
  for (int q = 0; q < R; ++q) tot += *cluster.map_shared_rank(&s_ssq, q);
  cluster.sync();  // peers may leave only after every CTA has read their sum
  if (!ok) return;
  if (tid < RB) {
    const float rms = 1.0f / sqrtf(tot / 128.0f + EPS);
    const int d = r * RB + tid;
    const float y = (s_o[tid] * rms) * a.ssm_norm[d] * silu_exact(s_z[tid]);
    a.out[(int64_t)b * 4096 + vh * HK + d] = f2bf(y);
  }
}

template <int R>
cudaError_t launch_r(const GdnArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(32 * R, a.n, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = R;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gdn_decode_kernel<R>, a);
}

}  // namespace

cudaError_t launch_gdn_decode(const GdnArgs& a, cudaStream_t s) {
  if (a.n <= 0) return cudaSuccess;
  // Small batches split each head over more CTAs to fill the 148 SMs.
  if (a.n <= 8) return launch_r<8>(a, s);
  return launch_r<4>(a, s);
}

}  // namespace qc
