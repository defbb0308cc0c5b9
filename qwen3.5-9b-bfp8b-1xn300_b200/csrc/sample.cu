// sample.cu — token sampling on sm_100a (sample_token, src/engine.cpp:
// 3979-4036): greedy argmax, or temperature softmax + top-p nucleus + one
// draw, for a batch of bf16 logit rows.
//
// The definition is the reference's with its open choices fixed (masses are
// integers, ties ordered by index, the draw passed in; see the header
// include/qsample.h), which makes the parallel result identical to a serial
// one: every sum below is an exact 64-bit integer sum.
//
// One cluster of SC = 8 CTAs per row, CTA r owning the logits
// [r * slice, (r + 1) * slice):
//   1. max and first argmax of the row (block reduction, then the 8 CTAs'
//      results exchanged through distributed shared memory);
//   2. each token's mass q = round(exp((l - max) / T) * 2^31) into shared
//      memory (exp evaluated with Cody-Waite reduction + Taylor series in
//      IEEE double, the same operations as the CPU restatement);
//   3. radix selection over the 32-bit masses, most significant byte first:
//      per pass a 256-bin histogram of (mass, count) of the tokens matching
//      the digits chosen so far — each thread sums runs of its tokens that
//      share a bin and adds them to its warp's histogram with integer
//      atomics; the histograms are summed per CTA and across the cluster —
//      then one warp scans the bins from the top for the one where the
//      running mass reaches the target.  Run once for the nucleus cut (target = top_p * Z) and once
//      for the draw (target = u * kept mass);
//   4. the drawn mass class holds equal-mass tokens in index order; the j-th
//      is located by per-CTA counts, a prefix over the cluster's ranks and a
//      block scan over contiguous per-thread sub-slices.
// No loop waits on another CTA except through the hardware cluster barrier.

#include <cooperative_groups.h>

#include <cstdint>
#include <string>

#include "../../include/qsample.h"
#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace qc {
namespace {

constexpr int SC = 8;                         // CTAs per row
constexpr int ST = 512;                       // threads per CTA
constexpr int SW = ST / 32;                   // warps per CTA
constexpr int SLICE_MAX = QC_SAMPLE_MAX_VOCAB / SC;

struct SampleSmem {
  uint32_t q[SLICE_MAX];                      // masses of this CTA's tokens
  unsigned long long wmass[SW][256];          // per-warp histograms
  uint32_t wcnt[SW][256];
  unsigned long long mass[256];               // this CTA's histogram
  uint32_t cnt[256];
  unsigned long long gmass[256];              // the cluster's histogram
  uint32_t gcnt[256];
  float red_f[SW];
  int red_i[SW];
  unsigned long long red_u[SW];
  float rank_max[SC];                         // written by every CTA of the cluster
  int rank_arg[SC];
  unsigned long long rank_sum[SC];
  int rank_cnt[SC];
  int sel_bin;
  unsigned long long sel_above;
  int scan[ST];
};

// exp(x) for x <= 0: Cody-Waite range reduction x = k ln2 + r, |r| <= ln2/2
// (ln2 as a 21-bit head, exact in k * head, plus a tail), the Taylor series
// of exp(r) to degree 13 by Horner's rule with fused multiply-adds, and the
// exact scaling by 2^k.  Only correctly rounded operations: the same bits as
// the CPU restatement.
__device__ __forceinline__ double exp_ref(double x) {
  if (x < -745.0) return 0.0;
  const double LN2_HI = 0.693145751953125;
  const double LN2_LO = 1.42860682030941723212e-06;
  const double k = rint(x * 1.4426950408889634074);
  const double r = fma(-k, LN2_LO, fma(-k, LN2_HI, x));
  double p = 1.0 / 6227020800.0;
  p = fma(p, r, 1.0 / 479001600.0);
  p = fma(p, r, 1.0 / 39916800.0);
  p = fma(p, r, 1.0 / 3628800.0);
  p = fma(p, r, 1.0 / 362880.0);
  p = fma(p, r, 1.0 / 40320.0);
  p = fma(p, r, 1.0 / 5040.0);
  p = fma(p, r, 1.0 / 720.0);
  p = fma(p, r, 1.0 / 120.0);
  p = fma(p, r, 1.0 / 24.0);
  p = fma(p, r, 1.0 / 6.0);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return scalbn(p, (int)k);
}

__device__ __forceinline__ uint32_t token_mass(float l, float max_l, float inv_t) {
  if (isnan(l)) return 0u;
  const float x = __fmul_rn(__fsub_rn(l, max_l), inv_t);
  // exp(-22.2) * 2^31 < 0.49: such tokens round to mass 0 (as they do in
  // the CPU restatement, which evaluates the exponential)
  if (x < -22.2f) return 0u;
  return (uint32_t)rint(exp_ref((double)x) * 2147483648.0);
}

// Selects the mass class at which the running mass (tokens in decreasing
// mass) first reaches `target`, restricted to nonempty classes.  Returns the
// class's mass value, the mass of all heavier tokens, and its token count.
// Tokens lighter than `lo` are left out: the caller knows the answer is at
// or above it (the draw lies inside the nucleus).
__device__ void radix_select(SampleSmem& sm, cg::cluster_group& cluster, int n_local,
                             uint32_t lo, unsigned long long target, uint32_t& value,
                             unsigned long long& above, uint32_t& count) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t prefix = 0, mask = 0;
  unsigned long long run = 0;
  for (int b = 3; b >= 0; --b) {
    for (int i = tid; i < SW * 256; i += ST) {
      (&sm.wmass[0][0])[i] = 0ull;
      (&sm.wcnt[0][0])[i] = 0u;
    }
    __syncthreads();
    // each thread sums runs of its own tokens that share a bin (most share
    // the lowest one) and flushes a run to its warp's histogram when the bin
    // changes: integer sums, so the order of the atomics does not matter
    int cur = -1;
    unsigned long long run_m = 0;
    uint32_t run_c = 0;
    for (int i = tid; i < n_local; i += ST) {
      const uint32_t q = sm.q[i];
      if (q < lo || (q & mask) != prefix) continue;
      const int bin = (int)((q >> (8 * b)) & 255u);
      if (bin != cur) {
        if (cur >= 0) {
          atomicAdd(&sm.wmass[warp][cur], run_m);
          atomicAdd(&sm.wcnt[warp][cur], run_c);
        }
        cur = bin;
        run_m = 0;
        run_c = 0;
      }
      run_m += q;
      ++run_c;
    }
    if (cur >= 0) {
      atomicAdd(&sm.wmass[warp][cur], run_m);
      atomicAdd(&sm.wcnt[warp][cur], run_c);
    }
    __syncthreads();
    if (tid < 256) {
      unsigned long long m = 0;
      uint32_t c = 0;
#pragma unroll
      for (int w = 0; w < SW; ++w) {
        m += sm.wmass[w][tid];
        c += sm.wcnt[w][tid];
      }
      sm.mass[tid] = m;
      sm.cnt[tid] = c;
    }
    cluster.sync();  // every CTA's histogram of this pass is complete
    if (tid < 256) {
      unsigned long long m = 0;
      uint32_t c = 0;
#pragma unroll
      for (int r = 0; r < SC; ++r) {
        m += *cluster.map_shared_rank(&sm.mass[tid], r);
        c += *cluster.map_shared_rank(&sm.cnt[tid], r);
      }
      sm.gmass[tid] = m;
      sm.gcnt[tid] = c;
    }
    cluster.sync();  // all peers have read this pass's histograms
    if (warp == 0) {
      // bins in decreasing order, 8 per lane: lane l owns bins 255-8l .. 248-8l
      unsigned long long bm[8], own = 0;
      uint32_t bc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        bm[e] = sm.gmass[255 - 8 * lane - e];
        bc[e] = sm.gcnt[255 - 8 * lane - e];
        own += bm[e];
      }
      unsigned long long before = own;
#pragma unroll
      for (int m = 1; m < 32; m <<= 1) {
        const unsigned long long o = __shfl_up_sync(FULL_MASK, before, m);
        if (lane >= m) before += o;
      }
      before -= own;  // mass of the heavier bins, owned by lower lanes
      int found = -1;
      unsigned long long r = run + before;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (found >= 0) continue;
        if (bc[e] != 0 && r + bm[e] >= target) found = e;
        else r += bm[e];
      }
      const unsigned hit = __ballot_sync(FULL_MASK, found >= 0);
      if (hit) {
        if (lane == __ffs(hit) - 1) {
          sm.sel_bin = 255 - 8 * lane - found;
          sm.sel_above = r;
        }
      } else if (lane == 0) {  // unreachable (targets never exceed the total): lightest class
        int sel = -1;
        unsigned long long rr = run;
        for (int bin = 0; bin < 256; ++bin)
          if (sm.gcnt[bin]) { sel = bin; break; }
        for (int bin = 255; bin > sel; --bin) rr += sm.gmass[bin];
        sm.sel_bin = sel;
        sm.sel_above = rr;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sm.sel_bin << (8 * b);
    mask |= 255u << (8 * b);
    run = sm.sel_above;
    if (b == 0) count = sm.gcnt[sm.sel_bin];
    __syncthreads();
  }
  value = prefix;
  above = run;
}

__global__ void __launch_bounds__(ST, 1) sample_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) unsigned char raw[];
  SampleSmem& sm = *reinterpret_cast<SampleSmem*>(raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster.block_rank(), row = blockIdx.x / SC;
  const int slice = a.slice;
  const int v0 = rank * slice;
  const int n_local = max(0, min(slice, a.vocab - v0));
  const uint16_t* lg = a.logits + (int64_t)row * a.ld + v0;

  // ---- 1. max and first argmax
  float best = -INFINITY;
  int arg = 0x7fffffff;
  for (int i = tid; i < n_local; i += ST) {
    const float l = bf2f(lg[i]);
    if (l > best) {  // i increases per thread: the first maximum is kept
      best = l;
      arg = v0 + i;
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float ob = __shfl_xor_sync(FULL_MASK, best, m);
    const int oa = __shfl_xor_sync(FULL_MASK, arg, m);
    if (ob > best || (ob == best && oa < arg)) { best = ob; arg = oa; }
  }
  if (lane == 0) { sm.red_f[warp] = best; sm.red_i[warp] = arg; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < SW; ++w)
      if (sm.red_f[w] > best || (sm.red_f[w] == best && sm.red_i[w] < arg)) {
        best = sm.red_f[w];
        arg = sm.red_i[w];
      }
    for (int r = 0; r < SC; ++r) {
      *cluster.map_shared_rank(&sm.rank_max[rank], r) = best;
      *cluster.map_shared_rank(&sm.rank_arg[rank], r) = arg;
    }
  }
  cluster.sync();
  best = -INFINITY;
  arg = 0x7fffffff;
  for (int r = 0; r < SC; ++r)
    if (sm.rank_max[r] > best || (sm.rank_max[r] == best && sm.rank_arg[r] < arg)) {
      best = sm.rank_max[r];
      arg = sm.rank_arg[r];
    }
  if (arg == 0x7fffffff) arg = 0;  // every logit NaN
  if (a.temperature <= 1e-7f) {
    if (rank == 0 && tid == 0) a.tokens[row] = arg;
    return;
  }

  // ---- 2. masses
  const float inv_t = __frcp_rn(a.temperature);
  unsigned long long zsum = 0;
  for (int i = tid; i < n_local; i += ST) {
    const uint32_t q = token_mass(bf2f(lg[i]), best, inv_t);
    sm.q[i] = q;
    zsum += q;
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) zsum += __shfl_xor_sync(FULL_MASK, zsum, m);
  if (lane == 0) sm.red_u[warp] = zsum;
  __syncthreads();
  if (tid == 0) {
    zsum = 0;
    for (int w = 0; w < SW; ++w) zsum += sm.red_u[w];
    for (int r = 0; r < SC; ++r) *cluster.map_shared_rank(&sm.rank_sum[rank], r) = zsum;
  }
  cluster.sync();
  unsigned long long z = 0;
  for (int r = 0; r < SC; ++r) z += sm.rank_sum[r];

  // ---- 3. nucleus cut, then the draw
  const unsigned long long target = (unsigned long long)((double)a.top_p * (double)z);
  uint32_t theta, cnt_theta;
  unsigned long long above;
  radix_select(sm, cluster, n_local, 0u, target, theta, above, cnt_theta);
  unsigned long long k = theta ? (target > above ? (target - above + theta - 1) / theta : 0) : 1;
  if (k < 1) k = 1;
  if (k > cnt_theta) k = cnt_theta;
  const unsigned long long kept = above + k * theta;
  const unsigned long long rdraw = (unsigned long long)(a.uniform[row] * (double)kept);
  uint32_t kappa, cnt_kappa;
  unsigned long long above2;
  radix_select(sm, cluster, n_local, theta, rdraw, kappa, above2, cnt_kappa);
  unsigned long long j = (rdraw > above2 && kappa) ? (rdraw - above2 + kappa - 1) / kappa : 1;
  if (j < 1) j = 1;

  // ---- 4. the j-th token (index order) of mass kappa
  const int per = (n_local + ST - 1) / ST;
  const int s0 = min(n_local, tid * per), s1 = min(n_local, s0 + per);
  int c = 0;
  for (int i = s0; i < s1; ++i) c += sm.q[i] == kappa;
  sm.scan[tid] = c;
  __syncthreads();
  {  // exclusive scan over the threads (warp shuffles, then the warp totals)
    int incl = c;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const int o = __shfl_up_sync(FULL_MASK, incl, m);
      if (lane >= m) incl += o;
    }
    if (lane == 31) sm.red_i[warp] = incl;
    __syncthreads();
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += sm.red_i[w];
    sm.scan[tid] = wbase + incl - c;
    if (tid == ST - 1) {
      const int total = wbase + incl;
      for (int r = 0; r < SC; ++r) *cluster.map_shared_rank(&sm.rank_cnt[rank], r) = total;
    }
  }
  cluster.sync();
  long long before = 0;
  for (int r = 0; r < rank; ++r) before += sm.rank_cnt[r];
  const long long want = (long long)j - 1;  // 0-based position in the class
  if (want >= before && want < before + sm.rank_cnt[rank]) {
    long long pos = before + sm.scan[tid];
    if (want >= pos && want < pos + c) {
      for (int i = s0; i < s1; ++i)
        if (sm.q[i] == kappa) {
          if (pos == want) {
            a.tokens[row] = v0 + i;
            break;
          }
          ++pos;
        }
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still read its memory
}

}  // namespace

size_t sample_smem_bytes() { return sizeof(SampleSmem); }

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t s) {
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(SampleSmem));
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(SC * a.batch, 1, 1);
  cfg.blockDim = dim3(ST, 1, 1);
  cfg.dynamicSmemBytes = sizeof(SampleSmem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = SC;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sample_kernel, a);
}

}  // namespace qc

extern "C" int qc_sample(const uint16_t* logits_dev, int64_t ld, int32_t vocab, int32_t batch,
                         float temperature, float top_p, const double* uniform_dev,
                         int32_t* tokens_dev, qc_stream stream) {
  qc::TraceRange trace_("qc_sample");
  if (!logits_dev || !tokens_dev || batch < 1 || vocab < 1 || vocab > QC_SAMPLE_MAX_VOCAB ||
      ld < vocab || !(top_p > 0.0f && top_p <= 1.0f) ||
      (temperature > 1e-7f && !uniform_dev)) {
    qc::set_thread_error("qc_sample: bad arguments");
    return QC_ERR_ARG;
  }
  qc::SampleArgs a{};
  a.logits = logits_dev;
  a.ld = ld;
  a.vocab = vocab;
  a.batch = batch;
  a.slice = (vocab + qc::SC - 1) / qc::SC;
  a.temperature = temperature;
  a.top_p = top_p;
  a.uniform = uniform_dev;
  a.tokens = tokens_dev;
  cudaError_t e = qc::launch_sample(a, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    qc::set_thread_error((std::string("qc_sample: ") + cudaGetErrorString(e)).c_str());
    return QC_ERR_CUDA;
  }
  return QC_OK;
}
