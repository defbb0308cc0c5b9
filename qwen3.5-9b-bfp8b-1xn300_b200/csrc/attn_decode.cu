// attn_decode.cu — full-attention decode over the paged bf16 KV cache
// (src/engine.cpp:3485-3564).
//
// Kernel 1, attn_partial_kernel: one CTA per SM, each given an equal share of
// the batch's "page-heads" (one 64-token page of one kv-head: 32 KiB of K and
// 32 KiB of V, contiguous in the pool) in (sequence, kv-head, page) order —
// a split-K over KV positions that balances the work exactly whatever the
// mix of context lengths.  Warp 8 is the producer: it streams each page-head
// into a 2-stage shared-memory ring with two bulk copies (cp.async.bulk, the
// untiled TMA path; no multicast).  Warps 0-7 are consumers; each takes 8 of
// the 64 positions of a tile for all 4 query heads of the GQA group
// (kv_h = h / 4, src/engine.cpp:3532), keeps its own online-softmax state
// (m, l, o) in registers and reduces the 32 (position, head) dot products of
// a tile with one transposing warp-shuffle reduction (31 shuffles).  When the
// CTA leaves a (sequence, kv-head) pair it merges its 8 warps' states and
// writes one partial record.
//
// Fused prologue per pair: per-head RMSNorm + partial RoPE of the 4 query
// heads (src/engine.cpp:3497-3519) and, in the CTA that owns the page of the
// new position, the same for the new K plus the bf16 append of K and V into
// the page (src/engine.cpp:3521-3526); the new token is attended from shared
// memory, so no CTA reads a row another CTA is writing.
//
// Kernel 2, attn_combine_kernel: per (sequence, kv-head) merges the partial
// records of the CTAs that covered it, divides by the softmax sum and applies
// the sigmoid output gate (src/engine.cpp:3560-3563), storing bf16.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace qc {
namespace {

constexpr int HD = 256;
constexpr int PAGE = 64;
constexpr int STAGES = 2;
constexpr int N_CONSUMER = 8;
constexpr int THREADS = (N_CONSUMER + 1) * 32;
constexpr int TILE_BYTES = PAGE * HD * 2;  // 32 KiB for K or for V
// score * 1/16 (src/model_config.h:40), kept in the log2 domain for exp2
constexpr float SCALE_LOG2 = 0.0625f * 1.4426950408889634f;

struct Smem {
  uint16_t k[STAGES][PAGE * HD];
  uint16_t v[STAGES][PAGE * HD];
  float red_o[N_CONSUMER][4][HD];
  float q[4][HD];
  float red_ml[N_CONSUMER][8];
  float p[N_CONSUMER][32];
  uint16_t knew[HD];
  uint16_t vnew[HD];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(N_CONSUMER * 32) : "memory");
}

// lane l returns the sum over the warp of v[l] (a transposing reduction:
// 16 + 8 + 4 + 2 + 1 shuffles for 32 independent sums).
__device__ __forceinline__ float transpose_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) {
    const bool hi = (lane & k) != 0;
#pragma unroll
    for (int j = 0; j < k; ++j) {
      const float send = hi ? v[j] : v[j + k];
      const float keep = hi ? v[j + k] : v[j];
      v[j] = keep + __shfl_xor_sync(FULL_MASK, send, k);
    }
  }
  return v[0];
}

// Walks page-heads u in (sequence b, kv-head, page) order.
struct Cursor {
  int b, kvh, pg, np;
  __device__ void seek(const AttnArgs& a, int u) {
    int lo = 0, hi = a.n - 1;  // largest b with seg[b] <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.seg[mid] <= u) lo = mid; else hi = mid - 1;
    }
    b = lo;
    np = (a.seg[b + 1] - a.seg[b]) >> 2;
    const int rel = u - a.seg[b];
    kvh = rel / np;
    pg = rel - kvh * np;
  }
  __device__ void next(const AttnArgs& a) {
    if (++pg < np) return;
    pg = 0;
    if (++kvh < 4) return;
    kvh = 0;
    // skip sequences with no pages in range
    do {
      ++b;
      np = (b < a.n) ? ((a.seg[b + 1] - a.seg[b]) >> 2) : 1;
    } while (np == 0);
  }
};

struct TileInfo {
  int page_id;      // physical page, -1 when out of bounds
  int rows_cached;  // rows [0, rows_cached) come from the pool
  int append_here;  // row rows_cached is the new token
  int tile_len;
};

__device__ __forceinline__ TileInfo tile_info(const AttnArgs& a, const Cursor& c) {
  TileInfo t;
  const int page_abs = a.page0[c.b] + c.pg;
  const int pos = a.pos[c.b];
  const int start = page_abs * PAGE;
  t.rows_cached = min(max(pos - start, 0), PAGE);
  t.append_here = (a.append[c.b] && pos >= start && pos < start + PAGE) ? 1 : 0;
  const int pid = a.page_table[(int64_t)a.slots[c.b] * a.pt_stride + page_abs];
  t.page_id = (pid >= 0 && pid < a.max_pages) ? pid : -1;
  t.tile_len = (t.page_id >= 0) ? t.rows_cached + t.append_here : 0;
  return t;
}

__global__ void __launch_bounds__(THREADS, 1) attn_partial_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int u_begin = blockIdx.x * a.per;
  const int u_end = min(a.total, u_begin + a.per);
  if (u_begin >= u_end) return;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], N_CONSUMER);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == N_CONSUMER) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    Cursor c;
    c.seek(a, u_begin);
    for (int i = 0, u = u_begin; u < u_end; ++i, ++u, c.next(a)) {
      const int s = i % STAGES;
      if (i >= STAGES && !mbar_wait(&sm.empty[s], ((i / STAGES) - 1) & 1, a.err)) return;
      const TileInfo t = tile_info(a, c);
      if (t.page_id < 0) record_error(a.err, QC_ERR_BOUNDS);
      const uint32_t bytes = (t.page_id >= 0) ? uint32_t(t.rows_cached) * HD * 2 : 0u;
      mbar_arrive_expect_tx(&sm.full[s], 2 * bytes);
      if (bytes) {
        const int64_t off = ((int64_t)t.page_id * 4 + c.kvh) * PAGE * HD;
        bulk_g2s(sm.k[s], a.k_pool + off, bytes, &sm.full[s]);
        bulk_g2s(sm.v[s], a.v_pool + off, bytes, &sm.full[s]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  Cursor c;
  c.seek(a, u_begin);
  bool aborted = false;
  float q[4][8];
  float o[4][8];
  float m_run[4], l_run[4];
  int cur_b = -1, cur_kvh = -1;

  auto flush = [&]() {
    if (lane == 0) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        sm.red_ml[warp][h] = m_run[h];
        sm.red_ml[warp][4 + h] = l_run[h];
      }
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float4* dst = reinterpret_cast<float4*>(&sm.red_o[warp][h][lane * 8]);
      dst[0] = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
      dst[1] = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
    }
    consumer_sync();
    const int slot = cur_b * 4 + cur_kvh + blockIdx.x;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < N_CONSUMER; ++w) M = fmaxf(M, sm.red_ml[w][h]);
      float O = 0.0f, L = 0.0f;
#pragma unroll
      for (int w = 0; w < N_CONSUMER; ++w) {
        const float mw = sm.red_ml[w][h];
        const float f = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
        O = fmaf(f, sm.red_o[w][h][tid], O);
        L = fmaf(f, sm.red_ml[w][4 + h], L);
      }
      a.part_o[((int64_t)slot * 4 + h) * HD + tid] = O;
      if (tid == 0) {
        a.part_m[slot * 4 + h] = M;
        a.part_l[slot * 4 + h] = L;
      }
    }
    consumer_sync();
  };

  for (int i = 0, u = u_begin; u < u_end; ++i, ++u, c.next(a)) {
    const int s = i % STAGES;
    const TileInfo t = tile_info(a, c);
    if (c.b != cur_b || c.kvh != cur_kvh) {
      if (cur_b >= 0) flush();
      cur_b = c.b;
      cur_kvh = c.kvh;
      // ---- fused prologue: Q norm + RoPE; K norm + RoPE + append
      const int pos = a.pos[c.b];
      const float* cs = a.rope_cos + (int64_t)pos * 32;
      const float* sn = a.rope_sin + (int64_t)pos * 32;
      const uint16_t* prow = a.proj + (int64_t)c.b * 10240;
      if (warp < 4) {
        const int h = c.kvh * 4 + warp;
        float x[8];
        unpack8(*reinterpret_cast<const uint4*>(prow + h * 2 * HD + lane * 8), x);
        norm_rope_lane(x, a.q_norm, cs, sn, lane);
        float4* dst = reinterpret_cast<float4*>(&sm.q[warp][lane * 8]);
        dst[0] = make_float4(x[0], x[1], x[2], x[3]);
        dst[1] = make_float4(x[4], x[5], x[6], x[7]);
      }
      // does this CTA own the page of the new token for this pair?
      const int u_app = a.seg[c.b] + c.kvh * c.np + (c.np - 1);
      const bool own_append = a.append[c.b] && u_app < u_end;
      if (own_append && (warp == 4 || warp == 5)) {
        const int page_abs = a.page0[c.b] + c.np - 1;
        const int pid = a.page_table[(int64_t)a.slots[c.b] * a.pt_stride + page_abs];
        const bool in_bounds = pid >= 0 && pid < a.max_pages && pos >= page_abs * PAGE &&
                               pos < (page_abs + 1) * PAGE;
        const int64_t row_off =
            (((int64_t)pid * 4 + c.kvh) * PAGE + (pos - page_abs * PAGE)) * HD + lane * 8;
        if (warp == 4) {
          float x[8];
          unpack8(*reinterpret_cast<const uint4*>(prow + 8192 + c.kvh * HD + lane * 8), x);
          norm_rope_lane(x, a.k_norm, cs, sn, lane);
          uint4 w;
          w.x = uint32_t(f2bf(x[0])) | (uint32_t(f2bf(x[1])) << 16);
          w.y = uint32_t(f2bf(x[2])) | (uint32_t(f2bf(x[3])) << 16);
          w.z = uint32_t(f2bf(x[4])) | (uint32_t(f2bf(x[5])) << 16);
          w.w = uint32_t(f2bf(x[6])) | (uint32_t(f2bf(x[7])) << 16);
          *reinterpret_cast<uint4*>(&sm.knew[lane * 8]) = w;
          if (in_bounds) *reinterpret_cast<uint4*>(a.k_pool + row_off) = w;
        } else {
          const uint4 w = *reinterpret_cast<const uint4*>(prow + 9216 + c.kvh * HD + lane * 8);
          *reinterpret_cast<uint4*>(&sm.vnew[lane * 8]) = w;
          if (in_bounds) *reinterpret_cast<uint4*>(a.v_pool + row_off) = w;
        }
        if (!in_bounds && lane == 0) record_error(a.err, QC_ERR_BOUNDS);
      }
      consumer_sync();
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float4 q0 = *reinterpret_cast<const float4*>(&sm.q[h][lane * 8]);
        const float4 q1 = *reinterpret_cast<const float4*>(&sm.q[h][lane * 8 + 4]);
        q[h][0] = q0.x; q[h][1] = q0.y; q[h][2] = q0.z; q[h][3] = q0.w;
        q[h][4] = q1.x; q[h][5] = q1.y; q[h][6] = q1.z; q[h][7] = q1.w;
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[h][e] = 0.0f;
      }
    }

    if (!aborted && !mbar_wait(&sm.full[s], (i / STAGES) & 1, a.err)) aborted = true;
    if (aborted) continue;

    const int r0 = warp * 8;
    if (r0 < t.tile_len) {
      const uint16_t* kbase = sm.k[s];
      const uint16_t* vbase = sm.v[s];
      const int new_row = t.append_here ? t.rows_cached : -1;
      float acc[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int row = r0 + j;
        uint4 kw = make_uint4(0, 0, 0, 0);
        if (row < t.tile_len) {
          const uint16_t* kr = (row == new_row) ? sm.knew : kbase + row * HD;
          kw = *reinterpret_cast<const uint4*>(kr + lane * 8);
        }
        float kf[8];
        unpack8(kw, kf);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float d = q[h][0] * kf[0];
#pragma unroll
          for (int e = 1; e < 8; ++e) d = fmaf(q[h][e], kf[e], d);
          acc[j * 4 + h] = d;
        }
      }
      const float dot = transpose_reduce32(acc, lane);
      const int my_row = r0 + (lane >> 2);
      const float sc = (my_row < t.tile_len) ? dot * SCALE_LOG2 : -INFINITY;
      float mx = sc;
      mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, 16));
      float m_new[4], corr[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        m_new[h] = fmaxf(m_run[h], __shfl_sync(FULL_MASK, mx, h));
        corr[h] = (m_new[h] == -INFINITY) ? 1.0f : exp2f(m_run[h] - m_new[h]);
      }
      const int hl = lane & 3;
      const float my_m = hl == 0 ? m_new[0] : hl == 1 ? m_new[1] : hl == 2 ? m_new[2] : m_new[3];
      const float p = (sc == -INFINITY) ? 0.0f : exp2f(sc - my_m);
      float ps = p;
      ps += __shfl_xor_sync(FULL_MASK, ps, 4);
      ps += __shfl_xor_sync(FULL_MASK, ps, 8);
      ps += __shfl_xor_sync(FULL_MASK, ps, 16);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        l_run[h] = fmaf(l_run[h], corr[h], __shfl_sync(FULL_MASK, ps, h));
        m_run[h] = m_new[h];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[h][e] *= corr[h];
      }
      sm.p[warp][lane] = p;
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int row = r0 + j;
        if (row < t.tile_len) {
          const uint16_t* vr = (row == new_row) ? sm.vnew : vbase + row * HD;
          float vf[8];
          unpack8(*reinterpret_cast<const uint4*>(vr + lane * 8), vf);
          const float4 pj = *reinterpret_cast<const float4*>(&sm.p[warp][j * 4]);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            o[0][e] = fmaf(pj.x, vf[e], o[0][e]);
            o[1][e] = fmaf(pj.y, vf[e], o[1][e]);
            o[2][e] = fmaf(pj.z, vf[e], o[2][e]);
            o[3][e] = fmaf(pj.w, vf[e], o[3][e]);
          }
        }
      }
      __syncwarp();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }
  if (cur_b >= 0) flush();
}

__global__ void __launch_bounds__(256) attn_combine_kernel(const CombineArgs c) {
  const int pair = blockIdx.x;
  const int b = pair >> 2, kvh = pair & 3, t = threadIdx.x;
  const int np = (c.seg[b + 1] - c.seg[b]) >> 2;
  const int u0 = c.seg[b] + kvh * np;
  const int c0 = u0 / c.per, c1 = (u0 + np - 1) / c.per;
  const uint16_t* prow = c.proj + (int64_t)b * 10240;
#pragma unroll
  for (int hh = 0; hh < 4; ++hh) {
    float M = -INFINITY;
    for (int k = c0; k <= c1; ++k) M = fmaxf(M, c.part_m[(pair + k) * 4 + hh]);
    float O = 0.0f, L = 0.0f;
    for (int k = c0; k <= c1; ++k) {
      const int sl = pair + k;
      const float mk = c.part_m[sl * 4 + hh];
      const float f = (mk == -INFINITY) ? 0.0f : exp2f(mk - M);
      L = fmaf(f, c.part_l[sl * 4 + hh], L);
      O = fmaf(f, c.part_o[((int64_t)sl * 4 + hh) * HD + t], O);
    }
    const int h = kvh * 4 + hh;
    const float g = bf2f(prow[h * 2 * HD + HD + t]);
    c.out[(int64_t)b * 4096 + h * HD + t] = f2bf((O / L) * sigmoid_exact(g));
  }
}

}  // namespace

int attn_smem_bytes() { return static_cast<int>(sizeof(Smem)); }

cudaError_t launch_attn_decode(const AttnArgs& a, const CombineArgs& c, cudaStream_t s) {
  if (a.n <= 0 || a.total <= 0) return cudaSuccess;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(attn_partial_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn_smem_bytes());
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  attn_partial_kernel<<<a.grid, THREADS, attn_smem_bytes(), s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_combine_kernel<<<c.n * 4, 256, 0, s>>>(c);
  return cudaGetLastError();
}

}  // namespace qc
