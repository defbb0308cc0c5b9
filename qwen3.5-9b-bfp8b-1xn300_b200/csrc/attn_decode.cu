// attn_decode.cu — full-attention decode over the paged bf16 KV cache
// (src/engine.cpp:3485-3564).
//
// Kernel 1, attn_partial_kernel: one CTA per SM, each given an equal share of
// the batch's "page-heads" (one 64-token page of one kv-head: 32 KiB of K and
// 32 KiB of V) in (sequence, kv-head, page) order — a split-K over KV
// positions that balances the work exactly whatever the mix of context
// lengths.  Warp 8 is the producer: it streams each page-head into a 3-stage
// shared-memory ring with tiled TMA loads (cp.async.bulk.tensor, 64-row x
// 128-byte boxes: 8 copies per 64 KiB page-head; 128-byte swizzle so that
// the ldmatrix reads below are free of bank conflicts; each CTA loads only
// for itself).  A partial last page is loaded whole; its rows past the
// cached length are never read.  Warps 0-7 are consumers; each takes 8 of
// the 64 positions of a tile for the 4 query heads of the GQA group
// (kv_h = h / 4, src/engine.cpp:3532) and keeps its own online-softmax state.
//
// The dot products run on the tensor cores (mma.sync, bf16 in, fp32
// accumulate), operands straight from the swizzled tiles via ldmatrix:
//   S^T[8 pos x 8 col] = K[8 pos x 256] . Qx^T, where the 8 columns hold the 4
//     heads' q rounded to bf16 (hi) and the bf16 rounding residual (lo), so
//     S = S_hi + S_lo carries ~16 mantissa bits of q;
//   O^T[256 x 8 col] += V^T[256 x 8 pos] . Px^T with the same hi/lo split of
//     the softmax weights, transposed from the S accumulators by movmatrix.
// K and V are bf16 in the cache, so the products are exact and the result
// matches an fp32 computation to ~1e-5 relative.
//
// Fused prologue per (sequence, kv-head) pair: per-head RMSNorm + partial RoPE
// of the 4 query heads (src/engine.cpp:3497-3519) and, in the CTA that owns
// the page of the new position, the same for the new K plus the bf16 append of
// K and V into the page (src/engine.cpp:3521-3526); the new token is attended
// from shared memory, so no CTA reads a row another CTA is writing.
//
// Kernel 1b, attn_partial_tc_kernel (the launcher picks it when each CTA
// streams at most QC_ATTN_TC_MAX_PER page-heads): the same split and records
// with the products on the fifth-generation tensor cores — tcgen05.mma issued
// by one thread, accumulators in tensor memory, softmax in four warps that
// read the scores with tcgen05.ld.  The new token's K / V row is written into
// the landed tile in shared memory before the MMAs read it, and V rows past a
// tile's valid length are zeroed (0 * Inf would otherwise reach O).
//
// Kernel 2, attn_combine_kernel: per (sequence, kv-head) merges the partial
// records of the CTAs that covered it, divides by the softmax sum and applies
// the sigmoid output gate (src/engine.cpp:3560-3563), storing bf16.
#include <atomic>
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace qc {
namespace {

constexpr int HD = 256;
constexpr int PAGE = 64;
#ifndef QC_ATTN_STAGES
#define QC_ATTN_STAGES 3
#endif
constexpr int STAGES = QC_ATTN_STAGES;
constexpr int N_CONSUMER = 8;
constexpr int THREADS = (N_CONSUMER + 1) * 32;
constexpr int TILE_ELEMS = PAGE * HD;     // one K or V page-head, 32 KiB
constexpr int BOX_ROWS = KV_BOX_ROWS;     // TMA box: rows x 64 bf16 (128 B per row)
constexpr int BOX_BYTES = BOX_ROWS * 128;
// score * 1/16 (src/model_config.h:40), kept in the log2 domain for exp2
constexpr float SCALE_LOG2 = 0.0625f * 1.4426950408889634f;
constexpr float RESCALE_SLACK = 8.0f;      // log2 of the largest unnormalised weight

struct __align__(1024) Smem {
  uint16_t k[STAGES][TILE_ELEMS];   // swizzled: [col block 4][row 64][128 B]
  uint16_t v[STAGES][TILE_ELEMS];
  float red_o[4][4][HD];            // flush: 4 warps at a time
  float q[4][HD];
  float red_ml[N_CONSUMER][8];
  uint16_t knew[HD];
  uint16_t vnew[HD];
  uint16_t zero[HD];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(N_CONSUMER * 32) : "memory");
}

// Byte offset of (row, dim) inside a swizzled 64 x 256 bf16 tile: four
// 64-column blocks of 64 rows x 128 B; the 16-byte chunk index within a row is
// XORed with row % 8 (the TMA 128-byte swizzle).
__device__ __forceinline__ uint32_t swz(int row, int dim) {
  return (uint32_t)((dim >> 6) * (PAGE * 128) + row * 128 + ((((dim & 63) >> 3) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D += A[16x16] . B[16x8], bf16 in, f32 accumulate (rows 8..15 of A are zero)
__device__ __forceinline__ void mma_k16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
// D += A[16x8] . B[8x8]
__device__ __forceinline__ void mma_k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo_elem, float hi_elem) {
  return uint32_t(f2bf(lo_elem)) | (uint32_t(f2bf(hi_elem)) << 16);
}
// split x into bf16 hi + bf16 lo (x - hi), as bit patterns
__device__ __forceinline__ void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
  hi = f2bf(x);
  lo = f2bf(x - bf2f(hi));
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
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
    do {  // skip sequences with no pages in range
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

// Rows of the tile; with_page also resolves the physical page through the
// page table (the producer's job; consumers do not need it).
__device__ __forceinline__ TileInfo tile_info(const AttnArgs& a, const Cursor& c,
                                              bool with_page) {
  TileInfo t;
  const int page_abs = a.page0[c.b] + c.pg;
  const int pos = a.pos[c.b];
  const int start = page_abs * PAGE;
  t.rows_cached = min(max(pos - start, 0), PAGE);
  t.append_here = (a.append[c.b] && pos >= start && pos < start + PAGE) ? 1 : 0;
  t.page_id = 0;
  if (with_page) {
    const int pid = a.page_table[(int64_t)a.slots[c.b] * a.pt_stride + page_abs];
    t.page_id = (pid >= 0 && pid < a.max_pages) ? pid : -1;
  }
  t.tile_len = t.rows_cached + t.append_here;
  return t;
}

// tile_info without the page for a cursor whose sequence changes rarely: the
// sequence's descriptor entries are loaded when it changes, so a loop of
// single-thread roles over the tiles issues no global loads per tile.
struct SeqRows {
  int b = -1, pos = 0, page0 = 0, append = 0;
  __device__ __forceinline__ TileInfo at(const AttnArgs& a, const Cursor& c) {
    if (c.b != b) {
      b = c.b;
      pos = a.pos[b];
      page0 = a.page0[b];
      append = a.append[b];
    }
    TileInfo t;
    const int start = (page0 + c.pg) * PAGE;
    t.rows_cached = min(max(pos - start, 0), PAGE);
    t.append_here = (append && pos >= start && pos < start + PAGE) ? 1 : 0;
    t.page_id = 0;
    t.tile_len = t.rows_cached + t.append_here;
    return t;
  }
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// The tensor-core kernel runs when each CTA streams at most this many
// page-heads: it wins on short ranges (shorter ramp), while on long ones the
// per-tile chain of its single MMA-issuing thread and four softmax warps
// lets the eight mma.sync consumer warps stream slightly faster.  Measured
// (attention time per step, 4096-token contexts): 8 / 16 sequences (15 / 29
// page-heads per CTA) 8 / 4% faster on the tensor-core kernel, 32 sequences
// (57) and one 131072-token sequence (56) even, 64 sequences (113) 4% slower.
#ifndef QC_ATTN_TC_MAX_PER
#define QC_ATTN_TC_MAX_PER 60
#endif
#ifndef QC_ATTN_PDL
#define QC_ATTN_PDL 1
#endif

__global__ void __launch_bounds__(THREADS, 1)
    attn_partial_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Programmatic dependent launch: with a.early the step descriptor, the
  // page table and this layer's cached K/V cannot have been written by the
  // previous kernel on the stream (nothing of the open step writes them
  // before this layer's own call), so the producer streams K/V while that
  // kernel drains; the projection rows, the append and the records wait.
  if (!a.early) griddep_wait();
  const int total = a.split[0], per = a.split[1];
  const int u_begin = blockIdx.x * per;
  const int u_end = min(total, u_begin + per);
  if (u_begin >= u_end) {
    griddep_wait();  // every thread: the grid completes after its predecessor
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], N_CONSUMER);
    }
    fence_mbar_init();
  }
  if (tid < HD) sm.zero[tid] = 0;
  __syncthreads();

  if (warp == N_CONSUMER) {
    // ------------------------------------------------------------ producer
    // Lane j resolves the page of tile base + j (page-table reads for 32 tiles
    // in flight at once), lane 0 then waits for free stages and issues the
    // TMA loads in order.
    int i = 0;
    for (int base = u_begin; base < u_end; base += 32) {
      const int u = base + lane;
      int pid = -1, rows = 0, kvh = 0;
      if (u < u_end) {
        Cursor c;
        c.seek(a, u);
        const TileInfo t = tile_info(a, c, true);
        pid = t.page_id;
        rows = t.rows_cached;
        kvh = c.kvh;
      }
      const int cnt = min(32, u_end - base);
      for (int j = 0; j < cnt; ++j, ++i) {
        const int pj = __shfl_sync(FULL_MASK, pid, j);
        const int rj = __shfl_sync(FULL_MASK, rows, j);
        const int kj = __shfl_sync(FULL_MASK, kvh, j);
        int ok = 1;
        if (lane == 0) {
          const int s = i % STAGES;
          if (i >= STAGES && !mbar_wait(&sm.empty[s], ((i / STAGES) - 1) & 1, a.err)) ok = 0;
          if (ok) {
            if (pj < 0) record_error(a.err, QC_ERR_BOUNDS);
            const int nbox = (pj >= 0) ? (rj + BOX_ROWS - 1) / BOX_ROWS : 0;
            mbar_arrive_expect_tx(&sm.full[s], uint32_t(nbox * 4 * BOX_BYTES * 2));
            const int row0 = (pj * 4 + kj) * PAGE;
            for (int rb = 0; rb < nbox; ++rb)
#pragma unroll
              for (int cb = 0; cb < 4; ++cb) {
                const int off = (cb * PAGE * 128 + rb * BOX_BYTES) / 2;
                tma_load_2d(&sm.k[s][off], &tmk, cb * 64, row0 + rb * BOX_ROWS, &sm.full[s]);
                tma_load_2d(&sm.v[s][off], &tmv, cb * 64, row0 + rb * BOX_ROWS, &sm.full[s]);
              }
          }
        }
        if (!__shfl_sync(FULL_MASK, ok, 0)) {
          griddep_wait();
          return;
        }
      }
    }
    griddep_wait();
    return;
  }

  // -------------------------------------------------------------- consumers
  griddep_wait();
  griddep_launch();
  const int g = lane >> 2, t4 = lane & 3;
  Cursor c;
  c.seek(a, u_begin);
  bool aborted = false;
  uint32_t qb[16][2];     // B fragments of Qx^T per 16-dim step
  float oacc[16][4];      // O^T accumulators, m-tile mt = dims 16mt..16mt+15
  float m_run[2], l_run[2];
  int cur_b = -1, cur_kvh = -1;

  auto reset_state = [&]() {
#pragma unroll
    for (int mt = 0; mt < 16; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[mt][e] = 0.0f;
    m_run[0] = m_run[1] = -INFINITY;
    l_run[0] = l_run[1] = 0.0f;
  };

  auto flush = [&]() {
    // fold the lo columns into the hi columns: lanes t4 < 2 keep heads
    // 2*t4, 2*t4 + 1
#pragma unroll
    for (int mt = 0; mt < 16; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[mt][e] += __shfl_xor_sync(FULL_MASK, oacc[mt][e], 2);
#pragma unroll
    for (int m = 4; m <= 16; m <<= 1) {  // per-lane l -> the warp's l per head
      l_run[0] += __shfl_xor_sync(FULL_MASK, l_run[0], m);
      l_run[1] += __shfl_xor_sync(FULL_MASK, l_run[1], m);
    }
    if (lane < 2) {
      sm.red_ml[warp][2 * lane] = m_run[0];
      sm.red_ml[warp][2 * lane + 1] = m_run[1];
      sm.red_ml[warp][4 + 2 * lane] = l_run[0];
      sm.red_ml[warp][4 + 2 * lane + 1] = l_run[1];
    }
    consumer_sync();
    float M[4], L[4], acc[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      M[h] = -INFINITY;
#pragma unroll
      for (int w = 0; w < N_CONSUMER; ++w) M[h] = fmaxf(M[h], sm.red_ml[w][h]);
      L[h] = 0.0f;
#pragma unroll
      for (int w = 0; w < N_CONSUMER; ++w) {
        const float mw = sm.red_ml[w][h];
        if (mw != -INFINITY) L[h] = fmaf(exp2f(mw - M[h]), sm.red_ml[w][4 + h], L[h]);
      }
      acc[h] = 0.0f;
    }
    const int hA = 2 * (t4 & 1);
    const float MA = (t4 & 1) ? M[2] : M[0], MB = (t4 & 1) ? M[3] : M[1];
    const float fA = (m_run[0] == -INFINITY) ? 0.0f : exp2f(m_run[0] - MA);
    const float fB = (m_run[1] == -INFINITY) ? 0.0f : exp2f(m_run[1] - MB);
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
      if ((warp >> 2) == grp && t4 < 2) {
        float* roA = sm.red_o[warp & 3][hA];
        float* roB = sm.red_o[warp & 3][hA + 1];
#pragma unroll
        for (int mt = 0; mt < 16; ++mt) {
          const int d = 16 * mt + g;
          roA[d] = oacc[mt][0] * fA;
          roB[d] = oacc[mt][1] * fB;
          roA[d + 8] = oacc[mt][2] * fA;
          roB[d + 8] = oacc[mt][3] * fB;
        }
      }
      consumer_sync();
#pragma unroll
      for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int h = 0; h < 4; ++h) acc[h] += sm.red_o[w][h][tid];
      consumer_sync();
    }
    const int slot = cur_b * 4 + cur_kvh + blockIdx.x;
#pragma unroll
    for (int h = 0; h < 4; ++h) a.part_o[((int64_t)slot * 4 + h) * HD + tid] = acc[h];
    if (tid < 4) {
      a.part_m[slot * 4 + tid] = M[tid];
      a.part_l[slot * 4 + tid] = L[tid];
    }
  };

  for (int i = 0, u = u_begin; u < u_end; ++i, ++u, c.next(a)) {
    const int s = i % STAGES;
    const TileInfo t = tile_info(a, c, false);
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
          w.x = pack_bf16(x[0], x[1]);
          w.y = pack_bf16(x[2], x[3]);
          w.z = pack_bf16(x[4], x[5]);
          w.w = pack_bf16(x[6], x[7]);
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
      // B fragments of Qx^T: column g holds head g & 3, hi part for g < 4 and
      // lo part for g >= 4; k-step j covers dims 16j..16j+15
      {
        const int hq = g & 3;
        const bool lo_part = g >= 4;
#pragma unroll
        for (int j = 0; j < 16; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int d = 16 * j + 8 * e + 2 * t4;
            uint16_t h0, l0, h1, l1;
            split_bf16(sm.q[hq][d], h0, l0);
            split_bf16(sm.q[hq][d + 1], h1, l1);
            qb[j][e] = lo_part ? (uint32_t(l0) | (uint32_t(l1) << 16))
                               : (uint32_t(h0) | (uint32_t(h1) << 16));
          }
      }
      reset_state();
    }

    if (!aborted && !mbar_wait(&sm.full[s], (i / STAGES) & 1, a.err)) aborted = true;
    if (aborted) continue;

    const int r0 = warp * 8;
    if (r0 < t.tile_len) {
      // this lane's ldmatrix row: position r0 + (lane & 7), 8-dim chunk lane >> 3
      const int row = r0 + (lane & 7);
      const int mi = lane >> 3;
      const int new_row = t.append_here ? t.rows_cached : -1;
      const bool plain = (row == new_row) || (row >= t.tile_len);
      const uint32_t kb = (row == new_row) ? smem_u32(sm.knew)
                          : (row >= t.tile_len) ? smem_u32(sm.zero) : smem_u32(sm.k[s]);
      const uint32_t vb = (row == new_row) ? smem_u32(sm.vnew)
                          : (row >= t.tile_len) ? smem_u32(sm.zero) : smem_u32(sm.v[s]);
      // ---- S^T = K . Qx^T  (four accumulator chains)
      float sa[4][4] = {};
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int d = 32 * jj + 8 * mi;
        const uint32_t addr = kb + (plain ? uint32_t(d * 2) : swz(row, d));
        uint32_t m0, m1, m2, m3;
        ldsm_x4(addr, m0, m1, m2, m3);
        mma_k16(sa[(2 * jj) & 3], m0, m1, qb[2 * jj][0], qb[2 * jj][1]);
        mma_k16(sa[(2 * jj + 1) & 3], m2, m3, qb[2 * jj + 1][0], qb[2 * jj + 1][1]);
      }
      // lane (g, t4): position r0 + g, columns 2t4, 2t4 + 1 -> heads hA, hA + 1
      float s0 = (sa[0][0] + sa[1][0]) + (sa[2][0] + sa[3][0]);
      float s1 = (sa[0][1] + sa[1][1]) + (sa[2][1] + sa[3][1]);
      s0 += __shfl_xor_sync(FULL_MASK, s0, 2);  // hi + lo columns
      s1 += __shfl_xor_sync(FULL_MASK, s1, 2);
      const bool valid = (r0 + g) < t.tile_len;
      const float sc0 = valid ? s0 * SCALE_LOG2 : -INFINITY;
      const float sc1 = valid ? s1 * SCALE_LOG2 : -INFINITY;
      // Lazy reference maximum: it moves only when a score exceeds it by more
      // than 2^RESCALE_SLACK, so p <= 2^RESCALE_SLACK and most tiles need
      // neither the max reduction over the warp's positions nor the rescale
      // of the accumulators.  (m, l, o) stays consistent either way: o / l is
      // the same softmax average.
      bool up0 = sc0 > m_run[0] + RESCALE_SLACK, up1 = sc1 > m_run[1] + RESCALE_SLACK;
      const bool rescale = __any_sync(FULL_MASK, up0 || up1);
      float c0 = 1.0f, c1 = 1.0f;
      if (rescale) {
        float mx0 = sc0, mx1 = sc1;
#pragma unroll
        for (int m = 4; m <= 16; m <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(FULL_MASK, mx0, m));
          mx1 = fmaxf(mx1, __shfl_xor_sync(FULL_MASK, mx1, m));
        }
        up0 = mx0 > m_run[0] + RESCALE_SLACK;
        up1 = mx1 > m_run[1] + RESCALE_SLACK;
        if (up0) { c0 = exp2f(m_run[0] - mx0); m_run[0] = mx0; }
        if (up1) { c1 = exp2f(m_run[1] - mx1); m_run[1] = mx1; }
      }
      const float p0 = (sc0 == -INFINITY) ? 0.0f : exp2f(sc0 - m_run[0]);
      const float p1 = (sc1 == -INFINITY) ? 0.0f : exp2f(sc1 - m_run[1]);
      // l is kept per lane (this lane's positions) and summed over the warp
      // at the flush
      l_run[0] = fmaf(l_run[0], c0, p0);
      l_run[1] = fmaf(l_run[1], c1, p1);
      if (rescale) {
#pragma unroll
        for (int mt = 0; mt < 16; ++mt) {
          oacc[mt][0] *= c0;
          oacc[mt][1] *= c1;
          oacc[mt][2] *= c0;
          oacc[mt][3] *= c1;
        }
      }
      // ---- Px^T B fragment: matrix [pos g][col], col 2t4, 2t4+1 = hi (t4 < 2)
      // or lo (t4 >= 2) parts of p for heads hA, hA + 1; transpose with movmatrix
      uint16_t h0, l0, h1, l1;
      split_bf16(p0, h0, l0);
      split_bf16(p1, h1, l1);
      const uint32_t pm = (t4 < 2) ? (uint32_t(h0) | (uint32_t(h1) << 16))
                                   : (uint32_t(l0) | (uint32_t(l1) << 16));
      const uint32_t pb = movmatrix_t(pm);
      // ---- O^T += V^T . Px^T
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int d = 32 * jj + 8 * mi;
        const uint32_t addr = vb + (plain ? uint32_t(d * 2) : swz(row, d));
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(addr, v0, v1, v2, v3);
        mma_k8(oacc[2 * jj], v0, v1, pb);
        mma_k8(oacc[2 * jj + 1], v2, v3, pb);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }
  if (cur_b >= 0) flush();
}

// ---------------------------------------------------------------------------
// Tensor-core (tcgen05) variant of the partial kernel, for short ranges per
// CTA (QC_ATTN_TC_MAX_PER): the same split, tiles and records, with the dot
// products issued by one thread into tensor memory (TMEM):
//   S^T[64 pos x 16] = K[64 x 256] . Qx^T     (M 64, N 16, both K-major)
//   O[128 x 256]    += Px[128 x 64] . V       (M 128, N 256, V MN-major)
// Qx and Px have 8 distinct rows (rows 0-3: the bf16 value of the 4 heads'
// q / p, rows 4-7: the bf16 rounding residual); their descriptors use a zero
// stride between 8-row groups, so every further group repeats those 8 rows.
// S^T: position 16w + l sits in TMEM lane 32w + l (l < 16), its 16 columns
// the scores against the 8 rows twice (four accumulators, one per 64-dim
// block of the head, added after the load), so lane l of softmax warp w holds the
// 4 heads' scores of one position.  O: row r in lane r, repeated in every
// 32-lane quarter; warp w rescales and stores columns 64w..64w+63 of its own
// copy.  Warps 5 and 6 stream the K and V rings separately (a K slot frees
// when its scores are done, a V slot after P . V); the four softmax warps
// agree on the lazy reference maximum through shared memory once per tile.
constexpr int TC_THREADS = 7 * 32;            // warps 0-3 softmax, 4 MMA, 5 TMA K, 6 TMA V
constexpr int TC_MMA = 4, TC_TMA = 5;
constexpr uint32_t TC_TMEM_COLS = 512;        // S x 2 (64 each) + O (256)

struct __align__(1024) TcSmem {
  uint16_t k[STAGES][TILE_ELEMS];   // swizzled: [col block 4][row 64][128 B]
  uint16_t v[STAGES][TILE_ELEMS];
  uint16_t q[2][4 * 8 * 64];        // per pair parity: [col block 4][row 8][128 B]
  uint16_t p[2][8 * 64];            // per tile parity: [row 8][128 B]
  uint16_t knew[2][HD];             // per pair parity: the appended K / V row
  uint16_t vnew[2][HD];
  float s_mx[2][4][4];              // per tile parity: [warp][head] max over 16 positions
  float s_l[4][4];                  // [warp][head] softmax sums at a flush
  uint64_t full[STAGES], empty[STAGES];      // K ring
  uint64_t full_v[STAGES], empty_v[STAGES];  // V ring
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2], q_full[2], fix, xch[2], lx;
  uint32_t tmem_base;
  int abort;
  int k_seen;                       // K tiles the MMA thread has seen land (monotonic)
};

__device__ __forceinline__ bool tc_need_fix(const TileInfo& t) {
  return t.tile_len < PAGE || t.append_here;
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    attn_partial_tc_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ unsigned char smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                          ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (!a.early) griddep_wait();
  const int total = a.split[0], per = a.split[1];
  const int u_begin = blockIdx.x * per;
  const int u_end = min(total, u_begin + per);
  if (u_begin >= u_end) {
    griddep_wait();  // every thread: the grid completes after its predecessor
    return;
  }
  const int nt = u_end - u_begin;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
      mbar_init(&sm.full_v[s], 1);
      mbar_init(&sm.empty_v[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.s_free[b], 4);
      mbar_init(&sm.p_full[b], 4);
      mbar_init(&sm.o_done[b], 1);
      mbar_init(&sm.q_full[b], 4);
      mbar_init(&sm.xch[b], 128);
    }
    mbar_init(&sm.fix, 4);
    mbar_init(&sm.lx, 128);
    sm.abort = 0;
    sm.k_seen = 0;
    fence_mbar_init();
  }
  if (warp == TC_MMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_o = tmem + 128;
  volatile int* abort_flag = &sm.abort;

  if (warp >= TC_TMA) {
    // ------------------------------------------------------------ producers
    // warp 5 streams the K ring, warp 6 the V ring: a K slot is free again as
    // soon as its scores are computed, a V slot only after P . V
    const bool is_v = warp == TC_TMA + 1;
    uint64_t* fbar = is_v ? sm.full_v : sm.full;
    uint64_t* ebar = is_v ? sm.empty_v : sm.empty;
    const CUtensorMap* tmap = is_v ? &tmv : &tmk;
    int i = 0;
    int last_issued[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; ++s) last_issued[s] = -1;
    bool ok_all = true;
    for (int base = u_begin; base < u_end && ok_all; base += 32) {
      const int u = base + lane;
      int pid = -1, rows = 0, kvh = 0;
      if (u < u_end) {
        Cursor c;
        c.seek(a, u);
        const TileInfo t = tile_info(a, c, true);
        pid = t.page_id;
        rows = t.rows_cached;
        kvh = c.kvh;
      }
      const int cnt = min(32, u_end - base);
      for (int j = 0; j < cnt; ++j, ++i) {
        const int pj = __shfl_sync(FULL_MASK, pid, j);
        const int rj = __shfl_sync(FULL_MASK, rows, j);
        const int kj = __shfl_sync(FULL_MASK, kvh, j);
        int ok = 1;
        if (lane == 0) {
          const int s = i % STAGES;
          if (*abort_flag) ok = 0;
          if (ok && is_v && i < STAGES) {
            // ramp: the first V tiles go out only once their K tile has
            // landed, so the first scores do not share the HBM burst with them
            const uint64_t t0 = globaltimer();
            while (*reinterpret_cast<volatile int*>(&sm.k_seen) <= i && !*abort_flag)
              if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                record_error(a.err, QC_ERR_TIMEOUT);
                ok = 0;
                break;
              }
          }
          if (ok && i >= STAGES && !mbar_wait(&ebar[s], ((i / STAGES) - 1) & 1, a.err)) ok = 0;
          if (ok) {
            if (pj < 0 && !is_v) record_error(a.err, QC_ERR_BOUNDS);
            const int nbox = (pj >= 0) ? (rj + BOX_ROWS - 1) / BOX_ROWS : 0;
            mbar_arrive_expect_tx(&fbar[s], uint32_t(nbox * 4 * BOX_BYTES));
            const int row0 = (pj * 4 + kj) * PAGE;
            uint16_t* dst = is_v ? sm.v[s] : sm.k[s];
            for (int rb = 0; rb < nbox; ++rb)
#pragma unroll
              for (int cb = 0; cb < 4; ++cb)
                tma_load_2d(dst + (cb * PAGE * 128 + rb * BOX_BYTES) / 2, tmap, cb * 64,
                            row0 + rb * BOX_ROWS, &fbar[s]);
            last_issued[s] = i;
          } else {
            *abort_flag = 1;
          }
        }
        if (!__shfl_sync(FULL_MASK, ok, 0)) {
          ok_all = false;
          break;
        }
      }
    }
    // on abort, wait (bounded) for this CTA's own copies in flight
    if (lane == 0 && *abort_flag) {
#pragma unroll
      for (int s = 0; s < STAGES; ++s)
        if (last_issued[s] >= 0) mbar_wait(&fbar[s], (last_issued[s] / STAGES) & 1, nullptr);
    }
    griddep_wait();
  } else if (warp == TC_MMA) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // S = Qx . K^T: M 128, N 64, A and B K-major; O^T += V^T . Px^T: M 128
      // per half, N 16, A (V [pos][dim]) MN-major, B K-major; bf16 operands,
      // f32 accumulators
      const uint32_t id_s = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((64u >> 4) << 24);
      const uint32_t id_o = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((256u >> 3) << 17) |
                            ((128u >> 4) << 24);
      Cursor cq;
      cq.seek(a, u_begin);
      SeqRows rows_q;
      int pq = -1, qb = -1, qk = -1, fixcnt = 0;
      bool firstp[2] = {false, false};
      int issued_s = -1, issued_o = -1;
      auto issue_qk = [&](int i) -> bool {
        const TileInfo t = rows_q.at(a, cq);
        const bool first = cq.b != qb || cq.kvh != qk;
        if (first) { ++pq; qb = cq.b; qk = cq.kvh; }
        const int s = i % STAGES, b = i & 1;
        if (!mbar_wait(&sm.full[s], (i / STAGES) & 1, a.err)) return false;
        *reinterpret_cast<volatile int*>(&sm.k_seen) = i + 1;
        if (tc_need_fix(t)) {
          if (!mbar_wait(&sm.fix, fixcnt & 1, a.err)) return false;
          ++fixcnt;
        }
        if (first && !mbar_wait(&sm.q_full[pq & 1], (pq >> 1) & 1, a.err)) return false;
        if (i >= 2 && !mbar_wait(&sm.s_free[b], ((i >> 1) - 1) & 1, a.err)) return false;
        tc_fence_after();
        // the start address is the descriptor's low field (address / 16, below
        // 2^14 for any shared-memory address): steps along the tile are adds
        const uint64_t dk = umma_desc(smem_u32(sm.k[s]), 16, 1024);
        const uint64_t dq = umma_desc(smem_u32(sm.q[pq & 1]), 16, 0);
        // four accumulators (one per 64-dim column block, columns 16cb of
        // the buffer) so that consecutive MMAs do not wait on each other's
        // accumulator; the softmax warps add them
        const uint32_t ts = tmem + b * 64;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
          for (int cb = 0; cb < 4; ++cb)
            umma(ts + 16 * cb, dk + uint64_t((cb * PAGE * 128 + ks * 32) >> 4),
                 dq + uint64_t((cb * 1024 + ks * 32) >> 4), id_s, ks != 0);
        umma_commit(&sm.s_full[b]);
        umma_commit(&sm.empty[s]);  // the K slot
        issued_s = i;
        firstp[b] = first;
        cq.next(a);
        return true;
      };
      bool ok = issue_qk(0);
      for (int i = 0; i < nt && ok; ++i) {
        if (*abort_flag) { ok = false; break; }
        // the next tile's scores run while the softmax works on this one
        if (i + 1 < nt && !(ok = issue_qk(i + 1))) break;
        if (!(ok = mbar_wait(&sm.p_full[i & 1], (i >> 1) & 1, a.err))) break;
        const int s = i % STAGES;
        if (!(ok = mbar_wait(&sm.full_v[s], (i / STAGES) & 1, a.err))) break;
        tc_fence_after();
        const uint64_t dp = umma_desc(smem_u32(sm.p[i & 1]), 16, 0);
        const uint64_t dv = umma_desc(smem_u32(sm.v[s]), PAGE * 128, 1024);
        const uint32_t acc0 = firstp[i & 1] ? 0u : 1u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma(t_o, dp + uint64_t((kk * 32) >> 4), dv + uint64_t((kk * 2048) >> 4), id_o,
               kk > 0 ? 1u : acc0);
        umma_commit(&sm.o_done[i & 1]);
        umma_commit(&sm.empty_v[s]);
        issued_o = i;
      }
      if (!ok) {
        *abort_flag = 1;
        // wait (bounded) for the products in flight before the memory goes
        if (issued_s >= 0) mbar_wait(&sm.s_full[issued_s & 1], (issued_s >> 1) & 1, nullptr);
        if (issued_o >= 0) mbar_wait(&sm.o_done[issued_o & 1], (issued_o >> 1) & 1, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------- softmax warps
    griddep_wait();
    griddep_launch();
    const int r = lane & 7, hq = r & 3;          // S / O row of this lane, its head
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    Cursor c;
    c.seek(a, u_begin);
    // Q rows (value, residual) and the appended K / V row of pair X, into the
    // buffers of parity X & 1 (src/engine.cpp:3497-3526)
    auto prep = [&](const Cursor& pc, int x) {
      const int pos = a.pos[pc.b];
      const float* cs = a.rope_cos + (int64_t)pos * 32;
      const float* sn = a.rope_sin + (int64_t)pos * 32;
      const uint16_t* prow = a.proj + (int64_t)pc.b * 10240;
      {
        const int h = pc.kvh * 4 + warp;
        float xv[8];
        unpack8(*reinterpret_cast<const uint4*>(prow + h * 2 * HD + lane * 8), xv);
        norm_rope_lane(xv, a.q_norm, cs, sn, lane);
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint16_t h0, l0, h1, l1;
          split_bf16(xv[2 * e], h0, l0);
          split_bf16(xv[2 * e + 1], h1, l1);
          hi[e] = uint32_t(h0) | (uint32_t(h1) << 16);
          lo[e] = uint32_t(l0) | (uint32_t(l1) << 16);
        }
        unsigned char* qs = reinterpret_cast<unsigned char*>(sm.q[x & 1]);
        const int cb = lane >> 3, ch = lane & 7;
        *reinterpret_cast<uint4*>(qs + cb * 1024 + warp * 128 + ((ch ^ warp) << 4)) =
            make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(qs + cb * 1024 + (warp + 4) * 128 + ((ch ^ (warp + 4)) << 4)) =
            make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      const int u_app = a.seg[pc.b] + pc.kvh * pc.np + (pc.np - 1);
      if (a.append[pc.b] && u_app < u_end && warp < 2) {
        const int page_abs = a.page0[pc.b] + pc.np - 1;
        const int pid = a.page_table[(int64_t)a.slots[pc.b] * a.pt_stride + page_abs];
        const bool in_bounds = pid >= 0 && pid < a.max_pages && pos >= page_abs * PAGE &&
                               pos < (page_abs + 1) * PAGE;
        const int64_t row_off =
            (((int64_t)pid * 4 + pc.kvh) * PAGE + (pos - page_abs * PAGE)) * HD + lane * 8;
        if (warp == 0) {
          float xv[8];
          unpack8(*reinterpret_cast<const uint4*>(prow + 8192 + pc.kvh * HD + lane * 8), xv);
          norm_rope_lane(xv, a.k_norm, cs, sn, lane);
          uint4 w;
          w.x = pack_bf16(xv[0], xv[1]);
          w.y = pack_bf16(xv[2], xv[3]);
          w.z = pack_bf16(xv[4], xv[5]);
          w.w = pack_bf16(xv[6], xv[7]);
          *reinterpret_cast<uint4*>(&sm.knew[x & 1][lane * 8]) = w;
          if (in_bounds) *reinterpret_cast<uint4*>(a.k_pool + row_off) = w;
        } else {
          const uint4 w = *reinterpret_cast<const uint4*>(prow + 9216 + pc.kvh * HD + lane * 8);
          *reinterpret_cast<uint4*>(&sm.vnew[x & 1][lane * 8]) = w;
          if (in_bounds) *reinterpret_cast<uint4*>(a.v_pool + row_off) = w;
        }
        if (!in_bounds && lane == 0) record_error(a.err, QC_ERR_BOUNDS);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_full[x & 1]);
    };
    // the cursor of the pair after the one at `pc` (within this CTA's range)
    auto next_pair = [&](Cursor pc, int u_pc, int& u_next) -> Cursor {
      const int left = pc.np - pc.pg;  // units of this pair from pc on
      u_next = u_pc + left;
      Cursor n = pc;
      n.pg = pc.np - 1;
      n.next(a);
      return n;
    };
    // per head: reference maximum (the same in every lane) and this lane's
    // share of the softmax sum
    float m_h[4], l_h[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) { m_h[h] = -INFINITY; l_h[h] = 0.0f; }
    int cur_b = -1, cur_kvh = -1, px = -1, first_i = 0, lxcnt = 0;
    bool ok = true;
    auto flush = [&](int il) {
      // O complete for the pair's last tile
      if (!(ok = mbar_wait(&sm.o_done[il & 1], (il >> 1) & 1, a.err))) return;
      tc_fence_after();
      const int slot = cur_b * 4 + cur_kvh + blockIdx.x;
#pragma unroll 1
      for (int hc = 0; hc < 2; ++hc) {
        float ov[32];
        tmem_ld32(t_o + lane_off + 64 * warp + 32 * hc, ov);
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] += __shfl_xor_sync(FULL_MASK, ov[j], 4);  // value + residual rows
        if (lane < 4) {
          float* dst = a.part_o + ((int64_t)slot * 4 + lane) * HD + 64 * warp + 32 * hc;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(ov[j], ov[j + 1], ov[j + 2], ov[j + 3]);
        }
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float lsum = warp_sum(l_h[h]);
        if (lane == 0) sm.s_l[warp][h] = lsum;
      }
      mbar_arrive(&sm.lx);
      if (!(ok = mbar_wait(&sm.lx, lxcnt & 1, a.err))) return;
      ++lxcnt;
      if (warp == 0 && lane < 4) {
        a.part_m[slot * 4 + lane] = lane == 0 ? m_h[0] : lane == 1 ? m_h[1] : lane == 2 ? m_h[2] : m_h[3];
        a.part_l[slot * 4 + lane] =
            (sm.s_l[0][lane] + sm.s_l[1][lane]) + (sm.s_l[2][lane] + sm.s_l[3][lane]);
      }
      tc_fence_before();
    };
    SeqRows rows_c;
    prep(c, 0);
    for (int i = 0, u = u_begin; i < nt && ok; ++i, ++u, c.next(a)) {
      if (*abort_flag) { ok = false; break; }
      const int s = i % STAGES, b = i & 1;
      const TileInfo t = rows_c.at(a, c);
      const bool first = c.b != cur_b || c.kvh != cur_kvh;
      const int pxt = px + (first ? 1 : 0);
      if (tc_need_fix(t)) {
        // rows past the tile's valid length hold what an earlier sequence
        // left in a reused page (possibly not finite): P is zero there, but
        // 0 * Inf would still reach O, so those V rows are zeroed; the new
        // token's K / V row goes in at its position.  Then the MMA may read.
        if (!(ok = mbar_wait(&sm.full[s], (i / STAGES) & 1, a.err))) break;
        if (!(ok = mbar_wait(&sm.full_v[s], (i / STAGES) & 1, a.err))) break;
        unsigned char* ks = reinterpret_cast<unsigned char*>(sm.k[s]);
        unsigned char* vs = reinterpret_cast<unsigned char*>(sm.v[s]);
        const int zr0 = t.tile_len;
        for (int k = tid; k < (PAGE - zr0) * 32; k += 128) {
          const int row = zr0 + k / 32, d = (k % 32) * 8;
          *reinterpret_cast<uint4*>(vs + swz(row, d)) = make_uint4(0, 0, 0, 0);
        }
        if (t.append_here && warp < 2) {
          const int row = t.rows_cached;
          const uint16_t* src = warp == 0 ? sm.knew[pxt & 1] : sm.vnew[pxt & 1];
          *reinterpret_cast<uint4*>((warp == 0 ? ks : vs) + swz(row, lane * 8)) =
              *reinterpret_cast<const uint4*>(src + lane * 8);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.fix);
      }
      if (first) {
        if (cur_b >= 0) {
          flush(i - 1);
          if (!ok) break;
        }
        cur_b = c.b;
        cur_kvh = c.kvh;
        px = pxt;
        first_i = i;
#pragma unroll
        for (int h = 0; h < 4; ++h) { m_h[h] = -INFINITY; l_h[h] = 0.0f; }
        // the next pair's operands, one pair ahead of the MMA issuer
        int u_next;
        const Cursor nc = next_pair(c, u, u_next);
        if (u_next < u_end) prep(nc, px + 1);
      }
      // ---- S^T of positions 16w..16w+15: lane l < 16 holds position
      // 16w + l, columns 0-7 its scores against the q value (0-3) and
      // residual (4-7) rows of the 4 heads
      if (!(ok = mbar_wait(&sm.s_full[b], (i >> 1) & 1, a.err))) break;
      tc_fence_after();
      float sv[16];
      {
        float s01[32], s23[32];
        tmem_ld32(tmem + b * 64 + lane_off, s01);
        tmem_ld32(tmem + b * 64 + lane_off + 32, s23);
#pragma unroll
        for (int j = 0; j < 16; ++j) sv[j] = (s01[j] + s01[16 + j]) + (s23[j] + s23[16 + j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free[b]);
      const int jp = 16 * warp + lane;  // position in the tile
      const bool valid = lane < 16 && jp < t.tile_len;
      float sc[4], mloc[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        sc[h] = valid ? (sv[h] + sv[4 + h]) * SCALE_LOG2 : -INFINITY;
        mloc[h] = warp_max(sc[h]);
      }
      // ---- lazy reference maximum, agreed by the four warps: it moves only
      // when a score exceeds it by more than 2^RESCALE_SLACK
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < 4; ++h) sm.s_mx[b][warp][h] = mloc[h];
      }
      mbar_arrive(&sm.xch[b]);
      if (!(ok = mbar_wait(&sm.xch[b], (i >> 1) & 1, a.err))) break;
      float cf[4];
      bool any_up = false;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float mt = fmaxf(fmaxf(sm.s_mx[b][0][h], sm.s_mx[b][1][h]),
                               fmaxf(sm.s_mx[b][2][h], sm.s_mx[b][3][h]));
        cf[h] = 1.0f;
        if (mt > m_h[h] + RESCALE_SLACK) {
          cf[h] = (m_h[h] == -INFINITY) ? 0.0f : exp2f(m_h[h] - mt);
          m_h[h] = mt;
          any_up = true;
        }
        l_h[h] *= cf[h];
      }
      // P buffer b was read by P . V of tile i - 2
      if (i >= 2 && !(ok = mbar_wait(&sm.o_done[b], ((i - 2) >> 1) & 1, a.err))) break;
      if (any_up && i > first_i) {
        // O up to tile i - 1, this warp's columns, every row by its head's factor
        if (!(ok = mbar_wait(&sm.o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err))) break;
        tc_fence_after();
        const float cr = hq == 0 ? cf[0] : hq == 1 ? cf[1] : hq == 2 ? cf[2] : cf[3];
#pragma unroll 1
        for (int hc = 0; hc < 2; ++hc) {
          float ov[32];
          tmem_ld32(t_o + lane_off + 64 * warp + 32 * hc, ov);
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] *= cr;
          tmem_st32(t_o + lane_off + 64 * warp + 32 * hc, ov);
        }
      }
      // ---- P = 2^(s - m) as bf16 value (rows 0-3) and residual (rows 4-7),
      // column jp of the [8][64] tile
      if (lane < 16) {
        unsigned char* ps = reinterpret_cast<unsigned char*>(sm.p[b]) + (jp & 7) * 2;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float pv = (sc[h] == -INFINITY) ? 0.0f : exp2f(sc[h] - m_h[h]);
          l_h[h] += pv;
          uint16_t hi, lo;
          split_bf16(pv, hi, lo);
          *reinterpret_cast<uint16_t*>(ps + h * 128 + (((jp >> 3) ^ h) << 4)) = hi;
          *reinterpret_cast<uint16_t*>(ps + (h + 4) * 128 + (((jp >> 3) ^ (h + 4)) << 4)) = lo;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[b]);
    }
    if (ok && cur_b >= 0) flush(nt - 1);
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TC_MMA) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

// Writes head h's record (m, l, o[thread]) into slot [step & 1][layer][rank]
// of every rank's mailbox over NVLink (plain peer stores), then — once the
// CTA's stores are visible system-wide — adds 1 to counter [layer][rank] of
// every rank.  Every CTA of the record kernel does this for its head, so a
// rank's record for a step is complete when the counter reaches 16 per step.
__device__ __forceinline__ void publish_record(const CombineArgs& c, int h, float m, float l,
                                               float o) {
  const int t = threadIdx.x;
  const int par = (int)((c.done[c.layer] + 1u) & 1u);  // this step's mailbox half
  const int64_t off =
      ((((int64_t)par * c.n_layers + c.layer) * c.world + c.rank) * 16 + h) * (HD + 2);
  if (t < HD) {
    for (int r = 0; r < c.world; ++r) {
      float* rec = c.mbox_rec[r] + off;
      if (t == 0) { rec[0] = m; rec[1] = l; }
      rec[2 + t] = o;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (t < c.world) atomicAdd_system(c.mbox_cnt[t] + c.layer * c.world + c.rank, 1u);
}

// One CTA per (sequence, kv-head pair, head of the group); the slots of the
// CTAs that covered the pair (at most one per SM, plus one) are weighed in
// parallel first, so the per-dimension merge below is a chain of independent
// loads rather than a serial max/sum walk.  G groups of 256 threads split
// that chain (group g takes slots g, g + G, ...): with few sequences a pair
// has dozens of slots and the chain's L2 latency is the kernel's time.
template <int G>
__global__ void __launch_bounds__(256 * G) attn_combine_kernel(const CombineArgs c) {
  constexpr int NT = 256 * G, NW = NT / 32;
  constexpr int KO = 8;  // o slots per thread loaded with m and l, before the weights are known
  static_assert(NT >= 256, "one slot per thread: a pair has at most one slot per CTA, plus one");
  __shared__ float s_w[512];
  __shared__ float s_rm[NW], s_rl[NW];
  __shared__ float s_o[G > 1 ? G - 1 : 1][HD];
  const int pair = blockIdx.x, hh = blockIdx.y;
  const int b = pair >> 2, kvh = pair & 3, t = threadIdx.x;
  const int h = kvh * 4 + hh;
  // Loads of what no kernel of the open step writes (the descriptor) or what
  // was complete when this grid was launched (the projection rows: the
  // partial kernel triggers its dependents only after its own wait on them)
  // go before the wait for the partial records.
  const int seg0 = c.seg[b], seg1 = c.seg[b + 1], per = c.split[1];
  const bool gated = c.world == 0 && c.record == nullptr;
  const float gt = (gated && t < HD) ? bf2f(c.proj[(int64_t)b * 10240 + h * 2 * HD + HD + t]) : 0.0f;
  griddep_wait();  // the partial records of the kernel before
  griddep_launch();
  const int np = (seg1 - seg0) >> 2;
  const int u0 = seg0 + kvh * np;
  if (np == 0) {  // empty page range (split over devices): an empty record
    if (c.world > 0) {
      publish_record(c, h, -INFINITY, 0.0f, 0.0f);
      return;
    }
    float* rec = c.record + h * (HD + 2);
    if (t == 0) { rec[0] = -INFINITY; rec[1] = 0.0f; }
    if (t < HD) rec[2 + t] = 0.0f;
    return;
  }
  const int c0 = u0 / per, ns = (u0 + np - 1) / per - c0 + 1;
  const int base = pair + c0;
  const int d = t & (HD - 1), g = t / HD;
  // every record load at once: m and l of slot t, o of this group's first
  // KO slots
  const float mk = t < ns ? c.part_m[(base + t) * 4 + hh] : -INFINITY;
  const float lk = t < ns ? c.part_l[(base + t) * 4 + hh] : 0.0f;
  const float* po = c.part_o + ((int64_t)base * 4 + hh) * HD + d;
  float ov[KO];
#pragma unroll
  for (int j = 0; j < KO; ++j) {
    const int k = g + j * G;
    ov[j] = k < ns ? po[(int64_t)k * 4 * HD] : 0.0f;
  }
  // max over the slots, then the slot weights and the softmax sum
  const float mw = warp_max(mk);
  if ((t & 31) == 0) s_rm[t >> 5] = mw;
  __syncthreads();
  float M = s_rm[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) M = fmaxf(M, s_rm[w]);
  const float f = (mk == -INFINITY) ? 0.0f : exp2f(mk - M);
  if (t < ns) s_w[t] = f;
  const float lw = warp_sum(f * lk);
  if ((t & 31) == 0) s_rl[t >> 5] = lw;
  __syncthreads();
  float L = 0.0f;
#pragma unroll
  for (int w = 0; w < NW; ++w) L += s_rl[w];
  float O = 0.0f;
#pragma unroll
  for (int j = 0; j < KO; ++j) {
    const int k = g + j * G;
    if (k < ns) O = fmaf(s_w[k], ov[j], O);
  }
#pragma unroll 8
  for (int k = g + KO * G; k < ns; k += G) O = fmaf(s_w[k], po[(int64_t)k * 4 * HD], O);
  if constexpr (G > 1) {
    if (g > 0) s_o[g - 1][d] = O;
    __syncthreads();
    if (g == 0) {
#pragma unroll
      for (int j = 0; j < G - 1; ++j) O += s_o[j][d];
    }
  }
  if (c.world > 0) {  // partial of a split over devices, sent to every rank
    publish_record(c, h, M, L, O);
    return;
  }
  if (t >= HD) return;
  if (c.record) {  // partial of a split over devices: keep it unnormalised
    float* rec = c.record + h * (HD + 2);
    if (t == 0) { rec[0] = M; rec[1] = L; }
    rec[2 + t] = O;
    return;
  }
  c.out[(int64_t)b * 4096 + h * HD + t] = f2bf((O / L) * gate_sigmoid(gt, c.ref_math));
}

// Cross-device merge: one CTA per head, thread = dimension.
__global__ void __launch_bounds__(256) attn_merge_records_kernel(const float* rec, int n_parts,
                                                                 const uint16_t* proj,
                                                                 uint16_t* out, int ref_math) {
  const int h = blockIdx.x, t = threadIdx.x;
  float M = -INFINITY;
  for (int g = 0; g < n_parts; ++g) M = fmaxf(M, rec[(g * 16 + h) * (HD + 2)]);
  float L = 0.0f, O = 0.0f;
  for (int g = 0; g < n_parts; ++g) {
    const float* r = rec + (g * 16 + h) * (HD + 2);
    const float f = (r[0] == -INFINITY) ? 0.0f : exp2f(r[0] - M);
    L = fmaf(f, r[1], L);
    O = fmaf(f, r[2 + t], O);
  }
  const float gt = bf2f(proj[h * 2 * HD + HD + t]);
  out[h * HD + t] = f2bf((O / L) * gate_sigmoid(gt, ref_math));
}

// The cross-device merge from this rank's mailbox.  The step is done[layer] + 1
// (this rank's merges so far, counted on the device, so captured and replayed
// calls number their steps the same way as direct ones).  Thread 0 waits until
// the counters of all ranks for this layer reach 16 * step (polling with
// acquire loads, bounded by WAIT_LIMIT_NS: on expiry the error word gets
// QC_ERR_TIMEOUT and the CTA returns without output), then the CTA merges
// the records, read through L2 (they were written by other GPUs).
__global__ void __launch_bounds__(256) attn_merge_mailbox_kernel(const MailboxMergeArgs m) {
  __shared__ int ok;
  const int h = blockIdx.x, t = threadIdx.x;
  // the next kernel may be scheduled now (its griddepcontrol.wait still waits
  // for this grid to complete); this grid was scheduled while the record
  // kernel ran and waits on the counters, not on the stream
  griddep_launch();
  // the gate half of the projection row was complete before the record
  // kernel triggered this launch: load it while the records travel
  const float gt = bf2f(m.proj[h * 2 * HD + HD + t]);
  if (t == 0) ok = 1;
  const uint32_t step = m.done[m.layer] + 1u;
  if (t == 0) {
    // a merge that gave up earlier left the step counts of the ranks apart:
    // every later merge refuses (no output) until qc_p2p_reset clears this
    if (*reinterpret_cast<volatile uint32_t*>(m.poison)) {
      record_error(m.err, QC_ERR_TIMEOUT);
      ok = 0;
    }
  }
  __syncthreads();
  if (t == 0 && ok != 0) {
    const uint32_t target = 16u * step;
    const uint32_t* cnt = m.cnt + m.layer * m.world;
    const uint64_t t0 = globaltimer();
    int done = 0;
    for (uint32_t it = 0;; ++it) {
      done = 1;
      for (int r = 0; r < m.world; ++r) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt + r) : "memory");
        if ((int32_t)(v - target) < 0) { done = 0; break; }
      }
      if (done) break;
      if ((it & 63u) == 0 && globaltimer() - t0 > WAIT_LIMIT_NS) {
        record_error(m.err, QC_ERR_TIMEOUT);
        atomicExch(m.poison, 1u);
        break;
      }
    }
    ok = done;
  }
  __syncthreads();
  if (!ok) return;
  const float* rec = m.rec + ((int64_t)(step & 1u) * m.n_layers + m.layer) * m.world * 16 * (HD + 2);
  float M = -INFINITY;
  for (int g = 0; g < m.world; ++g) M = fmaxf(M, __ldcg(rec + (g * 16 + h) * (HD + 2)));
  float L = 0.0f, O = 0.0f;
  for (int g = 0; g < m.world; ++g) {
    const float* r = rec + (g * 16 + h) * (HD + 2);
    const float mg = __ldcg(r);
    const float f = (mg == -INFINITY) ? 0.0f : exp2f(mg - M);
    L = fmaf(f, __ldcg(r + 1), L);
    O = fmaf(f, __ldcg(r + 2 + t), O);
  }
  m.out[h * HD + t] = f2bf((O / L) * gate_sigmoid(gt, m.ref_math));
  __syncthreads();
  // every CTA read done[layer] at its start; the 16th to get here advances it
  if (t == 0 && atomicAdd(m.consumed + m.layer, 1u) % 16u == 15u) atomicAdd(m.done + m.layer, 1u);
}

}  // namespace

cudaError_t launch_attn_merge_mailbox(const MailboxMergeArgs& m, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = QC_ATTN_PDL;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(16, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_merge_mailbox_kernel, m);
}

cudaError_t launch_attn_merge_records(const float* records, int32_t n_parts, const uint16_t* proj,
                                      uint16_t* out, int ref_math, cudaStream_t s) {
  attn_merge_records_kernel<<<16, 256, 0, s>>>(records, n_parts, proj, out, ref_math);
  return cudaGetLastError();
}

int attn_smem_bytes() {
  return static_cast<int>(sizeof(Smem) > sizeof(TcSmem) ? sizeof(Smem) : sizeof(TcSmem)) + 1024;
}

namespace {
std::atomic<int> g_attn_mode{QC_ATTN_KERNEL_AUTO};
}  // namespace

cudaError_t launch_attn_decode(const AttnArgs& a, const CombineArgs& c, const CUtensorMap& tmk,
                               const CUtensorMap& tmv, cudaStream_t s) {
  if (a.n <= 0) return cudaSuccess;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(attn_partial_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn_smem_bytes());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attn_partial_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             attn_smem_bytes());
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = QC_ATTN_PDL;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.grid, 1, 1);
  const int mode = g_attn_mode.load(std::memory_order_relaxed);
  const bool tc = mode == QC_ATTN_KERNEL_TC ||
                  (mode == QC_ATTN_KERNEL_AUTO && a.per_hint > 0 && a.per_hint <= QC_ATTN_TC_MAX_PER);
  cfg.blockDim = dim3(tc ? TC_THREADS : THREADS, 1, 1);
  cfg.dynamicSmemBytes = attn_smem_bytes();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e =
      cudaLaunchKernelEx(&cfg, tc ? attn_partial_tc_kernel : attn_partial_kernel, a, tmk, tmv);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cc = {};
  cc.gridDim = dim3(c.n * 4, 4, 1);
  cc.stream = s;
  cc.attrs = attr;
  cc.numAttrs = 1;
  // few sequences: many slots per pair, split the merge chain four ways
  if (c.n <= 2) {
    cc.blockDim = dim3(1024, 1, 1);
    return cudaLaunchKernelEx(&cc, attn_combine_kernel<4>, c);
  }
  cc.blockDim = dim3(256, 1, 1);
  return cudaLaunchKernelEx(&cc, attn_combine_kernel<1>, c);
}

}  // namespace qc

extern "C" int qc_attn_select_kernel(int mode) {
  if (mode != QC_ATTN_KERNEL_AUTO && mode != QC_ATTN_KERNEL_MMA && mode != QC_ATTN_KERNEL_TC)
    return -QC_ERR_ARG;
  return qc::g_attn_mode.exchange(mode);
}
