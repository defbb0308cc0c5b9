// bfp8.cu — BFP8_B tiled weights on sm_100a: the on-device packer and the
// split-K GEMV that streams the packed tiles (src/engine.cpp:371-727 on the
// reference's Tenstorrent cores).
//
// GEMV design.  The weights are the only large operand (1.0625 bytes per
// weight), so the kernel is an HBM stream.  Work is cut into units: one
// tile-row (32 output rows) times a run of `ku` consecutive k-tiles, a
// contiguous byte range of the packed matrix.  Every warp is an independent
// pipeline over its own units (u = global warp, += all warps): lane 0 keeps
// three stages of four tiles in flight with bulk copies (cp.async.bulk) into the
// warp's own shared-memory ring, and the warp dequantises in registers
// straight into mma.sync A fragments:
//   - a face (16x16) of a tile is exactly one m16 x k16 A operand;
//   - the MMA's k order is permuted so that lane (g, t) owns bytes 4t..4t+3
//     of face rows g and g + 8: one 32-bit shared load per row, conflict free;
//     the activations take the same permutation (one 8-byte load per lane);
//   - byte -> bf16: the bf16 with high byte sign|0x43 and low byte m is
//     +-(128 + m) exactly; one bf16x2 subtraction of +-128 leaves +-m.  Two
//     logic ops and four byte permutes serve four elements;
//   - each face row's shared exponent scales that face's MMA result (a
//     fresh f32 accumulator of 16 products) by 2^(e-127) into the running
//     sum; the decode rule's remaining 2^-6 is applied once per output.  Both
//     factors are powers of two, so the scaling itself rounds nothing: the
//     result is an f32 sum of the exactly decoded products (face rows whose
//     shared exponent is 0, i.e. zeros and bf16 subnormals, contribute 0).
// A warp ends a unit by writing its partial sums (or, without a k split, the
// outputs); a small merge kernel adds the partials in k order and writes the
// bf16 outputs, so the result does not depend on timing.  No CTA-wide
// barrier: warps of one CTA never wait for each other.  Both kernels are
// launched with programmatic dependent launch: a GEMV starts streaming its
// weights while the kernels before it drain, and waits (griddepcontrol.wait)
// only before it reads activations or writes outputs and scratch.

#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "../../include/qbfp8.h"
#include "common.cuh"
#include "kernels.h"

namespace qc {
namespace {

constexpr int TB = QC_BFP8_TILE_BYTES;  // 1088
constexpr int TPS = 4;                  // tiles per stage (one 4352-byte bulk copy)
constexpr int NSTW = 3;                 // stages per warp
constexpr int NWARP = 8;                // warps per CTA, each an independent pipeline
constexpr int GEMV_THREADS = NWARP * 32;
constexpr int NMAX = 16;                // batch columns per launch (two n8 MMA tiles)
constexpr int MERGE_BATCH = 8;          // split-K partials loaded at once per output

struct GemvSmem {
  uint8_t stage[NWARP][NSTW][TPS * TB];  // TPS * TB = 4352, a multiple of 16
  uint64_t full[NWARP][NSTW];
};

// Four sign/magnitude bytes of one face row -> their signed magnitudes +-m
// as two bf16x2 words (elements 0,1 and 2,3).  With the high byte s|0x43 and
// the low byte m, a bf16 is +-(128 + m) exactly; subtracting +-128 leaves +-m.
__device__ __forceinline__ void mags4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t mm = w & 0x7f7f7f7fu;
  const uint32_t hh = (w & 0x80808080u) | 0x43434343u;
  const uint32_t v_lo = __byte_perm(mm, hh, 0x5140);
  const uint32_t v_hi = __byte_perm(mm, hh, 0x7362);
  const uint32_t s_lo = __byte_perm(0u, hh, 0x5140);
  const uint32_t s_hi = __byte_perm(0u, hh, 0x7362);
  __nv_bfloat162 a, b;
  std::memcpy(&a, &v_lo, 4);
  std::memcpy(&b, &s_lo, 4);
  const __nv_bfloat162 r_lo = __hsub2(a, b);
  std::memcpy(&a, &v_hi, 4);
  std::memcpy(&b, &s_hi, 4);
  const __nv_bfloat162 r_hi = __hsub2(a, b);
  std::memcpy(&lo, &r_lo, 4);
  std::memcpy(&hi, &r_hi, 4);
}

// d = A.B (fresh accumulator), bf16 operands
__device__ __forceinline__ void mma_bf16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

__device__ __forceinline__ uint16_t bf_trunc(float f) { return uint16_t(__float_as_uint(f) >> 16); }

__device__ __forceinline__ void store_out(const Bfp8GemvArgs& a, int m, int b, float v) {
  uint16_t* p = (m < a.split) ? a.y0 + (int64_t)b * a.ld0 + m
                              : a.y1 + (int64_t)b * a.ld1 + (m - a.split);
  if (a.mode == 1)
    *p = bf_trunc(bf2f(f2bf(v)) + bf2f(*p));
  else
    *p = f2bf(v);
}

// A warp's position in its sequence of units (u = first, += W): unit u is
// k-chunk s = u / Mt of tile-row mt = u % Mt, the ku tiles from k-tile s*ku
// (contiguous bytes).  s and mt advance by addition (W = Wq * Mt + Wr).
struct UnitCursor {
  int u, s, mt, nt;
  __device__ __forceinline__ void init(const Bfp8GemvArgs& a, int u0) {
    u = u0;
    s = u0 / a.Mt;
    mt = u0 - s * a.Mt;
    nt = min(a.ku, a.Kt - s * a.ku);
  }
  __device__ __forceinline__ void next(const Bfp8GemvArgs& a, int W, int Wq, int Wr) {
    u += W;
    s += Wq;
    mt += Wr;
    if (mt >= a.Mt) { mt -= a.Mt; ++s; }
    nt = min(a.ku, a.Kt - s * a.ku);
  }
};

// One tile of the device layout times the activation fragments b (per n8
// column group q: k 4t..4t+3 and 16+4t..16+4t+3 of the tile), accumulated
// into acc[row block][q][4].
template <int NT>
__device__ __forceinline__ void tile_mma(const uint8_t* tile, int g, int lane,
                                         const uint32_t (&b)[NT][4], float (&acc)[2][NT][4]) {
  // this lane's 8 shared exponents and 8 words of mantissa bytes
  const uint2 ex = *reinterpret_cast<const uint2*>(tile + g * 8);
  const uint4 wa = *reinterpret_cast<const uint4*>(tile + 64 + lane * 16);
  const uint4 wb = *reinterpret_cast<const uint4*>(tile + 64 + 512 + lane * 16);
  const uint32_t wr[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int f = 0; f < 4; ++f) {
    // 2^(e - 127) per face row; the remaining 2^-6 of the decode rule is
    // applied once per output (exact: powers of two)
    const uint32_t ew = f < 2 ? ex.x : ex.y;
    const float sc0 = __uint_as_float(__byte_perm(ew, 0u, 0x4440 + (f & 1) * 2) << 23);
    const float sc1 = __uint_as_float(__byte_perm(ew, 0u, 0x4441 + (f & 1) * 2) << 23);
    uint32_t a0, a1, a2, a3;
    mags4(wr[2 * f], a0, a2);
    mags4(wr[2 * f + 1], a1, a3);
#pragma unroll
    for (int q = 0; q < NT; ++q) {
      float d[4];
      mma_bf16_z(d, a0, a1, a2, a3, b[q][(f & 1) * 2], b[q][(f & 1) * 2 + 1]);
      float(&c)[4] = acc[f >> 1][q];
      c[0] = fmaf(sc0, d[0], c[0]);
      c[1] = fmaf(sc0, d[1], c[1]);
      c[2] = fmaf(sc1, d[2], c[2]);
      c[3] = fmaf(sc1, d[3], c[3]);
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(GEMV_THREADS, 2) bfp8_gemv_kernel(const Bfp8GemvArgs a) {
  extern __shared__ __align__(128) unsigned char raw[];
  GemvSmem& sm = *reinterpret_cast<GemvSmem*>(raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = gridDim.x * NWARP, gw = blockIdx.x * NWARP + warp;
  const int Wq = W / a.Mt, Wr = W - Wq * a.Mt;
  uint64_t* full = sm.full[warp];
  if (lane == 0) {
    for (int i = 0; i < NSTW; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // copy cursor: the unit and first tile of the next stage to load
  UnitCursor fu;
  fu.init(a, gw);
  int fc0 = 0;
  auto issue = [&](int st) {  // loads the cursor's stage into slot st and advances
    if (lane == 0) {
      const int n = min(TPS, fu.nt - fc0);
      const uint8_t* src = a.w + ((int64_t)fu.mt * a.Kt + fu.s * a.ku + fc0) * TB;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&full[st], n * TB);
      bulk_g2s(sm.stage[warp][st], src, n * TB, &full[st]);
    }
    fc0 += TPS;
    if (fc0 >= fu.nt) {
      fu.next(a, W, Wq, Wr);
      fc0 = 0;
    }
  };

  const int g = lane >> 2, t = lane & 3;
  // activation fragments (bf16) of tiles kt_first .. kt_first + n - 1:
  // per tile and column group, k 4t..4t+3 and 16+4t..16+4t+3
  auto load_b = [&](uint32_t (&b)[TPS][NT][4], int kt_first, int n) {
#pragma unroll
    for (int j = 0; j < TPS; ++j)
#pragma unroll
      for (int q = 0; q < NT; ++q) {
        const int col = q * 8 + g;
        uint2 v0 = make_uint2(0u, 0u), v1 = make_uint2(0u, 0u);
        if (j < n && col < a.batch) {
          const uint16_t* xp = a.x + (int64_t)col * a.K + (kt_first + j) * 32 + 4 * t;
          v0 = __ldg(reinterpret_cast<const uint2*>(xp));
          v1 = __ldg(reinterpret_cast<const uint2*>(xp + 16));
        }
        b[j][q][0] = v0.x;
        b[j][q][1] = v0.y;
        b[j][q][2] = v1.x;
        b[j][q][3] = v1.y;
      }
  };

  // The next kernel on the stream may start as soon as SMs free up; it only
  // streams its own (read-only) weights until its griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int i = 0; i < NSTW && fu.u < a.n_units; ++i) issue(i);
  // Everything below reads the activations or writes outputs and scratch:
  // wait until the previous kernel on the stream has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  int st = 0;
  uint32_t ph = 0;
  bool ok = true;
  UnitCursor cu;
  cu.init(a, gw);
  for (; cu.u < a.n_units; cu.next(a, W, Wq, Wr)) {
    const int s = cu.s, mt = cu.mt, kt0 = s * a.ku, nt = cu.nt;
    float acc[2][NT][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int q = 0; q < NT; ++q) acc[i][q][0] = acc[i][q][1] = acc[i][q][2] = acc[i][q][3] = 0.0f;

    // one stage: wait, TPS tiles (or the unit's last n), release by loading
    // the next stage of the warp's sequence into the same slot
    auto stage = [&](const uint32_t (&b)[TPS][NT][4], int n) {
      if (!mbar_wait(&full[st], ph, a.err)) { ok = false; return; }
      const uint8_t* base = sm.stage[warp][st];
      if (n == TPS) {
#pragma unroll
        for (int j = 0; j < TPS; ++j) tile_mma<NT>(base + j * TB, g, lane, b[j], acc);
      } else {
#pragma unroll
        for (int j = 0; j < TPS - 1; ++j)
          if (j < n) tile_mma<NT>(base + j * TB, g, lane, b[j], acc);
      }
      __syncwarp();
      if (fu.u < a.n_units) issue(st);
      if (++st == NSTW) { st = 0; ph ^= 1u; }
    };
    // activation fragments ping-pong between two register sets: the next
    // stage's are loaded while the current stage is computed
    uint32_t bA[TPS][NT][4], bB[TPS][NT][4];
    load_b(bA, kt0, min(TPS, nt));
    for (int c0 = 0; c0 < nt; c0 += 2 * TPS) {
      if (c0 + TPS < nt) load_b(bB, kt0 + c0 + TPS, min(TPS, nt - c0 - TPS));
      stage(bA, min(TPS, nt - c0));
      if (!ok) return;
      if (c0 + TPS >= nt) break;
      if (c0 + 2 * TPS < nt) load_b(bA, kt0 + c0 + 2 * TPS, min(TPS, nt - c0 - 2 * TPS));
      stage(bB, min(TPS, nt - c0 - TPS));
      if (!ok) return;
    }

    // ---- unit epilogue: lane (g, t) holds rows g, g+8, g+16, g+24 of the
    // tile-row for columns q*8 + 2t, q*8 + 2t + 1
#pragma unroll
    for (int rb = 0; rb < 2; ++rb)
#pragma unroll
      for (int q = 0; q < NT; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e)  // 2^-6 of the decode rule
          acc[rb][q][e] *= 0.015625f;
#pragma unroll
    for (int rb = 0; rb < 2; ++rb)
#pragma unroll
      for (int q = 0; q < NT; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = rb * 16 + g + (e >> 1) * 8, c = q * 8 + 2 * t + (e & 1);
          if (c >= a.batch) continue;
          if (a.S == 1)
            store_out(a, mt * 32 + r, c, acc[rb][q][e]);
          else
            a.partial[((int64_t)s * NMAX + c) * a.M + mt * 32 + r] = acc[rb][q][e];
        }
  }
}

// Split-K merge: one thread per output, the S partials added in k order
// (the same order on every call).  Launched after the GEMV with programmatic
// serialization: it lets the next kernel start at once and waits for the
// GEMV to complete before reading the partials.
__global__ void __launch_bounds__(256) bfp8_merge_kernel(const Bfp8GemvArgs a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= (int64_t)a.batch * a.M) return;
  const int c = (int)(i / a.M), m = (int)(i - (int64_t)c * a.M);
  const float* src = a.partial + (int64_t)c * a.M + m;
  const int64_t step = (int64_t)NMAX * a.M;
  float sum = 0.0f;
  for (int k0 = 0; k0 < a.S; k0 += MERGE_BATCH) {
    float v[MERGE_BATCH];
#pragma unroll
    for (int k = 0; k < MERGE_BATCH; ++k) v[k] = (k0 + k < a.S) ? __ldcg(src + (k0 + k) * step) : 0.0f;
#pragma unroll
    for (int k = 0; k < MERGE_BATCH; ++k)
      if (k0 + k < a.S) sum += v[k];
  }
  store_out(a, m, c, sum);
}

// Device layout of a tile (the same 1088 bytes, permuted), built on upload
// from the GGUF layout and undone on download.  For MMA lane l = 4g + t:
//   bytes [g*8, g*8 + 8): shared exponents of face rows (f, g), (f, g + 8)
//     for f = 0..3, in that order;
//   bytes [64 + h*512 + l*16, +16), h = 0, 1: for faces 2h, 2h + 1 the
//     words (row g, bytes 4t..4t+3) and (row g + 8, bytes 4t..4t+3).
// Byte offset, in the GGUF layout, of device-layout byte i of a tile.
__device__ __forceinline__ int gguf_offset(int i) {
  if (i < 64) {
    const int g = i >> 3, k = i & 7, f = k >> 1;
    return f * 16 + g + (k & 1) * 8;
  }
  const int j = i - 64, h = j >> 9, l = (j >> 4) & 31, w = (j >> 2) & 3, b = j & 3;
  const int f = 2 * h + (w >> 1), r = (l >> 2) + (w & 1) * 8, t = l & 3;
  return 64 + f * 256 + r * 16 + 4 * t + b;
}

// One warp per tile, in place: to_device = 1 converts GGUF -> device layout,
// 0 the reverse.
__global__ void __launch_bounds__(256) bfp8_transcode_kernel(uint8_t* __restrict__ tiles,
                                                             int64_t n_tiles, int to_device) {
  __shared__ __align__(16) uint8_t buf[8][TB];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = (int64_t)blockIdx.x * 8 + w;
  if (tile >= n_tiles) return;
  uint8_t* t = tiles + tile * TB;
  for (int i = lane; i < TB / 16; i += 32)
    reinterpret_cast<uint4*>(buf[w])[i] = reinterpret_cast<const uint4*>(t)[i];
  __syncwarp();
  for (int i = lane; i < TB; i += 32) {
    const int o = gguf_offset(i);
    if (i < 64) {  // shared exponents
      if (to_device)
        t[i] = buf[w][o];
      else
        t[o] = buf[w][i];
    } else if (to_device) {
      t[i] = buf[w][o];
    } else {
      t[o] = buf[w][i];
    }
  }
}

// One warp per tile: lane l packs face rows l and l + 32 (face = row / 16).
__global__ void __launch_bounds__(256) bfp8_pack_kernel(const uint16_t* __restrict__ w, int32_t K,
                                                        int32_t Kt, int64_t n_tiles,
                                                        uint8_t* __restrict__ out) {
  const int64_t tile = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (tile >= n_tiles) return;
  const int lane = threadIdx.x & 31;
  const int64_t mt = tile / Kt, kt = tile - mt * Kt;
  uint8_t* t = out + tile * TB;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int fr = lane + hh * 32, f = fr >> 4, r = fr & 15;
    const uint16_t* src = w + (mt * 32 + (f >> 1) * 16 + r) * (int64_t)K + kt * 32 + (f & 1) * 16;
    uint32_t x[16];
    const uint4 p0 = *reinterpret_cast<const uint4*>(src);
    const uint4 p1 = *reinterpret_cast<const uint4*>(src + 8);
    const uint32_t pw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    uint32_t se = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[2 * i] = pw[i] << 16;
      x[2 * i + 1] = pw[i] & 0xffff0000u;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) se = max(se, (x[i] >> 23) & 0xffu);
    uint32_t packed[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t u = x[i];
      uint32_t byte = 0;
      if ((u & 0x7fffffffu) != 0) {
        const uint32_t diff = se - ((u >> 23) & 0xffu);
        uint32_t mant = (u & 0x7fffffu) | 0x800000u;
        mant = diff >= 24 ? 0u : (mant >> diff);
        mant = min((mant + (1u << 16)) >> 17, 127u);
        byte = mant == 0 ? 0u : (((u >> 31) << 7) | mant);
      }
      packed[i >> 2] |= byte << (8 * (i & 3));
    }
    t[f * 16 + r] = uint8_t(se);
    *reinterpret_cast<uint4*>(t + 64 + f * 256 + r * 16) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

}  // namespace

// Once per device, outside any stream capture.
cudaError_t bfp8_prepare_device() {
  const int smem = (int)sizeof(GemvSmem);
  cudaError_t e = cudaFuncSetAttribute(bfp8_gemv_kernel<1>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bfp8_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return e;
}

// Launched with programmatic stream serialization: consecutive GEMVs overlap
// the next one's weight streaming with the previous one's tail.
cudaError_t launch_bfp8_gemv(const Bfp8GemvArgs& a, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(GEMV_THREADS, 1, 1);
  cfg.dynamicSmemBytes = sizeof(GemvSmem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = a.batch <= 8 ? cudaLaunchKernelEx(&cfg, bfp8_gemv_kernel<1>, a)
                   : cudaLaunchKernelEx(&cfg, bfp8_gemv_kernel<2>, a);
  if (e != cudaSuccess || a.S == 1) return e;
  cfg.gridDim = dim3((unsigned)(((int64_t)a.batch * a.M + 255) / 256), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg, bfp8_merge_kernel, a);
}

cudaError_t launch_bfp8_pack(const uint16_t* w, int32_t M, int32_t K, uint8_t* out, cudaStream_t s) {
  const int64_t n_tiles = (int64_t)(M / 32) * (K / 32);
  bfp8_pack_kernel<<<(unsigned)((n_tiles + 7) / 8), 256, 0, s>>>(w, K, K / 32, n_tiles, out);
  return cudaGetLastError();
}

cudaError_t launch_bfp8_transcode(uint8_t* tiles, int64_t n_tiles, int to_device, cudaStream_t s) {
  bfp8_transcode_kernel<<<(unsigned)((n_tiles + 7) / 8), 256, 0, s>>>(tiles, n_tiles, to_device);
  return cudaGetLastError();
}

int bfp8_gemv_columns() { return NMAX; }
int bfp8_gemv_warps_per_cta() { return NWARP; }
int bfp8_gemv_ctas_per_sm(int batch) { return 2; }

}  // namespace qc

// ------------------------------------------------------------- host ABI

struct qc_bfp8_matrix {
  int device = 0;
  int32_t M = 0, K = 0, Mt = 0, Kt = 0;
  int32_t ku = 0, S = 0, grid = 0, nsm = 0;
  uint8_t* tiles = nullptr;
  int64_t bytes = 0;
  float* partial = nullptr;  // [S][16][M]
  int* err = nullptr;
};

namespace {

int fail(int code, const std::string& msg) {
  qc::set_thread_error(msg.c_str());
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(QC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Current device switched to m->device for the scope.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int run_gemv(qc_bfp8_matrix* m, const uint16_t* x, int32_t batch, uint16_t* y0, int64_t ld0,
             uint16_t* y1, int64_t ld1, int32_t split, int mode, qc_stream stream) {
  if (!m || !x || !y0 || batch < 1 || (split < m->M && !y1))
    return fail(QC_ERR_ARG, "bfp8 gemv: bad arguments");
  DeviceScope ds(m->device);
  const int cols = qc::bfp8_gemv_columns();
  for (int32_t b0 = 0; b0 < batch; b0 += cols) {
    qc::Bfp8GemvArgs a{};
    a.w = m->tiles;
    a.x = x + (int64_t)b0 * m->K;
    a.y0 = y0 + (int64_t)b0 * ld0;
    a.y1 = y1 ? y1 + (int64_t)b0 * ld1 : nullptr;
    a.ld0 = ld0;
    a.ld1 = ld1;
    a.split = split;
    a.mode = mode;
    a.partial = m->partial;
    a.ku = m->ku;
    a.S = m->S;
    a.n_units = m->Mt * m->S;
    a.err = m->err;
    a.M = m->M;
    a.K = m->K;
    a.Mt = m->Mt;
    a.Kt = m->Kt;
    a.batch = std::min(cols, batch - b0);
    cudaError_t e = qc::launch_bfp8_gemv(a, m->grid, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "bfp8 gemv launch");
  }
  return QC_OK;
}

}  // namespace

extern "C" {

int64_t qc_bfp8_packed_bytes(int32_t M, int32_t K) {
  if (M <= 0 || K <= 0 || M % 32 || K % 32) return -1;
  return (int64_t)(M / 32) * (K / 32) * QC_BFP8_TILE_BYTES;
}

int qc_bfp8_create(int device, int32_t M, int32_t K, qc_bfp8_matrix** out) {
  if (!out) return fail(QC_ERR_ARG, "qc_bfp8_create: out is NULL");
  *out = nullptr;
  if (M <= 0 || K <= 0 || M % 32 || K % 32)
    return fail(QC_ERR_ARG, "qc_bfp8_create: M and K must be positive multiples of 32");
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || device < 0 || device >= n_dev) {
    cudaGetLastError();
    return fail(QC_ERR_NODEVICE, "qc_bfp8_create: no such CUDA device");
  }
  DeviceScope ds(device);
  auto* m = new qc_bfp8_matrix();
  m->device = device;
  m->M = M;
  m->K = K;
  m->Mt = M / 32;
  m->Kt = K / 32;
  m->bytes = qc_bfp8_packed_bytes(M, K);
  int nsm = 0;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device);
  m->nsm = std::max(1, nsm);
  m->grid = m->nsm * qc::bfp8_gemv_ctas_per_sm(1);
  // k-chunks per tile-row: the split that minimises the critical path, i.e.
  // (units per warp) x (tiles per unit + the unit epilogue, worth ~1 tile
  // alone and ~3 with the split-K merge); chunks of whole 4-tile stages
  const int64_t n_warps = (int64_t)m->grid * qc::bfp8_gemv_warps_per_cta();
  double best = 1e300;
  m->S = 1;
  m->ku = m->Kt;
  for (int32_t S = 1; S <= m->Kt; ++S) {
    int32_t ku = (m->Kt + S - 1) / S;
    if (m->Kt >= 4) ku = (ku + 3) / 4 * 4;
    if ((m->Kt + ku - 1) / ku != S) continue;
    const int64_t units = (int64_t)m->Mt * S;
    const double cost = (double)((units + n_warps - 1) / n_warps) * (ku + (S > 1 ? 3 : 1));
    if (cost < best - 1e-9) {
      best = cost;
      m->S = S;
      m->ku = ku;
    }
  }
  cudaError_t e = qc::bfp8_prepare_device();
  if (e == cudaSuccess) e = cudaMalloc(&m->tiles, (size_t)m->bytes);
  if (e == cudaSuccess && m->S > 1)
    e = cudaMalloc(&m->partial, (size_t)m->S * qc::bfp8_gemv_columns() * M * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&m->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(m->tiles, 0, (size_t)m->bytes);
  if (e == cudaSuccess) e = cudaMemset(m->err, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    qc_bfp8_destroy(m);
    return e == cudaErrorMemoryAllocation ? fail(QC_ERR_OOM, "qc_bfp8_create: out of device memory")
                                          : cuda_fail(e, "qc_bfp8_create");
  }
  *out = m;
  return QC_OK;
}

void qc_bfp8_destroy(qc_bfp8_matrix* m) {
  if (!m) return;
  DeviceScope ds(m->device);
  cudaFree(m->tiles);
  cudaFree(m->partial);
  cudaFree(m->err);
  delete m;
}

void* qc_bfp8_tiles(const qc_bfp8_matrix* m) { return m ? m->tiles : nullptr; }

int qc_bfp8_upload(qc_bfp8_matrix* m, const void* packed_host, qc_stream stream) {
  qc::TraceRange trace_("qc_bfp8_upload");
  if (!m || !packed_host) return fail(QC_ERR_ARG, "qc_bfp8_upload: bad arguments");
  DeviceScope ds(m->device);
  cudaError_t e = cudaMemcpyAsync(m->tiles, packed_host, (size_t)m->bytes, cudaMemcpyHostToDevice,
                                  (cudaStream_t)stream);
  if (e == cudaSuccess) e = qc::launch_bfp8_transcode(m->tiles, m->bytes / QC_BFP8_TILE_BYTES, 1,
                                                      (cudaStream_t)stream);
  return e == cudaSuccess ? QC_OK : cuda_fail(e, "qc_bfp8_upload");
}

int qc_bfp8_download(qc_bfp8_matrix* m, void* packed_host, qc_stream stream) {
  if (!m || !packed_host) return fail(QC_ERR_ARG, "qc_bfp8_download: bad arguments");
  DeviceScope ds(m->device);
  // GGUF layout for the copy, device layout again afterwards (stream order)
  const int64_t n = m->bytes / QC_BFP8_TILE_BYTES;
  cudaError_t e = qc::launch_bfp8_transcode(m->tiles, n, 0, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(packed_host, m->tiles, (size_t)m->bytes, cudaMemcpyDeviceToHost,
                        (cudaStream_t)stream);
  if (e == cudaSuccess) e = qc::launch_bfp8_transcode(m->tiles, n, 1, (cudaStream_t)stream);
  return e == cudaSuccess ? QC_OK : cuda_fail(e, "qc_bfp8_download");
}

int qc_bfp8_pack_bf16(qc_bfp8_matrix* m, const uint16_t* w_dev, qc_stream stream) {
  qc::TraceRange trace_("qc_bfp8_pack_bf16");
  if (!m || !w_dev) return fail(QC_ERR_ARG, "qc_bfp8_pack_bf16: bad arguments");
  if (reinterpret_cast<uintptr_t>(w_dev) & 15u)
    return fail(QC_ERR_ARG, "qc_bfp8_pack_bf16: w_dev must be 16-byte aligned");
  DeviceScope ds(m->device);
  cudaError_t e = qc::launch_bfp8_pack(w_dev, m->M, m->K, m->tiles, (cudaStream_t)stream);
  if (e == cudaSuccess) e = qc::launch_bfp8_transcode(m->tiles, m->bytes / QC_BFP8_TILE_BYTES, 1,
                                                      (cudaStream_t)stream);
  return e == cudaSuccess ? QC_OK : cuda_fail(e, "qc_bfp8_pack_bf16");
}

int qc_bfp8_gemv(qc_bfp8_matrix* m, const uint16_t* x_dev, int32_t batch, uint16_t* y_dev,
                 qc_stream stream) {
  qc::TraceRange trace_("qc_bfp8_gemv");
  if (!m) return fail(QC_ERR_ARG, "qc_bfp8_gemv: matrix is NULL");
  return run_gemv(m, x_dev, batch, y_dev, m->M, nullptr, 0, m->M, 0, stream);
}

int qc_bfp8_gemv_resadd(qc_bfp8_matrix* m, const uint16_t* x_dev, int32_t batch,
                        uint16_t* residual_dev, qc_stream stream) {
  qc::TraceRange trace_("qc_bfp8_gemv_resadd");
  if (!m) return fail(QC_ERR_ARG, "qc_bfp8_gemv_resadd: matrix is NULL");
  return run_gemv(m, x_dev, batch, residual_dev, m->M, nullptr, 0, m->M, 1, stream);
}

int qc_bfp8_gemv_split(qc_bfp8_matrix* m, const uint16_t* x_dev, int32_t batch, int32_t split_m,
                       uint16_t* y0_dev, uint16_t* y1_dev, qc_stream stream) {
  qc::TraceRange trace_("qc_bfp8_gemv_split");
  if (!m) return fail(QC_ERR_ARG, "qc_bfp8_gemv_split: matrix is NULL");
  if (split_m <= 0 || split_m >= m->M)
    return fail(QC_ERR_ARG, "qc_bfp8_gemv_split: split_m must be in (0, M)");
  return run_gemv(m, x_dev, batch, y0_dev, split_m, y1_dev, m->M - split_m, split_m, 0, stream);
}

int qc_bfp8_check(qc_bfp8_matrix* m) {
  if (!m) return fail(QC_ERR_ARG, "qc_bfp8_check: matrix is NULL");
  DeviceScope ds(m->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "qc_bfp8_check");
  int code = 0;
  e = cudaMemcpy(&code, m->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "qc_bfp8_check");
  if (code != 0) {
    cudaMemset(m->err, 0, sizeof(int));
    return fail(code, "bfp8 gemv: a bounded device wait expired");
  }
  return QC_OK;
}

}  // extern "C"
