// bfp8.cpp — CPU restatement of the BFP8_B tiled weight format and of the
// GEMV family that reads it.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py may load this library; the
// product (libqcache.so) never links or calls it.
//
// Format (GGUF tensor type 200, src/gguf_loader.cpp:44-47,151-153): a [M][K]
// matrix (M, K multiples of 32) is stored as (M/32)*(K/32) tiles of 1088 bytes
// in row-major tile order (tile (mt, kt) at index mt*(K/32)+kt); the reference
// tiles the bf16 rows (tools/make_bfp8_gguf.cpp:160-182, src/engine.cpp:
// 1831-1852) and hands each 32x32 block to tt-metalium's
// pack_as_bfp_tiles<Bfp8_b>(row_major_input=true, is_exp_a=false).
//
// tt-metalium (v0.66.0, Dockerfile:10) is a third-party dependency that is
// absent here; its published packing algorithm is restated below:
//   - a tile is 4 faces of 16x16: face 0 rows 0-15 cols 0-15, face 1 rows 0-15
//     cols 16-31, face 2 rows 16-31 cols 0-15, face 3 rows 16-31 cols 16-31;
//   - bytes [0, 64): one shared exponent per face row, byte f*16 + r;
//   - bytes [64, 1088): one byte per element, face-major, rows of 16:
//     byte 64 + f*256 + r*16 + c = sign << 7 | 7-bit magnitude;
//   - shared exponent = max of the 8-bit float exponents of the row's 16
//     values; each magnitude = (1.mantissa) shifted right by (shared - own
//     exponent), rounded at 7 bits (add half, truncate), saturated at 127;
//     exact zeros encode as 0, and a magnitude that rounds to 0 drops its sign;
//   - decoded value = (-1)^sign * magnitude * 2^(shared_exp - 133).
// Parity of the PACKER is unpinned against tt-metalium (no golden tiles ship
// with the reference).  The decode rule is the format's definition, and the
// GPU kernels are checked against this file's decode + fp32 dot products.
//
// GEMV semantics (src/engine.cpp:371-486 dispatch_gemv, :498 dispatch_gemv_resadd,
// :619 dispatch_gemv_split): y[b][m] = sum_k W[m][k] * x[b][k], x bf16,
// accumulation f32, output rounded to bf16.  The resadd variant follows the
// reference's writer (src/kernels/dataflow/writer_gemv_resadd.cpp): the GEMV
// output is rounded to bf16 first, added to the bf16 residual in f32, and the
// sum is truncated to bf16.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr int TILE = 32, FACE = 16, TILE_BYTES = 1088, EXP_BYTES = 64;

inline uint32_t bits_of(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
inline float float_of(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline float bf(uint16_t b) { return float_of(uint32_t(b) << 16); }
inline uint16_t bf_rne(float f) {
  uint32_t u = bits_of(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
inline uint16_t bf_trunc(float f) { return uint16_t(bits_of(f) >> 16); }

// One element: f32 bits -> sign/magnitude byte under the row's shared exponent.
inline uint8_t encode(uint32_t u, uint32_t shared_exp) {
  if ((u & 0x7fffffffu) == 0) return 0;
  const uint32_t exp = (u >> 23) & 0xffu, sign = u >> 31;
  uint32_t mant = (u & 0x7fffffu) | 0x800000u;  // 24 bits with the hidden one
  const uint32_t diff = shared_exp - exp;       // shared_exp >= exp
  mant = diff >= 24 ? 0u : (mant >> diff);
  mant = (mant + (1u << 16)) >> 17;             // keep 7 bits, add half
  mant = std::min(mant, 127u);
  return uint8_t(mant == 0 ? 0u : ((sign << 7) | mant));
}

// Dequantises tile-row mt of a packed matrix into rows [mt*32, mt*32+32) of w.
void unpack_tile_row(const uint8_t* packed, int Kt, int mt, float* w, int K) {
  for (int kt = 0; kt < Kt; ++kt) {
    const uint8_t* t = packed + ((int64_t)mt * Kt + kt) * TILE_BYTES;
    for (int f = 0; f < 4; ++f)
      for (int r = 0; r < FACE; ++r) {
        const float scale = std::ldexp(1.0f, int(t[f * FACE + r]) - 133);
        const int row = (f >> 1) * FACE + r;
        const uint8_t* b = t + EXP_BYTES + f * 256 + r * FACE;
        float* dst = w + (int64_t)row * K + kt * TILE + (f & 1) * FACE;
        for (int c = 0; c < FACE; ++c) {
          const float mag = float(b[c] & 0x7f) * scale;  // exact: 7-bit integer times a power of two
          dst[c] = (b[c] & 0x80) ? -mag : mag;
        }
      }
  }
}

template <class F>
void parallel_rows(int n, int n_threads, F fn) {
  n_threads = std::max(1, std::min(n_threads, n));
  if (n_threads == 1) {
    for (int i = 0; i < n; ++i) fn(i);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < n_threads; ++t)
    th.emplace_back([=] {
      for (int i = t; i < n; i += n_threads) fn(i);
    });
  for (auto& x : th) x.join();
}

}  // namespace

extern "C" {

int64_t qo_bfp8_packed_bytes(int M, int K) { return (int64_t)(M / TILE) * (K / TILE) * TILE_BYTES; }

// Row-major bf16 [M][K] -> packed tiles (tools/make_bfp8_gguf.cpp:160-182).
void qo_bfp8_pack(const uint16_t* w, int M, int K, uint8_t* out) {
  const int Mt = M / TILE, Kt = K / TILE;
  for (int mt = 0; mt < Mt; ++mt)
    for (int kt = 0; kt < Kt; ++kt) {
      uint8_t* t = out + ((int64_t)mt * Kt + kt) * TILE_BYTES;
      for (int f = 0; f < 4; ++f)
        for (int r = 0; r < FACE; ++r) {
          const int row = mt * TILE + (f >> 1) * FACE + r;
          const uint16_t* src = w + (int64_t)row * K + kt * TILE + (f & 1) * FACE;
          uint32_t se = 0;
          for (int c = 0; c < FACE; ++c) se = std::max(se, (uint32_t(src[c]) >> 7) & 0xffu);
          t[f * FACE + r] = uint8_t(se);
          for (int c = 0; c < FACE; ++c)
            t[EXP_BYTES + f * 256 + r * FACE + c] = encode(uint32_t(src[c]) << 16, se);
        }
    }
}

void qo_bfp8_unpack(const uint8_t* packed, int M, int K, float* w) {
  const int Kt = K / TILE;
  for (int mt = 0; mt < M / TILE; ++mt) unpack_tile_row(packed, Kt, mt, w + (int64_t)mt * TILE * K, K);
}

// y32[b][m] (f32 sums, may be null) and y[b][m] (bf16) for b < batch.
// mode 0: y = bf16_rne(W x); mode 1 (resadd): y = bf16_trunc(bf16_rne(W x) + y_in).
// Rows are spread over n_threads host threads; each row sums k in order.
void qo_bfp8_gemv(const uint8_t* packed, int M, int K, const uint16_t* x, int batch, int mode,
                  uint16_t* y, float* y32, int n_threads) {
  const int Kt = K / TILE;
  std::vector<float> xf((size_t)batch * K);
  for (size_t i = 0; i < xf.size(); ++i) xf[i] = bf(x[i]);
  parallel_rows(M / TILE, n_threads, [&](int mt) {
    std::vector<float> w((size_t)TILE * K);
    unpack_tile_row(packed, Kt, mt, w.data(), K);
    for (int r = 0; r < TILE; ++r) {
      const int m = mt * TILE + r;
      const float* wr = w.data() + (size_t)r * K;
      for (int b = 0; b < batch; ++b) {
        const float* xb = xf.data() + (size_t)b * K;
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) acc += wr[k] * xb[k];
        if (y32) y32[(int64_t)b * M + m] = acc;
        uint16_t& dst = y[(int64_t)b * M + m];
        dst = mode == 1 ? bf_trunc(bf(bf_rne(acc)) + bf(dst)) : bf_rne(acc);
      }
    }
  });
}

}  // extern "C"
