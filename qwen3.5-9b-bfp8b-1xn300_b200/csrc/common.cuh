// common.cuh — device helpers shared by the cache-path kernels (sm_100a).
//
// Async copies use the Blackwell bulk-copy engine (cp.async.bulk, untiled
// TMA) completing on shared-memory mbarriers.  Every wait is bounded: on
// expiry the kernel records QC_ERR_TIMEOUT in the context's device error word
// and returns instead of spinning forever (no trap, no assert).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/qcache.h"

namespace qc {

constexpr unsigned FULL_MASK = 0xffffffffu;
constexpr uint64_t WAIT_LIMIT_NS = 1000ull * 1000ull * 1000ull;  // 1 s per wait

// ------------------------------------------------------------ error word

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// -------------------------------------------------------------- bf16 bits

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// Round to nearest even; the same bit recipe as the oracle's f32_to_bf16_rne.
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
__device__ __forceinline__ void unpack8(const uint4& w, float (&x)[8]) {
  x[0] = bf_lo(w.x); x[1] = bf_hi(w.x);
  x[2] = bf_lo(w.y); x[3] = bf_hi(w.y);
  x[4] = bf_lo(w.z); x[5] = bf_hi(w.z);
  x[6] = bf_lo(w.w); x[7] = bf_hi(w.w);
}

// -------------------------------------------------------- exact activations

__device__ __forceinline__ float sigmoid_exact(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_exact(float x) { return x * sigmoid_exact(x); }

// ------------------------------------ the reference's fast-math activations
// With QC_FLAG_REFERENCE_MATH the kernels compute what the reference computes
// (src/engine.cpp:2349-2376): Schraudolph's exp, i.e. clamp x to [-88, 88]
// and reinterpret the integer 12102203 * x + 1065353216 as float bits.  The
// scalar version (softplus, beta and gate sigmoids) converts by truncation;
// the AVX-512 SiLU (conv output, z gate) with _mm512_cvtps_epi32, which rounds
// to nearest even.  The reference's build (-ffast-math) contracts the
// multiply-add into one FMA, as here.
__device__ __forceinline__ float ref_exp_rz(float x) {
  x = fminf(fmaxf(x, -88.0f), 88.0f);
  return __int_as_float(__float2int_rz(fmaf(12102203.0f, x, 1065353216.0f)));
}
__device__ __forceinline__ float ref_exp_rn(float x) {
  x = fminf(fmaxf(x, -88.0f), 88.0f);
  return __int_as_float(__float2int_rn(fmaf(12102203.0f, x, 1065353216.0f)));
}
// the attention output gate and the DeltaNet beta (fast_sigmoidf)
__device__ __forceinline__ float gate_sigmoid(float x, int ref) {
  return ref ? 1.0f / (1.0f + ref_exp_rz(-x)) : sigmoid_exact(x);
}
// conv output and z gate (fast_silu_avx512)
__device__ __forceinline__ float act_silu(float x, int ref) {
  return ref ? x * (1.0f / (1.0f + ref_exp_rn(-x))) : silu_exact(x);
}
// the exp inside softplus (fast_expf)
__device__ __forceinline__ float softplus_exp(float x, int ref) {
  return ref ? ref_exp_rz(x) : expf(x);
}

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a barrier phase.  Returns false (and records a timeout)
// when the phase does not complete within WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0 && globaltimer() - t0 > WAIT_LIMIT_NS) {
      record_error(err, QC_ERR_TIMEOUT);
      return false;
    }
  }
}
// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a non-zero multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------- reductions

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(FULL_MASK, v, m);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, m));
  return v;
}

// Per-head RMSNorm + partial RoPE of one 256-wide head held by a warp, lane l
// owning dims 8l..8l+7 (src/engine.cpp:3497-3519 and 2422-2432).  Every
// operation is rounded explicitly (no contraction) in the order the oracle's
// qk_norm_rope documents, so the appended K bytes match it exactly.
__device__ __forceinline__ void norm_rope_lane(float (&x)[8], const float* __restrict__ w,
                                               const float* __restrict__ cs,
                                               const float* __restrict__ sn, int lane) {
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) s = __fmaf_rn(x[e], x[e], s);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) s = __fadd_rn(s, __shfl_xor_sync(FULL_MASK, s, m));
  const float var = __fadd_rn(__fdiv_rn(s, 256.0f), 1e-6f);
  const float rms = __fdiv_rn(1.0f, __fsqrt_rn(var));
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], rms), w[8 * lane + e]);
  float partner[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) partner[e] = __shfl_xor_sync(FULL_MASK, x[e], 4);
  if (lane < 4) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int p = 8 * lane + e;
      x[e] = __fsub_rn(__fmul_rn(x[e], cs[p]), __fmul_rn(partner[e], sn[p]));
    }
  } else if (lane < 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int p = 8 * (lane - 4) + e;
      x[e] = __fadd_rn(__fmul_rn(x[e], cs[p]), __fmul_rn(partner[e], sn[p]));
    }
  }
}

}  // namespace qc
