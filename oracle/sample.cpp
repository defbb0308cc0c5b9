// sample.cpp — CPU restatement of the reference's token sampler
// (sample_token, src/engine.cpp:3979-4036).
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py may load this library; the
// product (libqcache.so) never links or calls it.
//
// The reference, for one row of logits:
//   temperature <= 1e-7: the first index of the largest logit (strict >);
//   otherwise p_v = exp((l_v - max) / T), normalised; tokens in decreasing p
//   until the cumulative sum reaches top_p (0.9); one uniform draw r in
//   [0, kept sum) and the first token whose running sum reaches r.
// Restated with the choices the reference leaves open made explicit, so that
// a parallel implementation can match this one exactly:
//   - x_v = (l_v - max) * (1/T) in float, as the reference; the probability
//     mass of a token is the integer q_v = round(exp(x_v) * 2^31) (0 < q <=
//     2^31 for the largest logit), exp evaluated by exp_ref below (basic
//     IEEE double operations only, explicit fma: the same bits on any
//     IEEE machine).  Every sum is an exact 64-bit integer.
//   - tokens are ordered by q decreasing, then index increasing (the
//     reference's std::partial_sort leaves ties unspecified and sorts only
//     the first 1024 entries);
//   - the nucleus is the shortest prefix whose mass reaches
//     target = (uint64)(top_p * (double)Z), Z the total mass;
//   - the draw is an input: r = (uint64)(u * (double)kept) for a
//     caller-supplied u in [0, 1) (the reference draws from a process-global
//     mt19937); the sampled token is the first in order whose running mass
//     is >= r and whose own mass is not zero.
// NaN logits never win the argmax and have q = 0.  The logits are bf16 (the
// GEMV output that the reference widens to float).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

namespace {

inline float bf(uint16_t b) {
  uint32_t u = uint32_t(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// exp(x) for x <= 0 by Cody-Waite range reduction, x = k ln2 + r with
// |r| <= ln2 / 2 (ln2 split into a head with 21 significant bits, so k*head
// is exact for |k| < 2^11, and the tail), then the Taylor series of exp(r)
// to degree 13 (truncation error < 2^-60 relative) by Horner's rule with
// fused multiply-adds, and the exact scaling by 2^k.
double exp_ref(double x) {
  if (x < -745.0) return 0.0;
  const double LN2_HI = 0.693145751953125;           // 0x3FE62E4000000000
  const double LN2_LO = 1.42860682030941723212e-06;  // ln2 - LN2_HI
  const double k = std::nearbyint(x * 1.4426950408889634074);
  const double r = std::fma(-k, LN2_LO, std::fma(-k, LN2_HI, x));
  double p = 1.0 / 6227020800.0;                     // 1/13!
  const double inv_fact[13] = {1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0,
                               1.0 / 362880.0, 1.0 / 40320.0, 1.0 / 5040.0, 1.0 / 720.0,
                               1.0 / 120.0, 1.0 / 24.0, 1.0 / 6.0, 0.5, 1.0, 1.0};
  for (int i = 0; i < 13; ++i) p = std::fma(p, r, inv_fact[i]);
  return std::ldexp(p, (int)k);
}

}  // namespace

extern "C" {

double qo_exp_ref(double x) { return exp_ref(x); }

// Mass of one token: round(exp(x) * 2^31), x = (l - max) * inv_t in float.
uint32_t qo_sample_mass(float l, float max_l, float inv_t) {
  if (std::isnan(l)) return 0;
  const float x = (l - max_l) * inv_t;
  return (uint32_t)std::nearbyint(exp_ref((double)x) * 2147483648.0);
}

// Returns the sampled token of one row; *kept (may be null) receives the
// nucleus size.
int32_t qo_sample(const uint16_t* logits, int32_t vocab, float temperature, float top_p, double u,
                  int32_t* kept) {
  float max_l = -INFINITY;
  int32_t best = 0;
  for (int32_t v = 0; v < vocab; ++v) {
    const float l = bf(logits[v]);
    if (l > max_l) {
      max_l = l;
      best = v;
    }
  }
  if (temperature <= 1e-7f) {
    if (kept) *kept = 1;
    return best;
  }
  const float inv_t = 1.0f / temperature;
  std::vector<uint32_t> q(vocab);
  uint64_t z = 0;
  for (int32_t v = 0; v < vocab; ++v) {
    q[v] = qo_sample_mass(bf(logits[v]), max_l, inv_t);
    z += q[v];
  }
  std::vector<int32_t> idx(vocab);
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int32_t a, int32_t b) { return q[a] > q[b]; });
  const uint64_t target = (uint64_t)((double)top_p * (double)z);
  uint64_t cum = 0;
  int32_t cutoff = 0;
  for (int32_t i = 0; i < vocab; ++i) {
    cum += q[idx[i]];
    cutoff = i + 1;
    if (cum >= target) break;
  }
  if (kept) *kept = cutoff;
  const uint64_t r = (uint64_t)(u * (double)cum);
  uint64_t acc = 0;
  for (int32_t i = 0; i < cutoff; ++i) {
    acc += q[idx[i]];
    if (acc >= r && q[idx[i]] > 0) return idx[i];
  }
  return idx[0];
}

}  // extern "C"
