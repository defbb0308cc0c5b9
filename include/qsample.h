/*
 * qsample.h — C ABI of token sampling on B200 (sm_100a), part of
 * libqcache.so.  Replaces sample_token (src/engine.cpp:3979-4036), which the
 * reference runs on the host over float logits after every forward pass
 * (src/engine.cpp:4113, 4157).
 *
 * For each of `batch` rows of bf16 logits (row b at logits_dev + b * ld):
 *   temperature <= 1e-7: the first index of the largest logit;
 *   otherwise, with x_v = (l_v - max) * (1 / temperature) in float, each
 *   token's mass is the integer q_v = round(exp(x_v) * 2^31) (exp evaluated
 *   in IEEE double by Cody-Waite reduction and a Taylor series, so the CPU
 *   restatement reproduces it bit for bit); tokens are ordered by mass
 *   decreasing, then index increasing; the nucleus is the shortest prefix
 *   whose mass reaches (uint64)(top_p * Z), Z the total mass (the reference
 *   uses top_p = 0.9); with kept = the nucleus mass and
 *   r = (uint64)(uniform[b] * kept), the sampled token is the first of the
 *   nucleus whose running mass reaches r.
 * The reference normalises float probabilities and draws r from a
 * process-global mt19937; here the caller supplies one uniform double in
 * [0, 1) per row (uniform_dev, ignored and may be NULL for greedy rows), and
 * the result depends on nothing else: not on timing, not on the GPU.
 * NaN logits are never chosen.  vocab <= QC_SAMPLE_MAX_VOCAB (the model's
 * 248320 fits); ld >= vocab.  No allocation; one launch on `stream`.
 * Returns QC_OK or QC_ERR_ARG / QC_ERR_CUDA (qc_last_error(NULL)).
 */
#ifndef QSAMPLE_H
#define QSAMPLE_H

#include "qcache.h"

#ifdef __cplusplus
extern "C" {
#endif

#define QC_SAMPLE_MAX_VOCAB 262144

int qc_sample(const uint16_t* logits_dev, int64_t ld, int32_t vocab, int32_t batch,
              float temperature, float top_p, const double* uniform_dev, int32_t* tokens_dev,
              qc_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* QSAMPLE_H */
