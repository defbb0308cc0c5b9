"""GPU parity of qc_sample (include/qsample.h) with the CPU restatement of the
reference's sample_token (oracle/sample.cpp): the sampled token is compared
exactly — every sum in the definition is an exact integer."""
import numpy as np
import pytest
import torch

from gpu_util import dev

pytestmark = pytest.mark.gpu

VOCAB = 248320


def run(qcache, logits_bits, temperature, top_p, us):
    B, V = logits_bits.shape
    lg = dev(logits_bits)
    u = dev(np.asarray(us, np.float64))
    tok = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    qcache.sample(lg.data_ptr(), V, V, B, temperature, top_p, u.data_ptr(), tok.data_ptr())
    torch.cuda.synchronize()
    return tok.cpu().numpy()


@pytest.mark.parametrize("temp", [0.0, 0.6, 1.0, 1.7])
def test_full_vocab_batch(qcache, oracle, synth, temp):
    B = 6
    rng = np.random.default_rng(int(temp * 100) + 1)
    scale = rng.uniform(1.0, 6.0, size=(B, 1))
    logits = synth.bf16_bits((synth.normal(70 + int(temp * 10), (B, VOCAB)) * scale).astype(np.float32))
    us = rng.random(B)
    got = run(qcache, logits, temp, 0.9, us)
    for b in range(B):
        want, _ = oracle.sample(logits[b], temp, 0.9, us[b])
        assert got[b] == want, (b, got[b], want)


def test_many_draws_one_row(qcache, oracle, synth):
    """The same row under 64 draws: every boundary of the nucleus exercised."""
    rng = np.random.default_rng(5)
    row = synth.bf16_bits((synth.normal(81, (VOCAB,)) * 2.5).astype(np.float32))
    us = np.concatenate([[0.0, 1.0 - 2.0 ** -52], rng.random(62)])
    logits = np.repeat(row[None], us.size, axis=0)
    got = run(qcache, logits, 0.8, 0.9, us)
    for b, u in enumerate(us):
        assert got[b] == oracle.sample(row, 0.8, 0.9, u)[0], u


@pytest.mark.parametrize("vocab", [1, 7, 1000, 65537])
def test_small_and_ragged_vocab(qcache, oracle, synth, vocab):
    rng = np.random.default_rng(vocab)
    logits = synth.bf16_bits(rng.standard_normal((3, vocab)).astype(np.float32) * 2)
    us = rng.random(3)
    for temp in (0.0, 1.0):
        got = run(qcache, logits, temp, 0.9, us)
        for b in range(3):
            assert got[b] == oracle.sample(logits[b], temp, 0.9, us[b])[0]


def test_ties_nan_and_top_p_one(qcache, oracle, synth):
    flat = np.zeros((3, 5000), np.float32)
    flat[1, 100] = np.nan
    flat[2, ::7] = 1.0
    bits = synth.bf16_bits(flat)
    us = [0.0, 0.5, 0.9999]
    for temp, top_p in ((1.0, 0.9), (1.0, 1.0), (0.0, 0.9), (0.3, 0.05)):
        got = run(qcache, bits, temp, top_p, us)
        for b in range(3):
            assert got[b] == oracle.sample(bits[b], temp, top_p, us[b])[0], (temp, top_p, b)


def test_rejects_bad_arguments(qcache):
    with pytest.raises(qcache.QCacheError):
        qcache.sample(16, 10, 10, 1, 1.0, 0.9, 0, 16)      # no uniforms for a sampled row
    with pytest.raises(qcache.QCacheError):
        qcache.sample(16, 10, 300000, 1, 0.0, 0.9, 0, 16)  # vocab above the maximum
