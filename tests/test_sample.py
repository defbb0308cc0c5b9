"""CPU tests of the sampling restatement (oracle/sample.cpp): the exp it uses,
the greedy rule, the nucleus and the draw against a float64 numpy model of
the reference's sample_token (src/engine.cpp:3979-4036)."""
import numpy as np
import pytest


def np_sample(logits_f32, temperature, top_p, u):
    """numpy model with the same definitions (integer masses, index ties)."""
    if temperature <= 1e-7:
        return int(np.argmax(logits_f32)), 1
    mx = np.max(logits_f32)
    x = ((logits_f32 - mx).astype(np.float32) * np.float32(1.0 / np.float32(temperature))).astype(np.float32)
    q = np.rint(np.exp(x.astype(np.float64)) * 2.0 ** 31).astype(np.uint64)
    order = np.lexsort((np.arange(q.size), -q.astype(np.float64)))
    cum = np.cumsum(q[order])
    z = int(cum[-1])
    target = int(np.float64(np.float32(top_p)) * np.float64(z))
    cut = int(np.searchsorted(cum, target, side="left")) + 1
    kept = int(cum[cut - 1])
    r = int(u * np.float64(kept))
    i = int(np.searchsorted(cum[:cut], r, side="left"))
    while q[order[i]] == 0:
        i += 1
    return int(order[i]), cut


def test_exp_ref_accuracy(oracle):
    xs = np.concatenate([-np.logspace(-12, 2.85, 400), [0.0, -1e-300, -700.0, -744.9]])
    for x in xs:
        got, ref = oracle.exp_ref(x), np.exp(x)
        assert abs(got - ref) <= 4e-16 * ref + 1e-320, (x, got, ref)
    assert oracle.exp_ref(0.0) == 1.0
    assert oracle.exp_ref(-800.0) == 0.0


def test_greedy_first_max(oracle, synth):
    lg = np.zeros(1000, np.float32)
    lg[[17, 500, 999]] = 3.5
    lg[3] = np.nan
    tok, kept = oracle.sample(synth.bf16_bits(lg), 0.0)
    assert tok == 17 and kept == 1


@pytest.mark.parametrize("temp", [0.3, 0.7, 1.0, 2.5])
def test_matches_numpy_model(oracle, synth, temp):
    rng = np.random.default_rng(int(temp * 10))
    lg = synth.bf16_to_f32(synth.bf16_bits(rng.standard_normal(5000) * 3))
    bits = synth.bf16_bits(lg)
    for u in list(rng.random(40)) + [0.0, 0.999999999]:
        assert oracle.sample(bits, temp, 0.9, u) == np_sample(lg, temp, 0.9, u), u


def test_nucleus_edges(oracle, synth):
    lg = np.full(64, -20.0, np.float32)
    lg[5] = 10.0                                   # one dominant token: nucleus of 1
    tok, kept = oracle.sample(synth.bf16_bits(lg), 1.0, 0.9, 0.7)
    assert tok == 5 and kept == 1
    flat = np.zeros(64, np.float32)                # ties: index order, 90% of 64 = 58 (rounded up)
    for u, want in [(0.0, 0), (0.5, 28), (0.999, 57)]:
        tok, kept = oracle.sample(synth.bf16_bits(flat), 1.0, 0.9, u)
        assert kept == 58 and tok == want, (u, tok, kept)
    tok, kept = oracle.sample(synth.bf16_bits(flat), 1.0, 1.0, 0.999)
    assert kept == 64 and tok == 63
