"""CPU tests of the oracle: known-answer cases, an independent float64 numpy
restatement of the reference math, and the committed golden fixtures."""
import glob
import hashlib
import os

import numpy as np
import pytest

from conftest import load_pkg_module

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


# ---------------------------------------------------------------- numpy f64


def np_norm_rope(x, w, pos):
    x = x.astype(np.float64)
    y = x / np.sqrt(np.mean(x * x) + 1e-6) * w
    p = np.arange(32)
    th = pos * (1e7 ** (-2.0 * p / 64))
    c, s = np.cos(th), np.sin(th)
    y0, y1 = y[:32].copy(), y[32:64].copy()
    y[:32] = y0 * c - y1 * s
    y[32:64] = y1 * c + y0 * s
    return y


def np_attn(proj_bits, q_norm, k_norm, pos, k_cache_bits, v_cache_bits, synth):
    """float64 attention over a bf16 cache of pos rows plus the new token
    (src/engine.cpp:3485-3564)."""
    f = synth.bf16_to_f32(proj_bits).astype(np.float64)
    kn = np.stack([np_norm_rope(f[8192 + h * 256: 8192 + (h + 1) * 256], k_norm, pos)
                   for h in range(4)])
    knew = synth.bf16_to_f32(synth.bf16_bits(kn.astype(np.float32))).astype(np.float64)
    vnew = f[9216:10240].reshape(4, 256)
    K = np.concatenate([synth.bf16_to_f32(k_cache_bits[:pos]).astype(np.float64), knew[None]])
    V = np.concatenate([synth.bf16_to_f32(v_cache_bits[:pos]).astype(np.float64), vnew[None]])
    out = np.zeros((16, 256))
    for h in range(16):
        q = np_norm_rope(f[h * 512: h * 512 + 256], q_norm, pos)
        s = K[:, h // 4] @ q / 16.0
        p = np.exp(s - s.max())
        o = (p[:, None] * V[:, h // 4]).sum(0) / p.sum()
        g = f[h * 512 + 256: h * 512 + 512]
        out[h] = o / (1 + np.exp(-g))
    return out.reshape(-1)


def np_gdn(proj_bits, state, hist, p, synth):
    """float64 Gated DeltaNet step (src/engine.cpp:3204-3324)."""
    f = synth.bf16_to_f32(proj_bits).astype(np.float64)
    x = f[:8192]
    w = p["conv_w"].astype(np.float64)
    y = hist[0] * w[0] + hist[1] * w[1] + hist[2] * w[2] + x * w[3]
    y = y / (1 + np.exp(-y))
    z, alpha, beta = f[8192:12288], f[12288:12320], f[12320:12352]
    S = state.astype(np.float64).copy()
    out = np.zeros(4096)
    for vh in range(32):
        kh = vh % 16
        q = y[kh * 128:(kh + 1) * 128]
        k = y[2048 + kh * 128: 2048 + (kh + 1) * 128]
        v = y[4096 + vh * 128: 4096 + (vh + 1) * 128]
        q = q / np.sqrt((q * q).sum() + 1e-6)
        k = k / np.sqrt((k * k).sum() + 1e-6)
        b = alpha[vh] + p["dt_bias"][vh]
        sp = b if b > 20 else np.log1p(np.exp(b))
        decay = np.exp(sp * p["ssm_a"][vh])
        bt = 1 / (1 + np.exp(-beta[vh]))
        R = S[vh] * decay
        d = bt * (v - R @ k)
        R = R + d[:, None] * k[None, :]
        S[vh] = R
        o = (R @ q) / 11.3137
        rms = 1 / np.sqrt(np.mean(o * o) + 1e-6)
        zz = z[vh * 128:(vh + 1) * 128]
        out[vh * 128:(vh + 1) * 128] = o * rms * p["ssm_norm"] * zz / (1 + np.exp(-zz))
    return out, S


# ------------------------------------------------------------ known answers


def test_bf16_rne_known_values(oracle, synth):
    x = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -2.5, 65504.0, np.inf, 1e-40], np.float32)
    y = np.zeros(len(x), np.uint16)
    oracle.lib().qo_bf16_round(oracle._p(x), oracle._p(y), len(x))
    assert list(y[:4]) == [0x3F80, 0x3F80, 0x3F82, 0xC020]
    assert y[5] == 0x7F80
    np.testing.assert_array_equal(y, synth.bf16_bits(x))


def test_fast_expf_matches_schraudolph(oracle):
    L = oracle.lib()
    assert L.qo_fast_expf(0.0) == 1.0
    xs = np.linspace(-10, 10, 2001)
    rel = np.array([abs(L.qo_fast_expf(float(x)) - np.exp(x)) / np.exp(x) for x in xs])
    assert rel.max() < 0.065  # the reference's own approximation error (~6.2%)


def test_rope_identity_at_pos0(oracle):
    cs, sn = oracle.rope_table(0)
    np.testing.assert_array_equal(cs, np.ones(32, np.float32))
    np.testing.assert_array_equal(sn, np.zeros(32, np.float32))


def test_k_append_pos0_is_rmsnorm(oracle, synth):
    d = synth.attn_inputs(3, 1, 1)
    k = d["proj"][0][8192:9216]
    got = synth.bf16_to_f32(oracle.k_append(k, d["k_norm"], 0)).reshape(4, 256)
    x = synth.bf16_to_f32(k).reshape(4, 256).astype(np.float64)
    ref = x / np.sqrt((x * x).mean(1, keepdims=True) + 1e-6) * d["k_norm"]
    np.testing.assert_allclose(got, ref, rtol=2**-8, atol=1e-6)


def test_attention_single_position_is_gated_v(oracle, synth):
    d = synth.attn_inputs(4, 1, 0)
    k = np.zeros((1, 4, 256), np.uint16)
    v = np.zeros((1, 4, 256), np.uint16)
    out = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], 0, k, v).reshape(16, 256)
    f = synth.bf16_to_f32(d["proj"][0])
    for h in range(16):
        vv = f[9216 + (h // 4) * 256: 9216 + (h // 4 + 1) * 256]
        g = f[h * 512 + 256: h * 512 + 512]
        np.testing.assert_allclose(out[h], vv / (1 + np.exp(-g.astype(np.float64))), rtol=1e-6,
                                   atol=1e-7)


def test_gdn_identity_decay_zero_beta_keeps_state(oracle, synth):
    p = synth.gdn_params(5)
    p["ssm_a"] = np.zeros(32, np.float32)                  # decay = exp(0) = 1
    d = synth.gdn_inputs(5, 1)
    proj = d["proj"][0].copy()
    proj[12320:12352] = synth.bf16_bits(np.full(32, -60.0, np.float32))  # beta ~ 1e-26
    state = d["state"][0].copy()
    before = state.copy()
    hist = synth.bf16_to_f32(d["hist"][0]).copy()
    oracle.gdn_decode(proj, state, hist, p)
    np.testing.assert_allclose(state, before, rtol=1e-6, atol=1e-9)


def test_gdn_conv_history_shift(oracle, synth):
    p = synth.gdn_params(6)
    d = synth.gdn_inputs(6, 1)
    hist = synth.bf16_to_f32(d["hist"][0]).copy()
    h0 = hist.copy()
    oracle.gdn_decode(d["proj"][0], d["state"][0].copy(), hist, p)
    np.testing.assert_array_equal(hist[0], h0[1])
    np.testing.assert_array_equal(hist[1], h0[2])
    np.testing.assert_array_equal(hist[2], synth.bf16_to_f32(d["proj"][0][:8192]))


@pytest.mark.parametrize("cached,prompt,expect", [
    ([], [1, 2, 3], (0, False)),
    ([1, 2], [1, 2, 3, 4], (2, False)),
    ([1, 2, 9], [1, 2, 3, 4], (0, True)),      # divergence -> reset
    ([1, 2, 3], [1, 2, 3], (0, True)),          # fully cached -> reset
    ([1, 2, 3, 4], [1, 2], (0, True)),          # cache longer than prompt
])
def test_prefix_rule(oracle, cached, prompt, expect):
    assert oracle.prefix_decide(cached, prompt) == expect


# ---------------------------------------------- independent f64 restatement


@pytest.mark.parametrize("seed,ctx", [(31, 0), (32, 17), (33, 64), (34, 200)])
def test_attention_matches_f64_restatement(oracle, synth, seed, ctx):
    d = synth.attn_inputs(seed, 1, ctx)
    k = np.zeros((ctx + 1, 4, 256), np.uint16)
    v = np.zeros((ctx + 1, 4, 256), np.uint16)
    k[:ctx], v[:ctx] = d["k"][0], d["v"][0]
    ref = np_attn(d["proj"][0], d["q_norm"], d["k_norm"], ctx, d["k"][0], d["v"][0], synth)
    out = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], ctx, k, v)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("seed", [41, 42])
def test_gdn_matches_f64_restatement(oracle, synth, seed):
    p = synth.gdn_params(seed)
    d = synth.gdn_inputs(seed, 1)
    hist = synth.bf16_to_f32(d["hist"][0]).astype(np.float64)
    ref_out, ref_state = np_gdn(d["proj"][0], d["state"][0], hist, p, synth)
    state = d["state"][0].copy()
    h = synth.bf16_to_f32(d["hist"][0]).copy()
    out = oracle.gdn_decode(d["proj"][0], state, h, p)
    np.testing.assert_allclose(out, ref_out, rtol=1e-3, atol=1e-4)
    err = np.abs(state - ref_state).max() / np.abs(ref_state).max()
    assert err < 1e-5


def test_split_partials_recombine(oracle, synth):
    """Partials over disjoint position ranges merge to the one-pass result."""
    ctx = 150
    d = synth.attn_inputs(51, 1, ctx)
    k = np.zeros((ctx + 1, 4, 256), np.uint16)
    v = np.zeros((ctx + 1, 4, 256), np.uint16)
    k[:ctx], v[:ctx] = d["k"][0], d["v"][0]
    full = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], ctx, k, v)
    cuts = [0, 64, 128, ctx + 1]
    parts = np.stack([oracle.attn_partial(d["proj"][0], d["q_norm"], ctx, k, v, a, b)
                      for a, b in zip(cuts[:-1], cuts[1:])])
    np.testing.assert_allclose(oracle.attn_combine(parts, d["proj"][0]), full, rtol=1e-4, atol=1e-5)


def test_ref_approx_gap_is_bounded(oracle, synth):
    d = synth.attn_inputs(61, 1, 32)
    k = np.zeros((33, 4, 256), np.uint16)
    v = np.zeros((33, 4, 256), np.uint16)
    k[:32], v[:32] = d["k"][0], d["v"][0]
    a = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], 32, k.copy(), v.copy())
    b = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], 32, k.copy(), v.copy(),
                           mode=oracle.REF_APPROX)
    gap = np.abs(a - b).max()
    assert 0 < gap < 0.05


# ------------------------------------------------------------------- golden


def _golden(pattern):
    files = sorted(glob.glob(os.path.join(GOLDEN, pattern)))
    assert files, f"no golden fixtures {pattern}"
    return files


@pytest.mark.parametrize("path", _golden("attn_*.npz"))
def test_golden_attention(oracle, synth, path):
    g = np.load(path)
    seed, ctx = int(g["seed"]), int(g["ctx"])
    d = synth.attn_inputs(seed, 1, ctx)
    k = np.zeros((ctx + 1, 4, 256), np.uint16)
    v = np.zeros((ctx + 1, 4, 256), np.uint16)
    k[:ctx], v[:ctx] = d["k"][0], d["v"][0]
    out = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], ctx, k, v)
    np.testing.assert_array_equal(k[ctx], g["k_new"])
    np.testing.assert_array_equal(v[ctx], g["v_new"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("path", _golden("gdn_*.npz"))
def test_golden_gdn(oracle, synth, path):
    g = np.load(path)
    seed = int(g["seed"])
    p = synth.gdn_params(seed)
    d = synth.gdn_inputs(seed, 1)
    state = d["state"][0].copy()
    hist = synth.bf16_to_f32(d["hist"][0]).copy()
    out = oracle.gdn_decode(d["proj"][0], state, hist, p)
    np.testing.assert_allclose(out, g["out"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(state.reshape(-1)[::997], g["state_sample"], rtol=1e-6, atol=1e-9)
    np.testing.assert_array_equal(hist, g["hist"])
