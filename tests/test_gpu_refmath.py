"""The kernels against the REFERENCE's own outputs (QC_FLAG_REFERENCE_MATH).

tests/golden/ref_*.npz hold what the reference's host code computes
(src/engine.cpp:3198-3330 and :3484-3566, compiled unchanged from its source
by oracle/ref_harness.cpp).  A context created with QC_FLAG_REFERENCE_MATH
uses the reference's fast-math activations, so its outputs must match those
fixtures within the parity gate (max-abs 2e-2 / rel 1e-2 on the bf16 output,
1e-4 relative per element on the fp32 state).  The oracle's REF_APPROX mode,
pinned to the same fixtures on the CPU (tests/test_ref_pin.py), covers the
cases the fixtures do not: a ragged batch, prefill chunks."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from gpu_util import assert_out_close, assert_state_close, dev, empty_u16, host_f32, host_u16  # noqa: E402

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REF = 1  # QC_FLAG_REFERENCE_MATH


def fixtures(prefix):
    return sorted(f for f in os.listdir(GOLD) if f.startswith(prefix) and f.endswith(".npz"))


def ctx(qcache, **kw):
    args = dict(n_attn_layers=1, n_gdn_layers=1, max_seqs=8, max_pages=600, max_ctx=8192,
                max_batch=8, max_snapshots=1, device=0, flags=REF)
    args.update(kw)
    return qcache.QCache(**args)


@pytest.mark.parametrize("name", fixtures("ref_attn_"))
def test_attention_matches_reference_outputs(qcache, synth, name):
    z = np.load(os.path.join(GOLD, name))
    seed, L = int(z["seed"]), int(z["ctx"])
    d = synth.attn_inputs(seed, 1, L)
    q = ctx(qcache)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    if L:
        q.kv_write(s, 0, 0, L, dev(d["k"][0]).data_ptr(), dev(d["v"][0]).data_ptr())
    out = empty_u16(1, 4096)
    q.decode_begin([s])
    q.attn_decode(0, dev(d["proj"]).data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    assert_out_close(host_u16(out)[0], z["out"], synth)
    # the append is the reference's f32 row rounded to bf16 (RoPE table
    # differences aside, see test_ref_pin.py)
    kg, vg = empty_u16(1, 4, 256), empty_u16(1, 4, 256)
    q.kv_read(s, 0, L, 1, kg.data_ptr(), vg.data_ptr())
    kf = synth.bf16_to_f32(host_u16(kg)[0])
    tol = np.abs(z["k_new"]) * 2.0 ** -8 + 2.0 ** -22 * max(L, 1) * np.abs(z["k_new"]).max() + 1e-6
    assert np.all(np.abs(kf - z["k_new"]) <= tol)
    np.testing.assert_array_equal(synth.bf16_to_f32(host_u16(vg)[0]), z["v_new"])
    q.close()


@pytest.mark.parametrize("name", fixtures("ref_gdn_"))
@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_deltanet_matches_reference_outputs(qcache, synth, name, path):
    z = np.load(os.path.join(GOLD, name))
    seed, pseed, steps = int(z["seed"]), int(z["pseed"]), int(z["steps"])
    p = synth.gdn_params(pseed)
    d = synth.gdn_inputs(seed, 1)
    q = ctx(qcache)
    q.set_gdn_params(0, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    s = q.seq_alloc()
    q.gdn_state_write(s, 0, dev(d["state"][0]).data_ptr(), dev(d["hist"][0]).data_ptr())
    projs = dev(np.ascontiguousarray(z["proj"]))
    if path == "decode":
        for t in range(steps):
            out = empty_u16(1, 4096)
            q.decode_begin([s])
            q.gdn_decode(0, projs[t:t + 1].data_ptr(), out.data_ptr())
            q.decode_end()
            assert_out_close(host_u16(out)[0], z["out"][t], synth)
    else:
        out = empty_u16(steps, 4096)
        q.prefill_begin(s, steps)
        q.gdn_prefill(0, projs.data_ptr(), out.data_ptr())
        q.prefill_end()
        got = host_u16(out)
        for t in range(steps):
            assert_out_close(got[t], z["out"][t], synth)
    q.check_device()
    st, hi = torch.zeros(32, 128, 128, device="cuda"), empty_u16(3, 8192)
    q.gdn_state_read(s, 0, st.data_ptr(), hi.data_ptr())
    state = host_f32(st)
    assert_state_close(state[z["heads"]], z["state_heads"])
    sums = state.astype(np.float64).sum(axis=2)
    assert np.abs(sums - z["row_sums"][-1]).max() <= 1e-4 * np.abs(z["row_sums"][-1]).max()
    np.testing.assert_array_equal(synth.bf16_to_f32(host_u16(hi)), z["hist"])
    q.close()


def test_reference_math_batch_against_oracle(qcache, synth, oracle):
    """A ragged batch of 6 sequences in both layer types, reference math,
    against the oracle's REF_APPROX mode (itself pinned to the reference)."""
    lens = [0, 1, 63, 64, 700, 1500]
    n = len(lens)
    d = synth.attn_inputs(910, n, max(lens))
    p = synth.gdn_params(911)
    g = synth.gdn_inputs(912, n)
    q = ctx(qcache)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    q.set_gdn_params(0, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    seqs = [q.seq_alloc() for _ in range(n)]
    for b, (s, L) in enumerate(zip(seqs, lens)):
        q.seq_reserve(s, L)
        if L:
            q.kv_write(s, 0, 0, L, dev(d["k"][b][:L]).data_ptr(), dev(d["v"][b][:L]).data_ptr())
        q.gdn_state_write(s, 0, dev(g["state"][b]).data_ptr(), dev(g["hist"][b]).data_ptr())
    oa, og = empty_u16(n, 4096), empty_u16(n, 4096)
    q.decode_begin(seqs)
    q.attn_decode(0, dev(d["proj"]).data_ptr(), oa.data_ptr())
    q.gdn_decode(0, dev(g["proj"]).data_ptr(), og.data_ptr())
    q.decode_end()
    q.check_device()
    ga, gg = host_u16(oa), host_u16(og)
    for b, L in enumerate(lens):
        kc = np.zeros((L + 1, 4, 256), np.uint16)
        vc = np.zeros((L + 1, 4, 256), np.uint16)
        kc[:L], vc[:L] = d["k"][b][:L], d["v"][b][:L]
        ref = oracle.attn_decode(d["proj"][b], d["q_norm"], d["k_norm"], L, kc, vc,
                                 mode=oracle.REF_APPROX)
        assert_out_close(ga[b], ref, synth)
        st = g["state"][b].copy()
        hist = synth.bf16_to_f32(g["hist"][b]).copy()
        ref = oracle.gdn_decode(g["proj"][b], st, hist, p, mode=oracle.REF_APPROX)
        assert_out_close(gg[b], ref, synth)
    q.close()
