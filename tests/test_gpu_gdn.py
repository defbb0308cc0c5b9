"""GPU parity of the Gated-DeltaNet decode step (conv ring + delta rule + gated
RMSNorm) against the oracle, through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from gpu_util import (assert_out_close, assert_state_close, dev, empty_u16,  # noqa: E402
                      host_f32, host_u16)


def make_ctx(qcache, n_seq, n_gdn=2):
    return qcache.QCache(n_attn_layers=1, n_gdn_layers=n_gdn, max_seqs=max(n_seq, 2),
                         max_pages=2 * max(n_seq, 2), max_ctx=1024, max_batch=max(n_seq, 2), max_snapshots=1,
                         device=0)


def setup(qcache, synth, n_seq, seed, layer=1, pos=0):
    q = make_ctx(qcache, n_seq)
    p = synth.gdn_params(seed)
    q.set_gdn_params(layer, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    d = synth.gdn_inputs(seed, n_seq)
    seqs = []
    for b in range(n_seq):
        s = q.seq_alloc()
        if pos:
            q.seq_reserve(s, pos)   # ring phase = pos & 3
        q.gdn_state_write(s, layer, dev(d["state"][b]).data_ptr(), dev(d["hist"][b]).data_ptr())
        seqs.append(s)
    return q, p, d, seqs


@pytest.mark.parametrize("n_seq,pos", [(1, 0), (1, 5), (8, 2), (64, 7)])
def test_gdn_step_matches_oracle(qcache, synth, oracle, n_seq, pos):
    layer = 1
    q, p, d, seqs = setup(qcache, synth, n_seq, seed=100 + n_seq, layer=layer, pos=pos)
    proj = dev(d["proj"])
    out = empty_u16(n_seq, 4096)
    q.decode_begin(seqs)
    q.gdn_decode(layer, proj.data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    got = host_u16(out)
    st = torch.zeros(32, 128, 128, device="cuda")
    hi = empty_u16(3, 8192)
    for b, s in enumerate(seqs):
        state = d["state"][b].copy()
        hist = synth.bf16_to_f32(d["hist"][b]).copy()
        ref = oracle.gdn_decode(d["proj"][b], state, hist, p)
        assert_out_close(got[b], ref, synth)
        q.gdn_state_read(s, layer, st.data_ptr(), hi.data_ptr())
        assert_state_close(host_f32(st), state)
        # conv history after the step: bit-exact shift with the new input
        np.testing.assert_array_equal(synth.bf16_to_f32(host_u16(hi)), hist)


def test_gdn_multi_step_ring_phases(qcache, synth, oracle):
    """Five consecutive tokens walk the 4-slot ring through every phase."""
    layer = 0
    q, p, d, seqs = setup(qcache, synth, 2, seed=7, layer=layer, pos=3)
    states = [d["state"][b].copy() for b in range(2)]
    hists = [synth.bf16_to_f32(d["hist"][b]).copy() for b in range(2)]
    for t in range(5):
        pd = synth.gdn_inputs(300 + t, 2)
        out = empty_u16(2, 4096)
        q.decode_begin(seqs)
        q.gdn_decode(layer, dev(pd["proj"]).data_ptr(), out.data_ptr())
        q.decode_end()
        got = host_u16(out)
        for b in range(2):
            ref = oracle.gdn_decode(pd["proj"][b], states[b], hists[b], p)
            assert_out_close(got[b], ref, synth)
    q.check_device()
    st = torch.zeros(32, 128, 128, device="cuda")
    hi = empty_u16(3, 8192)
    for b, s in enumerate(seqs):
        q.gdn_state_read(s, layer, st.data_ptr(), hi.data_ptr())
        assert_state_close(host_f32(st), states[b])
        np.testing.assert_array_equal(synth.bf16_to_f32(host_u16(hi)), hists[b])


def test_gdn_golden_fixtures_on_gpu(qcache, synth):
    import glob
    import os
    gdir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    for path in sorted(glob.glob(os.path.join(gdir, "gdn_*.npz"))):
        g = np.load(path)
        seed, pos = int(g["seed"]), int(g["pos"])
        q, p, d, seqs = setup(qcache, synth, 1, seed=seed, layer=0, pos=pos)
        out = empty_u16(1, 4096)
        q.decode_begin(seqs)
        q.gdn_decode(0, dev(d["proj"]).data_ptr(), out.data_ptr())
        q.decode_end()
        assert_out_close(host_u16(out)[0], g["out"], synth)
        q.close()
