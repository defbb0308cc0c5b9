"""GPU parity of the attention path (fused Q/K norm + RoPE + bf16 KV append +
split-K paged flash-decode + gate) against the oracle, through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["mma", "tc"])
def attn_kernel(request, qcache):
    """Every test here runs on both decode-attention kernels (the launcher
    would pick by range length; forcing covers both on every case)."""
    mode = qcache.ATTN_KERNEL_MMA if request.param == "mma" else qcache.ATTN_KERNEL_TC
    qcache.attn_select_kernel(mode)
    yield request.param
    qcache.attn_select_kernel(qcache.ATTN_KERNEL_AUTO)

torch = pytest.importorskip("torch")

from gpu_util import (assert_out_close, dev, empty_u16, host_u16,  # noqa: E402
                      permute_free_pages)


def make_ctx(qcache, **kw):
    args = dict(n_attn_layers=2, n_gdn_layers=1, max_seqs=128, max_pages=512, max_ctx=8192,
                max_batch=16, max_snapshots=2, device=0)
    args.update(kw)
    return qcache.QCache(**args)


def oracle_step(oracle, d, b, ctx_len, kc, vc):
    return oracle.attn_decode(d["proj"][b], d["q_norm"], d["k_norm"], ctx_len, kc, vc)


def test_config0_single_layer_decode(qcache, synth, oracle):
    """Config 0: batch 1, 1024 cached positions, append at 1024."""
    L = 1024
    d = synth.attn_inputs(0, 1, L)
    q = make_ctx(qcache)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    k, v = dev(d["k"][0]), dev(d["v"][0])
    q.kv_write(s, 0, 0, L, k.data_ptr(), v.data_ptr())
    proj = dev(d["proj"])
    out = empty_u16(1, 4096)
    q.decode_begin([s])
    q.attn_decode(0, proj.data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    kc = np.zeros((L + 1, 4, 256), np.uint16)
    vc = np.zeros((L + 1, 4, 256), np.uint16)
    kc[:L], vc[:L] = d["k"][0], d["v"][0]
    ref = oracle_step(oracle, d, 0, L, kc, vc)
    assert_out_close(host_u16(out)[0], ref, synth)
    # gather the whole cache back: existing rows and the append are bit-exact
    kg, vg = empty_u16(L + 1, 4, 256), empty_u16(L + 1, 4, 256)
    q.kv_read(s, 0, 0, L + 1, kg.data_ptr(), vg.data_ptr())
    np.testing.assert_array_equal(host_u16(kg), kc)
    np.testing.assert_array_equal(host_u16(vg), vc)


@pytest.mark.parametrize("lens", [[0], [1], [65], [1500], [0, 1], [64, 65], [1, 1500],
                                  [0, 1, 63, 64, 65, 130, 700, 1500]])
def test_ragged_batch_permuted_pages(qcache, synth, oracle, lens):
    n = len(lens)
    q = make_ctx(qcache)
    permute_free_pages(q, 100, seed=7)
    d = synth.attn_inputs(5, n, max(lens))
    q.set_attn_params(1, d["q_norm"], d["k_norm"])
    seqs = [q.seq_alloc() for _ in range(n)]
    for s, L, b in zip(seqs, lens, range(n)):
        q.seq_reserve(s, L)
        if L:
            q.kv_write(s, 1, 0, L, dev(d["k"][b][:L]).data_ptr(), dev(d["v"][b][:L]).data_ptr())
    proj = dev(d["proj"])
    out = empty_u16(n, 4096)
    q.decode_begin(seqs)
    q.attn_decode(1, proj.data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    got = host_u16(out)
    for b, (s, L) in enumerate(zip(seqs, lens)):
        kc = np.zeros((L + 1, 4, 256), np.uint16)
        vc = np.zeros((L + 1, 4, 256), np.uint16)
        kc[:L], vc[:L] = d["k"][b][:L], d["v"][b][:L]
        ref = oracle_step(oracle, d, b, L, kc, vc)
        err = np.abs(synth.bf16_to_f32(got[b]) - ref).reshape(16, 256).max(1)
        assert err.max() < 0.05, (b, L, err)
        assert_out_close(got[b], ref, synth)
        kg, vg = empty_u16(L + 1, 4, 256), empty_u16(L + 1, 4, 256)
        q.kv_read(s, 1, 0, L + 1, kg.data_ptr(), vg.data_ptr())
        np.testing.assert_array_equal(host_u16(kg), kc)   # append bit-exact
        np.testing.assert_array_equal(host_u16(vg), vc)


def test_consecutive_steps_across_page_boundary(qcache, synth, oracle):
    L0, steps = 61, 6   # positions 61..66 cross the 64 boundary
    q = make_ctx(qcache)
    d = synth.attn_inputs(9, 1, L0)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L0)
    q.kv_write(s, 0, 0, L0, dev(d["k"][0]).data_ptr(), dev(d["v"][0]).data_ptr())
    kc = np.zeros((L0 + steps, 4, 256), np.uint16)
    vc = np.zeros((L0 + steps, 4, 256), np.uint16)
    kc[:L0], vc[:L0] = d["k"][0], d["v"][0]
    for t in range(steps):
        pd = synth.attn_inputs(100 + t, 1, 0)
        proj = dev(pd["proj"])
        out = empty_u16(1, 4096)
        q.decode_begin([s])
        q.attn_decode(0, proj.data_ptr(), out.data_ptr())
        q.decode_end()
        ref = oracle.attn_decode(pd["proj"][0], d["q_norm"], d["k_norm"], L0 + t, kc, vc)
        assert_out_close(host_u16(out)[0], ref, synth)
    q.check_device()
    assert q.seq_len(s) == L0 + steps and len(q.seq_pages(s)) == 2


def test_long_context_many_ctas_per_sequence(qcache, synth, oracle):
    """One sequence long enough that every SM holds a slice of it."""
    L = 20000
    q = make_ctx(qcache, max_pages=400, max_ctx=32768)
    d = synth.attn_inputs(21, 1, L)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    q.kv_write(s, 0, 0, L, dev(d["k"][0]).data_ptr(), dev(d["v"][0]).data_ptr())
    out = empty_u16(1, 4096)
    q.decode_begin([s])
    q.attn_decode(0, dev(d["proj"]).data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    kc = np.zeros((L + 1, 4, 256), np.uint16)
    vc = np.zeros((L + 1, 4, 256), np.uint16)
    kc[:L], vc[:L] = d["k"][0], d["v"][0]
    ref = oracle_step(oracle, d, 0, L, kc, vc)
    assert_out_close(host_u16(out)[0], ref, synth)


@pytest.mark.parametrize("path_pat", ["attn_*.npz"])
def test_golden_fixtures_on_gpu(qcache, synth, path_pat):
    import glob
    import os
    gdir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    for path in sorted(glob.glob(os.path.join(gdir, path_pat))):
        g = np.load(path)
        seed, L = int(g["seed"]), int(g["ctx"])
        d = synth.attn_inputs(seed, 1, L)
        q = make_ctx(qcache)
        q.set_attn_params(0, d["q_norm"], d["k_norm"])
        s = q.seq_alloc()
        q.seq_reserve(s, L)
        if L:
            q.kv_write(s, 0, 0, L, dev(d["k"][0]).data_ptr(), dev(d["v"][0]).data_ptr())
        out = empty_u16(1, 4096)
        q.decode_begin([s])
        q.attn_decode(0, dev(d["proj"]).data_ptr(), out.data_ptr())
        q.decode_end()
        assert_out_close(host_u16(out)[0], g["out"], synth)
        kg, vg = empty_u16(L + 1, 4, 256), empty_u16(L + 1, 4, 256)
        q.kv_read(s, 0, 0, L + 1, kg.data_ptr(), vg.data_ptr())
        np.testing.assert_array_equal(host_u16(kg)[L], g["k_new"])
        np.testing.assert_array_equal(host_u16(vg)[L], g["v_new"])
        q.close()


@pytest.mark.parametrize("shape", ["ramp", "spike_first", "spike_last"])
def test_softmax_reference_maximum_moves(qcache, synth, oracle, shape):
    """Scores built so that the online softmax's reference maximum must move
    by more than 2^8 from tile to tile (K rows of page t scaled by 1 + 3t,
    scores up to ~250: every tile rescales), never moves after the first page
    (the first page's keys scaled by 16), or moves only at the last page.
    Kernel and oracle read the same bf16 cache."""
    L = 1500
    d = synth.attn_inputs(11, 1, L)
    kf = synth.bf16_to_f32(d["k"][0]).copy()
    p = np.arange(L)
    if shape == "ramp":
        kf *= (1.0 + 3.0 * (p // 64)).astype(np.float32)[:, None, None]
    elif shape == "spike_first":
        kf[:64] *= 16.0
    else:
        kf[-40:] *= 16.0
    kb = synth.bf16_bits(kf)
    q = make_ctx(qcache)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    q.kv_write(s, 0, 0, L, dev(kb).data_ptr(), dev(d["v"][0]).data_ptr())
    proj = dev(d["proj"])
    out = empty_u16(1, 4096)
    q.decode_begin([s])
    q.attn_decode(0, proj.data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    kc = np.zeros((L + 1, 4, 256), np.uint16)
    vc = np.zeros((L + 1, 4, 256), np.uint16)
    kc[:L], vc[:L] = kb, d["v"][0]
    ref = oracle_step(oracle, d, 0, L, kc, vc)
    assert np.all(np.isfinite(ref))
    assert_out_close(host_u16(out)[0], ref, synth)
