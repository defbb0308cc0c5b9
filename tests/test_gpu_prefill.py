"""Chunked prefill against the oracle run token by token (the reference's
forward_prefill computes each token with the decode math), through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from gpu_util import (PREFILL_REL_FLOOR, assert_out_close, assert_state_close, dev,  # noqa: E402
                      empty_u16, host_f32, host_u16)


def ctx(qcache):
    return qcache.QCache(n_attn_layers=1, n_gdn_layers=1, max_seqs=4, max_pages=64,
                         max_ctx=4096, max_batch=4, max_snapshots=1, device=0)


@pytest.mark.parametrize("L,T", [(0, 1), (0, 32), (61, 7), (100, 32), (1000, 32), (64, 16)])
def test_attention_prefill_matches_token_by_token(qcache, synth, oracle, L, T):
    d = synth.attn_inputs(300 + L + T, 1, max(L, 1))
    pd = synth.attn_inputs(400 + T, T, 0)          # T projection rows
    q = ctx(qcache)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    if L:
        q.kv_write(s, 0, 0, L, dev(d["k"][0][:L]).data_ptr(), dev(d["v"][0][:L]).data_ptr())
    out = empty_u16(T, 4096)
    q.prefill_begin(s, T)
    q.attn_prefill(0, dev(pd["proj"]).data_ptr(), out.data_ptr())
    q.prefill_end()
    q.check_device()
    assert q.seq_len(s) == L + T
    kc = np.zeros((L + T, 4, 256), np.uint16)
    vc = np.zeros((L + T, 4, 256), np.uint16)
    kc[:L], vc[:L] = d["k"][0][:L], d["v"][0][:L]
    got = host_u16(out)
    for t in range(T):
        ref = oracle.attn_decode(pd["proj"][t], d["q_norm"], d["k_norm"], L + t, kc, vc)
        assert_out_close(got[t], ref, synth, PREFILL_REL_FLOOR)
    kg, vg = empty_u16(L + T, 4, 256), empty_u16(L + T, 4, 256)
    q.kv_read(s, 0, 0, L + T, kg.data_ptr(), vg.data_ptr())
    np.testing.assert_array_equal(host_u16(kg), kc)   # appends bit-exact
    np.testing.assert_array_equal(host_u16(vg), vc)


@pytest.mark.parametrize("pos,T", [(0, 1), (0, 32), (5, 3), (130, 32), (7, 2)])
def test_gdn_prefill_matches_token_by_token(qcache, synth, oracle, pos, T):
    p = synth.gdn_params(500 + T)
    d = synth.gdn_inputs(600 + pos, 1)
    pd = synth.gdn_inputs(700 + T, T)
    q = ctx(qcache)
    q.set_gdn_params(0, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    s = q.seq_alloc()
    if pos:
        q.seq_reserve(s, pos)
    q.gdn_state_write(s, 0, dev(d["state"][0]).data_ptr(), dev(d["hist"][0]).data_ptr())
    out = empty_u16(T, 4096)
    q.prefill_begin(s, T)
    q.gdn_prefill(0, dev(pd["proj"]).data_ptr(), out.data_ptr())
    q.prefill_end()
    q.check_device()
    state = d["state"][0].copy()
    hist = synth.bf16_to_f32(d["hist"][0]).copy()
    got = host_u16(out)
    for t in range(T):
        ref = oracle.gdn_decode(pd["proj"][t], state, hist, p)
        assert_out_close(got[t], ref, synth)
    st = torch.zeros(32, 128, 128, device="cuda")
    hi = empty_u16(3, 8192)
    q.gdn_state_read(s, 0, st.data_ptr(), hi.data_ptr())
    assert_state_close(host_f32(st), state)
    np.testing.assert_array_equal(synth.bf16_to_f32(host_u16(hi)), hist)


def test_prefill_then_decode_continues(qcache, synth, oracle):
    """A decode step after a prefill chunk sees the chunk's KV and state."""
    T = 20
    a = synth.attn_inputs(810, 1, 1)
    pa = synth.attn_inputs(811, T + 1, 0)
    q = ctx(qcache)
    q.set_attn_params(0, a["q_norm"], a["k_norm"])
    s = q.seq_alloc()
    out = empty_u16(T, 4096)
    q.prefill_begin(s, T, tokens=list(range(T)))
    q.attn_prefill(0, dev(pa["proj"][:T]).data_ptr(), out.data_ptr())
    q.prefill_end()
    o1 = empty_u16(1, 4096)
    q.decode_begin([s], tokens=[T])
    q.attn_decode(0, dev(pa["proj"][T:T + 1]).data_ptr(), o1.data_ptr())
    q.decode_end()
    q.check_device()
    kc = np.zeros((T + 1, 4, 256), np.uint16)
    vc = np.zeros((T + 1, 4, 256), np.uint16)
    for t in range(T):
        oracle.attn_decode(pa["proj"][t], a["q_norm"], a["k_norm"], t, kc, vc)
    ref = oracle.attn_decode(pa["proj"][T], a["q_norm"], a["k_norm"], T, kc, vc)
    assert_out_close(host_u16(o1)[0], ref, synth)
    assert q.match_prefix(s, list(range(T + 1)) + [99]) == T + 1


@pytest.mark.parametrize("poison", [0x7F80, 0x7FC0])   # bf16 +Inf, NaN
def test_prefill_ignores_stale_rows_of_a_reused_page(qcache, synth, oracle, poison):
    """A page freed by one sequence and reused by the next still holds the old
    rows past the new sequence's length.  Those rows enter the tensor-core
    P.V tile with P = 0; even non-finite leftovers must not reach the output."""
    T = 10
    q = qcache.QCache(n_attn_layers=1, n_gdn_layers=1, max_seqs=2, max_pages=2, max_ctx=128,
                      max_batch=1, max_snapshots=1, device=0)
    a = synth.attn_inputs(820, 1, 0)
    pa = synth.attn_inputs(821, T, 0)
    q.set_attn_params(0, a["q_norm"], a["k_norm"])
    old = q.seq_alloc()
    q.seq_reserve(old, 128)
    bad = np.full((128, 4, 256), poison, np.uint16)
    q.kv_write(old, 0, 0, 128, dev(bad).data_ptr(), dev(bad).data_ptr())
    torch.cuda.synchronize()
    q.seq_free(old)
    s = q.seq_alloc()
    out = empty_u16(T, 4096)
    q.prefill_begin(s, T)
    q.attn_prefill(0, dev(pa["proj"]).data_ptr(), out.data_ptr())
    q.prefill_end()
    q.check_device()
    kc = np.zeros((T, 4, 256), np.uint16)
    vc = np.zeros((T, 4, 256), np.uint16)
    got = host_u16(out)
    for t in range(T):
        ref = oracle.attn_decode(pa["proj"][t], a["q_norm"], a["k_norm"], t, kc, vc)
        assert_out_close(got[t], ref, synth, PREFILL_REL_FLOOR)
