"""GPU tests of the prefix cache: snapshot, page-list gather, tail-page
copy-on-write and DeltaNet/conv restore are bit-exact through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from gpu_util import dev, empty_u16, host_f32, host_u16  # noqa: E402


def make_ctx(qcache):
    return qcache.QCache(n_attn_layers=2, n_gdn_layers=2, max_seqs=8, max_pages=64,
                         max_ctx=2048, max_batch=4, max_snapshots=4, device=0)


def stand_up(q, synth, P, seed):
    """A sequence of length P with seeded KV in both attention layers and
    seeded DeltaNet state / conv history in both DeltaNet layers."""
    s = q.seq_alloc()
    q.seq_reserve(s, P)
    kv = {}
    for layer in range(2):
        d = synth.attn_inputs(seed + layer, 1, P)
        q.kv_write(s, layer, 0, P, dev(d["k"][0]).data_ptr(), dev(d["v"][0]).data_ptr())
        kv[layer] = (d["k"][0], d["v"][0])
        g = synth.gdn_inputs(seed + 10 + layer, 1)
        q.gdn_state_write(s, layer, dev(g["state"][0]).data_ptr(), dev(g["hist"][0]).data_ptr())
        kv[("g", layer)] = (g["state"][0], g["hist"][0])
    return s, kv


def read_all(q, s, P):
    res = {}
    for layer in range(2):
        k, v = empty_u16(P, 4, 256), empty_u16(P, 4, 256)
        q.kv_read(s, layer, 0, P, k.data_ptr(), v.data_ptr())
        res[layer] = (host_u16(k), host_u16(v))
        st = torch.zeros(32, 128, 128, device="cuda")
        hi = empty_u16(3, 8192)
        q.gdn_state_read(s, layer, st.data_ptr(), hi.data_ptr())
        res[("g", layer)] = (host_f32(st), host_u16(hi))
    return res


@pytest.mark.parametrize("P", [150, 128, 5])
def test_restore_is_bit_exact(qcache, synth, P):
    q = make_ctx(qcache)
    s, kv = stand_up(q, synth, P, seed=40)
    toks = list(range(7, 7 + P))
    e = q.prefix_insert(s, toks)
    matched, e2 = q.prefix_lookup(toks + [1, 2, 3])
    assert (matched, e2) == (P, e)
    t = q.seq_alloc()
    q.prefix_restore([e], [t])
    assert q.last_restore_bytes() > 0
    got = read_all(q, t, P)
    for layer in range(2):
        np.testing.assert_array_equal(got[layer][0], kv[layer][0])
        np.testing.assert_array_equal(got[layer][1], kv[layer][1])
        np.testing.assert_array_equal(got[("g", layer)][0], kv[("g", layer)][0])
        np.testing.assert_array_equal(got[("g", layer)][1], kv[("g", layer)][1])
    q.check_device()


def test_restored_sequence_decodes_like_the_original(qcache, synth):
    P = 150
    q = make_ctx(qcache)
    for layer in range(2):
        a = synth.attn_inputs(1, 1, 0)
        q.set_attn_params(layer, a["q_norm"], a["k_norm"])
        p = synth.gdn_params(2 + layer)
        q.set_gdn_params(layer, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    s, _ = stand_up(q, synth, P, seed=50)
    e = q.prefix_insert(s, list(range(P)))
    t = q.seq_alloc()
    q.prefix_restore([e], [t])
    pa = dev(synth.attn_inputs(60, 1, 0)["proj"])
    pg = dev(synth.gdn_inputs(61, 1)["proj"])
    outs = {}
    for seq in (s, t):
        oa, og = empty_u16(1, 4096), empty_u16(1, 4096)
        q.decode_begin([seq])
        q.gdn_decode(0, pg.data_ptr(), og.data_ptr())
        q.attn_decode(0, pa.data_ptr(), oa.data_ptr())
        q.decode_end()
        outs[seq] = (host_u16(oa), host_u16(og))
    np.testing.assert_array_equal(outs[s][0], outs[t][0])
    np.testing.assert_array_equal(outs[s][1], outs[t][1])
    # the decode appended into t's own tail page; the entry is untouched
    u = q.seq_alloc()
    q.prefix_restore([e], [u])
    assert q.seq_pages(u)[:2] == q.seq_pages(t)[:2]
    ku, _ = empty_u16(P, 4, 256), empty_u16(P, 4, 256)
    kt = empty_u16(P, 4, 256)
    q.kv_read(u, 0, 0, P, ku.data_ptr(), _.data_ptr())
    q.kv_read(t, 0, 0, P, kt.data_ptr(), _.data_ptr())
    np.testing.assert_array_equal(host_u16(ku), host_u16(kt))
    q.check_device()


def test_batched_restore_of_many_requests(qcache, synth):
    q = make_ctx(qcache)
    entries, data = [], []
    for i, P in enumerate([70, 200]):
        s, kv = stand_up(q, synth, P, seed=80 + 20 * i)
        entries.append(q.prefix_insert(s, [i] * P))
        data.append((P, kv))
    seqs = [q.seq_alloc() for _ in range(3)]
    pick = [1, 0, 1]
    q.prefix_restore([entries[i] for i in pick], seqs)
    for s, i in zip(seqs, pick):
        P, kv = data[i]
        got = read_all(q, s, P)
        np.testing.assert_array_equal(got[1][0], kv[1][0])
        np.testing.assert_array_equal(got[("g", 1)][0], kv[("g", 1)][0])
        np.testing.assert_array_equal(got[("g", 0)][1], kv[("g", 0)][1])
    q.check_device()
