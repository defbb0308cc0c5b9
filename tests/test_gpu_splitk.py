"""Split-K over KV positions across devices (long-context case), exercised on
one GPU: the page ranges that ranks would own are computed by qc_attn_partial
on one context, merged by qc_attn_combine and compared with the oracle."""
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

from gpu_util import assert_out_close, dev, empty_u16, host_f32, host_u16  # noqa: E402


@pytest.mark.parametrize("L,cuts", [(1000, [0, 5, 11, 16]), (4097, [0, 20, 40, 65]),
                                    (640, [0, 10, 10, 11])])
def test_partials_merge_to_the_full_decode(qcache, synth, oracle, L, cuts):
    d = synth.attn_inputs(90, 1, L)
    q = qcache.QCache(n_attn_layers=1, n_gdn_layers=1, max_seqs=2, max_pages=80, max_ctx=8192,
                      max_batch=2, max_snapshots=1, device=0)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    q.kv_write(s, 0, 0, L, dev(d["k"][0]).data_ptr(), dev(d["v"][0]).data_ptr())
    proj = dev(d["proj"])
    parts = torch.zeros(len(cuts) - 1, 16, 258, device="cuda")
    q.decode_begin([s])
    for g, (pb, pe) in enumerate(zip(cuts[:-1], cuts[1:])):
        last = g == len(cuts) - 2        # the range holding the new position appends
        q.attn_partial_range(pb, pe, int(last))
        q.attn_partial(0, proj.data_ptr(), parts[g].data_ptr())
    out = empty_u16(1, 4096)
    q.attn_combine(parts.data_ptr(), len(cuts) - 1, proj.data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    kc = np.zeros((L + 1, 4, 256), np.uint16)
    vc = np.zeros((L + 1, 4, 256), np.uint16)
    kc[:L], vc[:L] = d["k"][0], d["v"][0]
    ref = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], L, kc, vc)
    assert_out_close(host_u16(out)[0], ref, synth)
    # each record matches the oracle's partial over the same positions
    P = host_f32(parts)
    for g, (pb, pe) in enumerate(zip(cuts[:-1], cuts[1:])):
        p0, p1 = pb * 64, min(pe * 64, L + 1)
        r = oracle.attn_partial(d["proj"][0], d["q_norm"], L, kc, vc, p0, p1)
        if p1 <= p0:
            assert np.all(P[g][:, 0] == -np.inf) and np.all(P[g][:, 1] == 0)
            continue
        np.testing.assert_allclose(P[g][:, 0], r[:, 0], rtol=1e-5, atol=1e-4)
        scale = np.exp2(P[g][:, 0:1] - r[:, 0:1])
        np.testing.assert_allclose(P[g][:, 1:] , r[:, 1:] / scale, rtol=2e-3, atol=1e-3)
    # the append landed once, bit-exact
    kg, vg = empty_u16(L + 1, 4, 256), empty_u16(L + 1, 4, 256)
    q.kv_read(s, 0, 0, L + 1, kg.data_ptr(), vg.data_ptr())
    np.testing.assert_array_equal(host_u16(kg)[L], kc[L])
