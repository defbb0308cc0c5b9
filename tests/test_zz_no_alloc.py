"""qc_attn_decode_noalloc against qc_attn_decode, through the C ABI.

The no-allocation entry point serves callers that may not allocate device
memory themselves (an engine that owns all GPU memory in its own arena, a
plugin inside another framework's memory pool): they keep the KV pool, the
page table, the weights and the RoPE table in their own buffers, and the
kernel's scratch lives in a fixed array inside the library.  This test builds
such caller-owned buffers with the same contents as a context-managed
sequence, runs two consecutive decode steps through both entry points and
requires the same outputs (within the parity tolerance) and the same appended
K/V bytes, and checks both against the oracle; it also checks that the
kernels' error word reaches the caller through qc_attn_noalloc_check.  It
sits in its own file, collected last, so a failure here stops a
-x run only after every other test ran.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from gpu_util import assert_f32_close, assert_out_close, dev, empty_u16, host_u16  # noqa: E402


def test_noalloc_matches_context_decode_two_steps(qcache, synth, oracle):
    lens = [130, 1, 700]          # ragged batch: partial pages, one near-empty sequence
    n, steps = len(lens), 2
    max_pages, pt_stride = 64, 16
    d = synth.attn_inputs(77, n, max(lens))

    # --- context path (existing entry point)
    q = qcache.QCache(n_attn_layers=1, n_gdn_layers=1, max_seqs=n, max_pages=max_pages,
                      max_ctx=pt_stride * 64, max_batch=n, max_snapshots=1, device=0)
    q.set_attn_params(0, d["q_norm"], d["k_norm"])
    seqs = [q.seq_alloc() for _ in range(n)]
    for b, (s, L) in enumerate(zip(seqs, lens)):
        q.seq_reserve(s, L)
        q.kv_write(s, 0, 0, L, dev(d["k"][b][:L]).data_ptr(), dev(d["v"][b][:L]).data_ptr())

    # --- caller-owned buffers for the no-allocation path, same contents
    rng = np.random.default_rng(5)
    phys = rng.permutation(max_pages)[: n * pt_stride].reshape(n, pt_stride).astype(np.int32)
    kpool = torch.zeros(max_pages, 4, 64, 256, dtype=torch.int16, device="cuda")
    vpool = torch.zeros_like(kpool)
    for b, L in enumerate(lens):
        for p in range(L):
            kpool[phys[b, p // 64], :, p % 64] = dev(d["k"][b][p])
            vpool[phys[b, p // 64], :, p % 64] = dev(d["v"][b][p])
    ptab = dev(phys)
    maxpos = max(lens) + steps
    cs = np.zeros((maxpos, 32), np.float32)
    sn = np.zeros((maxpos, 32), np.float32)
    for p in range(maxpos):
        cs[p], sn[p] = oracle.rope_table(p)
    rope_c, rope_s = dev(cs), dev(sn)
    qn, kn = dev(d["q_norm"]), dev(d["k_norm"])

    for t in range(steps):
        proj = dev(synth.attn_inputs(200 + t, n, 0)["proj"])
        out_ctx = empty_u16(n, 4096)
        q.decode_begin(seqs)
        q.attn_decode(0, proj.data_ptr(), out_ctx.data_ptr())
        q.decode_end()
        out_na = empty_u16(n, 4096)
        pos = [L + t for L in lens]
        qcache.attn_decode_noalloc(proj.data_ptr(), kpool.data_ptr(), vpool.data_ptr(),
                                   max_pages, ptab.data_ptr(), pt_stride, pos, qn.data_ptr(),
                                   kn.data_ptr(), rope_c.data_ptr(), rope_s.data_ptr(),
                                   out_na.data_ptr())
        qcache.attn_noalloc_check()
        a = synth.bf16_to_f32(host_u16(out_na))
        b_ = synth.bf16_to_f32(host_u16(out_ctx))
        assert_f32_close(a, b_)
        # and both against the oracle, over the same cache contents
        for b, L in enumerate(lens):
            P = L + t
            kc = np.zeros((P + 1, 4, 256), np.uint16)
            vc = np.zeros((P + 1, 4, 256), np.uint16)
            kp, vp = host_u16(kpool), host_u16(vpool)
            for p in range(P):
                kc[p], vc[p] = kp[phys[b, p // 64], :, p % 64], vp[phys[b, p // 64], :, p % 64]
            ref = oracle.attn_decode(host_u16(proj)[b], d["q_norm"], d["k_norm"], P, kc, vc)
            assert_out_close(host_u16(out_na)[b], ref, synth)
    q.check_device()

    # the appends of both steps landed in the caller's pool, bit for bit
    for b, (s, L) in enumerate(zip(seqs, lens)):
        kg, vg = empty_u16(L + steps, 4, 256), empty_u16(L + steps, 4, 256)
        q.kv_read(s, 0, 0, L + steps, kg.data_ptr(), vg.data_ptr())
        kk, vv = host_u16(kg), host_u16(vg)
        kp, vp = host_u16(kpool), host_u16(vpool)
        for p in range(L, L + steps):
            np.testing.assert_array_equal(kp[phys[b, p // 64], :, p % 64], kk[p])
            np.testing.assert_array_equal(vp[phys[b, p // 64], :, p % 64], vv[p])


def test_noalloc_rejects_oversized_batch(qcache):
    with pytest.raises(qcache.QCacheError) as e:
        qcache.attn_decode_noalloc(16, 16, 16, 8, 16, 4, [0] * 65, 16, 16, 16, 16, 16)
    assert e.value.code == qcache.QC_ERR_ARG
    assert "limit" in str(e.value)


def test_noalloc_reports_out_of_range_page(qcache, synth):
    """A page-table entry outside [0, max_pages) makes the kernel skip that
    tile and record QC_ERR_BOUNDS; qc_attn_noalloc_check returns it once and
    clears it, so the next good call checks clean."""
    n, max_pages, pt_stride, L = 1, 8, 4, 130
    d = synth.attn_inputs(78, n, L)
    kpool = torch.zeros(max_pages, 4, 64, 256, dtype=torch.int16, device="cuda")
    vpool = torch.zeros_like(kpool)
    cs = np.zeros((L + 1, 32), np.float32)
    sn = np.zeros((L + 1, 32), np.float32)
    rope_c, rope_s = dev(cs), dev(sn)
    qn, kn = dev(d["q_norm"]), dev(d["k_norm"])
    proj = dev(d["proj"])
    out = empty_u16(n, 4096)
    good = np.array([[3, 5, 6, 0]], np.int32)
    bad = good.copy()
    bad[0, 1] = max_pages                     # the second page is out of range
    args = (kpool.data_ptr(), vpool.data_ptr(), max_pages)
    qcache.attn_noalloc_check()               # clean start, whatever ran before
    qcache.attn_decode_noalloc(proj.data_ptr(), *args, dev(bad).data_ptr(), pt_stride, [L],
                               qn.data_ptr(), kn.data_ptr(), rope_c.data_ptr(),
                               rope_s.data_ptr(), out.data_ptr())
    with pytest.raises(qcache.QCacheError) as e:
        qcache.attn_noalloc_check()
    assert e.value.code == 5                  # QC_ERR_BOUNDS
    qcache.attn_decode_noalloc(proj.data_ptr(), *args, dev(good).data_ptr(), pt_stride, [L],
                               qn.data_ptr(), kn.data_ptr(), rope_c.data_ptr(),
                               rope_s.data_ptr(), out.data_ptr())
    qcache.attn_noalloc_check()
