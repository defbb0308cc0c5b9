"""GPU parity at the benchmark configurations themselves, through the C ABI,
against the oracle (the scalar restatement of src/engine.cpp:3204-3327 and
:3485-3564):

- config 2: the full 32-layer stack (24 DeltaNet + 8 attention, attention at
  every 4th layer), 64 sequences at context 4096, pages mapped in a seeded
  random interleaving, one decode step; every attention output and append of
  every sequence, and a rotating sample of 16 sequences per DeltaNet layer
  (outputs and the fp32 state);
- config 4: one attention layer at context 131072, whole and split into 2, 4
  and 8 page ranges merged through qc_attn_partial / qc_attn_combine;
- config 3 at its sizes: 24 DeltaNet + 8 attention layers, prefixes of 512 to
  3584 tokens (and lengths that are not multiples of 64), bit-exact restore
  of every layer and decode-after-restore identical to the original;
- reset_state (src/engine.cpp:4164-4176): after qc_seq_reset, or a
  qc_seq_match_prefix that diverges, the state and conv history read back as
  zeros and the next decode matches the oracle from zero state.

Inputs are generated on the device from seeded torch generators and read
back for the oracle, so the sizes need no host-side generation."""
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from gpu_util import (assert_out_close, assert_state_close, empty_u16, host_f32,  # noqa: E402
                      host_u16)

BF16 = torch.bfloat16


def u16(t):
    """Device bf16/int16 tensor -> host uint16 bit patterns."""
    torch.cuda.synchronize()
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def rand_bf16(g, *shape, scale=1.0):
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(BF16)


def interleaved_reserve(q, seqs, ctx, seed):
    """Map each sequence's pages in a seeded random interleaving, so logical
    pages land on permuted physical pages."""
    rng = np.random.default_rng(seed)
    need = {s: (ctx + 63) // 64 for s in seqs}
    have = {s: 0 for s in seqs}
    live = list(seqs)
    while live:
        s = live[int(rng.integers(len(live)))]
        have[s] += 1
        q.seq_reserve(s, min(ctx, have[s] * 64))
        if have[s] == need[s]:
            live.remove(s)


def stack_kinds():
    return ["a" if (l + 1) % 4 == 0 else "g" for l in range(32)]


def test_config2_full_stack_one_step(qcache, synth, oracle):
    n, ctx = 64, 4096
    kinds = stack_kinds()
    q = qcache.QCache(n_attn_layers=8, n_gdn_layers=24, max_seqs=n, max_pages=n * 65,
                      max_ctx=ctx + 64, max_batch=n, max_snapshots=1, device=0)
    aparams = [synth.attn_inputs(500 + l, 1, 0) for l in range(8)]
    gparams = [synth.gdn_params(600 + l) for l in range(24)]
    for l in range(8):
        q.set_attn_params(l, aparams[l]["q_norm"], aparams[l]["k_norm"])
    for l in range(24):
        p = gparams[l]
        q.set_gdn_params(l, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    seqs = [q.seq_alloc() for _ in range(n)]
    interleaved_reserve(q, seqs, ctx, seed=2)
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    for s in seqs:
        for l in range(8):
            k, v = rand_bf16(g, ctx, 4, 256), rand_bf16(g, ctx, 4, 256)
            q.kv_write(s, l, 0, ctx, k.data_ptr(), v.data_ptr())
        for l in range(24):
            st = torch.randn(32, 128, 128, generator=g, device="cuda") * 0.02
            hi = rand_bf16(g, 3, 8192)
            q.gdn_state_write(s, l, st.data_ptr(), hi.data_ptr())
        torch.cuda.synchronize()
    # DeltaNet sample: 16 sequences per layer, rotating so every sequence is
    # checked in 6 layers; their state and history before the step
    rng = np.random.default_rng(3)
    order = rng.permutation(n)
    gsample = {gl: sorted(order[(16 * gl) % n:(16 * gl) % n + 16].tolist()) for gl in range(24)}
    before = {}
    st_d, hi_d = torch.empty(32, 128, 128, device="cuda"), empty_u16(3, 8192)
    for gl in range(24):
        for b in gsample[gl]:
            q.gdn_state_read(seqs[b], gl, st_d.data_ptr(), hi_d.data_ptr())
            before[(gl, b)] = (host_f32(st_d).copy(), host_u16(hi_d).copy())
    projs = [rand_bf16(g, n, 10240 if kd == "a" else 12352) for kd in kinds]
    outs = [empty_u16(n, 4096) for _ in kinds]
    q.decode_begin(seqs)
    ai = gi = 0
    for layer, kd in enumerate(kinds):
        if kd == "a":
            q.attn_decode(ai, projs[layer].data_ptr(), outs[layer].data_ptr())
            ai += 1
        else:
            q.gdn_decode(gi, projs[layer].data_ptr(), outs[layer].data_ptr())
            gi += 1
    q.decode_end()
    q.check_device()
    assert all(q.seq_len(s) == ctx + 1 for s in seqs)

    pool = ThreadPoolExecutor(8)
    attn_layers = [l for l, kd in enumerate(kinds) if kd == "a"]
    gdn_layers = [l for l, kd in enumerate(kinds) if kd == "g"]
    kd_, vd_ = empty_u16(ctx + 1, 4, 256), empty_u16(ctx + 1, 4, 256)
    for al, layer in enumerate(attn_layers):
        proj = u16(projs[layer])
        got = u16(outs[layer])
        jobs = []
        for b, s in enumerate(seqs):
            q.kv_read(s, al, 0, ctx + 1, kd_.data_ptr(), vd_.data_ptr())
            kc, vc = u16(kd_).copy(), u16(vd_).copy()
            appended = (kc[ctx].copy(), vc[ctx].copy())
            jobs.append((b, appended, kc, vc,
                         pool.submit(oracle.attn_decode, proj[b], aparams[al]["q_norm"],
                                     aparams[al]["k_norm"], ctx, kc, vc)))
        for b, appended, kc, vc, fut in jobs:
            ref = fut.result()
            # the oracle rewrote row ctx with its own append: bit-exact
            np.testing.assert_array_equal(appended[0], kc[ctx], err_msg=f"K append seq {b}")
            np.testing.assert_array_equal(appended[1], vc[ctx], err_msg=f"V append seq {b}")
            assert_out_close(got[b], ref, synth)
    for gl, layer in enumerate(gdn_layers):
        proj = u16(projs[layer])
        got = u16(outs[layer])
        jobs = []
        for b in gsample[gl]:
            st, hi = before[(gl, b)]
            st = st.copy()
            hist = synth.bf16_to_f32(hi).copy()
            jobs.append((b, st, hist, pool.submit(oracle.gdn_decode, proj[b], st, hist,
                                                  gparams[gl])))
        for b, st, hist, fut in jobs:
            ref = fut.result()
            assert_out_close(got[b], ref, synth)
            q.gdn_state_read(seqs[b], gl, st_d.data_ptr(), hi_d.data_ptr())
            assert_state_close(host_f32(st_d), st)
            np.testing.assert_array_equal(synth.bf16_to_f32(host_u16(hi_d)), hist)
    pool.shutdown()
    q.close()


def test_config4_long_context_whole_and_split(qcache, synth, oracle):
    L = 131072
    q = qcache.QCache(n_attn_layers=1, n_gdn_layers=1, max_seqs=1, max_pages=L // 64 + 1,
                      max_ctx=L + 64, max_batch=1, max_snapshots=1, device=0)
    a = synth.attn_inputs(700, 1, 0)
    q.set_attn_params(0, a["q_norm"], a["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, L)
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    k, v = rand_bf16(g, L, 4, 256), rand_bf16(g, L, 4, 256)
    q.kv_write(s, 0, 0, L, k.data_ptr(), v.data_ptr())
    kc = np.zeros((L + 1, 4, 256), np.uint16)
    vc = np.zeros((L + 1, 4, 256), np.uint16)
    kc[:L], vc[:L] = u16(k), u16(v)
    del k, v
    proj_h = u16(rand_bf16(g, 1, 10240))
    proj = torch.from_numpy(proj_h.view(np.int16)).cuda()
    ref = oracle.attn_decode(proj_h[0], a["q_norm"], a["k_norm"], L, kc, vc)
    n_pages = L // 64 + 1          # the last page holds only the new position
    for G in (2, 4, 8):
        cuts = [i * (L // 64) // G for i in range(G)] + [n_pages]
        parts = torch.zeros(G, 16, 258, device="cuda")
        q.decode_begin([s])
        for r in range(G):
            q.attn_partial_range(cuts[r], cuts[r + 1], int(r == G - 1))
            q.attn_partial(0, proj.data_ptr(), parts[r].data_ptr())
        out = empty_u16(1, 4096)
        q.attn_combine(parts.data_ptr(), G, proj.data_ptr(), out.data_ptr())
        q.decode_abort()
        q.check_device()
        assert_out_close(host_u16(out)[0], ref, synth)
    out = empty_u16(1, 4096)
    q.decode_begin([s])
    q.attn_decode(0, proj.data_ptr(), out.data_ptr())
    q.decode_end()
    q.check_device()
    assert_out_close(host_u16(out)[0], ref, synth)
    kd_, vd_ = empty_u16(1, 4, 256), empty_u16(1, 4, 256)
    q.kv_read(s, 0, L, 1, kd_.data_ptr(), vd_.data_ptr())
    np.testing.assert_array_equal(host_u16(kd_)[0], kc[L])
    np.testing.assert_array_equal(host_u16(vd_)[0], vc[L])
    q.close()


def _stack_ctx(qcache, synth, n_seqs, max_pages, max_ctx, snaps):
    q = qcache.QCache(n_attn_layers=8, n_gdn_layers=24, max_seqs=n_seqs, max_pages=max_pages,
                      max_ctx=max_ctx, max_batch=n_seqs, max_snapshots=snaps, device=0)
    ap = [synth.attn_inputs(800 + l, 1, 0) for l in range(8)]
    gp = [synth.gdn_params(900 + l) for l in range(24)]
    for l in range(8):
        q.set_attn_params(l, ap[l]["q_norm"], ap[l]["k_norm"])
    for l in range(24):
        q.set_gdn_params(l, gp[l]["ssm_a"], gp[l]["dt_bias"], gp[l]["ssm_norm"], gp[l]["conv_w"])
    return q, ap, gp


def _read_seq(q, s, P):
    """Every layer of a sequence, as device tensors (compared on the device)."""
    kv, st = [], []
    for l in range(8):
        k, v = empty_u16(max(P, 1), 4, 256), empty_u16(max(P, 1), 4, 256)
        if P:
            q.kv_read(s, l, 0, P, k.data_ptr(), v.data_ptr())
        kv.append((k, v))
    for l in range(24):
        a, h = torch.empty(32, 128, 128, device="cuda"), empty_u16(3, 8192)
        q.gdn_state_read(s, l, a.data_ptr(), h.data_ptr())
        st.append((a, h))
    torch.cuda.synchronize()
    return kv, st


def _decode_stack(q, seqs, projs):
    n = len(seqs)
    outs = []
    q.decode_begin(seqs)
    ai = gi = 0
    for layer, kd in enumerate(stack_kinds()):
        o = empty_u16(n, 4096)
        if kd == "a":
            q.attn_decode(ai, projs[layer].data_ptr(), o.data_ptr())
            ai += 1
        else:
            q.gdn_decode(gi, projs[layer].data_ptr(), o.data_ptr())
            gi += 1
        outs.append(o)
    q.decode_end()
    q.check_device()
    return outs


def test_config3_prefix_restore_at_full_sizes(qcache, synth, oracle):
    """16 prefixes at config-3 lengths (the endpoints 512 and 3584 and lengths
    that are not multiples of 64), 32 requests restored in one batched call;
    every layer of every request bit-exact; then one decode of all requests
    and of their source sequences, identical outputs; one request per prefix
    length class checked against the oracle."""
    rng = np.random.default_rng(33)
    P_list = [512, 3584, 1000, 2049] + [int(x) for x in rng.integers(512, 3585, 12)]
    n_pref, n_req = len(P_list), 32
    max_pages = sum(P // 64 + 2 for P in P_list) + n_req * 3 + 64
    q, ap, gp = _stack_ctx(qcache, synth, n_pref + n_req, max_pages, 3584 + 128, n_pref)
    g = torch.Generator(device="cuda")
    g.manual_seed(33)
    src, entries, toks = [], [], []
    for i, P in enumerate(P_list):
        s = q.seq_alloc()
        q.seq_reserve(s, P)
        for l in range(8):
            k, v = rand_bf16(g, P, 4, 256), rand_bf16(g, P, 4, 256)
            q.kv_write(s, l, 0, P, k.data_ptr(), v.data_ptr())
        for l in range(24):
            st = torch.randn(32, 128, 128, generator=g, device="cuda") * 0.02
            q.gdn_state_write(s, l, st.data_ptr(), rand_bf16(g, 3, 8192).data_ptr())
        torch.cuda.synchronize()
        t = [int(x) for x in rng.integers(0, 248320, P)]
        toks.append(t)
        entries.append(q.prefix_insert(s, t))
        src.append(s)
    pick = [int(x) for x in rng.integers(0, n_pref, n_req)]
    pick[:4] = [0, 1, 2, 3]
    want = []
    for i in pick:
        suffix = [int(x) for x in rng.integers(0, 248320, int(rng.integers(1, 65)))]
        m, e = q.prefix_lookup(toks[i] + suffix)
        assert (m, e) == (P_list[i], entries[i])
        want.append(e)
    reqs = [q.seq_alloc() for _ in range(n_req)]
    q.prefix_restore(want, reqs)
    q.check_device()
    ref_layers = {i: _read_seq(q, src[i], P_list[i]) for i in set(pick)}
    for r, i in zip(reqs, pick):
        assert q.seq_len(r) == P_list[i]
        kv, st = _read_seq(q, r, P_list[i])
        rkv, rst = ref_layers[i]
        for l in range(8):
            assert torch.equal(kv[l][0], rkv[l][0]) and torch.equal(kv[l][1], rkv[l][1]), (r, l)
        for l in range(24):
            assert torch.equal(st[l][0], rst[l][0]) and torch.equal(st[l][1], rst[l][1]), (r, l)
    del ref_layers
    # decode after restore: the four distinct-length requests, then their
    # sources, as two batches of the same layout (the split-K partition of an
    # attention batch depends on the batch's lengths and order, so equal
    # layouts give bit-identical outputs)
    projs = [rand_bf16(g, 4, 10240 if kd == "a" else 12352) for kd in stack_kinds()]
    # oracle inputs of request 2 (P = 1000) in attention layer 0 and DeltaNet layer 0
    P = P_list[2]
    kd_, vd_ = empty_u16(P + 1, 4, 256), empty_u16(P + 1, 4, 256)
    q.kv_read(reqs[2], 0, 0, P, kd_.data_ptr(), vd_.data_ptr())
    kc, vc = u16(kd_).copy(), u16(vd_).copy()
    st_d, hi_d = torch.empty(32, 128, 128, device="cuda"), empty_u16(3, 8192)
    q.gdn_state_read(reqs[2], 0, st_d.data_ptr(), hi_d.data_ptr())
    st0, hist0 = host_f32(st_d).copy(), synth.bf16_to_f32(host_u16(hi_d)).copy()
    outs = _decode_stack(q, reqs[:4], projs)
    outs_src = _decode_stack(q, [src[i] for i in pick[:4]], projs)
    for layer, (o, o2) in enumerate(zip(outs, outs_src)):
        np.testing.assert_array_equal(u16(o), u16(o2), err_msg=f"layer {layer}")
    ref_a = oracle.attn_decode(u16(projs[3])[2], ap[0]["q_norm"], ap[0]["k_norm"], P, kc, vc)
    assert_out_close(u16(outs[3])[2], ref_a, synth)
    ref_g = oracle.gdn_decode(u16(projs[0])[2], st0, hist0, gp[0])
    assert_out_close(u16(outs[0])[2], ref_g, synth)
    q.close()


@pytest.mark.parametrize("how", ["seq_reset", "match_prefix"])
def test_reset_zeroes_state_and_decodes_from_zero(qcache, synth, oracle, how):
    q, ap, gp = _stack_ctx(qcache, synth, 2, 64, 1024, 1)
    s = q.seq_alloc()
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    L = 70
    q.seq_reserve(s, L)
    for l in range(8):
        q.kv_write(s, l, 0, L, rand_bf16(g, L, 4, 256).data_ptr(),
                   rand_bf16(g, L, 4, 256).data_ptr())
    for l in range(24):
        st = torch.randn(32, 128, 128, generator=g, device="cuda") * 0.02
        q.gdn_state_write(s, l, st.data_ptr(), rand_bf16(g, 3, 8192).data_ptr())
    projs = [rand_bf16(g, 1, 10240 if kd == "a" else 12352) for kd in stack_kinds()]
    _decode_stack(q, [s], projs)           # one step with history recorded
    if how == "seq_reset":
        q.seq_reset(s)
    else:
        # the history was stood up without token ids, so no prompt matches
        # it: the rule resets the sequence (src/engine.cpp:4066-4070)
        assert q.match_prefix(s, [2, 3, 4]) == 0
    assert q.seq_len(s) == 0 and q.seq_pages(s) == []
    kv, st = _read_seq(q, s, 0)
    for a, h in st:
        assert not torch.any(a != 0) and not torch.any(h != 0)
    projs = [rand_bf16(g, 1, 10240 if kd == "a" else 12352) for kd in stack_kinds()]
    outs = _decode_stack(q, [s], projs)
    for layer, kd in enumerate(stack_kinds()):
        proj = u16(projs[layer])[0]
        if kd == "a":
            al = (layer + 1) // 4 - 1
            kc, vc = np.zeros((1, 4, 256), np.uint16), np.zeros((1, 4, 256), np.uint16)
            ref = oracle.attn_decode(proj, ap[al]["q_norm"], ap[al]["k_norm"], 0, kc, vc)
        else:
            gl = layer - (layer + 1) // 4
            ref = oracle.gdn_decode(proj, np.zeros((32, 128, 128), np.float32),
                                    np.zeros((3, 8192), np.float32), gp[gl])
        assert_out_close(u16(outs[layer])[0], ref, synth)
    q.close()
