"""CPU tests of the C ABI: the library loads and exports every declared symbol,
and the host logic (page allocator, sequences, decode bookkeeping, prefix
table) behaves on a host-only context.  No compute happens here."""
import ctypes as C

import pytest


def host_ctx(qcache, **kw):
    args = dict(n_attn_layers=8, n_gdn_layers=24, max_seqs=8, max_pages=64, max_ctx=4096,
                max_batch=8, max_snapshots=4, device=qcache.DEVICE_NONE)
    args.update(kw)
    return qcache.QCache(**args)


def test_library_exports_every_header_symbol(qcache):
    L = qcache.lib()
    names = qcache.header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n


def test_attention_kernel_selection(qcache):
    """The process-wide kernel choice: auto by default, either kernel forced,
    unknown modes refused without changing it."""
    prev = qcache.attn_select_kernel(qcache.ATTN_KERNEL_TC)
    try:
        assert prev == qcache.ATTN_KERNEL_AUTO
        assert qcache.attn_select_kernel(qcache.ATTN_KERNEL_MMA) == qcache.ATTN_KERNEL_TC
        with pytest.raises(qcache.QCacheError):
            qcache.attn_select_kernel(7)
        assert qcache.attn_select_kernel(qcache.ATTN_KERNEL_AUTO) == qcache.ATTN_KERNEL_MMA
    finally:
        qcache.attn_select_kernel(qcache.ATTN_KERNEL_AUTO)


def test_create_rejects_bad_config(qcache):
    with pytest.raises(qcache.QCacheError):
        qcache.QCache(max_seqs=0, device=qcache.DEVICE_NONE)
    with pytest.raises(qcache.QCacheError):
        qcache.QCache(max_batch=9, max_seqs=8, device=qcache.DEVICE_NONE)
    with pytest.raises(qcache.QCacheError):  # unknown flag bits
        qcache.QCache(max_seqs=8, max_batch=8, device=qcache.DEVICE_NONE, flags=2)
    host_ctx(qcache, flags=qcache.QC_FLAG_REFERENCE_MATH).close()


def test_device_calls_fail_loudly_on_host_only(qcache):
    q = host_ctx(qcache)
    s = q.seq_alloc()
    q.decode_begin([s])
    with pytest.raises(qcache.QCacheError) as e:
        q.attn_decode(0, 16, 16)
    assert e.value.code == qcache.QC_ERR_NODEVICE
    with pytest.raises(qcache.QCacheError) as e:
        q.gdn_decode(0, 16, 16)
    assert e.value.code == qcache.QC_ERR_NODEVICE
    with pytest.raises(qcache.QCacheError) as e:
        q.p2p_create(2, 0)
    assert e.value.code == qcache.QC_ERR_NODEVICE
    with pytest.raises(qcache.QCacheError) as e:
        q.attn_combine_p2p(0, 16, 16)
    assert e.value.code == qcache.QC_ERR_NODEVICE


def test_sequence_slots_and_pages(qcache):
    q = host_ctx(qcache, max_seqs=2, max_batch=2, max_pages=4)
    a, b = q.seq_alloc(), q.seq_alloc()
    with pytest.raises(qcache.QCacheError) as e:
        q.seq_alloc()
    assert e.value.code == qcache.QC_ERR_OOM
    q.seq_reserve(a, 130)                     # 3 pages
    assert q.seq_len(a) == 130 and len(q.seq_pages(a)) == 3
    with pytest.raises(qcache.QCacheError) as e:
        q.seq_reserve(b, 65)                  # needs 2, only 1 left
    assert e.value.code == qcache.QC_ERR_OOM
    assert q.seq_pages(b) == []               # rolled back
    q.seq_free(a)
    q.seq_reserve(b, 256)
    assert len(set(q.seq_pages(b))) == 4


def test_decode_maps_a_page_at_each_boundary(qcache):
    q = host_ctx(qcache)
    s = q.seq_alloc()
    for t in range(130):
        q.decode_begin([s], tokens=[t])
        q.decode_end()
        assert len(q.seq_pages(s)) == t // 64 + 1
    assert q.seq_len(s) == 130


def test_decode_step_protocol(qcache):
    q = host_ctx(qcache)
    s = q.seq_alloc()
    with pytest.raises(qcache.QCacheError):
        q.decode_end()
    q.decode_begin([s])
    with pytest.raises(qcache.QCacheError):
        q.decode_begin([s])
    q.decode_end()
    with pytest.raises(qcache.QCacheError):
        q.decode_begin([s, s])
    with pytest.raises(qcache.QCacheError):
        q.decode_begin([5])                   # not allocated


def test_match_prefix_follows_reference_rule(qcache):
    q = host_ctx(qcache)
    s = q.seq_alloc()
    for t in [1, 2, 3]:
        q.decode_begin([s], tokens=[t])
        q.decode_end()
    assert q.match_prefix(s, [1, 2, 3, 4, 5]) == 3       # reuse, prefill 4, 5
    assert q.seq_len(s) == 3
    assert q.match_prefix(s, [1, 2, 3]) == 0             # fully cached -> reset
    assert q.seq_len(s) == 0 and q.seq_pages(s) == []
    for t in [1, 2, 3]:
        q.decode_begin([s], tokens=[t])
        q.decode_end()
    assert q.match_prefix(s, [1, 9, 3, 4]) == 0          # diverged -> reset
    assert q.seq_len(s) == 0


def test_page_hashes_chain(qcache):
    toks = list(range(200))
    h = qcache.page_hashes(toks)
    assert len(h) == 3 and len(set(h)) == 3
    assert qcache.page_hashes(toks[:128]) == h[:2]
    toks2 = list(toks)
    toks2[5] = 999
    h2 = qcache.page_hashes(toks2)
    assert all(a != b for a, b in zip(h, h2))            # chained: all later pages differ


def test_prefix_insert_lookup_restore_refcounts(qcache):
    q = host_ctx(qcache, max_pages=32)
    s = q.seq_alloc()
    prefix = list(range(1000, 1000 + 150))               # 2 full pages + tail of 22
    q.seq_reserve(s, 150)
    e = q.prefix_insert(s, prefix)
    pages_s = q.seq_pages(s)
    assert q.prefix_lookup(prefix + [7, 8]) == (150, e)
    assert q.prefix_lookup(prefix) == (0, -1)            # P must be < n
    assert q.prefix_lookup(prefix[:149] + [5, 6]) == (0, -1)
    other = list(prefix)
    other[100] = 1
    assert q.prefix_lookup(other + [1]) == (0, -1)       # token ids verified
    t = q.seq_alloc()
    q.prefix_restore([e], [t])
    pt = q.seq_pages(t)
    assert q.seq_len(t) == 150 and len(pt) == 3
    assert pt[:2] == pages_s[:2]                         # full pages shared
    assert pt[2] != pages_s[2]                           # tail copied
    # a decode on t writes into its own tail page; full pages stay shared
    q.decode_begin([t])
    q.decode_end()
    assert q.seq_pages(t) == pt
    q.prefix_release(e)
    assert q.prefix_lookup(prefix + [7]) == (0, -1)
    q.seq_free(s)
    q.seq_free(t)
    # every page returned: a full reservation succeeds again
    u = q.seq_alloc()
    q.seq_reserve(u, 32 * 64)


def test_longest_prefix_wins(qcache):
    q = host_ctx(qcache, max_pages=64)
    base = list(range(300))
    ids = []
    for n in (70, 200, 64):
        s = q.seq_alloc()
        q.seq_reserve(s, n)
        ids.append((n, q.prefix_insert(s, base[:n])))
    assert q.prefix_lookup(base + [1]) == (200, ids[1][1])
    assert q.prefix_lookup(base[:150]) == (70, ids[0][1])
    assert q.prefix_lookup(base[:66]) == (64, ids[2][1])
    assert q.prefix_lookup(base[:64]) == (0, -1) or q.prefix_lookup(base[:64])[0] < 64


def test_restore_requires_empty_sequence(qcache):
    q = host_ctx(qcache)
    s = q.seq_alloc()
    q.seq_reserve(s, 10)
    e = q.prefix_insert(s, list(range(10)))
    with pytest.raises(qcache.QCacheError):
        q.prefix_restore([e], [s])                       # s is not empty
    with pytest.raises(qcache.QCacheError):
        q.prefix_restore([e + 5], [q.seq_alloc()])       # no such entry


def test_prefill_bookkeeping(qcache):
    q = host_ctx(qcache)
    s = q.seq_alloc()
    q.prefill_begin(s, 32, tokens=list(range(32)))
    with pytest.raises(qcache.QCacheError):
        q.decode_begin([s])                          # one open step at a time
    q.prefill_end()
    q.prefill_begin(s, 32, tokens=list(range(32, 64)))
    q.prefill_end()
    q.prefill_begin(s, 1, tokens=[64])
    q.prefill_end()
    assert q.seq_len(s) == 65 and len(q.seq_pages(s)) == 2
    assert q.match_prefix(s, list(range(65)) + [7]) == 65
    with pytest.raises(qcache.QCacheError):
        q.prefill_begin(s, 33)                       # chunk limit



def _two_boundary_sequences_one_free_page(qcache):
    """u, v: 128 tokens each (the next token of each needs a fresh page); the
    pool left with exactly one free page."""
    q = host_ctx(qcache, max_pages=32)
    u, v = q.seq_alloc(), q.seq_alloc()
    q.seq_reserve(u, 128)
    q.seq_reserve(v, 128)
    w = q.seq_alloc()
    q.seq_reserve(w, 27 * 64)                            # 32 - 2 - 2 - 27 = 1 free
    return q, u, v


def test_decode_oom_leaves_every_sequence_unchanged(qcache):
    """Two pages needed, one free: the step fails before any sequence of the
    batch takes a page, and the single page still serves a one-sequence step."""
    q, u, v = _two_boundary_sequences_one_free_page(qcache)
    before = (q.seq_pages(u), q.seq_pages(v))
    with pytest.raises(qcache.QCacheError) as e:
        q.decode_begin([u, v])
    assert e.value.code == qcache.QC_ERR_OOM
    assert (q.seq_pages(u), q.seq_pages(v)) == before
    q.decode_begin([v])
    q.decode_end()
    assert len(q.seq_pages(v)) == 3 and q.seq_pages(u) == before[0]


def test_prefill_oom_leaves_sequence_unchanged(qcache):
    """A chunk that crosses into two new pages with one free fails and leaves
    the sequence's pages as they were; a chunk inside one new page fits."""
    q, u, _ = _two_boundary_sequences_one_free_page(qcache)
    before = q.seq_pages(u)
    q.prefill_begin(u, 32)                               # positions 128..159: one page
    q.prefill_end()
    assert len(q.seq_pages(u)) == 3
    q2, u2, _ = _two_boundary_sequences_one_free_page(qcache)
    q2.seq_reserve(u2, 160)                              # takes the free page
    before = q2.seq_pages(u2)
    with pytest.raises(qcache.QCacheError) as e:
        q2.prefill_begin(u2, 32)                         # 160..191 fits; 192 would not
        q2.prefill_end()
        q2.prefill_begin(u2, 1)
    assert e.value.code == qcache.QC_ERR_OOM
    assert q2.seq_pages(u2) == before


def test_snapshot_slots_exhaust_and_return(qcache):
    """Every entry holds one DeltaNet/conv snapshot slot: inserts beyond
    max_snapshots fail with QC_ERR_OOM until an entry is released; releasing
    every entry returns every page reference."""
    q = host_ctx(qcache, max_pages=32, max_snapshots=2)
    seqs = [q.seq_alloc() for _ in range(3)]
    for i, s in enumerate(seqs):
        q.seq_reserve(s, 70 + i)                         # one full page + a tail
    e0 = q.prefix_insert(seqs[0], list(range(70)))
    e1 = q.prefix_insert(seqs[1], list(range(100, 171)))
    with pytest.raises(qcache.QCacheError) as e:
        q.prefix_insert(seqs[2], list(range(200, 272)))
    assert e.value.code == qcache.QC_ERR_OOM
    q.prefix_release(e0)
    e2 = q.prefix_insert(seqs[2], list(range(200, 272)))
    for ent in (e1, e2):
        q.prefix_release(ent)
    for s in seqs:
        q.seq_free(s)
    u = q.seq_alloc()
    q.seq_reserve(u, 32 * 64)                            # every page is free again
