"""Split-K long-context decode across two GPUs with the records exchanged
through peer memory (qc_p2p_* in include/qcache.h): each rank's output must
equal, bit for bit, the merge of the same records gathered on the host and
combined with qc_attn_combine.  Three steps, so both mailbox parities and the
arrival counters' growth are exercised.  Needs two GPUs; skipped otherwise."""
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _rank(rank, world, port, result_dir):
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from conftest import load_pkg_module
    qc = load_pkg_module("qcache")
    synth = load_pkg_module("synth")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ctx = 64 * 40 + 17
    q = qc.QCache(n_attn_layers=1, n_gdn_layers=1, max_seqs=1, max_pages=64, max_ctx=ctx + 64,
                  max_batch=1, max_snapshots=1, device=rank)
    a = synth.attn_inputs(5, 1, ctx)
    q.set_attn_params(0, a["q_norm"], a["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, ctx)
    k = torch.from_numpy(a["k"][0].view(np.int16)).cuda()
    v = torch.from_numpy(a["v"][0].view(np.int16)).cuda()
    q.kv_write(s, 0, 0, ctx, k.data_ptr(), v.data_ptr())
    torch.cuda.synchronize()
    handle = q.p2p_create(world, rank)
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    for r in range(world):
        if r != rank:
            q.p2p_open(r, handles[r])
    pages = ctx // 64 + 1
    cuts = [r * pages // world for r in range(world)]
    proj = torch.from_numpy(synth.bf16_bits(synth.normal(9, (3, 10240))).view(np.int16)).cuda()
    rec = torch.zeros(16, 258, device="cuda")
    out_p2p = torch.zeros(4096, dtype=torch.int16, device="cuda")
    out_ref = torch.zeros(4096, dtype=torch.int16, device="cuda")
    ok = []
    for step in range(3):
        q.decode_begin([s])
        pos = q.seq_len(s)
        end = cuts[rank + 1] if rank + 1 < world else pos // 64 + 1
        q.attn_partial_range(cuts[rank], end, int(rank == world - 1))
        p = proj[step].data_ptr()
        q.attn_partial_p2p(0, p)
        q.attn_combine_p2p(0, p, out_p2p.data_ptr())
        q.attn_partial(0, p, rec.data_ptr())        # the same record, the host way
        torch.cuda.synchronize()
        recs = [torch.zeros(16, 258) for _ in range(world)]
        dist.all_gather(recs, rec.cpu())
        g = torch.stack(recs).cuda()
        q.attn_combine(g.data_ptr(), world, p, out_ref.data_ptr())
        q.decode_end()
        q.check_device()
        ok.append(bool(torch.equal(out_p2p, out_ref)) and bool(out_ref.abs().sum() > 0))
        dist.barrier()
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write(" ".join(str(int(x)) for x in ok))
    dist.barrier()
    q.close()
    dist.destroy_process_group()


def test_p2p_split_matches_host_merge(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    port = 29600 + os.getpid() % 300
    mp.spawn(_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert open(tmp_path / f"rank{r}").read().split() == ["1", "1", "1"], r


def _rank_withhold(rank, world, port, result_dir, n_dev):
    """Rank 1 withholds its record for one step (a host-side fault: the rank
    skips a layer).  Rank 0's merge must give up after its bounded wait,
    report QC_ERR_TIMEOUT naming the merge kernel and layer, leave its output
    untouched, and refuse later merges until every rank has reset its
    mailbox.  With two GPUs the ranks then run a good step together; with one
    GPU they stop after the reset, because two ranks whose kernels wait on
    each other must not share a GPU."""
    import time

    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from conftest import load_pkg_module
    qc = load_pkg_module("qcache")
    synth = load_pkg_module("synth")
    dev = rank % n_dev
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    ctx = 64 * 8 + 3
    q = qc.QCache(n_attn_layers=2, n_gdn_layers=1, max_seqs=1, max_pages=16, max_ctx=ctx + 64,
                  max_batch=1, max_snapshots=1, device=dev)
    a = synth.attn_inputs(6, 1, ctx)
    for layer in range(2):
        q.set_attn_params(layer, a["q_norm"], a["k_norm"])
    s = q.seq_alloc()
    q.seq_reserve(s, ctx)
    k = torch.from_numpy(a["k"][0].view(np.int16)).cuda()
    v = torch.from_numpy(a["v"][0].view(np.int16)).cuda()
    for layer in range(2):
        q.kv_write(s, layer, 0, ctx, k.data_ptr(), v.data_ptr())
    torch.cuda.synchronize()
    handles = [None] * world
    dist.all_gather_object(handles, q.p2p_create(world, rank))
    for r in range(world):
        if r != rank:
            q.p2p_open(r, handles[r])
    pages = ctx // 64 + 1
    cuts = [r * pages // world for r in range(world)] + [pages]
    proj = torch.from_numpy(synth.bf16_bits(synth.normal(11, (10240,))).view(np.int16)).cuda()
    res = {}
    sentinel = torch.full((4096,), 0x7777, dtype=torch.int16, device="cuda")
    out = sentinel.clone()

    def open_step():
        q.decode_begin([s])
        q.attn_partial_range(cuts[rank], cuts[rank + 1], int(rank == world - 1))

    open_step()
    if rank == 0:
        q.attn_partial_p2p(1, proj.data_ptr())
        t0 = time.time()
        q.attn_combine_p2p(1, proj.data_ptr(), out.data_ptr())
        try:
            q.check_device()
            res["code"] = 0
        except qc.QCacheError as e:
            res["code"], res["msg"] = e.code, str(e)
        res["wait_s"] = time.time() - t0
        res["untouched"] = bool(torch.equal(out, sentinel))
        try:
            q.attn_combine_p2p(1, proj.data_ptr(), out.data_ptr())
            res["refused"] = 0
        except qc.QCacheError as e:
            res["refused"] = e.code
    q.decode_abort()
    torch.cuda.synchronize()
    dist.barrier()
    q.p2p_reset()
    dist.barrier()
    res["after_reset"] = -1
    if n_dev >= world:
        open_step()
        q.attn_partial_p2p(1, proj.data_ptr())
        q.attn_combine_p2p(1, proj.data_ptr(), out.data_ptr())
        q.decode_abort()
        q.check_device()
        rec = torch.zeros(16, 258, device="cuda")
        open_step()
        q.attn_partial(1, proj.data_ptr(), rec.data_ptr())
        torch.cuda.synchronize()
        recs = [torch.zeros(16, 258) for _ in range(world)]
        dist.all_gather(recs, rec.cpu())
        ref = torch.zeros(4096, dtype=torch.int16, device="cuda")
        q.attn_combine(torch.stack(recs).cuda().data_ptr(), world, proj.data_ptr(), ref.data_ptr())
        q.decode_abort()
        q.check_device()
        res["after_reset"] = int(torch.equal(out, ref))
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write(repr(res))
    dist.barrier()
    q.close()
    dist.destroy_process_group()


def test_withheld_record_times_out_and_reset_recovers(tmp_path):
    import ast

    import torch.multiprocessing as mp
    n_dev = torch.cuda.device_count()
    port = 29900 + os.getpid() % 90
    mp.spawn(_rank_withhold, args=(2, port, str(tmp_path), n_dev), nprocs=2, join=True)
    r0 = ast.literal_eval(open(tmp_path / "rank0").read())
    assert r0["code"] == 4, r0                       # QC_ERR_TIMEOUT
    assert "merge" in r0["msg"] and "layer 1" in r0["msg"], r0
    assert 0.9 <= r0["wait_s"] < 30, r0              # bounded at 1 s
    assert r0["untouched"], r0
    assert r0["refused"] == 1, r0                    # QC_ERR_ARG until reset
    if n_dev >= 2:
        for r in range(2):
            assert ast.literal_eval(open(tmp_path / f"rank{r}").read())["after_reset"] == 1, r
