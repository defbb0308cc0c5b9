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
