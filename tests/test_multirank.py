"""World-size-2 gloo tests (CPU) of the multi-GPU host protocols:
- independent sequences are sharded contiguously with no exchange;
- the long-context split-K exchange: each rank computes the (m, l, o) record
  of its position range, records are all-gathered, every rank merges them to
  the same output as a one-pass decode;
- a rank that fails before the exchange is detected by the others through the
  process group's timeout, not by a hang."""
import datetime
import os
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))


def shard(n_total, world, rank):
    """Contiguous sequence shard of a rank (bench.py's partition)."""
    per = n_total // world
    return list(range(rank * per, (rank + 1) * per))


def _splitk_worker(rank, world, port, q):
    import torch
    _init(rank, world, port)
    from conftest import load_pkg_module
    import oracle
    synth = load_pkg_module("synth")
    L = 300
    d = synth.attn_inputs(123, 1, L)
    kc = np.zeros((L + 1, 4, 256), np.uint16)
    vc = np.zeros((L + 1, 4, 256), np.uint16)
    kc[:L], vc[:L] = d["k"][0], d["v"][0]
    # the rank owning the new position appends it (oracle stands in for the
    # device); positions are split by whole 64-token pages
    kc[L] = oracle.k_append(d["proj"][0][8192:9216], d["k_norm"], L).reshape(4, 256)
    vc[L] = d["proj"][0][9216:10240].reshape(4, 256)
    pages = (L + 1 + 63) // 64
    cut = [0, pages // 2, pages]
    p0, p1 = cut[rank] * 64, min(cut[rank + 1] * 64, L + 1)
    rec = torch.from_numpy(oracle.attn_partial(d["proj"][0], d["q_norm"], L, kc, vc, p0, p1))
    got = [torch.zeros_like(rec) for _ in range(world)]
    dist.all_gather(got, rec)
    merged = oracle.attn_combine(torch.stack(got).numpy(), d["proj"][0])
    kf, vf = kc.copy(), vc.copy()
    full = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], L, kf, vf)
    q.put((rank, float(np.abs(merged - full).max()), shard(64, world, rank)))
    dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    import torch
    _init(rank, world, port, timeout_s=3)
    if rank == 1:
        q.put((rank, "raised"))
        raise SystemExit(0)      # leaves before the exchange
    try:
        dist.all_gather([torch.zeros(4) for _ in range(world)], torch.ones(4))
        q.put((rank, "no error"))
    except Exception as e:       # timeout / connection closed: detected, no hang
        q.put((rank, "detected: " + type(e).__name__))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    ps = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    return sorted(out, key=lambda x: x[0])


def test_splitk_exchange_matches_one_pass():
    res = _run(_splitk_worker)
    for rank, err, sh in res:
        assert err < 1e-4, (rank, err)
    assert res[0][2] == list(range(32)) and res[1][2] == list(range(32, 64))


def test_rank_failure_is_detected_not_hung():
    res = _run(_failing_worker)
    assert res[1][1] == "raised"
    assert res[0][1].startswith("detected"), res[0][1]
