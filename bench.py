"""Benchmark of the per-token cache path (headline metric: decode cache-path
µs/token/layer and HBM GB/s against 8 TB/s).

Default workload (config 2 of the benchmark configurations): the full 32-layer hybrid cache
stack (24 Gated-DeltaNet + 8 full-attention layers, attention at every 4th
layer), 64 sequences at context 4096 in a paged bf16 KV cache (64-token pages,
seeded random physical page order), one decode token per sequence per step,
sequences sharded over the GPUs (no collective).  Synthetic seeded inputs;
random-init per-layer weights of the real shapes.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

One JSON line on rank 0.  `value` = max-over-ranks device time of one step /
(64 tokens x 32 layers), in µs.  `e2e` = the same metric through the C ABI
with the step's projection inputs copied host->device from pinned memory and
all outputs copied back inside the timed region.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen3.5-9b-bfp8b-1xn300_b200")

N_SEQ, CTX, N_LAYERS = 64, 4096, 32
N_ATTN, N_GDN = 8, 24
HBM_NOMINAL_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0

# algorithmic bytes (HBM roofline; arithmetic intensity << ridge)
GDN_BYTES_PER_SEQ = (2 * 32 * 128 * 128 * 4      # state read + write
                     + 3 * 8192 * 2 + 8192 * 2   # conv ring: 3 taps read, 1 row written (bf16)
                     + 12352 * 2 + 4096 * 2)     # projection row in, output out
GDN_BYTES_PER_LAUNCH = 4 * 8192 * 4 + 32 * 4 * 2 + 128 * 4   # conv weights + small params


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the dominant kernel, per sequence, from single-launch ncu captures of the
# same kernels on smaller cases, scaled by the sequences processed:
PROFILED_TRAFFIC_PER_SEQ = {
    "stack": ("attn", (273.006592e6 + 4.397824e6) / 16,
              "ncu capture of one attention launch over 16 sequences at context 4096, scaled "
              "to the launch's sequences"),
    "long": ("attn", 537.116672e6 + 5.645312e6,
             "ncu capture of one attention launch at context 131072"),
    "gdn": ("gdn", (139.216640e6 + 77.228800e6) / 64,
            "ncu capture of one DeltaNet launch over 64 sequences (part of the state writes "
            "was still in L2 at the launch's end)"),
}


def attn_bytes_per_seq(pos: int) -> int:
    # K and V of the pos cached positions, the appended row, proj in, out
    return 4096 * pos + 4096 + 10240 * 2 + 4096 * 2


def is_attn(layer: int) -> bool:
    return (layer + 1) % 4 == 0   # src/model_config.h:36-38


def load_pkg(name):
    full = "qcache_b200_" + name
    if full in sys.modules:
        return sys.modules[full]
    spec = importlib.util.spec_from_file_location(full, os.path.join(PKG, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[full] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- GPU workload


class Stack:
    """A cache stack for this rank's n sequences on one GPU: `kinds` lists the
    layers in order ("a" attention, "g" DeltaNet)."""

    def __init__(self, qc, synth, torch, kinds, n, ctx, extra_tokens, seed, stream):
        self.torch, self.n, self.ctx, self.kinds = torch, n, ctx, kinds
        self.stream = stream
        n_attn, n_gdn = kinds.count("a"), kinds.count("g")
        pages_per_seq = (ctx + extra_tokens) // 64 + 1
        self.q = qc.QCache(n_attn_layers=n_attn, n_gdn_layers=n_gdn, max_seqs=n,
                           max_pages=n * pages_per_seq, max_ctx=ctx + extra_tokens + 64,
                           max_batch=n, max_snapshots=1, device=torch.cuda.current_device())
        q = self.q
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        for l in range(n_attn):
            a = synth.attn_inputs(seed + l, 1, 0)
            q.set_attn_params(l, a["q_norm"], a["k_norm"])
        for l in range(n_gdn):
            p = synth.gdn_params(seed + 100 + l)
            q.set_gdn_params(l, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
        self.seqs = [q.seq_alloc() for _ in range(n)]
        # map pages in a seeded random order: physical pages end up permuted
        rng = np.random.default_rng(seed)
        need = {s: (ctx + 63) // 64 for s in self.seqs}
        have = {s: 0 for s in self.seqs}
        while any(have[s] < need[s] for s in self.seqs):
            s = int(rng.choice([s for s in self.seqs if have[s] < need[s]]))
            have[s] += 1
            q.seq_reserve(s, min(ctx, have[s] * 64))
        bf16 = torch.bfloat16
        for s in self.seqs:
            for l in range(n_attn):
                k = torch.randn(ctx, 4, 256, generator=g, device="cuda").to(bf16)
                v = torch.randn(ctx, 4, 256, generator=g, device="cuda").to(bf16)
                q.kv_write(s, l, 0, ctx, k.data_ptr(), v.data_ptr(), stream)
                torch.cuda.synchronize()
            for l in range(n_gdn):
                st = torch.randn(32, 128, 128, generator=g, device="cuda") * 0.02
                hi = torch.randn(3, 8192, generator=g, device="cuda").to(bf16)
                q.gdn_state_write(s, l, st.data_ptr(), hi.data_ptr(), stream)
                torch.cuda.synchronize()
        # per-layer projection inputs and outputs: views into one contiguous
        # buffer each, so a step's inputs (outputs) move in one copy
        self.proj_flat, self.proj = Stack.layer_views(torch, kinds, n, bf16)
        self.proj_flat.copy_(torch.randn(self.proj_flat.numel(), generator=g, device="cuda"))
        self.out_flat = torch.empty(len(kinds) * n * 4096, device="cuda", dtype=bf16)
        self.out = [self.out_flat[i * n * 4096:(i + 1) * n * 4096].view(n, 4096)
                    for i in range(len(kinds))]
        torch.cuda.synchronize()
        q.check_device()

    @staticmethod
    def layer_views(torch, kinds, n, dtype):
        """One flat device buffer holding every layer's [n][row] projection
        input, and the per-layer views into it."""
        widths = [10240 if kd == "a" else 12352 for kd in kinds]
        flat = torch.empty(n * sum(widths), device="cuda", dtype=dtype)
        views, off = [], 0
        for w in widths:
            views.append(flat[off:off + n * w].view(n, w))
            off += n * w
        return flat, views

    def step(self, events=None):
        self.q.decode_begin(self.seqs, stream=self.stream)
        self.layers(self.stream, events)
        self.q.decode_end()

    def layers(self, st, events=None):
        q = self.q
        ai = gi = 0
        for layer, kind in enumerate(self.kinds):
            if events is not None:
                events[layer][0].record()
            if kind == "a":
                q.attn_decode(ai, self.proj[layer].data_ptr(), self.out[layer].data_ptr(), st)
                ai += 1
            else:
                q.gdn_decode(gi, self.proj[layer].data_ptr(), self.out[layer].data_ptr(), st)
                gi += 1
            if events is not None:
                events[layer][1].record()

    def step_bytes(self):
        """Algorithmic HBM bytes of ONE layer launch of each type in the next
        step (positions = current lengths)."""
        pos = [self.q.seq_len(s) for s in self.seqs]
        attn = sum(attn_bytes_per_seq(p) for p in pos)
        gdn = self.n * GDN_BYTES_PER_SEQ + GDN_BYTES_PER_LAUNCH
        return attn, gdn


WORKLOADS = {
    # name: (layer kinds, total sequences, context, description)
    "stack": ([("a" if is_attn(l) else "g") for l in range(N_LAYERS)], N_SEQ, CTX,
              "full cache stack: 24 DeltaNet + 8 attention layers (attention every 4th), "
              "{n} sequences at context {ctx}, 64-token bf16 pages (permuted), one decode "
              "token per sequence"),
    "gdn": (["g"] * N_GDN, 64, 0,
            "Gated DeltaNet decode step, 24 layers, batch {n}: fp32 state [32,128,128], "
            "conv ring, gated RMSNorm"),
    "attn": (["a"], 1, 1024,
             "single full-attention layer decode, batch {n}, {ctx} cached positions, fused "
             "Q/K norm + RoPE + append, L2 flushed between steps"),
    "long": (["a"] * N_ATTN, 1, 131072,
             "long-context single sequence: 8 attention layers at context {ctx}, split-K "
             "over KV pages"),
}


def run_ours(args, rank, world, dist, kinds, n_total, ctx):
    import torch
    qc = load_pkg("qcache")
    synth = load_pkg("synth")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    n = n_total // world
    stream = torch.cuda.current_stream().cuda_stream
    stack = Stack(qc, synth, torch, kinds, n, ctx, args.warmup + 2 * args.steps + 8,
                  seed=1000 + rank, stream=stream)
    nl = len(kinds)
    # inputs smaller than L2 (126 MB): flush it between steps, outside the events
    small = ctx * 4096 * kinds.count("a") * n + n * 2 ** 21 * 2 * kinds.count("g") < 512 * 2 ** 20
    flush_buf = torch.empty(512 * 2 ** 20, dtype=torch.uint8, device="cuda") if small else None

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        stack.step()
    barrier()

    # ---- capture the layer calls of one step into a CUDA graph (the
    # per-step inputs -- positions, split sizes -- are read from the device
    # descriptor that qc_decode_begin uploads, so the graph replays every step)
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    stack.q.decode_begin(stack.seqs, stream=stream)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=cap):
        stack.layers(torch.cuda.current_stream().cuda_stream)
    stack.q.decode_abort()
    torch.cuda.synchronize()

    def graph_step(kev=None):
        stack.q.decode_begin(stack.seqs, stream=stream)
        if kev is not None:
            kev[0].record()
        graph.replay()
        if kev is not None:
            kev[1].record()
        stack.q.decode_end()

    # ---- device-timed region: K graph steps
    attn_b = gdn_b = 0
    sev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.5)   # let the sampler come up before the timed region
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record()
    for k in range(args.steps):
        a, g_ = stack.step_bytes()
        attn_b += a
        gdn_b += g_
        if flush_buf is not None:
            flush_buf.zero_()
        sev[k][0].record()
        graph_step(kev[k])
        sev[k][1].record()
    t1.record()
    barrier()
    clk = clocks.stop()
    # with L2 flushes inside the region, the step time is the sum of the steps
    ms = (sum(e0.elapsed_time(e1) for e0, e1 in sev) / args.steps if small
          else t0.elapsed_time(t1) / args.steps)
    # the layer kernels alone (the graph replay), without qc_decode_begin's
    # descriptor upload: what small configurations spend in their kernels
    kernels_ms = sum(e0.elapsed_time(e1) for e0, e1 in kev) / args.steps
    # per-layer-type split: with one layer type it is the step; otherwise a few
    # extra non-graph steps with an event pair around every layer call (the
    # GPU stays saturated in these workloads, so the split is device time)
    if kinds.count("a") == 0 or kinds.count("g") == 0:
        attn_ms = ms if kinds.count("a") else 0.0
        gdn_ms = ms if kinds.count("g") else 0.0
    else:
        ks = min(args.steps, 10)
        ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(nl)]
              for _ in range(ks)]
        for k in range(ks):
            stack.step(ev[k])
        torch.cuda.synchronize()
        lt = [sum(ev[k][l][0].elapsed_time(ev[k][l][1]) for k in range(ks)) / ks
              for l in range(nl)]
        tot = sum(lt)
        attn_ms = ms * sum(t for t, kd in zip(lt, kinds) if kd == "a") / tot
        gdn_ms = ms * sum(t for t, kd in zip(lt, kinds) if kd == "g") / tot
    stack.q.check_device()

    # ---- end-to-end through the C ABI with host buffers: every step copies
    # its projection rows host -> device (pinned) and its outputs back.  Two
    # buffer sets, two captured graphs and two copy streams pipeline the
    # transfers of step k + 1 (inputs) and k - 1 (outputs) under step k.
    bf16 = torch.bfloat16
    h_in = torch.empty(stack.proj_flat.shape, dtype=bf16, pin_memory=True).copy_(
        stack.proj_flat.cpu())
    h_out = torch.empty(stack.out_flat.shape, dtype=bf16, pin_memory=True)
    h2d = h_in.numel() * 2
    d2h = h_out.numel() * 2
    sets = [(stack.proj_flat, stack.out_flat, graph)]
    proj2_flat, proj2 = Stack.layer_views(torch, kinds, n, bf16)
    out2_flat = torch.empty_like(stack.out_flat)
    out2 = [out2_flat[i * n * 4096:(i + 1) * n * 4096].view(n, 4096) for i in range(len(kinds))]
    saved = (stack.proj, stack.out)
    stack.proj, stack.out = proj2, out2
    graph2 = torch.cuda.CUDAGraph()
    stack.q.decode_begin(stack.seqs, stream=stream)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph2, stream=cap):
        stack.layers(torch.cuda.current_stream().cuda_stream)
    stack.q.decode_abort()
    stack.proj, stack.out = saved
    sets.append((proj2_flat, out2_flat, graph2))
    torch.cuda.synchronize()
    main = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def load_inputs(b, wait_done):
        with torch.cuda.stream(s_in):
            if wait_done:
                s_in.wait_event(ev_done[b])
            sets[b][0].copy_(h_in, non_blocking=True)
            ev_in[b].record(s_in)

    # every step copies its inputs in and its outputs out; the first load and
    # the last drain are inside the timed region too
    e2e_steps = max(2, args.steps)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(main)
    load_inputs(0, False)
    for k in range(e2e_steps):
        b = k % 2
        main.wait_event(ev_in[b])
        if k >= 2:
            main.wait_event(ev_out[b])     # step k-2's outputs left this buffer
        # the step (its small descriptor upload first) is queued before the
        # next step's 48 MB input copy, so that upload does not wait behind
        # the large copy on the host-to-device copy engine
        stack.q.decode_begin(stack.seqs, stream=stream)
        sets[b][2].replay()
        stack.q.decode_end()
        ev_done[b].record(main)
        if k + 1 < e2e_steps:
            load_inputs(1 - b, k >= 1)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[b])
            h_out.copy_(sets[b][1], non_blocking=True)
            ev_out[b].record(s_out)
    main.wait_event(ev_out[(e2e_steps - 1) % 2])
    e1.record(main)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps

    vals = torch.tensor([ms, e2e_ms, attn_ms, gdn_ms, kernels_ms], device="cuda",
                        dtype=torch.float64)
    rank_ms = [ms]
    if dist is not None:
        every = [torch.zeros_like(vals) for _ in range(world)]
        dist.all_gather(every, vals)
        rank_ms = [float(v[0]) for v in every]   # each rank's own step time
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms, attn_ms, gdn_ms, kernels_ms = vals.tolist()
    return dict(ms=ms, e2e_ms=e2e_ms, attn_ms=attn_ms, gdn_ms=gdn_ms, rank_ms=rank_ms,
                kernels_ms=kernels_ms,
                attn_layer_bytes=attn_b / args.steps, gdn_layer_bytes=gdn_b / args.steps,
                n_local=n, h2d=h2d, d2h=d2h, clocks=clk,
                l2="L2 flushed (512 MB write) between steps" if small
                else "inputs larger than L2 (126 MB) on every step")


def run_long_split(args, rank, world, dist, n_layers, ctx):
    """Config 4 over several GPUs: one sequence, split-K over KV pages.  Every
    rank maps the whole context (and holds the KV of all pages, so any range is
    valid); rank r attends pages [cut_r, cut_{r+1}) and the last rank also the
    new token (it owns the growing tail).  Per layer: qc_attn_partial -> NCCL
    all-gather of the [16][258] f32 records -> qc_attn_combine on every rank."""
    import torch
    qc = load_pkg("qcache")
    synth = load_pkg("synth")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream().cuda_stream
    kinds = ["a"] * n_layers
    stack = Stack(qc, synth, torch, kinds, 1, ctx, args.warmup + args.steps + 8, seed=1000,
                  stream=stream)
    q = stack.q
    pages0 = ctx // 64 + 1
    cuts = [r * pages0 // world for r in range(world)] + [None]
    recs = torch.zeros(n_layers, 16, 258, device="cuda")
    gathered = torch.zeros(n_layers, world, 16, 258, device="cuda")
    p2p = args.collective == "p2p"
    if p2p:  # mailboxes in peer memory: handles exchanged once over the process group
        handle = q.p2p_create(world, rank)
        handles = [None] * world
        dist.all_gather_object(handles, handle)
        for r in range(world):
            if r != rank:
                q.p2p_open(r, handles[r])

    def begin():
        q.decode_begin(stack.seqs, stream=stream)
        pos = q.seq_len(stack.seqs[0])
        pe = cuts[rank + 1] if rank + 1 < world else pos // 64 + 1
        q.attn_partial_range(cuts[rank], pe, int(rank == world - 1), stream)

    def layers(st):
        for l in range(n_layers):
            if p2p:
                q.attn_partial_p2p(l, stack.proj[l].data_ptr(), st)
                q.attn_combine_p2p(l, stack.proj[l].data_ptr(), stack.out[l].data_ptr(), st)
                continue
            q.attn_partial(l, stack.proj[l].data_ptr(), recs[l].data_ptr(), st)
            dist.all_gather_into_tensor(gathered[l], recs[l])
            q.attn_combine(gathered[l].data_ptr(), world, stack.proj[l].data_ptr(),
                           stack.out[l].data_ptr(), st)

    # one step captured into a CUDA graph (partials, NCCL all-gathers and
    # merges); the range descriptor is uploaded per step outside the graph
    begin()
    layers(stream)            # warm: NCCL communicator set up before capture
    q.decode_end()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    begin()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph):
        layers(torch.cuda.current_stream().cuda_stream)
    q.decode_abort()
    torch.cuda.synchronize()

    def step():
        begin()
        graph.replay()
        q.decode_end()

    for _ in range(args.warmup):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.5)
    attn_b = 0
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    t0.record()
    for _ in range(args.steps):
        attn_b += attn_bytes_per_seq(q.seq_len(stack.seqs[0]))
        step()
    t1.record()
    dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    q.check_device()
    vals = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms = vals.item()
    return dict(ms=ms, e2e_ms=None, attn_ms=ms, gdn_ms=0.0,
                attn_layer_bytes=attn_b / args.steps / world, gdn_layer_bytes=0.0, n_local=1,
                h2d=0, d2h=0, clocks=clk, l2="inputs larger than L2 on every step",
                collective=("records stored into every rank's mailbox in peer memory over "
                            "NVLink by the record kernel, arrival counters bumped at system "
                            "scope, bounded device-side wait in the merge; captured in a CUDA "
                            "graph" if p2p else
                            "NCCL all-gather of the (m, l, o) records, one per layer, "
                            "captured with the kernels in a CUDA graph"))


def run_prefix(args):
    """Config 3: prefix-cache reuse on one GPU."""
    import torch
    qc = load_pkg("qcache")
    synth = load_pkg("synth")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(3)
    batch = args.seqs or 64                 # requests per batched restore
    n_pref, n_req = 16, 4 * batch
    plen = rng.integers(512, 3585, n_pref)
    kinds = [("a" if is_attn(l) else "g") for l in range(N_LAYERS)]
    pages = int(sum((p + 63) // 64 for p in plen)) + batch * 4 + 16
    q = qc.QCache(n_attn_layers=N_ATTN, n_gdn_layers=N_GDN, max_seqs=n_pref + batch,
                  max_pages=pages, max_ctx=4096 + 128, max_batch=batch, max_snapshots=n_pref,
                  device=torch.cuda.current_device())
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    for l in range(N_ATTN):
        a = synth.attn_inputs(l, 1, 0)
        q.set_attn_params(l, a["q_norm"], a["k_norm"])
    for l in range(N_GDN):
        p = synth.gdn_params(100 + l)
        q.set_gdn_params(l, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    bf16 = torch.bfloat16
    prefixes, entries, src_seqs = [], [], []
    for i in range(n_pref):
        P = int(plen[i])
        toks = rng.integers(0, 248320, P).astype(np.int32)
        s = q.seq_alloc()
        q.seq_reserve(s, P)
        for l in range(N_ATTN):
            k = torch.randn(P, 4, 256, generator=g, device="cuda").to(bf16)
            v = torch.randn(P, 4, 256, generator=g, device="cuda").to(bf16)
            q.kv_write(s, l, 0, P, k.data_ptr(), v.data_ptr(), stream)
            torch.cuda.synchronize()
        for l in range(N_GDN):
            st = torch.randn(32, 128, 128, generator=g, device="cuda") * 0.02
            hi = torch.randn(3, 8192, generator=g, device="cuda").to(bf16)
            q.gdn_state_write(s, l, st.data_ptr(), hi.data_ptr(), stream)
            torch.cuda.synchronize()
        entries.append(q.prefix_insert(s, toks, stream))
        prefixes.append(toks)
        src_seqs.append(s)
    torch.cuda.synchronize()
    live = [q.seq_alloc() for _ in range(batch)]
    proj = [torch.randn(batch, 10240 if kd == "a" else 12352, generator=g, device="cuda").to(bf16)
            for kd in kinds]
    out = [torch.empty(batch, 4096, device="cuda", dtype=bf16) for _ in kinds]
    # requests: a prefix chosen uniformly + a distinct suffix of 1-64 tokens
    reqs = []
    for r in range(n_req):
        i = int(rng.integers(0, n_pref))
        suf = rng.integers(0, 248320, int(rng.integers(1, 65))).astype(np.int32)
        reqs.append((i, np.concatenate([prefixes[i], suf])))
    lookup_s, restore_ms, decode_ms, moved, hits = 0.0, 0.0, 0.0, 0, 0
    restore_host_ms = 0.0
    for rnd in range(-1, n_req // batch):      # round -1 warms up
        chunk = reqs[max(rnd, 0) * batch:(max(rnd, 0) + 1) * batch]
        t = time.perf_counter()
        found = [q.prefix_lookup(toks) for _, toks in chunk]
        lt = time.perf_counter() - t
        ents = [e for _, e in found]
        hits_r = sum(1 for (i, _), (m, e) in zip(chunk, found) if e == entries[i])
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        torch.cuda.synchronize()
        # the device time of the restore (the job upload and the copy kernel):
        # a spin kernel keeps the stream busy while the host builds the jobs,
        # so e0 fires after the host work is queued
        torch.cuda._sleep(int(4e7))
        e0.record()
        h0 = time.perf_counter()
        q.prefix_restore(ents, live, stream)
        host_ms = (time.perf_counter() - h0) * 1e3
        e1.record()
        q.decode_begin(live, stream=stream)
        ai = gi = 0
        for l, kd in enumerate(kinds):
            if kd == "a":
                q.attn_decode(ai, proj[l].data_ptr(), out[l].data_ptr(), stream)
                ai += 1
            else:
                q.gdn_decode(gi, proj[l].data_ptr(), out[l].data_ptr(), stream)
                gi += 1
        q.decode_end()
        e2.record()
        torch.cuda.synchronize()
        if rnd >= 0:
            lookup_s += lt
            restore_ms += e0.elapsed_time(e1)
            restore_host_ms += host_ms
            decode_ms += e1.elapsed_time(e2)
            moved += q.last_restore_bytes()
            hits += hits_r
        if rnd == 0:   # bit-exact check of one restored request against its source
            i0 = chunk[0][0]
            P = int(plen[i0])
            for l in (0, N_ATTN - 1):
                ka, va = (torch.empty(P, 4, 256, dtype=bf16, device="cuda") for _ in range(2))
                kb, vb = (torch.empty(P, 4, 256, dtype=bf16, device="cuda") for _ in range(2))
                q.kv_read(src_seqs[i0], l, 0, P, ka.data_ptr(), va.data_ptr(), stream)
                q.kv_read(live[0], l, 0, P, kb.data_ptr(), vb.data_ptr(), stream)
                torch.cuda.synchronize()
                exact = bool(torch.equal(ka.view(torch.int16), kb.view(torch.int16)) and
                             torch.equal(va.view(torch.int16), vb.view(torch.int16)))
        for s in live:
            q.seq_reset(s, stream)
        torch.cuda.synchronize()
    q.check_device()
    n = n_req
    return dict(lookup_us=lookup_s / n * 1e6, restore_ms=restore_ms, decode_ms=decode_ms,
                restore_host_ms=restore_host_ms, batch=batch,
                moved=moved, hits=hits, n=n, exact=exact,
                restore_gbs=moved / (restore_ms * 1e-3) / 1e9,
                decode_us_token_layer=decode_ms * 1e3 / (n * N_LAYERS))


def run_prefill(args, prompt=2048):
    """Prefill of one `prompt`-token sequence through the 32-layer stack in
    chunks of QC_PREFILL_CHUNK tokens (the reference prefills token by token,
    src/engine.cpp:2602, 2843), and the same prompt as one decode step per
    token for comparison."""
    import torch
    qc = load_pkg("qcache")
    synth = load_pkg("synth")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    stream = torch.cuda.current_stream().cuda_stream
    kinds = [("a" if is_attn(l) else "g") for l in range(N_LAYERS)]
    chunk = 32
    q = qc.QCache(n_attn_layers=N_ATTN, n_gdn_layers=N_GDN, max_seqs=2,
                  max_pages=2 * (prompt // 64 + 2), max_ctx=prompt + 64, max_batch=1,
                  max_snapshots=1, device=torch.cuda.current_device())
    for l in range(N_ATTN):
        a = synth.attn_inputs(l, 1, 0)
        q.set_attn_params(l, a["q_norm"], a["k_norm"])
    for l in range(N_GDN):
        p = synth.gdn_params(100 + l)
        q.set_gdn_params(l, p["ssm_a"], p["dt_bias"], p["ssm_norm"], p["conv_w"])
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    bf16 = torch.bfloat16
    proj = [torch.randn(chunk, 10240 if kd == "a" else 12352, generator=g, device="cuda").to(bf16)
            for kd in kinds]
    out = [torch.empty(chunk, 4096, device="cuda", dtype=bf16) for _ in kinds]

    def prefill(s, n_tok):
        for c0 in range(0, n_tok, chunk):
            n = min(chunk, n_tok - c0)
            q.prefill_begin(s, n, stream=stream)
            ai = gi = 0
            for l, kd in enumerate(kinds):
                if kd == "a":
                    q.attn_prefill(ai, proj[l].data_ptr(), out[l].data_ptr(), stream)
                    ai += 1
                else:
                    q.gdn_prefill(gi, proj[l].data_ptr(), out[l].data_ptr(), stream)
                    gi += 1
            q.prefill_end()

    def decode(s, n_tok):
        for _ in range(n_tok):
            q.decode_begin([s], stream=stream)
            ai = gi = 0
            for l, kd in enumerate(kinds):
                if kd == "a":
                    q.attn_decode(ai, proj[l].data_ptr(), out[l].data_ptr(), stream)
                    ai += 1
                else:
                    q.gdn_decode(gi, proj[l].data_ptr(), out[l].data_ptr(), stream)
                    gi += 1
            q.decode_end()

    s = q.seq_alloc()
    prefill(s, 256)                    # warm-up
    q.seq_reset(s, stream)
    torch.cuda.synchronize()
    res = {}
    for name, fn in (("prefill", prefill), ("decode", decode)):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn(s, prompt)
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1)
        q.seq_reset(s, stream)
        torch.cuda.synchronize()
    q.check_device()
    return res, prompt


def gemv_shapes():
    """The projection GEMVs around the cache path in one decode step, in layer
    order: per DeltaNet layer the combined in-projection (12352 x 4096) and the
    out-projection (4096 x 4096); per attention layer the QKV projection
    (10240 x 4096) and the out-projection (4096 x 4096)."""
    out = []
    for l in range(N_LAYERS):
        out.append((10240 if is_attn(l) else 12352, 4096))
        out.append((4096, 4096))
    return out


def run_gemv(args, batches=(1, 8, 16)):
    """BFP8_B projection GEMVs (include/qbfp8.h) of one decode step: 64
    distinct matrices (2.2 GB of tiles, far above L2), captured once per batch
    size in a CUDA graph.  Device time of the timed graph replays with CUDA
    events, and e2e with the step's activations copied in from pinned host
    memory and the outputs copied back inside the timed region."""
    import torch
    qc = load_pkg("qcache")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    shapes = gemv_shapes()
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    mats = []
    for M, K in shapes:
        w = (torch.randn(M, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        m = qc.Bfp8Matrix(M, K)
        m.pack_bf16(w.data_ptr())
        mats.append(m)
        del w
    torch.cuda.synchronize()
    tile_bytes = sum(qc.Bfp8Matrix.packed_bytes(M, K) for M, K in shapes)
    stream = torch.cuda.Stream()
    res = {}
    for B in batches:
        # every GEMV's activations (outputs) are views into one buffer, so a
        # step's inputs (outputs) move in one copy
        x_flat = torch.randn(B * sum(K for _, K in shapes), generator=g, device="cuda").to(
            torch.bfloat16)
        y_flat = torch.empty(B * sum(M for M, _ in shapes), device="cuda", dtype=torch.bfloat16)
        xs, ys, ox, oy = [], [], 0, 0
        for M, K in shapes:
            xs.append(x_flat[ox:ox + B * K].view(B, K))
            ys.append(y_flat[oy:oy + B * M].view(B, M))
            ox += B * K
            oy += B * M

        def step(st):
            for m, x, y in zip(mats, xs, ys):
                m.gemv(x.data_ptr(), B, y.data_ptr(), st)
        with torch.cuda.stream(stream):
            step(stream.cuda_stream)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(stream.cuda_stream)
            for _ in range(args.warmup):
                graph.replay()
            stream.synchronize()
            clk = ClockSampler(torch.cuda.current_device()) if B == 1 else None
            if clk:
                clk.start()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            stream.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            clocks = clk.stop() if clk else None
            # one launch alone (the largest matrix), for the kernel roofline
            big = max(range(len(shapes)), key=lambda i: shapes[i][0])
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 20
            f0.record(stream)
            for _ in range(reps):
                mats[big].gemv(xs[big].data_ptr(), B, ys[big].data_ptr(), stream.cuda_stream)
            f1.record(stream)
            stream.synchronize()
            one_ms = f0.elapsed_time(f1) / reps
            # e2e: activations in from pinned host memory, outputs back out
            hx = torch.empty_like(x_flat, device="cpu").pin_memory()
            hy = torch.empty_like(y_flat, device="cpu").pin_memory()
            stream.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(args.steps):
                x_flat.copy_(hx, non_blocking=True)
                graph.replay()
                hy.copy_(y_flat, non_blocking=True)
            t1.record(stream)
            stream.synchronize()
            e2e_ms = t0.elapsed_time(t1) / args.steps
        res[B] = dict(ms=ms, one_ms=one_ms, big=shapes[big], clocks=clocks, e2e_ms=e2e_ms,
                      h2d=x_flat.numel() * 2, d2h=y_flat.numel() * 2)
    for m in mats:
        m.check()
    return res, tile_bytes


def gemv_cpu_baseline(budget_s=10.0, threads=None):
    """The oracle's threaded BFP8_B GEMV (liboracle_fast.so) on a bounded sample:
    repeated 12352 x 4096 GEMVs at batch 1, scaled to the 64-matrix step by
    tile bytes.  Returns (us per step, threads, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    synth = load_pkg("synth")
    threads = threads or os.cpu_count() or 1
    M, K = 12352, 4096
    w = synth.bf16_bits(np.random.default_rng(1).standard_normal((M, K)).astype(np.float32) * 0.02)
    packed = oracle.bfp8_pack(w)
    x = synth.gemv_inputs(1, 1, K)
    oracle.bfp8_gemv(packed, M, K, x, n_threads=threads, fast=True)
    t0, reps = time.perf_counter(), 0
    while time.perf_counter() - t0 < budget_s:
        oracle.bfp8_gemv(packed, M, K, x, n_threads=threads, fast=True)
        reps += 1
    per = (time.perf_counter() - t0) / reps
    step_bytes = sum((Mi // 32) * (Ki // 32) * 1088 for Mi, Ki in gemv_shapes())
    return per * step_bytes / packed.size * 1e6, threads, f"{reps} GEMVs of 12352x4096 at batch 1"


# ------------------------------------------------------------ CPU baseline

REF_BUILD = ("oracle/_ref/libref.so: src/engine.cpp cache-path blocks, g++ -O3 -ffast-math "
             "-march=x86-64-v4 (the reference builds with clang++-20 -O3 -ffast-math "
             "-march=native)")


def oracle_build() -> str:
    """Which build of the timed CPU restatement this host runs."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    name = oracle.fast_build_name()
    isa = "x86-64-v4, AVX-512" if "512" in name else "x86-64-v3, AVX2"
    return f"{name} (-O3 -ffast-math, {isa})"


def cpu_baseline(budget_s: float = 12.0, threads: int | None = None):
    """The oracle's threaded C++ restatement of the reference's host math
    (liboracle_fast.so: the reference's -O3 -ffast-math), timed on this host
    over a bounded sample of the same workload: sequences at context 4096, one
    DeltaNet layer and one attention layer per sample, combined 24:8 per
    token.  Returns µs per token per layer."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ctypes as C

    import oracle

    synth = load_pkg("synth")
    L = oracle.lib(fast=True)
    threads = threads or os.cpu_count() or 1
    nb = max(1, min(threads, 16))              # sequences per batch call
    p = synth.gdn_params(1)
    g = synth.gdn_inputs(2, nb)
    hist = np.ascontiguousarray(synth.bf16_to_f32(g["hist"]))
    state = np.ascontiguousarray(g["state"])
    out = np.zeros((nb, 4096), np.float32)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    # attention: nb sequences sharing one seeded cache content (bounded memory)
    a = synth.attn_inputs(3, 1, CTX)
    cap = CTX + 64
    kc = np.zeros((nb, cap, 4, 256), np.uint16)
    vc = np.zeros((nb, cap, 4, 256), np.uint16)
    kc[:, :CTX], vc[:, :CTX] = a["k"][0], a["v"][0]
    aproj = np.ascontiguousarray(np.repeat(a["proj"], nb, axis=0))
    pos = np.full(nb, CTX, np.int32)
    aout = np.zeros((nb, 4096), np.float32)

    def gdn_once():
        L.qo_gdn_decode_batch(nb, ptr(g["proj"]), ptr(state), ptr(hist), ptr(p["conv_w"]),
                              ptr(p["ssm_a"]), ptr(p["dt_bias"]), ptr(p["ssm_norm"]), ptr(out),
                              0, threads)

    def attn_once():
        L.qo_attn_decode_batch(nb, ptr(aproj), ptr(a["q_norm"]), ptr(a["k_norm"]), ptr(pos),
                               ptr(kc), ptr(vc), cap, ptr(aout), 0, threads)

    def timed(fn, share):
        fn()  # warm
        t0 = time.perf_counter()
        reps = 0
        while True:
            fn()
            reps += 1
            el = time.perf_counter() - t0
            if el > budget_s * share:
                return el / (reps * nb), reps
    t_gdn, r_g = timed(gdn_once, 0.4)
    t_attn, r_a = timed(attn_once, 0.6)
    us = (24 * t_gdn + 8 * t_attn) / 32 * 1e6
    sample = (f"{r_g}x{nb} seq DeltaNet steps + {r_a}x{nb} seq attention steps at ctx {CTX}, "
              f"weighted 24:8 per token")
    return us, threads, sample, t_gdn * 1e6, t_attn * 1e6


def _ref_stack_worker(args):
    """One process of the reference arm: the reference's own host code for the
    cache path (oracle/_ref/libref.so, the src/engine.cpp blocks compiled
    unchanged) runs one sequence through the 32-layer stack, token after
    token, with its caches and state resident in the reference's own
    file-scope vectors (24 DeltaNet slots, 8 attention caches at the context).
    Returns (steps, seconds)."""
    budget_s, ctx, seed = args
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ctypes as C

    import ref
    L = ref.lib()
    rng = np.random.default_rng(seed)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    cap = ctx + 512
    for l in range(N_ATTN):
        k = rng.standard_normal((ctx, 4, 256), dtype=np.float32)
        v = rng.standard_normal((ctx, 4, 256), dtype=np.float32)
        L.ref_set_layer(l, ptr(k), ptr(v), ctx, cap, -1, None, None)
    for l in range(N_GDN):
        st = (rng.standard_normal((32, 128, 128), dtype=np.float32) * 0.02)
        hist = rng.standard_normal((3, 8192), dtype=np.float32)
        L.ref_set_layer(-1, None, None, 0, 0, l, ptr(st), ptr(hist))
    conv_w = (rng.standard_normal((4, 8192), dtype=np.float32) * 0.1)
    ssm_a = -np.exp(rng.normal(-2.0, 0.5, 32)).astype(np.float32)
    dt_bias = np.zeros(32, np.float32)
    norm = np.ones(128, np.float32)
    qn = np.ones(256, np.float32)
    gproj = rng.standard_normal(12352, dtype=np.float32)
    aproj = rng.standard_normal(10240, dtype=np.float32)
    out = np.zeros(4096, np.float32)

    def step(pos):
        ai = gi = 0
        for layer in range(N_LAYERS):
            if is_attn(layer):
                L.ref_attn_decode_resident(ai, ptr(aproj), ptr(qn), ptr(qn), pos, ptr(out))
                ai += 1
            else:
                L.ref_gdn_decode_resident(gi, ptr(gproj), ptr(conv_w), ptr(ssm_a), ptr(dt_bias),
                                          ptr(norm), ptr(out))
                gi += 1

    step(ctx)  # warm
    t0, n = time.perf_counter(), 1
    while time.perf_counter() - t0 < budget_s and n < cap - ctx:
        step(ctx + n)
        n += 1
    return n - 1, time.perf_counter() - t0


def reference_available() -> bool:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    try:
        import ref
        return ref.available()
    except Exception:
        return False


def reference_baseline(budget_s: float = 12.0, procs: int | None = None):
    """The reference's own CPU implementation of the path on this host: P
    processes, each one reference engine (one sequence at a time, its 4-thread
    WorkerPool for the DeltaNet heads, src/engine.cpp:1630-1693, single-thread
    attention), P = host cores / 4 so the pools fill the cores.  Returns
    (us per token per layer over all processes, threads used, sample)."""
    cores = os.cpu_count() or 1
    procs = procs or max(1, cores // 4)
    # one child interpreter per engine (the reference's state is process-wide);
    # each prints (steps, seconds) as JSON; bounded by a timeout
    kids = [subprocess.Popen([sys.executable, os.path.abspath(__file__), "--ref-worker",
                              f"{budget_s},{CTX},{100 + i}"], stdout=subprocess.PIPE,
                             stderr=subprocess.PIPE, text=True) for i in range(procs)]
    res = []
    for k in kids:
        try:
            out, err = k.communicate(timeout=budget_s * 4 + 120)
        except subprocess.TimeoutExpired:
            k.kill()
            raise RuntimeError("reference worker timed out")
        if k.returncode != 0:
            raise RuntimeError("reference worker failed: " + err.strip().splitlines()[-1:][0]
                               if err.strip() else "reference worker failed")
        res.append(tuple(json.loads(out.strip().splitlines()[-1])))
    steps = sum(r[0] for r in res)
    secs = max(r[1] for r in res)
    us = secs / (steps * N_LAYERS) * 1e6 if steps else float("inf")
    sample = (f"{procs} process(es) x {min(r[0] for r in res)}-{max(r[0] for r in res)} decode "
              f"tokens of one sequence through the 32-layer stack at context {CTX} "
              f"(reference code, 4-thread pool per process)")
    return us, procs * 4, sample


# ----------------------------------------------------------------- output


def emit(line):
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(WORKLOADS) + ["prefix", "prefill", "gemv"],
                    default="stack",
                    help="stack = the headline workload; the others are the baseline's "
                         "per-component configurations")
    ap.add_argument("--seqs", type=int, default=None,
                    help="total sequences (default: the configuration's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--collective", choices=["p2p", "nccl"], default="p2p",
                    help="config long over several GPUs: how the split-K records travel")
    ap.add_argument("--ref-worker", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.ref_worker:  # one engine of the reference arm (see reference_baseline)
        b, c, sd = args.ref_worker.split(",")
        print(json.dumps(_ref_stack_worker((float(b), int(c), int(sd)))), flush=True)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.config == "prefix" and args.impl == "ours":
        r = run_prefix(args)
        peak, peak_kind = measured_peaks()
        emit({"metric": "prefix-hit restore GB/s", "value": round(r["restore_gbs"], 1),
              "unit": "GB/s", "n_gpus": 1, "steps": 4, "warmup": 1,
              "higher_is_better": True, "dtype": "bytes", "data": "synthetic (seeded)",
              "config": {"workload": f"prefix-cache reuse: {r['n']} requests over 16 seeded prefixes "
                                     "(512-3584 tokens) + suffixes of 1-64 tokens; hash lookup, "
                                     f"batched restore of {r['batch']} requests (page-list gather, tail "
                                     "copy-on-write, DeltaNet/conv snapshot), one decode step",
                         "name": "prefix"},
              "hits": r["hits"], "requests": r["n"], "bit_exact": r["exact"],
              "restore_timing": "device time of each batched qc_prefix_restore (job upload + "
                                "copy kernel; a spin kernel ahead of it hides the host's job "
                                "building); host time of the call reported beside it",
              "restore_bytes_per_request": r["moved"] // r["n"],
              "restore_batch": r["batch"],
              "restore_ms_per_batch": round(r["restore_ms"] / 4, 4),
              "restore_host_ms_per_batch": round(r["restore_host_ms"] / 4, 4),
              "lookup_us_per_request": round(r["lookup_us"], 2),
              "decode_after_restore_us_token_layer": round(r["decode_us_token_layer"], 4),
              "roofline": {"kernel": "copy_jobs_bulk_kernel (restore)", "bound": "hbm",
                           "achieved": round(r["restore_gbs"], 1), "peak": peak,
                           "peak_kind": peak_kind, "unit": "GB/s",
                           "frac": round(r["restore_gbs"] / peak, 4), "traffic": None}})
        return
    if args.config == "prefill" and args.impl == "ours":
        r, prompt = run_prefill(args)
        emit({"metric": "prefill cache-path us/token/layer", "value":
              round(r["prefill"] * 1e3 / (prompt * N_LAYERS), 4), "unit": "us", "n_gpus": 1,
              "higher_is_better": False, "dtype": "f32", "data": "synthetic (seeded)",
              "config": {"workload": f"prefill of one {prompt}-token prompt through the 32-layer "
                                     "stack in chunks of 32 tokens", "name": "prefill"},
              "prefill_ms": round(r["prefill"], 3), "prefill_tokens_per_s":
              round(prompt / (r["prefill"] * 1e-3), 1),
              "token_by_token_decode_ms": round(r["decode"], 3),
              "speedup_vs_token_by_token": round(r["decode"] / r["prefill"], 2)})
        return
    if args.config == "gemv" and args.impl == "ours":
        r, tile_bytes = run_gemv(args)
        peak, peak_kind = measured_peaks()
        b1 = r[1]
        M, K = b1["big"]
        one_bytes = (M // 32) * (K // 32) * 1088 + M * 2 + K * 2
        k_gbs = one_bytes / (b1["one_ms"] * 1e-3) / 1e9
        line = {"metric": "projection GEMV us/decode step", "value": round(b1["ms"] * 1e3, 2),
                "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
                "dtype": "bfp8_b weights, bf16 activations, f32 accumulate",
                "data": "synthetic (seeded random weights ~N(0, 0.02) packed on device)",
                "config": {"workload": "the 64 BFP8_B projection GEMVs of one decode step of "
                                       "the 32-layer stack (24 x 12352x4096 + 8 x 10240x4096 "
                                       "in-projections, 32 x 4096x4096 out-projections), batch 1, "
                                       "CUDA graph; 2.2 GB of tiles per step (inputs > L2)",
                           "name": "gemv"},
                "tile_bytes_per_step": tile_bytes,
                "achieved_gbs": round(tile_bytes / (b1["ms"] * 1e-3) / 1e9, 1),
                "batches": {str(B): {"us_per_step": round(v["ms"] * 1e3, 2),
                                     "gbs": round(tile_bytes / (v["ms"] * 1e-3) / 1e9, 1)}
                            for B, v in r.items()},
                "roofline": {"kernel": f"bfp8_gemv_kernel ({M}x{K}, batch 1)", "bound": "hbm",
                             "achieved": round(k_gbs, 1), "peak": peak, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": round(k_gbs / peak, 4), "traffic": None,
                             "algorithmic_bytes_per_launch": one_bytes},
                "e2e": {"value": round(b1["e2e_ms"] * 1e3, 2), "unit": "us",
                        "h2d_bytes_per_step": b1["h2d"], "d2h_bytes_per_step": b1["d2h"]},
                "gpu_launches": args.steps * len(gemv_shapes()),
                "clocks": b1["clocks"]}
        if not args.no_cpu_baseline:
            cus, cores, sample = gemv_cpu_baseline()
            line["cpu_baseline"] = {"value": round(cus, 1), "unit": "us/decode step",
                                    "cores": cores, "kind": "port", "sample": sample, "build": oracle_build()}
        emit(line)
        return
    if args.config in ("prefix", "prefill", "gemv"):
        args.config = "stack"
    kinds, n_total, ctx, desc = WORKLOADS[args.config]
    if args.seqs:
        n_total = args.seqs
    n_attn, n_gdn = kinds.count("a"), kinds.count("g")
    config = {"workload": desc.format(n=n_total, ctx=ctx), "name": args.config,
              "sequences": n_total, "context": ctx, "layers": len(kinds),
              "attention_layers": n_attn, "deltanet_layers": n_gdn, "page_tokens": 64,
              "timing": "CUDA events on the launching stream, max over ranks; each step = "
                        "qc_decode_begin + CUDA-graph replay of the layer calls + qc_decode_end",
              "sharding": f"sequences over {world} GPU(s), no collective"}
    metric = "decode cache-path us/token/layer"

    if args.impl == "reference":
        if rank != 0:
            return
        if args.config == "stack" and reference_available():
            us, cores, sample = reference_baseline()
            kind, build = "reference", REF_BUILD
            what = ("the reference's own host code for the path (src/engine.cpp blocks compiled "
                    "unchanged into oracle/_ref), one engine per process, all host cores")
        else:
            us, cores, sample, _, _ = cpu_baseline()
            kind, build = "port", oracle_build()
            what = ("the CPU restatement of the reference's decode math (oracle port, all host "
                    "threads)")
        ref_config = dict(config, timing=f"host wall clock of {what} over a bounded sample of "
                          "the workload", sharding="rank 0 only, host cores")
        emit({"impl": "reference", "metric": metric, "value": round(us, 3), "unit": "us",
              "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": False, "dtype": "f32", "data": "synthetic",
              "config": ref_config,
              "cpu_baseline": {"value": round(us, 3), "unit": "us/token/layer", "cores": cores,
                               "kind": kind, "sample": sample, "build": build},
              "e2e": {"value": round(us, 3), "unit": "us", "h2d_bytes_per_step": 0,
                      "d2h_bytes_per_step": 0}})
        return

    dist = None
    if world > 1:
        import torch
        import torch.distributed as dist_mod
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist_mod.init_process_group("nccl")
        dist = dist_mod
    if args.config == "long" and world > 1:
        r = run_long_split(args, rank, world, dist, len(kinds), ctx)
        config["sharding"] = f"split-K over KV pages across {world} GPUs"
        config["collective"] = r["collective"]
    else:
        r = run_ours(args, rank, world, dist, kinds, n_total, ctx)
    if dist is not None:
        dist.barrier()
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    peak, peak_kind = measured_peaks()
    units = n_total * len(kinds)
    us = r["ms"] * 1e3 / units
    # every rank holds the same number of sequences at the same context
    step_bytes = (n_attn * r["attn_layer_bytes"] + n_gdn * r["gdn_layer_bytes"]) * world
    gbs = step_bytes / (r["ms"] * 1e-3) / 1e9
    config["l2"] = r["l2"]
    # dominant kernel: the layer type with the larger device time per step;
    # achieved = its algorithmic bytes per launch / its average launch time
    if r["attn_ms"] >= r["gdn_ms"]:
        kname, kbytes, kms = ("attn_partial_kernel + attn_combine_kernel (one attention layer)",
                              r["attn_layer_bytes"], r["attn_ms"] / n_attn)
    else:
        kname, kbytes, kms = ("gdn_decode (one DeltaNet layer)", r["gdn_layer_bytes"],
                              r["gdn_ms"] / n_gdn)
    k_gbs = kbytes / (kms * 1e-3) / 1e9
    traffic, traffic_src = None, None
    prof = PROFILED_TRAFFIC_PER_SEQ.get(args.config)
    kind_now = "attn" if r["attn_ms"] >= r["gdn_ms"] else "gdn"
    if prof and prof[0] == kind_now and world == 1:
        traffic, traffic_src = int(prof[1] * r["n_local"]), prof[2]
    line = {
        "metric": metric, "value": round(us, 4), "unit": "us", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 4),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded), random-init per-layer weights", "config": config,
        "hbm": {"algorithmic_bytes_per_step": int(step_bytes), "achieved_gbs": round(gbs, 1),
                "frac_of_8tbs": round(gbs / world / HBM_NOMINAL_GBS, 4),
                "frac_of_measured": round(gbs / world / peak, 4)},
        "layer_time_ms": {"attention_total": round(r["attn_ms"], 4),
                          "deltanet_total": round(r["gdn_ms"], 4)},
        "roofline": {"kernel": kname, "bound": "hbm", "achieved": round(k_gbs, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(k_gbs / peak, 4), "traffic": traffic,
                     "traffic_source": traffic_src,
                     "algorithmic_bytes_per_launch": int(kbytes)},
        "e2e": ({"value": round(r["e2e_ms"] * 1e3 / units, 4), "unit": "us",
                 "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]}
                if r["e2e_ms"] is not None else None),
        "gpu_launches": args.steps * (n_gdn + 2 * n_attn),
        "rank_ms_per_step": [round(x, 4) for x in r.get("rank_ms", [r["ms"]])],
        "layer_kernels_ms_per_step": (round(r["kernels_ms"], 4) if r.get("kernels_ms")
                                      is not None else None),
        "clocks": r["clocks"],
    }
    if not args.no_cpu_baseline and world == 1:
        if args.config == "stack" and reference_available():
            cus, cores, sample = reference_baseline(budget_s=10.0)
            line["cpu_baseline"] = {"value": round(cus, 3), "unit": "us/token/layer",
                                    "cores": cores, "kind": "reference", "sample": sample,
                                    "build": REF_BUILD}
            # the reference as it ships: one inference at a time
            cus1, c1, sample1 = reference_baseline(budget_s=6.0, procs=1)
            line["cpu_baseline_one_engine"] = {"value": round(cus1, 3), "unit": "us/token/layer",
                                               "cores": c1, "kind": "reference",
                                               "sample": sample1, "build": REF_BUILD}
        # the restatement (the parity oracle's fast build), all host threads
        cus, cores, sample, _, _ = cpu_baseline(budget_s=8.0)
        line["cpu_baseline_port"] = {"value": round(cus, 3), "unit": "us/token/layer",
                                     "cores": cores, "kind": "port", "sample": sample,
                                     "build": oracle_build()}
        if "cpu_baseline" not in line:
            line["cpu_baseline"] = dict(line["cpu_baseline_port"])
    emit(line)
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
