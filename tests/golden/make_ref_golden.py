"""Generates tests/golden/ref_*.npz: outputs of the REFERENCE's own host code
for the cache path (src/engine.cpp blocks compiled unchanged into
oracle/_ref/libref.so by oracle/ref_harness.cpp) on seeded synthetic inputs.

These fixtures pin the oracle (and, through it, the GPU kernels) to the
reference: tests/test_ref_pin.py checks the oracle against them on every
machine, whether or not the reference source is present there.  Inputs are
not stored; they regenerate from the seeds with the package's synth module.

Needs the reference source (the directory QC_REFERENCE_SRC names, default as
in oracle/ref.py) and an AVX-512 host.  Run from the repository root:
    python tests/golden/make_ref_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from conftest import load_pkg_module  # noqa: E402
import ref  # noqa: E402

synth = load_pkg_module("synth")

# config 0 (seed 0, 1024 cached positions) and cases around page edges and
# the config-2 context
ATTN_CASES = [(0, 1024), (41, 0), (42, 63), (43, 4096)]
# config 1 (batch-1 DeltaNet step), three consecutive tokens each so the conv
# history shift is covered; (seed, params seed)
GDN_CASES = [(1, 1), (51, 52)]
GDN_STEPS = 3
# heads of the state stored whole after the last step (the whole state is
# 2 MiB); after every step the sum of each state row is stored
STATE_HEADS = [0, 17, 31]
ROPE_POS = [0, 1, 63, 1024, 4096, 131072]


def prefix_cases():
    """(cached, prompt) pairs: the branches of the rule (extend, diverge,
    whole prompt cached, empty histories) on small seeded token lists."""
    rng = np.random.default_rng(61)
    cases = [([], []), ([], [5]), ([5], []), ([1, 2, 3], [1, 2, 3]), ([1, 2, 3], [1, 2, 3, 4]),
             ([1, 2, 3], [1, 2]), ([1, 2, 3], [1, 9, 3, 4]), ([7], [8, 9])]
    for _ in range(200):
        base = rng.integers(0, 3, 24)
        nc, npr = int(rng.integers(0, 16)), int(rng.integers(0, 16))
        c, p = base[:nc].copy(), base[:npr].copy()
        if npr and rng.random() < 0.3:
            p[int(rng.integers(npr))] += 1
        cases.append((c.tolist(), p.tolist()))
    return cases


def attn_case(seed, ctx):
    d = synth.attn_inputs(seed, 1, ctx)
    k = np.zeros((ctx + 1, 4, 256), np.float32)
    v = np.zeros((ctx + 1, 4, 256), np.float32)
    k[:ctx] = synth.bf16_to_f32(d["k"][0])
    v[:ctx] = synth.bf16_to_f32(d["v"][0])
    out = ref.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], ctx, k, v)
    return dict(out=out, k_new=k[ctx].copy(), v_new=v[ctx].copy())


def gdn_case(seed, pseed):
    p = synth.gdn_params(pseed)
    d = synth.gdn_inputs(seed, 1)
    state = d["state"][0].copy()
    hist = synth.bf16_to_f32(d["hist"][0]).copy()
    outs, row_sums, projs = [], [], []
    for t in range(GDN_STEPS):
        proj = d["proj"][0] if t == 0 else synth.bf16_bits(synth.normal(seed * 8 + 7 + t, (12352,)))
        projs.append(proj)
        outs.append(ref.gdn_decode(proj, state, hist, p))
        row_sums.append(state.astype(np.float64).sum(axis=2))
    return dict(out=np.stack(outs), row_sums=np.stack(row_sums), state_heads=state[STATE_HEADS],
                hist=hist, heads=np.array(STATE_HEADS, np.int32), proj=np.stack(projs))


def main():
    if not ref.available():
        sys.exit("reference library unavailable: needs the reference source and AVX-512")
    for seed, ctx in ATTN_CASES:
        np.savez_compressed(os.path.join(HERE, f"ref_attn_s{seed}_L{ctx}.npz"), seed=seed,
                            ctx=ctx, **attn_case(seed, ctx))
    for seed, pseed in GDN_CASES:
        np.savez_compressed(os.path.join(HERE, f"ref_gdn_s{seed}.npz"), seed=seed, pseed=pseed,
                            steps=GDN_STEPS, **gdn_case(seed, pseed))
    cases = prefix_cases()
    flat_c = np.concatenate([np.array(c, np.int32) for c, _ in cases] + [np.zeros(0, np.int32)])
    flat_p = np.concatenate([np.array(p, np.int32) for _, p in cases] + [np.zeros(0, np.int32)])
    res = np.array([ref.prefix_rule(c, p) for c, p in cases], np.int32)
    rope = np.stack([np.stack(ref.rope_row(pos)) for pos in ROPE_POS])
    np.savez_compressed(os.path.join(HERE, "ref_rules.npz"),
                        n_cached=np.array([len(c) for c, _ in cases], np.int32),
                        n_prompt=np.array([len(p) for _, p in cases], np.int32),
                        cached=flat_c, prompt=flat_p, result=res,
                        rope_pos=np.array(ROPE_POS, np.int32), rope=rope,
                        fast_exp_x=np.linspace(-100, 100, 2001, dtype=np.float32),
                        fast_exp_y=np.array([ref.fast_expf(float(x)) for x in
                                             np.linspace(-100, 100, 2001, dtype=np.float32)],
                                            np.float32))
    print("written to", HERE)


if __name__ == "__main__":
    main()
