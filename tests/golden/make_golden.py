"""Generates tests/golden/*.npz: oracle outputs on seeded synthetic inputs.

The inputs are not stored: they are regenerated from the seeds with the
package's synth module (SplitMix64 + Box-Muller, bit-reproducible).  Run from
the repository root:  python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from conftest import load_pkg_module  # noqa: E402
import oracle  # noqa: E402

synth = load_pkg_module("synth")

# (seed, cached positions): crosses 0, a page boundary, a full page, ragged
ATTN_CASES = [(11, 0), (12, 63), (13, 64), (14, 130)]
GDN_CASES = [(21, 0), (22, 5)]  # (seed, position of the token: ring phase)
BFP8_CASES = [(31, 64, 128, 3), (32, 96, 64, 1)]  # (seed, M, K, batch)


def attn_case(seed, ctx):
    d = synth.attn_inputs(seed, 1, ctx)
    k = np.zeros((ctx + 1, 4, 256), np.uint16)
    v = np.zeros((ctx + 1, 4, 256), np.uint16)
    k[:ctx] = d["k"][0]
    v[:ctx] = d["v"][0]
    out = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], ctx, k, v)
    out_ref = oracle.attn_decode(d["proj"][0], d["q_norm"], d["k_norm"], ctx, k.copy(), v.copy(),
                                 mode=oracle.REF_APPROX)
    return dict(out=out, out_ref_approx=out_ref, k_new=k[ctx].copy(), v_new=v[ctx].copy())


def gdn_case(seed, pos):
    p = synth.gdn_params(seed)
    d = synth.gdn_inputs(seed, 1)
    state = d["state"][0].copy()
    hist = synth.bf16_to_f32(d["hist"][0]).copy()
    out = oracle.gdn_decode(d["proj"][0], state, hist, p)
    return dict(out=out, state_sha=np.frombuffer(hashlib.sha256(state.tobytes()).digest(), np.uint8),
                state_sample=state.reshape(-1)[::997].copy(), hist=hist, pos=np.int32(pos))


def bfp8_case(seed, M, K, batch):
    w = synth.bfp8_weights(seed, M, K)
    packed = oracle.bfp8_pack(w)
    x = synth.gemv_inputs(seed, batch, K)
    y, y32 = oracle.bfp8_gemv(packed, M, K, x)
    res = synth.bf16_bits(synth.normal(seed * 8 + 3, (batch, M)))
    y_res, _ = oracle.bfp8_gemv(packed, M, K, x, residual_bits=res)
    return dict(packed=packed, y=y, y32=y32, y_resadd=y_res)


def main():
    for seed, ctx in ATTN_CASES:
        np.savez_compressed(os.path.join(HERE, f"attn_s{seed}_L{ctx}.npz"), seed=seed, ctx=ctx,
                            **attn_case(seed, ctx))
    for seed, pos in GDN_CASES:
        np.savez_compressed(os.path.join(HERE, f"gdn_s{seed}_p{pos}.npz"), seed=seed,
                            **gdn_case(seed, pos))
    for seed, M, K, batch in BFP8_CASES:
        np.savez_compressed(os.path.join(HERE, f"bfp8_s{seed}_{M}x{K}_b{batch}.npz"), seed=seed,
                            M=M, K=K, batch=batch, **bfp8_case(seed, M, K, batch))
    print("written to", HERE)


if __name__ == "__main__":
    main()
