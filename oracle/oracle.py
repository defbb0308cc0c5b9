"""ctypes binding of the CPU oracle (oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, never by the product.  Parity status: unpinned
by reference tests (the reference ships no golden vectors for this path); see
the header of oracle.cpp.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
EXACT, REF_APPROX = 0, 1

_libs = {}


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib(fast: bool = False) -> C.CDLL:
    name = "liboracle_fast.so" if fast else "liboracle.so"
    if name in _libs:
        return _libs[name]
    path = os.path.join(HERE, name)
    if not os.path.exists(path):
        build()
    L = C.CDLL(path)
    P = C.c_void_p
    I = C.c_int
    sig = {
        "qo_bf16_round": (None, [P, P, C.c_int64]),
        "qo_bf16_trunc": (None, [P, P, C.c_int64]),
        "qo_bf16_widen": (None, [P, P, C.c_int64]),
        "qo_fast_expf": (C.c_float, [C.c_float]),
        "qo_rope_table": (None, [I, P, P]),
        "qo_k_append": (None, [P, P, I, P]),
        "qo_attn_decode": (None, [P, P, P, I, P, P, P, I]),
        "qo_attn_partial": (None, [P, P, I, P, P, I, I, P]),
        "qo_attn_combine": (None, [P, I, P, P]),
        "qo_gdn_decode": (None, [P, P, P, P, P, P, P, P, I]),
        "qo_gdn_decode_batch": (None, [I, P, P, P, P, P, P, P, P, I, I]),
        "qo_attn_decode_batch": (None, [I, P, P, P, P, P, P, C.c_int64, P, I, I]),
        "qo_prefix_decide": (I, [P, I, P, I, P]),
    }
    for k, (r, a) in sig.items():
        f = getattr(L, k)
        f.restype = r
        f.argtypes = a
    _libs[name] = L
    return L


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def rope_table(pos: int):
    cs = np.zeros(32, np.float32)
    sn = np.zeros(32, np.float32)
    lib().qo_rope_table(pos, _p(cs), _p(sn))
    return cs, sn


def k_append(k_proj_bits: np.ndarray, k_norm: np.ndarray, pos: int) -> np.ndarray:
    out = np.zeros(1024, np.uint16)
    lib().qo_k_append(_p(np.ascontiguousarray(k_proj_bits, np.uint16)),
                      _p(np.ascontiguousarray(k_norm, np.float32)), pos, _p(out))
    return out


def attn_decode(proj_bits, q_norm, k_norm, pos, k_cache, v_cache, mode=EXACT):
    """One attention step.  k_cache / v_cache: uint16 [>= pos + 1][4][256], row
    pos is overwritten with the append.  Returns out [4096] f32."""
    out = np.zeros(4096, np.float32)
    assert k_cache.shape[0] > pos and v_cache.shape[0] > pos
    lib().qo_attn_decode(_p(np.ascontiguousarray(proj_bits, np.uint16)),
                         _p(np.ascontiguousarray(q_norm, np.float32)),
                         _p(np.ascontiguousarray(k_norm, np.float32)), pos, _p(k_cache),
                         _p(v_cache), _p(out), mode)
    return out


def attn_partial(proj_bits, q_norm, pos, k_cache, v_cache, p_begin, p_end):
    out = np.zeros((16, 258), np.float32)
    lib().qo_attn_partial(_p(np.ascontiguousarray(proj_bits, np.uint16)),
                          _p(np.ascontiguousarray(q_norm, np.float32)), pos, _p(k_cache),
                          _p(v_cache), p_begin, p_end, _p(out))
    return out


def attn_combine(partials: np.ndarray, proj_bits) -> np.ndarray:
    partials = np.ascontiguousarray(partials, np.float32)
    out = np.zeros(4096, np.float32)
    lib().qo_attn_combine(_p(partials), partials.shape[0],
                          _p(np.ascontiguousarray(proj_bits, np.uint16)), _p(out))
    return out


def gdn_decode(proj_bits, state, hist_f32, params, mode=EXACT):
    """One DeltaNet step.  state [32][128][128] f32 and hist_f32 [3][8192] f32
    are updated in place.  Returns out [4096] f32."""
    out = np.zeros(4096, np.float32)
    lib().qo_gdn_decode(_p(np.ascontiguousarray(proj_bits, np.uint16)), _p(state), _p(hist_f32),
                        _p(params["conv_w"]), _p(params["ssm_a"]), _p(params["dt_bias"]),
                        _p(params["ssm_norm"]), _p(out), mode)
    return out


def prefix_decide(cached, prompt):
    c = np.ascontiguousarray(cached, np.int32)
    p = np.ascontiguousarray(prompt, np.int32)
    reset = C.c_int()
    n = lib().qo_prefix_decide(_p(c), len(c), _p(p), len(p), C.byref(reset))
    return n, bool(reset.value)
