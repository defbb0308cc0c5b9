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


def host_has_avx512() -> bool:
    """True when the host CPU reports every x86-64-v4 feature (AVX-512 F, BW,
    CD, DQ, VL), so the AVX-512 build of the timed baseline may run."""
    try:
        with open("/proc/cpuinfo") as f:
            flags = next((ln.split(":", 1)[1].split() for ln in f if ln.startswith("flags")), [])
    except OSError:
        return False
    return {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= set(flags)


def fast_build_name() -> str:
    """The timed-baseline build this host runs: AVX-512 when it can."""
    return "liboracle_fast512.so" if host_has_avx512() else "liboracle_fast.so"


def lib(fast: bool = False) -> C.CDLL:
    name = fast_build_name() if fast else "liboracle.so"
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
        "qo_bfp8_packed_bytes": (C.c_int64, [I, I]),
        "qo_bfp8_pack": (None, [P, I, I, P]),
        "qo_bfp8_unpack": (None, [P, I, I, P]),
        "qo_bfp8_gemv": (None, [P, I, I, P, I, I, P, P, I]),
        "qo_exp_ref": (C.c_double, [C.c_double]),
        "qo_sample_mass": (C.c_uint32, [C.c_float, C.c_float, C.c_float]),
        "qo_sample": (C.c_int32, [P, I, C.c_float, C.c_float, C.c_double, P]),
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


def bfp8_pack(w_bits: np.ndarray) -> np.ndarray:
    """bf16 bits [M][K] -> BFP8_B tiles (uint8, GGUF type-200 layout)."""
    w = np.ascontiguousarray(w_bits, np.uint16)
    M, K = w.shape
    out = np.zeros(lib().qo_bfp8_packed_bytes(M, K), np.uint8)
    lib().qo_bfp8_pack(_p(w), M, K, _p(out))
    return out


def bfp8_unpack(packed: np.ndarray, M: int, K: int) -> np.ndarray:
    w = np.zeros((M, K), np.float32)
    lib().qo_bfp8_unpack(_p(np.ascontiguousarray(packed, np.uint8)), M, K, _p(w))
    return w


def bfp8_gemv(packed, M, K, x_bits, residual_bits=None, n_threads=1, fast=False):
    """y = W x for x bf16 bits [B][K]; with residual_bits, the reference's
    resadd rounding.  Returns (y bf16 bits [B][M], y32 f32 [B][M])."""
    x = np.ascontiguousarray(x_bits, np.uint16).reshape(-1, K)
    B = x.shape[0]
    y = (np.zeros((B, M), np.uint16) if residual_bits is None
         else np.array(residual_bits, np.uint16).reshape(B, M).copy())
    y32 = np.zeros((B, M), np.float32)
    lib(fast).qo_bfp8_gemv(_p(np.ascontiguousarray(packed, np.uint8)), M, K, _p(x), B,
                           0 if residual_bits is None else 1, _p(y), _p(y32), n_threads)
    return y, y32


def sample(logits_bits, temperature, top_p=0.9, u=0.0):
    """One row: (token, nucleus size) of the restated sample_token."""
    lg = np.ascontiguousarray(logits_bits, np.uint16).reshape(-1)
    kept = C.c_int32()
    tok = lib().qo_sample(_p(lg), lg.size, temperature, top_p, float(u), C.byref(kept))
    return tok, kept.value


def exp_ref(x: float) -> float:
    return lib().qo_exp_ref(float(x))
