"""ctypes binding of oracle/_ref/libref.so: the reference's own cache-path host
code (src/engine.cpp blocks, compiled unchanged by ref_harness.cpp).

TEST INFRASTRUCTURE ONLY: used by tests/ (to pin the oracle), by
tests/golden/make_ref_golden.py (to write the reference fixtures) and by the
reference arm of bench.py (as the timed CPU implementation).  The library can
only be built where the reference source is present; `available()` says
whether it is here.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PATH = os.path.join(HERE, "_ref", "libref.so")
REF_SRC = os.environ.get("QC_REFERENCE_SRC", "/root/reference/src")
_lib = None


def _host_ok() -> bool:
    try:
        from oracle import host_has_avx512
    except ImportError:  # loaded by path
        import importlib.util
        spec = importlib.util.spec_from_file_location("_qo", os.path.join(HERE, "oracle.py"))
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        host_has_avx512 = m.host_has_avx512
    return host_has_avx512()


def build() -> bool:
    """Build libref.so when the reference source is here.  True if it exists."""
    if not os.path.exists(PATH) and os.path.exists(os.path.join(REF_SRC, "engine.cpp")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF_SRC=" + REF_SRC], check=True)
    return os.path.exists(PATH)


def available() -> bool:
    return build() and _host_ok()


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError("oracle/_ref/libref.so is not built (reference source absent) "
                               "or this host lacks AVX-512")
        L = C.CDLL(PATH)
        P, I = C.c_void_p, C.c_int
        L.ref_gdn_decode.argtypes = [P] * 8
        L.ref_gdn_decode.restype = None
        L.ref_attn_decode.argtypes = [P, P, P, I, P, P, P]
        L.ref_attn_decode.restype = None
        L.ref_prefix_rule.argtypes = [P, I, P, I, P]
        L.ref_prefix_rule.restype = I
        L.ref_rope_row.argtypes = [I, P, P]
        L.ref_rope_row.restype = None
        L.ref_set_layer.argtypes = [I, P, P, I, I, I, P, P]
        L.ref_set_layer.restype = None
        L.ref_gdn_decode_resident.argtypes = [I, P, P, P, P, P, P]
        L.ref_gdn_decode_resident.restype = None
        L.ref_attn_decode_resident.argtypes = [I, P, P, P, I, P]
        L.ref_attn_decode_resident.restype = None
        L.ref_fast_expf.argtypes = [C.c_float]
        L.ref_fast_expf.restype = C.c_float
        _lib = L
    return _lib


def _p(a):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def gdn_decode(proj_bits, state, hist_f32, params):
    """The reference's DeltaNet step.  proj_bits [12352] bf16 bits (widened to
    f32 as the reference's GEMV read-out does); state [32][128][128] f32 and
    hist_f32 [3][8192] f32 are updated in place.  Returns out [4096] f32."""
    proj = np.ascontiguousarray(_f32(proj_bits), np.float32)
    out = np.zeros(4096, np.float32)
    lib().ref_gdn_decode(_p(proj), _p(hist_f32), _p(state),
                         _p(np.ascontiguousarray(params["conv_w"], np.float32)),
                         _p(np.ascontiguousarray(params["ssm_a"], np.float32)),
                         _p(np.ascontiguousarray(params["dt_bias"], np.float32)),
                         _p(np.ascontiguousarray(params["ssm_norm"], np.float32)), _p(out))
    return out


def attn_decode(proj_bits, q_norm, k_norm, pos, k_cache_f32, v_cache_f32):
    """The reference's attention step at position pos.  k/v caches: f32
    [>= pos + 1][4][256]; row pos is overwritten with the (f32) append.
    Returns out [4096] f32."""
    assert k_cache_f32.dtype == np.float32 and k_cache_f32.shape[0] > pos
    proj = np.ascontiguousarray(_f32(proj_bits), np.float32)
    out = np.zeros(4096, np.float32)
    lib().ref_attn_decode(_p(proj), _p(np.ascontiguousarray(q_norm, np.float32)),
                          _p(np.ascontiguousarray(k_norm, np.float32)), pos, _p(k_cache_f32),
                          _p(v_cache_f32), _p(out))
    return out


def prefix_rule(cached, prompt):
    c = np.ascontiguousarray(cached, np.int32)
    p = np.ascontiguousarray(prompt, np.int32)
    r = C.c_int()
    n = lib().ref_prefix_rule(_p(c), len(c), _p(p), len(p), C.byref(r))
    return n, bool(r.value)


def rope_row(pos):
    cs, sn = np.zeros(32, np.float32), np.zeros(32, np.float32)
    lib().ref_rope_row(pos, _p(cs), _p(sn))
    return cs, sn


def fast_expf(x: float) -> float:
    return lib().ref_fast_expf(x)
