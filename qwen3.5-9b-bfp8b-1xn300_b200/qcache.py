"""ctypes binding of libqcache.so (include/qcache.h) for tests and benchmarks.

The engine-side caller of this library is C++ (the reference's
src/engine.cpp); this module only gives Python the same C entry points.  Device
buffers are passed as integer addresses (e.g. torch.Tensor.data_ptr()), streams
as cudaStream_t handles (torch.cuda.Stream.cuda_stream).  Every non-zero status
raises QCacheError with the library's message.  There is no fallback: if the
shared library is missing the import of this module fails.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqcache.so")
HEADERS = [os.path.join(HERE, "..", "include", h) for h in ("qcache.h", "qbfp8.h", "qsample.h")]

QC_OK, QC_ERR_ARG, QC_ERR_OOM, QC_ERR_CUDA, QC_ERR_TIMEOUT, QC_ERR_BOUNDS, QC_ERR_NODEVICE = range(7)
QC_FLAG_REFERENCE_MATH = 1
DEVICE_NONE = -1
N_HEAD, N_HEAD_KV, HEAD_DIM = 16, 4, 256
ATTN_PROJ, ATTN_OUT = 10240, 4096
GDN_PROJ, GDN_OUT = 12352, 4096
GDN_STATE = 32 * 128 * 128
CONV_CH = 8192
PAGE = 64


class QCacheError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"qcache error {code}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [
        ("n_attn_layers", C.c_int32),
        ("n_gdn_layers", C.c_int32),
        ("max_seqs", C.c_int32),
        ("max_pages", C.c_int32),
        ("max_ctx", C.c_int32),
        ("max_batch", C.c_int32),
        ("max_snapshots", C.c_int32),
        ("flags", C.c_int32),
    ]


_lib = None

P = C.c_void_p
I32 = C.c_int32
PI32 = C.POINTER(C.c_int32)


def header_functions() -> list[str]:
    """Names of every function the headers in include/ declare."""
    text = ""
    for h in HEADERS:
        with open(h) as f:
            text += f.read()
    pat = r"^\s*(?:int64_t|int|void\s*\*|void|const char\*)\s*(qc_\w+)\s*\("
    return sorted(set(re.findall(pat, text, re.M)))


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built (run __graft_entry__.build())")
    L = C.CDLL(LIB_PATH)
    sig = {
        "qc_create": (C.c_int, [C.POINTER(Config), C.c_int, C.POINTER(P)]),
        "qc_destroy": (None, [P]),
        "qc_last_error": (C.c_char_p, [P]),
        "qc_check_device": (C.c_int, [P, P]),
        "qc_set_attn_params": (C.c_int, [P, C.c_int, P, P]),
        "qc_set_gdn_params": (C.c_int, [P, C.c_int, P, P, P, P]),
        "qc_seq_alloc": (C.c_int, [P, PI32]),
        "qc_seq_free": (C.c_int, [P, I32]),
        "qc_seq_reset": (C.c_int, [P, I32, P]),
        "qc_seq_len": (C.c_int, [P, I32, PI32]),
        "qc_seq_pages": (C.c_int, [P, I32, PI32, I32, PI32]),
        "qc_seq_reserve": (C.c_int, [P, I32, I32]),
        "qc_kv_write": (C.c_int, [P, I32, C.c_int, I32, I32, P, P, P]),
        "qc_kv_read": (C.c_int, [P, I32, C.c_int, I32, I32, P, P, P]),
        "qc_gdn_state_write": (C.c_int, [P, I32, C.c_int, P, P, P]),
        "qc_gdn_state_read": (C.c_int, [P, I32, C.c_int, P, P, P]),
        "qc_decode_begin": (C.c_int, [P, PI32, I32, PI32, P]),
        "qc_attn_decode": (C.c_int, [P, C.c_int, P, P, P]),
        "qc_gdn_decode": (C.c_int, [P, C.c_int, P, P, P]),
        "qc_decode_end": (C.c_int, [P]),
        "qc_decode_abort": (C.c_int, [P]),
        "qc_prefill_begin": (C.c_int, [P, I32, I32, PI32, P]),
        "qc_attn_prefill": (C.c_int, [P, C.c_int, P, P, P]),
        "qc_gdn_prefill": (C.c_int, [P, C.c_int, P, P, P]),
        "qc_prefill_end": (C.c_int, [P]),
        "qc_seq_match_prefix": (C.c_int, [P, I32, PI32, I32, PI32, P]),
        "qc_prefix_insert": (C.c_int, [P, I32, PI32, I32, PI32, P]),
        "qc_prefix_lookup": (C.c_int, [P, PI32, I32, PI32, PI32]),
        "qc_prefix_restore": (C.c_int, [P, PI32, PI32, I32, P]),
        "qc_prefix_release": (C.c_int, [P, I32]),
        "qc_prefix_last_restore_bytes": (C.c_int, [P, C.POINTER(C.c_int64)]),
        "qc_prefix_page_hashes": (C.c_int, [PI32, I32, C.POINTER(C.c_uint64)]),
        "qc_attn_partial_range": (C.c_int, [P, I32, I32, I32, P]),
        "qc_attn_partial": (C.c_int, [P, C.c_int, P, P, P]),
        "qc_attn_combine": (C.c_int, [P, P, I32, P, P, P]),
        "qc_p2p_create": (C.c_int, [P, I32, I32, P]),
        "qc_p2p_open": (C.c_int, [P, I32, P]),
        "qc_attn_partial_p2p": (C.c_int, [P, C.c_int, P, P]),
        "qc_attn_combine_p2p": (C.c_int, [P, C.c_int, P, P, P]),
        "qc_p2p_reset": (C.c_int, [P, P]),
        "qc_attn_decode_noalloc": (C.c_int, [P, P, P, I32, P, I32, PI32, I32, P, P, P, P, P, P]),
        "qc_attn_noalloc_check": (C.c_int, [P]),
        "qc_attn_select_kernel": (C.c_int, [C.c_int]),
        "qc_bfp8_packed_bytes": (C.c_int64, [I32, I32]),
        "qc_bfp8_create": (C.c_int, [C.c_int, I32, I32, C.POINTER(P)]),
        "qc_bfp8_destroy": (None, [P]),
        "qc_bfp8_tiles": (P, [P]),
        "qc_bfp8_upload": (C.c_int, [P, P, P]),
        "qc_bfp8_download": (C.c_int, [P, P, P]),
        "qc_bfp8_pack_bf16": (C.c_int, [P, P, P]),
        "qc_bfp8_gemv": (C.c_int, [P, P, I32, P, P]),
        "qc_bfp8_gemv_resadd": (C.c_int, [P, P, I32, P, P]),
        "qc_bfp8_gemv_split": (C.c_int, [P, P, I32, I32, P, P, P]),
        "qc_bfp8_check": (C.c_int, [P]),
        "qc_sample": (C.c_int, [P, C.c_int64, I32, I32, C.c_float, C.c_float, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _i32arr(xs):
    """int32 C array from a numpy array (no copy when already int32) or a list."""
    try:
        import numpy as np
        if isinstance(xs, np.ndarray):
            a = np.ascontiguousarray(xs, dtype=np.int32)
            return a.ctypes.data_as(PI32)
    except ImportError:
        pass
    xs = [int(x) for x in xs]
    return (C.c_int32 * max(1, len(xs)))(*xs)


def _f32ptr(a):
    """numpy float32 array -> pointer (keeps the caller's array alive)."""
    return a.ctypes.data_as(C.c_void_p)


class QCache:
    """One context on one GPU (or a host-only context with device=-1)."""

    def __init__(self, n_attn_layers=8, n_gdn_layers=24, max_seqs=64, max_pages=4096,
                 max_ctx=8192, max_batch=64, max_snapshots=16, device=0, flags=0):
        self.L = lib()
        self.cfg = Config(n_attn_layers, n_gdn_layers, max_seqs, max_pages, max_ctx, max_batch,
                          max_snapshots, flags)
        h = C.c_void_p()
        rc = self.L.qc_create(C.byref(self.cfg), device, C.byref(h))
        if rc:
            raise QCacheError(rc, self.L.qc_last_error(None).decode())
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self.L.qc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _ck(self, rc):
        if rc:
            raise QCacheError(rc, self.L.qc_last_error(self.h).decode())

    # ---- parameters
    def set_attn_params(self, layer, q_norm, k_norm):
        self._ck(self.L.qc_set_attn_params(self.h, layer, _f32ptr(q_norm), _f32ptr(k_norm)))

    def set_gdn_params(self, layer, ssm_a, dt_bias, ssm_norm, conv_w):
        self._ck(self.L.qc_set_gdn_params(self.h, layer, _f32ptr(ssm_a), _f32ptr(dt_bias),
                                          _f32ptr(ssm_norm), _f32ptr(conv_w)))

    def check_device(self, stream=0):
        self._ck(self.L.qc_check_device(self.h, stream))

    # ---- sequences
    def seq_alloc(self) -> int:
        s = C.c_int32()
        self._ck(self.L.qc_seq_alloc(self.h, C.byref(s)))
        return s.value

    def seq_free(self, s):
        self._ck(self.L.qc_seq_free(self.h, s))

    def seq_reset(self, s, stream=0):
        self._ck(self.L.qc_seq_reset(self.h, s, stream))

    def seq_len(self, s) -> int:
        n = C.c_int32()
        self._ck(self.L.qc_seq_len(self.h, s, C.byref(n)))
        return n.value

    def seq_pages(self, s) -> list[int]:
        n = C.c_int32()
        self._ck(self.L.qc_seq_pages(self.h, s, None, 0, C.byref(n)))
        arr = (C.c_int32 * max(1, n.value))()
        self._ck(self.L.qc_seq_pages(self.h, s, arr, n.value, C.byref(n)))
        return list(arr[: n.value])

    def seq_reserve(self, s, new_len):
        self._ck(self.L.qc_seq_reserve(self.h, s, new_len))

    def kv_write(self, s, layer, pos0, n, k_ptr, v_ptr, stream=0):
        self._ck(self.L.qc_kv_write(self.h, s, layer, pos0, n, k_ptr, v_ptr, stream))

    def kv_read(self, s, layer, pos0, n, k_ptr, v_ptr, stream=0):
        self._ck(self.L.qc_kv_read(self.h, s, layer, pos0, n, k_ptr, v_ptr, stream))

    def gdn_state_write(self, s, layer, state_ptr, hist_ptr, stream=0):
        self._ck(self.L.qc_gdn_state_write(self.h, s, layer, state_ptr, hist_ptr, stream))

    def gdn_state_read(self, s, layer, state_ptr, hist_ptr, stream=0):
        self._ck(self.L.qc_gdn_state_read(self.h, s, layer, state_ptr, hist_ptr, stream))

    # ---- decode step
    def decode_begin(self, seqs, tokens=None, stream=0):
        arr = _i32arr(seqs)
        tok = _i32arr(tokens) if tokens is not None else None
        self._ck(self.L.qc_decode_begin(self.h, arr, len(seqs), tok, stream))

    def attn_decode(self, layer, proj_ptr, out_ptr, stream=0):
        self._ck(self.L.qc_attn_decode(self.h, layer, proj_ptr, out_ptr, stream))

    def gdn_decode(self, layer, proj_ptr, out_ptr, stream=0):
        self._ck(self.L.qc_gdn_decode(self.h, layer, proj_ptr, out_ptr, stream))

    def decode_end(self):
        self._ck(self.L.qc_decode_end(self.h))

    def decode_abort(self):
        self._ck(self.L.qc_decode_abort(self.h))

    # ---- prefill
    def prefill_begin(self, s, n, tokens=None, stream=0):
        tok = _i32arr(tokens) if tokens is not None else None
        self._ck(self.L.qc_prefill_begin(self.h, s, n, tok, stream))

    def attn_prefill(self, layer, proj_ptr, out_ptr, stream=0):
        self._ck(self.L.qc_attn_prefill(self.h, layer, proj_ptr, out_ptr, stream))

    def gdn_prefill(self, layer, proj_ptr, out_ptr, stream=0):
        self._ck(self.L.qc_gdn_prefill(self.h, layer, proj_ptr, out_ptr, stream))

    def prefill_end(self):
        self._ck(self.L.qc_prefill_end(self.h))

    # ---- prefix cache
    def match_prefix(self, s, tokens, stream=0) -> int:
        out = C.c_int32()
        self._ck(self.L.qc_seq_match_prefix(self.h, s, _i32arr(tokens), len(tokens),
                                            C.byref(out), stream))
        return out.value

    def prefix_insert(self, s, tokens, stream=0) -> int:
        e = C.c_int32()
        self._ck(self.L.qc_prefix_insert(self.h, s, _i32arr(tokens), len(tokens), C.byref(e),
                                         stream))
        return e.value

    def prefix_lookup(self, tokens):
        m, e = C.c_int32(), C.c_int32()
        self._ck(self.L.qc_prefix_lookup(self.h, _i32arr(tokens), len(tokens), C.byref(m),
                                         C.byref(e)))
        return m.value, e.value

    def prefix_restore(self, entries, seqs, stream=0):
        self._ck(self.L.qc_prefix_restore(self.h, _i32arr(entries), _i32arr(seqs), len(seqs),
                                          stream))

    def prefix_release(self, entry):
        self._ck(self.L.qc_prefix_release(self.h, entry))

    def last_restore_bytes(self) -> int:
        b = C.c_int64()
        self._ck(self.L.qc_prefix_last_restore_bytes(self.h, C.byref(b)))
        return b.value

    # ---- split-K across devices
    def attn_partial_range(self, page_begin, page_end, append, stream=0):
        self._ck(self.L.qc_attn_partial_range(self.h, page_begin, page_end, append, stream))

    def attn_partial(self, layer, proj_ptr, partial_ptr, stream=0):
        self._ck(self.L.qc_attn_partial(self.h, layer, proj_ptr, partial_ptr, stream))

    def p2p_create(self, world, rank) -> bytes:
        """Allocates the peer mailbox; returns its IPC handle for the peers."""
        buf = (C.c_char * 64)()
        self._ck(self.L.qc_p2p_create(self.h, world, rank, buf))
        return bytes(buf)

    def p2p_open(self, peer, handle: bytes):
        buf = (C.c_char * 64).from_buffer_copy(handle)
        self._ck(self.L.qc_p2p_open(self.h, peer, buf))

    def attn_partial_p2p(self, layer, proj_ptr, stream=0):
        self._ck(self.L.qc_attn_partial_p2p(self.h, layer, proj_ptr, stream))

    def attn_combine_p2p(self, layer, proj_ptr, out_ptr, stream=0):
        self._ck(self.L.qc_attn_combine_p2p(self.h, layer, proj_ptr, out_ptr, stream))

    def p2p_reset(self, stream=0):
        self._ck(self.L.qc_p2p_reset(self.h, stream))

    def attn_combine(self, partials_ptr, n_parts, proj_ptr, out_ptr, stream=0):
        self._ck(self.L.qc_attn_combine(self.h, partials_ptr, n_parts, proj_ptr, out_ptr, stream))


def page_hashes(tokens) -> list[int]:
    n = len(tokens)
    out = (C.c_uint64 * max(1, n // PAGE))()
    rc = lib().qc_prefix_page_hashes(_i32arr(tokens), n, out)
    if rc:
        raise QCacheError(rc, "qc_prefix_page_hashes")
    return list(out[: n // PAGE])


def attn_decode_noalloc(proj_ptr, k_pool_ptr, v_pool_ptr, max_pages, page_table_ptr, pt_stride,
                        pos, q_norm_ptr, k_norm_ptr, rope_cos_ptr, rope_sin_ptr, out_ptr,
                        stream=0):
    """qc_attn_decode_noalloc: attention decode over caller-owned buffers, with
    no device allocation (see include/qcache.h)."""
    L = lib()
    rc = L.qc_attn_decode_noalloc(proj_ptr, k_pool_ptr, v_pool_ptr, max_pages, page_table_ptr,
                                  pt_stride, _i32arr(pos), len(pos), q_norm_ptr, k_norm_ptr,
                                  rope_cos_ptr, rope_sin_ptr, out_ptr, stream)
    if rc:
        raise QCacheError(rc, L.qc_last_error(None).decode())


def attn_noalloc_check(stream=0):
    """qc_attn_noalloc_check: raise the error the no-allocation kernels
    recorded on the current device since the last check (and clear it)."""
    rc = lib().qc_attn_noalloc_check(stream)
    if rc:
        raise QCacheError(rc, lib().qc_last_error(None).decode())


ATTN_KERNEL_AUTO, ATTN_KERNEL_MMA, ATTN_KERNEL_TC = 0, 1, 2


def attn_select_kernel(mode):
    """qc_attn_select_kernel: pick the decode-attention kernel process-wide
    (auto / mma.sync / tcgen05); returns the previous mode."""
    rc = lib().qc_attn_select_kernel(mode)
    if rc < 0:
        raise QCacheError(-rc, f"unknown attention kernel mode {mode}")
    return rc


class Bfp8Matrix:
    """One BFP8_B weight matrix on one GPU (include/qbfp8.h)."""

    def __init__(self, M: int, K: int, device: int = 0):
        self.M, self.K = M, K
        self._m = P()
        rc = lib().qc_bfp8_create(device, M, K, C.byref(self._m))
        if rc:
            raise QCacheError(rc, lib().qc_last_error(None).decode())

    def close(self):
        if self._m:
            lib().qc_bfp8_destroy(self._m)
            self._m = P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _ck(self, rc):
        if rc:
            raise QCacheError(rc, lib().qc_last_error(None).decode())

    @staticmethod
    def packed_bytes(M: int, K: int) -> int:
        return lib().qc_bfp8_packed_bytes(M, K)

    @property
    def tiles_ptr(self) -> int:
        return lib().qc_bfp8_tiles(self._m)

    def upload(self, host_ptr, stream=0):
        self._ck(lib().qc_bfp8_upload(self._m, host_ptr, stream))

    def download(self, host_ptr, stream=0):
        self._ck(lib().qc_bfp8_download(self._m, host_ptr, stream))

    def pack_bf16(self, w_ptr, stream=0):
        self._ck(lib().qc_bfp8_pack_bf16(self._m, w_ptr, stream))

    def gemv(self, x_ptr, batch, y_ptr, stream=0):
        self._ck(lib().qc_bfp8_gemv(self._m, x_ptr, batch, y_ptr, stream))

    def gemv_resadd(self, x_ptr, batch, residual_ptr, stream=0):
        self._ck(lib().qc_bfp8_gemv_resadd(self._m, x_ptr, batch, residual_ptr, stream))

    def gemv_split(self, x_ptr, batch, split_m, y0_ptr, y1_ptr, stream=0):
        self._ck(lib().qc_bfp8_gemv_split(self._m, x_ptr, batch, split_m, y0_ptr, y1_ptr, stream))

    def check(self):
        self._ck(lib().qc_bfp8_check(self._m))


def sample(logits_ptr, ld, vocab, batch, temperature, top_p, uniform_ptr, tokens_ptr, stream=0):
    """qc_sample (include/qsample.h): one token per row of bf16 logits."""
    L = lib()
    rc = L.qc_sample(logits_ptr, ld, vocab, batch, temperature, top_p, uniform_ptr, tokens_ptr,
                     stream)
    if rc:
        raise QCacheError(rc, L.qc_last_error(None).decode())
