"""CPU tests of the BFP8_B oracle (oracle/bfp8.cpp): known-answer tiles, the
format's layout, packing properties, the GEMV against float64 numpy, the
committed golden fixtures, and the C ABI's host-side checks."""
import ctypes as C
import glob
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def one_tile(rows):
    """A 32x32 bf16 matrix whose first rows are given (rest zero)."""
    w = np.zeros((32, 32), np.float32)
    for i, r in enumerate(rows):
        w[i, : len(r)] = r
    return w


def test_known_answer_bytes(oracle, synth):
    w = one_tile([[1.0, 0.5, -0.25, 0.0, 1.9921875, 0.75]])
    t = oracle.bfp8_pack(synth.bf16_bits(w))
    assert t.size == 1088
    assert t[0] == 127                            # face 0 row 0: shared exponent of 1.0..1.99
    assert list(t[64:70]) == [64, 32, 0x80 | 16, 0, 127, 48]   # 1.99 saturates at 127
    assert np.all(t[1:64] == 0) and np.all(t[70:] == 0)


def test_face_layout(oracle, synth):
    """Element (row, col) lands in face (row//16)*2 + col//16, byte
    64 + face*256 + (row%16)*16 + col%16; exponent at face*16 + row%16."""
    for row, col in [(0, 0), (5, 20), (20, 5), (31, 31), (16, 16)]:
        w = np.zeros((32, 32), np.float32)
        w[row, col] = 2.0
        t = oracle.bfp8_pack(synth.bf16_bits(w))
        f = (row // 16) * 2 + col // 16
        assert t[f * 16 + row % 16] == 128
        nz = np.nonzero(t[64:])[0]
        assert list(nz) == [f * 256 + (row % 16) * 16 + col % 16]
        assert t[64 + nz[0]] == 64


def test_tile_order_is_row_major(oracle, synth):
    M, K = 64, 96
    w = np.zeros((M, K), np.float32)
    w[33, 70] = 1.0                               # tile (1, 2)
    t = oracle.bfp8_pack(synth.bf16_bits(w)).reshape(-1, 1088)
    assert [i for i in range(t.shape[0]) if t[i].any()] == [1 * 3 + 2]


def test_decode_error_bound_and_idempotence(oracle, synth):
    M, K = 64, 128
    wb = synth.bfp8_weights(7, M, K)
    w = synth.bf16_to_f32(wb)
    p = oracle.bfp8_pack(wb)
    d = oracle.bfp8_unpack(p, M, K)
    # per face row: |w - d| <= half a step of 2^(e-133), except saturation at 127
    for r in range(M):
        for c0 in range(0, K, 16):
            seg = w[r, c0:c0 + 16]
            e = int(((synth.bf16_bits(seg).astype(np.uint32) >> 7) & 0xFF).max())
            step = 2.0 ** (e - 133)
            err = np.abs(seg - d[r, c0:c0 + 16])
            sat = np.abs(seg) >= 127.5 * step
            assert np.all(err[~sat] <= 0.5 * step * (1 + 1e-6)), (r, c0)
    # decoded values are bf16-exact, so packing them again gives the same bytes
    assert np.array_equal(oracle.bfp8_pack(synth.bf16_bits(d)), p)


def test_sign_of_rounded_zero_and_negative_zero(oracle, synth):
    w = one_tile([[1.0, -2.0 ** -12, -0.0]])
    t = oracle.bfp8_pack(synth.bf16_bits(w))
    assert t[64 + 1] == 0 and t[64 + 2] == 0


def test_gemv_matches_float64(oracle, synth):
    M, K, B = 96, 160, 5
    p = oracle.bfp8_pack(synth.bfp8_weights(3, M, K))
    x = synth.gemv_inputs(3, B, K)
    y, y32 = oracle.bfp8_gemv(p, M, K, x, n_threads=3)
    ref = synth.bf16_to_f32(x).astype(np.float64) @ oracle.bfp8_unpack(p, M, K).astype(np.float64).T
    np.testing.assert_allclose(y32, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    assert np.array_equal(y, synth.bf16_bits(y32))


def test_gemv_resadd_rounding(oracle, synth):
    """bf16_trunc(bf16_rne(Wx) + residual), as the reference writer does."""
    M, K = 64, 64
    p = oracle.bfp8_pack(synth.bfp8_weights(4, M, K))
    x = synth.gemv_inputs(4, 2, K)
    res = synth.bf16_bits(synth.normal(99, (2, M)))
    y, y32 = oracle.bfp8_gemv(p, M, K, x, residual_bits=res)
    s = synth.bf16_to_f32(synth.bf16_bits(y32)) + synth.bf16_to_f32(res)
    assert np.array_equal(y, (s.view(np.uint32) >> 16).astype(np.uint16))


def test_fast_build_agrees(oracle, synth):
    M, K = 64, 256
    p = oracle.bfp8_pack(synth.bfp8_weights(5, M, K))
    x = synth.gemv_inputs(5, 2, K)
    _, a = oracle.bfp8_gemv(p, M, K, x)
    _, b = oracle.bfp8_gemv(p, M, K, x, n_threads=4, fast=True)
    np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-4 * np.abs(a).max())


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "bfp8_*.npz"))))
def test_golden(oracle, synth, path):
    g = np.load(path)
    seed, M, K, B = int(g["seed"]), int(g["M"]), int(g["K"]), int(g["batch"])
    p = oracle.bfp8_pack(synth.bfp8_weights(seed, M, K))
    assert np.array_equal(p, g["packed"])
    x = synth.gemv_inputs(seed, B, K)
    y, y32 = oracle.bfp8_gemv(p, M, K, x)
    assert np.array_equal(y, g["y"])
    np.testing.assert_allclose(y32, g["y32"], rtol=1e-6, atol=1e-6 * np.abs(g["y32"]).max())
    res = synth.bf16_bits(synth.normal(seed * 8 + 3, (B, M)))
    y_res, _ = oracle.bfp8_gemv(p, M, K, x, residual_bits=res)
    assert np.array_equal(y_res, g["y_resadd"])


def test_golden_fixtures_present():
    assert len(glob.glob(os.path.join(GOLDEN, "bfp8_*.npz"))) >= 2


# ---------------------------------------------------------------- C ABI


def test_abi_packed_bytes(qcache):
    L = qcache.lib()
    assert L.qc_bfp8_packed_bytes(12352, 4096) == 386 * 128 * 1088
    assert L.qc_bfp8_packed_bytes(32, 32) == 1088
    assert L.qc_bfp8_packed_bytes(33, 32) == -1
    assert L.qc_bfp8_packed_bytes(0, 32) == -1


def test_abi_create_rejects_bad_shapes(qcache):
    with pytest.raises(qcache.QCacheError) as e:
        qcache.Bfp8Matrix(100, 64, device=0)
    assert e.value.code == qcache.QC_ERR_ARG


def test_abi_null_arguments(qcache):
    L = qcache.lib()
    assert L.qc_bfp8_gemv(None, None, 1, None, None) == qcache.QC_ERR_ARG
    assert L.qc_bfp8_check(None) == qcache.QC_ERR_ARG
    assert L.qc_bfp8_create(0, 32, 32, None) == qcache.QC_ERR_ARG
    assert L.qc_bfp8_tiles(None) is None
    L.qc_bfp8_destroy(None)


def test_abi_create_without_device(qcache):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    m = C.c_void_p()
    rc = qcache.lib().qc_bfp8_create(0, 64, 64, C.byref(m))
    assert rc == qcache.QC_ERR_NODEVICE and not m.value
