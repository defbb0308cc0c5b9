"""GPU parity of the BFP8_B path (include/qbfp8.h) against the CPU oracle:
the on-device packer byte for byte, and the GEMV family within the output
tolerance (f32 accumulation in a different order, one bf16 rounding)."""
import numpy as np
import pytest
import torch

from gpu_util import KEEP, dev, host_u16

pytestmark = pytest.mark.gpu

# y is bf16: within one bf16 rounding of the oracle's f32 sum plus a small
# f32 reordering term; the parity gate of the path (max-abs 2e-2, rel 1e-2)
# is checked as well.
def assert_gemv_close(got_bits, y32, synth):
    got = synth.bf16_to_f32(got_bits).reshape(y32.shape).astype(np.float64)
    ref = y32.astype(np.float64)
    scale = np.abs(ref).max()
    err = np.abs(got - ref)
    assert np.all(err <= 2.0 ** -8 * np.abs(ref) + 1e-5 * scale), err.max()
    np.testing.assert_allclose(got, ref, atol=2e-2, rtol=1e-2)


def upload(qcache, oracle, synth, seed, M, K):
    w = synth.bfp8_weights(seed, M, K)
    packed = oracle.bfp8_pack(w)
    m = qcache.Bfp8Matrix(M, K)
    m.upload(packed.ctypes.data)
    torch.cuda.synchronize()
    return m, packed, w


@pytest.mark.parametrize("M,K", [(64, 96), (12352, 4096), (96, 1024)])
def test_pack_on_device_is_byte_exact(qcache, oracle, synth, M, K):
    w = synth.bfp8_weights(40 + M % 7, M, K)
    m = qcache.Bfp8Matrix(M, K)
    m.pack_bf16(dev(w).data_ptr())
    m.check()
    got = np.empty(qcache.Bfp8Matrix.packed_bytes(M, K), np.uint8)
    m.download(got.ctypes.data)
    torch.cuda.synchronize()
    assert np.array_equal(got, oracle.bfp8_pack(w))


@pytest.mark.parametrize("M,K,B", [(64, 96, 1), (96, 64, 3), (4096, 4096, 1), (12352, 4096, 1),
                                   (10240, 4096, 8), (4096, 12288, 2), (1024, 4096, 16),
                                   (2048, 4096, 17), (512, 4096, 64)])
def test_gemv_matches_oracle(qcache, oracle, synth, M, K, B):
    m, packed, _ = upload(qcache, oracle, synth, 50 + B, M, K)
    x = synth.gemv_inputs(50 + B, B, K)
    y = torch.zeros(B, M, dtype=torch.int16, device="cuda")
    m.gemv(dev(x).data_ptr(), B, y.data_ptr())
    m.check()
    _, y32 = oracle.bfp8_gemv(packed, M, K, x, n_threads=8, fast=True)
    assert_gemv_close(host_u16(y), y32, synth)


def test_golden_fixtures_on_device(qcache, synth):
    import glob, os
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    for path in sorted(glob.glob(os.path.join(here, "bfp8_*.npz"))):
        g = np.load(path)
        seed, M, K, B = int(g["seed"]), int(g["M"]), int(g["K"]), int(g["batch"])
        m = qcache.Bfp8Matrix(M, K)
        m.pack_bf16(dev(synth.bfp8_weights(seed, M, K)).data_ptr())
        got = np.empty(g["packed"].size, np.uint8)
        m.download(got.ctypes.data)
        torch.cuda.synchronize()
        assert np.array_equal(got, g["packed"]), path
        y = torch.zeros(B, M, dtype=torch.int16, device="cuda")
        m.gemv(dev(synth.gemv_inputs(seed, B, K)).data_ptr(), B, y.data_ptr())
        assert_gemv_close(host_u16(y), g["y32"], synth)


def test_resadd_in_place(qcache, oracle, synth):
    M, K, B = 4096, 4096, 2
    m, packed, _ = upload(qcache, oracle, synth, 61, M, K)
    x = synth.gemv_inputs(61, B, K)
    res = synth.bf16_bits(synth.normal(611, (B, M)))
    r = dev(res)
    m.gemv_resadd(dev(x).data_ptr(), B, r.data_ptr())
    m.check()
    got = host_u16(r)
    want, y32 = oracle.bfp8_gemv(packed, M, K, x, residual_bits=res, n_threads=8, fast=True)
    # the two roundings (RNE of Wx, truncation of the sum) follow the oracle;
    # the GPU's f32 sum may sit one bf16 step away before the first rounding
    exact = np.mean(got == want)
    assert exact > 0.95, exact
    ref = synth.bf16_to_f32(res).astype(np.float64) + y32
    np.testing.assert_allclose(synth.bf16_to_f32(got), ref, atol=2e-2, rtol=1e-2)


def test_split_outputs(qcache, oracle, synth):
    M, K, B, split = 2 * 1024, 4096, 3, 1024        # the fused gate|up layout
    m, packed, _ = upload(qcache, oracle, synth, 62, M, K)
    x = synth.gemv_inputs(62, B, K)
    y0 = torch.zeros(B, split, dtype=torch.int16, device="cuda")
    y1 = torch.zeros(B, M - split, dtype=torch.int16, device="cuda")
    m.gemv_split(dev(x).data_ptr(), B, split, y0.data_ptr(), y1.data_ptr())
    m.check()
    _, y32 = oracle.bfp8_gemv(packed, M, K, x, n_threads=8, fast=True)
    assert_gemv_close(host_u16(y0), y32[:, :split], synth)
    assert_gemv_close(host_u16(y1), y32[:, split:], synth)


def test_deterministic_and_graph_replay(qcache, oracle, synth):
    """Same bits on every call (fixed-order split-K merge), including replays
    of a captured CUDA graph, which also exercises the counter reset."""
    M, K, B = 12352, 4096, 4
    m, _, _ = upload(qcache, oracle, synth, 63, M, K)
    x = dev(synth.gemv_inputs(63, B, K))
    y = torch.zeros(B, M, dtype=torch.int16, device="cuda")
    m.gemv(x.data_ptr(), B, y.data_ptr())
    first = host_u16(y).copy()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        m.gemv(x.data_ptr(), B, y.data_ptr(), s.cuda_stream)   # warm-up on the capture stream
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            m.gemv(x.data_ptr(), B, y.data_ptr(), s.cuda_stream)
    for _ in range(3):
        y.zero_()
        g.replay()
        assert np.array_equal(host_u16(y), first)
    m.check()


def test_bad_split_and_batch(qcache):
    m = qcache.Bfp8Matrix(64, 64)
    with pytest.raises(qcache.QCacheError):
        m.gemv_split(16, 1, 64, 16, 16)
    with pytest.raises(qcache.QCacheError):
        m.gemv(16, 0, 16)
    KEEP.clear()
