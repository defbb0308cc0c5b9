"""Helpers for the GPU tests: device buffers from numpy and back, tolerances."""
import numpy as np
import torch

# Output tolerance of the parity gate: max-abs 2e-2 / rel 1e-2 on the bf16
# outputs; the fp32 DeltaNet state within 1e-4 relative.
OUT_ATOL, OUT_RTOL = 2e-2, 1e-2
STATE_RTOL = 1e-4


# Device copies made by dev() stay referenced until the test ends, so that a
# pointer taken from a temporary (dev(x).data_ptr()) stays valid while the
# asynchronous kernels that read it run.
KEEP = []


def dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()
    KEEP.append(t)
    return t


def host_u16(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint16)


def host_f32(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def empty_u16(*shape) -> torch.Tensor:
    return torch.zeros(*shape, dtype=torch.int16, device="cuda")


def assert_out_close(got_bits: np.ndarray, ref_f32: np.ndarray, synth):
    got = synth.bf16_to_f32(got_bits).reshape(ref_f32.shape)
    np.testing.assert_allclose(got, ref_f32, atol=OUT_ATOL, rtol=OUT_RTOL)


def assert_state_close(got: np.ndarray, ref: np.ndarray):
    scale = np.abs(ref).max()
    err = np.abs(got - ref)
    assert err.max() <= STATE_RTOL * scale, (err.max(), scale)
    np.testing.assert_allclose(got, ref, rtol=STATE_RTOL, atol=STATE_RTOL * 1e-2 * scale)


def permute_free_pages(q, n_pages: int, seed: int):
    """Leave the context's page free list in a seeded random order, so that
    later allocations map logical pages to permuted physical pages."""
    rng = np.random.default_rng(seed)
    seqs = [q.seq_alloc() for _ in range(n_pages)]
    for s in seqs:
        q.seq_reserve(s, 1)
    for i in rng.permutation(n_pages):
        q.seq_free(seqs[i])
