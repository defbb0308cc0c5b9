"""Seeded synthetic inputs for the cache path (no datasets, no weights).

SplitMix64 counters + Box-Muller in float64, then rounding to the stored
dtype, so every test and fixture is reproducible bit for bit on any machine.
The distributions are those of the benchmark configurations: K/V, q/k/v and
gates ~ N(0, 1); norm weights 1 + N(0, 0.02); DeltaNet state ~ N(0, 0.02);
conv weights ~ N(0, 0.1) (bf16-valued); ssm_a = -exp(N(-2, 0.5)); alpha,
beta ~ N(0, 1) with dt_bias = 0.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix64(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) * _M2 + np.arange(1, n + 1, dtype=np.uint64) * _GOLDEN
        x = x ^ (x >> np.uint64(30))
        x = x * _M1
        x = x ^ (x >> np.uint64(27))
        x = x * _M2
        x = x ^ (x >> np.uint64(31))
    return x


def uniform(seed: int, shape) -> np.ndarray:
    """float64 uniform in (0, 1]."""
    n = int(np.prod(shape))
    u = (_splitmix64(seed, n) >> np.uint64(11)).astype(np.float64)
    return ((u + 1.0) * (1.0 / 9007199254740992.0)).reshape(shape)


def normal(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """float64 N(mean, std^2) by Box-Muller."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u1 = uniform(seed, (m,))
    u2 = uniform(seed ^ 0x5DEECE66D, (m,))
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)])[:n]
    return (mean + std * z).reshape(shape)


def bf16_bits(x) -> np.ndarray:
    """float -> bf16 bit patterns (uint16), round to nearest even."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def attn_inputs(seed: int, n_seq: int, ctx: int):
    """Config-0 style inputs for n_seq sequences with `ctx` cached positions.

    Returns dict: k, v [n_seq][ctx][4][256] bf16 bits; proj [n_seq][10240]
    bf16 bits; q_norm, k_norm [256] f32.
    """
    k = bf16_bits(normal(seed * 8 + 1, (n_seq, ctx, 4, 256)))
    v = bf16_bits(normal(seed * 8 + 2, (n_seq, ctx, 4, 256)))
    proj = bf16_bits(normal(seed * 8 + 3, (n_seq, 10240)))
    q_norm = (1.0 + normal(seed * 8 + 4, (256,), std=0.02)).astype(np.float32)
    k_norm = (1.0 + normal(seed * 8 + 5, (256,), std=0.02)).astype(np.float32)
    return dict(k=k, v=v, proj=proj, q_norm=q_norm, k_norm=k_norm)


def gdn_params(seed: int):
    """Per-layer DeltaNet weights: ssm_a, dt_bias [32], ssm_norm [128], conv_w [4][8192]."""
    ssm_a = (-np.exp(normal(seed * 8 + 1, (32,), mean=-2.0, std=0.5))).astype(np.float32)
    dt_bias = np.zeros(32, dtype=np.float32)
    ssm_norm = (1.0 + normal(seed * 8 + 2, (128,), std=0.02)).astype(np.float32)
    conv_w = bf16_to_f32(bf16_bits(normal(seed * 8 + 3, (4, 8192), std=0.1)))
    return dict(ssm_a=ssm_a, dt_bias=dt_bias, ssm_norm=ssm_norm, conv_w=conv_w)


def gdn_inputs(seed: int, n_seq: int):
    """Per-sequence DeltaNet inputs: state [n][32][128][128] f32 ~ N(0, 0.02),
    conv history [n][3][8192] bf16 bits ~ N(0, 1), proj [n][12352] bf16 bits."""
    state = normal(seed * 8 + 4, (n_seq, 32, 128, 128), std=0.02).astype(np.float32)
    hist = bf16_bits(normal(seed * 8 + 5, (n_seq, 3, 8192)))
    proj = bf16_bits(normal(seed * 8 + 6, (n_seq, 12352)))
    return dict(state=state, hist=hist, proj=proj)


def bfp8_weights(seed: int, M: int, K: int, std: float = 0.02, edges: bool = True) -> np.ndarray:
    """bf16 bits [M][K] ~ N(0, std).  With `edges`, the first tile-row carries
    the format's edge cases: an all-zero face row, a face row whose values
    span 2^-30 .. 1 (magnitudes that shift out), exact powers of two, values
    that round up to the saturated magnitude, and negative zeros."""
    w = normal(seed, (M, K), std=std).astype(np.float32)
    if edges and M >= 32 and K >= 32:
        w[0, :16] = 0.0
        w[1, :16] = np.float32(2.0) ** -np.arange(0, 32, 2, dtype=np.float32)
        w[1, 3::4] *= -1
        w[2, :16] = [1.0, 0.5, -0.25, 0.125, 2.0, -4.0, 0.0, 1.0 / 64, 1.5, -1.5, 3.0, 0.75,
                     -0.375, 1.0 / 128, 1.0 / 256, -1.0 / 512]
        w[3, :16] = np.float32(1.9921875)  # bf16 0x3fff: rounds to 128 -> saturates
        w[3, 8:16] = np.float32(-1.9921875)
        w[4, 16:32] = -0.0
    return bf16_bits(w)


def gemv_inputs(seed: int, batch: int, K: int) -> np.ndarray:
    """Activations bf16 bits [batch][K] ~ N(0, 1) (post-RMSNorm hidden rows)."""
    return bf16_bits(normal(seed * 8 + 7, (batch, K)))
