"""Seeded and edge-case weight matrices shared by the CPU and GPU parity tests.

Generators only (numpy); both the oracle pins and the device parity tests
draw from here so they cover the same inputs.
"""
import numpy as np

F32_MAX = np.float32(3.4028235e38)


def weights(O, N, K, seed=0, std=0.02):
    """W ~ N(0, std) from the build's documented generator (oracle/or_randn)."""
    return O.randn(seed, 1, N * K, 0.0, std).reshape(N, K)


def edge_matrix(N=8, K=256, seed=7):
    """Rows that exercise every special branch of the packers
    (pack.hpp:424-542): all-zero blocks, signed zeros, subnormal blocks whose
    scale underflows, a block at the float maximum, +-inf, exact ties of the
    E2M1 and rounding grids, and ordinary values."""
    assert N >= 8 and K % 128 == 0
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[0, :] = 0.0                                            # empty groups
    W[1, :] = -0.0                                           # signed zeros
    W[2, :] = np.float32(1e-45) * rng.integers(-3, 4, K)      # subnormal blocks
    W[3, :64] = F32_MAX * np.sign(rng.standard_normal(64)).astype(np.float32)
    W[3, 64:] = np.float32(3e38)
    W[4, 5] = np.inf                                         # one +inf per row/block
    W[4, 70] = -np.inf
    W[5, :] = np.tile(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0], np.float32), K // 8)
    W[5, 1::2] *= -1                                         # E2M1 ties, both signs
    W[6, :] = np.arange(K, dtype=np.float32) * np.float32(0.5) - np.float32(K / 4)  # int grid ties
    W[7, :] = np.float32(1e30) * np.sign(rng.standard_normal(K)).astype(np.float32)
    return W


def random_bits(n, seed=3):
    """Uniformly random float32 bit patterns (all classes, incl. NaN/inf)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 2**32, size=n, dtype=np.uint64).astype(np.uint32).view(np.float32)
