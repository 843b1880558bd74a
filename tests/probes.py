"""Code-level probe matrices for exact GEMM checks (numpy only).

The reference's structured probes (include/qgemm/correctness.hpp:31-110:
one-hot weights, prime block scales, a ramp of codes) make index and scale
mistakes exact and local instead of hiding them in a reduction.  Here they are
built directly as packed bytes in the reference layout (pack.hpp:14-25: code
of element 2i in the low nibble, scales in a separate array indexed
n*(K/block) + k/block), as the reference's pack_*_codes helpers do
(pack.hpp:611-674), and every product and partial sum they lead to is exactly
representable in FP32, so the device result must equal the oracle bit for bit
whatever the summation order.
"""
import numpy as np

BLOCK = {"mxfp4": 32, "nvfp4": 16}


def pack_codes(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8).reshape(-1)
    return (c[0::2] & 0xF) | ((c[1::2] & 0xF) << 4)


def fp16_bits(v) -> np.ndarray:
    return np.asarray(v, dtype=np.float16).view(np.uint16)


def e4m3_code(e: int, m: int) -> int:
    """Positive normal E4M3 code with exponent field e (1..15) and mantissa m."""
    return (e << 3) | m


def random_weights(fmt: str, group: int, N: int, K: int, seed: int):
    """Random codes and scales in a narrow exponent range.

    MXFP4: E8M0 scales 2^-4 .. 2^4; NVFP4: E4M3 scales in [0.5, 15] and a
    power-of-two tensor scale; INT4: FP16 group scales equal to primes
    (correctness.hpp:31-49, the reference's prime-scale probe).
    Returns (data, scales, tensor_scale)."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, N * K, dtype=np.uint8)
    if fmt == "mxfp4":
        scales = rng.integers(123, 132, N * (K // 32), dtype=np.uint8)
        return pack_codes(codes), scales, 1.0
    if fmt == "nvfp4":
        e = rng.integers(6, 11, N * (K // 16))
        m = rng.integers(0, 8, N * (K // 16))
        return pack_codes(codes), ((e << 3) | m).astype(np.uint8), 0.25
    primes = np.array([2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53, 59, 61, 67, 71, 73, 79, 83,
                       89, 97, 101, 103, 107, 109, 113, 127, 131], np.float32)
    g = N * (K // group)
    return pack_codes(codes), fp16_bits(primes[np.arange(g) % len(primes)]), 1.0


def sparse_activations(M: int, K: int, seed: int, density: float = 1.0 / 16) -> np.ndarray:
    """bf16 bits of X with about `density` nonzeros, each +-{0.5, 1, 2}."""
    rng = np.random.default_rng(seed)
    vals = rng.choice(np.array([0.5, 1.0, 2.0, -0.5, -1.0, -2.0], np.float32), size=(M, K))
    keep = rng.random((M, K)) < density
    X = np.where(keep, vals, np.float32(0.0)).astype(np.float32)
    return (X.view(np.uint32) >> 16).astype(np.uint16)


def permutation_probe(fmt: str, group: int, N: int, K: int):
    """One nonzero weight per row: W[n, pi(n)] with pi(n) = 37 n mod K, a
    distinct k per row (N <= K), of value code 0x5 (3.0) or 0xD (-3.0) times a
    row-dependent scale.  Returns (data, scales, tensor_scale, pi)."""
    assert N <= K
    pi = (37 * np.arange(N)) % K
    assert len(set(pi.tolist())) == N
    codes = np.zeros(N * K, np.uint8)
    codes[np.arange(N) * K + pi] = np.where(np.arange(N) % 2 == 0, 0x5, 0xD)
    if fmt == "mxfp4":
        scales = (127 + (np.arange(N * (K // 32)) // (K // 32)) % 5 - 2).astype(np.uint8)
        return pack_codes(codes), scales, 1.0, pi
    if fmt == "nvfp4":
        rows = np.arange(N * (K // 16)) // (K // 16)
        scales = np.array([e4m3_code(7, int(r % 8)) for r in rows], np.uint8)
        return pack_codes(codes), scales, 2.0, pi
    codes[np.arange(N) * K + pi] = np.where(np.arange(N) % 2 == 0, 3, 0xD)  # INT4 +3 / -3
    rows = np.arange(N * (K // group)) // (K // group)
    return pack_codes(codes), fp16_bits(1 + (rows % 7)), 1.0, pi


def one_hot_rows(M: int, K: int, cols) -> np.ndarray:
    """bf16 bits of X with X[m, cols[m]] = 1 and zeros elsewhere."""
    X = np.zeros((M, K), np.float32)
    X[np.arange(M), np.asarray(cols)] = 1.0
    return (X.view(np.uint32) >> 16).astype(np.uint16)
