"""The arithmetic the tcgen05 kernels use for INT4, modelled on the CPU.

k_umma_ts (csrc/umma.cu) and k_umma_sk (csrc/umma_sk.cu) feed the tensor
core f16 weights: q (exact in f16) times the FP16 group scale s, rounded to
f16, after the row was folded by 2^-b, b = max(0, e - 26) with e the largest
FP16 exponent field among the row's scales; the epilogue multiplies by 2^b.
X enters as f16 scaled by a power of two per row (exact for bf16 values in
range), products are exact in the FP32 accumulator, so W's rounding is the
only difference from the reference's exact q * s (dequant_int4,
pack.hpp:548-604; ref_gemm.hpp:15-27) beyond summation order.

This model, in float64 on the oracle's packed bytes, shows:
* q * s is exact while it needs at most 11 significant bits (scales of up to
  8 significant bits), so such weights reproduce the reference to summation
  order;
* with full 11-bit scales the error of Y stays below the 1e-3 relative
  Frobenius bound the GPU tests hold INT4 on these kernels to, and above the
  1e-5 bound of the other formats (which is why INT4 has its own bound);
* rows whose scales reach f16's top binades overflow without the fold and
  stay finite with it;
* the bit operations that widen eight INT4 codes to f16 give exact values
  in the pair order of k_xprep's INT4 permutation of X.
No GPU is involved: this is the tolerance's derivation, not a parity test.
"""
import numpy as np
import pytest


def _pack(O, orc, N, K, group, seed, row_gain=None):
    W = O.randn(seed, 1, N * K, 0.0, 0.02).reshape(N, K)
    if row_gain is not None:
        W[::4] *= row_gain
    st, d, s = orc.pack("int4", W, group=group)
    assert st == 0
    return d, s


def _x(O, M, K, seed):
    bits = O.randn_bf16(seed, 2, M * K).reshape(M, K)
    return bits, O.bf16_bits_to_f32(bits).reshape(M, K).astype(np.float64)


def _fold(s, N, group, K):
    """Per-row fold exponent b = max(0, e - 26), infinity / NaN fields as 0."""
    e = ((s.reshape(N, K // group).astype(np.int32) >> 10) & 0x1F)
    e = np.where(e == 31, 0, e)
    return np.maximum(0, e.max(axis=1) - 26)


def _model_w(orc, d, s, N, K, group, fold=True):
    Wq = orc.dequant("int4", d, s, N, K, group=group).astype(np.float64)  # q * s, exact
    b = _fold(s, N, group, K) if fold else np.zeros(N, np.int64)
    f = np.ldexp(1.0, -b)[:, None]
    with np.errstate(over="ignore"):
        w16 = (Wq * f).astype(np.float16)  # the kernels' f16 operand (round to nearest even)
    return w16.astype(np.float64) / f, Wq


def _rel(A, B):
    return float(np.linalg.norm(A - B) / max(np.linalg.norm(B), 1e-300))


@pytest.mark.parametrize("group", [128, 64])
def test_short_scales_are_exact(O, orc, group):
    N, K, M = 128, 1024, 8
    d, s = _pack(O, orc, N, K, group, seed=41)
    s8 = (s & np.uint16(0xFFF8)).astype(np.uint16)  # 8 significant bits: q * s needs <= 11
    w, Wq = _model_w(orc, d, s8, N, K, group)
    assert np.array_equal(w, Wq)
    bits, X = _x(O, M, K, seed=42)
    Yref = orc.w4a16_gemm("int4", d, s8, N, K, bits, group=group)
    assert _rel(X @ w.T, Yref) < 1e-6


@pytest.mark.parametrize("group", [128, 64])
def test_full_scales_within_the_int4_bound(O, orc, group):
    N, K, M = 256, 2048, 16
    d, s = _pack(O, orc, N, K, group, seed=43)
    w, Wq = _model_w(orc, d, s, N, K, group)
    # per weight: at most half an f16 unit in the last place, 2^-11 relative
    nz = Wq != 0
    assert np.max(np.abs(w[nz] - Wq[nz]) / np.abs(Wq[nz])) <= 2.0 ** -11
    bits, X = _x(O, M, K, seed=44)
    Yref = orc.w4a16_gemm("int4", d, s, N, K, bits, group=group)
    rel = _rel(X @ w.T, Yref)
    assert 1e-5 < rel < 1e-3, rel


def test_fold_keeps_large_rows_finite(O, orc):
    N, K, M, group = 64, 1024, 4, 128
    d, s = _pack(O, orc, N, K, group, seed=45, row_gain=2e6)
    assert int(_fold(s, N, group, K).max()) > 0  # some rows need the fold
    bits, X = _x(O, M, K, seed=46)
    Yref = orc.w4a16_gemm("int4", d, s, N, K, bits, group=group)
    unfolded, _ = _model_w(orc, d, s, N, K, group, fold=False)
    assert not np.isfinite(unfolded).all()  # q * s leaves f16's range
    w, _ = _model_w(orc, d, s, N, K, group)
    Y = X @ w.T
    assert np.isfinite(Y).all()
    assert _rel(Y, Yref) < 1e-3


def _halves(w):
    """The two f16 halves (low, high) of a 32-bit word, as float64."""
    h = np.array([w & 0xFFFF, w >> 16], np.uint16).view(np.float16)
    return h.astype(np.float64)


def test_int4_widening_pairs_match_the_x_permutation():
    """int4x8_to_f16 (gemv_core.cuh) restated with its bit operations: one
    32-bit word of eight two's-complement nibbles c0..c7 (c0 in bits 0-3)
    becomes four f16 pairs (c0, c4), (c1, c5), (c2, c6), (c3, c7), each value
    exact, which is the order k_xprep's INT4 permutation gives X
    (f16 pair i = (x_i, x_{i+4}))."""
    magic, sub, k16, neg72 = 0x6400, 1032.0, 1.0 / 16.0, -72.0
    rng = np.random.default_rng(5)
    words = list(rng.integers(0, 2 ** 32, 2000, dtype=np.uint64)) + [0, 0xFFFFFFFF, 0x88888888, 0x77777777]
    for q in words:
        q = int(q)
        nib = [(q >> (4 * i)) & 0xF for i in range(8)]
        val = [n - 16 if n >= 8 else n for n in nib]
        lo = q ^ 0x88888888
        hi = lo >> 8
        w0 = (lo & 0x000F000F) | (magic | magic << 16)
        w1 = (lo & 0x00F000F0) | (magic | magic << 16)
        w2 = (hi & 0x000F000F) | (magic | magic << 16)
        w3 = (hi & 0x00F000F0) | (magic | magic << 16)
        pairs = [_halves(w0) - sub, _halves(w1) * k16 + neg72, _halves(w2) - sub, _halves(w3) * k16 + neg72]
        for i, p in enumerate(pairs):
            assert p.tolist() == [val[i], val[i + 4]], (hex(q), i)
