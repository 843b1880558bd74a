"""The block-scaled kernel's two-term E4M3 split of X, checked exhaustively on the CPU.

k_xprep_bs (csrc/umma_bs.cu) gives each 32-block of an activation row the
E8M0 scale 2^s0, s0 = E - 7 with E the block's largest bf16 exponent (the
byte kept in [4, 254]), and writes t0 = e4m3(x / 2^s0) and
t1 = e4m3((x / 2^s0 - t0) * 16), both rounded to nearest even and saturated
(cvt.rn.satfinite.e4m3x2.f32).  The tensor core then sees
x' = 2^s0 (t0 + t1 / 16).  This restates those steps in numpy and runs them
over every positive finite bf16 value x under every block exponent E >= its
own: x' == x for every x within 13 binades of E, and |x' - x| <= 2^(E - 21)
below that, which is the bound the kernel's comment states.  No GPU is
involved; the GPU tests check the hardware conversion against the oracle.
"""
import numpy as np


def _e4m3_rne(v):
    """Nearest E4M3 value (ties to even, saturated at 448), as float64."""
    a = np.abs(v)
    nz = a > 0
    e = np.maximum(np.floor(np.log2(np.where(nz, a, 1.0))), -6.0)  # subnormals share 2^-6's step
    ulp = np.exp2(e - 3.0)
    q = np.minimum(np.round(a / ulp) * ulp, 448.0)                  # np.round: half to even
    return np.copysign(np.where(nz, q, 0.0), v)


def _split(xs, ebits):
    sb0 = min(max(ebits - 7, 4), 254)
    s = 2.0 ** (sb0 - 127)
    v0 = xs / s                       # a power of two: exact
    q0 = _e4m3_rne(v0)
    q1 = _e4m3_rne((v0 - q0) * 16.0)  # the remainder is exact in FP32
    return s * (q0 + q1 / 16.0)


_BITS = np.arange(1, 0x7F80, dtype=np.uint32)  # every positive finite bf16
_X = (_BITS << 16).view(np.float32).astype(np.float64)
_XE = (_BITS >> 7) & 0xFF                       # biased exponent field


def test_e4m3_model_matches_the_format():
    # spot values of E4M3: max 448, min normal 2^-6, min subnormal 2^-9, ties to even
    got = _e4m3_rne(np.array([448.0, 500.0, 2.0 ** -6, 2.0 ** -9, 17.0, 19.0]))
    assert got.tolist() == [448.0, 448.0, 2.0 ** -6, 2.0 ** -9, 16.0, 20.0]
    assert _e4m3_rne(np.array([2.0 ** -10]))[0] == 0.0  # half the smallest step: to even (zero)


def test_two_terms_exact_within_13_binades_for_every_block_exponent():
    for ebits in range(0, 255):
        sel = _XE <= ebits
        xs, xe = _X[sel], _XE[sel]
        err = np.abs(_split(xs, ebits) - xs)
        near = xe >= max(ebits - 13, 0)
        assert not err[near].any(), ebits
        assert (err[~near] <= 2.0 ** (ebits - 127 - 21)).all(), ebits


def test_the_13_binade_band_is_tight():
    fails = 0
    for ebits in range(20, 255):
        sel = (_XE <= ebits) & (_XE == ebits - 14)
        xs = _X[sel]
        fails += int((_split(xs, ebits) != xs).sum())
    assert fails > 0
