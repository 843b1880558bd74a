"""The f16 weights the dequantising tcgen05 kernels build, checked on the CPU.

k_umma_ts (csrc/umma.cu) and k_umma_sk (csrc/umma_sk.cu) widen E2M1 codes to
f16 (cvt.rn.f16x2.e2m1x2, exact) and multiply by an f16 block factor with one
f16x2 multiply, rounded to nearest even; the tensor core then multiplies f16
operands exactly into FP32.  Over every code and scale byte:

* NVFP4: the factor is the E4M3 scale itself, decoded by bit placement for
  normal codes (the exact decoder for the rest), and e2m1 x e4m3 is exact
  in f16 for every finite pair (the FP32 tensor scale is applied in the
  epilogue), so the kernels see the reference's dequantised values
  (pack.hpp:548-604) exactly.
* MXFP4: the factor is 2^(e - 127 - b) with b = (largest E8M0 byte of the
  row or segment) - 140, made by f16x2_pow2 (tc.cuh: 2^k for k >= -24, else
  zero), and the epilogue multiplies by 2^b.  Products never exceed 49152
  (no overflow) and are exact for every block within 36 binades of the
  largest; the next binade rounds to f16's smallest subnormals and blocks
  below it get a zero factor.
No GPU is involved; the GPU tests check the kernels against the oracle.
"""
import numpy as np
import pytest

_E2M1 = None


def _e2m1(orc):
    global _E2M1
    if _E2M1 is None:
        _E2M1 = np.array([orc.e2m1_decode(c) for c in range(16)], np.float64)
    return _E2M1


def _f16_pow2(k):
    """f16x2_pow2 (tc.cuh) restated: 2^k for k >= -24, zero below."""
    k = np.asarray(k)
    return np.where(k >= -24, np.exp2(k.astype(np.float64)), 0.0)


def _f16_mul(a, b):
    """One f16 multiply, rounded to nearest even (the FP32 product of two
    f16 values is exact, so rounding it once to f16 is the f16 result)."""
    with np.errstate(over="ignore"):
        return (np.float16(a).astype(np.float32) * np.float16(b).astype(np.float32)).astype(np.float16)


def test_nvfp4_products_are_exact_in_f16(orc):
    codes = _e2m1(orc)
    scales = np.array([orc.e4m3_decode(b) for b in range(256) if b & 0x7F != 0x7F], np.float64)
    assert np.all(np.float16(scales).astype(np.float64) == scales)  # every finite E4M3 is an f16
    prod = codes[:, None] * scales[None, :]
    assert np.all(_f16_mul(codes[:, None], scales[None, :]).astype(np.float64) == prod)


@pytest.mark.parametrize("mx", [0, 1, 40, 127, 200, 254])
def test_mxfp4_folded_products(orc, mx):
    codes = _e2m1(orc)
    e = np.arange(0, mx + 1)
    b = mx - 140
    factor = _f16_pow2(e - 127 - b)
    got = _f16_mul(codes[:, None], factor[None, :]).astype(np.float64)
    exact = codes[:, None] * np.exp2((e - 127 - b).astype(np.float64))[None, :]
    assert np.all(np.isfinite(got)) and got.max() <= 49152.0
    near = e >= mx - 36
    assert np.all(got[:, near] == exact[:, near]), mx
    if mx >= 37:
        assert np.any(got[:, e == mx - 37] != exact[:, e == mx - 37])  # the band is tight
        assert not got[:, e < mx - 37].any()                           # zero factor below


def test_e4m3_decode_by_bit_placement(orc):
    """e4m3x2_to_f16x2_fast (gemv_core.cuh) restated: a normal E4M3 byte's
    exponent and mantissa bits, shifted into f16 position with the exponent
    rebased (+8), are the f16 of its value; it declines exactly the zero,
    subnormal and NaN codes, which the kernels decode with the exact path."""
    for b in range(256):
        e, m7 = (b >> 3) & 0xF, b & 0x7F
        ok = e != 0 and m7 != 0x7F
        h = ((b & 0x80) << 8) | ((m7 << 7) + 0x2000)
        ref = orc.e4m3_decode(b)
        if ok:
            assert float(np.array([h], np.uint16).view(np.float16)[0]) == ref, b
        else:
            assert e == 0 or np.isnan(ref), b
