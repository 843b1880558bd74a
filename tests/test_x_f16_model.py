"""The decode kernel's f16 copy of X, checked exhaustively on the CPU.

k_xprep_units (csrc/gemv_tma.cu) scales each activation row's 256-k unit by
2^-s, s = ilogb(largest |x| of the unit) - 14 (kept in [-126, 114]), so the
largest lands in [2^14, 2^15), and converts to f16 rounding to nearest even;
the consumers multiply the unit's partial sum by 2^s, an exact power of two.
This restates those steps in numpy over every positive finite bf16 value x
under every possible largest exponent of its unit: nothing overflows f16,
every x within 31 binades of the largest's binade converts exactly (its 8
significant bits fit f16's 11, down to the subnormal grid), the first
value that can round is 32 binades down, and no value is off by more than
2^(ilogb(largest) - 39), half a subnormal step.  k_xprep (csrc/gemv.cu), the
copy the LDG-fed and tcgen05 kernels read, uses the same rule per row.  No
GPU is involved.
"""
import numpy as np

_BITS = np.arange(1, 0x7F80, dtype=np.uint32)  # every positive finite bf16
_X32 = (_BITS << 16).view(np.float32)
_X = _X32.astype(np.float64)
_ILOGB = np.floor(np.log2(_X)).astype(np.int64)


def test_unit_scaling_is_exact_within_31_binades():
    first_inexact = set()
    for lg in range(-133, 128):  # ilogb of the unit's largest |x| (bf16 subnormals from -133)
        sel = _ILOGB <= lg
        s = min(max(lg - 14, -126), 114)
        h = (_X32[sel] * np.float32(2.0 ** -s)).astype(np.float16)  # f32 scale, then RN to f16
        assert np.isfinite(h).all(), lg
        back = h.astype(np.float64) * 2.0 ** s
        off = _ILOGB[sel] - lg
        exact = back == _X[sel]
        assert exact[off >= -31].all(), lg
        assert (np.abs(back - _X[sel]) <= 2.0 ** (lg - 39)).all(), lg  # half a subnormal step
        if not exact.all():
            first_inexact.add(int(off[~exact].max()))
    assert first_inexact == {-32}
