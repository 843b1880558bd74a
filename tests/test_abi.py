"""The C-ABI library loads without a GPU, exports every entry point declared
in include/*.h, and its host-only parts behave like the reference: byte
accounting (formats.cuh), packed sizes (pack.hpp:113-153) and the argument
checks on which the reference throws (pack.hpp:426-430, 466-468, 504-509)."""
import ctypes as C
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(qgemm_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("qgemm_pack_mxfp4", "qgemm_pack_nvfp4", "qgemm_pack_int4", "qgemm_gemm_w4a16",
                 "qgemm_dequant", "qgemm_workspace_size"):
        assert must in names


def test_library_exports_every_declared_symbol(qg):
    lib = qg.lib()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_byte_accounting_matches_reference_formulas(qg):  # test_formats.cpp:49-117
    assert qg.bytes_per_weight(qg.MXFP4) == 0.53125
    assert qg.bytes_per_weight(qg.NVFP4) == 0.5625
    assert qg.bytes_per_weight(qg.INT4_G128) == 0.515625
    assert qg.bytes_per_weight(qg.INT4_G64) == 0.53125
    assert qg.bytes_per_weight(qg.BF16) == 2.0 and qg.bytes_per_weight(qg.FP8_E4M3) == 1.0
    assert qg.weight_bytes(qg.INT4_G128, 4096, 4096) == 8_650_752
    assert qg.weight_bytes(qg.MXFP4, 4096, 4096) == 8_912_896
    assert qg.total_bytes(qg.MXFP4, 1, 4096, 4096) == 8_912_896 + 8192 + 8192
    assert qg.flops(2, 3, 4) == 48.0


def test_accounting_equals_reference_build(qg, ref):
    for f, rf in [(qg.MXFP4, 0), (qg.NVFP4, 1), (qg.INT4_G128, 2), (qg.INT4_G64, 3)]:
        for (M, N, K) in [(1, 4096, 4096), (256, 28672, 4096), (7, 2880, 2880), (64, 57344, 8192)]:
            assert qg.weight_bytes(f, N, K) == ref.lib.ref_weight_bytes(rf, N, K)
            assert qg.total_bytes(f, M, N, K) == ref.lib.ref_total_bytes(rf, M, N, K)


def test_packed_sizes(qg):  # test_formats.cpp:81-106 (N=64, K=256)
    N, K = 64, 256
    for f, bpw in [(qg.MXFP4, 0.53125), (qg.NVFP4, 0.5625), (qg.INT4_G128, 0.515625), (qg.INT4_G64, 0.53125)]:
        d, s = qg.packed_sizes(f, N, K)
        assert (d + s) / (N * K) == bpw
    with pytest.raises(ValueError):
        qg.packed_sizes(qg.MXFP4, 3, 48)


def test_argument_checks_return_invalid_arg(qg):
    """The reference's throw conditions come back as QGEMM_ERR_INVALID_ARG,
    decided on the host before any device work."""
    lib = qg.lib()
    null = C.c_void_p(0)
    assert lib.qgemm_pack_mxfp4(null, 4, 48, null, null, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_pack_nvfp4(null, 4, 40, 1.0, null, null, null) == qg.ERR_INVALID_ARG
    for ts in (0.0, -2.0, float("inf"), float("nan")):
        assert lib.qgemm_pack_nvfp4(null, 4, 32, ts, null, null, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_pack_int4(null, 4, 128, 32, null, null, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_pack_int4(null, 4, 96, 64, null, null, null) == qg.ERR_INVALID_ARG
    assert b"group" in lib.qgemm_last_error_message() or b"divisible" in lib.qgemm_last_error_message()
    w = qg._Weights(qg.MXFP4, 0, 64, 256, None, None, 1.0)
    assert lib.qgemm_gemm_w4a16(C.byref(w), null, 1, null, null, 0, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_codec_encode(9, null, null, 4, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_probe_launch(0, null, null, 17, null) == qg.ERR_INVALID_ARG


def test_grouped_argument_checks(qg):
    """qgemm_grouped_gemm_w4a16 rejects mixed shapes and negative counts, and
    returns at once for E = 0 or all-empty routing, before any device work."""
    lib = qg.lib()
    null = C.c_void_p(0)
    fake = C.c_void_p(1 << 20)  # never dereferenced: every call below returns on the host
    W3 = qg._Weights * 3
    ws = W3(qg._Weights(qg.MXFP4, 0, 256, 512, 1 << 20, 1 << 21, 1.0),
            qg._Weights(qg.MXFP4, 0, 256, 512, 1 << 22, 1 << 23, 1.0),
            qg._Weights(qg.MXFP4, 0, 128, 512, 1 << 24, 1 << 25, 1.0))
    I3, O3 = C.c_int32 * 3, C.c_int64 * 3
    args = lambda E, m, o: (ws, E, fake, I3(*m), O3(*o), fake, null, 0, null)
    assert lib.qgemm_grouped_gemm_w4a16(*args(0, [1, 1, 1], [0, 1, 2])) == qg.OK
    assert lib.qgemm_grouped_gemm_w4a16(*args(2, [0, 0, 0], [0, 0, 0])) == qg.OK
    assert lib.qgemm_grouped_gemm_w4a16(*args(3, [1, 1, 1], [0, 1, 2])) == qg.ERR_INVALID_ARG
    assert b"expert 2" in lib.qgemm_last_error_message()
    assert lib.qgemm_grouped_gemm_w4a16(*args(2, [1, -1, 0], [0, 1, 2])) == qg.ERR_INVALID_ARG
    assert lib.qgemm_grouped_gemm_w4a16(*args(2, [1, 1, 0], [0, -4, 2])) == qg.ERR_INVALID_ARG
    assert lib.qgemm_grouped_gemm_w4a16(*args(-1, [1, 1, 1], [0, 1, 2])) == qg.ERR_INVALID_ARG
    assert lib.qgemm_grouped_gemm_w4a16(ws, 2, null, I3(1, 1, 1), O3(0, 1, 2), fake, null, 0, null) \
        == qg.ERR_INVALID_ARG
    assert lib.qgemm_grouped_workspace_size(ws, 0, 4) == 0


def test_code_packer_argument_checks(qg):
    """qgemm_pack_codes / qgemm_unpack_codes refuse what the reference's
    pack_*_codes throws on (pack.hpp:113-139), on the host."""
    lib = qg.lib()
    null = C.c_void_p(0)
    fake = C.c_void_p(1 << 20)
    assert lib.qgemm_pack_codes(9, fake, fake, 4, 64, fake, fake, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_pack_codes(qg.MXFP4, fake, fake, 3, 33, fake, fake, null) == qg.ERR_INVALID_ARG  # N*K odd
    assert lib.qgemm_pack_codes(qg.MXFP4, fake, fake, 4, 48, fake, fake, null) == qg.ERR_INVALID_ARG  # K % 32
    assert lib.qgemm_pack_codes(qg.NVFP4, fake, fake, 4, 40, fake, fake, null) == qg.ERR_INVALID_ARG  # K % 16
    assert lib.qgemm_pack_codes(qg.INT4_G128, fake, fake, 4, 192, fake, fake, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_pack_codes(qg.INT4_G64, null, fake, 4, 128, fake, fake, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_pack_codes(qg.MXFP4, null, null, 0, 64, null, null, null) == qg.OK  # empty
    assert lib.qgemm_unpack_codes(qg.MXFP4, fake, 3, 33, fake, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_unpack_codes(7, fake, 4, 64, fake, null) == qg.ERR_INVALID_ARG


def test_layout_sizes_and_checks(qg):
    """The scale-checked layout keeps the canonical sizes; the host-side
    refusals: unknown layouts, INT4 in the scale-checked layout, a
    non-canonical repack source."""
    assert qg.layout_sizes(qg.MXFP4, qg.CANONICAL, 300, 2048) == qg.packed_sizes(qg.MXFP4, 300, 2048)
    assert qg.layout_sizes(qg.MXFP4, qg.SCALE_CHECKED, 300, 2048) == qg.packed_sizes(qg.MXFP4, 300, 2048)
    assert qg.layout_sizes(qg.NVFP4, qg.SCALE_CHECKED, 1000, 2880) == qg.packed_sizes(qg.NVFP4, 1000, 2880)
    with pytest.raises(ValueError):
        qg.layout_sizes(qg.INT4_G128, qg.SCALE_CHECKED, 128, 256)
    with pytest.raises(ValueError):
        qg.layout_sizes(qg.MXFP4, 5, 128, 256)
    lib = qg.lib()
    null = C.c_void_p(0)
    fake = C.c_void_p(1 << 20)
    w = qg._Weights(qg.MXFP4, 7, 256, 512, 1 << 20, 1 << 21, 1.0)
    assert lib.qgemm_gemm_w4a16(C.byref(w), fake, 1, fake, fake, 1 << 20, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_gemm_w4a16_noalloc(C.byref(w), fake, 1, fake, null) == qg.ERR_INVALID_ARG
    w = qg._Weights(qg.INT4_G128, qg.SCALE_CHECKED, 256, 512, 1 << 20, 1 << 21, 1.0)
    assert lib.qgemm_gemm_w4a16(C.byref(w), fake, 1, fake, fake, 1 << 20, null) == qg.ERR_INVALID_ARG
    w = qg._Weights(qg.MXFP4, qg.SCALE_CHECKED, 256, 512, 1 << 20, 1 << 21, 1.0)
    assert lib.qgemm_repack(C.byref(w), qg.SCALE_CHECKED, fake, fake, null) == qg.ERR_INVALID_ARG  # not canonical
    assert lib.qgemm_unpack(C.byref(qg._Weights(qg.INT4_G64, 1, 8, 64, 1 << 20, 1 << 21, 1.0)), fake, fake,
                            null) == qg.ERR_INVALID_ARG


def test_launch_count_mirrors_dispatch(qg):
    """qgemm_launch_count is host-only: which kernel a call uses and how many
    launches it makes (MXFP4 with 9 <= M <= 128, K % 128 == 0 and a 32-byte
    aligned code array: k_xprep_bs + k_umma_bs, plus k_bs_fixup when the
    device's stream-K ranges split tiles, which needs its SM count: 2 without
    a device; an X-preparation kernel + one GEMM kernel per 16-row block on
    the decode paths; k_xprep + one tcgen05 kernel for M >= 32)."""
    lib = qg.lib()
    kern = qg._i32(0)

    def count(fmt, N, K, M, scales=0x1000, data=0x2000):
        w = qg._Weights(fmt, 0, N, K, C.c_void_p(data), C.c_void_p(scales), 1.0)
        n = lib.qgemm_launch_count(C.byref(w), M, C.byref(kern))
        return n, qg.KERNEL_NAMES.get(kern.value)

    assert count(qg.MXFP4, 8192, 8192, 1) == (2, "k_gemv_tma")
    assert count(qg.MXFP4, 8192, 8192, 8) == (2, "k_gemv_tma")
    assert count(qg.MXFP4, 8192, 8192, 9) == (2, "k_umma_bs")
    assert count(qg.MXFP4, 8192, 8192, 20) == (2, "k_umma_bs")
    assert count(qg.MXFP4, 8192, 8192, 128) == (2, "k_umma_bs")
    assert count(qg.MXFP4, 8192, 4224, 64) == (2, "k_umma_bs")      # K % 128 == 0
    assert count(qg.MXFP4, 8192, 8192, 129) == (2, "k_umma_ts")
    assert count(qg.MXFP4, 8192, 8192, 20, data=0x2010) == (4, "k_gemv_tma")  # codes not 32-byte aligned
    assert count(qg.NVFP4, 8192, 8192, 16) == (2, "k_gemv_tma")
    assert count(qg.NVFP4, 8192, 8192, 17) == (2, "k_umma_sk")             # one pass, X padded to 32 rows
    assert count(qg.NVFP4, 8192, 8192, 32) == (2, "k_umma_sk")
    assert count(qg.NVFP4, 8192, 8192, 127) == (2, "k_umma_sk")
    assert count(qg.NVFP4, 8192, 8192, 128) == (2, "k_umma_ts")
    assert count(qg.MXFP4, 8192, 4160, 64) == (2, "k_umma_ts")      # K % 128 != 0
    assert count(qg.MXFP4, 8192, 4160, 1) == (2, "k_gemv")          # decode, LDG-fed
    assert count(qg.NVFP4, 8192, 8192, 1, scales=0x1002) == (2, "k_gemv")  # scales not 4-byte aligned
    assert count(qg.INT4_G128, 8192, 8192, 1) == (2, "k_gemv_tma")
    assert count(qg.INT4_G64, 8192, 8192, 16) == (2, "k_gemv_tma")
    assert count(qg.INT4_G64, 8192, 8192, 20) == (2, "k_umma_sk")            # M >= 17: tcgen05
    assert count(qg.INT4_G128, 8192, 8192, 17) == (2, "k_umma_sk")
    assert count(qg.INT4_G64, 8192, 8192, 64) == (2, "k_umma_sk")
    assert count(qg.INT4_G128, 8192, 8192, 127) == (2, "k_umma_sk")
    assert count(qg.INT4_G128, 8192, 8192, 128) == (2, "k_umma_ts")
    assert count(qg.INT4_G128, 8192, 8064, 24) == (2, "k_umma_ts")           # K % 256 != 0
    assert count(qg.INT4_G128, 4096, 8192, 24) == (2, "k_umma_ts")           # below 2^26 weights
    assert count(qg.NVFP4, 8192, 8192, 40) == (2, "k_umma_sk")           # 2^26 weights
    assert count(qg.NVFP4, 8191, 8192, 40) == (2, "k_umma_ts")
    assert count(qg.INT4_G128, 8192, 8192, 2048) == (2, "k_umma_ts")
    assert count(qg.INT4_G128, 8192, 8064, 1) == (2, "k_gemv")              # K % 256 != 0: LDG-fed
    assert count(qg.INT4_G64, 8192, 8192, 1, scales=0x1004) == (2, "k_gemv")  # scales not 8-byte aligned
    w = qg._Weights(qg.MXFP4, 0, 64, 256, None, None, 1.0)
    assert lib.qgemm_launch_count(C.byref(w), 0, C.byref(kern)) == -1
    # K only needs each format's own divisibility; the rest is refused as the GEMM refuses it
    assert count(qg.MXFP4, 2880, 2880, 1) == (2, "k_gemv")          # gpt_oss 2880: K % 128 = 64
    assert count(qg.MXFP4, 2880, 2880, 33) == (2, "k_umma_ts")
    assert count(qg.NVFP4, 200, 48, 1) == (2, "k_gemv")             # K % 32 = 16
    assert count(qg.INT4_G64, 2880, 2880, 20) == (2, "k_umma_ts")          # K % 64 == 0
    assert count(qg.INT4_G64, 2880, 2880, 16) == (2, "k_gemv")
    assert count(qg.INT4_G128, 2880, 2880, 1)[0] == -1              # 2880 % 128 != 0
    assert count(qg.MXFP4, 64, 48, 1)[0] == -1                      # not whole 32-blocks
    assert count(qg.NVFP4, 64, 40, 1)[0] == -1
