"""Pin the CPU oracle to the reference's own known-answer tests.

Each test restates one check of titoatwork/qgemm-mx tests/test_pack_roundtrip.cpp,
tests/test_formats.cpp or tests/test_ref_gemm.cpp (cited per test) and runs it
against the oracle (oracle/qgemm_oracle.c) and, where it was built here,
against the reference's own headers (oracle/_ref/libqgemm_ref.so).
"""
import math

import numpy as np
import pytest

PRIMES = [2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53, 59, 61, 67, 71, 73, 79, 83,
          89, 97, 101, 103, 107, 109, 113, 127, 131, 137, 139, 149, 151, 157, 163, 167, 173, 179,
          181, 191, 193, 197, 199, 211, 223, 227, 229, 233, 239, 241, 251, 257, 263, 269, 271, 277,
          281, 283, 293, 307, 311]  # correctness.hpp:35-41




def pack_codes(codes):
    """Nibble packing of pack.hpp:159-169 (even index low, odd index high)."""
    c = np.asarray(codes, dtype=np.uint8).reshape(-1)
    return (c[0::2] & 0xF) | ((c[1::2] & 0xF) << 4)


@pytest.fixture(params=["oracle", "reference"])
def impl(request, O):
    if request.param == "oracle":
        return O.oracle()
    r = O.reference()
    if r is None:
        pytest.skip("reference build absent")
    return r


# ---- test_pack_roundtrip.cpp:47-110 scalar codecs -------------------------------

def test_e2m1_table(impl):  # :47-62
    for c in range(16):
        if c == 8:
            continue
        assert impl.e2m1_encode(impl.e2m1_decode(c)) == c
    assert impl.e2m1_encode(impl.e2m1_decode(8)) == 0
    assert impl.e2m1_decode(0x0) == 0.0 and impl.e2m1_decode(0x1) == 0.5
    assert impl.e2m1_decode(0x7) == 6.0 and impl.e2m1_decode(0xF) == -6.0
    assert impl.e2m1_decode(0x8) == 0.0


def test_e8m0(impl):  # :64-76
    assert impl.e8m0_decode(127) == 1.0 and impl.e8m0_decode(128) == 2.0
    assert impl.e8m0_decode(126) == 0.5 and math.isnan(impl.e8m0_decode(0xFF))
    assert impl.e8m0_encode(1.0) == 127 and impl.e8m0_encode(2.0) == 128
    assert impl.e8m0_encode(0.5) == 126 and impl.e8m0_encode(3.0) == 129


def test_e4m3_roundtrip(impl):  # :78-90
    for c in range(256):
        if (c & 0x7F) == 0x7F:
            continue
        assert impl.e4m3_encode(impl.e4m3_decode(c)) == c
    assert impl.e4m3_decode(0x00) == 0.0
    assert abs(impl.e4m3_decode(0x38) - 1.0) <= 1e-6
    assert math.isnan(impl.e4m3_decode(0x7F))


def test_fp16_roundtrip(impl):  # :92-104
    for v in [0.0, 1.0, -1.0, 0.5, 2.0, 7.0, 0.0001, 65504.0]:
        back = impl.fp16_bits_to_float(impl.float_to_fp16_bits(v))
        tol = 0.0 if v == 0.0 else abs(v) * 1e-3 + 1e-6
        assert abs(back - v) <= tol


def test_int4_nibble(impl):  # :106-110
    for v in range(-8, 8):
        assert impl.int4_from_nibble(impl.int4_to_nibble(v)) == v


def test_nibble_pack_order():  # :116-129  0xA,0xB,0xC,0xD -> 0xBA, 0xDC
    assert list(pack_codes([0xA, 0xB, 0xC, 0xD])) == [0xBA, 0xDC]


def test_tie_breaking_rules(impl):
    # ties go to the smaller magnitude / lower code (pack.hpp:278-286, 362-370)
    for v, code in [(0.25, 0x0), (0.75, 0x1), (1.75, 0x3), (2.5, 0x4), (3.5, 0x5), (5.0, 0x6),
                    (-0.75, 0x9), (100.0, 0x7), (-100.0, 0xF)]:
        assert impl.e2m1_encode(v) == code, v
    # Beyond 2^27 every float-rounded |a - t| is the same number, so the
    # first-minimum search keeps candidate 0: the reference encodes 1e9 as 0.
    assert impl.e2m1_encode(1e9) == 0x0 and impl.e2m1_encode(-1e9) == 0x0
    assert impl.e4m3_decode(impl.e4m3_encode(1.1875)) == 1.125
    assert impl.e4m3_encode(1000.0) == 0x7E


# ---- test_pack_roundtrip.cpp:135-216 exact code-level probes --------------------

def test_int4_prime_probe(impl):  # :135-145  N=4, K=256, group 128
    N, K, g = 4, 256, 128
    q = np.ones(N * K, dtype=np.int64)
    nib = (q & 0xF).astype(np.uint8)
    data = pack_codes(nib)
    scales = np.array([impl.float_to_fp16_bits(float(PRIMES[i % 64])) for i in range(N * K // g)],
                      dtype=np.uint16)
    got = impl.dequant("int4", data, scales, N, K, group=g)
    exp = np.array([[impl.fp16_bits_to_float(int(scales[n * (K // g) + k // g])) for k in range(K)]
                    for n in range(N)], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
    assert got[0, 0] == 2.0


def test_int4_one_hot_probe(impl):  # :147-170
    N, K = 8, 128
    for n0 in (0, 3, N - 1):
        for k0 in (0, 17, K - 1):
            codes = np.zeros(N * K, dtype=np.uint8)
            codes[n0 * K + k0] = 5
            sc = np.full(N, impl.float_to_fp16_bits(2.0), dtype=np.uint16)
            got = impl.dequant("int4", pack_codes(codes), sc, N, K, group=128)
            exp = np.zeros((N, K), np.float32)
            exp[n0, k0] = 10.0
            assert np.array_equal(got, exp)


def test_mxfp4_prime_probe(impl):  # :172-179 via correctness.hpp:176-201
    N, K = 3, 64
    cnt = N * K // 32
    bits = np.array([min(254, max(0, 127 + (PRIMES[i % 64] % 13) - 6)) for i in range(cnt)], np.uint8)
    data = pack_codes(np.full(N * K, 0x2, np.uint8))
    got = impl.dequant("mxfp4", data, bits, N, K)
    exp = np.array([[impl.e8m0_decode(int(bits[n * 2 + k // 32])) for k in range(K)] for n in range(N)],
                   np.float32)
    assert np.array_equal(got, exp)


def test_mxfp4_one_hot_probe(impl):  # :181-191  code 0x5 (3.0) x e8m0 128 (2.0) at (2,7)
    N, K = 4, 32
    codes = np.zeros(N * K, np.uint8)
    codes[2 * K + 7] = 0x5
    got = impl.dequant("mxfp4", pack_codes(codes), np.full(N, 128, np.uint8), N, K)
    assert got[2, 7] == 6.0 and got[0, 0] == 0.0 and np.count_nonzero(got) == 1


def test_mxfp4_ramp_probe(impl):  # :193-204
    N, K = 2, 32
    codes = (np.arange(N * K) % 8).astype(np.uint8)
    got = impl.dequant("mxfp4", pack_codes(codes), np.full(N, 127, np.uint8), N, K)
    assert list(got.reshape(-1)[:8]) == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def test_nvfp4_prime_probe(impl):  # :206-216  tensor scale 2
    N, K = 2, 32
    sc = np.array([impl.e4m3_encode(float(PRIMES[i])) for i in range(N * K // 16)], np.uint8)
    got = impl.dequant("nvfp4", pack_codes(np.full(N * K, 0x2, np.uint8)), sc, N, K, tensor_scale=2.0)
    exp = np.array([[impl.e4m3_decode(int(sc[n * 2 + k // 16])) * 2.0 for k in range(K)] for n in range(N)],
                   np.float32)
    assert np.array_equal(got, exp)
    assert abs(got[0, 0] - impl.e4m3_decode(impl.e4m3_encode(2.0)) * 2.0) <= 1e-5


def test_gpt_oss_dims_mxfp4(impl):  # :294-305  K=96 (32 | K, 128 does not)
    N, K = 96, 96
    codes = np.zeros(N * K, np.uint8)
    codes[10 * K + 33] = 0x6
    got = impl.dequant("mxfp4", pack_codes(codes), np.full(N * 3, 127, np.uint8), N, K)
    assert got[10, 33] == 4.0 and np.count_nonzero(got) == 1


# ---- test_pack_roundtrip.cpp:222-266 quantize-path round trips ------------------

def test_int4_quantize_roundtrip(impl):  # :222-237
    N, K = 4, 128
    W = ((np.arange(N * K) % 15) - 7).astype(np.float32).reshape(N, K)
    st, d, s = impl.pack("int4", W, group=128)
    assert st == 0
    got = impl.dequant("int4", d, s, N, K, group=128)
    assert np.all(np.abs(got - W) <= 0.05 + 0.05 * np.abs(W))


def test_mxfp4_quantize_roundtrip(impl):  # :239-252  exact-set values recover exactly
    N, K = 2, 32
    W = np.array([impl.e2m1_decode(i % 16) * 4.0 for i in range(N * K)], np.float32).reshape(N, K)
    st, d, s = impl.pack("mxfp4", W)
    assert st == 0
    got = impl.dequant("mxfp4", d, s, N, K)
    assert np.all(np.abs(got - W) <= 1e-5 + 1e-5 * np.abs(W))


def test_nvfp4_quantize_roundtrip(impl):  # :254-266
    N, K = 2, 16
    W = np.array([impl.e2m1_decode((i * 3) % 16) for i in range(N * K)], np.float32).reshape(N, K)
    st, d, s = impl.pack("nvfp4", W, tensor_scale=1.0)
    assert st == 0
    got = impl.dequant("nvfp4", d, s, N, K, tensor_scale=1.0)
    assert np.all(np.abs(got - W) <= 0.05 + 0.05 * np.abs(W))


def test_pack_rejects_like_reference(impl):  # pack.hpp:426-430, 466-468, 504-509
    W = np.zeros((2, 48), np.float32)
    assert impl.pack("mxfp4", W)[0] == 1           # K % 32
    assert impl.pack("int4", W, group=32)[0] == 1  # group not 64/128
    assert impl.pack("int4", np.zeros((2, 96), np.float32), group=64)[0] == 1
    assert impl.pack("nvfp4", np.zeros((2, 40), np.float32))[0] == 1  # K % 16
    for ts in (0.0, -1.0, float("inf"), float("nan")):
        assert impl.pack("nvfp4", np.zeros((2, 32), np.float32), tensor_scale=ts)[0] == 1


# ---- test_ref_gemm.cpp ------------------------------------------------------------

def test_gemm_hand_product(impl):  # :23-37
    Y = impl.gemm_ref(np.array([[1, 2], [3, 4]], np.float32), np.array([[5, 6], [7, 8]], np.float32))
    assert Y.tolist() == [[17.0, 23.0], [39.0, 53.0]]


def test_int4_dequant_gemm_matches_fp_weights(impl):  # :39-70
    M, N, K = 3, 8, 128
    n, k = np.meshgrid(np.arange(N), np.arange(K), indexing="ij")
    W = (np.float32(0.1) * ((n + k) % 7).astype(np.float32) - np.float32(0.3)).astype(np.float32)
    st, d, s = impl.pack("int4", W, group=128)
    Wdq = impl.dequant("int4", d, s, N, K, group=128)
    m, kk = np.meshgrid(np.arange(M), np.arange(K), indexing="ij")
    X = (((kk + m) % 5) * 0.25).astype(np.float32)
    Yr, Yf = impl.gemm_ref(X, Wdq), impl.gemm_ref(X, W)
    tol = max(1e-2, 0.15 * np.abs(Yf).max() + 1e-3 * K)
    assert np.abs(Yr - Yf).max() <= tol


# ---- test_formats.cpp (byte accounting, through the reference build) -------------

def test_weight_bytes_formula(ref):  # test_formats.cpp:108-117
    assert ref.lib.ref_weight_bytes(2, 4096, 4096) == 8_650_752
    assert ref.lib.ref_weight_bytes(0, 4096, 4096) == 8_912_896
