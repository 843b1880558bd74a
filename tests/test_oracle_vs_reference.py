"""The C oracle is bit-identical to the reference's own code on seeded random
and edge inputs (codecs on random float bit patterns, all three packers,
dequantisers and the W4A16 CPU path).  Skipped where the reference build
(oracle/_ref) is absent."""
import numpy as np
import pytest

from edge_cases import edge_matrix, random_bits, weights


@pytest.mark.parametrize("kind", ["e2m1", "e8m0", "fp16"])
def test_codecs_random_bits(orc, ref, kind):
    v = random_bits(1 << 20)
    assert np.array_equal(orc.encode_n(kind, v), ref.encode_n(kind, v))


def test_e4m3_random_bits(orc, ref):
    v = random_bits(1 << 16, seed=5)
    assert np.array_equal(orc.encode_n("e4m3", v), ref.encode_n("e4m3", v))
    # dense sweep of the finite range, including every midpoint region
    w = np.linspace(-500, 500, 200001, dtype=np.float32)
    assert np.array_equal(orc.encode_n("e4m3", w), ref.encode_n("e4m3", w))


def _packs(orc, ref, W, fmt, **kw):
    a = orc.pack(fmt, W, **kw)
    b = ref.pack(fmt, W, **kw)
    assert a[0] == b[0]
    if a[0] == 0:
        assert np.array_equal(a[1], b[1]), f"{fmt} data"
        assert np.array_equal(a[2], b[2]), f"{fmt} scales"
    return a


@pytest.mark.parametrize("shape", [(64, 256), (33, 384), (7, 128)])
def test_pack_seeded(O, orc, ref, shape):
    N, K = shape
    W = weights(O, N, K, seed=N)
    _packs(orc, ref, W, "mxfp4")
    _packs(orc, ref, W, "nvfp4", tensor_scale=O.nvfp4_tensor_scale(W))
    _packs(orc, ref, W, "nvfp4", tensor_scale=1.0)
    _packs(orc, ref, W, "int4", group=128)
    _packs(orc, ref, W, "int4", group=64)


def test_pack_edge_matrix(orc, ref):
    W = edge_matrix()
    _packs(orc, ref, W, "mxfp4")
    _packs(orc, ref, W, "nvfp4", tensor_scale=1.0)
    _packs(orc, ref, W, "nvfp4", tensor_scale=1e-30)   # inverse overflows to inf
    _packs(orc, ref, W, "nvfp4", tensor_scale=3e38)
    _packs(orc, ref, W, "int4", group=128)
    _packs(orc, ref, W, "int4", group=64)


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4", "int4"])
def test_dequant_random_bytes(orc, ref, fmt):
    rng = np.random.default_rng(11)
    N, K = 16, 256
    data = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
    if fmt == "int4":
        sc = rng.integers(0, 2**16, N * K // 128, dtype=np.uint16)
        a = orc.dequant(fmt, data, sc, N, K, group=128)
        b = ref.dequant(fmt, data, sc, N, K, group=128)
    else:
        sc = rng.integers(0, 256, N * K // (32 if fmt == "mxfp4" else 16), dtype=np.uint8)
        a = orc.dequant(fmt, data, sc, N, K, tensor_scale=0.37)
        b = ref.dequant(fmt, data, sc, N, K, tensor_scale=0.37)
    nan = np.isnan(a) & np.isnan(b)
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))
    assert np.array_equal(np.isnan(a), np.isnan(b))


@pytest.mark.parametrize("fmt,group", [("mxfp4", 32), ("nvfp4", 16), ("int4", 128), ("int4", 64)])
def test_w4a16_cpu_path(O, orc, ref, fmt, group):
    N, K, M = 40, 256, 3
    W = weights(O, N, K, seed=2)
    ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
    st, d, s = orc.pack(fmt, W, group=group, tensor_scale=ts)
    X = O.randn_bf16(0, 2, M * K).reshape(M, K)
    a = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=3)
    b = ref.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=2)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # and equal to dequant + gemm_fp32_ref done separately
    Wd = ref.dequant(fmt, d, s, N, K, group=group, tensor_scale=ts)
    c = ref.gemm_ref(O.bf16_bits_to_f32(X), Wd)
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


@pytest.mark.parametrize("fmt,group,K", [("mxfp4", 32, 96), ("mxfp4", 32, 2880), ("nvfp4", 16, 48),
                                         ("nvfp4", 16, 112), ("nvfp4", 16, 2880), ("int4", 64, 192),
                                         ("int4", 64, 2880)])
def test_unaligned_k_pack_and_cpu_path(O, orc, ref, fmt, group, K):
    """K that is a whole number of the format's blocks but not of 128 (the
    reference's gpt_oss_2880 and K = 96 shapes, shapes.hpp:33,
    test_pack_roundtrip.cpp:291-305): packing and the W4A16 CPU path stay
    bit-identical to the reference's."""
    N, M = 24, 2
    W = weights(O, N, K, seed=K)
    ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
    st, d, s = _packs(orc, ref, W, fmt, group=group, tensor_scale=ts)
    assert st == 0
    X = O.randn_bf16(1, 2, M * K).reshape(M, K)
    a = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=2)
    b = ref.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=2)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
