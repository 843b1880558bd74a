"""Device codecs, packers and dequantisers are bit-exact against the oracle
(the CPU restatement of titoatwork/qgemm-mx include/qgemm/pack.hpp) and the
golden fixtures produced by the reference itself."""
import os

import numpy as np
import pytest
import torch

from edge_cases import edge_matrix, random_bits, weights
from gpu_util import same_bits, to_dev_f32, u16, u8

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FORMATS = [("mxfp4", 32), ("nvfp4", 16), ("int4", 128), ("int4", 64)]


def dev_pack(qg, fmt, group, W, ts):
    Wd = to_dev_f32(W)
    if fmt == "mxfp4":
        return qg.pack_mxfp4(Wd)
    if fmt == "nvfp4":
        return qg.pack_nvfp4(Wd, ts)
    return qg.pack_int4(Wd, group)


def host_scales(p):
    return u16(p.scales) if p.format in (2, 3) else u8(p.scales)


@pytest.mark.parametrize("kind", ["e2m1", "e8m0", "fp16"])
def test_codec_random_bits(qg, cuda, orc, kind):
    v = random_bits(1 << 22, seed=17)
    got = qg.codec_encode(kind, to_dev_f32(v)).cpu().numpy()
    exp = orc.encode_n(kind, v)
    if kind == "fp16":
        got = got.view(np.uint16)
    assert np.array_equal(got, exp)


def test_codec_e8m0_dense_and_subnormal(qg, cuda, orc):
    # every subnormal pattern (first 2^23 bit patterns), and a dense normal sweep
    v = np.concatenate([np.arange(1, 1 << 23, dtype=np.uint32).view(np.float32),
                        np.linspace(1e-30, 1e30, 1 << 20, dtype=np.float32)])
    assert np.array_equal(qg.codec_encode("e8m0", to_dev_f32(v)).cpu().numpy(), orc.encode_n("e8m0", v))


def test_codec_e4m3(qg, cuda, orc):
    v = np.concatenate([random_bits(1 << 16, seed=23), np.linspace(-600, 600, 300001, dtype=np.float32),
                        np.linspace(-0.01, 0.01, 100001, dtype=np.float32)])
    assert np.array_equal(qg.codec_encode("e4m3", to_dev_f32(v)).cpu().numpy(), orc.encode_n("e4m3", v))


@pytest.mark.parametrize("shape", [(64, 256), (33, 384), (256, 1024), (5, 128)])
@pytest.mark.parametrize("fmt,group", FORMATS)
def test_pack_seeded_bit_exact(qg, cuda, O, orc, shape, fmt, group):
    N, K = shape
    W = weights(O, N, K, seed=N + K)
    ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
    st, d, s = orc.pack(fmt, W, group=group, tensor_scale=ts)
    p = dev_pack(qg, fmt, group, W, ts)
    torch.cuda.synchronize()
    assert np.array_equal(u8(p.data), d)
    assert np.array_equal(host_scales(p), s)
    # dequant of the device-packed bytes equals the oracle's dequant bit for bit
    assert same_bits(qg.dequant(p).cpu().numpy(), orc.dequant(fmt, d, s, N, K, group=group, tensor_scale=ts))


@pytest.mark.parametrize("fmt,group", FORMATS)
def test_pack_edge_bit_exact(qg, cuda, orc, fmt, group):
    W = edge_matrix(16, 512)
    for ts in ([1.0, 1e-30, 3e38, 0.37] if fmt == "nvfp4" else [1.0]):
        st, d, s = orc.pack(fmt, W, group=group, tensor_scale=ts)
        p = dev_pack(qg, fmt, group, W, ts)
        assert np.array_equal(u8(p.data), d), ts
        assert np.array_equal(host_scales(p), s), ts


def test_pack_unaligned_source(qg, cuda, O, orc):
    """Scalar-load path: W starting 4 bytes past a 16-byte boundary."""
    N, K = 16, 256
    W = weights(O, N, K, seed=3)
    buf = torch.zeros(N * K + 1, dtype=torch.float32, device="cuda")
    buf[1:] = to_dev_f32(W).reshape(-1)
    Wd = buf[1:].view(N, K)
    assert Wd.data_ptr() % 16 != 0
    p = qg.pack_mxfp4(Wd)
    st, d, s = orc.pack("mxfp4", W)
    assert np.array_equal(u8(p.data), d) and np.array_equal(u8(p.scales), s)


@pytest.mark.parametrize("fmt,group", FORMATS)
def test_dequant_random_bytes(qg, cuda, orc, fmt, group):
    rng = np.random.default_rng(29)
    N, K = 32, 512
    data = rng.integers(0, 256, N * K // 2, dtype=np.uint8)
    fcode = {"mxfp4": qg.MXFP4, "nvfp4": qg.NVFP4}.get(fmt, qg.INT4_G128 if group == 128 else qg.INT4_G64)
    if fmt == "int4":
        sc = rng.integers(0, 2**16, N * K // group, dtype=np.uint16)
    else:
        sc = rng.integers(0, 256, N * K // group, dtype=np.uint8)
    p = qg.from_host(fcode, N, K, data, sc, tensor_scale=0.37)
    got = qg.dequant(p).cpu().numpy()
    exp = orc.dequant(fmt, data, sc, N, K, group=group, tensor_scale=0.37)
    assert same_bits(got, exp)


def test_nvfp4_tensor_scale(qg, cuda, O):
    W = weights(O, 300, 256, seed=9)
    W[17, 3] = -0.9
    assert qg.nvfp4_tensor_scale(to_dev_f32(W)) == O.nvfp4_tensor_scale(W)


@pytest.mark.parametrize("name", ["seeded_64x256", "edge_8x256"])
def test_pack_matches_reference_fixtures(qg, cuda, O, name):
    f = np.load(os.path.join(GOLD, name + ".npz"))
    N, K = int(f["N"]), int(f["K"])
    W = (O.randn(0, 1, N * K, 0.0, 0.02).reshape(N, K) if name.startswith("seeded") else edge_matrix(N, K))
    for fmt, group in FORMATS:
        tag = f"{fmt}{group}"
        p = dev_pack(qg, fmt, group, W, float(f[f"{tag}_ts"]))
        assert np.array_equal(u8(p.data), f[f"{tag}_data"]), tag
        assert np.array_equal(host_scales(p), f[f"{tag}_scales"]), tag
        assert same_bits(qg.dequant(p).cpu().numpy(), f[f"{tag}_dequant"]), tag


def test_pack_rejects_like_reference(qg, cuda):
    W = torch.zeros((4, 48), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        qg.pack_mxfp4(W)
    with pytest.raises(ValueError):
        qg.pack_int4(torch.zeros((4, 96), dtype=torch.float32, device="cuda"), 64)
    with pytest.raises(ValueError):
        qg.pack_nvfp4(torch.zeros((4, 32), dtype=torch.float32, device="cuda"), 0.0)


# ---- code-level packers (pack.hpp:611-674) against the reference's own ---------------

def _ref_code_fns(ref):
    import ctypes as C
    L = ref.lib
    vp, sz = C.c_void_p, C.c_size_t
    L.ref_pack_int4_codes.argtypes = [vp, vp, sz, sz, C.c_int, vp, vp]
    L.ref_pack_mxfp4_codes.argtypes = [vp, vp, sz, sz, vp, vp]
    L.ref_pack_nvfp4_codes.argtypes = [vp, vp, sz, sz, C.c_float, vp, vp]
    L.ref_unpack_int4_codes.argtypes = [vp, sz, sz, vp]
    L.ref_unpack_e2m1_codes.argtypes = [vp, sz, sz, vp]
    return L


@pytest.mark.parametrize("shape", [(64, 256), (7, 384), (130, 1024)])
@pytest.mark.parametrize("fmt,group", FORMATS)
def test_code_packers_match_reference(qg, cuda, ref, fmt, group, shape):
    """qgemm_pack_codes / qgemm_unpack_codes equal the reference's
    pack_*_codes / unpack_*_codes byte for byte, out-of-range INT4 codes
    (clamped), FP4 codes with high bits set (masked), and FP16 scale edge
    values (overflow, underflow, inf, NaN) included."""
    import ctypes as C
    N, K = shape
    rng = np.random.default_rng(N * K + group)
    L = _ref_code_fns(ref)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    nsc = N * (K // group)
    d_ref = np.zeros(N * K // 2, np.uint8)
    if fmt == "int4":
        codes = rng.integers(-12, 12, N * K).astype(np.int32)
        sc = (rng.standard_normal(nsc) * 0.05).astype(np.float32)
        sc[:5] = [131008.0, 1e-8, np.inf, np.nan, -3e-6]
        s_ref = np.zeros(nsc, np.uint16)
        assert L.ref_pack_int4_codes(ptr(codes), ptr(sc), N, K, group, ptr(d_ref), ptr(s_ref)) == 0
        fcode = qg.INT4_G128 if group == 128 else qg.INT4_G64
        p = qg.pack_codes(fcode, torch.from_numpy(codes).cuda(), torch.from_numpy(sc).cuda(), N, K)
        assert np.array_equal(u8(p.data), d_ref)
        assert np.array_equal(u16(p.scales), s_ref)
        back = qg.unpack_codes(p).cpu().numpy()
        q_ref = np.zeros(N * K, np.int32)
        L.ref_unpack_int4_codes(ptr(d_ref), N, K, ptr(q_ref))
        assert np.array_equal(back, q_ref)
        assert np.array_equal(back, np.clip(codes, -8, 7))
        again = qg.pack_codes(fcode, torch.from_numpy(back).cuda(), torch.from_numpy(sc).cuda(), N, K)
        assert np.array_equal(u8(again.data), d_ref)
    else:
        codes = rng.integers(0, 256, N * K).astype(np.uint8)
        sb = rng.integers(0, 256, nsc).astype(np.uint8)
        s_ref = np.zeros(nsc, np.uint8)
        if fmt == "mxfp4":
            assert L.ref_pack_mxfp4_codes(ptr(codes), ptr(sb), N, K, ptr(d_ref), ptr(s_ref)) == 0
            p = qg.pack_codes(qg.MXFP4, torch.from_numpy(codes).cuda(), torch.from_numpy(sb).cuda(), N, K)
        else:
            assert L.ref_pack_nvfp4_codes(ptr(codes), ptr(sb), N, K, 0.37, ptr(d_ref), ptr(s_ref)) == 0
            p = qg.pack_codes(qg.NVFP4, torch.from_numpy(codes).cuda(), torch.from_numpy(sb).cuda(), N, K,
                              tensor_scale=0.37)
            assert p.tensor_scale == 0.37
        assert np.array_equal(u8(p.data), d_ref)
        assert np.array_equal(u8(p.scales), s_ref)
        back = qg.unpack_codes(p).cpu().numpy()
        c_ref = np.zeros(N * K, np.uint8)
        L.ref_unpack_e2m1_codes(ptr(d_ref), N, K, ptr(c_ref))
        assert np.array_equal(back, c_ref)
        assert np.array_equal(back, codes & 0xF)
