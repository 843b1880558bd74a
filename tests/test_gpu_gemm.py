"""Device W4A16 GEMM against the oracle (dequant + double-accumulated
reference GEMM, titoatwork/qgemm-mx ref_gemm.hpp:15-27), through the C-ABI.

Tolerance (tests/gpu_util.py): per row max-abs <= 1e-2 * ||Y_ref row||_inf and
relative Frobenius <= 1e-3; bf16 output is compared with the reference value
rounded to bf16.  Small shapes check every output; the full BASELINE shapes
check sampled row blocks against the oracle plus exact size-independent
properties (Y(2X) = 2Y(X), determinism, row independence)."""
import os

import numpy as np
import pytest
import torch

from edge_cases import weights
from gpu_util import bf16_to_np_f32, same_bits, to_dev_bf16, to_dev_f32, u8, u16, within_tolerance

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FORMATS = [("mxfp4", 32), ("nvfp4", 16), ("int4", 128), ("int4", 64)]


def fcode(qg, fmt, group):
    return {"mxfp4": qg.MXFP4, "nvfp4": qg.NVFP4}.get(fmt, qg.INT4_G128 if group == 128 else qg.INT4_G64)


def packed_pair(qg, O, orc, fmt, group, N, K, seed):
    """Device-packed weights plus the oracle's host copy of the same bytes."""
    W = weights(O, N, K, seed=seed)
    ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
    Wd = to_dev_f32(W)
    p = {"mxfp4": lambda: qg.pack_mxfp4(Wd), "nvfp4": lambda: qg.pack_nvfp4(Wd, ts)}.get(
        fmt, lambda: qg.pack_int4(Wd, group))()
    del Wd
    d = u8(p.data)
    s = u16(p.scales) if fmt == "int4" else u8(p.scales)
    return p, d, s, ts


def run(qg, p, Xbits, f32=False):
    X = to_dev_bf16(Xbits)
    Y = qg.gemm_w4a16(p, X, out_f32=f32)
    torch.cuda.synchronize()
    return Y.cpu().numpy() if f32 else bf16_to_np_f32(Y)


@pytest.mark.parametrize("fmt,group", FORMATS)
@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 16, 17, 31, 32, 33, 64])
def test_gemm_small_all_outputs(qg, cuda, O, orc, fmt, group, M):
    N, K = 200, 512
    p, d, s, ts = packed_pair(qg, O, orc, fmt, group, N, K, seed=M)
    X = O.randn_bf16(M, 2, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=8)
    ok, ratio, rel = within_tolerance(run(qg, p, X, f32=True), Yref)
    assert ok, (ratio, rel)
    # fp32 output: only summation order differs, except INT4 from M = 17,
    # whose tcgen05 path rounds q x scale to f16 (relative 2^-11 per weight)
    assert rel < (1e-3 if fmt == "int4" and M >= 17 else 1e-5), rel
    Yb = run(qg, p, X, f32=False)
    ok, ratio, rel = within_tolerance(Yb, O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(M, N))
    assert ok, (ratio, rel)


@pytest.mark.parametrize("N,K", [(16, 128), (48, 28672), (1, 256), (1000, 4096), (4096, 128)])
def test_gemm_stream_k_shapes(qg, cuda, O, orc, N, K):
    """Shapes whose tiles split across many warps (deep K, few rows), a single
    row, and many one-chunk tiles."""
    for fmt, group in [("mxfp4", 32), ("int4", 128)]:
        p, d, s, ts = packed_pair(qg, O, orc, fmt, group, N, K, seed=N)
        for M in (1, 7):
            X = O.randn_bf16(N + M, 2, M * K).reshape(M, K)
            Yref = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=8)
            ok, ratio, rel = within_tolerance(run(qg, p, X, f32=True), Yref)
            assert ok, (fmt, M, ratio, rel)


@pytest.mark.parametrize("fmt,group", [("mxfp4", 32), ("nvfp4", 16)])
@pytest.mark.parametrize("M", [32, 64, 200])
def test_gemm_split_k_tcgen05(qg, cuda, O, orc, fmt, group, M):
    """Few 128-row tiles and a long K: the tcgen05 path splits K across CTAs
    and reduces the FP32 partials in split order (deterministic)."""
    N, K = 300, 8192
    p, d, s, ts = packed_pair(qg, O, orc, fmt, group, N, K, seed=M)
    X = O.randn_bf16(M, 2, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=8)
    Xd = to_dev_bf16(X)
    ws = qg.make_workspace(p, M)
    a = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
    b = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
    assert same_bits(a, b)
    ok, ratio, rel = within_tolerance(a, Yref)
    assert ok and rel < 1e-5, (ratio, rel)


@pytest.mark.parametrize("group", [128, 64])
@pytest.mark.parametrize("M,K", [(20, 8192), (32, 8192), (64, 8192), (127, 4096), (200, 8192), (40, 8064)])
def test_gemm_int4_tcgen05(qg, cuda, O, orc, group, M, K):
    """INT4 from M = 17 on weights below 2^26 codes runs the tile tcgen05
    kernel, K split across CTAs (the stream-K kernel takes larger weights,
    covered with the layer shapes): two calls give the same bits, and Y is
    within the contract's tolerance (W enters the tensor core as q x scale
    rounded to f16)."""
    N = 300
    p, d, s, ts = packed_pair(qg, O, orc, "int4", group, N, K, seed=M + group)
    assert qg.launch_count(p, M)[1] == "k_umma_ts"
    X = O.randn_bf16(M, 2, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm("int4", d, s, N, K, X, group=group, nthreads=8)
    Xd = to_dev_bf16(X)
    ws = qg.make_workspace(p, M)
    a = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
    b = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
    assert same_bits(a, b)
    ok, ratio, rel = within_tolerance(a, Yref)
    assert ok and rel < 1e-3, (ratio, rel)


@pytest.mark.parametrize("group,K", [(128, 1024), (64, 1088)])
def test_gemm_int4_tcgen05_large_scales(qg, cuda, O, orc, group, K):
    """INT4 rows with FP16 group scales near 2^14 (|W| ~ 1e5) next to ordinary
    rows: q x scale would leave f16's range, so the tile tcgen05 kernel folds
    those rows by a power of two and multiplies it back in the epilogue (the
    stream-K kernel's fold is covered with the layer shapes)."""
    kernel = "k_umma_ts"
    N, M = 256, 64
    W = weights(O, N, K, seed=17)
    W[::4] *= 4e6
    Wd = to_dev_f32(W)
    p = qg.pack_int4(Wd, group)
    assert qg.launch_count(p, M)[1] == kernel
    d, s = u8(p.data), u16(p.scales)
    assert int(s.max() >> 10 & 0x1F) > 26  # the folded case is reached
    X = O.randn_bf16(9, 2, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm("int4", d, s, N, K, X, group=group, nthreads=8)
    Y = run(qg, p, X, f32=True)
    assert np.isfinite(Y).all()
    ok, ratio, rel = within_tolerance(Y, Yref)
    assert ok and rel < 1e-3, (ratio, rel)


def test_gemm_mxfp4_wide_scale_rows(qg, cuda, O, orc):
    """MXFP4 rows whose blocks span ~30 binades (1e-9 next to 1): the tcgen05
    path folds block scales relative to a per-row base exponent."""
    N, K, M = 256, 1024, 64
    W = weights(O, N, K, seed=11)
    W[:, :256] *= 1e-9
    W[::3, 512:544] *= 1000.0
    Wd = to_dev_f32(W)
    p = qg.pack_mxfp4(Wd)
    d, s = u8(p.data), u8(p.scales)
    X = O.randn_bf16(3, 2, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=8)
    ok, ratio, rel = within_tolerance(run(qg, p, X, f32=True), Yref)
    assert ok and rel < 1e-5, (ratio, rel)


def test_gemm_deterministic_and_scaling(qg, cuda, O, orc):
    N, K, M = 3000, 4096, 8
    for fmt, group in FORMATS:
        p, d, s, ts = packed_pair(qg, O, orc, fmt, group, N, K, seed=5)
        X = O.randn_bf16(5, 2, M * K).reshape(M, K)
        Xd = to_dev_bf16(X)
        ws = qg.make_workspace(p, M)
        a = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
        b = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
        assert same_bits(a, b)                    # stream-K reduction is ordered
        c = qg.gemm_w4a16(p, Xd * 2, workspace=ws, out_f32=True).cpu().numpy()
        assert same_bits(c, 2 * a)                # power-of-two scaling is exact
        # the workspace is left zeroed: a fresh one gives the same bits
        e = qg.gemm_w4a16(p, Xd, out_f32=True).cpu().numpy()
        assert same_bits(e, a)


def test_gemm_config1_fixture(qg, cuda, O):
    """MXFP4 M=1 N=K=4096 seed 0: device pack equals the reference's bytes,
    and Y is within tolerance of the reference's Y (stored bf16)."""
    import hashlib
    f = np.load(os.path.join(GOLD, "config1_mxfp4_4096.npz"))
    N, K = int(f["N"]), int(f["K"])
    W = O.randn(0, 1, N * K, 0.0, 0.02).reshape(N, K)
    p = qg.pack_mxfp4(to_dev_f32(W))
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()  # noqa: E731
    assert h(u8(p.data)) == str(f["data_sha"]) and h(u8(p.scales)) == str(f["scales_sha"])
    X = O.randn_bf16(0, 2, K).reshape(1, K)
    Yref = f["Y"]
    ok, ratio, rel = within_tolerance(run(qg, p, X, f32=True), Yref)
    assert ok and rel < 1e-5, (ratio, rel)
    Yb = run(qg, p, X)
    ok, ratio, rel = within_tolerance(Yb, O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(1, N))
    assert ok, (ratio, rel)


@pytest.mark.parametrize("fmt,group", FORMATS)
def test_gemm_reference_fixture(qg, cuda, O, fmt, group):
    f = np.load(os.path.join(GOLD, "seeded_64x256.npz"))
    N, K = int(f["N"]), int(f["K"])
    tag = f"{fmt}{group}"
    p = qg.from_host(fcode(qg, fmt, group), N, K, f[f"{tag}_data"], f[f"{tag}_scales"], float(f[f"{tag}_ts"]))
    for M in f["ms"]:
        X = O.randn_bf16(int(f["seed"]), 2, int(M) * K).reshape(int(M), K)
        ok, ratio, rel = within_tolerance(run(qg, p, X, f32=True), f[f"{tag}_Y_M{M}"])
        assert ok, (tag, M, ratio, rel)


# Full shapes of the path's configurations: sampled row blocks vs the oracle.
FULL = [
    ("nvfp4", 16, 14336, 4096, [1, 4, 8, 16]),
    ("int4", 128, 14336, 4096, [1, 4, 8, 16]),
    ("mxfp4", 32, 6144, 4096, [1, 2, 32, 64]),
    ("mxfp4", 32, 4096, 14336, [1, 16]),
    ("mxfp4", 32, 28672, 4096, [1, 8, 256]),
    ("mxfp4", 32, 8192, 28672, [1, 8]),
]


@pytest.mark.parametrize("fmt,group,N,K,ms", FULL)
def test_gemm_full_shape_sampled(qg, cuda, O, orc, fmt, group, N, K, ms):
    p, d, s, ts = packed_pair(qg, O, orc, fmt, group, N, K, seed=0)
    rng = np.random.default_rng(N ^ K)
    for M in ms:
        X = O.randn_bf16(0, 2, M * K).reshape(M, K)
        Y = run(qg, p, X, f32=True)
        for n0 in rng.integers(0, N - 64, 3):
            n0 = int(n0) // 16 * 16
            Yref = np.zeros((M, N), np.float32)
            orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, n_begin=n0, n_end=n0 + 64,
                           nthreads=8, Y=Yref)
            ok, ratio, rel = within_tolerance(Y[:, n0:n0 + 64], Yref[:, n0:n0 + 64])
            assert ok, (M, n0, ratio, rel)


def test_gemm_matches_cublas_on_dequantised_weights(qg, cuda, O, orc):
    """MXFP4 weights are exact in bf16, so a dense cuBLAS BF16 GEMM over the
    dequantised matrix is an independent full-size check."""
    N, K, M = 6144, 4096, 16
    p, d, s, ts = packed_pair(qg, O, orc, "mxfp4", 32, N, K, seed=1)
    Wb = qg.dequant(p).to(torch.bfloat16)
    X = to_dev_bf16(O.randn_bf16(1, 2, M * K).reshape(M, K))
    Yc = qg.cublas_bf16_gemm(Wb, X).float().cpu().numpy()
    Y = qg.gemm_w4a16(p, X).float().cpu().numpy()
    ok, ratio, rel = within_tolerance(Y, Yc, frob_tol=2e-3)  # both rounded to bf16 independently
    assert ok, (ratio, rel)


def test_gemm_errors(qg, cuda, O, orc):
    p, d, s, ts = packed_pair(qg, O, orc, "mxfp4", 32, 64, 256, seed=0)
    X = torch.zeros((4, 256), dtype=torch.bfloat16, device="cuda")
    small = torch.zeros(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(qg.QGemmError) as e:
        qg.gemm_w4a16(p, X, workspace=small)
    assert e.value.status == qg.ERR_WORKSPACE
    # K that is not a whole number of NVFP4 blocks (the buffers are those of
    # K = 48, larger than K = 40 needs)
    p48, *_ = packed_pair(qg, O, orc, "nvfp4", 16, 64, 48, seed=0)
    p2 = qg.Packed(p48.format, 64, 40, p48.data, p48.scales)
    with pytest.raises(qg.QGemmError) as e:
        qg.gemm_w4a16(p2, torch.zeros((1, 40), dtype=torch.bfloat16, device="cuda"))
    assert e.value.status == qg.ERR_UNSUPPORTED_SHAPE
