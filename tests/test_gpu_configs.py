"""Parity on the configurations the benchmark numbers are quoted on, and the
reference's structured probes routed through every GEMM kernel.

Against the oracle (dequant + double-accumulated reference GEMM,
titoatwork/qgemm-mx include/qgemm/ref_gemm.hpp:15-27), through the C-ABI:

* the 70B-class MXFP4 layer set (QKV 10240x8192, gate-up 57344x8192, down
  8192x28672; M in {1, 8, 32, 64}) -- the bench workload, one kernel per
  M range (TMA decode for M <= 8, block-scaled tcgen05 for M = 32, 64);
* the 8B-class MXFP4 layer set at the M values no other test covers, the
  O projection 4096x4096 included;
* NVFP4 and INT4 layers of 2^26 weights or more at 17 <= M < 128 (the
  stream-K tcgen05 kernel), INT4 rows with scales that need folding among them;
* compute-bound prefill, NVFP4 (28672, 8192) and (8192, 28672) at M = 2048;
* exact probes (one nonzero weight per row, random codes with prime / narrow
  scales, sparse power-of-two activations): every product and partial sum is
  representable in FP32, so the device result must equal the oracle's bits
  (the reference's acceptance rule "structured correctness probes exact",
  docs/PROJECT-v2.0-fp4-hopper.md:223).

Large shapes draw W on the device from torch's seeded generator (the bytes the
oracle sees are the device-packed bytes, themselves checked against the
oracle's packer on sampled rows) and check sampled 64-column blocks of every
activation row, or sampled activation rows for prefill.  Tolerance
(tests/gpu_util.py): per row max-abs <= 1e-2 * ||Y_ref row||_inf and relative
Frobenius <= 1e-3; bf16 output against the oracle rounded to bf16.
"""
import numpy as np
import pytest
import torch

import probes as P
from gpu_util import same_bits, to_dev_bf16, u8, u16, within_tolerance

pytestmark = pytest.mark.gpu


def _dev_pack(qg, fmt, group, N, K, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    W = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float32) * 0.02
    if fmt == "mxfp4":
        p = qg.pack_mxfp4(W)
    elif fmt == "nvfp4":
        p = qg.pack_nvfp4(W)
    else:
        p = qg.pack_int4(W, group)
    return W, p


def _check_packed_rows(orc, fmt, group, W, p, rows):
    """Device bytes of sampled rows equal the oracle packer's (rows pack
    independently; the NVFP4 tensor scale is the one the device used)."""
    N, K = W.shape
    blk = {"mxfp4": 32, "nvfp4": 16}.get(fmt, group)
    d_all, s_all = u8(p.data), (u16(p.scales) if fmt == "int4" else u8(p.scales))
    for n0 in rows:
        Wr = W[n0:n0 + 16].cpu().numpy()
        st, d, s = orc.pack(fmt, Wr, group=group, tensor_scale=p.tensor_scale)
        assert st == 0
        assert np.array_equal(d_all[n0 * K // 2:(n0 + 16) * K // 2], d), (fmt, n0)
        assert np.array_equal(s_all[n0 * (K // blk):(n0 + 16) * (K // blk)], s), (fmt, n0)


def _host_bytes(fmt, p):
    return u8(p.data), (u16(p.scales) if fmt == "int4" else u8(p.scales))


def _sampled_blocks(qg, orc, O, fmt, group, p, d, s, M, seed, nblocks=4, expect_kernel=None, rel_f32=1e-5,
                    frob_bf16=1e-3):
    N, K = p.N, p.K
    if expect_kernel:
        assert qg.launch_count(p, M)[1] == expect_kernel, (M, qg.launch_count(p, M))
    X = O.randn_bf16(seed, 2, M * K).reshape(M, K)
    Xd = to_dev_bf16(X)
    Yb = qg.gemm_w4a16(p, Xd).float().cpu().numpy()
    Yf = qg.gemm_w4a16(p, Xd, out_f32=True).cpu().numpy()
    rng = np.random.default_rng(seed * 7919 + M)
    for n0 in sorted(set(int(v) // 16 * 16 for v in rng.integers(0, N - 64, nblocks))) + [N - 64]:
        Yref = np.zeros((M, N), np.float32)
        orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=p.tensor_scale, n_begin=n0,
                       n_end=n0 + 64, nthreads=16, Y=Yref)
        ref = Yref[:, n0:n0 + 64]
        ok, ratio, rel = within_tolerance(Yf[:, n0:n0 + 64], ref)
        assert ok and rel < rel_f32, ("f32", M, n0, ratio, rel)
        refb = O.bf16_bits_to_f32(O.f32_to_bf16_bits(ref)).reshape(ref.shape)
        ok, ratio, rel = within_tolerance(Yb[:, n0:n0 + 64], refb, frob_tol=frob_bf16)
        assert ok, ("bf16", M, n0, ratio, rel)


# ---- the bench workload: 70B-class MXFP4 layer set -----------------------------------

CFG70B = [("qkv", 10240, 8192), ("gate_up", 57344, 8192), ("down", 8192, 28672)]


@pytest.mark.parametrize("name,N,K", CFG70B)
def test_70b_layer_set_all_m(qg, cuda, O, orc, name, N, K):
    W, p = _dev_pack(qg, "mxfp4", 32, N, K, seed=N + K)
    _check_packed_rows(orc, "mxfp4", 32, W, p, [0, N // 2 + 16, N - 16])
    del W
    torch.cuda.empty_cache()
    d, s = _host_bytes("mxfp4", p)
    for M, kern in ((1, "k_gemv_tma"), (8, "k_gemv_tma"), (32, "k_umma_bs"), (64, "k_umma_bs")):
        _sampled_blocks(qg, orc, O, "mxfp4", 32, p, d, s, M, seed=M, expect_kernel=kern)


# ---- 8B-class MXFP4 layer set at the remaining M of the sweep ------------------------

CFG8B = [
    ("o_proj", 4096, 4096, [1, 2, 4, 16, 32, 128, 256]),
    ("qkv", 6144, 4096, [4, 8, 16, 128, 256]),
    ("gate_up", 28672, 4096, [2, 4, 16, 32, 64, 128]),
    ("down", 4096, 14336, [2, 4, 8, 32, 64, 128, 256]),
]


@pytest.mark.parametrize("name,N,K,ms", CFG8B)
def test_8b_layer_set_sweep(qg, cuda, O, orc, name, N, K, ms):
    W, p = _dev_pack(qg, "mxfp4", 32, N, K, seed=N ^ K)
    _check_packed_rows(orc, "mxfp4", 32, W, p, [16, N - 16])
    del W
    d, s = _host_bytes("mxfp4", p)
    for M in ms:
        _sampled_blocks(qg, orc, O, "mxfp4", 32, p, d, s, M, seed=M + 3, nblocks=3)


# ---- NVFP4 / INT4 layers of 2^26 weights and more at 17 <= M < 128 ----------------------
# The stream-K tcgen05 kernel: tiles split across CTAs and summed by the last
# arriver, per-segment INT4 row folds; M = 17 and 20 pad X to 32 rows.  INT4
# enters the tensor core as q x scale rounded to f16 (relative Frobenius
# bound 1e-3 on the FP32 output, as for the tile kernel).

CFG_SK = [
    ("nvfp4", 16, 10240, 8192, [17, 40, 64, 100]),
    ("int4", 128, 10240, 8192, [20, 32, 64, 127]),
    ("int4", 64, 8192, 28672, [24, 96]),
]


@pytest.mark.parametrize("fmt,group,N,K,ms", CFG_SK)
def test_stream_k_layers(qg, cuda, O, orc, fmt, group, N, K, ms):
    W, p = _dev_pack(qg, fmt, group, N, K, seed=N + 3 * K + group)
    _check_packed_rows(orc, fmt, group, W, p, [16, N - 16])
    del W
    d, s = _host_bytes(fmt, p)
    for M in ms:
        _sampled_blocks(qg, orc, O, fmt, group, p, d, s, M, seed=M + 5, nblocks=3, expect_kernel="k_umma_sk",
                        rel_f32=1e-3 if fmt == "int4" else 1e-5)


def test_stream_k_int4_large_scales(qg, cuda, O, orc):
    """Every fourth row's FP16 group scales near 2^14 (|W| ~ 1e5): the
    stream-K kernel folds those rows by a power of two per segment and
    multiplies it back in the epilogue.  The bf16 output is held to 2e-3
    relative Frobenius: the FP32 result's error from q x scale rounded to f16
    (below 1e-3) flips the bf16 rounding of some outputs by one unit (2^-8
    relative), which the columns of the large rows carry."""
    N, K = 8192, 8192
    g = torch.Generator(device="cuda")
    g.manual_seed(29)
    W = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float32) * 0.02
    W[::4] *= 2e6  # group scales ~1.5e4, the largest below f16's 65504
    p = qg.pack_int4(W, 128)
    del W
    d, s = _host_bytes("int4", p)
    assert int(s.max() >> 10 & 0x1F) > 26  # the folded case is reached
    for M in (24, 64):
        _sampled_blocks(qg, orc, O, "int4", 128, p, d, s, M, seed=M + 7, nblocks=3, expect_kernel="k_umma_sk",
                        rel_f32=1e-3, frob_bf16=2e-3)


# ---- compute-bound prefill (NVFP4, M = 2048) ------------------------------------------

@pytest.mark.parametrize("N,K", [(28672, 8192), (8192, 28672)])
def test_prefill_sampled_rows(qg, cuda, O, orc, N, K):
    M = 2048
    W, p = _dev_pack(qg, "nvfp4", 16, N, K, seed=N * 3 + K)
    _check_packed_rows(orc, "nvfp4", 16, W, p, [32, N - 16])
    del W
    torch.cuda.empty_cache()
    assert qg.launch_count(p, M)[1] == "k_umma_ts"
    d, s = _host_bytes("nvfp4", p)
    X = O.randn_bf16(11, 2, M * K).reshape(M, K)
    Y = qg.gemm_w4a16(p, to_dev_bf16(X), out_f32=True)
    rng = np.random.default_rng(N + K)
    rows = np.sort(rng.choice(M, 64, replace=False))
    rows[-1] = M - 1
    Ys = Y[torch.from_numpy(rows).cuda()].cpu().numpy()
    del Y
    Xs = np.ascontiguousarray(X[rows])
    for n0 in sorted(set(int(v) // 16 * 16 for v in rng.integers(0, N - 64, 8))):
        Yref = np.zeros((64, N), np.float32)
        orc.w4a16_gemm("nvfp4", d, s, N, K, Xs, tensor_scale=p.tensor_scale, n_begin=n0, n_end=n0 + 64,
                       nthreads=16, Y=Yref)
        ok, ratio, rel = within_tolerance(Ys[:, n0:n0 + 64], Yref[:, n0:n0 + 64])
        # FP32 output: only the summation order differs from the double-accumulated
        # reference, ~1e-5 relative over K = 28672
        assert ok and rel < 1e-4, (n0, ratio, rel)


# ---- exact probes through every kernel -------------------------------------------------

PROBE_FORMATS = [("mxfp4", 32), ("nvfp4", 16), ("int4", 128), ("int4", 64)]
# M values that route to each kernel: 1 and 8 decode (TMA or LDG), 12 block-scaled
# (MXFP4) / decode, 40 block-scaled (MXFP4) / tile tcgen05 (NVFP4, INT4), 130
# tile tcgen05 (every format).  The stream-K tcgen05 kernel takes weights of
# 2^26 codes and more: test_exact_random_codes_stream_k below.
PROBE_M = [1, 8, 12, 40, 130]


def _fcode(qg, fmt, group):
    return {"mxfp4": qg.MXFP4, "nvfp4": qg.NVFP4}.get(fmt, qg.INT4_G128 if group == 128 else qg.INT4_G64)


def _exact(qg, O, orc, fmt, group, N, K, d, s, ts, X):
    p = qg.from_host(_fcode(qg, fmt, group), N, K, d, s, ts)
    M = X.shape[0]
    Yref = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=16)
    Xd = to_dev_bf16(X)
    Yf = qg.gemm_w4a16(p, Xd, out_f32=True).cpu().numpy()
    assert same_bits(Yf, Yref), (fmt, M, qg.launch_count(p, M), float(np.abs(Yf - Yref).max()))
    Yb = qg.gemm_w4a16(p, Xd).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(Yb, O.f32_to_bf16_bits(Yref).reshape(M, N)), (fmt, M)
    return Yref


@pytest.mark.parametrize("fmt,group", PROBE_FORMATS)
@pytest.mark.parametrize("M", PROBE_M)
def test_exact_random_codes(qg, cuda, O, orc, fmt, group, M):
    """Random codes over the full code set with narrow-range scales (primes for
    INT4) against sparse +-{0.5, 1, 2} activations: exact in FP32."""
    N, K = 256, 1024
    d, s, ts = P.random_weights(fmt, group, N, K, seed=M)
    X = P.sparse_activations(M, K, seed=100 + M)
    Yref = _exact(qg, O, orc, fmt, group, N, K, d, s, ts, X)
    assert np.count_nonzero(Yref) > Yref.size // 2  # the probe is not trivially zero


@pytest.mark.parametrize("fmt,group", PROBE_FORMATS)
@pytest.mark.parametrize("M", PROBE_M)
def test_exact_one_hot_permutation(qg, cuda, O, orc, fmt, group, M):
    """One nonzero weight per row at k = pi(n), one-hot activation rows at
    k = pi(m mod N): Y[m, n] is that weight when n = m mod N and zero
    elsewhere, so a wrong row, column, nibble or scale index shows up."""
    N, K = 256, 1024
    d, s, ts, pi = P.permutation_probe(fmt, group, N, K)
    X = P.one_hot_rows(M, K, pi[np.arange(M) % N])
    Yref = _exact(qg, O, orc, fmt, group, N, K, d, s, ts, X)
    nz = np.argwhere(Yref != 0)
    assert np.array_equal(nz[:, 1], np.arange(M) % N)


@pytest.mark.parametrize("fmt,group", [("nvfp4", 16), ("int4", 128), ("int4", 64)])
def test_exact_random_codes_stream_k(qg, cuda, O, orc, fmt, group):
    """The random-code probe on 65536 x 1024 weights (2^26 codes), which
    route M = 40 to the stream-K tcgen05 kernel.  K as in the probes above
    keeps every partial sum exact, so the split tiles' partials, parked by
    several CTAs and summed by the last, must give the oracle's bits."""
    N, K, M = 65536, 1024, 40
    d, s, ts = P.random_weights(fmt, group, N, K, seed=M + group)
    assert qg.launch_count(qg.from_host(_fcode(qg, fmt, group), N, K, d, s, ts), M)[1] == "k_umma_sk"
    X = P.sparse_activations(M, K, seed=140 + group)
    Yref = _exact(qg, O, orc, fmt, group, N, K, d, s, ts, X)
    assert np.count_nonzero(Yref) > Yref.size // 2
