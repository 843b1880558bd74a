"""Block-scaled tcgen05 path (k_umma_bs: MXFP4, 9 <= M <= 128) against the
oracle (dequant + double-accumulated reference GEMM, titoatwork/qgemm-mx
ref_gemm.hpp:15-27), through the C-ABI.

The kernel feeds the packed E2M1 codes and E8M0 scales straight to
tcgen05.mma.kind::mxf8f6f4.block_scale and splits X into two E4M3 terms with
their own block scales.  These cases aim at what that adds: activation tiles
of 16..128 rows (one and two scale atoms for the stacked operand), K with an
odd number of 128-k sub-steps, partial weight tiles, the E8M0 codes 0x00
(2^-127) and 0xFF (NaN), non-finite and extreme-range activations, and exact
properties (determinism, power-of-two scaling)."""
import numpy as np
import pytest
import torch

from edge_cases import weights
from gpu_util import bf16_to_np_f32, same_bits, to_dev_bf16, to_dev_f32, u8, within_tolerance

pytestmark = pytest.mark.gpu


def _uses_block_scaled(qg, p, M):
    return qg.launch_count(p, M)[1] == "k_umma_bs"


def _pack(qg, O, N, K, seed):
    W = weights(O, N, K, seed=seed)
    p = qg.pack_mxfp4(to_dev_f32(W))
    return p, u8(p.data), u8(p.scales)


def _run(qg, p, X, f32=True):
    Y = qg.gemm_w4a16(p, to_dev_bf16(X), out_f32=f32)
    torch.cuda.synchronize()
    return Y.cpu().numpy() if f32 else bf16_to_np_f32(Y)


def _x_bits(a: np.ndarray) -> np.ndarray:
    """float32 values -> bf16 bits (the values given are bf16-exact)."""
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("M", [9, 16, 40, 65, 100, 128])
def test_block_scaled_all_outputs(qg, cuda, O, orc, M):
    N, K = 300, 384  # partial second tile; K = 3 sub-steps of 128
    p, d, s = _pack(qg, O, N, K, seed=40 + M)
    assert _uses_block_scaled(qg, p, M)
    X = O.randn_bf16(M, 3, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=8)
    Y = _run(qg, p, X, f32=True)
    ok, ratio, rel = within_tolerance(Y, Yref)
    assert ok and rel < 1e-5, (ratio, rel)
    Yb = _run(qg, p, X, f32=False)
    ok, ratio, rel = within_tolerance(Yb, O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(M, N))
    assert ok, (ratio, rel)


def test_block_scaled_special_scale_codes(qg, cuda, O, orc):
    """E8M0 0x00 is 2^-127 and 0xFF is NaN (pack.hpp e8m0_decode): a NaN
    block makes its weight row's outputs NaN, a 2^-127 block contributes its
    (tiny) products."""
    N, K, M = 256, 512, 24
    p, d, s = _pack(qg, O, N, K, seed=7)
    sc = p.scales.view(torch.uint8).view(N, K // 32)
    sc[3, 5] = 0xFF          # NaN block in row 3
    sc[10, :] = 0x00         # every block of row 10 at 2^-127
    sc[20, 2] = 0x00
    torch.cuda.synchronize()
    s2 = u8(p.scales)
    X = O.randn_bf16(2, 3, M * K).reshape(M, K)
    Yref = orc.w4a16_gemm("mxfp4", d, s2, N, K, X, nthreads=8)
    Y = _run(qg, p, X, f32=True)
    assert np.array_equal(np.isnan(Y), np.isnan(Yref))
    assert np.isnan(Y[:, 3]).all()
    fin = ~np.isnan(Yref)
    err = np.abs(Y - Yref)[fin]
    scale = np.abs(Yref[fin]).max()
    assert err.max() <= 1e-5 * scale


def test_block_scaled_nonfinite_activations(qg, cuda, O, orc):
    """A NaN or infinity in X makes every output of that activation row
    non-finite, as in the reference; the other rows are unaffected."""
    N, K, M = 200, 256, 12
    p, d, s = _pack(qg, O, N, K, seed=8)
    X = O.randn_bf16(4, 3, M * K).reshape(M, K).copy()
    Xf = O.bf16_bits_to_f32(X).reshape(M, K)
    Xf[2, 37] = np.nan
    Xf[5, 200] = np.inf
    Xf[7, 0] = -np.inf
    X = _x_bits(Xf)
    Yref = orc.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=8)
    Y = _run(qg, p, X, f32=True)
    bad = [2, 5, 7]
    assert not np.isfinite(Y[bad]).any()
    assert not np.isfinite(Yref[bad]).any()
    good = [m for m in range(M) if m not in bad]
    ok, ratio, rel = within_tolerance(Y[good], Yref[good])
    assert ok and rel < 1e-5, (ratio, rel)


def test_block_scaled_activation_range(qg, cuda, O, orc):
    """Activation rows spanning the bf16 range: huge and tiny values in the
    same 32-block, a zero row.  The two E4M3 terms hold every value within 13
    binades of its block's largest exactly.  (Rows made only of bf16
    subnormals are outside this path's range: their products fall below the
    FP32 normal range inside the tensor core.)"""
    N, K, M = 256, 512, 16
    p, d, s = _pack(qg, O, N, K, seed=9)
    rng = np.random.default_rng(3)
    Xf = rng.standard_normal((M, K)).astype(np.float32)
    Xf[0] *= 1e30
    Xf[1] *= 1e-30
    Xf[2] = 0.0
    Xf[3] *= 1e-33                                   # far down the normal range
    Xf[4, ::2] *= 1e20                               # 67 binades apart inside each block
    Xf[5, ::7] *= 4096.0
    X = _x_bits(Xf)
    Yref = orc.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=8)
    Y = _run(qg, p, X, f32=True)
    assert np.array_equal(Y[2], np.zeros(N, np.float32))
    ok, ratio, rel = within_tolerance(Y, Yref)
    assert ok, (ratio, rel)
    for m in range(M):
        if m == 2:
            continue
        ok, ratio, rel = within_tolerance(Y[m:m + 1], Yref[m:m + 1])
        assert ok, (m, ratio, rel)


def test_block_scaled_deterministic_and_scaling(qg, cuda, O, orc):
    N, K, M = 3000, 4096, 32
    p, d, s = _pack(qg, O, N, K, seed=10)
    X = O.randn_bf16(6, 3, M * K).reshape(M, K)
    Xd = to_dev_bf16(X)
    ws = qg.make_workspace(p, M)
    a = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
    b = qg.gemm_w4a16(p, Xd, workspace=ws, out_f32=True).cpu().numpy()
    assert same_bits(a, b)                    # stream-K reduction is ordered
    c = qg.gemm_w4a16(p, Xd * 2, workspace=ws, out_f32=True).cpu().numpy()
    assert same_bits(c, 2 * a)                # power-of-two scaling moves only the block scales
    Yref = orc.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=16)
    ok, ratio, rel = within_tolerance(a, Yref)
    assert ok and rel < 1e-5, (ratio, rel)
