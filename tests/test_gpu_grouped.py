"""Grouped (mixture-of-experts) GEMM and workspace sharing, through the C-ABI.

qgemm_grouped_gemm_w4a16 runs E experts of one format and shape; expert e
owns rows offs[e] .. offs[e] + M[e] of X and Y.  The reference plans this
variant ("grouped / MoE with variable M per expert",
docs/PROJECT-v2.0-fp4-hopper.md:89-90) without building it, so parity is
per expert against the oracle GEMM (ref_gemm.hpp:15-27, tolerance of
tests/gpu_util.py) and against the library's own single-expert call:

* skewed routing (empty experts, 1-row experts, experts above the 16-row
  fused limit) for MXFP4, NVFP4 with a different tensor scale per expert,
  and INT4 g128;
* more than 32 active experts (two fused launches);
* one active expert: the fused launch plans exactly like the single call, so
  the bits must match; experts above 16 rows run the single-call kernels:
  bits match; fused INT4 experts agree with their single calls within the
  contract (their stream-K split points differ);
* rows that no expert owns keep their contents;
* a realistic decode step: 32 experts of 4096 x 4096, top-2 routing of 64
  tokens with skew, sampled output blocks;
* one workspace shared by calls of different M (the tickets sit at the
  start of every layout): results equal those of fresh workspaces, bit for
  bit.
"""
import numpy as np
import pytest
import torch

from gpu_util import to_dev_bf16, u8, u16, within_tolerance

pytestmark = pytest.mark.gpu


def _experts(qg, fmt, E, N, K, seed, group=128):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    out = []
    for e in range(E):
        W = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float32) * (0.01 + 0.005 * (e % 5))
        if fmt == "mxfp4":
            out.append(qg.pack_mxfp4(W))
        elif fmt == "nvfp4":
            out.append(qg.pack_nvfp4(W))  # each expert its own tensor scale
        else:
            out.append(qg.pack_int4(W, group))
    return out


def _host(fmt, p):
    return u8(p.data), (u16(p.scales) if fmt == "int4" else u8(p.scales))


def _check_expert(orc, O, fmt, group, p, X, Y, off, m, cols=None):
    """Rows off .. off + m of the bf16 result Y against the oracle."""
    if m == 0:
        return
    d, s = _host(fmt, p)
    N, K = p.N, p.K
    Xe = X[off:off + m]
    blocks = cols or [(0, N)]
    for n0, n1 in blocks:
        Yref = np.zeros((m, N), np.float32)
        orc.w4a16_gemm(fmt, d, s, N, K, Xe, group=group, tensor_scale=p.tensor_scale, n_begin=n0, n_end=n1,
                       nthreads=16, Y=Yref)
        ref = Yref[:, n0:n1]
        refb = O.bf16_bits_to_f32(O.f32_to_bf16_bits(ref)).reshape(ref.shape)
        ok, ratio, rel = within_tolerance(Y[off:off + m, n0:n1], refb)
        assert ok, (fmt, off, m, n0, ratio, rel)


@pytest.mark.parametrize("fmt,group", [("mxfp4", 32), ("nvfp4", 16), ("int4", 128)])
def test_skewed_routing(qg, cuda, O, orc, fmt, group):
    N, K = 640, 1024
    counts = [0, 1, 3, 16, 7, 0, 2, 24, 9, 1]
    experts = _experts(qg, fmt, len(counts), N, K, seed=5 + len(fmt))
    rows = sum(counts)
    X = O.randn_bf16(17, 2, rows * K).reshape(rows, K)
    Y = qg.grouped_gemm_w4a16(experts, to_dev_bf16(X), counts).float().cpu().numpy()
    off = 0
    for p, m in zip(experts, counts):
        _check_expert(orc, O, fmt, group, p, X, Y, off, m)
        off += m


def test_more_than_32_experts(qg, cuda, O, orc):
    N, K = 384, 512
    rng = np.random.default_rng(3)
    counts = [int(c) for c in rng.integers(1, 5, 41)]
    counts[7] = 0
    experts = _experts(qg, "mxfp4", len(counts), N, K, seed=41)
    rows = sum(counts)
    X = O.randn_bf16(23, 2, rows * K).reshape(rows, K)
    Y = qg.grouped_gemm_w4a16(experts, to_dev_bf16(X), counts).float().cpu().numpy()
    off = 0
    for p, m in zip(experts, counts):
        _check_expert(orc, O, "mxfp4", 32, p, X, Y, off, m)
        off += m


@pytest.mark.parametrize("fmt,m", [("mxfp4", 5), ("nvfp4", 13), ("int4", 6), ("mxfp4", 40)])
def test_single_active_expert_matches_single_call(qg, cuda, O, fmt, m):
    N, K = 1024, 2048
    experts = _experts(qg, fmt, 4, N, K, seed=77)
    counts = [0, 0, m, 0]
    X = O.randn_bf16(31, 2, m * K).reshape(m, K)
    Xd = to_dev_bf16(X)
    Yg = qg.grouped_gemm_w4a16(experts, Xd, counts)
    Ys = qg.gemm_w4a16(experts[2], Xd)
    assert torch.equal(Yg.view(torch.int16), Ys.view(torch.int16))


def test_int4_experts_match_single_calls(qg, cuda, O):
    N, K = 512, 1024
    counts = [2, 0, 17, 1]
    experts = _experts(qg, "int4", len(counts), N, K, seed=9)
    rows = sum(counts)
    X = to_dev_bf16(O.randn_bf16(37, 2, rows * K).reshape(rows, K))
    Yg = qg.grouped_gemm_w4a16(experts, X, counts)
    off = 0
    for p, m in zip(experts, counts):
        if m:
            Ys = qg.gemm_w4a16(p, X[off:off + m])
            if m > 16:  # a regular call: the same kernels and plan
                assert torch.equal(Yg[off:off + m].view(torch.int16), Ys.view(torch.int16)), off
            else:       # fused with the other small expert
                ok, ratio, rel = within_tolerance(Yg[off:off + m].float().cpu().numpy(), Ys.float().cpu().numpy())
                assert ok, (off, ratio, rel)
        off += m


def test_uncovered_rows_untouched(qg, cuda, O):
    N, K = 256, 512
    experts = _experts(qg, "mxfp4", 3, N, K, seed=13)
    counts, offs = [2, 3, 1], [1, 6, 10]
    X = to_dev_bf16(O.randn_bf16(43, 2, 12 * K).reshape(12, K))
    out = torch.full((12, N), 7.0, dtype=torch.bfloat16, device="cuda")
    qg.grouped_gemm_w4a16(experts, X, counts, offsets=offs, out=out)
    covered = set()
    for o, c in zip(offs, counts):
        covered.update(range(o, o + c))
    for r in range(12):
        if r not in covered:
            assert bool((out[r] == 7.0).all()), r
        else:
            assert not bool((out[r] == 7.0).all()), r


def test_moe_decode_step_32x4096(qg, cuda, O, orc):
    """32 experts of 4096 x 4096 (MXFP4), 64 tokens routed top-2 with skew."""
    E, N, K, tokens = 32, 4096, 4096, 64
    rng = np.random.default_rng(2024)
    pop = rng.zipf(1.5, 4 * E) % E
    picks = np.concatenate([rng.choice(pop, 2, replace=False) for _ in range(tokens)])
    counts = [int((picks == e).sum()) for e in range(E)]
    assert sum(counts) == 2 * tokens
    experts = _experts(qg, "mxfp4", E, N, K, seed=99)
    rows = sum(counts)
    X = O.randn_bf16(53, 2, rows * K).reshape(rows, K)
    Y = qg.grouped_gemm_w4a16(experts, to_dev_bf16(X), counts).float().cpu().numpy()
    off = 0
    for e, (p, m) in enumerate(zip(experts, counts)):
        n0 = int(rng.integers(0, N // 64)) * 64
        _check_expert(orc, O, "mxfp4", 32, p, X, Y, off, m, cols=[(n0, n0 + 64), (N - 64, N)])
        off += m


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4", "int4"])
def test_workspace_shared_across_m(qg, cuda, O, fmt):
    """One workspace for calls of M = 1, 8, 130, 32, 64, 3, 16 in stream order."""
    N, K = 2048, 4096
    p = _experts(qg, fmt, 1, N, K, seed=61)[0]
    ms = [1, 8, 130, 32, 64, 3, 16]
    size = max(qg.workspace_size(p, m) for m in ms)
    ws = torch.zeros(size, dtype=torch.uint8, device="cuda")
    Xs = {m: to_dev_bf16(O.randn_bf16(m, 2, m * K).reshape(m, K)) for m in ms}
    shared = [qg.gemm_w4a16(p, Xs[m], workspace=ws) for m in ms]
    for m, y in zip(ms, shared):
        fresh = qg.gemm_w4a16(p, Xs[m])
        assert torch.equal(y.view(torch.int16), fresh.view(torch.int16)), (fmt, m)
    assert not bool(ws[:256].any())  # tickets back at zero
