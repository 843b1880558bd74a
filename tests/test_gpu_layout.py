"""The scale-checked layout (QGEMM_LAYOUT_SCALE_CHECKED): the kernel-optimal
layout as an offline transform, with the canonical bytes (pack.hpp:14-85) as
the parity format.

* qgemm_repack accepts weights whose scales are all inside the decode
  kernel's fast range and refuses, with QGEMM_ERR_INVALID_ARG, weights with a
  single byte outside it (MXFP4 E8M0 0x00 / 0xFF; NVFP4 E4M3 zero, subnormal
  and NaN), whatever its position; the bytes are untouched either way.
* qgemm_unpack returns the canonical bytes exactly.
* GEMM results of checked weights are bit-identical to those of the same
  canonical weights on every dispatch path (decode kernels, block-scaled and
  dequantising tcgen05 kernels, the allocation-free, grouped and
  tensor-parallel-shard entry points), and within the contract of the oracle.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import same_bits, to_dev_bf16, u8, within_tolerance

pytestmark = pytest.mark.gpu


def _weights(qg, fmt, N, K, seed, special=None):
    """Random codes and ordinary scale bytes; special = (row, block, byte) to plant."""
    rng = np.random.default_rng(seed)
    blk = 32 if fmt == "mxfp4" else 16
    codes = rng.integers(0, 16, N * K).astype(np.uint8)
    if fmt == "mxfp4":
        sb = rng.integers(0x74, 0x86, N * (K // blk)).astype(np.uint8)
    else:
        sb = rng.integers(0x30, 0x48, N * (K // blk)).astype(np.uint8)  # E4M3 normals around 1
    if special is not None:
        r, b, v = special
        sb[r * (K // blk) + b] = v
    f = qg.MXFP4 if fmt == "mxfp4" else qg.NVFP4
    p = qg.pack_codes(f, torch.from_numpy(codes).cuda(), torch.from_numpy(sb).cuda(), N, K,
                      tensor_scale=0.75)
    return p, sb


SPECIALS = {"mxfp4": [0x00, 0xFF], "nvfp4": [0x00, 0x80, 0x03, 0x85, 0x7F, 0xFF]}


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
def test_repack_accepts_clean_and_refuses_special_scales(qg, cuda, fmt):
    N, K = 1000, 2880
    blk = 32 if fmt == "mxfp4" else 16
    p, sb = _weights(qg, fmt, N, K, seed=3)
    c = qg.repack(p)
    assert c.layout == qg.SCALE_CHECKED
    assert c.data.data_ptr() == p.data.data_ptr() and np.array_equal(u8(c.scales), sb)
    back = qg.unpack(c)
    assert np.array_equal(u8(back.data), u8(p.data)) and np.array_equal(u8(back.scales), sb)
    spr = K // blk
    for i, v in enumerate(SPECIALS[fmt]):
        for r, b in ((0, 0), (N - 1, spr - 1), (517, 33 + i)):
            q, qsb = _weights(qg, fmt, N, K, seed=3, special=(r, b, v))
            with pytest.raises(ValueError):
                qg.repack(q)
            assert np.array_equal(u8(q.scales), qsb)


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
def test_checked_gemm_bits_equal_canonical(qg, cuda, O, fmt):
    N, K = 1000, 4096
    p, _ = _weights(qg, fmt, N, K, seed=7)
    c = qg.repack(p)
    for M in (1, 5, 8, 13, 16, 40, 130):
        X = to_dev_bf16(O.randn_bf16(M, 2, M * K).reshape(M, K))
        for out_f32 in (False, True):
            a = qg.gemm_w4a16(p, X, out_f32=out_f32).float().cpu().numpy()
            b = qg.gemm_w4a16(c, X, out_f32=out_f32).float().cpu().numpy()
            assert same_bits(a, b), (fmt, M, out_f32)


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
def test_checked_gemm_against_oracle(qg, cuda, O, orc, fmt):
    N, K = 640, 2048
    p, sb = _weights(qg, fmt, N, K, seed=11)
    c = qg.repack(p)
    d = u8(p.data)
    grp = 32 if fmt == "mxfp4" else 16
    for M in (1, 8, 16):
        Xh = O.randn_bf16(M + 3, 2, M * K).reshape(M, K)
        Y = qg.gemm_w4a16(c, to_dev_bf16(Xh), out_f32=True).cpu().numpy()
        Yref = orc.w4a16_gemm(fmt, d, sb, N, K, Xh, group=grp, tensor_scale=c.tensor_scale, nthreads=16)
        ok, ratio, rel = within_tolerance(Y, Yref)
        assert ok, (fmt, M, ratio, rel)


def test_checked_noalloc_grouped_and_shards(qg, cuda, O):
    N, K = 512, 2048
    ps = [_weights(qg, "mxfp4", N, K, seed=20 + e)[0] for e in range(3)]
    cs = [qg.repack(p) for p in ps]
    # allocation-free entry (LDG-fed decode kernel): reads the bytes as canonical
    M = 3
    X = to_dev_bf16(O.randn_bf16(3, 2, M * K).reshape(M, K))
    ya = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    yb = torch.empty_like(ya)
    for p, y in ((ps[0], ya), (cs[0], yb)):
        d = p.desc()
        st = qg.lib().qgemm_gemm_w4a16_noalloc(C.byref(d), C.c_void_p(X.data_ptr()), M, C.c_void_p(y.data_ptr()),
                                                C.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == qg.OK
    assert same_bits(ya.float().cpu().numpy(), yb.float().cpu().numpy())
    # grouped: one active expert plans like the single call (same bits), checked or mixed
    counts = [0, 7, 0]
    Xg = to_dev_bf16(O.randn_bf16(4, 2, 7 * K).reshape(7, K))
    ys = qg.gemm_w4a16(ps[1], Xg)
    for experts in (cs, [ps[0], cs[1], ps[2]], [cs[0], ps[1], cs[2]]):
        yg = qg.grouped_gemm_w4a16(experts, Xg, counts)
        assert same_bits(yg.float().cpu().numpy(), ys.float().cpu().numpy())
    # a row shard of checked weights is checked
    sh = cs[2].shard_rows(128, 384)
    assert sh.layout == qg.SCALE_CHECKED
    assert same_bits(qg.gemm_w4a16(sh, X).float().cpu().numpy(),
                     qg.gemm_w4a16(ps[2].shard_rows(128, 384), X).float().cpu().numpy())
