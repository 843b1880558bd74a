"""The allocation-free entry point, qgemm_gemm_w4a16_noalloc, against the
oracle and against the regular workspace entry point, called through the
C-ABI.

It exists for callers that cannot hand the library a workspace buffer: an
operator slot that passes only inputs, outputs and a stream, a plugin inside
a framework that owns the device memory pool and forbids raw cudaMalloc, or
code running while another component captures the stream in global mode.
Its scratch is one fixed device array shared by every call, so each shape is
run twice in a row: the second call must not be disturbed by what the first
left in that array.  The file sorts last so that a run stopping at its first
failure has already run every other test; it also passes alone in a fresh
process (the first call performs the one-time symbol lookup).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from edge_cases import weights
from gpu_util import to_dev_bf16, to_dev_f32, within_tolerance

pytestmark = pytest.mark.gpu

CASES = [  # (format, group, N, K, M): split tiles, several 16-row blocks, all formats
    ("mxfp4", 32, 48, 28672, 1),
    ("mxfp4", 32, 3000, 4096, 20),
    ("nvfp4", 16, 1000, 4096, 7),
    ("int4", 128, 4096, 8192, 16),
    ("int4", 64, 200, 512, 33),
    # a 16-row block followed by a tail block of 1 or 8 rows, which plans on
    # its own (one activation tile, its own occupancy and warp count)
    ("int4", 128, 14336, 4096, 17),
    ("int4", 128, 14336, 4096, 24),
]


def _pack(qg, O, fmt, group, N, K, seed):
    W = weights(O, N, K, seed=seed)
    ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
    Wd = to_dev_f32(W)
    if fmt == "mxfp4":
        return qg.pack_mxfp4(Wd), ts
    if fmt == "nvfp4":
        return qg.pack_nvfp4(Wd, ts), ts
    return qg.pack_int4(Wd, group), ts


@pytest.mark.parametrize("fmt,group,N,K,M", CASES)
def test_noalloc_matches_oracle_and_workspace_entry_point(qg, cuda, O, orc, fmt, group, N, K, M):
    lib = qg.lib()
    p, ts = _pack(qg, O, fmt, group, N, K, seed=N + M)
    Xh = O.randn_bf16(M, 2, M * K).reshape(M, K)
    X = to_dev_bf16(Xh)
    d = p.data.cpu().numpy().view(np.uint8)
    s = p.scales.cpu().numpy().view(np.uint16 if fmt == "int4" else np.uint8)
    Yref = orc.w4a16_gemm(fmt, d, s, N, K, Xh, group=group, tensor_scale=ts, nthreads=16)
    Yref_b = O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(M, N)    # stored bf16
    expected = qg.gemm_w4a16(p, X).float().cpu().numpy()   # workspace entry point
    desc = p.desc()
    if M > 16 and M % 16 and qg.launch_count(p, M)[1] in ("k_gemv", "k_gemv_tma"):
        # both entry points run the decode kernel in 16-row blocks: the
        # scratch reserved covers the tail block's plan as well as the first
        # block's
        need = lib.qgemm_workspace_size(C.byref(desc), M)
        assert need >= lib.qgemm_workspace_size(C.byref(desc), 16)
        assert need >= lib.qgemm_workspace_size(C.byref(desc), M % 16)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        Y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.qgemm_gemm_w4a16_noalloc(C.byref(desc), C.c_void_p(X.data_ptr()), M,
                                          C.c_void_p(Y.data_ptr()), stream)
        assert st == qg.OK, lib.qgemm_last_error_message()
        torch.cuda.synchronize()
        got = Y.float().cpu().numpy()
        ok, ratio, rel = within_tolerance(got, Yref_b)
        assert ok, ("oracle", call, ratio, rel)
        ok, ratio, rel = within_tolerance(got, expected)
        assert ok, ("workspace entry point", call, ratio, rel)


def test_noalloc_rejects_plans_larger_than_its_array(qg, cuda):
    """A plan whose scratch exceeds the fixed array is refused up front."""
    lib = qg.lib()
    N, K, M = 16, 600064, 16               # the f16 copy of X alone needs ~19 MB
    data = torch.zeros(N * K // 2, dtype=torch.uint8, device="cuda")
    scales = torch.full((N * K // 32,), 127, dtype=torch.uint8, device="cuda")
    p = qg.Packed(qg.MXFP4, N, K, data, scales)
    X = torch.zeros((M, K), dtype=torch.bfloat16, device="cuda")
    Y = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    desc = p.desc()
    st = lib.qgemm_gemm_w4a16_noalloc(C.byref(desc), C.c_void_p(X.data_ptr()), M, C.c_void_p(Y.data_ptr()),
                                      C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == qg.ERR_WORKSPACE
    assert b"scratch" in lib.qgemm_last_error_message()
    assert np.all(Y.float().cpu().numpy() == 0.0)
