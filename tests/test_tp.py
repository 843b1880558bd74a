"""Tensor-parallel path: W sharded along N over the GPUs of one node, each
rank computing its Y slice and the slices gathered into every rank's Y.

CPU (gloo, world sizes 2, 4, 8): the sharding the multi-GPU path relies on -- a
rank's shard of packed W is a contiguous slice of the full packing's data
and scales, its Y slice is the full GEMM's column block, and the gathered
slices are the full result -- checked with the oracle; plus the C-ABI's
argument checks, which return before any device work.

GPU (two processes, one GPU each, skipped with fewer than two GPUs):
qgemm_tp_gemm_w4a16 through CUDA IPC peer mappings against the oracle.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

from gpu_util import within_tolerance

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------------------
# CPU: sharding with the oracle, 2 / 4 / 8 gloo ranks
# ---------------------------------------------------------------------------

def _cpu_rank(rank, world, port, fmt, N, K, M, out):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist
    import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        orc = O.oracle()
        W = O.randn(11, 1, N * K, 0.0, 0.02).reshape(N, K)
        X = O.randn_bf16(11, 2, M * K).reshape(M, K)
        n_loc = N // world
        shard = np.ascontiguousarray(W[rank * n_loc:(rank + 1) * n_loc])
        st, d, s = orc.pack(fmt, shard)
        assert st == 0
        y = orc.w4a16_gemm(fmt, d, s, n_loc, K, X)                       # [M][n_loc]
        parts = [torch.zeros((M, n_loc), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(y))
        packs = [None] * world
        dist.all_gather_object(packs, (d.tobytes(), s.tobytes()))
        if rank == 0:
            out.put((np.concatenate([p.numpy() for p in parts], axis=1), packs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,N,K,M,world", [("mxfp4", 256, 512, 3, 2), ("nvfp4", 128, 256, 1, 2),
                                              ("mxfp4", 256, 512, 3, 4), ("mxfp4", 1024, 256, 2, 8)])
def test_shards_are_row_slices_and_gather_to_full_result(O, orc, fmt, N, K, M, world):
    """World sizes of the scaling runs (2, 4, 8): every rank's packed shard is
    its contiguous row slice and the gathered Y equals the full result."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank, args=(r, world, port, fmt, N, K, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        Ygath, packs = q.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    W = O.randn(11, 1, N * K, 0.0, 0.02).reshape(N, K)
    X = O.randn_bf16(11, 2, M * K).reshape(M, K)
    st, d, s = orc.pack(fmt, W)
    assert st == 0
    Yfull = orc.w4a16_gemm(fmt, d, s, N, K, X)
    # bit-exact: packing and the reference GEMM are row-independent
    assert np.array_equal(Ygath, Yfull)
    n_loc = N // world
    dpr, spr = K // 2, s.size // N
    for r, (db, sb) in enumerate(packs):
        assert db == d[r * n_loc * dpr:(r + 1) * n_loc * dpr].tobytes()
        assert sb == s[r * n_loc * spr:(r + 1) * n_loc * spr].tobytes()


def test_tp_argument_checks_return_before_device_work(qg):
    lib = qg.lib()
    null = C.c_void_p(0)
    w = qg._Weights(qg.MXFP4, 0, 64, 256, C.c_void_p(0x1000), C.c_void_p(0x2000), 1.0)
    yp = (C.c_void_p * 2)(0x10000, 0x20000)
    sp = (C.c_void_p * 2)(0x30000, 0x40000)
    x = C.c_void_p(0x50000)
    assert lib.qgemm_tp_gemm_w4a16(C.byref(w), x, 1, 0, 0, yp, sp, null, 0, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_tp_gemm_w4a16(C.byref(w), x, 1, 9, 0, yp, sp, null, 0, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_tp_gemm_w4a16(C.byref(w), x, 1, 2, 2, yp, sp, null, 0, null) == qg.ERR_INVALID_ARG
    assert lib.qgemm_tp_gemm_w4a16(C.byref(w), x, 0, 2, 0, yp, sp, null, 0, null) == qg.ERR_INVALID_ARG
    bad = (C.c_void_p * 2)(0x10000, 0)
    assert lib.qgemm_tp_gemm_w4a16(C.byref(w), x, 1, 2, 0, bad, sp, null, 0, null) == qg.ERR_INVALID_ARG
    mis = (C.c_void_p * 2)(0x10008, 0x20000)
    assert lib.qgemm_tp_gemm_w4a16(C.byref(w), x, 1, 2, 0, mis, sp, null, 0, null) == qg.ERR_INVALID_ARG
    assert qg.tp_sync_bytes(8) >= 9 * 4


# ---------------------------------------------------------------------------
# GPU: two ranks, one GPU each, peer mappings by CUDA IPC
# ---------------------------------------------------------------------------

def _gpu_rank(rank, world, port, cases, out):
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    import oracle as O
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    qg = importlib.import_module("qgemm-mx_b200")
    res = []
    opened = []
    try:
        for fmt, N, K, M in cases:
            fcode = {"mxfp4": qg.MXFP4, "nvfp4": qg.NVFP4, "int4": qg.INT4_G128}[fmt]
            W = O.randn(21, 1, N * K, 0.0, 0.02).reshape(N, K)
            X = O.randn_bf16(21, 2, M * K).reshape(M, K)
            n_loc = N // world
            Wl = torch.from_numpy(np.ascontiguousarray(W[rank * n_loc:(rank + 1) * n_loc])).cuda()
            # NVFP4: one tensor scale for the whole W, shared by every shard
            p = qg.pack_nvfp4(Wl, O.nvfp4_tensor_scale(W)) if fmt == "nvfp4" else qg.pack(fcode, Wl)
            Xd = torch.from_numpy(X.view(np.int16)).cuda().view(torch.bfloat16)
            buf = torch.zeros(256 + M * N * 2, dtype=torch.uint8, device="cuda")
            handles = [None] * world
            dist.all_gather_object(handles, qg.ipc_handle(buf))
            bases = []
            for r in range(world):
                if r == rank:
                    bases.append(buf.data_ptr())
                else:
                    b0, ptr = qg.ipc_open(*handles[r])
                    opened.append(b0)
                    bases.append(ptr)
            ws = qg.make_tp_workspace(p, M)
            torch.cuda.synchronize()
            dist.barrier()
            for _ in range(3):  # repeated calls: the epoch counter advances in step on both ranks
                qg.tp_gemm(p, Xd, world, rank, [b + 256 for b in bases], bases, ws)
            torch.cuda.synchronize()
            qg.tp_status()
            Y = buf[256:].view(torch.bfloat16).view(M, N).float().cpu().numpy()
            dist.barrier()  # peers finished writing before this buffer is released
            for b0 in opened:
                qg.ipc_close(b0)
            opened.clear()
            res.append(Y)
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_tp_gemm_two_gpus_matches_oracle(O, orc):
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    # decode (TMA and LDG-fed), block-scaled tcgen05 with split tiles (its
    # fixup kernel stores the slices and runs the exchange), NVFP4 and INT4
    # on the stream-K tcgen05 kernel (shards of 2^26 weights; M = 20 has X
    # padded to 32 rows), and NVFP4 / INT4 shards below that size, or with
    # K % 256 != 0, on the tile tcgen05 kernel (slice computed, then gathered)
    cases = [("mxfp4", 1024, 1024, 1), ("mxfp4", 2048, 4096, 8), ("nvfp4", 768, 1024, 40), ("int4", 512, 1024, 5),
             ("mxfp4", 1024, 512, 70), ("mxfp4", 2048, 8192, 32), ("nvfp4", 1024, 1024, 20),
             ("int4", 512, 1024, 24), ("int4", 1024, 2048, 64), ("int4", 512, 1152, 24),
             ("nvfp4", 16384, 8192, 20), ("int4", 16384, 8192, 40)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=300) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for ci, (fmt, N, K, M) in enumerate(cases):
        W = O.randn(21, 1, N * K, 0.0, 0.02).reshape(N, K)
        X = O.randn_bf16(21, 2, M * K).reshape(M, K)
        n_loc = N // world
        parts = []
        ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
        for r in range(world):
            st, d, s = orc.pack(fmt, np.ascontiguousarray(W[r * n_loc:(r + 1) * n_loc]), tensor_scale=ts)
            parts.append(orc.w4a16_gemm(fmt, d, s, n_loc, K, X, tensor_scale=ts, nthreads=16))
        Yref = np.concatenate(parts, axis=1)
        Yref = O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(M, N)  # Y is stored bf16, like the reference
        for r in range(world):
            ok, ratio, rel = within_tolerance(got[r][ci], Yref)
            assert ok, (fmt, N, K, M, r, ratio, rel)
        assert np.array_equal(got[0][ci], got[1][ci])  # every rank holds the same Y
