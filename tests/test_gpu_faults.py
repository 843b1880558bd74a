"""Scratch bounds and the bounded waits, on one GPU, through the C-ABI.

* Every dispatch path refuses a workspace one byte short of
  qgemm_workspace_size (the size covers all launches of the call, the tail
  block of a call with M % 16 != 0 included) and is correct with exactly
  that size.
* A tensor-parallel call whose peer never announces its slice: rank 0 of a
  world of 2 whose "peer" buffers are local ones nobody else writes.  The
  exchange's wait is bounded (2 s): the call ends, qgemm_tp_status reports
  QGEMM_ERR_TIMEOUT, and after the documented recovery (zero the sync blocks,
  qgemm_clear_faults) the next call is correct.  Nothing faults or hangs the
  GPU: the wait runs out on a counter that nothing raises.
"""
import ctypes as C
import time

import numpy as np
import pytest
import torch

from edge_cases import weights
from gpu_util import to_dev_bf16, to_dev_f32, within_tolerance

pytestmark = pytest.mark.gpu


def _packed(qg, O, fmt, group, N, K, seed=0):
    W = weights(O, N, K, seed=seed)
    ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
    Wd = to_dev_f32(W)
    p = {"mxfp4": lambda: qg.pack_mxfp4(Wd), "nvfp4": lambda: qg.pack_nvfp4(Wd, ts)}.get(
        fmt, lambda: qg.pack_int4(Wd, group))()
    d = p.data.cpu().numpy().view(np.uint8)
    s = p.scales.cpu().numpy().view(np.uint16 if fmt == "int4" else np.uint8)
    return p, d, s, ts


WS_CASES = [  # (format, group, N, K, M values): one per dispatch path, and INT4 tails
    ("int4", 128, 14336, 4096, [16, 17, 18, 20, 24, 40, 130]),  # TMA decode, then the tile tcgen05 kernel
    ("int4", 64, 4096, 4096, [1, 16, 33]),
    ("int4", 64, 8192, 8192, [24, 100]),                # stream-K tcgen05 (2^26 weights)
    ("mxfp4", 32, 4096, 4096, [1, 8, 16, 64]),          # TMA decode, block-scaled
    ("nvfp4", 16, 4096, 4096, [1, 16, 40, 130]),        # TMA decode, tile tcgen05
    ("nvfp4", 16, 8192, 8192, [20, 64]),                # stream-K tcgen05
    ("mxfp4", 32, 2880, 2880, [1, 40, 200]),            # LDG decode (K % 256 != 0), tile tcgen05
]


@pytest.mark.parametrize("fmt,group,N,K,ms", WS_CASES)
def test_workspace_one_byte_short_is_refused(qg, cuda, O, orc, fmt, group, N, K, ms):
    p, d, s, ts = _packed(qg, O, fmt, group, N, K)
    for M in ms:
        need = qg.workspace_size(p, M)
        assert need > 0
        Xh = O.randn_bf16(M, 2, M * K).reshape(M, K)
        X = to_dev_bf16(Xh)
        short = torch.zeros(need - 1, dtype=torch.uint8, device="cuda")
        with pytest.raises(qg.QGemmError) as e:
            qg.gemm_w4a16(p, X, workspace=short)
        assert e.value.status == qg.ERR_WORKSPACE, (M, str(e.value))
        exact = torch.zeros(need, dtype=torch.uint8, device="cuda")
        Y = qg.gemm_w4a16(p, X, workspace=exact, out_f32=True).cpu().numpy()
        Yref = orc.w4a16_gemm(fmt, d, s, N, K, Xh, group=group, tensor_scale=ts, nthreads=16)
        ok, ratio, rel = within_tolerance(Y, Yref)
        assert ok, (fmt, M, ratio, rel)


def _tp_call(qg, p, X, world, y_bufs, syncs, ws):
    qg.tp_gemm(p, X, world, 0, [y.data_ptr() for y in y_bufs], [s.data_ptr() for s in syncs], ws)


@pytest.mark.parametrize("M,kernel", [(1, "k_gemv_tma"), (32, "k_umma_bs")])
def test_tp_wait_gives_up_when_a_peer_never_arrives(qg, cuda, O, orc, M, kernel):
    fmt, N_loc, K = "mxfp4", 512, 1024
    p, d, s, ts = _packed(qg, O, fmt, 32, N_loc, K, seed=M)
    assert qg.launch_count(p, M)[1] == kernel
    Xh = O.randn_bf16(M, 2, M * K).reshape(M, K)
    X = to_dev_bf16(Xh)
    nsync = qg.tp_sync_bytes(2) // 4
    qg.clear_faults()
    # world 2: rank 1's Y_full and sync block are local buffers that no rank 1 writes
    y = [torch.zeros((M, 2 * N_loc), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    sync = [torch.zeros(nsync, dtype=torch.int32, device="cuda") for _ in range(2)]
    ws = qg.make_tp_workspace(p, M)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    _tp_call(qg, p, X, 2, y, sync, ws)
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 1.5 < waited < 30.0, waited
    flag = C.c_int32(0)
    st = qg.lib().qgemm_tp_status(C.byref(flag))
    assert st == qg.ERR_TIMEOUT and flag.value != 0
    # the GEMM status names the kernel family whose flag the exchange set
    # (1: the exchange's wait, not an mbarrier site)
    st = qg.lib().qgemm_umma_status(C.byref(flag))
    family = {"k_gemv_tma": "decode", "k_umma_bs": "block-scaled"}[kernel]
    assert st == qg.ERR_TIMEOUT and f"{family} 00000001" in qg.lib().qgemm_last_error_message().decode()
    # this rank's own slice still landed in its Y_full
    Yref = orc.w4a16_gemm(fmt, d, s, N_loc, K, Xh, nthreads=16)
    Yb = O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(M, N_loc)
    ok, ratio, rel = within_tolerance(y[0][:, :N_loc].float().cpu().numpy(), Yb)
    assert ok, (ratio, rel)
    # recovery: zero the sync blocks, clear the flags; the next call is correct
    for t in sync:
        t.zero_()
    qg.clear_faults()
    assert qg.lib().qgemm_tp_status(C.byref(flag)) == qg.OK and flag.value == 0
    y1 = torch.zeros((M, N_loc), dtype=torch.bfloat16, device="cuda")
    t0 = time.monotonic()
    _tp_call(qg, p, X, 1, [y1], [sync[0]], ws)
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 1.0
    assert qg.lib().qgemm_tp_status(C.byref(flag)) == qg.OK
    ok, ratio, rel = within_tolerance(y1.float().cpu().numpy(), Yb)
    assert ok, (ratio, rel)
    # the plain entry point is unaffected (its tickets returned to zero)
    Yp = qg.gemm_w4a16(p, X).float().cpu().numpy()
    ok, ratio, rel = within_tolerance(Yp, Yb)
    assert ok, (ratio, rel)
    qg.umma_status()
