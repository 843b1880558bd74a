"""The cuBLASLt FP8 baseline (qgemm_cublaslt_fp8_gemm), the dense "vs FP8"
comparison the reference plans (docs/BASELINE_STUDY.md:23), against a
float64 host product of the same E4M3 values: Y = (X8 sx) (W8 sw)^T with
per-tensor scales amax / 448, bf16 output within the tolerance of
tests/gpu_util.py (per row max-abs <= 1e-2 ||row||_inf, relative Frobenius
<= 1e-3) of the reference rounded to bf16."""
import numpy as np
import pytest
import torch

from gpu_util import bf16_to_np_f32, within_tolerance

pytestmark = pytest.mark.gpu


def _e4m3(A: torch.Tensor):
    s = float(A.abs().max()) / 448.0
    return (A / s).to(torch.float8_e4m3fn), torch.tensor([s], dtype=torch.float32, device=A.device)


@pytest.mark.parametrize("N,K,M", [(256, 512, 1), (256, 512, 16), (1024, 4096, 33), (4096, 1024, 64)])
def test_fp8_baseline_matches_reference(qg, cuda, N, K, M):
    g = torch.Generator(device="cuda").manual_seed(N + K + M)
    W = torch.randn((N, K), generator=g, device="cuda") * 0.02
    X = torch.randn((M, K), generator=g, device="cuda")
    W8, sw = _e4m3(W)
    X8, sx = _e4m3(X)
    Y = qg.cublaslt_fp8_gemm(W8.view(torch.uint8), X8.view(torch.uint8), sw, sx)
    torch.cuda.synchronize()
    Wd = W8.float().cpu().double().numpy() * float(sw.item())
    Xd = X8.float().cpu().double().numpy() * float(sx.item())
    ref = torch.from_numpy((Xd @ Wd.T).astype(np.float32)).to(torch.bfloat16).float().numpy()
    ok, ratio, rel = within_tolerance(bf16_to_np_f32(Y), ref)
    assert ok, (ratio, rel)


def test_fp8_baseline_rejects_bad_shapes(qg, cuda):
    W8 = torch.zeros((64, 40), dtype=torch.uint8, device="cuda")  # K % 16 != 0
    X8 = torch.zeros((2, 40), dtype=torch.uint8, device="cuda")
    one = torch.ones(1, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        qg.cublaslt_fp8_gemm(W8, X8, one, one)
