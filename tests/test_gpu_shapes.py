"""Shapes whose K is not a multiple of 128, or whose N leaves a partial
tile, against the oracle through the C-ABI.

The reference lists them as layer archetypes (include/qgemm/shapes.hpp:27-34):
gpt_oss_2880 (N = K = 2880, "not 128-aligned -- live bug class") and kv_gqa
(N = 1024, K = 4096, "small N -- tails / occupancy"); its packer tests use
K = 96 as the awkward shape (tests/test_pack_roundtrip.cpp:291-305).  K only
has to be a multiple of the format's block (32 for MXFP4, 16 for NVFP4, 64
for INT4 g64).  The last 128-k chunk of the decode kernel then holds part of
a chunk (K % 128 = 16 .. 112), M >= 32 with K % 64 == 0 goes to
the tcgen05 kernels, and every output is compared (tolerance of
tests/gpu_util.py: per row max-abs <= 1e-2 ||row||_inf, relative Frobenius
<= 1e-3; FP32 output also within 1e-5 relative Frobenius)."""
import pytest

from gpu_util import bf16_to_np_f32, to_dev_bf16, within_tolerance
from test_gpu_gemm import packed_pair

pytestmark = pytest.mark.gpu

CASES = [
    ("mxfp4", 32, 2880, 2880, [1, 7, 16, 17, 33, 100]),   # gpt_oss_2880: K % 128 = 64
    ("nvfp4", 16, 2880, 2880, [1, 9, 33]),
    ("int4", 64, 2880, 2880, [1, 16, 20]),
    ("mxfp4", 32, 200, 96, [1, 5, 17, 40]),               # K = 96: one chunk of three blocks
    ("nvfp4", 16, 200, 96, [1, 5, 40]),
    ("mxfp4", 32, 300, 160, [3, 12]),                     # K % 128 = 32
    ("mxfp4", 32, 300, 224, [3, 12]),                     # K % 128 = 96
    ("nvfp4", 16, 300, 160, [2]),
    ("nvfp4", 16, 200, 48, [1, 5, 40]),                   # K % 32 = 16: rows on 8-byte boundaries
    ("nvfp4", 16, 200, 112, [1, 9, 33]),                  # last lane holds one 16-block
    ("nvfp4", 16, 300, 2896, [1, 16, 40]),                # K % 128 = 80
    ("int4", 64, 300, 192, [4, 18]),                      # one 64-group in the last chunk
    ("mxfp4", 32, 1024, 4096, [1, 16, 64]),               # kv_gqa
]


@pytest.mark.parametrize("fmt,group,N,K,ms", CASES)
def test_layer_shape_all_outputs(qg, cuda, O, orc, fmt, group, N, K, ms):
    p, d, s, ts = packed_pair(qg, O, orc, fmt, group, N, K, seed=N + K)
    for M in ms:
        X = O.randn_bf16(M + K, 2, M * K).reshape(M, K)
        Yref = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=8)
        Xd = to_dev_bf16(X)
        Y = qg.gemm_w4a16(p, Xd, out_f32=True).cpu().numpy()
        ok, ratio, rel = within_tolerance(Y, Yref)
        # INT4 from M = 17 runs the tcgen05 path, which rounds q x scale to f16
        assert ok and rel < (1e-3 if fmt == "int4" and M >= 17 else 1e-5), (M, ratio, rel)
        Yb = bf16_to_np_f32(qg.gemm_w4a16(p, Xd, out_f32=False))
        ok, ratio, rel = within_tolerance(Yb, O.bf16_bits_to_f32(O.f32_to_bf16_bits(Yref)).reshape(M, N))
        assert ok, (M, ratio, rel)


def test_layer_shape_launch_choice(qg):
    """The decode kernel takes the unaligned K at small M; the tcgen05
    kernels take M >= 32 when K % 64 == 0."""
    import ctypes as C
    import torch
    lib, kern = qg.lib(), C.c_int(0)
    for fmt, K, M, name in [(qg.MXFP4, 2880, 1, "k_gemv"), (qg.MXFP4, 2880, 16, "k_gemv"),
                            (qg.MXFP4, 2880, 33, "k_umma_ts"), (qg.MXFP4, 96, 40, "k_gemv"),
                            (qg.INT4_G64, 2880, 16, "k_gemv"), (qg.INT4_G64, 2880, 20, "k_umma_ts")]:
        data = torch.empty(16, dtype=torch.uint8, device="cuda")
        w = qg._Weights(fmt, 0, 2880, K, C.c_void_p(data.data_ptr()), C.c_void_p(data.data_ptr()), 1.0)
        assert lib.qgemm_launch_count(C.byref(w), M, C.byref(kern)) > 0
        assert qg.KERNEL_NAMES.get(kern.value) == name, (K, M, qg.KERNEL_NAMES.get(kern.value))
