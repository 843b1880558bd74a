"""The library driven from C++ through the reference's own harness.

oracle/_ref/time_graphed_w4a16 (tests/cpp/time_graphed_w4a16.cu, built by
tests/cpp/Makefile from the reference's include/ tree) quantises W with the
reference's host packers (pack.hpp:424-542), calls qgemm_gemm_w4a16 inside
the reference's time_graphed / time_looped lambda protocol
(timing.cuh:250-336, as bench_cublas.cu:144-158 drives cuBLAS) and checks
the result with the reference's gemm_fp32_ref on dequant_reference_* rows
and compare_close (correctness.hpp:317-346) under the W4A16 contract's row
bound and the 1e-3 relative Frobenius bound.  The cases are the benchmarked
configurations: the 70B MXFP4 layers on each kernel, config 2 (NVFP4 and
INT4 14336 x 4096), NVFP4 prefill at M = 2048 and an unaligned 2880 shape.
"""
import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "time_graphed_w4a16")

CASES = [  # format, N, K, M, checked weight rows
    ("mxfp4", 10240, 8192, 1, 256),      # QKV, TMA decode
    ("mxfp4", 57344, 8192, 64, 128),     # gate-up, block-scaled tcgen05 + fixup
    ("mxfp4", 8192, 28672, 32, 128),     # down, block-scaled tcgen05
    ("nvfp4", 14336, 4096, 16, 256),     # config 2, TMA decode (two n-tiles)
    ("int4_g128", 14336, 4096, 8, 256),  # config 2 INT4, TMA decode
    ("nvfp4", 28672, 8192, 2048, 16),    # prefill, tile-per-CTA tcgen05
    ("mxfp4", 2880, 2880, 7, 256),       # unaligned K (gpt_oss_2880)
]


def test_driver_is_built():
    assert os.path.exists(BIN), "tests/cpp/Makefile output missing (build() makes it from the reference headers)"


@pytest.mark.parametrize("fmt,N,K,M,rows", CASES)
def test_reference_harness_drives_the_library(cuda, fmt, N, K, M, rows):
    r = subprocess.run([BIN, fmt, str(N), str(K), str(M), str(rows)], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["ok"] and not d["wait_timed_out"], d
    assert d["cold_us"] > 0 and d["hot_us"] > 0 and d["looped_us"] >= d["cold_us"] * 0.5, d
