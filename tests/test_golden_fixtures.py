"""The oracle reproduces the committed golden fixtures, which were produced by
the reference's own code (tests/golden/make_golden.py).  These run without the
reference tree, so they pin the oracle on any machine."""
import hashlib
import os

import numpy as np
import pytest

from edge_cases import edge_matrix

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FORMATS = [("mxfp4", 32), ("nvfp4", 16), ("int4", 128), ("int4", 64)]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("name", ["seeded_64x256", "edge_8x256"])
def test_small_fixtures(O, orc, name):
    f = np.load(os.path.join(GOLD, name + ".npz"))
    N, K, seed = int(f["N"]), int(f["K"]), int(f["seed"])
    W = (O.randn(0, 1, N * K, 0.0, 0.02).reshape(N, K) if name.startswith("seeded") else edge_matrix(N, K))
    for fmt, group in FORMATS:
        tag = f"{fmt}{group}"
        ts = float(f[f"{tag}_ts"])
        st, d, s = orc.pack(fmt, W, group=group, tensor_scale=ts)
        assert st == 0
        assert np.array_equal(d, f[f"{tag}_data"]), tag
        assert np.array_equal(s, f[f"{tag}_scales"]), tag
        assert same_bits(orc.dequant(fmt, d, s, N, K, group=group, tensor_scale=ts), f[f"{tag}_dequant"])
        for M in f["ms"]:
            X = O.randn_bf16(seed, 2, int(M) * K).reshape(int(M), K)
            Y = orc.w4a16_gemm(fmt, d, s, N, K, X, group=group, tensor_scale=ts, nthreads=4)
            assert same_bits(Y, f[f"{tag}_Y_M{M}"]), (tag, M)


def test_config1_fixture(O, orc):
    """MXFP4 M=1 N=K=4096, seed 0: packed bytes (by digest) and Y."""
    f = np.load(os.path.join(GOLD, "config1_mxfp4_4096.npz"))
    N, K = int(f["N"]), int(f["K"])
    W = O.randn(0, 1, N * K, 0.0, 0.02).reshape(N, K)
    assert sha(W) == str(f["W_sha"])
    st, d, s = orc.pack("mxfp4", W)
    assert sha(d) == str(f["data_sha"]) and sha(s) == str(f["scales_sha"])
    X = O.randn_bf16(0, 2, K).reshape(1, K)
    assert sha(X) == str(f["X_sha"])
    Y = orc.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=8)
    assert same_bits(Y, f["Y"])
