"""Generate the committed golden fixtures from the reference's own code.

Run where the reference tree is available (it builds oracle/_ref from the
reference headers through oracle/Makefile):

    python tests/golden/make_golden.py

Inputs come from the build's documented generator (oracle/qgemm_oracle.c:
splitmix64-seeded xoshiro256** + Box-Muller): W ~ N(0, 0.02) fp32 on stream 1,
X ~ N(0, 1) rounded to bf16 on stream 2, seed as named per fixture.  Every
output (packed bytes, scales, dequantised values, Y) is produced by the
reference's pack_* / dequant_* / gemm_fp32_ref (titoatwork/qgemm-mx
include/qgemm/pack.hpp, ref_gemm.hpp).  Large packed buffers are stored as a
SHA-256 digest.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle as O  # noqa: E402
from edge_cases import edge_matrix  # noqa: E402

FORMATS = [("mxfp4", 32), ("nvfp4", 16), ("int4", 128), ("int4", 64)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def small_case(ref, name, W, ms, seed):
    N, K = W.shape
    out = {}
    for fmt, group in FORMATS:
        ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
        if not (np.isfinite(ts) and ts > 0):  # the edge matrix holds +-inf
            ts = 1.0
        st, d, s = ref.pack(fmt, W, group=group, tensor_scale=ts)
        assert st == 0
        tag = f"{fmt}{group}"
        out[f"{tag}_data"] = d
        out[f"{tag}_scales"] = s
        out[f"{tag}_ts"] = np.float32(ts)
        out[f"{tag}_dequant"] = ref.dequant(fmt, d, s, N, K, group=group, tensor_scale=ts)
        for M in ms:
            X = O.randn_bf16(seed, 2, M * K).reshape(M, K)
            out[f"{tag}_Y_M{M}"] = ref.w4a16_gemm(fmt, d, s, N, K, X, group=group,
                                                  tensor_scale=ts, nthreads=8)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), N=N, K=K, seed=seed,
                        ms=np.array(ms), **out)


def config1(ref):
    """MXFP4, M=1, N=K=4096, W ~ N(0,0.02), X ~ N(0,1) bf16, seed 0."""
    N = K = 4096
    W = O.randn(0, 1, N * K, 0.0, 0.02).reshape(N, K)
    st, d, s = ref.pack("mxfp4", W)
    assert st == 0
    X = O.randn_bf16(0, 2, K).reshape(1, K)
    Y = ref.w4a16_gemm("mxfp4", d, s, N, K, X, nthreads=8)
    np.savez_compressed(os.path.join(HERE, "config1_mxfp4_4096.npz"), N=N, K=K, seed=0,
                        W_sha=sha(W), X_sha=sha(X), data_sha=sha(d), scales_sha=sha(s),
                        scales_head=s[:4096], Y=Y)


def main():
    O.build()
    ref = O.reference()
    if ref is None:
        raise SystemExit("reference build (oracle/_ref) not available")
    W = O.randn(0, 1, 64 * 256, 0.0, 0.02).reshape(64, 256)
    small_case(ref, "seeded_64x256", W, [1, 5, 16], seed=0)
    small_case(ref, "edge_8x256", edge_matrix(8, 256), [1, 3], seed=4)
    config1(ref)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
