"""ctypes loader for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/liboracle.so`` (the C restatement of the reference's host
numerics, titoatwork/qgemm-mx include/qgemm/pack.hpp and ref_gemm.hpp) and,
when it was built, ``oracle/_ref/libqgemm_ref.so`` (the reference's own
headers compiled through ``oracle/ref_shim.cpp``).  Only tests/, the smoke
check in __graft_entry__.py and bench.py's CPU-baseline leg import this
module; the CUDA product path never does.

Both libraries expose the same functions under the prefixes ``or_`` (oracle)
and ``ref_`` (reference); :class:`CpuPath` wraps either behind one numpy API.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqgemm_ref.so")

FMT_MXFP4, FMT_NVFP4, FMT_INT4 = 0, 1, 2
_p = C.c_void_p
_sz = C.c_size_t


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (builds liboracle.so and, if the reference tree is
    present on this machine, _ref/libqgemm_ref.so)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_p)


class CpuPath:
    """One of the two CPU implementations: prefix 'or' (oracle) or 'ref'."""

    def __init__(self, path: str, prefix: str):
        self.lib = C.CDLL(path)
        self.prefix = prefix
        L = self.lib
        f = lambda name: getattr(L, f"{prefix}_{name}")  # noqa: E731
        self._f = f
        for name, res, args in [
            ("fp16_bits_to_float", C.c_float, [C.c_uint16]),
            ("float_to_fp16_bits", C.c_uint16, [C.c_float]),
            ("e2m1_decode", C.c_float, [C.c_uint8]),
            ("e2m1_encode", C.c_uint8, [C.c_float]),
            ("e8m0_decode", C.c_float, [C.c_uint8]),
            ("e8m0_encode", C.c_uint8, [C.c_float]),
            ("e4m3_decode", C.c_float, [C.c_uint8]),
            ("e4m3_encode", C.c_uint8, [C.c_float]),
            ("int4_from_nibble", C.c_int, [C.c_uint8]),
            ("int4_to_nibble", C.c_uint8, [C.c_int]),
            ("e2m1_encode_n", None, [_p, _p, _sz]),
            ("e8m0_encode_n", None, [_p, _p, _sz]),
            ("e4m3_encode_n", None, [_p, _p, _sz]),
            ("fp16_encode_n", None, [_p, _p, _sz]),
            ("pack_int4", C.c_int, [_p, _sz, _sz, C.c_int, _p, _p]),
            ("pack_mxfp4", C.c_int, [_p, _sz, _sz, _p, _p]),
            ("pack_nvfp4", C.c_int, [_p, _sz, _sz, C.c_float, _p, _p]),
            ("dequant_int4", None, [_p, _p, _sz, _sz, C.c_int, _p]),
            ("dequant_mxfp4", None, [_p, _p, _sz, _sz, _p]),
            ("dequant_nvfp4", None, [_p, _p, _sz, _sz, C.c_float, _p]),
            ("w4a16_gemm", C.c_int, [C.c_int, _p, _p, _sz, _sz, C.c_int, C.c_float,
                                     _p, _sz, _p, _sz, _sz, C.c_int]),
        ]:
            fn = f(name)
            fn.restype = res
            fn.argtypes = args
        gemm = getattr(L, "or_gemm_ref" if prefix == "or" else "ref_gemm_fp32")
        gemm.restype = None
        gemm.argtypes = [_p, _p, _p, _sz, _sz, _sz]
        self._gemm = gemm

    # -- scalar / batch codecs ------------------------------------------------
    def __getattr__(self, name):
        return self._f(name)

    def encode_n(self, kind: str, v: np.ndarray) -> np.ndarray:
        v = np.ascontiguousarray(v, dtype=np.float32)
        dt = np.uint16 if kind == "fp16" else np.uint8
        out = np.empty(v.shape, dtype=dt)
        self._f(f"{kind}_encode_n")(_ptr(v), _ptr(out), v.size)
        return out

    # -- packers ----------------------------------------------------------------
    def pack(self, fmt: str, W: np.ndarray, group: int = 128, tensor_scale: float = 1.0):
        """Returns (status, data, scales) with the reference's byte layout."""
        W = np.ascontiguousarray(W, dtype=np.float32)
        N, K = W.shape
        data = np.zeros(N * K // 2, dtype=np.uint8)
        if fmt == "mxfp4":
            sc = np.zeros(N * (K // 32) if K % 32 == 0 else 1, dtype=np.uint8)
            st = self._f("pack_mxfp4")(_ptr(W), N, K, _ptr(data), _ptr(sc))
        elif fmt == "nvfp4":
            sc = np.zeros(N * (K // 16) if K % 16 == 0 else 1, dtype=np.uint8)
            st = self._f("pack_nvfp4")(_ptr(W), N, K, C.c_float(tensor_scale), _ptr(data), _ptr(sc))
        elif fmt == "int4":
            ok = group > 0 and K % group == 0
            sc = np.zeros(N * (K // group) if ok else 1, dtype=np.uint16)
            st = self._f("pack_int4")(_ptr(W), N, K, group, _ptr(data), _ptr(sc))
        else:
            raise ValueError(fmt)
        return st, data, sc

    def dequant(self, fmt: str, data, scales, N, K, group=128, tensor_scale=1.0):
        out = np.empty((N, K), dtype=np.float32)
        if fmt == "mxfp4":
            self._f("dequant_mxfp4")(_ptr(data), _ptr(scales), N, K, _ptr(out))
        elif fmt == "nvfp4":
            self._f("dequant_nvfp4")(_ptr(data), _ptr(scales), N, K, C.c_float(tensor_scale), _ptr(out))
        else:
            self._f("dequant_int4")(_ptr(data), _ptr(scales), N, K, group, _ptr(out))
        return out

    def gemm_ref(self, X: np.ndarray, W: np.ndarray) -> np.ndarray:
        X = np.ascontiguousarray(X, dtype=np.float32)
        W = np.ascontiguousarray(W, dtype=np.float32)
        M, K = X.shape
        N = W.shape[0]
        Y = np.empty((M, N), dtype=np.float32)
        self._gemm(_ptr(X), _ptr(W), _ptr(Y), M, N, K)
        return Y

    def w4a16_gemm(self, fmt: str, data, scales, N, K, X_bf16: np.ndarray, group=128,
                   tensor_scale=1.0, n_begin=0, n_end=None, nthreads=1, Y=None):
        """dequant + reference GEMM, X given as bf16 bits (uint16 [M,K])."""
        f = {"mxfp4": FMT_MXFP4, "nvfp4": FMT_NVFP4, "int4": FMT_INT4}[fmt]
        X_bf16 = np.ascontiguousarray(X_bf16, dtype=np.uint16)
        M = X_bf16.shape[0]
        if Y is None:
            Y = np.zeros((M, N), dtype=np.float32)
        n_end = N if n_end is None else n_end
        st = self._f("w4a16_gemm")(f, _ptr(data), _ptr(scales), N, K, group,
                                   C.c_float(tensor_scale), _ptr(X_bf16), M, _ptr(Y),
                                   n_begin, n_end, nthreads)
        if st != 0:
            raise ValueError("w4a16_gemm: invalid arguments")
        return Y


_ORACLE = None
_REF = None


def oracle() -> CpuPath:
    global _ORACLE
    if _ORACLE is None:
        if not os.path.exists(ORACLE_SO):
            build()
        _ORACLE = CpuPath(ORACLE_SO, "or")
        o = _ORACLE.lib
        o.or_randn.restype = None
        o.or_randn.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_float, _p, _sz]
        o.or_randn_bf16.restype = None
        o.or_randn_bf16.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_float, _p, _sz]
        o.or_nvfp4_tensor_scale.restype = C.c_float
        o.or_nvfp4_tensor_scale.argtypes = [_p, _sz]
        o.or_f32_to_bf16_bits.restype = C.c_uint16
        o.or_f32_to_bf16_bits.argtypes = [C.c_float]
    return _ORACLE


def reference() -> CpuPath | None:
    """The reference's own code, or None where it was never built."""
    global _REF
    if _REF is None and os.path.exists(REF_SO):
        _REF = CpuPath(REF_SO, "ref")
        r = _REF.lib
        for nm in ("ref_weight_bytes",):
            getattr(r, nm).restype = _sz
            getattr(r, nm).argtypes = [C.c_int, _sz, _sz]
        r.ref_total_bytes.restype = _sz
        r.ref_total_bytes.argtypes = [C.c_int, _sz, _sz, _sz]
    return _REF


# -- seeded inputs (the build's documented generator) --------------------------

def randn(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    oracle().lib.or_randn(seed, stream, mean, std, _ptr(out), n)
    return out


def randn_bf16(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    oracle().lib.or_randn_bf16(seed, stream, mean, std, _ptr(out), n)
    return out


def nvfp4_tensor_scale(W: np.ndarray) -> float:
    W = np.ascontiguousarray(W, dtype=np.float32)
    return float(oracle().lib.or_nvfp4_tensor_scale(_ptr(W), W.size))


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r
