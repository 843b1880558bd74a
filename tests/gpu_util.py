"""Helpers for the GPU parity tests: upload oracle inputs, pull results back,
and the tolerance of the W4A16 contract.

Tolerance (stated by the path's specification): against the reference GEMM
(double accumulation, ref_gemm.hpp:15-27) every output row m must satisfy
max_n |Y - Y_ref| <= 1e-2 * max_n |Y_ref[m, :]|, and the whole result
||Y - Y_ref||_F <= 1e-3 * ||Y_ref||_F.  For bf16 output the reference value
is rounded to bf16 the same way ("stored bf16").
"""
import numpy as np
import torch

ROW_TOL = 1e-2
FROB_TOL = 1e-3


def to_dev_f32(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def to_dev_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def bf16_to_np_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def u8(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint8)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def same_bits(a, b) -> bool:
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return bool(np.array_equal(nan, np.isnan(b)) and
                np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32)))


def within_tolerance(Y: np.ndarray, Yref: np.ndarray, row_tol=ROW_TOL, frob_tol=FROB_TOL):
    """Returns (ok, worst_row_ratio, rel_frobenius)."""
    Y = np.asarray(Y, np.float64)
    R = np.asarray(Yref, np.float64)
    rowmax = np.abs(R).max(axis=1, keepdims=True)
    err = np.abs(Y - R)
    ratio = float((err / np.maximum(rowmax, 1e-30)).max())
    rel = float(np.linalg.norm(Y - R) / max(np.linalg.norm(R), 1e-30))
    return (ratio <= row_tol and rel <= frob_tol), ratio, rel
