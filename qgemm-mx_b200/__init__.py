"""qgemm-mx B200: host-side mirror of titoatwork/qgemm-mx's W4A16 API.

Thin Python layer over the C-ABI in ``include/qgemm_b200.h`` (the shared
library ``libqgemm_b200.so`` next to this file, built for sm_100a).  Names and
error behaviour follow the reference's header-only C++ API
(include/qgemm/pack.hpp, formats.cuh): ``pack_mxfp4`` / ``pack_nvfp4`` /
``pack_int4`` return packed containers, ``dequant_*`` expand them, and
``gemm_w4a16`` computes ``Y = X . W^T``.  Where the reference throws
``std::invalid_argument`` these raise ``ValueError``.  Device memory and
streams come from PyTorch; every compute step runs in the CUDA library, and
importing this package fails if that library is missing.

The directory name contains a hyphen, so import it with
``importlib.import_module("qgemm-mx_b200")``.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqgemm_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `make -C qgemm-mx_b200/csrc` "
        "(or __graft_entry__.build()); there is no CPU fallback")

_lib = C.CDLL(LIB_PATH)

# status codes (qgemm_status_t)
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED_SHAPE, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_WORKSPACE = range(7)
# formats (qgemm_format_t), mirroring qgemm::Format
MXFP4, NVFP4, INT4_G128, INT4_G64, BF16, FP16, FP8_E4M3 = range(7)
FORMAT_NAMES = {MXFP4: "mxfp4", NVFP4: "nvfp4", INT4_G128: "int4_g128", INT4_G64: "int4_g64",
                BF16: "bf16", FP16: "fp16", FP8_E4M3: "fp8_e4m3"}

_vp, _sz, _i32, _f32, _u16p = C.c_void_p, C.c_size_t, C.c_int32, C.c_float, C.c_void_p


class _Weights(C.Structure):
    _fields_ = [("format", _i32), ("layout", _i32), ("N", _sz), ("K", _sz),
                ("data", _vp), ("scales", _vp), ("tensor_scale", _f32)]


def _sig(name, res, args):
    f = getattr(_lib, name)
    f.restype = res
    f.argtypes = args
    return f


_sig("qgemm_version", C.c_char_p, [])
_sig("qgemm_status_string", C.c_char_p, [_i32])
_sig("qgemm_last_error_message", C.c_char_p, [])
_sig("qgemm_bytes_per_weight", C.c_double, [_i32])
_sig("qgemm_weight_bytes", _sz, [_i32, _sz, _sz])
_sig("qgemm_total_bytes", _sz, [_i32, _sz, _sz, _sz])
_sig("qgemm_flops", C.c_double, [_sz, _sz, _sz])
_sig("qgemm_packed_sizes", _i32, [_i32, _sz, _sz, C.POINTER(_sz), C.POINTER(_sz)])
_sig("qgemm_pack_mxfp4", _i32, [_vp, _sz, _sz, _vp, _vp, _vp])
_sig("qgemm_pack_nvfp4", _i32, [_vp, _sz, _sz, _f32, _vp, _vp, _vp])
_sig("qgemm_pack_int4", _i32, [_vp, _sz, _sz, _i32, _vp, _vp, _vp])
_sig("qgemm_nvfp4_tensor_scale", _i32, [_vp, _sz, _vp, _vp])
_sig("qgemm_dequant", _i32, [C.POINTER(_Weights), _vp, _vp])
_sig("qgemm_codec_encode", _i32, [_i32, _vp, _vp, _sz, _vp])
_sig("qgemm_pack_codes", _i32, [_i32, _vp, _vp, _sz, _sz, _vp, _vp, _vp])
_sig("qgemm_unpack_codes", _i32, [_i32, _vp, _sz, _sz, _vp, _vp])
_sig("qgemm_layout_sizes", _i32, [_i32, _i32, _sz, _sz, C.POINTER(_sz), C.POINTER(_sz)])
_sig("qgemm_repack", _i32, [C.POINTER(_Weights), _i32, _vp, _vp, _vp])
_sig("qgemm_unpack", _i32, [C.POINTER(_Weights), _vp, _vp, _vp])
_sig("qgemm_workspace_size", _sz, [C.POINTER(_Weights), _i32])
_sig("qgemm_launch_count", _i32, [C.POINTER(_Weights), _i32, C.POINTER(_i32)])
_sig("qgemm_workspace_init", _i32, [_vp, _sz, _vp])
_sig("qgemm_gemm_w4a16", _i32, [C.POINTER(_Weights), _vp, _i32, _vp, _vp, _sz, _vp])
_sig("qgemm_gemm_w4a16_f32", _i32, [C.POINTER(_Weights), _vp, _i32, _vp, _vp, _sz, _vp])
_sig("qgemm_gemm_w4a16_noalloc", _i32, [C.POINTER(_Weights), _vp, _i32, _vp, _vp])
_sig("qgemm_grouped_workspace_size", _sz, [C.POINTER(_Weights), _i32, _i32])
_sig("qgemm_grouped_gemm_w4a16", _i32, [C.POINTER(_Weights), _i32, _vp, C.POINTER(_i32), C.POINTER(C.c_int64),
                                        _vp, _vp, _sz, _vp])
_sig("qgemm_cublas_bf16_gemm", _i32, [_vp, _vp, _i32, _sz, _sz, _vp, _vp])
_sig("qgemm_probe_launch", _i32, [_i32, _vp, _vp, _sz, _vp])
_sig("qgemm_cublaslt_fp8_gemm", _i32, [_vp, _vp, _i32, _sz, _sz, _vp, _vp, _vp, _vp, _sz, _vp])
_sig("qgemm_device_info", _i32, [C.POINTER(_i32), C.POINTER(_sz)])
_sig("qgemm_probe_status", _i32, [C.POINTER(_i32)])
_sig("qgemm_umma_status", _i32, [C.POINTER(_i32)])
_sig("qgemm_clear_faults", _i32, [])
_sig("qgemm_tp_sync_bytes", _sz, [_i32])
_sig("qgemm_tp_workspace_size", _sz, [C.POINTER(_Weights), _i32])
_sig("qgemm_tp_gemm_w4a16", _i32, [C.POINTER(_Weights), C.c_void_p, _i32, _i32, _i32, C.POINTER(C.c_void_p),
                                   C.POINTER(C.c_void_p), C.c_void_p, _sz, C.c_void_p])
_sig("qgemm_tp_status", _i32, [C.POINTER(_i32)])
_sig("qgemm_ipc_handle", _i32, [C.c_void_p, C.POINTER(C.c_uint8), C.POINTER(_sz)])
_sig("qgemm_ipc_open", _i32, [C.POINTER(C.c_uint8), C.POINTER(C.c_void_p)])
_sig("qgemm_ipc_close", _i32, [C.c_void_p])

EXPORTED = [n for n in dir(_lib) if n.startswith("qgemm_")]


class QGemmError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = _lib.qgemm_last_error_message().decode()
        super().__init__(f"{where}: {_lib.qgemm_status_string(status).decode()}: {msg}")


def _check(status: int, where: str) -> None:
    if status == OK:
        return
    if status == ERR_INVALID_ARG:
        raise ValueError(f"{where}: {_lib.qgemm_last_error_message().decode()}")
    raise QGemmError(status, where)


def lib() -> C.CDLL:
    """The loaded C-ABI library (for callers that bind symbols directly)."""
    return _lib


def version() -> str:
    return _lib.qgemm_version().decode()


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t: torch.Tensor | None):
    return C.c_void_p(0 if t is None else t.data_ptr())


# ---- byte accounting (formats.cuh) ------------------------------------------

def bytes_per_weight(fmt: int) -> float:
    return _lib.qgemm_bytes_per_weight(fmt)


def weight_bytes(fmt: int, N: int, K: int) -> int:
    return _lib.qgemm_weight_bytes(fmt, N, K)


def total_bytes(fmt: int, M: int, N: int, K: int) -> int:
    return _lib.qgemm_total_bytes(fmt, M, N, K)


def flops(M: int, N: int, K: int) -> float:
    return _lib.qgemm_flops(M, N, K)


def packed_sizes(fmt: int, N: int, K: int) -> tuple[int, int]:
    d, s = _sz(0), _sz(0)
    _check(_lib.qgemm_packed_sizes(fmt, N, K, C.byref(d), C.byref(s)), "packed_sizes")
    return d.value, s.value


# ---- packed containers (pack.hpp:396-417, device-resident) -------------------

@dataclass
class Packed:
    """A packed weight matrix on the device.  ``data`` is uint8 [N*K/2];
    ``scales`` is uint8 (MXFP4/NVFP4) or int16 holding FP16 bits (INT4)."""
    format: int
    N: int
    K: int
    data: torch.Tensor
    scales: torch.Tensor
    tensor_scale: float = 1.0
    layout: int = 0  # CANONICAL or SCALE_CHECKED (include/qgemm_b200.h)

    @property
    def group(self) -> int:
        return {MXFP4: 32, NVFP4: 16, INT4_G128: 128, INT4_G64: 64}[self.format]

    def desc(self) -> _Weights:
        return _Weights(self.format, self.layout, self.N, self.K, self.data.data_ptr(),
                        self.scales.data_ptr(), float(self.tensor_scale))

    def shard_rows(self, n0: int, n1: int) -> "Packed":
        """Rows [n0, n1) as a view: contiguous slices of data and scales, in
        the same layout (a row subset of checked scales is checked)."""
        bpr = self.K // 2
        spr = self.K // self.group
        return Packed(self.format, n1 - n0, self.K, self.data[n0 * bpr:n1 * bpr],
                      self.scales[n0 * spr:n1 * spr], self.tensor_scale, self.layout)


def _alloc_packed(fmt: int, N: int, K: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    d, s = packed_sizes(fmt, N, K)
    data = torch.empty(max(d, 16), dtype=torch.uint8, device=device)[:d]
    if fmt in (INT4_G128, INT4_G64):
        scales = torch.empty(max(s // 2, 8), dtype=torch.int16, device=device)[: s // 2]
    else:
        scales = torch.empty(max(s, 16), dtype=torch.uint8, device=device)[:s]
    return data, scales


def _as_f32_2d(W: torch.Tensor) -> torch.Tensor:
    if W.dim() != 2 or W.dtype != torch.float32 or not W.is_cuda:
        raise ValueError("W must be a 2-D float32 CUDA tensor [N, K]")
    return W.contiguous()


def pack_mxfp4(W: torch.Tensor, stream=None) -> Packed:
    """pack.hpp:465-497 on the device (bit-exact)."""
    W = _as_f32_2d(W)
    N, K = W.shape
    if K % 32:
        raise ValueError("pack_mxfp4: K must be divisible by 32")
    data, scales = _alloc_packed(MXFP4, N, K, W.device)
    _check(_lib.qgemm_pack_mxfp4(_ptr(W), N, K, _ptr(data), _ptr(scales), _stream(stream)), "pack_mxfp4")
    return Packed(MXFP4, N, K, data, scales)


def nvfp4_tensor_scale(W: torch.Tensor, stream=None) -> float:
    """max|W| / (448*6) computed on the device; returns the host float."""
    W = _as_f32_2d(W) if W.dim() == 2 else W.contiguous()
    out = torch.empty(1, dtype=torch.float32, device=W.device)
    _check(_lib.qgemm_nvfp4_tensor_scale(_ptr(W), W.numel(), _ptr(out), _stream(stream)), "nvfp4_tensor_scale")
    return float(out.item())


def pack_nvfp4(W: torch.Tensor, tensor_scale: float | None = None, stream=None) -> Packed:
    """pack.hpp:502-542 on the device (bit-exact).  tensor_scale defaults to
    max|W|/(448*6)."""
    W = _as_f32_2d(W)
    N, K = W.shape
    if tensor_scale is None:
        tensor_scale = nvfp4_tensor_scale(W, stream)
    if K % 16:
        raise ValueError("pack_nvfp4: K must be divisible by 16")
    data, scales = _alloc_packed(NVFP4, N, K, W.device)
    _check(_lib.qgemm_pack_nvfp4(_ptr(W), N, K, float(tensor_scale), _ptr(data), _ptr(scales),
                                 _stream(stream)), "pack_nvfp4")
    return Packed(NVFP4, N, K, data, scales, float(tensor_scale))


def pack_int4(W: torch.Tensor, group: int = 128, stream=None) -> Packed:
    """pack.hpp:424-462 on the device (bit-exact)."""
    W = _as_f32_2d(W)
    N, K = W.shape
    if group not in (64, 128):
        raise ValueError("pack_int4: group must be 64 or 128")
    if K % group:
        raise ValueError("pack_int4: K must be divisible by group")
    fmt = INT4_G128 if group == 128 else INT4_G64
    data, scales = _alloc_packed(fmt, N, K, W.device)
    _check(_lib.qgemm_pack_int4(_ptr(W), N, K, group, _ptr(data), _ptr(scales), _stream(stream)), "pack_int4")
    return Packed(fmt, N, K, data, scales)


def pack(fmt: int, W: torch.Tensor, stream=None) -> Packed:
    if fmt == MXFP4:
        return pack_mxfp4(W, stream)
    if fmt == NVFP4:
        return pack_nvfp4(W, None, stream)
    if fmt == INT4_G128:
        return pack_int4(W, 128, stream)
    if fmt == INT4_G64:
        return pack_int4(W, 64, stream)
    raise ValueError(f"pack: not a 4-bit format: {fmt}")


def from_host(fmt: int, N: int, K: int, data, scales, tensor_scale: float = 1.0, device="cuda") -> Packed:
    """Wrap host-packed bytes (numpy arrays in the reference layout)."""
    import numpy as np
    d = torch.from_numpy(np.ascontiguousarray(data).view(np.uint8)).to(device)
    if fmt in (INT4_G128, INT4_G64):
        s = torch.from_numpy(np.ascontiguousarray(scales).view(np.int16)).to(device)
    else:
        s = torch.from_numpy(np.ascontiguousarray(scales).view(np.uint8)).to(device)
    return Packed(fmt, N, K, d, s, float(tensor_scale))


def dequant(p: Packed, stream=None) -> torch.Tensor:
    """pack.hpp:548-585 on the device (bit-exact FP32 [N, K])."""
    out = torch.empty((p.N, p.K), dtype=torch.float32, device=p.data.device)
    d = p.desc()
    _check(_lib.qgemm_dequant(C.byref(d), _ptr(out), _stream(stream)), "dequant")
    return out


dequant_mxfp4 = dequant_nvfp4 = dequant_int4 = dequant


def pack_codes(fmt: int, codes: torch.Tensor, scales: torch.Tensor, N: int, K: int,
               tensor_scale: float = 1.0, stream=None) -> Packed:
    """Already-quantised codes to the canonical layout (pack.hpp:611-665):
    FP4 formats take uint8 E2M1 codes [N*K] and uint8 scale bytes; INT4 takes
    int32 codes in [-8, 7] (clamped) and float32 group scales."""
    int4 = fmt in (INT4_G128, INT4_G64)
    want_c, want_s = (torch.int32, torch.float32) if int4 else (torch.uint8, torch.uint8)
    if codes.dtype != want_c or scales.dtype != want_s:
        raise ValueError(f"pack_codes: codes must be {want_c}, scales {want_s}")
    codes, scales = codes.contiguous(), scales.contiguous()
    data, sc = _alloc_packed(fmt, N, K, codes.device)
    _check(_lib.qgemm_pack_codes(fmt, _ptr(codes), _ptr(scales), N, K, _ptr(data), _ptr(sc), _stream(stream)),
           "pack_codes")
    return Packed(fmt, N, K, data, sc, tensor_scale if fmt == NVFP4 else 1.0)


def unpack_codes(p: Packed, stream=None) -> torch.Tensor:
    """The packed codes back (pack.hpp:667-682): uint8 E2M1 codes, or int32
    INT4 values, [N*K]."""
    int4 = p.format in (INT4_G128, INT4_G64)
    out = torch.empty(p.N * p.K, dtype=torch.int32 if int4 else torch.uint8, device=p.data.device)
    _check(_lib.qgemm_unpack_codes(p.format, _ptr(p.data), p.N, p.K, _ptr(out), _stream(stream)), "unpack_codes")
    return out


# ---- layouts (the kernel-optimal layout as an offline transform) --------------

CANONICAL, SCALE_CHECKED = 0, 1


def layout_sizes(fmt: int, layout: int, N: int, K: int) -> tuple[int, int]:
    d, s = _sz(0), _sz(0)
    _check(_lib.qgemm_layout_sizes(fmt, layout, N, K, C.byref(d), C.byref(s)), "layout_sizes")
    return d.value, s.value


def repack(p: Packed, layout: int = SCALE_CHECKED, stream=None) -> Packed:
    """Canonical weights in `layout`.  The scale-checked layout keeps the
    bytes (shared with p, nothing is copied) once a scan of the scales finds
    none outside the decode kernel's fast range; ValueError otherwise (such
    weights stay canonical).  Waits for the stream."""
    if p.layout != CANONICAL:
        raise ValueError("repack: source must be canonical")
    d = p.desc()
    _check(_lib.qgemm_repack(C.byref(d), layout, _ptr(p.data), _ptr(p.scales), _stream(stream)), "repack")
    return Packed(p.format, p.N, p.K, p.data, p.scales, p.tensor_scale, layout)


def unpack(p: Packed, stream=None) -> Packed:
    """The canonical bytes of p (any layout), in new buffers."""
    data, sc = _alloc_packed(p.format, p.N, p.K, p.data.device)
    d = p.desc()
    _check(_lib.qgemm_unpack(C.byref(d), _ptr(data), _ptr(sc), _stream(stream)), "unpack")
    return Packed(p.format, p.N, p.K, data, sc, p.tensor_scale, CANONICAL)


def codec_encode(kind: str, x: torch.Tensor, stream=None) -> torch.Tensor:
    """Device scalar encoders (pack.hpp): 'e2m1' | 'e8m0' | 'e4m3' | 'fp16'."""
    k = {"e2m1": 0, "e8m0": 1, "e4m3": 2, "fp16": 3}[kind]
    x = x.contiguous().float()
    out = torch.empty(x.shape, dtype=torch.int16 if k == 3 else torch.uint8, device=x.device)
    _check(_lib.qgemm_codec_encode(k, _ptr(x), _ptr(out), x.numel(), _stream(stream)), "codec_encode")
    return out


# ---- GEMM ---------------------------------------------------------------------

def workspace_size(p: Packed, M: int) -> int:
    d = p.desc()
    return _lib.qgemm_workspace_size(C.byref(d), M)


KERNEL_NAMES = {0: "k_gemv", 1: "k_gemv_tma", 2: "k_umma_sk", 3: "k_umma_ts", 4: "k_umma_bs"}


def launch_count(p: Packed, M: int) -> tuple[int, str]:
    """(kernel launches one gemm_w4a16 call makes, name of its GEMM kernel)."""
    d = p.desc()
    k = _i32(0)
    n = _lib.qgemm_launch_count(C.byref(d), M, C.byref(k))
    if n < 0:
        raise QGemmError(-1, "launch_count: invalid arguments")
    return n, KERNEL_NAMES[k.value]


def make_workspace(p: Packed, M: int, stream=None) -> torch.Tensor:
    n = max(workspace_size(p, M), 256)
    ws = torch.empty(n, dtype=torch.uint8, device=p.data.device)
    _check(_lib.qgemm_workspace_init(_ptr(ws), n, _stream(stream)), "workspace_init")
    return ws


def gemm_w4a16(p: Packed, X: torch.Tensor, out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None, out_f32: bool = False, stream=None) -> torch.Tensor:
    """Y[M,N] = X[M,K] . W[N,K]^T with X bf16; Y bf16 (or fp32 if out_f32)."""
    if X.dim() != 2 or X.dtype != torch.bfloat16 or X.shape[1] != p.K:
        raise ValueError("gemm_w4a16: X must be bf16 [M, K]")
    X = X.contiguous()
    M = X.shape[0]
    if out is None:
        out = torch.empty((M, p.N), dtype=torch.float32 if out_f32 else torch.bfloat16, device=X.device)
    if workspace is None:
        workspace = make_workspace(p, M, stream)
    d = p.desc()
    fn = _lib.qgemm_gemm_w4a16_f32 if out.dtype == torch.float32 else _lib.qgemm_gemm_w4a16
    _check(fn(C.byref(d), _ptr(X), M, _ptr(out), _ptr(workspace), workspace.numel(), _stream(stream)),
           "gemm_w4a16")
    return out


# ---- grouped GEMM (mixture of experts) ------------------------------------------

def _expert_descs(experts: list[Packed]):
    return (_Weights * len(experts))(*[p.desc() for p in experts])


def grouped_workspace_size(experts: list[Packed], max_m: int) -> int:
    """Workspace bytes for grouped_gemm_w4a16 calls whose experts have <= max_m rows."""
    if not experts:
        return 0
    return _lib.qgemm_grouped_workspace_size(_expert_descs(experts), len(experts), max_m)


def make_grouped_workspace(experts: list[Packed], max_m: int, stream=None) -> torch.Tensor:
    n = max(grouped_workspace_size(experts, max_m), 256)
    ws = torch.empty(n, dtype=torch.uint8, device=experts[0].data.device)
    _check(_lib.qgemm_workspace_init(_ptr(ws), n, _stream(stream)), "workspace_init")
    return ws


def grouped_gemm_w4a16(experts: list[Packed], X: torch.Tensor, counts, offsets=None,
                       out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                       stream=None) -> torch.Tensor:
    """Mixture-of-experts GEMM: rows offsets[e] .. offsets[e] + counts[e] of X
    (bf16 [rows, K]) go through expert e; Y holds the same rows (bf16 [rows, N]).
    offsets defaults to the exclusive prefix sum of counts (rows sorted by
    expert).  Rows no expert covers are left as they are in ``out``."""
    E = len(experts)
    counts = [int(c) for c in counts]
    if len(counts) != E:
        raise ValueError("grouped_gemm_w4a16: one count per expert")
    if offsets is None:
        offsets, acc = [], 0
        for c in counts:
            offsets.append(acc)
            acc += c
    offsets = [int(o) for o in offsets]
    if X.dim() != 2 or X.dtype != torch.bfloat16 or (E and X.shape[1] != experts[0].K):
        raise ValueError("grouped_gemm_w4a16: X must be bf16 [rows, K]")
    for c, o in zip(counts, offsets):
        if c > 0 and o + c > X.shape[0]:
            raise ValueError("grouped_gemm_w4a16: expert rows beyond X")
    X = X.contiguous()
    if out is None:
        out = torch.zeros((X.shape[0], experts[0].N if E else 0), dtype=torch.bfloat16, device=X.device)
    if E == 0:
        return out
    if workspace is None:
        workspace = make_grouped_workspace(experts, max(max(counts), 1), stream)
    Ms = (_i32 * E)(*counts)
    Os = (C.c_int64 * E)(*offsets)
    _check(_lib.qgemm_grouped_gemm_w4a16(_expert_descs(experts), E, _ptr(X), Ms, Os, _ptr(out), _ptr(workspace),
                                         workspace.numel(), _stream(stream)), "grouped_gemm_w4a16")
    return out


def cublas_bf16_gemm(W: torch.Tensor, X: torch.Tensor, out: torch.Tensor | None = None, stream=None):
    """Dense cuBLAS BF16 baseline of the same shape (bench_cublas.cu:144-151)."""
    N, K = W.shape
    M = X.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=X.device)
    _check(_lib.qgemm_cublas_bf16_gemm(_ptr(W), _ptr(X), M, N, K, _ptr(out), _stream(stream)), "cublas")
    return out


def cublaslt_fp8_gemm(W8: torch.Tensor, X8: torch.Tensor, scale_w: torch.Tensor, scale_x: torch.Tensor,
                      out: torch.Tensor | None = None, workspace: torch.Tensor | None = None, stream=None):
    """cuBLASLt FP8 dense baseline: Y[M,N] bf16 = (X8.scale_x) . (W8.scale_w)^T.
    W8 [N,K] / X8 [M,K] hold E4M3 bytes (uint8 or float8_e4m3fn); scale_w and
    scale_x are one-element float32 CUDA tensors."""
    N, K = W8.shape
    M = X8.shape[0]
    if X8.shape[1] != K or scale_w.dtype != torch.float32 or scale_x.dtype != torch.float32:
        raise ValueError("cublaslt_fp8_gemm: W8 [N,K], X8 [M,K], float32 scales")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=X8.device)
    nws = 0 if workspace is None else workspace.numel()
    _check(_lib.qgemm_cublaslt_fp8_gemm(_ptr(W8), _ptr(X8), M, N, K, _ptr(scale_w), _ptr(scale_x), _ptr(out),
                                        _ptr(workspace), nws, _stream(stream)), "cublaslt_fp8_gemm")
    return out


def probe_launch(kind: int, src: torch.Tensor | None, dst: torch.Tensor | None, nbytes: int, stream=None):
    _check(_lib.qgemm_probe_launch(kind, _ptr(src), _ptr(dst), nbytes, _stream(stream)), "probe")


def probe_status() -> None:
    """Raises QGemmError if a bounded wait inside a TMA bulk probe gave up."""
    f = _i32(0)
    _check(_lib.qgemm_probe_status(C.byref(f)), "probe_status")


def umma_status() -> None:
    """Raises QGemmError if a bounded wait inside the tcgen05 kernel gave up."""
    f = _i32(0)
    _check(_lib.qgemm_umma_status(C.byref(f)), "umma_status")


def clear_faults() -> None:
    """Waits for the device and resets its fault flags (after a reported
    timeout; tp sync blocks must be zeroed again first)."""
    _check(_lib.qgemm_clear_faults(), "clear_faults")


# ---- tensor parallel (W sharded along N over the GPUs of one node) ------------

def tp_sync_bytes(world: int) -> int:
    return _lib.qgemm_tp_sync_bytes(world)


def make_tp_workspace(p: Packed, M: int, stream=None) -> torch.Tensor:
    """Zeroed workspace for tp_gemm of this rank's shard p."""
    d = p.desc()
    n = max(_lib.qgemm_tp_workspace_size(C.byref(d), M), 256)
    ws = torch.empty(n, dtype=torch.uint8, device=p.data.device)
    _check(_lib.qgemm_workspace_init(_ptr(ws), n, _stream(stream)), "workspace_init")
    return ws


def tp_gemm(p: Packed, X: torch.Tensor, world: int, rank: int, y_peers: list[int], sync_peers: list[int],
            workspace: torch.Tensor, stream=None) -> None:
    """This rank's slice of Y = X . W^T written into every rank's Y_full
    (y_peers[d]: rank d's Y_full [M][N] as mapped here, device addresses),
    then a bounded wait until all ranks' slices are in this rank's Y_full."""
    if X.dtype != torch.bfloat16 or not X.is_contiguous():
        raise ValueError("X must be contiguous bf16")
    d = p.desc()
    yp = (C.c_void_p * world)(*y_peers)
    sp = (C.c_void_p * world)(*sync_peers)
    _check(_lib.qgemm_tp_gemm_w4a16(C.byref(d), _ptr(X), X.shape[0], world, rank, yp, sp, _ptr(workspace),
                                    workspace.numel(), _stream(stream)), "tp_gemm")


def tp_status() -> None:
    """Raises QGemmError if a tp wait gave up (a peer never announced)."""
    f = _i32(0)
    _check(_lib.qgemm_tp_status(C.byref(f)), "tp_status")


def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding t, t's byte offset in it)."""
    h = (C.c_uint8 * 64)()
    off = _sz(0)
    _check(_lib.qgemm_ipc_handle(_ptr(t), h, C.byref(off)), "ipc_handle")
    return bytes(h), off.value


def ipc_open(handle: bytes, offset: int) -> tuple[int, int]:
    """Maps another process's allocation; returns (base to close later, address of the shared pointer)."""
    h = (C.c_uint8 * 64)(*handle)
    ptr = C.c_void_p(0)
    _check(_lib.qgemm_ipc_open(h, C.byref(ptr)), "ipc_open")
    return ptr.value, ptr.value + offset


def ipc_close(base: int) -> None:
    _check(_lib.qgemm_ipc_close(C.c_void_p(base)), "ipc_close")


def device_info() -> tuple[int, int]:
    sm, l2 = _i32(0), _sz(0)
    _check(_lib.qgemm_device_info(C.byref(sm), C.byref(l2)), "device_info")
    return sm.value, l2.value
