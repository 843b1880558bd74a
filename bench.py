"""W4A16 GEMM benchmark on B200: achieved HBM GB/s of the decode path.

Workload (default "llama70b_mxfp4"): the 70B-class decoder layer set with
MXFP4 weights, (N, K) in {(10240, 8192) QKV, (57344, 8192) gate-up,
(8192, 28672) down}, M in {1, 8, 32, 64}, X ~ N(0,1) bf16, W ~ N(0,0.02)
packed on the device.  One step = the 12 GEMMs, ordered M-major so that each
call is L2-cold: between two uses of any layer at least 170 MB of other
weights stream through the 126 MB L2, and the step's working set (419 MB of
packed weights) exceeds L2.  With --gpus N each rank owns N/world contiguous
rows of every W (and its scales), and qgemm_tp_gemm_w4a16 computes its Y
slice and writes it into every rank's full Y over NVLink peer memory (CUDA
IPC mappings), then waits for the other slices; the step time is the max
over ranks (NCCL carries only barriers and the max reduction).

  value   Sum_calls total_bytes(MXFP4, M, N/world, K) over all ranks / step
          time (formats.cuh:80-83 accounting), device-resident inputs, each
          step one CUDA-graph replay (the reference's time_graphed protocol).
  e2e     the same bytes / time of the same step through the C-ABI with host
          buffers: every step copies its distinct activations in from pinned
          host memory and reads every Y back to pinned host memory.
  roofline  for the GEMM kernel with the largest share of the step
          (qgemm_launch_count names it per call): its algorithmic bytes per
          launch / its mean launch time, measured per (layer, M) with CUDA
          events over graph replays of weight-rotated launches (L2-cold),
          against the measured HBM peak; "kernels" lists every GEMM kernel's
          figures; traffic is the ncu DRAM bytes per launch recorded in
          profiles/dram_traffic.json for the same shapes.

--impl reference times the reference's own CPU path (dequant_* +
gemm_fp32_ref, threaded over rows; oracle/_ref, else the oracle port) on a
bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (format name, [(layer, N, K)], [M])
    "llama70b_mxfp4": ("mxfp4", [("qkv", 10240, 8192), ("gate_up", 57344, 8192), ("down", 8192, 28672)],
                       [1, 8, 32, 64]),
    "decode_14336x4096": ("nvfp4", [("gate_up", 14336, 4096)], [1, 4, 8, 16]),
    "decode_14336x4096_int4": ("int4", [("gate_up", 14336, 4096)], [1, 4, 8, 16]),
    "llama8b_mxfp4": ("mxfp4", [("qkv", 6144, 4096), ("o_proj", 4096, 4096), ("gate_up", 28672, 4096),
                                ("down", 4096, 14336)], [1, 2, 4, 8, 16, 32, 64, 128, 256]),
}
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama70b_mxfp4", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cublas", action="store_true", help="skip the cuBLAS BF16 column of the per-call table")
    ap.add_argument("--table", action="store_true", help="print the per-(layer, M) table to stderr")
    ap.add_argument("--fp8", action="store_true",
                    help="also time the cuBLASLt FP8 dense baseline on the same calls (1 GPU)")
    ap.add_argument("--prefill", action="store_true",
                    help="compute-bound table: NVFP4 (28672,8192) and (8192,28672), M in {2048,4096,8192}, "
                         "tcgen05 path vs cuBLAS BF16 of the same shape")
    ap.add_argument("--layout", default="checked", choices=["canonical", "checked"],
                    help="MXFP4 / NVFP4 weights as the reference's bytes, or the same bytes in the "
                         "scale-checked layout (qgemm_repack; every kernel reads it)")
    ap.add_argument("--moe", default=None, choices=sorted(MOE_STEPS),
                    help="mixture-of-experts decode step: one grouped call vs one call per active expert")
    ap.add_argument("--case", default=None,
                    help="fmt,N,K,M: run only that GEMM --steps times (for profilers), print its mean time")
    return ap.parse_args()


def run_case(args):
    """One GEMM configuration launched --warmup + --steps times (eager, one
    weight buffer); used for ncu captures of a single kernel."""
    import ctypes as C
    import torch
    qg = importlib.import_module("qgemm-mx_b200")
    fmt, N, K, M = args.case.split(",")
    N, K, M = int(N), int(K), int(M)
    fcode = {"mxfp4": qg.MXFP4, "nvfp4": qg.NVFP4, "int4": qg.INT4_G128, "int4g64": qg.INT4_G64}[fmt]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1)
    W = torch.randn((N, K), generator=gen, device="cuda").mul_(0.02)
    p = qg.pack(fcode, W)
    del W
    if args.layout == "checked" and fcode in (qg.MXFP4, qg.NVFP4):
        p = qg.repack(p)
    X = torch.randn((M, K), generator=gen, device="cuda").to(torch.bfloat16)
    Y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    ws = qg.make_workspace(p, M)
    for _ in range(args.warmup):
        qg.gemm_w4a16(p, X, out=Y, workspace=ws)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        qg.gemm_w4a16(p, X, out=Y, workspace=ws)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / args.steps
    nb = qg.total_bytes(fcode, M, N, K)
    f = C.c_int32(0)
    st = qg.lib().qgemm_umma_status(C.byref(f))  # nonzero: a bounded wait gave up (times and outputs invalid)
    line = {"case": args.case, "us_per_call": round(us, 3), "gbs": round(nb / us / 1e3, 1),
            "wait_timed_out": bool(f.value)}
    if st != qg.OK:
        line["status"] = qg.lib().qgemm_last_error_message().decode()
    print(json.dumps(line))


# Mixture-of-experts decode steps (expert gate-up projections, MXFP4):
# (experts, N, K, experts per token, tokens).  Shapes of DeepSeek-V3-class
# (256 experts, 2 x 2048 x 7168) and Mixtral-8x7B-class (8 experts,
# 2 x 14336 x 4096) models; random weights, seeded skewed routing.
MOE_STEPS = {
    "deepseek_v3_gate_up": (256, 4096, 7168, 8, 32),
    "mixtral_gate_up": (8, 28672, 4096, 2, 16),
}


def moe_routing(E, topk, tokens, seed=0):
    """Per-expert row counts of one step: every token picks topk distinct
    experts with probability proportional to 1 / (rank + 1) ** 1.1 over a
    shuffled expert order (a skewed, Zipf-like popularity)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    pop = 1.0 / (np.arange(E) + 1.0) ** 1.1
    pop = pop[rng.permutation(E)]
    pop /= pop.sum()
    counts = np.zeros(E, np.int64)
    for _ in range(tokens):
        counts[rng.choice(E, topk, replace=False, p=pop)] += 1
    return [int(c) for c in counts]


def run_moe(args):
    """One MoE decode step's expert GEMMs: qgemm_grouped_gemm_w4a16 (decode-
    sized experts fused 32 per launch) against one qgemm_gemm_w4a16 per active
    expert, both captured as CUDA graphs and replayed (CUDA events, median);
    the active experts' weights exceed L2, so every replay reads them from
    HBM."""
    import torch
    qg = importlib.import_module("qgemm-mx_b200")
    E, N, K, topk, tokens = MOE_STEPS[args.moe]
    counts = moe_routing(E, topk, tokens)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    experts = []
    for _ in range(E):
        W = torch.randn((N, K), generator=gen, device="cuda").mul_(0.02)
        p = qg.pack_mxfp4(W)
        experts.append(qg.repack(p) if args.layout == "checked" else p)
        del W, p
    torch.cuda.empty_cache()
    rows = sum(counts)
    offs = [sum(counts[:e]) for e in range(E)]
    X = torch.randn((rows, K), generator=gen, device="cuda").to(torch.bfloat16)
    Yg = torch.zeros((rows, N), dtype=torch.bfloat16, device="cuda")
    Yl = torch.zeros_like(Yg)
    active = [e for e in range(E) if counts[e]]
    wsg = qg.make_grouped_workspace(experts, max(counts))
    wsl = torch.zeros(max(qg.workspace_size(experts[e], counts[e]) for e in active), dtype=torch.uint8,
                      device="cuda")
    stream = torch.cuda.Stream()

    def grouped(_):
        qg.grouped_gemm_w4a16(experts, X, counts, offsets=offs, out=Yg, workspace=wsg)

    def loop(_):
        for e in active:
            o, m = offs[e], counts[e]
            qg.gemm_w4a16(experts[e], X[o:o + m], out=Yl[o:o + m], workspace=wsl)

    us_g = time_graphed(grouped, 4, stream)
    us_l = time_graphed(loop, 4, stream)
    torch.cuda.synchronize()
    diff = float(((Yg.float() - Yl.float()).norm() / Yl.float().norm().clamp_min(1e-30)).item())
    nbytes = sum(qg.total_bytes(qg.MXFP4, counts[e], N, K) for e in active)
    fused = sum(1 for e in active if counts[e] <= 16)
    launches_g = 2 * ((fused + 31) // 32) + sum(qg.launch_count(experts[e], counts[e])[0]
                                                for e in active if counts[e] > 16)
    launches_l = sum(qg.launch_count(experts[e], counts[e])[0] for e in active)
    print(json.dumps({
        "moe": args.moe, "experts": E, "N": N, "K": K, "topk": topk, "tokens": tokens,
        "active_experts": len(active), "max_rows": max(counts), "rows": rows,
        "grouped_us": round(us_g, 2), "per_expert_calls_us": round(us_l, 2),
        "speedup": round(us_l / us_g, 3),
        "grouped_gbs": round(nbytes / us_g / 1e3, 1), "per_expert_calls_gbs": round(nbytes / us_l / 1e3, 1),
        "launches_grouped": launches_g, "launches_per_expert_calls": launches_l,
        "rel_frobenius_grouped_vs_calls": diff}))


def run_prefill(args):
    """TFLOP/s of the tcgen05 path on the compute-bound shapes, next to a
    cuBLAS BF16 GEMM of the same shape (weights dequantised to bf16), both
    timed as CUDA-graph replays with CUDA events, against the measured BF16
    peak.  Prints a table to stderr and one JSON line."""
    import torch
    qg = importlib.import_module("qgemm-mx_b200")
    peak = 1632.0
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            peak = float(json.load(f)["bf16_tflops"])
    gen = torch.Generator(device="cuda")
    rows = []
    for (N, K) in [(28672, 8192), (8192, 28672)]:
        gen.manual_seed(N + K)
        W = torch.randn((N, K), generator=gen, device="cuda").mul_(0.02)
        p = qg.pack(qg.NVFP4, W)
        del W
        Wb = qg.dequant(p).to(torch.bfloat16)
        for M in [2048, 4096, 8192]:
            X = torch.randn((M, K), generator=gen, device="cuda").to(torch.bfloat16)
            Y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
            Yc = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
            ws = qg.make_workspace(p, M)

            def timed(fn, reps=5):
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    for _ in range(2):
                        fn()
                torch.cuda.current_stream().wait_stream(s)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(reps):
                        fn()
                g.replay()
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                g.replay()
                b.record()
                torch.cuda.synchronize()
                return a.elapsed_time(b) / reps * 1e-3

            t_ours = timed(lambda: qg.gemm_w4a16(p, X, out=Y, workspace=ws))
            t_cub = timed(lambda: qg.cublas_bf16_gemm(Wb, X, out=Yc))
            fl = 2.0 * M * N * K
            rows.append({"N": N, "K": K, "M": M, "ours_tflops": round(fl / t_ours / 1e12, 1),
                         "cublas_bf16_tflops": round(fl / t_cub / 1e12, 1),
                         "ours_frac_of_peak": round(fl / t_ours / 1e12 / peak, 4),
                         "ours_over_cublas": round(t_cub / t_ours, 3)})
            print(json.dumps(rows[-1]), file=sys.stderr, flush=True)
            del X, Y, Yc, ws
        del p, Wb
        torch.cuda.empty_cache()
    print(json.dumps({"prefill": rows, "bf16_peak_tflops": peak}))


def fmt_code(qg, name):
    return {"mxfp4": qg.MXFP4, "nvfp4": qg.NVFP4, "int4": qg.INT4_G128}[name]


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """Polls SM clock, power and clock-event reasons through NVML every few
    milliseconds while the timed region runs (nvidia-smi's 100 ms loop can
    miss a short region entirely)."""
    # nvmlClocksEventReason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index: int, period_s: float = 0.005):
        self.gpu = gpu_index
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(cvd.split(",")[self.gpu]) if cvd and cvd.split(",")[0].isdigit() else self.gpu
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:  # no NVML: report no samples
            self._t = None
        return self

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def probe_read_gbs(qg, dev, kind=0, nbytes=1 << 30):
    """The reference's bandwidth denominator, measured in the same run: a
    read-only stream over a buffer 8x the L2 (its src/probe/bandwidth.cu:92-97
    and :111-117), ten launches per CUDA-graph replay, median of ten replays.
    kind 0: 128-bit loads; kind 1: TMA bulk copies into shared memory (no
    multicast)."""
    import torch
    buf = torch.ones(nbytes // 4, dtype=torch.int32, device=dev)
    for _ in range(3):
        qg.probe_launch(kind, buf, None, nbytes)
    torch.cuda.synchronize()
    inner, g = 10, torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(inner):
            qg.probe_launch(kind, buf, None, nbytes)
    samples = []
    for _ in range(10):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        samples.append(a.elapsed_time(b) * 1e-3 / inner)
    qg.probe_status()
    del g, buf
    torch.cuda.empty_cache()
    return nbytes / statistics.median(samples) / 1e9


def fp8_baseline(qg, dev, calls, table, l2, stream):
    """The reference's planned "vs FP8" comparison (docs/BASELINE_STUDY.md:23,
    docs/MASTER_EXECUTION_PLAN.md:280: MXFP4 >= 1.5x FP8 at M = 1): every call
    of the step as a cuBLASLt FP8 GEMM (E4M3 W and X, per-tensor scales, bf16
    Y), timed like the per-call table (weights rotated past L2, a graph of
    launches, median of ten replays)."""
    import torch
    ours = {(r["layer"], r["M"]): r["cold_us"] for r in table}
    wsp = torch.empty(32 << 20, dtype=torch.uint8, device=dev)
    one = torch.ones(1, dtype=torch.float32, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    per_call, t8, t4 = {}, 0.0, 0.0
    w8_cache = {}
    for M, name, N, K in calls:
        if (N, K) not in w8_cache:
            Wf = torch.randn((N, K), generator=gen, device=dev).mul_(0.02)
            sw = float(Wf.abs().max()) / 448.0
            w8_cache[(N, K)] = ((Wf / sw).to(torch.float8_e4m3fn).view(torch.uint8), torch.tensor([sw], device=dev))
            del Wf
        W8, sw = w8_cache[(N, K)]
        rot = max(2, math.ceil(2 * l2 / (N * K)))
        copies = [W8] + [W8.clone() for _ in range(rot - 1)]
        X8 = torch.randn((M, K), generator=gen, device=dev).clamp_(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
        Y8 = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        inner = max(rot, 8)
        with torch.cuda.stream(stream):
            for j in range(inner):
                qg.cublaslt_fp8_gemm(copies[j % rot], X8, sw, one, out=Y8, workspace=wsp)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for j in range(inner):
                qg.cublaslt_fp8_gemm(copies[j % rot], X8, sw, one, out=Y8, workspace=wsp)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        samples = []
        for _ in range(10):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            b.synchronize()
            samples.append(a.elapsed_time(b) * 1e3 / inner)
        us8 = statistics.median(samples)
        us4 = ours[(name, M)]
        per_call[f"{name}:M={M}"] = {"fp8_us": round(us8, 2), "mxfp4_us": round(us4, 2),
                                     "mxfp4_vs_fp8": round(us8 / us4, 3)}
        t8, t4 = t8 + us8, t4 + us4
        del copies, g
        torch.cuda.empty_cache()
    return {"fp8_us_per_step": round(t8, 2), "mxfp4_us_per_step": round(t4, 2),
            "mxfp4_vs_fp8": round(t8 / t4, 3), "per_call": per_call,
            "how": "qgemm_cublaslt_fp8_gemm (cuBLASLt, E4M3 x E4M3, per-tensor scales, bf16 out), same shapes, "
                   "weights rotated past L2, graph of launches, median of 10; X is given already in E4M3 (its "
                   "quantisation is not timed, while mxfp4_us includes the X preparation kernel); mxfp4_us from "
                   "the per-call table"}


def _median_us(run_once, inner, samples=20):
    """Median over `samples` of (device time of run_once()) / inner, in us."""
    import torch
    out = []
    for _ in range(samples):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run_once()
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b) * 1e3 / inner)
    return statistics.median(out)


def time_graphed(fn, inner, stream):
    """The reference's time_graphed (timing.cuh:288-336): `inner` calls
    fn(j) captured into one CUDA graph, warmed, median of replays, per call."""
    import torch
    with torch.cuda.stream(stream):
        for j in range(inner):
            fn(j)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for j in range(inner):
            fn(j)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    us = _median_us(g.replay, inner)
    del g
    return us


def time_looped(fn, inner, stream):
    """The reference's time_looped (timing.cuh:250-277): the same calls
    launched one by one from the host, so launch overhead is inside."""
    import torch
    with torch.cuda.stream(stream):
        for j in range(inner):
            fn(j)
        torch.cuda.synchronize()

        def loop():
            for j in range(inner):
                fn(j)
        us = _median_us(loop, inner)
    return us


def per_call_table(qg, dev, calls, shards, X, Y, ws, fcode, l2, stream, kernel_of, cublas=True):
    """Per (layer, M), as the reference's bench_cublas.cu:152-175 reports:
    cold = graphed with the weights rotated past L2 (rot = max(2, ceil(2 L2 /
    W bytes)), timing.cuh:152-158, inner = max(rot, 8)); hot = graphed on one
    weight buffer; looped = the cold calls launched one by one;
    l2_inflation = cold / hot; launch_share = 100 (looped - cold) / looped;
    GB/s and %% of peak from the algorithmic bytes (formats.cuh:80-83);
    TFLOP/s = 2 M N K / cold and its fraction of the measured BF16 peak; and a
    cuBLAS BF16 GEMM of the same shape (dense bf16 W, rotated likewise)."""
    import torch
    peak_hbm, _ = measured_peaks()
    bf16_peak = measured_bf16_tflops()
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    wb16 = {}
    rows = []
    for M, name, N, K in calls:
        p = shards[name]
        wbytes = qg.weight_bytes(fcode, p.N, K)
        rot = max(2, math.ceil(2 * l2 / max(wbytes, 1)))
        copies = [p] + [qg.Packed(p.format, p.N, p.K, p.data.clone(), p.scales.clone(), p.tensor_scale, p.layout)
                        for _ in range(rot - 1)]
        inner = max(rot, 8)
        Xm, Ym, wsm = X[(M, K)], Y[(M, name)], ws[(M, name)]

        def cold(j):
            qg.gemm_w4a16(copies[j % rot], Xm, out=Ym, workspace=wsm)

        def hot(j):
            qg.gemm_w4a16(p, Xm, out=Ym, workspace=wsm)
        c_us = time_graphed(cold, inner, stream)
        h_us = time_graphed(hot, inner, stream)
        l_us = time_looped(cold, inner, stream)
        nb = qg.total_bytes(fcode, M, p.N, K)
        fl = 2.0 * M * p.N * K
        r = {"layer": name, "M": M, "N": p.N, "K": K, "rot": rot, "kernel": kernel_of[(M, name)],
             "cold_us": round(c_us, 3), "hot_us": round(h_us, 3), "looped_us": round(l_us, 3),
             "bytes": nb, "gbs": round(nb / (c_us * 1e-6) / 1e9, 1),
             "pct_of_hbm_peak": round(100 * nb / (c_us * 1e-6) / 1e9 / peak_hbm, 2),
             "tflops": round(fl / (c_us * 1e-6) / 1e12, 2),
             "frac_of_bf16_peak": round(fl / (c_us * 1e-6) / 1e12 / bf16_peak, 4),
             "l2_inflation": round(c_us / h_us, 3), "launch_share_pct": round(100 * (l_us - c_us) / l_us, 2)}
        del copies
        if cublas:
            key = (p.N, K)
            if key not in wb16:
                wb16.clear()
                torch.cuda.empty_cache()
                wb16[key] = torch.randn((p.N, K), generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
            W16 = wb16[key]
            rot16 = max(2, math.ceil(2 * l2 / (2 * p.N * K)))
            c16 = [W16] + [W16.clone() for _ in range(rot16 - 1)]
            Yc = torch.empty((M, p.N), dtype=torch.bfloat16, device=dev)

            def cub(j):
                qg.cublas_bf16_gemm(c16[j % rot16], Xm, out=Yc)
            cu_us = time_graphed(cub, max(rot16, 8), stream)
            r["cublas_bf16_us"] = round(cu_us, 3)
            r["vs_cublas_bf16"] = round(cu_us / c_us, 3)
            del c16, Yc
        rows.append(r)
        torch.cuda.empty_cache()
    wb16.clear()
    torch.cuda.empty_cache()
    return rows


def measured_bf16_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# CPU path (the reference's own host code, or the oracle port)
# ---------------------------------------------------------------------------

def cpu_path():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not os.path.exists(O.ORACLE_SO):
        O.build()
    r = O.reference()
    return O, (r if r is not None else O.oracle()), ("reference" if r is not None else "port")


def cpu_sample_run(fmt, layers, ms, rows, threads, O, impl, packed_cache):
    """Times dequant + reference GEMM over `rows` rows of every (layer, M);
    returns (seconds, algorithmic bytes of that sample)."""
    tot_bytes, secs = 0, 0.0
    for M in ms:
        for name, N, K in layers:
            key = (name, K, rows)
            if key not in packed_cache:
                W = O.randn(7, hash(name) & 0xFFFF, rows * K, 0.0, 0.02).reshape(rows, K)
                ts = O.nvfp4_tensor_scale(W) if fmt == "nvfp4" else 1.0
                st, d, s = impl.pack(fmt, W, tensor_scale=ts)
                packed_cache[key] = (d, s, ts)
            d, s, ts = packed_cache[key]
            X = O.randn_bf16(1, M, M * K).reshape(M, K)
            t0 = time.perf_counter()
            impl.w4a16_gemm(fmt, d, s, rows, K, X, tensor_scale=ts, nthreads=threads)
            secs += time.perf_counter() - t0
            wb = {"mxfp4": 0.53125, "nvfp4": 0.5625, "int4": 0.515625}[fmt]
            tot_bytes += int(wb * rows * K) + M * K * 2 + M * rows * 2
    return secs, tot_bytes


def calibrate_rows(fmt, layers, ms, threads, O, impl, target_s):
    cache = {}
    rows = 16
    secs, _ = cpu_sample_run(fmt, layers, ms, rows, threads, O, impl, cache)
    scale = target_s / max(secs, 1e-3)
    return max(16, min(4096, int(rows * scale) // 16 * 16))


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    fmt, layers, ms = WORKLOADS[args.workload]
    O, impl, kind = cpu_path()
    threads = os.cpu_count() or 1
    budget = 150.0
    step_target = min(3.0, budget / max(1, args.steps + args.warmup))
    rows = calibrate_rows(fmt, layers, ms, threads, O, impl, step_target)
    cache = {}
    for _ in range(args.warmup):
        cpu_sample_run(fmt, layers, ms, rows, threads, O, impl, cache)
    tsum, bsum = 0.0, 0
    for _ in range(args.steps):
        s, b = cpu_sample_run(fmt, layers, ms, rows, threads, O, impl, cache)
        tsum += s
        bsum += b
    gbs = bsum / tsum / 1e9
    sample = (f"{rows} rows of each of {len(layers)} layers x M in {ms} per step "
              f"(dequant + gemm_fp32_ref, {threads} threads)")
    line = {
        "impl": "reference", "metric": "W4A16 GEMM achieved HBM GB/s (% of probed B200 peak)",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * tsum / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": args.workload, "format": fmt, "layers": [[n, N, K] for n, N, K in layers],
                   "M": ms, "sample_rows": rows},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def main():
    args = parse()
    if args.case:
        run_case(args)
        return
    if args.prefill:
        run_prefill(args)
        return
    if args.moe:
        run_moe(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    qg = importlib.import_module("qgemm-mx_b200")
    fmt, layers, ms = WORKLOADS[args.workload]
    fcode = fmt_code(qg, fmt)
    sms, l2 = qg.device_info()

    # ---- weights: each rank packs its own contiguous row shard -------------
    gen = torch.Generator(device=dev)
    shards = {}
    for li, (name, N, K) in enumerate(layers):
        if N % world:
            raise SystemExit(f"N={N} not divisible by world={world}")
        n_loc = N // world
        gen.manual_seed(1000 + li)  # same full W on every rank; take this rank's rows
        W = torch.randn((N, K), generator=gen, device=dev, dtype=torch.float32).mul_(0.02)
        Wl = W[rank * n_loc:(rank + 1) * n_loc].contiguous()
        del W
        shards[name] = qg.pack(fcode, Wl)
        if args.layout == "checked" and fcode in (qg.MXFP4, qg.NVFP4):
            shards[name] = qg.repack(shards[name])
        del Wl
        torch.cuda.empty_cache()
    Kset = sorted({K for _, _, K in layers})
    gen.manual_seed(7)
    X = {(M, K): torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16) for M in ms for K in Kset}
    Y = {(M, name): torch.empty((M, N // world), dtype=torch.bfloat16, device=dev)
         for M in ms for name, N, _ in layers}
    ws = {}
    for M in ms:
        for name, N, K in layers:
            ws[(M, name)] = qg.make_workspace(shards[name], M)
    calls = [(M, name, N, K) for M in ms for name, N, K in layers]

    # ---- world > 1: every rank's Y_full buffers and sync block in one
    # allocation shared by CUDA IPC; tp_gemm writes each slice into every
    # rank's Y_full over NVLink and waits for the other slices -------------
    Yfull, y_peers, sync_peers, tpws, opened = {}, {}, [], {}, []
    Yfull2, y_peers2 = {}, {}  # a second Y_full set for the end-to-end run's double buffering
    if world > 1:
        offs, off = {}, 256
        for M, name, N, K in calls:
            offs[(M, name)] = off
            off += (M * N * 2 + 255) // 256 * 256
        payload = off - 256  # [sync block | set 0 | set 1], one allocation, one IPC handle
        tpbuf = torch.zeros(256 + 2 * payload, dtype=torch.uint8, device=dev)
        handles = [None] * world
        dist.all_gather_object(handles, qg.ipc_handle(tpbuf))
        bases = []
        for r in range(world):
            if r == rank:
                bases.append(tpbuf.data_ptr())
            else:
                b0, ptr = qg.ipc_open(*handles[r])
                opened.append(b0)
                bases.append(ptr)
        sync_peers = bases
        for M, name, N, K in calls:
            o = offs[(M, name)]
            y_peers[(M, name)] = [b + o for b in bases]
            Yfull[(M, name)] = tpbuf[o:o + M * N * 2].view(torch.bfloat16).view(M, N)
            y_peers2[(M, name)] = [b + o + payload for b in bases]
            Yfull2[(M, name)] = tpbuf[o + payload:o + payload + M * N * 2].view(torch.bfloat16).view(M, N)
            tpws[(M, name)] = qg.make_tp_workspace(shards[name], M)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # every rank's buffers exist before any rank's first tp_gemm
    kernel_of = {(M, name): qg.launch_count(shards[name], M)[1] for M, name, N, K in calls}
    launches_per_step = sum(qg.launch_count(shards[name], M)[0] for M, name, N, K in calls)
    bytes_rank = sum(qg.total_bytes(fcode, M, N // world, K) for M, name, N, K in calls)
    bytes_step = bytes_rank * world

    def gemm(M, name, Xin):
        if world == 1:
            qg.gemm_w4a16(shards[name], Xin, out=Y[(M, name)], workspace=ws[(M, name)])
        else:
            qg.tp_gemm(shards[name], Xin, world, rank, y_peers[(M, name)], sync_peers, tpws[(M, name)])

    def step():
        for M, name, N, K in calls:
            gemm(M, name, X[(M, K)])

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        # first warm-up step call by call, each followed by a synchronise, so
        # that a device fault names the call that raised it
        for M, name, N, K in calls:
            try:
                gemm(M, name, X[(M, K)])
                torch.cuda.synchronize()
            except Exception as e:
                raise SystemExit(f"warm-up call (layer {name}, M={M}) failed: {e}")
        for _ in range(max(3, args.warmup) - 1):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    # ---- timed region: device-resident, one graph replay per step ---------
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(0.02)  # let the sampler take its first reading
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    if world > 1:
        qg.tp_status()
        dist.barrier()
    ms_step = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms_step], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item())
    value = bytes_step / (ms_step * 1e-3) / 1e9
    clk = clocks.summary()

    # ---- e2e: same step through the C-ABI with host buffers ----------------
    # Every step copies its distinct activations host -> device (pinned), runs
    # the 12 GEMMs and reads every Y back to pinned host memory.  Two device
    # buffer sets, so step i + 1's inputs travel on one copy stream and each
    # finished Y of step i on another while step i's GEMMs run; events keep a
    # buffer set from being reused before its copies and GEMMs are done.
    # Several GPUs: the two sets of Y_full are shared by every rank, and each
    # rank reads back its own 1/world of every result (the job reads Y once).
    Xh = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True).copy_(v.cpu()) for k, v in X.items()}
    Xd = {(M, K): torch.empty_like(X[(M, K)]) for (M, K) in X}
    h2d = sum(v.numel() * 2 for v in Xh.values())
    d2h = sum(M * N * 2 for M, name, N, K in calls)  # all of Y, once per step for the whole job
    if world == 1:
        Yh = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in Y.items()}
    else:
        Yh = {(M, name): torch.empty(M * N // world, dtype=torch.bfloat16, pin_memory=True)
              for M, name, N, K in calls}

    if world == 1:
        Xd2 = [Xd, {k: torch.empty_like(v) for k, v in Xd.items()}]
        Yd2 = [Y, {k: torch.empty_like(v) for k, v in Y.items()}]
        hs, ds = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        x_ready = [torch.cuda.Event(), torch.cuda.Event()]
        x_free = [torch.cuda.Event(), torch.cuda.Event()]
        y_free = [torch.cuda.Event(), torch.cuda.Event()]
        ydone = {k: torch.cuda.Event() for k in Y}

        def h2d_into(i):
            b = i % 2
            hs.wait_event(x_free[b])  # the GEMMs of step i - 2 have read this set
            with torch.cuda.stream(hs):
                for key in Xd2[b]:
                    Xd2[b][key].copy_(Xh[key], non_blocking=True)
            x_ready[b].record(hs)

        def e2e_run(nsteps):
            main = torch.cuda.current_stream()
            for ev in x_ready + x_free + y_free:
                ev.record(main)
            h2d_into(0)
            for i in range(nsteps):
                b = i % 2
                if i + 1 < nsteps:
                    h2d_into(i + 1)
                main.wait_event(x_ready[b])
                main.wait_event(y_free[b])  # step i - 2's results from this set are on the host
                for M, name, N, K in calls:
                    qg.gemm_w4a16(shards[name], Xd2[b][(M, K)], out=Yd2[b][(M, name)], workspace=ws[(M, name)])
                    ydone[(M, name)].record(main)
                    ds.wait_event(ydone[(M, name)])
                    with torch.cuda.stream(ds):
                        Yh[(M, name)].copy_(Yd2[b][(M, name)], non_blocking=True)
                x_free[b].record(main)
                y_free[b].record(ds)
            main.wait_stream(ds)  # the run ends when every result is on the host
            main.wait_stream(hs)
    else:
        # A rank's step i + 1 writes set (i + 1) % 2 of every rank's Y_full,
        # and it starts only after the exchange of the last call of step i
        # completed on every rank.  Each rank enters that last call after its
        # own read-back of step i - 1 (the same set) finished, so no rank
        # overwrites a set another rank is still reading.
        Xd2 = [Xd, {k: torch.empty_like(v) for k, v in Xd.items()}]
        Yf2, yp2 = [Yfull, Yfull2], [y_peers, y_peers2]
        hs, ds = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        x_ready = [torch.cuda.Event(), torch.cuda.Event()]
        x_free = [torch.cuda.Event(), torch.cuda.Event()]
        y_free = [torch.cuda.Event(), torch.cuda.Event()]
        ydone = {(M, name): torch.cuda.Event() for M, name, N, K in calls}

        def h2d_into(i):
            b = i % 2
            hs.wait_event(x_free[b])
            with torch.cuda.stream(hs):
                for key in Xd2[b]:
                    Xd2[b][key].copy_(Xh[key], non_blocking=True)
            x_ready[b].record(hs)

        def e2e_run(nsteps):
            main = torch.cuda.current_stream()
            for ev in x_ready + x_free + y_free:
                ev.record(main)
            h2d_into(0)
            for i in range(nsteps):
                b = i % 2
                if i + 1 < nsteps:
                    h2d_into(i + 1)
                main.wait_event(x_ready[b])
                for ci, (M, name, N, K) in enumerate(calls):
                    if ci == len(calls) - 1:
                        main.wait_event(y_free[1 - b])  # this rank's read-back of step i - 1 is done
                    qg.tp_gemm(shards[name], Xd2[b][(M, K)], world, rank, yp2[b][(M, name)], sync_peers,
                               tpws[(M, name)])
                    ydone[(M, name)].record(main)
                    ds.wait_event(ydone[(M, name)])
                    part = M * N // world
                    with torch.cuda.stream(ds):
                        Yh[(M, name)].copy_(Yf2[b][(M, name)].view(-1)[rank * part:(rank + 1) * part],
                                            non_blocking=True)
                x_free[b].record(main)
                y_free[b].record(ds)
            main.wait_stream(ds)  # the run ends when every result is on the host
            main.wait_stream(hs)

    e2e_run(max(3, args.warmup))
    torch.cuda.synchronize()
    # the end-to-end run is captured as one graph of all its steps: bounded so
    # the capture stays small (the device-side region above runs --steps)
    e2e_steps = min(args.steps, 100)
    # the whole run (every step's copies in and out and its 12 C-ABI calls) as
    # one CUDA graph, as the device-side number is taken: the host then does
    # not pace the GPU; one untimed replay, then the timed one (several GPUs:
    # the exchange inside the kernels is the only cross-rank step, no library
    # collective is captured)
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e):
        e2e_run(e2e_steps)
    if world > 1:
        dist.barrier()
    g_e2e.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g_e2e.replay()
    e1.record()
    torch.cuda.synchronize()
    if world == 1:  # the read-backs of the last step equal a fresh call (the kernels are deterministic)
        for M, name, N, K in calls:
            ref_y = qg.gemm_w4a16(shards[name], Xd[(M, K)].copy_(Xh[(M, K)]), workspace=ws[(M, name)])
            if not torch.equal(ref_y.cpu().view(torch.int16), Yh[(M, name)].view(torch.int16)):
                raise SystemExit(f"e2e: read-back of {name} M={M} differs from a fresh call")
    te = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = bytes_step / (float(te.item()) * 1e-3) / 1e9

    # ---- per-call table: the reference's protocol (bench_cublas.cu:152-175) --
    table = per_call_table(qg, dev, calls, shards, X, Y, ws, fcode, l2, s, kernel_of,
                           cublas=(world == 1 and not args.no_cublas))
    fp8 = fp8_baseline(qg, dev, calls, table, l2, s) if (args.fp8 and world == 1) else None
    # no number is reported from a run in which a kernel's bounded wait gave up
    # (its outputs are then wrong): that raises here and the bench exits non-zero
    qg.umma_status()
    peak, peak_src = measured_peaks()
    probe_ldg = probe_read_gbs(qg, dev, 0) if rank == 0 else None
    probe_tma = probe_read_gbs(qg, dev, 1) if rank == 0 else None
    probe_gbs = max(probe_ldg, probe_tma) if rank == 0 else None
    # per GEMM kernel: algorithmic bytes per launch / mean launch time; the
    # roofline entry is the kernel with the largest share of the step
    per_kernel = {}
    for r in table:
        d = per_kernel.setdefault(r["kernel"], {"us": 0.0, "bytes": 0, "launches": 0, "shapes": []})
        d["us"] += r["cold_us"]
        d["bytes"] += r["bytes"]
        d["launches"] += 1
        d["shapes"].append(f"{r['layer']}:M={r['M']}")
    dom = max(per_kernel, key=lambda k: per_kernel[k]["us"])
    achieved = per_kernel[dom]["bytes"] / (per_kernel[dom]["us"] * 1e-6) / 1e9
    traffic = None
    tr_path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(tr_path) and world == 1:
        with open(tr_path) as f:
            trd = json.load(f).get(args.workload, {}).get(dom, {})
        got = [trd[sh] for sh in per_kernel[dom]["shapes"] if sh in trd]
        if got and len(got) == len(per_kernel[dom]["shapes"]):
            traffic = round(sum(got) / len(got))  # DRAM bytes per launch, ncu capture

    # ---- CPU baseline (rank 0 at N=1 only) ---------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        O, impl, kind = cpu_path()
        threads = os.cpu_count() or 1
        rows = calibrate_rows(fmt, layers, ms, threads, O, impl, 12.0)
        cache = {}
        secs, nb, reps = 0.0, 0, 0
        while secs < 12.0 and reps < 64:  # repeat the bounded sample to ~12 s of CPU work
            s1, b1 = cpu_sample_run(fmt, layers, ms, rows, threads, O, impl, cache)
            secs, nb, reps = secs + s1, nb + b1, reps + 1
        cpu = {"value": round(nb / secs / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": f"{rows} rows of each layer x M in {ms} (dequant + gemm_fp32_ref), "
                         f"{reps} passes, {secs:.1f} s"}

    if args.table and rank == 0:
        print(f"{'layer':8s} {'M':>4s} {'N':>6s} {'K':>6s} {'rot':>3s} {'cold_us':>9s} {'hot_us':>8s} "
              f"{'loop_us':>8s} {'GB/s':>8s} {'%peak':>6s} {'TF/s':>7s} {'l2inf':>6s} {'launch%':>7s} "
              f"{'cublas':>8s}  kernel", file=sys.stderr)
        for r in table:
            print(f"{r['layer']:8s} {r['M']:4d} {r['N']:6d} {r['K']:6d} {r['rot']:3d} {r['cold_us']:9.2f} "
                  f"{r['hot_us']:8.2f} {r['looped_us']:8.2f} {r['gbs']:8.1f} {100 * r['gbs'] / peak:6.1f} "
                  f"{r['tflops']:7.1f} {r['l2_inflation']:6.2f} {r['launch_share_pct']:7.1f} "
                  f"{(r.get('cublas_bf16_us') or 0):8.2f}  {r['kernel']}", file=sys.stderr)

    if rank == 0:
        line = {
            "metric": "W4A16 GEMM achieved HBM GB/s (% of probed B200 peak)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) X, N(0,0.02) W packed on device)",
            "config": {"workload": args.workload, "format": fmt,
                       "layers": [[n, N, K] for n, N, K in layers], "M": ms,
                       "layout": args.layout if fmt in ("mxfp4", "nvfp4") else "canonical",
                       "parallelism": f"N-shard x{world}" + (" + all-gather of Y over NVLink peer stores "
                                                              "(qgemm_tp_gemm_w4a16)" if world > 1 else ""),
                       "l2": "cold: step working set 419 MB > 126 MB L2, calls M-major",
                       "pct_of_hbm_peak": round(100 * value / peak, 2)},
            "probe": {"read_only_gbs": round(probe_gbs, 1), "pct_of_probe": round(100 * value / probe_gbs, 2),
                      "ldg_gbs": round(probe_ldg, 1), "tma_bulk_gbs": round(probe_tma, 1),
                      "how": "max of qgemm_probe_launch kinds 0 (128-bit loads) and 1 (TMA bulk copies), "
                             "1 GiB, graph of 10, median of 10; the reference's denominator "
                             "(src/probe/bandwidth.cu:111-117), measured in this run"},
            "per_call": [{k: v for k, v in r.items() if k != "bytes"} for r in table],
            "per_call_how": "cold/hot/looped as the reference's bench_cublas.cu:152-175 (graph of max(rot, 8) "
                            "calls, median of 20); cublas_bf16_us: dense bf16 W of the same shape, rotated",
            **({"fp8_baseline": fp8} if fp8 else {}),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "copies": "whole job per step: every rank's X in; Y out once (each rank its 1/world)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": dom, "share": round(per_kernel[dom]["us"] / sum(v["us"] for v in per_kernel.values()), 3),
                         "algorithmic_bytes_per_launch": round(per_kernel[dom]["bytes"] / per_kernel[dom]["launches"]),
                         "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                         else "fallback 6650 GB/s",
                         "kernels": {k: {"achieved": round(v["bytes"] / (v["us"] * 1e-6) / 1e9, 1),
                                         "frac": round(v["bytes"] / (v["us"] * 1e-6) / 1e9 / peak, 4),
                                         "us_per_step": round(v["us"], 2), "launches_per_step": v["launches"]}
                                     for k, v in per_kernel.items()}},
            "cpu_baseline": cpu,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
            "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        qg.tp_status()
        del graph, g_e2e
        dist.barrier()  # no rank unmaps while a peer may still write into it
        for b0 in opened:
            qg.ipc_close(b0)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
