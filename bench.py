#!/usr/bin/env python3
"""Benchmark of the sm_100a NVFP4 x NVFP4 -> BF16 GEMM (one JSON line on rank 0).

Workload: M = N = K = 8192, A and B drawn from N(0,1) on the device
(seeded torch generator), quantised to NVFP4 by this library's GPU quantiser (global scale
amax/(448*6), per-16 UE4M3 block scales, E2M1 RNE), alpha = gA*gB, BF16 output.
With --gpus P > 1 the GEMM is split along N: every rank owns an 8192-column slice of B
(weak scaling: global N = 8192*P) and A is replicated; no collective sits on the data path.
The optional NCCL all-gather of the C slices is timed separately ("gather").

A "step" is one GEMM launch.  Steps run back to back, cycling through ROT independent input
sets whose total size exceeds the 126 MB L2 (4 x 72 MB), so no step finds its inputs in L2;
`value` = whole-job TFLOP/s from CUDA events around the K timed steps (max over ranks).
A second figure times single launches after a 256 MB L2-flush write ("per_launch_l2_flush").
`e2e` is the same GEMM through the C ABI with pinned host buffers: H2D of A/SFA/B/SFB and D2H
of D of every step inside the timed region, the steps pipelined over upload / compute /
download streams.  The decode shape (configs[2], M=16 N=28672 K=8192) is
reported under "decode" in HBM GB/s, back to back over 3 rotating weight sets (396 MB), with
M = 1, 64, 128 under "decode.sweep_by_M".  "prefill" is configs[3] (M=16384 N=8192 K=28672,
1% outlier activations) and "nsplit" configs[4] (M=32768, N=65536 split over the ranks,
K=8192; strong scaling; at P > 1 also, unless --no-gather, the NCCL all-gather, the fused
gather with its NVLink figures and the tensor-parallel decode leg, each checked against the
oracle on a sample).  "parity" holds every rank's check of its own timed output.
"library_baseline" times cuBLASLt's NVFP4 GEMM on the same 8192^3 operands, for comparison.

The CPU leg ("cpu_baseline") times the host reference loop and, as the checker, compares its
output with the first 128 rows of the bench's own 8192^3 GPU result ("parity_vs_gpu").

--impl reference runs the reference's host GEMM (the CPU oracle's restatement of
example/nvfp4_bf16_gemm.cu:161-168) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SPEC_FP4_TFLOPS = 9000.0      # B200 dense FP4 (4 x the 2250 TF/s dense BF16 figure)
SPEC_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0     # used only when the measured-peaks file is absent
FALLBACK_BF16_TFLOPS = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192, help="columns per GPU")
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--case", default="all", choices=["all", "main", "decode", "quantize", "compare"],
                    help="main: only the 8192^3-class GEMM; decode: only the M=16 GEMM; "
                         "quantize: only the quantiser leg; compare: this library's and cuBLASLt's "
                         "NVFP4 GEMM alternating on the same operands (small runs for profiler "
                         "captures; the JSON line then lacks the others)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--decode-warmup", type=int, default=4000,
                    help="decode warm-up launches (~0.1 s at 4000; fewer for profiler captures)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the configs[3] prefill and configs[4] N-split legs")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-gather", action="store_true",
                    help="P > 1: skip the gather legs (NCCL all-gather, the fused gather and the "
                         "tensor-parallel decode leg), which run by default")
    ap.add_argument("--no-library", action="store_true",
                    help="skip the cuBLASLt NVFP4 comparison leg (torch._scaled_mm, same operands)")
    ap.add_argument("--schedule", default="auto", choices=["auto", "1sm", "2sm"],
                    help="GEMM schedule for the main workload (auto: one-SM for M > 128)")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profiled_traffic(key):
    """DRAM bytes per launch from a committed ncu capture (profiles/traffic.json)."""
    try:
        return json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))[key]["bytes_per_launch"]
    except Exception:
        return None


# ---------------------------------------------------------------------------------------
# clocks during the timed region (NVML, the library behind nvidia-smi)
# ---------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index, interval=0.0002, enabled=True):
        """enabled=False (ranks other than 0, whose record is not printed) samples nothing:
        eight ranks querying NVML at once slow each other down to ~1 sample per timed region."""
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        self.nv = None
        if not enabled:
            self.interval = interval
            return
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
        self.interval = interval

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------
def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def dist_rank():
    """This process's rank (0 without a process group)."""
    import torch.distributed as dist
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------------------
def make_operand(rows, K, seed, std, dev, outlier_p=0.0, outlier_x=20.0):
    import torch
    import blackhole_b200 as bh

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((rows, K), generator=g, device=dev, dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    if outlier_p > 0:  # configs[3]: a fraction of the entries multiplied (outlier channels)
        mask = torch.rand((rows, K), generator=g, device=dev) < outlier_p
        x[mask] *= outlier_x
        del mask
    packed, sf, scales = bh.quantize_tensor(x)
    torch.cuda.synchronize()
    del x
    return packed, sf, scales


def sf_bytes(mn, k):
    return ((mn + 127) // 128) * ((k // 16 + 3) // 4) * 512


def gemm_bytes(M, N, K):
    return M * K // 2 + N * K // 2 + M * K // 16 + N * K // 16 + 2 * M * N


def time_gemm(M, N, K, sets, D, steps, warmup, world, schedule="auto", fmt="nvfp4", clk=None):
    """Back-to-back launches cycling through the input sets; returns total ms of `steps`
    launches from CUDA events on the launching stream (one event pair around all of them).
    A ClockSampler passed as `clk` samples exactly the timed region (after the warm-up
    barrier, until the closing one)."""
    import torch
    import blackhole_b200 as bh

    stream = torch.cuda.current_stream()

    def launch(A, SFA, B, SFB, alpha):
        if fmt == "mxfp4":
            bh.mxfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha, schedule=schedule)
        elif fmt == "mxf8f4":
            bh.mxf8f4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha, schedule=schedule)
        elif schedule == "auto":
            bh.nvfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha)
        else:
            bh.nvfp4_bf16_gemm_ex(M, N, K, A, SFA, B, SFB, D, alpha, schedule=schedule)

    for i in range(warmup):
        launch(*sets[i % len(sets)])
    barrier(world)
    if clk is not None:
        clk.__enter__()
    try:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        h0 = time.perf_counter()
        for i in range(steps):
            launch(*sets[i % len(sets)])
        host_us = (time.perf_counter() - h0) * 1e6 / steps
        e.record(stream)
        barrier(world)
    finally:
        if clk is not None:
            clk.__exit__(None, None, None)
    time_gemm.host_us_per_launch = host_us
    return s.elapsed_time(e)


def time_gemm_flushed(M, N, K, A, SFA, B, SFB, D, alpha, steps, flush, world):
    """Single launches, each after a 256 MB write that flushes L2; per-launch event times."""
    import torch
    import blackhole_b200 as bh

    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    barrier(world)
    for s, e in ev:
        flush.zero_()
        s.record(stream)
        bh.nvfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha)
        e.record(stream)
    barrier(world)
    return [s.elapsed_time(e) for s, e in ev]


def run_e2e(M, N, K, A, SFA, B, SFB, alpha, steps, world):
    """The C-ABI call with pinned host buffers, H2D of every step's inputs and D2H of every
    step's result inside the timed region, pipelined the way a serving loop runs it: step
    i+1's inputs upload (copy stream) while step i computes and step i-1's result downloads
    (a second copy stream; PCIe is full duplex), over two device buffer sets ordered by
    events.  A step costs about its slowest part instead of the sum of the three."""
    import torch
    import blackhole_b200 as bh

    dev = A.device
    hIn = [t.cpu().pin_memory() for t in (A, SFA, B, SFB)]
    dIn = [[torch.empty_like(t) for t in (A, SFA, B, SFB)] for _ in range(2)]
    dD = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    hD = [torch.empty((M, N), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s_cmp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_done = [torch.cuda.Event() for _ in range(2)]
    cmp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in hIn)
    d2h = hD[0].numel() * hD[0].element_size()
    # every event starts recorded, so the first waits on each buffer pass at once
    for b in range(2):
        for ev in (in_done[b], cmp_done[b], out_done[b]):
            ev.record(s_cmp)

    def step(k):
        b = k % 2
        s_in.wait_event(cmp_done[b])              # the GEMM that last read dIn[b] is done
        with torch.cuda.stream(s_in):
            for d, h in zip(dIn[b], hIn):
                d.copy_(h, non_blocking=True)
        in_done[b].record(s_in)
        s_cmp.wait_event(in_done[b])
        s_cmp.wait_event(out_done[b])             # the download that last read dD[b] is done
        bh.nvfp4_bf16_gemm(M, N, K, *dIn[b], dD[b], alpha, stream=s_cmp)
        cmp_done[b].record(s_cmp)
        s_out.wait_event(cmp_done[b])
        with torch.cuda.stream(s_out):
            hD[b].copy_(dD[b], non_blocking=True)
        out_done[b].record(s_out)

    step(0)
    step(1)
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(s_cmp)
    s_in.wait_event(s)
    s_out.wait_event(s)
    for k in range(steps):
        step(k)
    s_cmp.wait_stream(s_in)
    s_cmp.wait_stream(s_out)
    e.record(s_cmp)
    barrier(world)
    ms = s.elapsed_time(e) / steps
    return ms, h2d, d2h


# ---------------------------------------------------------------------------------------
# CPU legs (the oracle restatement of the reference's host loop)
# ---------------------------------------------------------------------------------------
def decoded_operands(A, SFA, B, SFB, rows_a, rows_b, K):
    """The float arrays the reference example builds before its host loop (element values
    and per-16 scale values, example/nvfp4_bf16_gemm.cu:159-168 reads them as refA / sfaVal):
    rows_a rows of A and rows_b rows of B.  Made once, outside any timed region."""
    from oracle import oracle as O
    vA, sA = O.decode_operand(A[:rows_a * K // 2], SFA, rows_a, K)
    vB, sB = O.decode_operand(B[:rows_b * K // 2], SFB, rows_b, K)
    return vA, sA, vB, sB


def cpu_loop_seconds(dec, rows, alpha, threads):
    """The example's host loop (a = vA*sA, b = vB*sB, acc += a*b in k order, then
    bf16(alpha*acc)) on `rows` full output rows against every decoded row of B; seconds."""
    from oracle import oracle as O
    vA, sA, vB, sB = dec
    t0 = time.perf_counter()
    O.ref_loop(vA[:rows], sA[:rows], vB, sB, alpha, nthreads=threads)
    return time.perf_counter() - t0


def cpu_parity(A, SFA, B, SFB, N, K, alpha, gpu_rows, threads):
    """The checker half of the CPU leg: the host reference on the first rows of the timed
    workload (untimed, with the per-element sum |a*b| the tolerance needs) against the bench's
    own GPU output for the same operands.  Tolerance per element: one BF16 ulp of the larger
    magnitude + |alpha| * sqrt(K) * 2^-24 * sum_k |a_k b_k| (FP32 reassociation), the one the
    parity tests assert; the worst-case K * 2^-24 bound is reported beside it."""
    from oracle import oracle as O
    rows = gpu_rows.shape[0]
    ref, absdot = O.gemm_full(rows, N, K, A, SFA, B, SFB, alpha=alpha, nthreads=threads)
    r = O.check_report(ref, gpu_rows, alpha, K, absdot)
    r.update({"rows": rows,
              "tolerance": "ulp_bf16 + |alpha|*sqrt(K)*2^-24*sum|a*b| per element (worst-case "
                           "bound: K*2^-24); reference_rel_max is the example's own "
                           "|got-ref|/(|ref|+1e-3) (it accepts <= 0.05)"})
    return r


def cpu_baseline(A, SFA, B, SFB, N, K, alpha, M, budget_s=12.0, gpu_rows=None):
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    cal = min(threads, M)
    dec = decoded_operands(A, SFA, B, SFB, cal, N, K)
    # calibrate on `cal` full rows, then size the sample (whole output rows) to the budget
    t = cpu_loop_seconds(dec, cal, alpha, threads)
    per_row = t / cal
    rows = max(cal, min(M, int(budget_s / per_row) // threads * threads))
    vA, sA = O.decode_operand(A[:rows * K // 2], SFA, rows, K)
    dec = (vA, sA, dec[2], dec[3])
    t = cpu_loop_seconds(dec, rows, alpha, threads)
    tflops = 2.0 * rows * N * K / t / 1e12
    out = {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
           "sample": f"{rows} full output rows x N={N} x K={K} of the host reference loop in the "
                     f"example's form (example/nvfp4_bf16_gemm.cu:159-168: a = vA*sA, "
                     f"b = vB*sB, acc += a*b, values and scales decoded before the loop), "
                     f"{threads} threads, {t:.1f} s; TFLOP/s = 2*rows*N*K/t"}
    if gpu_rows is not None:
        out["parity_vs_gpu"] = cpu_parity(A, SFA, B, SFB, N, K, alpha, gpu_rows, threads)
    return out


def reference_arm(args, world, rank):
    """--impl reference: the reference's host GEMM loop on the host cores, rank 0 only.  Each
    step is the loop on 4 full output rows per thread (all N columns, all K): the same loop,
    form and sample shape as this bench's cpu_baseline leg, with the operands decoded once
    before the timed steps as the example does before its loop."""
    import numpy as np
    from oracle import oracle as O

    if rank != 0:
        return None
    M, N, K = args.m, args.n, args.k
    threads = os.cpu_count() or 1
    # Inputs: the same recipe on the host (seeded): the rows a step touches.
    xa = O.gen_normal(1, 4 * threads * K).reshape(4 * threads, K)
    xb = O.gen_normal(2, N * K).reshape(N, K)
    A, SFA, ga = O.quantize(xa)
    B, SFB, gb = O.quantize(xb)
    del xa, xb
    alpha = float(np.float32(ga) * np.float32(gb))
    dec = decoded_operands(A, SFA, B, SFB, 4 * threads, N, K)
    # per-step sample: 4 rows per thread x N columns x K (several rows per thread, as in the
    # cpu_baseline leg's sample), fewer if the run would be long
    rows = 4 * threads
    t_one = cpu_loop_seconds(dec, rows, alpha, threads)
    total_steps = args.steps + args.warmup
    budget = 150.0
    if t_one * total_steps > budget:
        rows = max(1, int(rows * budget / (t_one * total_steps)))
    for _ in range(args.warmup):
        cpu_loop_seconds(dec, rows, alpha, threads)
    times = []
    for _ in range(args.steps):
        times.append(cpu_loop_seconds(dec, rows, alpha, threads))
    t = sum(times)
    flops = 2.0 * rows * N * K * args.steps
    v = flops / t / 1e12
    sample = (f"{rows} full output rows x N={N} x K={K} per step of the host reference loop in "
              f"the example's form (example/nvfp4_bf16_gemm.cu:159-168), {threads} threads; "
              f"operands decoded once before the steps, as the example builds refA / sfaVal "
              f"before its loop")
    return {
        "metric": "NVFP4 GEMM TFLOPS @8192^3 (% FP4 peak); M=16 decode GEMM HBM GB/s",
        "impl": "reference", "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": {"workload": f"nvfp4 gemm M={M} N={N} K={K} (sampled on CPU)"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def library_baseline(M, N, K, sets, steps, warmup, world):
    """The same GEMM through NVIDIA's library (cuBLASLt block-scaled NVFP4 kernel, reached via
    torch._scaled_mm) on the same operands, timed the same way: a comparison, not our path.
    The 128x4 scale-factor layout of this library is the one cuBLASLt expects."""
    import torch

    def launch(A, SFA, B, SFB, alpha):
        torch._scaled_mm(A.view(torch.float4_e2m1fn_x2).view(M, K // 2),
                         B.view(torch.float4_e2m1fn_x2).view(N, K // 2).t(),
                         SFA.view(torch.float8_e4m3fn), SFB.view(torch.float8_e4m3fn),
                         out_dtype=torch.bfloat16)

    for i in range(warmup):
        launch(*sets[i % len(sets)])
    barrier(world)
    time.sleep(1.0)  # let the power limiter settle as before our own timed region
    with ClockSampler(torch.cuda.current_device(), enabled=not dist_rank()) as clk:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(steps):
            launch(*sets[i % len(sets)])
        e.record()
        barrier(world)
    ms = max_over_ranks(s.elapsed_time(e) / steps, world)
    return {"impl": "cuBLASLt NVFP4 block-scaled GEMM via torch._scaled_mm (comparison only)",
            "tflops": 2.0 * M * N * K * world / (ms * 1e-3) / 1e12, "ms_per_step": ms,
            "steps": steps, "clocks": clk.summary()}


def run_compare(args, dev, M, N, K):
    """--case compare: this library's GEMM and cuBLASLt's block-scaled NVFP4 GEMM
    (torch._scaled_mm) alternating on the same operands, `warmup` + `steps` launches of each,
    one event pair per launch; for profiler captures of the two kernels side by side."""
    import torch
    import blackhole_b200 as bh

    A, SFA, sa = make_operand(M, K, 1, 1.0, dev)
    B, SFB, sb = make_operand(N, K, 1000, 1.0, dev)
    alpha = float(sa[1].item() * sb[1].item())
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

    def lib():
        return torch._scaled_mm(A.view(torch.float4_e2m1fn_x2).view(M, K // 2),
                                B.view(torch.float4_e2m1fn_x2).view(N, K // 2).t(),
                                SFA.view(torch.float8_e4m3fn), SFB.view(torch.float8_e4m3fn),
                                out_dtype=torch.bfloat16)

    times = {"ours": [], "cublaslt": []}
    for i in range(args.warmup + args.steps):
        for name, fn in (("ours", lambda: bh.nvfp4_bf16_gemm(M, N, K, A, SFA, B, SFB, D, alpha)),
                         ("cublaslt", lib)):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            if i >= args.warmup:
                times[name].append((s, e))
    torch.cuda.synchronize()
    assert bh.device_status(torch.cuda.current_device()) == 0
    us = {k: [round(s.elapsed_time(e) * 1e3, 1) for s, e in v] for k, v in times.items()}
    return {"case": "compare", "shape": [M, N, K], "us_per_launch": us,
            "gpu_launches": args.warmup + args.steps}


# Decode legs warm up with ~0.1 s of decode launches: measured on B200, a decode timed right
# after the power-capped GEMM legs with 20 warm-up launches ran at 30-33 us instead of its
# steady 25 us (the clocks recover over tens of milliseconds), i.e. it timed the previous
# leg's state, not the decode's.  (--decode-warmup, default 4000.)


def run_decode(args, dev, rank, world, hbm_peak, peak_src, Ms=(16, 1, 64, 128)):
    """M x 28672 x 8192 decode GEMMs over 3 rotating weight sets (396 MB), back to
    back.  Returns the M=16 line plus a per-M sweep."""
    import torch

    Nd, Kd = 28672, 8192
    bsets = []
    for i in range(3):
        Bd, SFBd, scBd = make_operand(Nd, Kd, 2000 + rank + 7 * i, 0.02, dev)
        bsets.append((Bd, SFBd, float(scBd[1].item())))
    out, sweep = None, {}
    for Md in Ms:
        dsets = []
        for i in range(3):
            Ad, SFAd, scAd = make_operand(Md, Kd, 2 + 7 * i, 1.0, dev)
            Bd, SFBd, gB = bsets[i]
            dsets.append((Ad, SFAd, Bd, SFBd, float(scAd[1].item()) * gB))
        Dd = torch.empty((Md, Nd), dtype=torch.bfloat16, device=dev)
        dsteps = max(30, args.steps)
        dtot = time_gemm(Md, Nd, Kd, dsets, Dd, dsteps, max(args.warmup, args.decode_warmup), world)
        dms = max_over_ranks(dtot / dsteps, world)
        nbytes = gemm_bytes(Md, Nd, Kd)
        gbs = nbytes / (dms * 1e-3) / 1e9
        line = {"workload": f"M={Md} N={Nd} K={Kd} (BASELINE configs[2]) per GPU",
                "value": gbs * world, "unit": "GB/s", "ms_per_step": dms,
                "bytes_per_launch": nbytes, "roofline_frac": gbs / hbm_peak,
                "peak": hbm_peak, "peak_source": peak_src,
                "frac_of_spec_8tbs": gbs / SPEC_HBM_GBS, "steps": dsteps,
                "l2": "3 rotating weight sets (396 MB > 126 MB L2), back to back",
                "warmup_launches": max(args.warmup, args.decode_warmup),
                "host_enqueue_us_per_launch": time_gemm.host_us_per_launch,
                "traffic": profiled_traffic(f"gemm_{Md}x{Nd}x{Kd}")}
        if Md == 16:
            out = line
        sweep[str(Md)] = {k: line[k] for k in ("value", "ms_per_step", "roofline_frac",
                                                "frac_of_spec_8tbs")}
        del dsets, Dd
    out = dict(out or line)
    out["sweep_by_M"] = sweep
    return out


def run_mx(args, dev, rank, world, fp4_peak, hbm_peak, fmt="mxfp4"):
    """A sibling format on configs[1]'s and configs[2]'s M=16 shapes, same sources (N(0,1);
    decode weights N(0, 0.02^2)), quantised on the device: "mxfp4" (UE8M0 scale per 32) or
    "mxf8f4" (MXFP8 activations x MXFP4 weights; kind::mxf8f6f4, half the FP4 MMA rate)."""
    import torch
    import blackhole_b200 as bh

    def mx_operand(rows, K, seed, std, fp8=False):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        x = torch.randn((rows, K), generator=g, device=dev, dtype=torch.float32)
        if std != 1.0:
            x.mul_(std)
        q, sf = bh.quantize_tensor_mxfp8(x) if fp8 else bh.quantize_tensor_mxfp4(x)
        torch.cuda.synchronize()
        return q, sf

    a8 = fmt == "mxf8f4"
    peak = fp4_peak / 2 if a8 else fp4_peak
    out = {}
    M = N = K = 8192
    sets = [mx_operand(M, K, 1 + 7 * i, 1.0, a8) + mx_operand(N, K, 1000 + rank + 7 * i, 1.0) + (1.0,)
            for i in range(4)]
    set_mb = sum(t.numel() for t in sets[0][:4]) / 1e6
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    steps = max(10, min(args.steps, 400))
    tot = time_gemm(M, N, K, sets, D, steps, max(3, args.warmup), world, fmt=fmt)
    ms = max_over_ranks(tot / steps, world)
    tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    out["gemm_8192"] = {"value": tf * world, "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps,
                        "roofline_frac": tf / peak, "peak": peak,
                        "l2": f"4 rotating input sets ({set_mb * 4:.0f} MB > 126 MB L2), back to back"}
    del sets, D
    Md, Nd, Kd = 16, 28672, 8192
    dsets = [mx_operand(Md, Kd, 2 + 7 * i, 1.0, a8) + mx_operand(Nd, Kd, 2000 + rank + 7 * i, 0.02) + (1.0,)
             for i in range(3)]
    Dd = torch.empty((Md, Nd), dtype=torch.bfloat16, device=dev)
    dsteps = max(30, min(args.steps, 2000))
    tot = time_gemm(Md, Nd, Kd, dsets, Dd, dsteps, max(args.warmup, args.decode_warmup), world, fmt=fmt)
    dms = max_over_ranks(tot / dsteps, world)
    a_bytes = Md * Kd if a8 else Md * Kd // 2   # MXFP8: one byte per element
    nbytes = a_bytes + Nd * Kd // 2 + (Md + Nd) * Kd // 32 + 2 * Md * Nd
    gbs = nbytes / (dms * 1e-3) / 1e9
    out["decode_m16"] = {"value": gbs * world, "unit": "GB/s", "ms_per_step": dms, "steps": dsteps,
                         "bytes_per_launch": nbytes, "roofline_frac": gbs / hbm_peak,
                         "l2": "3 rotating weight sets (~380 MB > 126 MB L2), back to back"}
    del dsets, Dd
    out["steps"] = steps + dsteps
    return out


def run_quantize(args, dev, world, hbm_peak, rows=28672, K=8192):
    """The NVFP4 quantiser (the step before the GEMM) on configs[2]'s weight shape, FP32 input
    (940 MB > L2), calls back to back.  One call is two HBM passes over X -- the tensor amax,
    then the quantiser proper -- so its minimal traffic is 2 reads of X plus the codes and
    scale factors written; `frac` is that traffic's rate over the measured HBM peak."""
    import torch
    import blackhole_b200 as bh

    g = torch.Generator(device=dev)
    g.manual_seed(99)
    x = torch.randn((rows, K), generator=g, device=dev, dtype=torch.float32)
    packed = torch.empty((rows, K // 2), dtype=torch.uint8, device=dev)
    sf = torch.empty(bh.sf_storage_bytes(rows, K), dtype=torch.uint8, device=dev)
    scales = torch.empty(2, dtype=torch.float32, device=dev)
    steps = max(5, min(args.steps, 50))
    for _ in range(3):
        bh.nvfp4_quantize(x, rows, K, packed, sf, scales)
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        bh.nvfp4_quantize(x, rows, K, packed, sf, scales)
    e.record()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e) / steps, world)
    read = rows * K * 4
    written = rows * K // 2 + sf_bytes(rows, K)
    traffic = 2 * read + written
    del x, packed, sf, scales
    return {"workload": f"{rows} x {K} FP32 -> NVFP4 (packed E2M1 + UE4M3 128x4 scale factors)",
            "ms_per_call": ms, "steps": steps,
            "gbs_two_pass": traffic / (ms * 1e-3) / 1e9, "frac": traffic / (ms * 1e-3) / 1e9 / hbm_peak,
            "bytes_per_call": {"read_x_twice": 2 * read, "written": written},
            "gbs_one_read": (read + written) / (ms * 1e-3) / 1e9,
            "launches_per_call": 2, "peak": hbm_peak}


def run_prefill(args, dev, rank, world, fp4_peak):
    """M=16384 N=8192 K=28672, A from N(0,1) with 1% of entries x20, B from
    N(0, 0.02^2); 2 rotating input sets (~800 MB), back to back."""
    import torch

    M, N, K = 16384, 8192, 28672
    sets = []
    for i in range(2):
        A, SFA, sa = make_operand(M, K, 3 + 7 * i, 1.0, dev, outlier_p=0.01)
        B, SFB, sb = make_operand(N, K, 3000 + rank + 7 * i, 0.02, dev)
        sets.append((A, SFA, B, SFB, float(sa[1].item() * sb[1].item())))
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    steps = max(5, min(args.steps, 40))
    tot = time_gemm(M, N, K, sets, D, steps, max(3, min(args.warmup, 5)), world)
    ms = max_over_ranks(tot / steps, world)
    tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    del sets, D
    return {"workload": f"M={M} N={N} K={K}, A with 1% outliers x20 (BASELINE configs[3]) per GPU",
            "value": tf * world, "unit": "TFLOP/s", "ms_per_step": ms, "steps": steps,
            "roofline_frac": tf / fp4_peak, "l2": "2 rotating input sets (~800 MB), back to back"}


NVLINK_GBS = 770.0   # measured peer copy on this pool's B200s, GB/s per direction per GPU


def all_gather_objects(obj, world):
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def gathered_parity(M, N, K, A, SFA, B, SFB, alpha, rank, world, row0, buf, S=1024,
                    own_slice=False):
    """Checks S sampled elements of this rank's gathered row-major M x N buffer against the
    oracle.  Every rank draws the same sample points; each computes the oracle at the points in
    its own N-slice (the only slice of B it holds), the ranks exchange those values, and every
    rank compares its buffer (tiles written by every rank) with the whole set.  With
    own_slice=True, buf is this rank's M x N/P slice and only the points inside it are checked
    (no exchange)."""
    import numpy as np
    import torch
    from oracle import oracle as O

    rows = B.shape[0] if B.dim() == 2 else B.numel() * 2 // K
    rng = np.random.default_rng(77)
    ms = rng.integers(0, M, S)
    ns = rng.integers(0, N, S)
    mine = np.nonzero((ns >= row0) & (ns < row0 + rows))[0]
    hA, hSFA, hB, hSFB = (t.cpu().numpy().reshape(-1) for t in (A, SFA, B, SFB))
    threads = max(1, (os.cpu_count() or 1) // world)
    ref, ad = O.gemm_sampled(M, rows, K, hA, hSFA, hB, hSFB, ms[mine], ns[mine] - row0, alpha,
                             nthreads=threads)
    dev = buf.device
    if own_slice:
        tm = torch.from_numpy(ms[mine]).to(dev)
        tn = torch.from_numpy(ns[mine] - row0).to(dev)
        got = buf[tm, tn].view(torch.int16).cpu().numpy().view(np.uint16)
        r = O.check_report(ref, got, alpha, K, ad)
        r["sample"] = f"the points of {S} random elements of M x N that fall in each rank's slice"
        return r
    # each slice has its own alpha (its B was quantised with its own global scale)
    parts = all_gather_objects((mine, ref, ad, alpha), world)
    full_ref = np.zeros(S, dtype=np.uint16)
    full_ad = np.zeros(S, dtype=np.float64)
    full_alpha = np.zeros(S, dtype=np.float64)
    for idx, r, a, al in parts:
        full_ref[idx] = r
        full_ad[idx] = a
        full_alpha[idx] = al
    got = buf[torch.from_numpy(ms).to(dev), torch.from_numpy(ns).to(dev)]
    got = got.view(torch.int16).cpu().numpy().view(np.uint16)
    r = O.check_report(full_ref, got, full_alpha, K, full_ad)
    r["sample"] = f"{S} random elements of the whole gathered M x N buffer, on every rank"
    return r


def run_nsplit(args, dev, rank, world, fp4_peak):
    """M=32768, N=65536 split evenly over the P ranks, K=8192, seed 4; A replicated.
    Strong scaling (the whole GEMM is fixed).  At P > 1 also (unless --no-gather) the NCCL
    all-gather of the C slices after the GEMM, and the gather fused into the GEMM (every rank
    ends with the row-major M x N result), each with its parity against the oracle."""
    import torch
    import torch.distributed as dist
    from blackhole_b200.nsplit import shard

    M, N, K = 32768, 65536, 8192
    sh = shard(N, K, rank, world)
    A, SFA, sa = make_operand(M, K, 4, 1.0, dev)
    B, SFB, sb = make_operand(sh.rows, K, 4000 + rank, 1.0, dev)  # this rank's rows of B
    alpha = float(sa[1].item() * sb[1].item())
    D = torch.empty((M, sh.rows), dtype=torch.bfloat16, device=dev)
    steps = max(3, min(args.steps, 10))
    tot = time_gemm(M, sh.rows, K, [(A, SFA, B, SFB, alpha)], D, steps, 2, world)
    ms = max_over_ranks(tot / steps, world)
    flops = 2.0 * M * N * K
    out = {"workload": f"M={M} N={N} K={K} split along N over {world} GPU(s) (BASELINE configs[4])",
           "unit": "TFLOP/s", "scaling": "strong", "n_gpus": world,
           "ms_per_step": ms, "value": flops / (ms * 1e-3) / 1e12,
           "roofline_frac": flops / world / (ms * 1e-3) / 1e12 / fp4_peak, "steps": steps}
    # parity of every rank's slice (the plain GEMM) at the same sample points as the gathered
    # buffer below: the slice's own columns, checked on each rank
    par = gathered_parity(M, N, K, A, SFA, B, SFB, alpha, rank, world, sh.row0, D, own_slice=True)
    out["parity_slices"] = _merge_parity(all_gather_objects(par, world))
    if world > 1 and not args.no_gather:
        g = torch.empty((world, M, sh.rows), dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(g, D)
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(3):
            dist.all_gather_into_tensor(g, D)
        e.record()
        barrier(world)
        gms = max_over_ranks(s.elapsed_time(e) / 3, world)
        nbytes_in = (world - 1) * M * sh.rows * 2
        out["gather"] = {"ms_per_step": gms, "layout": "[P][M][N/P] bf16",
                         "bytes_per_gpu_in": nbytes_in,
                         "nvlink_gbs_per_gpu": nbytes_in / (gms * 1e-3) / 1e9,
                         "with_gather_ms_per_step": ms + gms,
                         "with_gather_tflops": flops / ((ms + gms) * 1e-3) / 1e12}
        del g
        # the gather fused into the GEMM: each rank's epilogue stores its tiles into every
        # rank's row-major M x N buffer (CUDA IPC mappings, two buffers alternating by step)
        # while it computes the next tiles; the flag barrier over NVLink ends each step
        import blackhole_b200 as bh
        from blackhole_b200.nsplit import GatheredOutput

        go = GatheredOutput(M, N, rank, world)

        def fused():
            bh.nvfp4_bf16_gemm_gather(M, sh.rows, K, A, SFA, B, SFB, go.dst_c, sh.row0, N, alpha)
            go.barrier()

        for _ in range(2):
            fused()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fused()
        e.record()
        barrier(world)
        fms = max_over_ranks(s.elapsed_time(e) / steps, world)
        assert bh.device_status(torch.cuda.current_device()) == 0
        nbytes_out = (world - 1) * M * sh.rows * 2
        t_link = nbytes_out / (NVLINK_GBS * 1e9) * 1e3
        t_math = flops / world / (fp4_peak * 1e12) * 1e3
        bound = max(t_link, t_math)
        out["fused_gather"] = {
            "ms_per_step": fms, "tflops": flops / (fms * 1e-3) / 1e12,
            "layout": "row-major M x N on every GPU",
            "nvlink_bytes_out_per_gpu": nbytes_out,
            "nvlink_gbs_per_gpu": nbytes_out / (fms * 1e-3) / 1e9,
            "roofline": {"bound_ms": bound, "limiter": "nvlink" if t_link > t_math else "tensor",
                         "nvlink_ms_at_770_gbs": t_link, "tensor_ms_at_fp4_peak": t_math,
                         "frac": bound / fms},
            "speedup_vs_gemm_then_nccl": (ms + gms) / fms, "steps": steps,
            "parity": _merge_parity(all_gather_objects(
                gathered_parity(M, N, K, A, SFA, B, SFB, alpha, rank, world, sh.row0, go.out),
                world))}
        out["steps"] += steps + 2
        go.close()
        del go
    del A, SFA, B, SFB, D
    if world > 1 and not args.no_gather:
        out["decode_gather"] = run_decode_gather(dev, rank, world)
        out["steps"] += out["decode_gather"]["steps"]
    return out


def _merge_parity(reports):
    """One record from the ranks' parity reports."""
    n = sum(r["elements"] for r in reports)
    return {"elements": n, "mismatches": sum(r["mismatches"] for r in reports),
            "bit_identical_frac": sum(r["bit_identical_frac"] * r["elements"] for r in reports) / max(n, 1),
            "max_err_over_tol": max(r["max_err_over_tol"] for r in reports),
            "max_err_over_worst_case_bound": max(r["max_err_over_worst_case_bound"] for r in reports),
            "ranks": len(reports), "sample": reports[0].get("sample", "")}


def run_decode_gather(dev, rank, world, steps=50):
    """Tensor-parallel decode: configs[2]'s M=16, K=8192 GEMM with the N=28672 weights split
    over the ranks and the output all-gathered, per step either GEMM + NCCL all-gather
    ([P][M][N/P]) or the gather fused into the skinny GEMM + the flag barrier over NVLink that
    ends each step (row-major M x N on every GPU, two buffers alternating by step so that a
    step never writes the buffer a slower rank may still read)."""
    import torch
    import torch.distributed as dist
    import blackhole_b200 as bh
    from blackhole_b200.nsplit import GatheredOutput, shard

    M, N, K = 16, 28672, 8192
    sh = shard(N, K, rank, world)
    A, SFA, sa = make_operand(M, K, 2, 1.0, dev)
    B, SFB, sb = make_operand(sh.rows, K, 2000 + rank, 0.02, dev)
    alpha = float(sa[1].item() * sb[1].item())
    D = torch.empty((M, sh.rows), dtype=torch.bfloat16, device=dev)
    g = torch.empty((world, M, sh.rows), dtype=torch.bfloat16, device=dev)
    go = GatheredOutput(M, N, rank, world)

    def nccl_step():
        bh.nvfp4_bf16_gemm(M, sh.rows, K, A, SFA, B, SFB, D, alpha)
        dist.all_gather_into_tensor(g, D)

    def fused_step():
        bh.nvfp4_bf16_gemm_gather(M, sh.rows, K, A, SFA, B, SFB, go.dst_c, sh.row0, N, alpha)
        go.barrier()

    res = {}
    for name, step in (("gemm_then_nccl", nccl_step), ("fused", fused_step)):
        for _ in range(5):
            step()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            step()
        e.record()
        barrier(world)
        res[name] = max_over_ranks(s.elapsed_time(e) / steps, world) * 1e3
    assert bh.device_status(torch.cuda.current_device()) == 0
    parity = _merge_parity(all_gather_objects(
        gathered_parity(M, N, K, A, SFA, B, SFB, alpha, rank, world, sh.row0, go.out), world))
    go.close()
    del A, SFA, B, SFB, D, g, go
    return {"workload": f"M={M} N={N} K={K}, N split over {world} GPUs, output all-gathered",
            "us_per_step_gemm_then_nccl": res["gemm_then_nccl"], "us_per_step_fused": res["fused"],
            "speedup": res["gemm_then_nccl"] / res["fused"], "steps": 2 * steps,
            "parity": parity,
            "note": "each step includes its cross-GPU synchronisation (the all-gather, or the "
                    "fused path's flag barrier)"}


# ---------------------------------------------------------------------------------------
def main():
    args = parse()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        out = reference_arm(args, world, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    import torch
    import blackhole_b200 as bh

    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", torch.cuda.current_device())
    hbm_peak, bf16_peak, peak_src = measured_peaks()
    fp4_peak = 4.0 * bf16_peak
    M, N, K = args.m, args.n, args.k
    if args.case == "decode":
        with ClockSampler(torch.cuda.current_device(), enabled=rank == 0) as clk:
            d = run_decode(args, dev, rank, world, hbm_peak, peak_src)
        assert bh.device_status(torch.cuda.current_device()) == 0
        if rank == 0:
            print(json.dumps({"case": "decode", "decode": d,
                              "gpu_launches": d["steps"] * len(d["sweep_by_M"]),
                              "clocks": clk.summary()}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == "quantize":
        q = run_quantize(args, dev, world, hbm_peak)
        if rank == 0:
            print(json.dumps({"case": "quantize", "quantize": q,
                              "gpu_launches": 2 * (q["steps"] + 3)}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == "compare":
        print(json.dumps(run_compare(args, dev, M, N, K)), flush=True)
        return
    if args.case == "main":
        args.no_decode = True
        args.no_configs = True

    ROT = 4
    sets = []
    for i in range(ROT):
        A_, SFA_, scA_ = make_operand(M, K, 1 + 7 * i, 1.0, dev)            # A replicated
        B_, SFB_, scB_ = make_operand(N, K, 1000 + rank + 7 * i, 1.0, dev)  # this rank's N slice
        sets.append((A_, SFA_, B_, SFB_, float(scA_[1].item() * scB_[1].item())))
    A, SFA, B, SFB, alpha = sets[0]
    D = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)

    clk = ClockSampler(torch.cuda.current_device(), enabled=rank == 0)
    total_ms = time_gemm(M, N, K, sets, D, args.steps, args.warmup, world, args.schedule, clk=clk)
    fsteps = min(args.steps, 20)
    ftimes = time_gemm_flushed(M, N, K, A, SFA, B, SFB, D, alpha, fsteps, flush, world)
    assert bh.device_status(torch.cuda.current_device()) == 0
    # D now holds the GEMM of input set 0: its first 128 rows go to the CPU leg's parity check
    check_rows = D[:min(M, 128)].view(torch.int16).cpu().numpy().view("uint16")
    total_ms = max_over_ranks(total_ms, world)
    ms_step = total_ms / args.steps
    flops_rank = 2.0 * M * N * K
    value = flops_rank * world * args.steps / (total_ms * 1e-3) / 1e12
    achieved = flops_rank / (ms_step * 1e-3) / 1e12
    fms = max_over_ranks(statistics.mean(ftimes), world)
    in_bytes = ROT * (M * K // 2 + N * K // 2 + sf_bytes(M, K) + sf_bytes(N, K))

    result = {
        "metric": "NVFP4 GEMM TFLOPS @8192^3 (% FP4 peak); M=16 decode GEMM HBM GB/s",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4",
        "data": "synthetic: N(0,1) via seeded torch.randn on device, NVFP4-quantised on device",
        "config": {"workload": f"nvfp4 gemm M={M} N={N}/gpu K={K} (BASELINE configs[1]; N-split "
                               f"across {world} GPU(s), A replicated)",
                   "M": M, "N_per_gpu": N, "N_total": N * world, "K": K,
                   "parallelism": f"n-split{world}", "schedule": args.schedule,
                   "l2": f"inputs larger than L2: {ROT} rotating input sets "
                         f"({in_bytes / 1e6:.0f} MB > 126 MB L2), launched back to back, no flush"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s",
                     "frac": achieved / fp4_peak,
                     "peak_source": f"4 x {peak_src} dense bf16 ({bf16_peak} TF/s); FP4 dense = 4x BF16 per SM-clock",
                     "frac_of_spec_9pf": achieved / SPEC_FP4_TFLOPS,
                     "traffic": profiled_traffic(f"gemm_{M}x{N}x{K}")},
        "per_launch_l2_flush": {"tflops": flops_rank / (fms * 1e-3) / 1e12, "ms": fms, "steps": fsteps,
                                "method": "256 MB write before each launch, one event pair per launch "
                                          "(includes ~5-7 us of event/launch overhead per launch)"},
        "gpu_launches": args.steps + fsteps,
    }

    if not args.no_decode:
        result["decode"] = run_decode(args, dev, rank, world, hbm_peak, peak_src)
        result["gpu_launches"] += result["decode"]["steps"] * len(result["decode"]["sweep_by_M"])

    if not args.no_configs:
        result["quantize"] = run_quantize(args, dev, world, hbm_peak)
        result["gpu_launches"] += 2 * result["quantize"]["steps"]
        result["prefill"] = run_prefill(args, dev, rank, world, fp4_peak)
        result["nsplit"] = run_nsplit(args, dev, rank, world, fp4_peak)
        result["gpu_launches"] += result["prefill"]["steps"] + result["nsplit"]["steps"]
        result["mxfp4"] = run_mx(args, dev, rank, world, fp4_peak, hbm_peak, "mxfp4")
        result["gpu_launches"] += result["mxfp4"]["steps"]
        result["mxf8f4"] = run_mx(args, dev, rank, world, fp4_peak, hbm_peak, "mxf8f4")
        result["gpu_launches"] += result["mxf8f4"]["steps"]

    if world > 1 and not args.no_gather:
        import torch.distributed as dist
        out = torch.empty((world, M, N), dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            dist.all_gather_into_tensor(out, D)
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(10):
            dist.all_gather_into_tensor(out, D)
        e.record()
        barrier(world)
        gms = max_over_ranks(s.elapsed_time(e) / 10, world)
        nbytes_in = (world - 1) * M * N * 2
        result["gather"] = {"ms_per_step": gms, "layout": "[P][M][N/P] bf16",
                            "bytes_per_gpu_in": nbytes_in,
                            "nvlink_gbs_per_gpu": nbytes_in / (gms * 1e-3) / 1e9,
                            "with_gather_tflops": flops_rank * world / ((ms_step + gms) * 1e-3) / 1e12}
        del out

    if not args.no_e2e:
        esteps = max(3, min(args.steps, 20))
        ems, h2d, d2h = run_e2e(M, N, K, A, SFA, B, SFB, alpha, esteps, world)
        ems = max_over_ranks(ems, world)
        result["e2e"] = {"value": flops_rank * world / (ems * 1e-3) / 1e12, "unit": "TFLOP/s",
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "ms_per_step": ems, "steps": esteps,
                         "path": "blackhole_sm100_nvfp4_bf16_gemm (C ABI) + pinned host copies, "
                                 "steps pipelined over upload / compute / download streams",
                         # the ceiling: every step moves its inputs and its 134 MB result over
                         # PCIe and through host memory, shared by all GPUs of the node
                         "host_link": {"h2d_gbs_per_gpu": h2d / (ems * 1e-3) / 1e9,
                                       "d2h_gbs_per_gpu": d2h / (ems * 1e-3) / 1e9,
                                       "d2h_gbs_all_gpus": world * d2h / (ems * 1e-3) / 1e9,
                                       "h2d_gbs_all_gpus": world * h2d / (ems * 1e-3) / 1e9,
                                       "gemm_share_of_step": ms_step / ems,
                                       "limiter": "host copies (PCIe / host memory), not the GEMM"}}
        result["gpu_launches"] += esteps

    result["clocks"] = clk.summary()

    # last, so that it cannot disturb our own legs (the GPU is left hot and power capped)
    if not args.no_library:
        try:
            lib = library_baseline(M, N, K, sets, args.steps, args.warmup, world)
            lib["ours_over_library"] = value / lib["tflops"]
            result["library_baseline"] = lib
        except Exception as exc:  # an older torch without FP4 _scaled_mm
            result["library_baseline"] = {"unavailable": repr(exc)[:200]}

    hA = A.cpu().numpy().reshape(-1)
    hSFA = SFA.cpu().numpy()
    hB = B.cpu().numpy().reshape(-1)
    hSFB = SFB.cpu().numpy()
    # every rank checks the first 16 full rows of its own timed output (input set 0) against
    # the oracle; rank 0 reports each rank's record
    threads = max(1, (os.cpu_count() or 1) // world)
    par = cpu_parity(hA, hSFA, hB, hSFB, N, K, alpha, check_rows[:16], threads)
    par["rank"] = rank
    per_rank = all_gather_objects(par, world)
    result["parity"] = dict(_merge_parity(per_rank),
                            sample="first 16 full output rows of every rank's timed GEMM "
                                   "(input set 0) against the host reference",
                            per_rank=[{k: r[k] for k in ("rank", "elements", "mismatches",
                                                         "bit_identical_frac", "max_err_over_tol")}
                                      for r in per_rank])

    if rank == 0 and world == 1 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(hA, hSFA, hB, hSFB, N, K, alpha, M,
                                              gpu_rows=check_rows)

    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
