"""Shared helpers for the NVFP4 GEMM tests: seeded operands made by the oracle's generator
and quantiser (host), the CUDA path run through the C ABI, and the tolerance check."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O


def make_operands(M, N, K, seed=0, std_a=1.0, std_b=1.0, outlier_p=0.0, outlier_x=20.0):
    """Quantised A (M x K) and B (N x K) following the BASELINE recipe."""
    xa = O.gen_normal(seed, M * K, 0.0, std_a).reshape(M, K)
    if outlier_p > 0:
        O.apply_outliers(seed, xa.reshape(-1), outlier_p, outlier_x)
    xb = O.gen_normal(seed + 1000003, N * K, 0.0, std_b).reshape(N, K)
    A, SFA, ga = O.quantize(xa)
    B, SFB, gb = O.quantize(xb)
    alpha = float(np.float32(ga) * np.float32(gb))
    return A, SFA, B, SFB, alpha


def run_gpu(M, N, K, A, SFA, B, SFB, alpha, repeat=1, schedule="auto", workspace=None):
    """Runs the CUDA GEMM through the C ABI; returns D as uint16 bf16 bits [M, N]."""
    import torch
    import blackhole_b200 as bh

    dev = torch.device("cuda:0")
    tA = torch.from_numpy(A).to(dev)
    tB = torch.from_numpy(B).to(dev)
    tSFA = torch.from_numpy(SFA).to(dev)
    tSFB = torch.from_numpy(SFB).to(dev)
    D = torch.full((M, N), -1, dtype=torch.int16, device=dev)  # NaN pattern: catches unwritten
    outs = []
    for _ in range(repeat):
        if schedule == "auto" and workspace is None:
            bh.nvfp4_bf16_gemm(M, N, K, tA, tSFA, tB, tSFB, D, alpha)
        else:
            bh.nvfp4_bf16_gemm_ex(M, N, K, tA, tSFA, tB, tSFB, D, alpha, schedule=schedule,
                                  workspace=workspace)
        torch.cuda.synchronize()
        outs.append(D.cpu().numpy().view(np.uint16).copy())
    assert bh.device_status(0) == 0
    return outs if repeat > 1 else outs[0]


def check_full(M, N, K, A, SFA, B, SFB, alpha, got):
    ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    return O.check(ref, got, alpha, K, ad), ref


def check_sampled(M, N, K, A, SFA, B, SFB, alpha, got, S=4096, seed=7, record=True):
    rng = np.random.default_rng(seed)
    ms = rng.integers(0, M, S)
    ns = rng.integers(0, N, S)
    # always include the corners of the output
    ms[:4] = [0, 0, M - 1, M - 1]
    ns[:4] = [0, N - 1, 0, N - 1]
    ref, ad = O.gemm_sampled(M, N, K, A, SFA, B, SFB, ms, ns, alpha)
    return O.check(ref, got[ms, ns], alpha, K, ad, record=record)
