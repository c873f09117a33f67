"""The bench's CPU leg on the host alone: its timing sample and the parity check it runs
against a GPU output (here stood in for by the oracle's own result, with one element
altered on the CPU to show that a wrong value is counted)."""
import numpy as np

import bench
from oracle import oracle as O


def _operands(M, N, K):
    xa = O.gen_normal(11, M * K).reshape(M, K)
    xb = O.gen_normal(12, N * K, std=0.02).reshape(N, K)
    A, SFA, ga = O.quantize(xa)
    B, SFB, gb = O.quantize(xb)
    return A, SFA, B, SFB, float(np.float32(ga) * np.float32(gb))


def test_cpu_leg_reports_parity_of_matching_rows():
    M, N, K = 256, 384, 512
    A, SFA, B, SFB, alpha = _operands(M, N, K)
    ref, _ = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    out = bench.cpu_baseline(A, SFA, B, SFB, N, K, alpha, M, budget_s=0.2,
                             gpu_rows=ref[:128].copy())
    assert out["kind"] == "port" and out["cores"] >= 1 and out["value"] > 0
    par = out["parity_vs_gpu"]
    assert par["rows"] == 128 and par["elements"] == 128 * N
    assert par["mismatches"] == 0 and par["bit_identical_frac"] == 1.0
    assert par["max_err_over_tol"] == 0.0


def test_cpu_parity_counts_a_wrong_element():
    M, N, K = 128, 256, 512
    A, SFA, B, SFB, alpha = _operands(M, N, K)
    ref, _ = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
    rows = ref.copy()
    rows[7, 9] ^= np.uint16(0x0100)   # two exponent steps off
    par = bench.cpu_parity(A, SFA, B, SFB, N, K, alpha, rows, 2)
    assert par["mismatches"] == 1
    assert par["max_err_over_tol"] > 1.0
    assert par["bit_identical_frac"] == 1.0 - 1.0 / (M * N)
