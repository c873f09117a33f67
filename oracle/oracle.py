"""Python access to the CPU oracle (oracle/liboracle.so) -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path.  Only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference leg import it; the shipped package (blackhole_b200)
never does.  The C code it wraps restates the reference's host path
(example/nvfp4_bf16_gemm.cu:60-71 and :161-168, include/blackhole/sm120/nvfp4_gemm.hpp:293-302);
see oracle/nvfp4_oracle.h.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_SHIM_PATH = os.path.join(HERE, "_ref", "libref_shim.so")

_lib = None
_ref = None

c_i64 = ctypes.c_int64
c_ptr = ctypes.c_void_p


def build(force: bool = False) -> None:
    """Compile liboracle.so (gcc) if it is missing or stale."""
    src = os.path.join(HERE, "nvfp4_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE, "liboracle.so"])


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        L.bho_e2m1_from_float.restype = ctypes.c_uint8
        L.bho_e2m1_from_float.argtypes = [ctypes.c_float]
        L.bho_e2m1_to_float.restype = ctypes.c_float
        L.bho_e2m1_to_float.argtypes = [ctypes.c_uint8]
        L.bho_ue4m3_from_float.restype = ctypes.c_uint8
        L.bho_ue4m3_from_float.argtypes = [ctypes.c_float]
        L.bho_ue4m3_to_float.restype = ctypes.c_float
        L.bho_ue4m3_to_float.argtypes = [ctypes.c_uint8]
        L.bho_bf16_from_float.restype = ctypes.c_uint16
        L.bho_bf16_from_float.argtypes = [ctypes.c_float]
        L.bho_sf_offset.restype = c_i64
        L.bho_sf_offset.argtypes = [c_i64, c_i64, c_i64]
        L.bho_sf_storage_bytes.restype = c_i64
        L.bho_sf_storage_bytes.argtypes = [c_i64, c_i64]
        L.bho_gen_normal.restype = None
        L.bho_gen_normal.argtypes = [ctypes.c_uint64, c_i64, c_i64, ctypes.c_float, ctypes.c_float, c_ptr]
        L.bho_apply_outliers.restype = None
        L.bho_apply_outliers.argtypes = [ctypes.c_uint64, c_i64, ctypes.c_double, ctypes.c_float, c_ptr]
        L.bho_quantize_nvfp4.restype = ctypes.c_float
        L.bho_quantize_nvfp4.argtypes = [c_ptr, c_i64, c_i64, c_ptr, c_ptr]
        L.bho_gemm_ref_full.restype = None
        L.bho_gemm_ref_full.argtypes = [c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
                                        ctypes.c_float, c_ptr, c_ptr, ctypes.c_int]
        L.bho_gemm_ref_sampled.restype = None
        L.bho_gemm_ref_sampled.argtypes = [c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
                                           ctypes.c_float, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
                                           ctypes.c_int]
        L.bho_ue8m0_to_float.restype = ctypes.c_float
        L.bho_ue8m0_to_float.argtypes = [ctypes.c_uint8]
        L.bho_sf_offset_vs.restype = c_i64
        L.bho_sf_offset_vs.argtypes = [c_i64, c_i64, c_i64, ctypes.c_int]
        L.bho_sf_storage_bytes_vs.restype = c_i64
        L.bho_sf_storage_bytes_vs.argtypes = [c_i64, c_i64, ctypes.c_int]
        L.bho_quantize_mxfp4.restype = None
        L.bho_quantize_mxfp4.argtypes = [c_ptr, c_i64, c_i64, c_ptr, c_ptr]
        L.bho_e4m3_from_float.restype = ctypes.c_uint8
        L.bho_e4m3_from_float.argtypes = [ctypes.c_float]
        L.bho_e4m3_to_float.restype = ctypes.c_float
        L.bho_e4m3_to_float.argtypes = [ctypes.c_uint8]
        L.bho_quantize_mxfp8.restype = None
        L.bho_quantize_mxfp8.argtypes = [c_ptr, c_i64, c_i64, c_ptr, c_ptr]
        L.bho_gemm_ref_full_fmt.restype = None
        L.bho_gemm_ref_full_fmt.argtypes = [ctypes.c_int, c_i64, c_i64, c_i64, c_ptr, c_ptr, c_ptr,
                                            c_ptr, ctypes.c_float, c_ptr, c_ptr, ctypes.c_int]
        L.bho_gemm_ref_sampled_fmt.restype = None
        L.bho_gemm_ref_sampled_fmt.argtypes = [ctypes.c_int, c_i64, c_i64, c_i64, c_ptr, c_ptr,
                                               c_ptr, c_ptr, ctypes.c_float, c_i64, c_ptr, c_ptr,
                                               c_ptr, c_ptr, ctypes.c_int]
        L.bho_tolerance.restype = ctypes.c_double
        L.bho_tolerance.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float, c_i64, ctypes.c_double]
        L.bho_tolerance_worst.restype = ctypes.c_double
        L.bho_tolerance_worst.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float, c_i64,
                                          ctypes.c_double]
        L.bho_decode_operand.restype = None
        L.bho_decode_operand.argtypes = [ctypes.c_int, c_ptr, c_ptr, c_i64, c_i64, c_ptr, c_ptr]
        L.bho_ref_loop.restype = None
        L.bho_ref_loop.argtypes = [c_i64, c_i64, c_i64, ctypes.c_int, c_ptr, c_ptr, c_ptr, c_ptr,
                                   ctypes.c_float, c_ptr, ctypes.c_int]
        _lib = L
    return _lib


def ref_shim():
    """The reference-backed shim (oracle/_ref), or None when it was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_SHIM_PATH):
        R = ctypes.CDLL(REF_SHIM_PATH)
        R.ref_sf_offset.restype = c_i64
        R.ref_sf_offset.argtypes = [c_i64, c_i64, c_i64, c_i64, ctypes.c_int]
        R.ref_sf_cosize.restype = c_i64
        R.ref_sf_cosize.argtypes = [c_i64, c_i64, ctypes.c_int]
        R.ref_e2m1.restype = ctypes.c_uint8
        R.ref_e2m1.argtypes = [ctypes.c_float]
        R.ref_ue4m3.restype = ctypes.c_uint8
        R.ref_ue4m3.argtypes = [ctypes.c_float]
        R.ref_bf16.restype = ctypes.c_uint16
        R.ref_bf16.argtypes = [ctypes.c_float]
        _ref = R
    return _ref


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(c_ptr)


# ---- vectorised helpers (numpy in, numpy out) -------------------------------------------

def sf_storage_bytes(mn: int, k: int) -> int:
    return int(lib().bho_sf_storage_bytes(mn, k))


def sf_offset(mn: int, kg: int, k: int) -> int:
    return int(lib().bho_sf_offset(mn, kg, k))


def sf_offsets(mn: int, k: int) -> np.ndarray:
    """Offsets for every (row, k-group) of an (mn, k) tensor, same rule as the C code."""
    kgb = (k // 16 + 3) // 4
    r = np.arange(mn, dtype=np.int64)[:, None]
    g = np.arange(k // 16, dtype=np.int64)[None, :]
    return ((r // 128) * kgb + g // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + (g % 4)


def gen_normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().bho_gen_normal(seed, offset, n, mean, std, _p(out))
    return out


def apply_outliers(seed: int, x: np.ndarray, p: float, factor: float) -> None:
    lib().bho_apply_outliers(seed, x.size, p, factor, _p(x))


def quantize(X: np.ndarray):
    """NVFP4-quantise a (rows, K) float32 matrix: returns (packed u8, sf u8, global_scale)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    rows, k = X.shape
    packed = np.zeros(rows * k // 2, dtype=np.uint8)
    sf = np.zeros(sf_storage_bytes(rows, k), dtype=np.uint8)
    g = lib().bho_quantize_nvfp4(_p(X), rows, k, _p(packed), _p(sf))
    return packed, sf, float(g)


FORMATS = {"nvfp4": 0, "mxfp4": 1, "mxf8f4": 2}   # mxf8f4: MXFP8 A x MXFP4 B


def sf_storage_bytes_vs(mn: int, k: int, vs: int) -> int:
    return int(lib().bho_sf_storage_bytes_vs(mn, k, vs))


def sf_offset_vs(mn: int, kg: int, k: int, vs: int) -> int:
    return int(lib().bho_sf_offset_vs(mn, kg, k, vs))


def quantize_mxfp4(X: np.ndarray):
    """MXFP4-quantise a (rows, K) float32 matrix (K % 32 == 0): returns (packed u8, sf u8)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    rows, k = X.shape
    packed = np.zeros(rows * k // 2, dtype=np.uint8)
    sf = np.zeros(sf_storage_bytes_vs(rows, k, 32), dtype=np.uint8)
    lib().bho_quantize_mxfp4(_p(X), rows, k, _p(packed), _p(sf))
    return packed, sf


def quantize_mxfp8(X: np.ndarray):
    """MXFP8 (E4M3)-quantise a (rows, K) float32 matrix (K % 32 == 0): returns (q u8 [rows*K],
    sf u8)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    rows, k = X.shape
    q = np.zeros(rows * k, dtype=np.uint8)
    sf = np.zeros(sf_storage_bytes_vs(rows, k, 32), dtype=np.uint8)
    lib().bho_quantize_mxfp8(_p(X), rows, k, _p(q), _p(sf))
    return q, sf


def gemm_full(M, N, K, A, SFA, B, SFB, alpha=1.0, nthreads=0, want_absdot=True, fmt="nvfp4"):
    """Full host reference: returns (D bf16 bits as uint16 [M,N], absdot [M,N] or None)."""
    D = np.empty((M, N), dtype=np.uint16)
    ad = np.empty((M, N), dtype=np.float64) if want_absdot else None
    nt = nthreads if nthreads > 0 else (os.cpu_count() or 1)
    lib().bho_gemm_ref_full_fmt(FORMATS[fmt], M, N, K, _p(A), _p(SFA), _p(B), _p(SFB), alpha,
                                _p(D), _p(ad) if ad is not None else None, nt)
    return D, ad


def gemm_sampled(M, N, K, A, SFA, B, SFB, ms, ns, alpha=1.0, nthreads=0, fmt="nvfp4"):
    ms = np.ascontiguousarray(ms, dtype=np.int64)
    ns = np.ascontiguousarray(ns, dtype=np.int64)
    S = ms.size
    D = np.empty(S, dtype=np.uint16)
    ad = np.empty(S, dtype=np.float64)
    nt = nthreads if nthreads > 0 else (os.cpu_count() or 1)
    lib().bho_gemm_ref_sampled_fmt(FORMATS[fmt], M, N, K, _p(A), _p(SFA), _p(B), _p(SFB),
                                   alpha, S, _p(ms), _p(ns), _p(D), _p(ad), nt)
    return D, ad


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def decode_operand(P: np.ndarray, SF: np.ndarray, rows: int, K: int, kind: str = "nvfp4"):
    """Element values (rows x K float32) and per-group scale values (rows x K/vs float32) of a
    quantised operand: the arrays the reference example builds before its host loop
    (example/nvfp4_bf16_gemm.cu:159-168 reads them as refA / sfaVal)."""
    k = {"nvfp4": 0, "mxfp4": 1, "mxfp8": 2}[kind]
    vs = 16 if k == 0 else 32
    vals = np.empty((rows, K), dtype=np.float32)
    scales = np.empty((rows, K // vs), dtype=np.float32)
    lib().bho_decode_operand(k, _p(np.ascontiguousarray(P)), _p(np.ascontiguousarray(SF)), rows, K,
                             _p(vals), _p(scales))
    return vals, scales


def ref_loop(vA, sA, vB, sB, alpha=1.0, nthreads=0):
    """The example's host loop on decoded operands (decode_operand): D[m, n] = bf16(alpha *
    sum_k (vA*sA)*(vB*sB)) in k order, for every row of vA against every row of vB.  Returns
    bf16 bits [rows_a, rows_b]; bit-identical to gemm_full."""
    M, K = vA.shape
    N = vB.shape[0]
    vs = K // sA.shape[1]
    D = np.empty((M, N), dtype=np.uint16)
    nt = nthreads if nthreads > 0 else (os.cpu_count() or 1)
    lib().bho_ref_loop(M, N, K, vs, _p(vA), _p(sA), _p(vB), _p(sB), alpha, _p(D), nt)
    return D


def tolerance(ref: np.ndarray, got: np.ndarray, alpha: float, K: int, absdot: np.ndarray,
              worst: bool = False) -> np.ndarray:
    """Vectorised bho_tolerance: ulp_bf16(max|.|) + |alpha|*sqrt(K)*2^-24*absdot (FP32
    reassociation slack for rounding errors of random sign), or with worst=True the
    worst-case bound bho_tolerance_worst, ulp_bf16 + |alpha|*K*2^-24*absdot."""
    a = np.maximum(np.abs(ref.astype(np.float64)), np.abs(got.astype(np.float64)))
    a = np.maximum(a, np.float64(np.finfo(np.float32).tiny))
    _, e = np.frexp(a)
    ulp = np.ldexp(1.0, (e - 1) - 7)
    slack = float(K) if worst else float(np.sqrt(K))
    return ulp + abs(alpha) * slack * 2.0 ** -24 * absdot


# Every check made in this process, as (pytest test id or "", report): the test session
# prints them (tests/conftest.py), so each parity test's bit-identical fraction and
# err/tol figures are on record, not only its pass/fail.
REPORTS: list = []


def check(ref_bits: np.ndarray, got_bits: np.ndarray, alpha: float, K: int, absdot: np.ndarray,
          record: bool = True):
    """Returns (n_bad, max_abs_err, max_err_over_tol, reference_rel_max) for BF16 outputs,
    under the tolerance every parity test asserts (tolerance(), sqrt(K) slack).  record=False
    keeps the figures out of REPORTS (checks of results with a planted mistake)."""
    r = check_report(ref_bits, got_bits, alpha, K, absdot)
    r["K"] = int(K)
    if record:
        REPORTS.append((os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], r))
    return r["mismatches"], r["max_abs_err"], r["max_err_over_tol"], r["reference_rel_max"]


def check_report(ref_bits: np.ndarray, got_bits: np.ndarray, alpha: float, K: int,
                 absdot: np.ndarray) -> dict:
    """Parity figures of a GPU result against the oracle's, element by element:
    mismatches / max_err_over_tol under the asserted tolerance (sqrt(K) slack), the same under
    the worst-case bound (the outer limit), the fraction of bit-identical elements, and the
    reference example's own relative error |got-ref|/(|ref|+1e-3) (it accepts <= 0.05)."""
    ref = bf16_bits_to_f32(ref_bits.ravel())
    got = bf16_bits_to_f32(got_bits.ravel())
    err = np.abs(ref.astype(np.float64) - got.astype(np.float64))
    ad = absdot.ravel()
    tol = tolerance(ref, got, alpha, K, ad)
    tol_w = tolerance(ref, got, alpha, K, ad, worst=True)
    rel = err / (np.abs(ref.astype(np.float64)) + 1e-3)
    n = int(ref.size)
    return {
        "elements": n,
        "mismatches": int(np.count_nonzero(~(err <= tol))),
        "max_err_over_tol": float((err / tol).max(initial=0.0)),
        "mismatches_worst_case_bound": int(np.count_nonzero(~(err <= tol_w))),
        "max_err_over_worst_case_bound": float((err / tol_w).max(initial=0.0)),
        "bit_identical_frac": float(np.mean(ref_bits.ravel() == got_bits.ravel())) if n else 1.0,
        "max_abs_err": float(err.max(initial=0.0)),
        "reference_rel_max": float(rel.max(initial=0.0)),
    }


def format_report(r: dict) -> str:
    return (f"{r['elements']} elements: {r['mismatches']} outside tolerance, "
            f"bit-identical {r['bit_identical_frac']:.6f}, max err/tol {r['max_err_over_tol']:.3g} "
            f"(worst-case bound {r['max_err_over_worst_case_bound']:.3g}), "
            f"max |err| {r['max_abs_err']:.3g}, example rel {r['reference_rel_max']:.3g}")
