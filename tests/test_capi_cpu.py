"""C-ABI host checks that need no GPU: the library loads, exports every symbol that
include/*.h declares, agrees with the oracle on the scale-factor layout, and rejects bad
arguments with cudaErrorInvalidValue before any device work."""
import os
import re
import subprocess

import numpy as np
import pytest

import blackhole_b200 as bh
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            syms |= set(re.findall(r"BLACKHOLE_SM100_API\s+[\w\s\*]+?\b(blackhole_\w+)\s*\(", src))
    return syms


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert "blackhole_sm100_nvfp4_bf16_gemm" in syms and len(syms) >= 5
    out = subprocess.run(["nm", "-D", "--defined-only", bh.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    missing = syms - exported
    assert not missing, f"declared but not exported: {missing}"
    L = bh.load()
    for s in syms:
        assert hasattr(L, s)
    assert L.blackhole_sm100_abi_version() == 6
    assert "blackhole_sm100_mxfp4_bf16_gemm_ex" in syms and "blackhole_sm100_mxfp4_quantize" in syms


@pytest.mark.parametrize("mn,k", [(1, 256), (16, 8192), (200, 768), (28672, 8192), (8192, 8192)])
def test_sf_layout_matches_oracle(mn, k):
    assert bh.sf_storage_bytes(mn, k) == O.sf_storage_bytes(mn, k)
    for m in (0, 1, 31, 32, 127, 128, mn - 1):
        if m >= mn:
            continue
        for kg in (0, 1, 3, 4, k // 16 - 1):
            assert bh.sf_offset(m, kg, k) == O.sf_offset(m, kg, k)


@pytest.mark.parametrize("mn,k", [(1, 128), (16, 8192), (200, 768), (130, 320), (8192, 8192)])
def test_mx_sf_layout_matches_oracle(mn, k):
    assert bh.mxfp4_sf_storage_bytes(mn, k) == O.sf_storage_bytes_vs(mn, k, 32)


@pytest.mark.parametrize("M,N,K", [(0, 128, 256), (128, 100, 256), (128, 128, 16), (128, 128, 48),
                                   (128, 4, 256)])
def test_mx_bad_shapes_rejected_before_launch(M, N, K):
    for sched in ("auto", "1sm", "2sm", "skinny"):
        with pytest.raises(bh.BlackholeError) as ei:
            bh.mxfp4_bf16_gemm(M, N, K, 4096, 4096, 4096, 4096, 4096, 1.0, stream=0, schedule=sched)
        assert ei.value.code == 1


@pytest.mark.parametrize("M,N,K", [(0, 128, 256), (128, 0, 256), (128, 100, 256), (128, 128, 0),
                                   (128, 128, 16), (128, 128, 80), (-1, 128, 256), (128, 4, 256),
                                   (128, 12, 256)])
def test_bad_shapes_rejected_before_launch(M, N, K):
    with pytest.raises(bh.BlackholeError) as ei:
        bh.nvfp4_bf16_gemm(M, N, K, 4096, 4096, 4096, 4096, 4096, 1.0, stream=0)
    assert ei.value.code == 1  # cudaErrorInvalidValue


def test_null_and_misaligned_pointers_rejected():
    good = 1 << 20
    for args in [(0, good, good, good, good), (good, 0, good, good, good), (good, good, good, good, 0),
                 (good + 8, good, good, good, good), (good, good, good + 4, good, good),
                 (good, good, good, good, good + 2)]:
        with pytest.raises(bh.BlackholeError) as ei:
            bh.nvfp4_bf16_gemm(128, 128, 256, *args, 1.0, stream=0)
        assert ei.value.code == 1


@pytest.mark.parametrize("ndst,col0,ldd,N", [(0, 0, 256, 256), (9, 0, 256, 256), (2, 4, 264, 256),
                                             (2, 0, 260, 256), (2, 8, 256, 256), (2, -8, 256, 256),
                                             (2, 0, 256, 100)])
def test_gather_bad_arguments_rejected_before_launch(ndst, col0, ldd, N):
    good = 1 << 20
    with pytest.raises(bh.BlackholeError) as ei:
        bh.nvfp4_bf16_gemm_gather(128, N, 256, good, good, good, good, [good] * ndst, col0, ldd,
                                  1.0, stream=0)
    assert ei.value.code == 1


def test_gather_misaligned_destination_rejected():
    good = 1 << 20
    with pytest.raises(bh.BlackholeError) as ei:
        bh.nvfp4_bf16_gemm_gather(128, 256, 256, good, good, good, good, [good, good + 8], 0, 256,
                                  1.0, stream=0)
    assert ei.value.code == 1


def test_ipc_helpers_reject_null_arguments():
    L = bh.load()
    assert L.blackhole_sm100_ipc_get_handle(None, None, None) == 1
    assert L.blackhole_sm100_ipc_open(None, 0, None) == 1
    assert L.blackhole_sm100_ipc_close(12345) == 1


@pytest.mark.parametrize("M,N,K", [(128, 128, 256 + 32), (128, 128, 64), (128, 100, 256), (0, 128, 256)])
def test_mxf8f4_bad_shapes_rejected_before_launch(M, N, K):
    for sched in ("auto", "1sm", "2sm", "skinny"):
        with pytest.raises(bh.BlackholeError) as ei:
            bh.mxf8f4_bf16_gemm(M, N, K, 4096, 4096, 4096, 4096, 4096, 1.0, stream=0, schedule=sched)
        assert ei.value.code == 1


def test_mxf8f4_b_needs_32_byte_alignment():
    with pytest.raises(bh.BlackholeError) as ei:
        bh.mxf8f4_bf16_gemm(128, 128, 256, 4096, 4096, 4096 + 16, 4096, 4096, 1.0, stream=0)
    assert ei.value.code == 1


@pytest.mark.parametrize("world,rank,epoch,limit", [(0, 0, 1, 10**9), (9, 0, 1, 10**9), (2, 2, 1, 10**9),
                                                    (2, -1, 1, 10**9), (2, 0, 0, 10**9), (2, 0, 1, 0),
                                                    (2, 0, 1, 2 * 10**10)])
def test_peer_barrier_bad_arguments_rejected(world, rank, epoch, limit):
    good = 1 << 20
    with pytest.raises(bh.BlackholeError) as ei:
        bh.peer_barrier([good] * max(world, 1), world, rank, epoch, limit, stream=0)
    assert ei.value.code == 1


def test_peer_barrier_null_or_misaligned_flags_rejected():
    good = 1 << 20
    for flags in ([good, 0], [good, good + 4]):
        with pytest.raises(bh.BlackholeError) as ei:
            bh.peer_barrier(flags, 2, 0, 1, 10**9, stream=0)
        assert ei.value.code == 1


@pytest.mark.parametrize("schedule", [-1, 5, 6, 1 << 20])
@pytest.mark.parametrize("entry", ["blackhole_sm100_nvfp4_bf16_gemm_ex",
                                   "blackhole_sm100_mxfp4_bf16_gemm_ex",
                                   "blackhole_sm100_mxf8f4_bf16_gemm_ex"])
def test_ex_rejects_unknown_schedules(entry, schedule):
    """Schedules are 0 (by shape) to 4; anything else is cudaErrorInvalidValue before any
    device work (valid shapes and aligned pointers, so only the schedule is wrong)."""
    import ctypes
    fn = getattr(bh.load(), entry)
    good = 1 << 20
    rc = fn(ctypes.c_int(128), ctypes.c_int(128), ctypes.c_int(256),
            *(ctypes.c_void_p(good) for _ in range(5)), ctypes.c_float(1.0), ctypes.c_int(schedule),
            ctypes.c_void_p(0), ctypes.c_int64(0), ctypes.c_void_p(0))
    assert rc == 1
    assert set(bh.SCHEDULES.values()) == set(range(5))
