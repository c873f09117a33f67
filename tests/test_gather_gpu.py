"""GEMM with the N-split's all-gather fused into the epilogue, on one GPU.

Ranks are emulated one after another on a single device: "rank" r computes its N-slice and
writes it into every rank's row-major buffer (its own by TMA stores, the others with the
epilogue's plain 16-byte stores, here to local memory instead of a peer GPU's).  Nothing
waits on another launch, so this runs on one GPU; the real multi-GPU exchange is covered by
test_gather_multigpu.py.  Every buffer must end bit-identical, equal to the oracle's full
M x N GEMM, with columns outside [col0, col0 + N) untouched."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import nvfp4_cases as C

pytestmark = pytest.mark.gpu


def _bits(t):
    import torch

    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("M,N,K,world", [(256, 1024, 512, 2), (300, 1024, 768, 4),
                                         (200, 2048, 256, 8), (1000, 1024, 1024, 2),
                                         (16, 2048, 1024, 4), (1, 1024, 512, 2),
                                         (100, 1024, 768, 8), (128, 4096, 2048, 2)])
def test_emulated_ranks_all_hold_the_full_result(M, N, K, world):
    import torch
    import blackhole_b200 as bh
    from blackhole_b200.nsplit import shard, shard_views

    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=M + N + world)
    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    outs = [torch.full((M, N), -1, dtype=torch.int16, device=dev) for _ in range(world)]
    for r in range(world):
        s = shard(N, K, r, world)
        b, sfb = shard_views(tB, tSFB, N, K, r, world)
        dst = [outs[r]] + [outs[q] for q in range(world) if q != r]
        bh.nvfp4_bf16_gemm_gather(M, s.rows, K, tA, tSFA, b, sfb, dst, s.row0, N, alpha)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    got = [_bits(o) for o in outs]
    for g in got[1:]:
        assert np.array_equal(g, got[0]), "buffers differ between emulated ranks"
    assert not np.any(got[0] == 0xFFFF), "unwritten elements"
    (bad, maxerr, ratio, _), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, got[0])
    assert bad == 0, f"{bad} elements beyond tolerance (max err {maxerr}, err/tol {ratio})"


@pytest.mark.parametrize("M,schedule", [(130, "2sm"), (16, "skinny"), (77, "skinny")])
def test_single_destination_equals_plain_gemm_and_respects_columns(M, schedule):
    """ndst = 1 writes exactly the plain GEMM's bits into the column window of a wider buffer;
    a ragged window (col0 = 8, N = 264) and ragged M leave every other column untouched."""
    import torch
    import blackhole_b200 as bh

    N, K, col0, ldd = 264, 512, 8, 288
    A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=5)
    dev = torch.device("cuda:0")
    tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
    plain = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    bh.nvfp4_bf16_gemm_ex(M, N, K, tA, tSFA, tB, tSFB, plain, alpha, schedule=schedule)
    wide = [torch.full((M, ldd), 0x1234, dtype=torch.int16, device=dev) for _ in range(3)]
    bh.nvfp4_bf16_gemm_gather(M, N, K, tA, tSFA, tB, tSFB, wide, col0, ldd, alpha)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    ref = _bits(plain)
    for w in wide:
        g = _bits(w)
        assert np.array_equal(g[:, col0:col0 + N], ref)
        assert np.all(g[:, :col0] == 0x1234) and np.all(g[:, col0 + N:] == 0x1234)


def test_back_to_back_gathers_without_sync():
    """Two gathers into the same buffers back to back (programmatic dependent launch): the
    second's stores are ordered after the first's."""
    import torch
    import blackhole_b200 as bh

    M, N, K = 512, 512, 1024
    ops = [C.make_operands(M, N, K, seed=s) for s in (11, 12)]
    dev = torch.device("cuda:0")
    outs = [torch.full((M, N), -1, dtype=torch.int16, device=dev) for _ in range(2)]
    for A, SFA, B, SFB, alpha in ops:
        tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
        bh.nvfp4_bf16_gemm_gather(M, N, K, tA, tSFA, tB, tSFB, outs, 0, N, alpha)
    torch.cuda.synchronize()
    assert bh.device_status(0) == 0
    A, SFA, B, SFB, alpha = ops[1]
    for o in outs:
        (bad, _, _, _), _ = C.check_full(M, N, K, A, SFA, B, SFB, alpha, _bits(o))
        assert bad == 0


def test_ipc_handle_roundtrip_in_process():
    """The handle of a buffer inside a larger allocation carries its offset."""
    import torch
    import blackhole_b200 as bh

    base = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda:0")
    h0, off0 = bh.ipc_get_handle(base)
    h1, off1 = bh.ipc_get_handle(base[4096:])
    assert len(h0) == 64 and h0 == h1
    assert off1 == off0 + 4096
