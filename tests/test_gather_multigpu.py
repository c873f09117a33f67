"""The fused GEMM + all-gather across real GPUs: 2, 4 and 8 ranks (each skipped when the box
has fewer GPUs).

One process per GPU, NCCL for the process group; the output buffers are exchanged as CUDA
IPC handles and every rank's kernel writes its N-slice into every GPU's row-major M x N buffer.
NVLink SHARP is switched off (NCCL_NVLS_ENABLE=0) and no NVLS object is made: the peers'
buffers are plain IPC mappings written with ordinary stores.

Each shape runs several steps whose inputs differ (another A or alpha per step).  Before each
step every rank fills the buffer that step writes with NaN and the ranks synchronise, so a tile
that a step fails to write, or a write that lands in the wrong step's buffer, shows up as NaN
or as the previous step's values.  After each step every rank checks its whole buffer (small
shapes) or a sample of it (the configs[4] shape) against the oracle."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (M, N, K): two-SM schedule, skinny (decode) schedule, a ragged M on the two-SM schedule
SHAPES = [(512, 2048, 1024), (16, 4096, 2048), (300, 1024, 512)]
STEPS = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check_small(rank, world, errs):
    import torch

    from oracle import oracle as O
    from tests import nvfp4_cases as C
    from blackhole_b200.nsplit import GatheredOutput, nsplit_gemm_gathered
    import blackhole_b200 as bh

    dev = torch.device("cuda", rank)
    threads = max(1, (os.cpu_count() or 1) // world)
    for M, N, K in SHAPES:
        _, _, B, SFB, _ = C.make_operands(M, N, K, seed=21 + M)
        tB, tSFB = torch.from_numpy(B).to(dev), torch.from_numpy(SFB).to(dev)
        out = GatheredOutput(M, N, rank, world)
        for step in range(STEPS):
            A, SFA, _, _, alpha = C.make_operands(M, N, K, seed=100 * step + M)
            alpha *= (1.0, -0.5, 2.0)[step % 3]
            tA, tSFA = torch.from_numpy(A).to(dev), torch.from_numpy(SFA).to(dev)
            out.bufs[out.step_buf].fill_(float("nan"))
            out.sync()          # every rank's fill lands before any rank's stores of this step
            res = nsplit_gemm_gathered(M, N, K, tA, tSFA, tB, tSFB, alpha, rank, world, out)
            torch.cuda.synchronize()
            assert bh.device_status(rank) == 0
            got = res.view(torch.int16).cpu().numpy().view(np.uint16)
            ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha, nthreads=threads)
            r = O.check_report(ref, got, alpha, K, ad)
            if r["mismatches"]:
                errs.append(f"rank {rank} {M}x{N}x{K} step {step}: {O.format_report(r)}")
        out.sync()
        torch.cuda.synchronize()
        out.close()


def _device_operand(rows, K, seed, dev, std=1.0):
    import torch
    import blackhole_b200 as bh

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((rows, K), generator=g, device=dev)
    if std != 1.0:
        x.mul_(std)
    packed, sf, sc = bh.quantize_tensor(x)
    del x
    return packed, sf, float(sc[1].item())


def _check_config4(rank, world, errs, S=2048):
    """M = 32768, N = 65536 split over the ranks, K = 8192, A replicated; every
    rank makes the same full A and B on its GPU (seeded, this library's quantiser, which is
    bit-exact with the oracle's) and uses its N-slice of B."""
    import torch

    from oracle import oracle as O
    from blackhole_b200.nsplit import GatheredOutput, nsplit_gemm_gathered
    import blackhole_b200 as bh

    M, N, K = 32768, 65536, 8192
    dev = torch.device("cuda", rank)
    A, SFA, ga = _device_operand(M, K, 4, dev)
    B, SFB, gb = _device_operand(N, K, 4004, dev)
    hA, hSFA, hB, hSFB = (t.cpu().numpy().reshape(-1) for t in (A, SFA, B, SFB))
    rng = np.random.default_rng(1000 + rank)
    ms = rng.integers(0, M, S)
    ns = rng.integers(0, N, S)
    ms[:4] = [0, 0, M - 1, M - 1]
    ns[:4] = [0, N - 1, 0, N - 1]
    tm, tn = torch.from_numpy(ms).to(dev), torch.from_numpy(ns).to(dev)
    out = GatheredOutput(M, N, rank, world)
    for step, scale in enumerate((1.0, -0.5)):
        alpha = ga * gb * scale
        out.bufs[out.step_buf].fill_(float("nan"))
        out.sync()
        res = nsplit_gemm_gathered(M, N, K, A, SFA, B, SFB, alpha, rank, world, out)
        torch.cuda.synchronize()
        assert bh.device_status(rank) == 0
        got = res[tm, tn].view(torch.int16).cpu().numpy().view(np.uint16)
        ref, ad = O.gemm_sampled(M, N, K, hA, hSFA, hB, hSFB, ms, ns, alpha,
                                 nthreads=max(1, (os.cpu_count() or 1) // world))
        r = O.check_report(ref, got, alpha, K, ad)
        if r["mismatches"]:
            errs.append(f"rank {rank} configs[4] step {step}: {O.format_report(r)}")
    out.sync()
    torch.cuda.synchronize()
    out.close()


def _worker(rank, world, port, errfile):
    import datetime

    import torch
    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        errs = []
        _check_small(rank, world, errs)
        _check_config4(rank, world, errs)
        dist.barrier()
        dist.destroy_process_group()
        if errs:
            raise AssertionError("; ".join(errs))
    except BaseException as exc:  # reported to the parent through the file
        with open(errfile + f".{rank}", "w") as f:
            f.write(repr(exc))
        raise


@pytest.mark.parametrize("world", [2, 4, 8])
def test_every_gpu_holds_the_full_result(world, tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    errfile = str(tmp_path / "err")
    mp.start_processes(_worker, args=(world, _free_port(), errfile), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        assert not os.path.exists(errfile + f".{r}"), open(errfile + f".{r}").read()
