"""The fused GEMM + all-gather across real GPUs (skipped with fewer than two).

Two ranks, one process per GPU, NCCL for the process group; the output buffers are
exchanged as CUDA IPC handles and each rank's kernel writes its N-slice into both GPUs'
row-major M x N buffers.  After the barrier each rank checks its whole buffer against the
oracle.  NVLink SHARP is switched off (NCCL_NVLS_ENABLE=0) and no NVLS object is made:
the peers' buffers are plain IPC mappings written with ordinary stores."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(512, 2048, 1024), (16, 4096, 2048)]   # two-SM and skinny (decode) schedules


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errfile):
    import datetime

    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from tests import nvfp4_cases as C
    from blackhole_b200.nsplit import GatheredOutput, nsplit_gemm_gathered
    import blackhole_b200 as bh

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        dev = torch.device("cuda", rank)
        for M, N, K in SHAPES:
            A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=21 + M)
            tA, tSFA, tB, tSFB = (torch.from_numpy(x).to(dev) for x in (A, SFA, B, SFB))
            out = GatheredOutput(M, N, rank, world)
            out.out.fill_(float("nan"))
            out.barrier()
            for _ in range(2):
                nsplit_gemm_gathered(M, N, K, tA, tSFA, tB, tSFB, alpha, rank, world, out)
            torch.cuda.synchronize()
            assert bh.device_status(rank) == 0
            got = out.out.view(torch.int16).cpu().numpy().view(np.uint16)
            ref, ad = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha)
            bad, maxerr, ratio, _ = O.check(ref, got, alpha, K, ad)
            assert bad == 0, f"rank {rank} {M}x{N}x{K}: {bad} bad (max err {maxerr}, err/tol {ratio})"
            out.barrier()
            torch.cuda.synchronize()
            out.close()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # reported to the parent through the file
        with open(errfile + f".{rank}", "w") as f:
            f.write(repr(exc))
        raise


def test_two_gpus_each_hold_the_full_result(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    errfile = str(tmp_path / "err")
    mp.start_processes(_worker, args=(2, _free_port(), errfile), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        assert not os.path.exists(errfile + f".{r}"), open(errfile + f".{r}").read()
