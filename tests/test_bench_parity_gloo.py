"""The bench's multi-GPU parity records on CPU: two gloo ranks each hold their N-slice of B, run
bench.gathered_parity on a gathered M x N buffer (here the oracle's own full result, so the
record must be clean) and on their own slice, and see a planted wrong element counted.  The
same host logic runs on every rank of `bench.py --gpus P` at P > 1.  No GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, errfile):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench
    from blackhole_b200 import nsplit
    from oracle import oracle as O
    from tests import nvfp4_cases as C

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=5)
        ref, _ = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha, nthreads=2, want_absdot=False)
        s = nsplit.shard(N, K, rank, world)
        b, sfb = nsplit.shard_views(B, SFB, N, K, rank, world)
        t = [torch.from_numpy(np.ascontiguousarray(x)) for x in (A, SFA, b, sfb)]

        def bf16(bits):
            return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)

        full = bench.gathered_parity(M, N, K, *t, alpha, rank, world, s.row0, bf16(ref), S=512)
        assert full["mismatches"] == 0 and full["bit_identical_frac"] == 1.0, full
        assert full["elements"] == 512
        mine = bench.gathered_parity(M, N, K, *t, alpha, rank, world, s.row0,
                                     bf16(ref[:, s.row0:s.row0 + s.rows]), S=512, own_slice=True)
        assert mine["mismatches"] == 0 and 0 < mine["elements"] < 512, mine
        merged = bench._merge_parity(bench.all_gather_objects(mine, world))
        assert merged["elements"] == 512 and merged["mismatches"] == 0, merged
        # a wrong element at a sampled point of the gathered buffer is counted, on that rank only
        rng = np.random.default_rng(77)          # the sample points gathered_parity draws
        ms, ns = rng.integers(0, M, 512), rng.integers(0, N, 512)
        m0, n0 = int(ms[0]), int(ns[0])
        bad = ref.copy()
        if rank == 1:
            bad[m0, n0] ^= np.uint16(0x0100)
        r = bench.gathered_parity(M, N, K, *t, alpha, rank, world, s.row0, bf16(bad), S=512)
        assert r["mismatches"] == (1 if rank == 1 else 0), r
        dist.barrier()
    except BaseException as exc:
        with open(errfile + f".{rank}", "w") as f:
            f.write(repr(exc))
        raise
    finally:
        dist.destroy_process_group()


def test_gathered_parity_two_ranks(tmp_path):
    errfile = str(tmp_path / "err")
    mp.spawn(_worker, args=(2, _free_port(), 64, 512, 256, errfile), nprocs=2, join=True)
    for r in range(2):
        assert not os.path.exists(errfile + f".{r}"), open(errfile + f".{r}").read()
