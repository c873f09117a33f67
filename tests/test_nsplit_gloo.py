"""Host logic of the multi-GPU N-split on CPU: two gloo ranks each take their shard of B and
SFB (views of whole 128-row scale-factor blocks), compute their M x N/P slice with the CPU
oracle, all-gather the slices and check that the assembled [M][N] result is bit-identical
to the unsplit GEMM.  No GPU."""
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


def _worker(rank, world, port, M, N, K):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from oracle import oracle as O
    from blackhole_b200 import nsplit
    from tests import nvfp4_cases as C

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        A, SFA, B, SFB, alpha = C.make_operands(M, N, K, seed=42)
        s = nsplit.shard(N, K, rank, world)
        b, sfb = nsplit.shard_views(B, SFB, N, K, rank, world)
        assert b.size == s.rows * K // 2 and sfb.size == s.sf_bytes
        mine, _ = O.gemm_full(M, s.rows, K, A, SFA, np.ascontiguousarray(b),
                              np.ascontiguousarray(sfb), alpha, nthreads=2, want_absdot=False)
        out = [torch.empty((M, s.rows), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(mine.astype(np.int32)))
        gathered = torch.stack(out).numpy().astype(np.uint16)       # [P][M][N/P]
        full = nsplit.assemble(gathered, world)
        if rank == 0:
            ref, _ = O.gemm_full(M, N, K, A, SFA, B, SFB, alpha, nthreads=2, want_absdot=False)
            assert np.array_equal(full, ref), "assembled N-split result differs from the unsplit GEMM"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M,N,K", [(2, 64, 512, 512), (2, 130, 1024, 256), (4, 16, 1024, 768)])
def test_nsplit_gloo_matches_unsplit(world, M, N, K):
    mp.spawn(_worker, args=(world, _free_port(), M, N, K), nprocs=world, join=True)


def test_shard_geometry():
    from blackhole_b200 import nsplit, sf_storage_bytes
    N, K = 65536, 8192
    for world in (1, 2, 4, 8):
        shards = [nsplit.shard(N, K, r, world) for r in range(world)]
        assert sum(s.rows for s in shards) == N
        assert shards[-1].sf_offset + shards[-1].sf_bytes == sf_storage_bytes(N, K)
        assert shards[-1].b_offset + shards[-1].b_bytes == N * K // 2
    with pytest.raises(ValueError):
        nsplit.shard(384, 256, 0, 2)   # 192-row shards are not whole SF blocks
