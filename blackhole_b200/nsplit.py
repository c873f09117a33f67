"""N-split of the NVFP4 GEMM across the GPUs of one node (host-side plumbing).

Rank r of P owns rows [r*N/P, (r+1)*N/P) of B (the GEMM's N dimension) and the matching
scale factors; A and its scale factors are replicated.  Each rank runs the single-GPU
operator on (M, N/P, K) and produces an M x N/P slice of D; no GPU reads another GPU's
memory.  The slices are assembled either by an NCCL all-gather after the GEMM ([P][M][N/P],
`nsplit_gemm(gather=True)`), or inside the GEMM itself (`GatheredOutput` +
`nsplit_gemm_gathered`): every rank's kernel writes its tiles straight into every rank's
row-major M x N buffer over NVLink while it computes the next tiles.

Because a shard is a whole number of 128-row blocks, its SFB is one contiguous byte range of
the full SFB tensor (the 128x4 layout advances along K inside a row block, then to the next
block), so shards are plain views: no repacking.
"""
from __future__ import annotations

from dataclasses import dataclass

from blackhole_b200 import sf_storage_bytes


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    row0: int        # first row of B owned by this rank
    rows: int        # rows owned (N / world)
    b_offset: int    # byte offset of the shard in packed B
    b_bytes: int
    sf_offset: int   # byte offset of the shard's scale factors in SFB
    sf_bytes: int


def shard(N: int, K: int, rank: int, world: int) -> Shard:
    """Rows of B (and bytes of B / SFB) that `rank` owns in an even N-split."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    if N % (128 * world) != 0:
        raise ValueError(f"N={N} must split into {world} shards of whole 128-row blocks")
    rows = N // world
    row0 = rank * rows
    sf_per_shard = sf_storage_bytes(rows, K)
    return Shard(rank, world, row0, rows, row0 * (K // 2), rows * (K // 2),
                 rank * sf_per_shard, sf_per_shard)


def shard_views(B, SFB, N: int, K: int, rank: int, world: int):
    """Views of this rank's rows of packed B and of its SFB bytes (1-D byte tensors or
    arrays, or 2-D [N, K/2] B); no copy."""
    s = shard(N, K, rank, world)
    if getattr(B, "ndim", 1) == 2:
        b = B[s.row0:s.row0 + s.rows]
    else:
        b = B[s.b_offset:s.b_offset + s.b_bytes]
    return b, SFB[s.sf_offset:s.sf_offset + s.sf_bytes]


def assemble(gathered, world: int):
    """[P][M][N/P] slices (the all-gather layout) -> row-major [M][N]."""
    P, M, n = gathered.shape
    assert P == world
    if hasattr(gathered, "permute"):
        return gathered.permute(1, 0, 2).reshape(M, P * n)
    return gathered.transpose(1, 0, 2).reshape(M, P * n)


def nsplit_gemm(M: int, N: int, K: int, A, SFA, B, SFB, alpha: float, rank: int, world: int,
                gather: bool = False, group=None, stream=None):
    """Runs this rank's slice on the current CUDA device; returns the M x N/P slice, or with
    gather=True the assembled M x N result (NCCL all-gather through torch.distributed)."""
    import torch

    import blackhole_b200 as bh

    s = shard(N, K, rank, world)
    b, sfb = shard_views(B, SFB, N, K, rank, world)
    D = torch.empty((M, s.rows), dtype=torch.bfloat16, device=A.device)
    bh.nvfp4_bf16_gemm(M, s.rows, K, A, SFA, b, sfb, D, alpha, stream=stream)
    if not gather or world == 1:
        return D
    import torch.distributed as dist

    out = torch.empty((world, M, s.rows), dtype=torch.bfloat16, device=A.device)
    dist.all_gather_into_tensor(out, D, group=group)
    return assemble(out, world)


class GatheredOutput:
    """Two row-major M x N BF16 buffers on every rank, each mapped into every other rank
    (CUDA IPC), plus the ranks' barrier flags.  Step s of a gathered N-split writes buffer
    s % 2 on every rank.

    Collective: every rank of `group` constructs it with the same M and N.

    Why two buffers: a step's gather kernels store into the OTHER ranks' buffers.  With one
    buffer, a rank that passed step s's barrier could start step s+1 and overwrite a slower
    rank's buffer while that rank still reads its step-s result.  With two, step s+1 writes the
    buffer of step s-1, and a rank reaches step s+1 only after every rank arrived at step s's
    barrier, which each rank does after the work it queued before step s on the same stream,
    its reads of the step s-1 result included.

    Rule for callers: read a step's result (`out`, or the tensor nsplit_gemm_gathered returns)
    on the stream passed to the step, before enqueueing the step after next; a step's result
    is overwritten two steps later.  `dst_c` is this step's destination list for the gather
    call (own buffer first, then the peers' mappings), `barrier()` the stream-ordered flag
    barrier that ends a step and makes every rank's tiles visible to work after it.
    """

    def __init__(self, M: int, N: int, rank: int, world: int, group=None,
                 barrier_limit_ns: int = 1_000_000_000):
        import torch
        import torch.distributed as dist

        import blackhole_b200 as bh

        self.M, self.N, self.rank, self.world = M, N, rank, world
        dev = torch.cuda.current_device()
        self.bufs = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.flags = torch.zeros(world, dtype=torch.int64, device=dev)
        self._mapped = []
        ptrs = [{rank: b.data_ptr()} for b in self.bufs]
        flag_ptrs = {rank: self.flags.data_ptr()}
        if world > 1:
            handles = [None] * world
            mine = tuple(bh.ipc_get_handle(t) for t in (*self.bufs, self.flags))
            dist.all_gather_object(handles, mine, group=group)
            for q in range(world):
                if q != rank:
                    for i in range(2):
                        ptrs[i][q] = bh.ipc_open(*handles[q][i])
                        self._mapped.append(ptrs[i][q])
                    flag_ptrs[q] = bh.ipc_open(*handles[q][2])
                    self._mapped.append(flag_ptrs[q])
        self._dst = [[self.bufs[i]] + [ptrs[i][q] for q in range(world) if q != rank]
                     for i in range(2)]
        self._dst_c = [bh.pointer_array(d) for d in self._dst]
        self.flags_c = bh.pointer_array([flag_ptrs[q] for q in range(world)])
        self.epoch = 0          # flag barriers issued so far (the barrier kernel's epoch)
        self.steps = 0          # steps completed (barrier() calls)
        self.limit_ns = barrier_limit_ns

    @property
    def step_buf(self) -> int:
        """Index of the buffer the next step writes."""
        return self.steps % 2

    @property
    def dst(self):
        return self._dst[self.step_buf]

    @property
    def dst_c(self):
        return self._dst_c[self.step_buf]

    @property
    def out(self):
        """This rank's buffer holding the result of the last completed step."""
        return self.bufs[(self.steps - 1) % 2] if self.steps > 0 else self.bufs[0]

    def sync(self, stream=None):
        """A flag barrier that does not end a step: every rank's work queued before it (on
        the stream given) is complete before work after it runs on any rank.  Collective; e.g.
        after each rank re-initialises the buffer the next step writes."""
        import blackhole_b200 as bh

        self.epoch += 1
        bh.peer_barrier(self.flags_c, self.world, self.rank, self.epoch, self.limit_ns,
                        stream=stream)

    def barrier(self, stream=None):
        """Ends a step (stream-ordered): work after it on this rank's stream sees every rank's
        gather writes of this step.  Every rank calls it once per step, after the step's
        gather call."""
        self.sync(stream)
        self.steps += 1

    def close(self):
        import blackhole_b200 as bh

        for p in self._mapped:
            bh.ipc_close(p)
        self._mapped = []
        self._dst = [[b] for b in self.bufs]
        self._dst_c = [bh.pointer_array(d) for d in self._dst]


def nsplit_gemm_gathered(M: int, N: int, K: int, A, SFA, B, SFB, alpha: float, rank: int,
                         world: int, out: GatheredOutput, stream=None):
    """One step of the N-split with the gather fused into the GEMM: this rank's N-slice goes
    to the step's buffer on every rank, then the step's barrier.  Returns this rank's buffer,
    which (for work after the call on `stream`) holds the whole row-major M x N result until
    the step after next overwrites it (GatheredOutput)."""
    import blackhole_b200 as bh

    if out.M != M or out.N != N:
        raise ValueError("GatheredOutput was made for another shape")
    s = shard(N, K, rank, world)
    b, sfb = shard_views(B, SFB, N, K, rank, world)
    bh.nvfp4_bf16_gemm_gather(M, s.rows, K, A, SFA, b, sfb, out.dst_c, s.row0, N, alpha,
                              stream=stream)
    out.barrier(stream=stream)
    return out.out
