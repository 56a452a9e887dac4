"""Output-row sharding of a set of GEMV/GEMM weights across GPUs (one process per GPU).

The reference splits work by disjoint output-row ranges (``gemv_repacked_rows``,
repack.rs:4014; ``gemm_repacked_rows``, :4087; stitched bit-identically in
tests/test_repack_gemv_gemm.rs:805-826). Rows are independent, so rank p of P owns rows
``shard_rows(rows, P, p)`` of every matrix, computes them with the same kernels as a
single-GPU call, and one all-gather per step collects the slices. No K split is used: it would
need an all-reduce and change the f32 summation order.

Layout of one rank's flat output buffer: the matrices in order, each contributing its slice,
padded to the largest rank's total so that ``all_gather_into_tensor`` sees equal sizes.

Failures of the collective (a peer that died or never joins, a process-group timeout) surface
as ``CollectiveError`` on the host; every rank takes the same collective steps in the same order.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["shard_rows", "ShardedOutputs", "CollectiveError"]


class CollectiveError(RuntimeError):
    """The all-gather of output slices failed (peer lost, timeout, communicator aborted)."""


def shard_rows(rows: int, world: int, rank: int) -> range:
    """Rows [r0, r1) of a `rows`-row matrix owned by `rank` of `world`: contiguous, in rank
    order, the first ``rows % world`` ranks one row more than the others."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(rows, world)
    r0 = rank * base + min(rank, extra)
    return range(r0, r0 + base + (1 if rank < extra else 0))


@dataclass
class _Mat:
    name: str
    rows: int
    slices: list  # per rank: range of rows
    offs: list    # per rank: offset of the slice in that rank's flat buffer


class ShardedOutputs:
    """Flat per-rank output buffer for a list of (name, rows) matrices, its all-gather, and the
    reassembly of full output vectors from the gathered slices."""

    def __init__(self, mats, world: int, rank: int, device="cuda", dtype=torch.float32):
        self.world, self.rank = world, rank
        self.mats: dict[str, _Mat] = {}
        totals = [0] * world
        for name, rows in mats:
            slices, offs = [], []
            for r in range(world):
                sl = shard_rows(rows, world, r)
                slices.append(sl)
                offs.append(totals[r])
                totals[r] += len(sl)
            self.mats[name] = _Mat(name, rows, slices, offs)
        self.local_len = max(totals)
        self.local = torch.zeros(self.local_len, dtype=dtype, device=device)
        self.gathered = (torch.empty(self.local_len * world, dtype=dtype, device=device)
                         if world > 1 else self.local)

    def rows_of(self, name: str) -> range:
        """This rank's rows of matrix `name`."""
        return self.mats[name].slices[self.rank]

    def local_slice(self, name: str) -> torch.Tensor:
        """View of this rank's output slice of matrix `name` in the flat buffer."""
        m = self.mats[name]
        o = m.offs[self.rank]
        return self.local[o:o + len(m.slices[self.rank])]

    def gather(self, group=None):
        """All-gather the flat buffers (one collective, every rank must call it)."""
        if self.world == 1:
            return
        try:
            dist.all_gather_into_tensor(self.gathered, self.local, group=group)
        except Exception as e:  # noqa: BLE001 -- any backend failure is a lost step
            raise CollectiveError(f"all-gather of output slices failed on rank {self.rank}: "
                                  f"{type(e).__name__}: {e}") from e

    def output(self, name: str) -> torch.Tensor:
        """The full output vector of matrix `name` assembled from the gathered slices (valid
        after gather(); a new tensor)."""
        m = self.mats[name]
        parts = [self.gathered[r * self.local_len + m.offs[r]:
                               r * self.local_len + m.offs[r] + len(m.slices[r])]
                 for r in range(self.world)]
        return torch.cat(parts)
