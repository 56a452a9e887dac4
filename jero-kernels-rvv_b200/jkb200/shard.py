"""Output-row sharding of a set of GEMV/GEMM weights across GPUs (one process per GPU).

The reference splits work by disjoint output-row ranges (``gemv_repacked_rows``,
repack.rs:4014; ``gemm_repacked_rows``, :4087; stitched bit-identically in
tests/test_repack_gemv_gemm.rs:805-826). Rows are independent, so rank p of P owns rows
``shard_rows(rows, P, p)`` of every matrix, computes them with the same kernels as a
single-GPU call, and one all-gather per step collects the slices. No K split is used: it would
need an all-reduce and change the f32 summation order.

Layout of one rank's flat output buffer: the matrices in order, each contributing its slice,
padded to the largest rank's total so that ``all_gather_into_tensor`` sees equal sizes. With a
batch of m tokens a rank's slice of a matrix is its [m][rows of the shard] block (the layout
jkb_gemv_batch writes), so every rank's part stays one contiguous range; ``output()``
reassembles the [m][rows] matrix.

Two ways to collect the slices:
* ``ShardedOutputs``: each rank computes into a flat local buffer, one NCCL all-gather per step
  collects them, and ``output()`` reassembles a full vector. Failures of the collective (a peer
  that died or never joins, a process-group timeout) surface as ``CollectiveError``.
* ``PeerOutputs``: every rank holds the full output vectors in a peer-group buffer (the same
  layout on every rank) and computes its rows straight into their global positions; one kernel
  per step (jkb_peer_group_allgather) copies them to every peer over NVLink and waits for the
  peers' rows. The full vectors are then in place on every rank, in one of two slots alternated
  by step parity (a fast rank never overwrites rows a slow rank is still reading: it cannot start
  step s + 2 before every rank has finished step s). A wait that expires sets bit 1 of
  jkb200.device_status().
Every rank takes the same collective steps in the same order.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["shard_rows", "ShardedOutputs", "PeerOutputs", "CollectiveError"]


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

    def __init__(self, mats, world: int, rank: int, device="cuda", dtype=torch.float32,
                 batch: int = 1):
        self.world, self.rank, self.batch = world, rank, batch
        self.mats: dict[str, _Mat] = {}
        totals = [0] * world
        for name, rows in mats:
            slices, offs = [], []
            for r in range(world):
                sl = shard_rows(rows, world, r)
                slices.append(sl)
                offs.append(totals[r])
                totals[r] += batch * len(sl)
            self.mats[name] = _Mat(name, rows, slices, offs)
        self.local_len = max(totals)
        self.local = torch.zeros(self.local_len, dtype=dtype, device=device)
        self.gathered = (torch.empty(self.local_len * world, dtype=dtype, device=device)
                         if world > 1 else self.local)

    def rows_of(self, name: str) -> range:
        """This rank's rows of matrix `name`."""
        return self.mats[name].slices[self.rank]

    def local_slice(self, name: str) -> torch.Tensor:
        """View of this rank's output slice of matrix `name` in the flat buffer ([batch][rows
        of the shard], flattened)."""
        m = self.mats[name]
        o = m.offs[self.rank]
        return self.local[o:o + self.batch * len(m.slices[self.rank])]

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
        """The full output of matrix `name` assembled from the gathered slices (valid after
        gather(); a new tensor): [rows] for a batch of 1, else [batch][rows]."""
        m, b = self.mats[name], self.batch
        parts = [self.gathered[r * self.local_len + m.offs[r]:
                               r * self.local_len + m.offs[r] + b * len(m.slices[r])]
                 for r in range(self.world)]
        if b == 1:
            return torch.cat(parts)
        return torch.cat([p.view(b, -1) for p in parts], dim=1)


class PeerOutputs:
    """Full output vectors of a list of (name, rows) matrices in a peer-group buffer on every
    rank: rank p computes rows shard_rows(rows, world, p) of each into ``local_slice(name,
    slot)``; after ``gather(slot)`` every rank holds all rows of every matrix in
    ``output(name, slot)``. With a batch of m tokens a matrix takes m * rows floats of a slot,
    rank p's part being its [m][rows of the shard] block at offset m * (first row of the shard),
    so each rank still pushes one contiguous chunk per matrix.

    push=True: the GEMVs that write ``local_slice`` store their rows into every peer's buffer
    as they compute them (PeerGroup.set_push), and ``gather`` only signals and waits
    (PeerGroup.signal); outputs must then come from the GEMV entry points."""

    SLOTS = 2

    def __init__(self, mats, world: int, rank: int, group=None, batch: int = 1,
                 push: bool = False):
        from .api import PeerGroup

        self.world, self.rank, self.batch, self.push = world, rank, batch, push
        self.offs, self.rows = {}, {}
        total = 0
        for name, rows in mats:
            self.offs[name], self.rows[name] = total, rows
            total += batch * rows
        self.total = total
        self.pitch = (total + 3) // 4 * 4  # floats per slot (16-byte multiple)
        self.group = PeerGroup(self.SLOTS * self.pitch * 4, world, rank, group)
        if push:
            self.group.set_push(True)
        self.slots = self.group.buffer[:self.SLOTS * self.pitch].view(self.SLOTS, self.pitch)

    def rows_of(self, name: str) -> range:
        return shard_rows(self.rows[name], self.world, self.rank)

    def local_slice(self, name: str, slot: int) -> torch.Tensor:
        rr, b = self.rows_of(name), self.batch
        o = self.offs[name]
        return self.slots[slot, o + b * rr.start:o + b * rr.stop]

    def output(self, name: str, slot: int) -> torch.Tensor:
        """[rows] (a view) for a batch of 1, else the [batch][rows] matrix (a new tensor)."""
        o, b, rows = self.offs[name], self.batch, self.rows[name]
        if b == 1:
            return self.slots[slot, o:o + rows]
        parts = []
        for r in range(self.world):
            rr = shard_rows(rows, self.world, r)
            parts.append(self.slots[slot, o + b * rr.start:o + b * rr.stop].view(b, -1))
        return torch.cat(parts, dim=1)

    def full(self, slot: int) -> torch.Tensor:
        """All matrices' outputs of a slot, in list order."""
        return self.slots[slot, :self.total]

    def chunks(self, slot: int):
        """(byte offset, byte length) of this rank's rows of every matrix in a slot."""
        out, b = [], self.batch
        for name in self.offs:
            rr = self.rows_of(name)
            if len(rr):
                out.append((4 * (slot * self.pitch + self.offs[name] + b * rr.start),
                            4 * b * len(rr)))
        return out

    def gather(self, slot: int, stream=None):
        """One kernel: this rank's rows of the slot to every peer (already there with push),
        then wait for theirs."""
        if self.push:
            self.group.signal(stream)
            return
        if not hasattr(self, "_chunks"):
            self._chunks = [self.group.chunk_arrays(self.chunks(s)) for s in range(self.SLOTS)]
        self.group.allgather_arrays(self._chunks[slot], stream)

    def destroy(self):
        self.group.destroy()
