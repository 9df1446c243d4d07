"""Row-sharded GEMV across the ranks of a torch.distributed process group.

A GEMV's rows are independent, so a weight matrix is split into contiguous row
blocks, one per rank; each rank keeps its block resident on its own GPU,
computes those outputs, and the output slices are all-gathered so every rank
ends with the full vector.  Each rank's slice is bitwise the single-GPU result
for those rows.  The input vector is replicated.

One process per GPU; the collective is NCCL over NVLink on GPUs (gloo on CPU
for the host-logic tests).  Every rank takes the same collective steps in the
same order.  The per-rank compute is injectable so the partition and gather
logic can be tested on CPU against the oracle; on a GPU it is the library's
asynchronous GEMV on the caller's stream.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous row block [r0, r1) of `rank`: the first rows % world ranks get one more row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(rows, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def padded_shard(rows: int, world: int) -> int:
    """Per-rank slot length of the gathered buffer (all slots equal for all-gather)."""
    return -(-rows // world)


@dataclass
class RowSharding:
    rows: int
    world: int
    rank: int

    @property
    def bounds(self) -> tuple[int, int]:
        return shard_rows(self.rows, self.world, self.rank)

    @property
    def local_rows(self) -> int:
        r0, r1 = self.bounds
        return r1 - r0

    @property
    def slot(self) -> int:
        return padded_shard(self.rows, self.world)

    def unpack(self, gathered, out=None):
        """[world * slot] gathered slots -> [rows] full vector (drops the padding)."""
        pieces = []
        for r in range(self.world):
            a, b = shard_rows(self.rows, self.world, r)
            pieces.append(gathered[r * self.slot : r * self.slot + (b - a)])
        import torch

        full = torch.cat(pieces)
        if out is not None:
            out.copy_(full)
            return out
        return full


def sharded_gemv_allgather(
    sharding: RowSharding,
    compute_local: Callable[[object], None],
    y_slot,
    y_gathered,
    group=None,
    async_op: bool = False,
):
    """Compute this rank's rows into y_slot[:local_rows] and all-gather the slots.

    compute_local(out) writes the local outputs into `out` (a view of y_slot).
    y_slot has `sharding.slot` elements, y_gathered world * slot.  Returns the
    collective's work handle when async_op, else None.
    """
    import torch.distributed as dist

    compute_local(y_slot[: sharding.local_rows])
    if sharding.world == 1:
        y_gathered[: sharding.slot].copy_(y_slot)
        return None
    return dist.all_gather_into_tensor(y_gathered, y_slot, group=group, async_op=async_op)


def w4a8_compute_fn(x, w_shard, s_shard, cols: int, group: int, sx: float, scale_type: int, status=None,
                    stream=None, zx: int = 0, zw: int = 0):
    """The library's asynchronous W4A8 GEMV over this rank's row block (GPU)."""
    import kernelsmith_b200 as K

    rows = w_shard.shape[0]
    scale_bytes = 2 if scale_type == K.SCALE_F16 else 4

    def run(out):
        K.matvec_w4a8_async(x, w_shard, w_shard.stride(0) * w_shard.element_size(), s_shard,
                            s_shard.stride(0) * s_shard.element_size() // scale_bytes, out, rows, cols, group, sx,
                            zx, zw, scale_type=scale_type, status=status, stream=stream)

    return run
