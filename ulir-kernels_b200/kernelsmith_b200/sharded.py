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

import ctypes
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


class PeerGatherW4A8:
    """Sharded W4A8 batch whose outputs are gathered by peer stores over NVLink.

    Every rank holds `rows` rows (its block) of each of up to `count` matrices
    and a gathered buffer `y` of shape [count, world * rows]: after `run()` and
    the arrival wait it queues, y[m] is the full output of matrix m on every
    rank.  The buffers are exchanged once with CUDA IPC; the data path is the
    GEMV kernel's own stores plus a one-warp arrival wait -- no collective
    library.  Each rank keeps one arrival counter word per source rank
    (`sync[s]` counts the CTA signals from rank s), so the wait checks every
    source separately.  Use two instances (or alternate buffers) when a
    consumer of y may still be reading while the next run starts.

    Create and close on every rank in the same order (the constructor runs one
    all_gather_object on `group`).  `timeout_ns` bounds each wait (0: the
    library's one second).
    """

    EXPECTED_WORD = 32  # sync[0:world]: counters per source rank; sync[32]: the wait's running target

    def __init__(self, count: int, rows: int, device, group=None, timeout_ns: int = 0):
        import torch
        import torch.distributed as dist

        import kernelsmith_b200 as K

        self.K = K
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.count, self.rows = count, rows
        self.timeout_ns = timeout_ns
        self.y = torch.zeros((count, self.world * rows), dtype=torch.float32, device=device)
        self.sync = torch.zeros(64, dtype=torch.int32, device=device)
        self.status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=device)
        mine = []
        for t in (self.y, self.sync):
            h = (ctypes.c_ubyte * K.IPC_HANDLE_BYTES)()
            off = ctypes.c_size_t()
            K.check(K.lib().ks_b200_ipc_get_handle(t.data_ptr(), h, ctypes.byref(off)))
            mine.append((bytes(h), off.value))
        everyone = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(everyone, mine, group=group)
        else:
            everyone = [mine]
        self._opened = []
        y_ptrs, c_ptrs = [], []
        for p in range(self.world):
            if p == self.rank:
                y_ptrs.append(self.y.data_ptr())
                c_ptrs.append(self.sync.data_ptr() + 4 * self.rank)
                continue
            ptrs = []
            for hb, off in everyone[p]:
                out = ctypes.c_void_p()
                K.check(K.lib().ks_b200_ipc_open_handle((ctypes.c_ubyte * len(hb)).from_buffer_copy(hb), off,
                                                        ctypes.byref(out)))
                self._opened.append((out.value, off))
                ptrs.append(out.value)
            y_ptrs.append(ptrs[0])
            c_ptrs.append(ptrs[1] + 4 * self.rank)  # rank p's word for arrivals from this rank
        self._y_ptrs = list(y_ptrs)
        self._c_ptrs = (ctypes.c_void_p * self.world)(*c_ptrs)

    def run(self, xs, ws, ss, cols, group, sx, scale_type, stream=None, w_stride=None, s_stride=None,
            wait: bool = True, m0: int = 0) -> int:
        """Queue this rank's GEMVs (gathered by peer stores into y[m0 : m0 + len(xs)])
        and, if `wait`, the arrival wait.

        Returns the signals each rank receives from this rank (the arrivals
        to pass to wait() when several runs share one wait).
        """
        K = self.K
        n = len(xs)
        assert m0 + n <= self.count and len(ws) == len(ss) == n
        sig = ctypes.c_uint32()
        row_bytes = self.world * self.rows * 4
        y_ptrs = (ctypes.c_void_p * self.world)(*[p + m0 * row_bytes for p in self._y_ptrs])
        K.check(K.lib().ks_b200_matvec_w4a8_batch_gather_async(
            n, K._ptr_array(xs), K._ptr_array(ws), K._ptr_array(ss), self.world, y_ptrs, self._c_ptrs,
            self.world * self.rows, self.rank * self.rows, w_stride or cols // 2, scale_type,
            s_stride or cols // group, self.rows, cols, group, sx, 0, 0,
            ctypes.byref(sig), K.addr(self.status), K.stream_handle(stream)))
        if wait:
            self.wait(sig.value, stream)
        return sig.value

    def wait(self, signals_per_rank: int, stream=None) -> None:
        """Queue the wait for every rank's signals of the preceding runs."""
        K = self.K
        K.check(K.lib().ks_b200_peer_arrival_wait_ranks_async(
            self.sync.data_ptr(), self.world, self.sync.data_ptr() + 4 * self.EXPECTED_WORD, signals_per_rank,
            self.timeout_ns, K.addr(self.status), K.stream_handle(stream)))

    def close(self) -> None:
        for ptr, off in self._opened:
            self.K.lib().ks_b200_ipc_close_handle(ptr, off)
        self._opened = []


class NcclGatherW4A8:
    """The same sharded W4A8 batch with the output slices gathered by NCCL.

    Each rank computes its rows of `count` matrices into `y_local` [count,
    rows] with one batched GEMV launch on `stream`, then
    `all_gather_into_tensor` (on `comm_stream` if given, after the launch)
    fills `y_all` [world, count, rows]: full(m) is matrix m's full output.
    Every rank issues the same collectives in the same order.
    """

    def __init__(self, count: int, rows: int, device, group=None):
        import torch
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.count, self.rows = count, rows
        self.y_local = torch.zeros((count, rows), dtype=torch.float32, device=device)
        self.y_all = torch.zeros((self.world, count, rows), dtype=torch.float32, device=device)
        self.status = None

    def run(self, xs, ws, ss, cols, group, sx, scale_type, stream=None, comm_stream=None, status=None,
            w_stride=None, s_stride=None) -> None:
        import torch
        import torch.distributed as dist

        import kernelsmith_b200 as K

        n = len(xs)
        assert n <= self.count
        K.matvec_w4a8_batch_async(xs, ws, ss, [self.y_local[m] for m in range(n)], w_stride or cols // 2,
                                  s_stride or -(-cols // group), self.rows, cols, group, sx, scale_type=scale_type,
                                  status=status, stream=stream)
        cur = stream or torch.cuda.current_stream()
        if self.world == 1:
            with torch.cuda.stream(cur):
                self.y_all[0].copy_(self.y_local)
            return
        if comm_stream is None:
            with torch.cuda.stream(cur):
                dist.all_gather_into_tensor(self.y_all, self.y_local, group=self.group)
            return
        ev = torch.cuda.Event()
        ev.record(cur)
        comm_stream.wait_event(ev)
        with torch.cuda.stream(comm_stream):
            dist.all_gather_into_tensor(self.y_all, self.y_local, group=self.group)

    def full(self, m: int):
        """Matrix m's gathered output, [world * rows] (a copy)."""
        return self.y_all[:, m, :].reshape(-1)
