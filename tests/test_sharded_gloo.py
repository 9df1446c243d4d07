"""Row-sharded GEMV host logic on CPU: world_size-2 gloo ranks, the oracle as
each rank's compute, NCCL's role played by gloo.  Rows are independent, so the
gathered vector must be bitwise the single-process oracle result.  A rank that
fails before the gather must make the other rank's collective fail within the
process-group timeout instead of hanging."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, cols, group, fail_rank, q):
    for p in (ROOT / "oracle", ROOT / "ulir-kernels_b200"):
        sys.path.insert(0, str(p))
    import torch
    import torch.distributed as dist

    import oracle as O
    from kernelsmith_b200.sharded import RowSharding, sharded_gemv_allgather

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
        orc = O.Oracle()
        g = np.random.default_rng(77)
        x = g.integers(-128, 128, cols, dtype=np.int8)
        w = g.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        s = g.uniform(1e-3, 1e-2, (rows, cols // group)).astype(np.float32)
        sh = RowSharding(rows, world, rank)
        r0, r1 = sh.bounds

        def compute(out):
            if rank == fail_rank:
                raise RuntimeError("injected failure before the gather")
            _, y = orc.matvec_w4a8(x, np.ascontiguousarray(w[r0:r1]), cols // 2, np.ascontiguousarray(s[r0:r1]),
                                   cols // group, r1 - r0, cols, group, 0.05)
            out.copy_(torch.from_numpy(y))

        y_slot = torch.zeros(sh.slot, dtype=torch.float32)
        y_all = torch.zeros(world * sh.slot, dtype=torch.float32)
        sharded_gemv_allgather(sh, compute, y_slot, y_all)
        full = sh.unpack(y_all).numpy()
        _, ref = orc.matvec_w4a8(x, w, cols // 2, s, cols // group, rows, cols, group, 0.05)
        q.put((rank, "ok", bool(np.array_equal(full.view(np.uint32), ref.view(np.uint32)))))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, rows, cols, group, fail_rank=-1, timeout=60):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, cols, group, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, kind, val = q.get(timeout=timeout)
        results[rank] = (kind, val)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


def test_shard_rows_partition():
    from kernelsmith_b200.sharded import padded_shard, shard_rows

    for rows in (1, 7, 11008, 28672, 128256):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
            assert max(sizes) == padded_shard(rows, world) or rows < world
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


@pytest.mark.parametrize("rows", [64, 11])
def test_two_rank_gather_matches_single_oracle(rows):
    res = _run(2, rows, 256, 32)
    assert res[0] == ("ok", True) and res[1] == ("ok", True), res


def test_failed_rank_does_not_hang_the_other():
    res = _run(2, 64, 256, 32, fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    # rank 0's all-gather ends with an error (peer gone / timeout), not a hang
    assert res[0][0] == "error", res
