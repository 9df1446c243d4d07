"""Sharded W4A8 GEMV across 2 GPUs with the gather done by peer stores over
NVLink (CUDA IPC pointers, plain stores, no multicast) and a bounded arrival
wait.  One process per GPU; needs at least 2 GPUs (skipped otherwise).  The
gathered output on every rank must be bitwise the single-GPU result of the
full matrix, since rows are independent."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    for p in (ROOT / "oracle", ROOT / "ulir-kernels_b200"):
        sys.path.insert(0, str(p))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    import kernelsmith_b200 as K
    from kernelsmith_b200.sharded import PeerGatherW4A8

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    pg = None
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        count, rows, cols, group = 3, 3000, 4096, 32
        g = np.random.default_rng(5)
        xs = [g.integers(-127, 128, cols, dtype=np.int8) for _ in range(count)]
        ws = [g.integers(0, 256, (world * rows, cols // 2), dtype=np.uint8) for _ in range(count)]
        ss = [g.uniform(1e-3, 1e-2, (world * rows, cols // group)).astype(np.float16) for _ in range(count)]
        dx = [torch.from_numpy(x).to(dev) for x in xs]
        dw = [torch.from_numpy(np.ascontiguousarray(w[rank * rows:(rank + 1) * rows])).to(dev) for w in ws]
        ds = [torch.from_numpy(np.ascontiguousarray(s[rank * rows:(rank + 1) * rows]).view(np.uint16)).to(dev)
              for s in ss]
        pg = PeerGatherW4A8(count, rows, dev)
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))  # zero-filled buffers first
        with torch.cuda.stream(stream):
            for step in range(3):  # several runs: counters and targets keep growing
                pg.run(dx, dw, ds, cols, group, 0.02, K.SCALE_F16, stream=stream)
        stream.synchronize()
        status = pg.status.cpu().tolist()
        # single-GPU reference: the full matrices on this GPU
        ok = status == [0, 0]
        for m in range(count):
            full_w = torch.from_numpy(ws[m]).to(dev)
            full_s = torch.from_numpy(ss[m].view(np.uint16)).to(dev)
            y1 = torch.zeros(world * rows, dtype=torch.float32, device=dev)
            K.matvec_w4a8_async(dx[m], full_w, cols // 2, full_s, cols // group, y1, world * rows, cols, group,
                                0.02, scale_type=K.SCALE_F16)
            torch.cuda.synchronize()
            ok = ok and torch.equal(y1, pg.y[m])
        dist.barrier()
        pg.close()
        pg = None
        q.put((rank, "ok", bool(ok), status))
    except Exception as e:
        q.put((rank, "error", repr(e), None))
    finally:
        if pg is not None:
            pg.close()
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_peer_gather_two_gpus_matches_single_gpu():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, kind, val, status = q.get(timeout=300)
        res[rank] = (kind, val, status)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res[0][:2] == ("ok", True) and res[1][:2] == ("ok", True), res
