"""Row-sharded W4A8 GEMV across 2 GPUs, the large sharded configuration:
K = 8192 with N = 28672 (a 70B-class MLP up-projection) and N = 128256 (an
LM head), int4 group 128, f16 scales, int8 x replicated on every rank.  Each
rank holds its contiguous row block resident and the output slices are
gathered to every rank two ways:

  peer  the GEMV kernel stores each CTA's rows straight into every rank's
        gathered buffer (CUDA IPC pointers, plain coalesced stores, no
        multicast) and a bounded arrival wait closes the run;
  nccl  the GEMV writes local slices and NCCL all-gathers them.

Rows are independent (the reference's functions are reentrant,
include/kernelsmith/ks_quantized.h:12), so every rank's gathered output must
be bitwise the single-GPU result of the full matrix, and on sampled rows
within the W4A8 tolerance of the oracle.  One process per GPU; needs at least
2 GPUs (skipped otherwise).  NVLS is off (NCCL_NVLS_ENABLE=0).
"""

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

COLS, GROUP, SX = 8192, 128, 0.02
# (name, rows, matrices per run): two matrices take the batched kernel, one
# the single-GEMV kernel; both carry the fused gather
SHAPES = [("up_28672", 28672, 2), ("lm_head_128256", 128256, 1)]
GATHERS = ["peer", "nccl"]
SAMPLE_ROWS = 256


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


def _matrices(name, rows, count):
    """Full matrices, identical in every process (seeded numpy)."""
    import oracle as O

    seed = 20261201 + sum(map(ord, name))
    xs = [O.rng(seed, 10 * m).integers(-127, 128, COLS, dtype=np.int8) for m in range(count)]
    ws = [O.rng(seed, 10 * m + 1).integers(0, 256, (rows, COLS // 2), dtype=np.uint8) for m in range(count)]
    ss = [O.rng(seed, 10 * m + 2).uniform(1e-3, 1e-2, (rows, COLS // GROUP)).astype(np.float16)
          for m in range(count)]
    return xs, ws, ss


def _worker(rank, world, port, q):
    for p in (ROOT / "oracle", ROOT / "ulir-kernels_b200"):
        sys.path.insert(0, str(p))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist

    import kernelsmith_b200 as K
    import oracle as O
    from kernelsmith_b200.sharded import NcclGatherW4A8, PeerGatherW4A8

    results = {}
    opened = []
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        orc = O.Oracle()
        stream = torch.cuda.Stream(device=dev)
        for name, rows, count in SHAPES:
            R = rows // world
            xs, ws, ss = _matrices(name, rows, count)
            dx = [torch.from_numpy(x).to(dev) for x in xs]
            dw = [torch.from_numpy(np.ascontiguousarray(w[rank * R:(rank + 1) * R])).to(dev) for w in ws]
            ds = [torch.from_numpy(np.ascontiguousarray(s[rank * R:(rank + 1) * R]).view(np.uint16)).to(dev)
                  for s in ss]
            # single-GPU reference on this GPU: the full matrices
            full = []
            for m in range(count):
                y1 = torch.zeros(rows, dtype=torch.float32, device=dev)
                K.matvec_w4a8_async(dx[m], torch.from_numpy(ws[m]).to(dev), COLS // 2,
                                    torch.from_numpy(ss[m].view(np.uint16)).to(dev), COLS // GROUP, y1, rows, COLS,
                                    GROUP, SX, scale_type=K.SCALE_F16)
                full.append(y1)
            torch.cuda.synchronize()
            pick = np.sort(O.rng(rank + 7, 99).choice(rows, SAMPLE_ROWS, replace=False))
            pick[0], pick[-1] = 0, rows - 1
            oracle_rows = []
            for m in range(count):
                _, yr = orc.matvec_w4a8_f16(xs[m], np.ascontiguousarray(ws[m][pick]), COLS // 2,
                                            np.ascontiguousarray(ss[m][pick]).view(np.uint16), COLS // GROUP,
                                            len(pick), COLS, GROUP, SX)
                oracle_rows.append(yr)
            for gather in GATHERS:
                stream.wait_stream(torch.cuda.current_stream(dev))  # zero-filled buffers first
                if gather == "peer":
                    pg = PeerGatherW4A8(count, R, dev, timeout_ns=5_000_000_000)
                    opened.append(pg)
                    with torch.cuda.stream(stream):
                        for _ in range(3):  # counters and targets keep growing across runs
                            pg.run(dx, dw, ds, COLS, GROUP, SX, K.SCALE_F16, stream=stream)
                    stream.synchronize()
                    status = pg.status.cpu().tolist()
                    outs = [pg.y[m] for m in range(count)]
                else:
                    ng = NcclGatherW4A8(count, R, dev)
                    st = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
                    with torch.cuda.stream(stream):
                        for _ in range(2):
                            ng.run(dx, dw, ds, COLS, GROUP, SX, K.SCALE_F16, stream=stream, status=st)
                    stream.synchronize()
                    status = st.cpu().tolist()
                    outs = [ng.full(m) for m in range(count)]
                bitwise = all(torch.equal(outs[m], full[m]) for m in range(count))
                tol = []
                for m in range(count):
                    ok, worst = O.w4a8_tolerance_ok(outs[m].cpu().numpy()[pick], oracle_rows[m])
                    tol.append((bool(ok), float(worst)))
                results[(name, gather)] = {"status": status, "bitwise": bool(bitwise), "oracle": tol}
                dist.barrier()
                if gather == "peer":
                    pg.close()
                    opened.remove(pg)
            del dx, dw, ds, full
            torch.cuda.empty_cache()
        q.put((rank, "ok", results))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, "error", repr(e)))
    finally:
        for pg in opened:
            pg.close()
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.fixture(scope="module")
def two_gpu_results():
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, kind, val = q.get(timeout=900)
            res[rank] = (kind, val)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for rank in (0, 1):
        assert rank in res and res[rank][0] == "ok", res
    return {rank: res[rank][1] for rank in (0, 1)}


@pytest.mark.parametrize("gather", GATHERS)
@pytest.mark.parametrize("name", [s[0] for s in SHAPES])
def test_sharded_two_gpus_match_single_gpu(two_gpu_results, name, gather):
    for rank in (0, 1):
        r = two_gpu_results[rank][(name, gather)]
        assert r["status"] == [0, 0], (rank, r)
        assert r["bitwise"], f"rank {rank}: gathered output differs from the single-GPU result"
        for ok, worst in r["oracle"]:
            assert ok, f"rank {rank}: sampled rows vs oracle, worst err/bound {worst:.3g}"
