"""Batched (grouped) GEMV launches: every matrix of a batch must give bitwise
the same output as its own single launch, and match the oracle."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _w4a8_set(seed, n, rows, cols, group, f16=True):
    xs, ws, ss = [], [], []
    for i in range(n):
        g = np.random.default_rng(seed * 1000 + i)
        xs.append(g.integers(-128, 128, cols, dtype=np.int8))
        ws.append(g.integers(0, 256, (rows, cols // 2), dtype=np.uint8))
        ss.append(g.uniform(1e-3, 1e-2, (rows, cols // group)).astype(np.float16 if f16 else np.float32))
    return xs, ws, ss


def _to(torch, cuda, arrs, view16=False):
    return [torch.from_numpy(a.view(np.uint16) if view16 else a).to(cuda) for a in arrs]


@pytest.mark.parametrize("case", [
    # n, rows, cols, group, f16, zx, zw
    (5, 3000, 4096, 32, True, 0, 0),
    (3, 1000, 8192, 128, True, 0, 0),
    (2, 500, 16384, 32, False, 3, -2),
    (70, 40, 256, 32, True, 0, 0),       # more than one launch (64 per launch)
    (4, 7, 1024, 64, False, -9, 1),      # fewer rows than SMs
])
def test_w4a8_batch_matches_single_and_oracle(ks, cuda, oracle, case):
    import torch

    n, rows, cols, group, f16, zx, zw = case
    xs, ws, ss = _w4a8_set(sum(case[:4]), n, rows, cols, group, f16)
    dx, dw, ds = _to(torch, cuda, xs), _to(torch, cuda, ws), _to(torch, cuda, ss, view16=f16)
    ys = [torch.zeros(rows, dtype=torch.float32, device=cuda) for _ in range(n)]
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    st = ks.SCALE_F16 if f16 else ks.SCALE_F32
    ks.matvec_w4a8_batch_async(dx, dw, ds, ys, cols // 2, cols // group, rows, cols, group, 0.03, zx, zw,
                               scale_type=st, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    for i in range(n):
        y1 = torch.zeros(rows, dtype=torch.float32, device=cuda)
        ks.matvec_w4a8_async(dx[i], dw[i], cols // 2, ds[i], cols // group, y1, rows, cols, group, 0.03, zx, zw,
                             scale_type=st)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ys[i].cpu().numpy().view(np.uint32), y1.cpu().numpy().view(np.uint32))
    for i in (0, n - 1):
        if f16:
            _, y_ref = oracle.matvec_w4a8_f16(xs[i], ws[i], cols // 2, ss[i].view(np.uint16), cols // group, rows,
                                              cols, group, 0.03, zx, zw)
        else:
            _, y_ref = oracle.matvec_w4a8(xs[i], ws[i], cols // 2, ss[i], cols // group, rows, cols, group, 0.03,
                                          zx, zw)
        ok, worst = O.w4a8_tolerance_ok(ys[i].cpu().numpy(), y_ref)
        assert ok, worst


def test_w4a8_batch_bad_scale_sets_status(ks, cuda):
    import torch

    n, rows, cols, group = 6, 2000, 4096, 32
    xs, ws, ss = _w4a8_set(3, n, rows, cols, group)
    ss[4][1234, 77] = np.float16(np.nan)
    dx, dw, ds = _to(torch, cuda, xs), _to(torch, cuda, ws), _to(torch, cuda, ss, view16=True)
    ys = [torch.zeros(rows, dtype=torch.float32, device=cuda) for _ in range(n)]
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    ks.matvec_w4a8_batch_async(dx, dw, ds, ys, cols // 2, cols // group, rows, cols, group, 0.03, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [1, 0]


@pytest.mark.parametrize("dequant", [False, True])
def test_i8_batch_matches_single(ks, cuda, oracle, dequant):
    import torch

    n, rows, cols = 6, 4096, 4096
    g = np.random.default_rng(9)
    xs = [g.integers(-128, 128, cols, dtype=np.int8) for _ in range(n)]
    ws = [g.integers(-128, 128, (rows, cols), dtype=np.int8) for _ in range(n)]
    sc = [g.uniform(1e-3, 1e-2, rows).astype(np.float32) for _ in range(n)]
    dx, dw, ds = _to(torch, cuda, xs), _to(torch, cuda, ws), _to(torch, cuda, sc)
    dt = torch.float32 if dequant else torch.int32
    ys = [torch.zeros(rows, dtype=dt, device=cuda) for _ in range(n)]
    ks.matvec_i8_batch_async(dx, dw, ys, cols, rows, cols, 2, -3, w_scales=ds if dequant else None, sa=0.02)
    torch.cuda.synchronize()
    for i in range(n):
        if dequant:
            _, ref = oracle.matvec_i8_dequant(xs[i], ws[i], rows, cols, cols, sc[i], 0.02, 2, -3)
            np.testing.assert_array_equal(ys[i].cpu().numpy().view(np.uint32), ref.view(np.uint32))
        else:
            _, ref = oracle.matvec_i8(xs[i], ws[i], rows, cols, cols, 2, -3)
            np.testing.assert_array_equal(ys[i].cpu().numpy(), ref)


def test_w4a8_batch_graph_capture(ks, cuda):
    import torch

    n, rows, cols, group = 8, 11008, 4096, 32
    xs, ws, ss = _w4a8_set(4, n, rows, cols, group)
    dx, dw, ds = _to(torch, cuda, xs), _to(torch, cuda, ws), _to(torch, cuda, ss, view16=True)
    ys = [torch.zeros(rows, dtype=torch.float32, device=cuda) for _ in range(n)]
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())  # zero-filled outputs first
    with torch.cuda.stream(stream):
        ks.matvec_w4a8_batch_async(dx, dw, ds, ys, cols // 2, cols // group, rows, cols, group, 0.03, stream=stream)
    stream.synchronize()
    ref = [y.clone() for y in ys]
    for y in ys:
        y.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        ks.matvec_w4a8_batch_async(dx, dw, ds, ys, cols // 2, cols // group, rows, cols, group, 0.03,
                                   stream=torch.cuda.current_stream())
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(ys, ref):
        assert torch.equal(a, b)
