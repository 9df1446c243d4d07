"""Batched W4A8 GEMM on the tensor cores (ks_b200_gemm_w4a8_async) against the
oracle: every token's row equals the oracle W4A8 GEMV for that token within
the W4A8 tolerance (|y - y_ref| <= 1e-4 * max(|y_ref|, rms(y_ref)))."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _case(seed, m, n, k, group, f16, sstride=None):
    g = np.random.default_rng(seed)
    a = g.integers(-127, 128, (m, k), dtype=np.int8)
    sx = g.uniform(0.01, 0.03, m).astype(np.float32)
    w = g.integers(0, 256, (n, k // 2), dtype=np.uint8)
    per16 = 8 if f16 else 4  # scale rows padded to a multiple of 16 bytes
    ss = sstride or -(-(k // group) // per16) * per16
    s = g.uniform(1e-3, 1e-2, (n, ss)).astype(np.float32)
    if f16:
        s = s.astype(np.float16)
    return a, sx, w, s


def _run(ks, torch, cuda, a, sx, w, s, group, f16):
    m, k = a.shape
    n = w.shape[0]
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
    da, dsx, dw = dev(a), dev(sx), dev(w)
    ds = dev(s.view(np.uint16)) if f16 else dev(s)
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    ks.gemm_w4a8_async(da, dsx, dw, ds, y, m, n, k, group, s_stride=s.shape[1],
                       scale_type=ks.SCALE_F16 if f16 else ks.SCALE_F32, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    return y.cpu().numpy()


def _check(oracle, a, sx, w, s, group, f16, y, rows=None):
    m, k = a.shape
    rows = np.arange(w.shape[0]) if rows is None else rows
    wr = np.ascontiguousarray(w[rows])
    sr = np.ascontiguousarray(s[rows])
    for t in range(m):
        if f16:
            rc, ref = oracle.matvec_w4a8_f16(a[t], wr, k // 2, sr.view(np.uint16), s.shape[1], len(rows), k, group,
                                             float(sx[t]))
        else:
            rc, ref = oracle.matvec_w4a8(a[t], wr, k // 2, sr, s.shape[1], len(rows), k, group, float(sx[t]))
        assert rc == 0
        ok, worst = O.w4a8_tolerance_ok(y[t, rows], ref)
        assert ok, f"token {t}: worst err/bound {worst:.3g}"


@pytest.mark.parametrize("m", [8, 64])
def test_bench_shape_sampled_rows(ks, cuda, oracle, m):
    """M x 4096 x 14336, G 32, f16 scales; every token, 768 sampled weight rows."""
    import torch

    n, k, group = 14336, 4096, 32
    a, sx, w, s = _case(90 + m, m, n, k, group, True)
    y = _run(ks, torch, cuda, a, sx, w, s, group, True)
    assert np.isfinite(y).all()
    rows = np.unique(np.concatenate([np.arange(0, 256), np.arange(n - 256, n),
                                     np.random.default_rng(m).choice(n, 256, replace=False)]))
    _check(oracle, a, sx, w, s, group, True, y, rows)


@pytest.mark.parametrize("shape", [(1, 256, 128, 128, True), (16, 1000, 4096, 64, False), (33, 500, 11008, 32, True),
                                   (64, 384, 2048, 32, False), (5, 130, 512, 128, False), (48, 208, 4096, 64, True),
                                   (8, 300, 384, 32, True), (8, 300, 640, 64, True), (12, 96, 1152, 128, False),
                                   (32, 300, 2048, 32, True), (24, 200, 1024, 128, False), (64, 256, 4096, 64, True),
                                   (40, 150, 512, 128, True), (64, 200, 640, 128, False), (20, 100, 384, 64, True),
                                   (17, 64, 33 * 128, 32, False), (2, 4000, 2048, 32, True)])
def test_shapes_all_rows(ks, cuda, oracle, shape):
    import torch

    m, n, k, group, f16 = shape
    a, sx, w, s = _case(sum(shape[:4]), m, n, k, group, f16)
    y = _run(ks, torch, cuda, a, sx, w, s, group, f16)
    _check(oracle, a, sx, w, s, group, f16, y)


def test_partial_last_stage_and_padded_scale_rows(ks, cuda, oracle):
    """k = 4128 (32 past a multiple of 128): the last stage is zero-filled past
    k; scale rows padded to 136 entries (272 bytes, a multiple of 16)."""
    import torch

    m, n, k, group = 12, 200, 4128, 32
    a, sx, w, s = _case(4128, m, n, k, group, True, sstride=136)
    y = _run(ks, torch, cuda, a, sx, w, s, group, True)
    _check(oracle, a, sx, w, s, group, True, y)


def test_unsupported_shapes(ks, cuda):
    import torch

    z = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    L = ks.lib()
    p = z.data_ptr()
    U = ks.KS_ERR_UNSUPPORTED
    assert L.ks_b200_gemm_w4a8_async(p, 128, p, p, 64, p, 1, 8, p, 64, 65, 64, 128, 32, None, None) == U  # m > 64
    assert L.ks_b200_gemm_w4a8_async(p, 128, p, p, 64, p, 1, 8, p, 64, 8, 64, 128, 256, None, None) == U  # group
    assert L.ks_b200_gemm_w4a8_async(p, 130, p, p, 64, p, 1, 8, p, 64, 8, 64, 128, 32, None, None) == U  # lda % 16


@pytest.mark.parametrize("m", [1, 8, 16, 33, 64])
def test_no_bounded_wait_runs_out(ks, cuda, m):
    """Every wait in the kernel is bounded at about a second and records a
    timeout in the status word; a wait that ran out unreported would still
    give correct results, one second late.  20 launches of the bench shape
    must take far less than one second in all."""
    import torch

    n, k, group = 14336, 4096, 32
    g = torch.Generator(device=cuda)
    g.manual_seed(m)
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=cuda, generator=g)
    sx = torch.rand(m, device=cuda, generator=g) * 0.02 + 0.01
    w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=cuda, generator=g)
    s = (torch.rand((n, k // group), device=cuda, generator=g) * 9e-3 + 1e-3).half()
    y = torch.zeros((m, n), dtype=torch.float32, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    ks.gemm_w4a8_async(a, sx, w, s, y, m, n, k, group, status=status)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        ks.gemm_w4a8_async(a, sx, w, s, y, m, n, k, group, status=status)
    e1.record()
    e1.synchronize()
    assert status.cpu().tolist() == [0, 0]
    assert e0.elapsed_time(e1) < 100.0, f"20 launches took {e0.elapsed_time(e1):.1f} ms"
