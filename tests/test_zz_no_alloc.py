"""The no-allocation W4A8 GEMV entry point (ks_b200_matvec_w4a8_f16_noalloc).

Callers that must not let a library allocate memory -- loops that reserve all
device memory up front, processes whose device memory belongs to their own
allocator, threads where an allocation is not allowed -- use this entry point.
Its scratch is a fixed array in device memory rather than allocations made on
first use.  It runs the same kernels as the allocating entry point,
ks_b200_matvec_w4a8_f16, so its results must be bitwise the same on every
call; the scratch array keeps the previous call's contents, so calls are
checked two in a row.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

SX = 0.02
W4A8_REL_TOL = 1e-4  # the W4A8 tolerance of the other parity tests

# (rows, cols, group): the streaming kernel at the benchmark shape, the two
# size limits of the fixed array, and an odd column count (generic kernel)
SHAPES = [(11008, 4096, 32), (64, 16384, 32), (131072, 256, 32), (300, 4095, 32)]


def _inputs(seed, rows, cols, group):
    x = O.rng(seed, 0).integers(-127, 128, cols, dtype=np.int8)
    w = O.rng(seed, 1).integers(0, 256, (rows, (cols + 1) // 2), dtype=np.uint8)
    s = O.rng(seed, 2).uniform(1e-3, 1e-2, (rows, -(-cols // group))).astype(np.float16)
    return x, w, s


def _call(ks, name, x, dw, ds, y, rows, cols, group):
    fn = getattr(ks.lib(), name)
    return fn(ks.addr(x), ks.addr(dw), (cols + 1) // 2, ks.addr(ds), -(-cols // group), ks.addr(y), rows, cols,
              group, SX, 0, 0)


def _allocating(ks, x, dw, ds, rows, cols, group):
    """The existing allocating entry point on the same inputs."""
    y = np.zeros(rows, np.float32)
    assert _call(ks, "ks_b200_matvec_w4a8_f16", x, dw, ds, y, rows, cols, group) == 0, ks.last_error()
    return y


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_no_alloc_bitwise_equal_to_allocating_entry(ks, cuda, oracle, shape):
    import torch

    rows, cols, group = shape
    x1, w, s = _inputs(101, rows, cols, group)
    x2 = O.rng(202, 0).integers(-127, 128, cols, dtype=np.int8)
    dw = torch.from_numpy(w).to(cuda)
    ds = torch.from_numpy(s.view(np.uint16)).to(cuda)
    outs = []
    # host activations and outputs, twice in a row with different inputs
    for x in (x1, x2):
        y = np.full(rows, np.nan, np.float32)
        assert _call(ks, "ks_b200_matvec_w4a8_f16_noalloc", x, dw, ds, y, rows, cols, group) == 0, ks.last_error()
        ref = _allocating(ks, x, dw, ds, rows, cols, group)
        np.testing.assert_array_equal(y.view(np.uint32), ref.view(np.uint32))
        outs.append(y)
    assert not np.array_equal(outs[0], outs[1])
    # device activations and outputs (used in place), twice in a row
    for x in (x2, x1):
        dx = torch.from_numpy(x).to(cuda)
        dy = torch.full((rows,), float("nan"), dtype=torch.float32, device=cuda)
        assert _call(ks, "ks_b200_matvec_w4a8_f16_noalloc", dx, dw, ds, dy, rows, cols, group) == 0, ks.last_error()
        np.testing.assert_array_equal(dy.cpu().numpy().view(np.uint32),
                                      _allocating(ks, x, dw, ds, rows, cols, group).view(np.uint32))
    # and once directly against the oracle (sampled rows of the large shapes)
    pick = np.unique(np.concatenate([[0, rows - 1], O.rng(5, 9).integers(0, rows, min(rows, 512))]))
    _, y_ref = oracle.matvec_w4a8_f16(x1, np.ascontiguousarray(w[pick]), (cols + 1) // 2,
                                      np.ascontiguousarray(s[pick]).view(np.uint16), -(-cols // group), len(pick),
                                      cols, group, SX)
    ok, worst = O.w4a8_tolerance_ok(outs[0][pick], y_ref, W4A8_REL_TOL)
    assert ok, f"worst err/bound {worst}"


@pytest.mark.parametrize("out_on", ["host", "device"])
def test_no_alloc_bad_scale_leaves_rows_like_the_reference(ks, cuda, oracle, out_on):
    """A bad scale is reported; rows before the first bad row hold results,
    that row and the later ones keep their contents (as in the reference and
    in the allocating entry point); the next good call is not affected by the
    status word the bad call left in the shared scratch array."""
    import torch

    rows, cols, group = 11008, 4096, 32
    x, w, s = _inputs(303, rows, cols, group)
    dw = torch.from_numpy(w).to(cuda)
    bad = s.copy()
    bad[500, 3] = np.float16(0.0)
    bad[9000, 1] = np.float16(np.nan)
    dbad = torch.from_numpy(bad.view(np.uint16)).to(cuda)
    fill = np.linspace(-3, 3, rows).astype(np.float32)
    results = []
    for name in ("ks_b200_matvec_w4a8_f16_noalloc", "ks_b200_matvec_w4a8_f16"):
        y = torch.from_numpy(fill.copy()).to(cuda) if out_on == "device" else fill.copy()
        assert _call(ks, name, x, dw, dbad, y, rows, cols, group) == ks.KS_ERR_INVALID_ARG
        results.append(y.cpu().numpy() if out_on == "device" else y)
    np.testing.assert_array_equal(results[0].view(np.uint32), results[1].view(np.uint32))
    o = fill.copy()
    rc, _ = oracle.matvec_w4a8_f16(x, w, cols // 2, bad.view(np.uint16), cols // group, rows, cols, group, SX, out=o)
    assert rc == -1
    ok, worst = O.w4a8_tolerance_ok(results[0][:500], o[:500], W4A8_REL_TOL)
    assert ok, worst
    np.testing.assert_array_equal(results[0][500:].view(np.uint32), o[500:].view(np.uint32))
    ds = torch.from_numpy(s.view(np.uint16)).to(cuda)
    y = np.zeros(rows, np.float32)
    assert _call(ks, "ks_b200_matvec_w4a8_f16_noalloc", x, dw, ds, y, rows, cols, group) == 0
    np.testing.assert_array_equal(y.view(np.uint32), _allocating(ks, x, dw, ds, rows, cols, group).view(np.uint32))


def test_no_alloc_rejects_what_it_cannot_serve(ks, cuda):
    """Sizes beyond the fixed array and host-resident weights are valid
    arguments this entry point cannot serve: KS_ERR_UNSUPPORTED."""
    import torch

    L = ks.lib()
    x = np.zeros(32768, np.int8)
    dw = torch.zeros(16, dtype=torch.uint8, device=cuda)
    ds = torch.zeros(8, dtype=torch.uint16, device=cuda)
    y = np.zeros(8, np.float32)
    # cols beyond 16384
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), 16400, ks.addr(ds), 1024, ks.addr(y),
                                             1, 32768, 32, 1.0, 0, 0) == ks.KS_ERR_UNSUPPORTED
    assert "16384" in ks.last_error()
    # rows beyond 131072
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), 16, ks.addr(ds), 1, ks.addr(y),
                                             131073, 32, 32, 1.0, 0, 0) == ks.KS_ERR_UNSUPPORTED
    assert "131072" in ks.last_error()
    # weights in host memory are not staged
    hw = np.zeros(16, np.uint8)
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(hw), 16, ks.addr(ds), 1, ks.addr(y), 1, 32, 32,
                                             1.0, 0, 0) == ks.KS_ERR_UNSUPPORTED
    assert "device memory" in ks.last_error()
    # invalid arguments keep the reference's code
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), 16, ks.addr(ds), 1, ks.addr(y), 1, 32, 0,
                                             1.0, 0, 0) == ks.KS_ERR_INVALID_ARG


def test_no_alloc_keeps_the_callers_current_device(ks, cuda):
    """The call makes the weights' device current for its work and puts the
    caller's current device back; with two GPUs, a device output on the other
    GPU is refused."""
    import torch

    rows, cols, group = 256, 512, 32
    x, w, s = _inputs(404, rows, cols, group)
    dw = torch.from_numpy(w).to(cuda)
    ds = torch.from_numpy(s.view(np.uint16)).to(cuda)
    y = np.zeros(rows, np.float32)
    n = torch.cuda.device_count()
    other = 1 if n > 1 else 0
    torch.cuda.set_device(other)
    try:
        assert _call(ks, "ks_b200_matvec_w4a8_f16_noalloc", x, dw, ds, y, rows, cols, group) == 0
        assert torch.cuda.current_device() == other
        if n > 1:
            dy = torch.zeros(rows, dtype=torch.float32, device=torch.device("cuda", 1))
            assert _call(ks, "ks_b200_matvec_w4a8_f16_noalloc", x, dw, ds, dy, rows, cols, group) == \
                ks.KS_ERR_INVALID_ARG
            assert "different devices" in ks.last_error()
    finally:
        torch.cuda.set_device(cuda)
