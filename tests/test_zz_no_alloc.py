"""The no-allocation W4A8 GEMV entry point (ks_b200_matvec_w4a8_f16_noalloc).

Callers that must not let a library allocate memory -- loops that reserve all
device memory up front, processes whose device memory belongs to their own
allocator, threads where an allocation is not allowed -- use this entry point.
Its scratch is a fixed array in device memory rather than allocations made on
first use.  Its results must match the allocating entry point,
ks_b200_matvec_w4a8_f16, on every call; the scratch array keeps the previous
call's contents, so two calls in a row are checked.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

ROWS, COLS, GROUP, SX = 11008, 4096, 32, 0.02
W4A8_REL_TOL = 1e-4  # the W4A8 tolerance of the other parity tests


def _inputs(seed):
    x = O.rng(seed, 0).integers(-127, 128, COLS, dtype=np.int8)
    w = O.pack_int4(O.rng(seed, 1).integers(-8, 8, (ROWS, COLS), dtype=np.int8))
    s = O.rng(seed, 2).uniform(1e-3, 1e-2, (ROWS, COLS // GROUP)).astype(np.float16)
    return x, w, s


def _reference_entry(ks, x, dw, ds):
    """The existing allocating entry point on the same inputs."""
    y = np.zeros(ROWS, np.float32)
    rc = ks.lib().ks_b200_matvec_w4a8_f16(ks.addr(x), ks.addr(dw), COLS // 2, ks.addr(ds), COLS // GROUP,
                                          ks.addr(y), ROWS, COLS, GROUP, SX, 0, 0)
    assert rc == 0, ks.last_error()
    return y


def test_no_alloc_matches_allocating_entry_two_calls(ks, cuda):
    import torch

    L = ks.lib()
    x1, w, s = _inputs(101)
    x2 = O.rng(202, 0).integers(-127, 128, COLS, dtype=np.int8)
    dw = torch.from_numpy(w).to(cuda)
    ds = torch.from_numpy(s.view(np.uint16)).to(cuda)
    # host activations and outputs, twice in a row with different inputs
    outs = []
    for x in (x1, x2):
        y = np.full(ROWS, np.nan, np.float32)
        rc = L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), COLS // 2, ks.addr(ds), COLS // GROUP,
                                               ks.addr(y), ROWS, COLS, GROUP, SX, 0, 0)
        assert rc == 0, ks.last_error()
        ref = _reference_entry(ks, x, dw, ds)
        ok, worst = O.w4a8_tolerance_ok(y, ref, W4A8_REL_TOL)
        assert ok, f"worst err/bound {worst}"
        outs.append(y)
    assert not np.array_equal(outs[0], outs[1])
    # device activations and outputs, twice in a row
    for x in (x2, x1):
        dx = torch.from_numpy(x).to(cuda)
        dy = torch.full((ROWS,), float("nan"), dtype=torch.float32, device=cuda)
        rc = L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(dx), ks.addr(dw), COLS // 2, ks.addr(ds), COLS // GROUP,
                                               ks.addr(dy), ROWS, COLS, GROUP, SX, 0, 0)
        assert rc == 0, ks.last_error()
        ok, worst = O.w4a8_tolerance_ok(dy.cpu().numpy(), _reference_entry(ks, x, dw, ds), W4A8_REL_TOL)
        assert ok, f"worst err/bound {worst}"


def test_no_alloc_status_cleared_between_calls(ks, cuda):
    """A bad scale is reported, and the next good call is not affected by the
    status word the bad call left in the shared scratch array."""
    import torch

    L = ks.lib()
    x, w, s = _inputs(303)
    dw = torch.from_numpy(w).to(cuda)
    bad = s.copy()
    bad[500, 3] = np.float16(0.0)
    y = np.zeros(ROWS, np.float32)
    dbad = torch.from_numpy(bad.view(np.uint16)).to(cuda)
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), COLS // 2, ks.addr(dbad), COLS // GROUP,
                                             ks.addr(y), ROWS, COLS, GROUP, SX, 0, 0) == ks.KS_ERR_INVALID_ARG
    ds = torch.from_numpy(s.view(np.uint16)).to(cuda)
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), COLS // 2, ks.addr(ds), COLS // GROUP,
                                             ks.addr(y), ROWS, COLS, GROUP, SX, 0, 0) == 0
    ok, worst = O.w4a8_tolerance_ok(y, _reference_entry(ks, x, dw, ds), W4A8_REL_TOL)
    assert ok, worst


def test_no_alloc_rejects_sizes_beyond_its_limit(ks, cuda):
    import torch

    L = ks.lib()
    x = np.zeros(32768, np.int8)
    dw = torch.zeros(16, dtype=torch.uint8, device=cuda)
    ds = torch.zeros(8, dtype=torch.uint16, device=cuda)
    y = np.zeros(8, np.float32)
    # cols beyond 16384
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), 16400, ks.addr(ds), 1024, ks.addr(y),
                                             1, 32768, 32, 1.0, 0, 0) == ks.KS_ERR_INVALID_ARG
    assert "16384" in ks.last_error()
    # rows beyond 131072
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(dw), 16, ks.addr(ds), 1, ks.addr(y),
                                             131073, 32, 32, 1.0, 0, 0) == ks.KS_ERR_INVALID_ARG
    assert "131072" in ks.last_error()
    # weights in host memory are not staged
    hw = np.zeros(16, np.uint8)
    assert L.ks_b200_matvec_w4a8_f16_noalloc(ks.addr(x), ks.addr(hw), 16, ks.addr(ds), 1, ks.addr(y), 1, 32, 32,
                                             1.0, 0, 0) == ks.KS_ERR_INVALID_ARG
    assert "device memory" in ks.last_error()
