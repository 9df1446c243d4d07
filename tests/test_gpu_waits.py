"""Bounded device-side waits on one GPU.

Every spin in this library's kernels gives up after a time limit, records a
timeout in status word 1 and returns, so a lost signal can never hang the GPU.
These tests make the peer-arrival wait run out for real: its counters are
zero-filled device memory that no kernel ever increments.  Nothing faults;
the wait kernel only polls until its limit and returns.  The synchronous
status check then turns the status word into KS_ERR_DEVICE (the reference's
return codes, include/kernelsmith/ks_common.h:25-28, plus the library's -4).
"""

from __future__ import annotations

import time

import pytest

pytestmark = pytest.mark.gpu

EXPECTED = 32  # word of the running target in the 64-word sync buffer (as kernelsmith_b200.sharded uses it)


def _wait(ks, sync, nranks, arrivals, timeout_ns, status):
    return ks.lib().ks_b200_peer_arrival_wait_ranks_async(sync.data_ptr(), nranks, sync.data_ptr() + 4 * EXPECTED,
                                                          arrivals, timeout_ns, status.data_ptr(), None)


def test_wait_that_nothing_satisfies_times_out(ks, cuda):
    import torch

    sync = torch.zeros(64, dtype=torch.int32, device=cuda)
    status = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert _wait(ks, sync, 2, 1, 20_000_000, status) == ks.KS_OK  # 20 ms limit
    rc = ks.lib().ks_b200_status_check(status.data_ptr(), None)
    dt = time.perf_counter() - t0
    assert rc == ks.KS_ERR_DEVICE, rc
    assert "timed out" in ks.last_error()
    assert status.cpu().tolist() == [0, 1]
    assert 0.015 <= dt < 5.0, dt  # it waited for its limit, and no longer
    assert int(sync[EXPECTED]) == 1  # the running target still advanced
    # the context is still usable: a satisfied wait passes with a clean status
    status.zero_()
    sync[0] = 2
    sync[1] = 2
    assert _wait(ks, sync, 2, 1, 20_000_000, status) == ks.KS_OK
    assert ks.lib().ks_b200_status_check(status.data_ptr(), None) == ks.KS_OK
    assert int(sync[EXPECTED]) == 2


def test_wait_checks_every_source(ks, cuda):
    """Two arrivals from source 0 do not stand in for the missing one of source 1."""
    import torch

    sync = torch.zeros(64, dtype=torch.int32, device=cuda)
    sync[0] = 2
    status = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
    assert _wait(ks, sync, 2, 1, 10_000_000, status) == ks.KS_OK
    assert ks.lib().ks_b200_status_check(status.data_ptr(), None) == ks.KS_ERR_DEVICE
    assert status.cpu().tolist() == [0, 1]


def test_single_counter_wait_and_default_limit(ks, cuda):
    """The single-counter form (one-second limit) passes at once when its
    target is already met, and status_check reports a clean status."""
    import torch

    sync = torch.zeros(64, dtype=torch.int32, device=cuda)
    sync[0] = 5
    status = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
    t0 = time.perf_counter()
    assert ks.lib().ks_b200_peer_arrival_wait_async(sync.data_ptr(), sync.data_ptr() + 4 * EXPECTED, 5,
                                                     status.data_ptr(), None) == ks.KS_OK
    assert ks.lib().ks_b200_status_check(status.data_ptr(), None) == ks.KS_OK
    assert time.perf_counter() - t0 < 0.5
    assert int(sync[EXPECTED]) == 5


def test_status_check_reports_bad_scale(ks, cuda):
    """The status check maps word 0 (a bad scale found by an asynchronous
    call) to KS_ERR_INVALID_ARG, as the synchronous calls return it."""
    import numpy as np
    import torch

    import oracle as O

    rows, cols, group = 64, 256, 32
    x = torch.from_numpy(O.rng(3, 0).integers(-127, 128, cols, dtype=np.int8)).to(cuda)
    w = torch.from_numpy(O.rng(3, 1).integers(0, 256, (rows, cols // 2), dtype=np.uint8)).to(cuda)
    s = O.rng(3, 2).uniform(1e-3, 1e-2, (rows, cols // group)).astype(np.float16)
    s[10, 2] = np.float16(np.inf)
    ds = torch.from_numpy(s.view(np.uint16)).to(cuda)
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    status = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
    ks.matvec_w4a8_async(x, w, cols // 2, ds, cols // group, y, rows, cols, group, 0.1, status=status)
    assert ks.lib().ks_b200_status_check(status.data_ptr(), None) == ks.KS_ERR_INVALID_ARG
    assert status.cpu().tolist() == [1, 0]
