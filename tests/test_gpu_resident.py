"""Resident W4A8 weights (ks_b200_w4a8_register): a matrix, or a rank's row
shard of it, uploaded once in the ABI layout and used by later GEMVs.  The
GEMV on the registered copy must be bitwise the GEMV on the original device
weights (the same kernel on the same bytes); a shard's outputs must be those
rows of the full matrix's outputs."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cols,group,f16", [(4096, 32, True), (8192, 128, True), (4095, 32, False)],
                         ids=["4096_g32_f16", "8192_g128_f16", "4095_g32_f32_generic"])
def test_registered_gemv_bitwise_equals_direct(ks, cuda, cols, group, f16):
    import torch

    L = ks.lib()
    rows = 3000
    prb, groups = (cols + 1) // 2, -(-cols // group)
    x = O.rng(61, 0).integers(-127, 128, cols, dtype=np.int8)
    w = O.rng(61, 1).integers(0, 256, (rows, prb), dtype=np.uint8)
    s = O.rng(61, 2).uniform(1e-3, 1e-2, (rows, groups)).astype(np.float16 if f16 else np.float32)
    st = ks.SCALE_F16 if f16 else ks.SCALE_F32
    s_arg = s.view(np.uint16) if f16 else s
    dx, dw, ds = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (x, w, s_arg))
    ref = torch.zeros(rows, dtype=torch.float32, device=cuda)
    ks.matvec_w4a8_async(dx, dw, prb, ds, groups, ref, rows, cols, group, 0.02, scale_type=st)
    torch.cuda.synchronize()
    for src in ("host", "device"):
        for r0, n in ((0, rows), (1000, 1000), (2999, 1)):  # the whole matrix and two shards
            h = ctypes.c_void_p()
            wsrc, ssrc = (w, s_arg) if src == "host" else (dw, ds)
            assert L.ks_b200_w4a8_register(ks.addr(wsrc), prb, ks.addr(ssrc), st, groups, rows, cols, group, r0, n,
                                           ks.KS_QUANT_LAYOUT_VERSION, ctypes.byref(h)) == 0, ks.last_error()
            try:
                stride, held, first = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
                assert L.ks_b200_w4a8_weights_info(h, None, ctypes.byref(stride), None, None, ctypes.byref(held),
                                                   ctypes.byref(first)) == 0
                assert held.value == n and first.value == r0 and stride.value % 16 == 0
                y = torch.full((n,), float("nan"), dtype=torch.float32, device=cuda)
                assert L.ks_b200_w4a8_matvec_registered_async(h, ks.addr(dx), 0.02, 0, 0, ks.addr(y), None,
                                                              None) == 0, ks.last_error()
                torch.cuda.synchronize()
                assert torch.equal(y, ref[r0:r0 + n]), (src, r0, n)
            finally:
                assert L.ks_b200_w4a8_release(h) == 0
