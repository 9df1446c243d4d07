"""GGML Q4_0 -> native W4A8 importer on the GPU (ks_b200_import_ggml_q4_0_async)
against the oracle: packed int4 bytes and group scales bit-exact, for every
group size, f32 and f16 scales, padded strides and the edge blocks (d = 0,
negative d, f16 subnormal and maximal d).  The imported weights then run
through the W4A8 GEMV like any native weights."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _blocks(rows, cols, seed):
    g = np.random.default_rng(seed)
    nb = cols // 32
    b = np.zeros((rows, nb, 18), np.uint8)
    d = g.uniform(-0.05, 0.05, (rows, nb)).astype(np.float16)
    d[0, 0] = 0                          # zero block
    d[0, 1] = np.float16(6e-8)           # subnormal
    d[0, 2] = np.float16(65504)          # largest finite
    d[0, 3] = np.float16(-65504)
    b[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    b[:, :, 2:] = g.integers(0, 256, (rows, nb, 16), dtype=np.uint8)
    return b.reshape(rows, nb * 18)


def _run(ks, torch, cuda, blocks, rows, cols, group, f16, src_pad=0, dst_pad=0):
    src = np.zeros((rows, blocks.shape[1] + src_pad), np.uint8)
    src[:, :blocks.shape[1]] = blocks
    pstride = cols // 2 + dst_pad
    sstride = cols // group + (3 if dst_pad else 0)
    dsrc = torch.from_numpy(src).to(cuda)
    packed = torch.full((rows, pstride), 0xEE, dtype=torch.uint8, device=cuda)
    scales = torch.zeros((rows, sstride), dtype=torch.float16 if f16 else torch.float32, device=cuda)
    ks.import_ggml_q4_0_async(dsrc, src.shape[1], rows, cols, group, packed, pstride, scales,
                              scale_type=ks.SCALE_F16 if f16 else ks.SCALE_F32, scale_stride=sstride)
    torch.cuda.synchronize()
    p = packed.cpu().numpy()
    s = scales.cpu().numpy()
    if dst_pad:
        assert (p[:, cols // 2:] == 0xEE).all()  # padding untouched
    return p[:, :cols // 2], s[:, :cols // group]


@pytest.mark.parametrize("group", [32, 64, 128, 256])
@pytest.mark.parametrize("f16", [False, True])
def test_import_bit_exact(ks, cuda, group, f16):
    import torch

    rows, cols = 300, 4096
    blocks = _blocks(rows, cols, group + (1 if f16 else 0))
    p, s = _run(ks, torch, cuda, blocks, rows, cols, group, f16)
    p_ref, s_ref = O.q4_0_import(blocks, rows, cols, group, f16)
    np.testing.assert_array_equal(p, p_ref)
    np.testing.assert_array_equal(s.view(np.uint16 if f16 else np.uint32),
                                  s_ref.view(np.uint16 if f16 else np.uint32))


def test_import_strided(ks, cuda):
    import torch

    rows, cols, group = 37, 1024, 64
    blocks = _blocks(rows, cols, 3)
    p, s = _run(ks, torch, cuda, blocks, rows, cols, group, True, src_pad=6, dst_pad=16)
    p_ref, s_ref = O.q4_0_import(blocks, rows, cols, group, True)
    np.testing.assert_array_equal(p, p_ref)
    np.testing.assert_array_equal(s.view(np.uint16), s_ref)


def test_imported_weights_in_the_gemv(ks, cuda, oracle):
    """Imported weights feed ks_b200_matvec_w4a8_f16 unchanged: the GPU GEMV on
    them matches the oracle GEMV on the same bytes."""
    import torch

    rows, cols, group = 512, 4096, 32
    blocks = _blocks(rows, cols, 99)
    p, s = _run(ks, torch, cuda, blocks, rows, cols, group, True)
    x = np.random.default_rng(7).integers(-127, 128, cols, dtype=np.int8)
    dx, dp, ds = (torch.from_numpy(a).to(cuda) for a in (x, p, s.view(np.uint16)))
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    ks.matvec_w4a8_async(dx, dp, cols // 2, ds, cols // group, y, rows, cols, group, 0.02)
    torch.cuda.synchronize()
    _, y_ref = oracle.matvec_w4a8_f16(x, p, cols // 2, s.view(np.uint16), cols // group, rows, cols, group, 0.02)
    ok, worst = O.w4a8_tolerance_ok(y.cpu().numpy(), y_ref)
    assert ok, worst


def test_import_rejects_bad_args(ks):
    L = ks.lib()
    buf = np.zeros(64, np.uint8)
    E = ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_import_ggml_q4_0_async(ks.addr(buf), 18, 1, 48, 32, ks.addr(buf), 32, ks.addr(buf), 0, 1,
                                            None) == E  # cols not a multiple of 32
    assert L.ks_b200_import_ggml_q4_0_async(ks.addr(buf), 18, 1, 32, 48, ks.addr(buf), 32, ks.addr(buf), 0, 1,
                                            None) == E  # group size
    assert L.ks_b200_import_ggml_q4_0_async(ks.addr(buf), 10, 1, 32, 32, ks.addr(buf), 32, ks.addr(buf), 0, 1,
                                            None) == E  # block stride too small
    assert L.ks_b200_quant_layout_version() == 1
