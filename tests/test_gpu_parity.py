"""GPU parity of libkernelsmith (B200) against the CPU oracle, through the C ABI.

Bar (from the reference's own contract, lib/kernelsmith/ks_quantized.c):
  * INT8 int32 results and the INT8 f32 dequant epilogue: bit-exact.
  * W4A8 f32 results: |y - y_ref| <= 1e-4 * max(|y_ref[n]|, rms(y_ref)).
    The reference sums W4A8 products one element at a time in f32
    (ks_quantized.c:116-123); the GPU sums exact int32 chunk dots scaled by
    their group scale, so results differ by rounding only; the floor at the
    RMS covers rows whose terms cancel.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from conftest import bundle_array

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
W4A8_REL_TOL = 1e-4


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def host(t):
    return t.cpu().numpy()


def assert_w4a8_close(y, y_ref, what=""):
    ok, worst = O.w4a8_tolerance_ok(y, y_ref, W4A8_REL_TOL)
    assert ok, f"{what}: worst err/bound = {worst:.3g} (tolerance {W4A8_REL_TOL})"


def call_matvec_w4a8(ks, x, w, wstride, s, sstride, y, rows, cols, group, sx, zx=0, zw=0, f16=False):
    L = ks.lib()
    a = ks.addr
    if f16:
        return L.ks_b200_matvec_w4a8_f16(a(x), a(w), wstride, a(s), sstride, a(y), rows, cols, group, sx, zx, zw)
    return L.ks_matvec_w4a8(a(x), a(w), wstride, a(s), sstride, a(y), rows, cols, group, sx, zx, zw, None, 0)


def call_matvec_i8(ks, x, w, stride, y, rows, cols, zx=0, zw=0):
    a = ks.addr
    return ks.lib().ks_matvec_i8(a(x), a(w), stride, a(y), rows, cols, zx, zw, None, 0)


def make_w4a8(seed, rows, cols, group, wstride=None, sstride=None, lo=1e-3, hi=1e-2, f16=False):
    prb = (cols + 1) // 2
    groups = -(-cols // group)
    wstride = wstride or prb
    sstride = sstride or groups
    g = O.rng(seed, 0)
    x = g.integers(-128, 128, cols, dtype=np.int8)
    w = O.rng(seed, 1).integers(0, 256, (rows, wstride), dtype=np.uint8)
    s = O.rng(seed, 2).uniform(lo, hi, (rows, sstride)).astype(np.float16 if f16 else np.float32)
    return x, w, s, wstride, sstride


# ------------------------------------------------------------ golden bundles


def test_golden_bundles_on_device(ks, cuda, smoke_bundles, oracle):
    import torch

    b = smoke_bundles["matvec_w4a8"]
    q = b["quantization_policy"]
    lay = b["tensors"]["W_packed"]["layout"]
    slay = b["tensors"]["W_scales"]["layout"]
    rows, cols = lay["logical_shape"]
    x, w, s = (dev(bundle_array(b, n), cuda) for n in ("X", "W_packed", "W_scales"))
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    rc = call_matvec_w4a8(ks, x, w, lay["packed_stride_bytes"], s, slay["scale_stride"], y, rows, cols,
                          lay["group_size"], q["input_scale"], q["input_zero_point"], q["weight_zero_point"])
    assert rc == 0, ks.last_error()
    c = b["compare"]
    np.testing.assert_allclose(host(y), bundle_array(b, "Y"), rtol=c["rtol"], atol=c["atol"])

    b = smoke_bundles["dot_w4a8"]
    q = b["quantization_policy"]
    xs = bundle_array(b, "X")
    out = torch.zeros(1, dtype=torch.float32, device=cuda)
    # keep every device buffer referenced until the call returns
    dxs, dws, dss = dev(xs, cuda), dev(bundle_array(b, "W_packed"), cuda), dev(bundle_array(b, "W_scales"), cuda)
    rc = ks.lib().ks_dot_w4a8(ks.addr(dxs), ks.addr(dws), ks.addr(dss), xs.size,
                              b["tensors"]["W_packed"]["layout"]["group_size"], q["input_scale"],
                              q["input_zero_point"], q["weight_zero_point"], ks.addr(out), None, 0)
    assert rc == 0
    np.testing.assert_allclose(host(out), bundle_array(b, "Y"), rtol=b["compare"]["rtol"], atol=b["compare"]["atol"])

    b = smoke_bundles["matvec_i8"]
    q = b["quantization_policy"]
    wm = bundle_array(b, "W")
    y = torch.zeros(wm.shape[0], dtype=torch.int32, device=cuda)
    rc = call_matvec_i8(ks, dev(bundle_array(b, "X"), cuda), dev(wm, cuda), b["tensors"]["W"]["layout"]["weight_stride"],
                        y, wm.shape[0], wm.shape[1], q["input_zero_point"], q["weight_zero_point"])
    assert rc == 0
    np.testing.assert_array_equal(host(y), bundle_array(b, "Y"))

    b = smoke_bundles["dot_i8"]
    q = b["quantization_policy"]
    xs = bundle_array(b, "X")
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    dxs, dws = dev(xs, cuda), dev(bundle_array(b, "W"), cuda)
    rc = ks.lib().ks_dot_i8(ks.addr(dxs), ks.addr(dws), xs.size, q["input_zero_point"], q["weight_zero_point"],
                            ks.addr(out), None, 0)
    assert rc == 0
    np.testing.assert_array_equal(host(out), bundle_array(b, "Y"))


def _pp(lo, hi):
    return ((lo & 0x0F) | ((hi & 0x0F) << 4)) & 0xFF


def test_reference_kats_host_pointers(ks, cuda):
    """reference tests/capi/test_quantized.c:33-126, called with host buffers
    exactly as that test does (the staged path)."""
    L, a = ks.lib(), ks.addr
    # every buffer is bound to a name so it outlives the call
    x1, w1, out = np.array([3, -2, 7, 1], np.int8), np.array([2, -5, 4, -3], np.int8), np.zeros(1, np.int32)
    assert L.ks_dot_i8(a(x1), a(w1), 4, 1, -1, a(out), None, 0) == 0
    assert out[0] == 48
    x2, w2, y = np.array([1, 2, 3], np.int8), np.array([1, 0, -1, 0, -2, 2, 3, 9], np.int8), np.array([-1, -1], np.int32)
    assert L.ks_matvec_i8(a(x2), a(w2), 4, a(y), 2, 3, 0, 0, None, 0) == 0
    assert y.tolist() == [-2, 11]
    x3 = np.array([4, -2, 3, 1], np.int8)
    w3 = np.array([_pp(1, -2), _pp(3, -4)], np.uint8)
    s3 = np.array([0.5, 0.25], np.float32)
    f = np.zeros(1, np.float32)
    assert L.ks_dot_w4a8(a(x3), a(w3), a(s3), 4, 2, 0.25, 0, 0, a(f), None, 0) == 0
    assert abs(f[0] - 1.3125) <= 1e-5
    x4 = np.array([2, -1, 3], np.int8)
    pw = np.array([_pp(1, 2), _pp(-3, 0), _pp(-1, 0), _pp(4, 0)], np.uint8)
    s4 = np.array([0.5, 0.25], np.float32)
    y4 = np.zeros(2, np.float32)
    assert L.ks_matvec_w4a8(a(x4), a(pw), 2, a(s4), 1, a(y4), 2, 3, 3, 0.5, 0, 0, None, 0) == 0
    np.testing.assert_allclose(y4, [-2.25, 1.25], atol=1e-5)


def test_seeded_reference_fixtures(ks, cuda, seeded):
    """Outputs written by the reference's compiled C; GPU via the C ABI."""
    import torch

    meta, arr = seeded
    for name, m in meta.items():
        x, w, y_ref = dev(arr[f"{name}.x"], cuda), dev(arr[f"{name}.w"], cuda), arr[f"{name}.y"]
        if m["kind"] == "w4a8":
            y = torch.zeros(m["rows"], dtype=torch.float32, device=cuda)
            rc = call_matvec_w4a8(ks, x, w, m["wstride"], dev(arr[f"{name}.s"], cuda), m["sstride"], y, m["rows"],
                                  m["cols"], m["group"], m["sx"], m["zx"], m["zw"])
            assert rc == 0, (name, ks.last_error())
            assert_w4a8_close(host(y), y_ref, name)
        else:
            y = torch.zeros(m["rows"], dtype=torch.int32, device=cuda)
            rc = call_matvec_i8(ks, x, w, m["wstride"], y, m["rows"], m["cols"], m["zx"], m["zw"])
            assert rc == 0, (name, ks.last_error())
            np.testing.assert_array_equal(host(y), y_ref, err_msg=name)


# ------------------------------------------------------ shapes and paths ----

W4A8_SHAPES = [
    # rows, cols, group, wstride_pad, sstride_pad, zx, zw, f16, expected path
    (1, 32, 32, 0, 0, 0, 0, False, 0),        # 4-byte scale rows cannot be bulk-copied
    (3, 64, 32, 0, 0, 5, -3, True, 0),         # (bulk copies move multiples of 16 bytes)
    (5, 128, 32, 0, 0, 5, -3, False, 1),
    (7, 256, 32, 0, 0, 0, 0, True, 1),
    (149, 4096, 32, 0, 0, 0, 0, True, 1),
    (300, 2048, 64, 16, 4, -7, 2, False, 1),
    (77, 8192, 128, 0, 0, 0, 0, True, 1),
    (64, 1024, 256, 0, 0, 127, -8, False, 1),
    (100, 96, 96, 0, 0, 0, 0, False, 0),       # group/32 not a power of two -> generic
    (50, 130, 10, 3, 1, 1, 1, False, 0),       # cols % 32 != 0
    (13, 77, 7, 0, 0, -128, 7, True, 0),       # odd cols
    (40, 640, 32, 1, 0, 0, 0, False, 0),       # stride not a multiple of 16
    (20, 9216, 32, 0, 0, 0, 0, False, 1),      # activations staged in shared memory
    (6, 16416, 32, 0, 0, 0, 0, True, 0),       # beyond the staged row limit (513 chunks)
]


@pytest.mark.parametrize("shape", W4A8_SHAPES, ids=lambda s: "x".join(map(str, s[:3])))
def test_w4a8_shapes(ks, cuda, oracle, shape):
    import torch

    rows, cols, group, wpad, spad, zx, zw, f16, path = shape
    prb = (cols + 1) // 2
    groups = -(-cols // group)
    x, w, s, wstride, sstride = make_w4a8(hash(shape) % 10000, rows, cols, group, prb + wpad, groups + spad, f16=f16)
    sx = 0.0625
    dx, dw, ds = dev(x, cuda), dev(w, cuda), dev(s.view(np.uint16) if f16 else s, cuda)
    got_path = ks.lib().ks_b200_w4a8_kernel_path(ks.addr(dx), ks.addr(dw), wstride, ks.addr(ds),
                                                 ks.SCALE_F16 if f16 else ks.SCALE_F32, sstride, rows, cols, group)
    assert got_path == path
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    rc = call_matvec_w4a8(ks, dx, dw, wstride, ds, sstride, y, rows, cols, group, sx, zx, zw, f16=f16)
    assert rc == 0, ks.last_error()
    if f16:
        rc, y_ref = oracle.matvec_w4a8_f16(x, w, wstride, s.view(np.uint16), sstride, rows, cols, group, sx, zx, zw)
    else:
        rc, y_ref = oracle.matvec_w4a8(x, w, wstride, s, sstride, rows, cols, group, sx, zx, zw)
    assert rc == 0
    assert_w4a8_close(host(y), y_ref, str(shape))


I8_SHAPES = [
    # rows, cols, stride_pad, zx, zw, expected path
    (1, 16, 0, 0, 0, 1),
    (5, 4096, 0, 3, -4, 1),
    (4096, 4096, 0, 0, 0, 1),
    (333, 1024, 16, -128, 127, 1),
    (77, 2000, 0, 1, 1, 1),
    (40, 100, 12, -3, 2, 0),    # cols % 16 != 0
    (20, 6000, 0, 5, 5, 1),     # activations staged in shared memory
    (4, 8208, 0, 1, -1, 0),     # beyond the staged row limit (513 chunks)
    (9, 64, 3, 0, 0, 0),        # stride not a multiple of 16
]


@pytest.mark.parametrize("shape", I8_SHAPES, ids=lambda s: "x".join(map(str, s[:3])))
def test_i8_shapes_bit_exact(ks, cuda, oracle, shape):
    import torch

    rows, cols, spad, zx, zw, path = shape
    stride = cols + spad
    g = O.rng(hash(shape) % 10000, 0)
    x = g.integers(-128, 128, cols, dtype=np.int8)
    w = O.rng(hash(shape) % 10000, 1).integers(-128, 128, (rows, stride), dtype=np.int8)
    dx, dw = dev(x, cuda), dev(w, cuda)
    assert ks.lib().ks_b200_i8_kernel_path(ks.addr(dx), ks.addr(dw), stride, rows, cols) == path
    y = torch.zeros(rows, dtype=torch.int32, device=cuda)
    assert call_matvec_i8(ks, dx, dw, stride, y, rows, cols, zx, zw) == 0, ks.last_error()
    rc, y_ref = oracle.matvec_i8(x, w, rows, cols, stride, zx, zw)
    np.testing.assert_array_equal(host(y), y_ref)
    ws = O.rng(hash(shape) % 10000, 2).uniform(1e-3, 1e-2, rows).astype(np.float32)
    yf = torch.zeros(rows, dtype=torch.float32, device=cuda)
    dws = dev(ws, cuda)
    rc = ks.lib().ks_b200_matvec_i8_dequant(ks.addr(dx), ks.addr(dw), stride, ks.addr(dws), 0.02,
                                            ks.addr(yf), rows, cols, zx, zw)
    assert rc == 0, ks.last_error()
    rc, yf_ref = oracle.matvec_i8_dequant(x, w, rows, cols, stride, ws, 0.02, zx, zw)
    np.testing.assert_array_equal(host(yf).view(np.uint32), yf_ref.view(np.uint32))


def test_i8_wraparound(ks, cuda, oracle):
    import torch

    cols = 40000
    x = np.full(cols, 127, np.int8)
    w = np.full((3, cols), -128, np.int8)
    y = torch.zeros(3, dtype=torch.int32, device=cuda)
    assert call_matvec_i8(ks, dev(x, cuda), dev(w, cuda), cols, y, 3, cols, -128, 127) == 0
    _, y_ref = oracle.matvec_i8(x, w, 3, cols, cols, -128, 127)
    np.testing.assert_array_equal(host(y), y_ref)


def test_unaligned_pointers(ks, cuda, oracle):
    """Base addresses off the 16-byte grid take the generic path, same answers."""
    import torch

    rows, cols, group = 64, 512, 32
    x, w, s, wstride, sstride = make_w4a8(5, rows, cols, group)
    bx = torch.zeros(cols + 1, dtype=torch.int8, device=cuda)
    bx[1:] = dev(x, cuda)
    bw = torch.zeros(rows * wstride + 1, dtype=torch.uint8, device=cuda)
    bw[1:] = dev(w.ravel(), cuda)
    y = torch.zeros(rows + 1, dtype=torch.float32, device=cuda)
    rc = call_matvec_w4a8(ks, bx.data_ptr() + 1, bw.data_ptr() + 1, wstride, dev(s, cuda), sstride,
                          y.data_ptr() + 4, rows, cols, group, 0.1)
    assert rc == 0, ks.last_error()
    _, y_ref = oracle.matvec_w4a8(x, w, wstride, s, sstride, rows, cols, group, 0.1)
    assert_w4a8_close(host(y)[1:], y_ref)


# -------------------------------------------------------- BASELINE configs --


def test_config_int8_gemv_4096(ks, cuda, oracle):
    """INT8 GEMV 4096x4096, f32 out = acc * w_scale[n] * a_scale: bit-exact."""
    import torch

    n = k = 4096
    x = O.rng(20261201, 0).integers(-127, 128, k, dtype=np.int8)
    w = O.rng(20261201, 1).integers(-127, 128, (n, k), dtype=np.int8)
    ws = O.rng(20261201, 2).uniform(1e-3, 1e-2, n).astype(np.float32)
    dx, dw = dev(x, cuda), dev(w, cuda)
    yi = torch.zeros(n, dtype=torch.int32, device=cuda)
    assert call_matvec_i8(ks, dx, dw, k, yi, n, k) == 0
    _, yi_ref = oracle.matvec_i8(x, w, n, k, k)
    np.testing.assert_array_equal(host(yi), yi_ref)
    yf = torch.zeros(n, dtype=torch.float32, device=cuda)
    dws = dev(ws, cuda)
    assert ks.lib().ks_b200_matvec_i8_dequant(ks.addr(dx), ks.addr(dw), k, ks.addr(dws), 0.02,
                                              ks.addr(yf), n, k, 0, 0) == 0
    _, yf_ref = oracle.matvec_i8_dequant(x, w, n, k, k, ws, 0.02)
    np.testing.assert_array_equal(host(yf).view(np.uint32), yf_ref.view(np.uint32))


@pytest.mark.parametrize("f16", [True, False])
def test_config_w4a8_gemv_11008x4096(ks, cuda, oracle, f16):
    """W4A8 11008x4096 G32; f16 scales (extension) and f32 scales (reference ABI)."""
    import torch

    n, k, g = 11008, 4096, 32
    x = O.rng(20261202, 0).integers(-127, 128, k, dtype=np.int8)
    w4 = O.rng(20261202, 1).integers(-8, 8, (n, k), dtype=np.int8)
    w = O.pack_int4(w4)
    s16 = O.rng(20261202, 2).uniform(1e-3, 1e-2, (n, k // g)).astype(np.float16)
    y = torch.zeros(n, dtype=torch.float32, device=cuda)
    if f16:
        rc = call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), k // 2, dev(s16.view(np.uint16), cuda), k // g, y, n,
                              k, g, 0.02, f16=True)
    else:
        rc = call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), k // 2, dev(s16.astype(np.float32), cuda), k // g,
                              y, n, k, g, 0.02)
    assert rc == 0, ks.last_error()
    _, y_ref = oracle.matvec_w4a8(x, w, k // 2, s16.astype(np.float32), k // g, n, k, g, 0.02)
    assert_w4a8_close(host(y), y_ref, "cfg2")
    # the GPU answer is also close to the exact (f64) dot, as the reference's is
    exact = (w4.astype(np.float64) * np.repeat(s16.astype(np.float64), g, axis=1)) @ (x.astype(np.float64) * 0.02)
    assert_w4a8_close(host(y), exact, "cfg2 vs f64")


@pytest.mark.parametrize("n", [28672, 128256])
def test_config_sharded_shapes_rows_sample(ks, cuda, oracle, n):
    """K=8192, G=128, f16: full GEMV on the GPU, oracle on 512 sampled rows."""
    import torch

    k, g = 8192, 128
    gen = np.random.default_rng(n)
    x = gen.integers(-127, 128, k, dtype=np.int8)
    w = gen.integers(0, 256, (n, k // 2), dtype=np.uint8)
    s16 = gen.uniform(1e-3, 1e-2, (n, k // g)).astype(np.float16)
    y = torch.zeros(n, dtype=torch.float32, device=cuda)
    rc = call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), k // 2, dev(s16.view(np.uint16), cuda), k // g, y, n, k,
                          g, 0.02, f16=True)
    assert rc == 0, ks.last_error()
    rows = np.sort(gen.choice(n, 512, replace=False))
    rows[0], rows[-1] = 0, n - 1
    _, y_ref = oracle.matvec_w4a8_f16(x, np.ascontiguousarray(w[rows]), k // 2,
                                      np.ascontiguousarray(s16[rows]).view(np.uint16), k // g, len(rows), k, g, 0.02)
    assert_w4a8_close(host(y)[rows], y_ref, f"N={n}")


# ------------------------------------------------------- semantics ---------


@pytest.mark.parametrize("f16", [False, True], ids=["f32_scales", "f16_scales"])
@pytest.mark.parametrize("out_on", ["device", "host"])
@pytest.mark.parametrize("cols", [1024, 1000], ids=["streaming", "generic"])
def test_bad_scale_returns_invalid_arg(ks, cuda, oracle, f16, out_on, cols):
    """A bad scale returns KS_ERR_INVALID_ARG and leaves the WHOLE output buffer
    as the reference leaves it: rows before the first bad row written, that row
    and every later one untouched (ks_quantized.c:148-156, scale check :112-114)."""
    import torch

    rows, group = 300, 32
    x, w, s, wstride, sstride = make_w4a8(9, rows, cols, group, f16=f16)
    for bad_row, bad in ((211, 0.0), (211, -1.0), (211, np.inf), (211, np.nan), (0, 0.0), (rows - 1, -0.0),
                         (37, 0.0)):
        s2 = s.copy()
        s2[bad_row, 7] = bad
        if bad_row == 37:  # two bad rows: the first one decides
            s2[250, 1] = np.nan
        first = 37 if bad_row == 37 else bad_row
        fill = np.full(rows, 7.0, np.float32)
        fill[::3] = -2.5  # untouched rows must keep their own contents, not one fill value
        s_arg = s2.view(np.uint16) if f16 else s2
        y = dev(fill, cuda) if out_on == "device" else fill.copy()
        rc = call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), wstride, dev(s_arg, cuda), sstride, y, rows, cols,
                              group, 0.5, f16=f16)
        assert rc == ks.KS_ERR_INVALID_ARG, (rc, ks.last_error())
        o = fill.copy()
        if f16:
            rc_ref, _ = oracle.matvec_w4a8_f16(x, w, wstride, s_arg, sstride, rows, cols, group, 0.5, out=o)
        else:
            rc_ref, _ = oracle.matvec_w4a8(x, w, wstride, s2, sstride, rows, cols, group, 0.5, out=o)
        assert rc_ref == -1
        got = host(y) if out_on == "device" else y
        if first > 0:
            assert_w4a8_close(got[:first], o[:first], "rows before the first bad row")
        np.testing.assert_array_equal(got[first:].view(np.uint32), o[first:].view(np.uint32),
                                      err_msg=f"rows from the first bad row ({first}) must be untouched")
    # the next good call succeeds (status is per call) and writes every row
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    s_arg = s.view(np.uint16) if f16 else s
    assert call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), wstride, dev(s_arg, cuda), sstride, y, rows, cols,
                            group, 0.5, f16=f16) == 0
    o = np.zeros(rows, np.float32)
    if f16:
        oracle.matvec_w4a8_f16(x, w, wstride, s_arg, sstride, rows, cols, group, 0.5, out=o)
    else:
        oracle.matvec_w4a8(x, w, wstride, s, sstride, rows, cols, group, 0.5, out=o)
    assert_w4a8_close(host(y), o, "good call after a bad one")


def test_dot_w4a8_bad_scale_leaves_output(ks, cuda):
    """ks_dot_w4a8 with a bad scale returns KS_ERR_INVALID_ARG and does not write *output."""
    k, group = 256, 32
    x, w, s, _, _ = make_w4a8(11, 1, k, group)
    s[0, 3] = np.nan
    for out_on in ("device", "host"):
        out = dev(np.array([42.0], np.float32), cuda) if out_on == "device" else np.array([42.0], np.float32)
        a = ks.addr
        rc = ks.lib().ks_dot_w4a8(a(dev(x, cuda)), a(dev(w, cuda)), a(dev(s, cuda)), k, group, 0.5, 0, 0, a(out),
                                  None, 0)
        assert rc == ks.KS_ERR_INVALID_ARG
        assert float((host(out) if out_on == "device" else out)[0]) == 42.0


def test_bad_f16_scale(ks, cuda):
    import torch

    rows, cols, group = 20, 256, 32
    x, w, s, wstride, sstride = make_w4a8(10, rows, cols, group, f16=True)
    s[5, 1] = np.float16(-0.0)
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    rc = call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), wstride, dev(s.view(np.uint16), cuda), sstride, y, rows,
                          cols, group, 0.5, f16=True)
    assert rc == ks.KS_ERR_INVALID_ARG


def test_host_and_pinned_buffers_match_device(ks, cuda):
    import torch

    rows, cols, group = 500, 2048, 32
    x, w, s, wstride, sstride = make_w4a8(12, rows, cols, group)
    yd = torch.zeros(rows, dtype=torch.float32, device=cuda)
    assert call_matvec_w4a8(ks, dev(x, cuda), dev(w, cuda), wstride, dev(s, cuda), sstride, yd, rows, cols, group, 0.3) == 0
    yh = np.zeros(rows, np.float32)
    assert call_matvec_w4a8(ks, x, w, wstride, s, sstride, yh, rows, cols, group, 0.3) == 0
    np.testing.assert_array_equal(yh.view(np.uint32), host(yd).view(np.uint32))
    px, pw, ps = (torch.from_numpy(a).pin_memory() for a in (x, w, s))
    yp = torch.zeros(rows, dtype=torch.float32).pin_memory()
    assert call_matvec_w4a8(ks, px, pw, wstride, ps, sstride, yp, rows, cols, group, 0.3) == 0
    np.testing.assert_array_equal(yp.numpy().view(np.uint32), yh.view(np.uint32))
    # mixed: weights on device, activations and output on the host
    ym = np.zeros(rows, np.float32)
    assert call_matvec_w4a8(ks, x, dev(w, cuda), wstride, dev(s, cuda), sstride, ym, rows, cols, group, 0.3) == 0
    np.testing.assert_array_equal(ym.view(np.uint32), yh.view(np.uint32))


def test_deterministic_repeat(ks, cuda):
    import torch

    rows, cols, group = 11008, 4096, 32
    x, w, s, wstride, sstride = make_w4a8(13, rows, cols, group, f16=True)
    args = (dev(x, cuda), dev(w, cuda), wstride, dev(s.view(np.uint16), cuda), sstride)
    ys = []
    for _ in range(3):
        y = torch.zeros(rows, dtype=torch.float32, device=cuda)
        assert call_matvec_w4a8(ks, *args, y, rows, cols, group, 0.02, f16=True) == 0
        ys.append(host(y).view(np.uint32))
    assert (ys[0] == ys[1]).all() and (ys[1] == ys[2]).all()


def test_async_status_and_streams(ks, cuda, oracle):
    import torch

    rows, cols, group = 1000, 4096, 32
    x, w, s, wstride, sstride = make_w4a8(14, rows, cols, group, f16=True)
    dx, dw, ds = dev(x, cuda), dev(w, cuda), dev(s.view(np.uint16), cuda)
    status = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
    stream = torch.cuda.Stream()
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    stream.wait_stream(torch.cuda.current_stream())  # zero-filled buffers first
    with torch.cuda.stream(stream):
        ks.matvec_w4a8_async(dx, dw, wstride, ds, sstride, y, rows, cols, group, 0.02, status=status, stream=stream)
    stream.synchronize()
    assert host(status).tolist() == [0, 0]
    _, y_ref = oracle.matvec_w4a8_f16(x, w, wstride, s.view(np.uint16), sstride, rows, cols, group, 0.02)
    assert_w4a8_close(host(y), y_ref)
    s_bad = s.copy()
    s_bad[999, 127] = np.float16(np.inf)
    with torch.cuda.stream(stream):
        ks.matvec_w4a8_async(dx, dw, wstride, dev(s_bad.view(np.uint16), cuda), sstride, y, rows, cols, group, 0.02,
                             status=status, stream=stream)
    stream.synchronize()
    assert host(status).tolist() == [1, 0]


def test_async_graph_capture(ks, cuda, oracle):
    """The async entry point allocates nothing and can be captured."""
    import torch

    rows, cols, group = 2000, 4096, 32
    x, w, s, wstride, sstride = make_w4a8(15, rows, cols, group, f16=True)
    dx, dw, ds = dev(x, cuda), dev(w, cuda), dev(s.view(np.uint16), cuda)
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())  # zero-filled output first
    with torch.cuda.stream(stream):  # warm-up outside capture
        ks.matvec_w4a8_async(dx, dw, wstride, ds, sstride, y, rows, cols, group, 0.02, stream=stream)
    stream.synchronize()
    y.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        ks.matvec_w4a8_async(dx, dw, wstride, ds, sstride, y, rows, cols, group, 0.02,
                             stream=torch.cuda.current_stream())
    graph.replay()
    torch.cuda.synchronize()
    _, y_ref = oracle.matvec_w4a8_f16(x, w, wstride, s.view(np.uint16), sstride, rows, cols, group, 0.02)
    assert_w4a8_close(host(y), y_ref)


# --------------------------------------- the reference's own C callers -------


def _bin(name):
    p = ROOT / "oracle" / "_ref" / name
    if not p.exists():
        pytest.skip(f"{p} not built (make -C oracle ref-b200)")
    return p


def test_reference_capi_test_linked_against_b200(cuda):
    """tests/capi/test_quantized.c of the reference, compiled unmodified and
    linked against libkernelsmith (B200): all its checks pass."""
    exe = _bin("test_quantized_b200")
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "Target: b200-sm100a" in res.stdout
    assert "7/7 tests passed" in res.stdout


def test_reference_host_runner_linked_against_b200(cuda, smoke_bundles, tmp_path):
    """tests/host_reference/host_reference_runner.c of the reference, unmodified,
    linked against libkernelsmith (B200), on the reference's golden bundles."""
    exe = _bin("host_reference_runner_b200")

    def raw(name, a):
        p = tmp_path / f"{name}.raw"
        np.ascontiguousarray(a).tofile(p)
        return str(p)

    b = smoke_bundles["matvec_w4a8"]
    q = b["quantization_policy"]
    rows, cols = b["tensors"]["W_packed"]["layout"]["logical_shape"]
    out = tmp_path / "y.raw"
    cmd = [str(exe), "matvec_w4a8", raw("x", bundle_array(b, "X")), raw("w", bundle_array(b, "W_packed")),
           raw("s", bundle_array(b, "W_scales")), str(out), str(rows), str(cols),
           str(b["tensors"]["W_packed"]["layout"]["group_size"]), repr(q["input_scale"]),
           str(q["input_zero_point"]), str(q["weight_zero_point"])]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    np.testing.assert_allclose(np.fromfile(out, np.float32), bundle_array(b, "Y"), rtol=1e-6, atol=1e-6)

    b = smoke_bundles["matvec_i8"]
    q = b["quantization_policy"]
    wm = bundle_array(b, "W")
    cmd = [str(exe), "matvec_i8", raw("x8", bundle_array(b, "X")), raw("w8", wm), str(out), str(wm.shape[0]),
           str(wm.shape[1]), str(q["input_zero_point"]), str(q["weight_zero_point"])]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    np.testing.assert_array_equal(np.fromfile(out, np.int32), bundle_array(b, "Y"))


def test_library_loaded_is_in_tree(ks, cuda):
    """The process runs the in-tree libkernelsmith.so (no pip copy)."""
    maps = Path("/proc/self/maps").read_text()
    assert str(ks.LIB_PATH) in maps
    assert ctypes.CDLL(str(ks.LIB_PATH)).ks_target_name
