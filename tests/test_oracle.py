"""Pins the CPU oracle (oracle/ks_oracle.c) before any GPU result is trusted.

* against the reference's own golden bundles (tests/golden/generated/*_smoke
  in the reference, copied with their sha256 checked);
* against the hand-computed known answers of the reference's C API test
  (tests/capi/test_quantized.c:33-171);
* bit-for-bit against the reference's C implementation itself: the seeded
  fixtures were produced by it, and, where oracle/_ref is built, live calls
  on fresh random inputs including the error paths.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import bundle_array

# ---------------------------------------------------------------- golden --


def test_golden_dot_i8(oracle, smoke_bundles):
    b = smoke_bundles["dot_i8"]
    q = b["quantization_policy"]
    rc, y = oracle.dot_i8(bundle_array(b, "X"), bundle_array(b, "W"), q["input_zero_point"], q["weight_zero_point"])
    assert rc == 0
    assert y == int(bundle_array(b, "Y")[0])


def test_golden_matvec_i8(oracle, smoke_bundles):
    b = smoke_bundles["matvec_i8"]
    q = b["quantization_policy"]
    w = bundle_array(b, "W")
    stride = b["tensors"]["W"]["layout"]["weight_stride"]
    rc, y = oracle.matvec_i8(bundle_array(b, "X"), w, w.shape[0], w.shape[1], stride,
                             q["input_zero_point"], q["weight_zero_point"])
    assert rc == 0
    np.testing.assert_array_equal(y, bundle_array(b, "Y"))


def _compare_policy(b, got, exp):
    c = b["compare"]
    np.testing.assert_allclose(got, exp, rtol=c["rtol"], atol=c["atol"])


def test_golden_dot_w4a8(oracle, smoke_bundles):
    b = smoke_bundles["dot_w4a8"]
    q = b["quantization_policy"]
    x = bundle_array(b, "X")
    lay = b["tensors"]["W_packed"]["layout"]
    rc, y = oracle.dot_w4a8(x, bundle_array(b, "W_packed"), bundle_array(b, "W_scales"), x.size,
                            lay["group_size"], q["input_scale"], q["input_zero_point"], q["weight_zero_point"])
    assert rc == 0
    _compare_policy(b, np.float32(y), bundle_array(b, "Y")[0])


def test_golden_matvec_w4a8(oracle, smoke_bundles):
    b = smoke_bundles["matvec_w4a8"]
    q = b["quantization_policy"]
    lay = b["tensors"]["W_packed"]["layout"]
    slay = b["tensors"]["W_scales"]["layout"]
    rows, cols = lay["logical_shape"]
    rc, y = oracle.matvec_w4a8(bundle_array(b, "X"), bundle_array(b, "W_packed"), lay["packed_stride_bytes"],
                               bundle_array(b, "W_scales"), slay["scale_stride"], rows, cols, lay["group_size"],
                               q["input_scale"], q["input_zero_point"], q["weight_zero_point"])
    assert rc == 0
    _compare_policy(b, y, bundle_array(b, "Y"))


def test_golden_matmul_i8_via_gemm(oracle, smoke_bundles):
    """matmul_i8_smoke pins int32 C = (A - za)(B - zb); the skinny GEMM oracle
    (zero points 0) reproduces it after shifting the operands in int32."""
    b = smoke_bundles["matmul_i8"]
    q = b["quantization_policy"]
    a = bundle_array(b, "A").astype(np.int32) - q["input_zero_point"]
    bm = bundle_array(b, "B").astype(np.int32) - q["weight_zero_point"]
    # shifted operands still fit int8 for this bundle (values in [-8, 8])
    a8 = a.astype(np.int8)
    w8 = np.ascontiguousarray(bm.T).astype(np.int8)
    rc, _, acc = oracle.gemm_i8_requant(a8, np.ones(a8.shape[0], np.float32), w8,
                                        np.ones(w8.shape[0], np.float32), 1.0, want_acc=True)
    assert rc == 0
    np.testing.assert_array_equal(acc, bundle_array(b, "C"))


def test_golden_rms_norm(oracle, smoke_bundles):
    b = smoke_bundles["rms_norm_f32"]
    x = bundle_array(b, "X")
    eps = b["compare"].get("epsilon", b["quantization_policy"].get("epsilon", 1e-5))
    rc, y = oracle.rms_norm(x, bundle_array(b, "W"), eps)
    assert rc == 0
    c = b["compare"]
    np.testing.assert_allclose(y, bundle_array(b, "Y"), rtol=c.get("rtol", 1e-6), atol=c.get("atol", 1e-6))


# ------------------------------------------- known answers (test_quantized.c)


def _pack_pair(lo, hi):
    return ((lo & 0x0F) | ((hi & 0x0F) << 4)) & 0xFF


def test_kat_dot_i8(oracle):
    # reference tests/capi/test_quantized.c:33-47
    rc, y = oracle.dot_i8(np.array([3, -2, 7, 1], np.int8), np.array([2, -5, 4, -3], np.int8), 1, -1)
    assert (rc, y) == (0, 48)


def test_kat_matvec_i8(oracle):
    # :49-67 -- stride 4 over 3 columns
    w = np.array([1, 0, -1, 0, -2, 2, 3, 9], np.int8)
    rc, y = oracle.matvec_i8(np.array([1, 2, 3], np.int8), w, 2, 3, 4)
    assert rc == 0 and y.tolist() == [-2, 11]


def test_kat_helpers(oracle):
    # :69-83
    L = oracle.lib
    assert L.kso_w4a8_packed_row_bytes(5) == 3
    assert L.kso_w4a8_scale_groups(17, 8) == 3
    assert L.kso_w4a8_scale_groups(17, 0) == 0


def test_kat_dot_w4a8(oracle):
    # :85-103
    pw = np.array([_pack_pair(1, -2), _pack_pair(3, -4)], np.uint8)
    rc, y = oracle.dot_w4a8(np.array([4, -2, 3, 1], np.int8), pw, np.array([0.5, 0.25], np.float32), 4, 2, 0.25)
    assert rc == 0 and abs(y - 1.3125) <= 1e-5


def test_kat_matvec_w4a8(oracle):
    # :105-126 -- stride 2 bytes, one scale per row, group 3
    pw = np.array([_pack_pair(1, 2), _pack_pair(-3, 0), _pack_pair(-1, 0), _pack_pair(4, 0)], np.uint8)
    rc, y = oracle.matvec_w4a8(np.array([2, -1, 3], np.int8), pw, 2, np.array([0.5, 0.25], np.float32), 1,
                               2, 3, 3, 0.5)
    assert rc == 0
    np.testing.assert_allclose(y, [-2.25, 1.25], atol=1e-5)


def test_kat_error_cases(oracle):
    # :143-171
    L = oracle.lib
    x = np.array([1], np.int8)
    w = np.array([1], np.int8)
    packed = np.array([0], np.uint8)
    scale = np.array([1.0], np.float32)
    i32 = np.zeros(1, np.int32)
    f32 = np.zeros(1, np.float32)
    p = lambda a: a.ctypes.data  # noqa: E731
    assert L.kso_dot_i8(None, p(w), 1, 0, 0, p(i32)) == -1
    assert L.kso_dot_i8(p(x), p(w), 1, 129, 0, p(i32)) == -1
    assert L.kso_matvec_i8(p(x), p(w), 0, p(i32), 1, 1, 0, 0) == -1
    assert L.kso_dot_w4a8(p(x), p(packed), p(scale), 1, 0, 1.0, 0, 0, p(f32)) == -1
    assert L.kso_dot_w4a8(p(x), p(packed), p(scale), 1, 1, -1.0, 0, 0, p(f32)) == -1
    assert L.kso_dot_w4a8(p(x), p(packed), p(scale), 1, 1, 1.0, 0, 8, p(f32)) == -1


# ------------------------------------------- reference C, bit for bit ------


def test_seeded_fixtures_bit_exact(oracle, seeded):
    """Expected outputs were written by the reference's compiled C."""
    meta, arr = seeded
    for name, m in meta.items():
        x, w, y_ref = arr[f"{name}.x"], arr[f"{name}.w"], arr[f"{name}.y"]
        if m["kind"] == "w4a8":
            rc, y = oracle.matvec_w4a8(x, w, m["wstride"], arr[f"{name}.s"], m["sstride"], m["rows"], m["cols"],
                                       m["group"], m["sx"], m["zx"], m["zw"])
            assert rc == 0
            np.testing.assert_array_equal(y.view(np.uint32), y_ref.view(np.uint32), err_msg=name)
        else:
            rc, y = oracle.matvec_i8(x, w, m["rows"], m["cols"], m["wstride"], m["zx"], m["zw"])
            assert rc == 0
            np.testing.assert_array_equal(y, y_ref, err_msg=name)


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (make -C oracle ref)")


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_live_w4a8_vs_reference(oracle, seed):
    ref = O.RefLib("generic")
    g = np.random.default_rng(1000 + seed)
    rows, cols = int(g.integers(1, 40)), int(g.integers(1, 300))
    group = int(g.integers(1, 70))
    prb = (cols + 1) // 2
    groups = -(-cols // group)
    wstride = prb + int(g.integers(0, 5))
    sstride = groups + int(g.integers(0, 3))
    x = g.integers(-128, 128, cols, dtype=np.int8)
    w = g.integers(0, 256, (rows, wstride), dtype=np.uint8)
    s = g.uniform(1e-3, 1.0, (rows, sstride)).astype(np.float32)
    zx, zw = int(g.integers(-128, 128)), int(g.integers(-8, 8))
    sx = float(np.float32(g.uniform(0.01, 1)))
    rc1, y1 = oracle.matvec_w4a8(x, w, wstride, s, sstride, rows, cols, group, sx, zx, zw)
    rc2, y2 = ref.matvec_w4a8(x, w, wstride, s, sstride, rows, cols, group, sx, zx, zw)
    assert rc1 == rc2 == 0
    np.testing.assert_array_equal(y1.view(np.uint32), y2.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_live_i8_vs_reference(oracle, seed):
    ref = O.RefLib("generic")
    g = np.random.default_rng(2000 + seed)
    rows, cols = int(g.integers(1, 40)), int(g.integers(1, 700))
    stride = cols + int(g.integers(0, 9))
    x = g.integers(-128, 128, cols, dtype=np.int8)
    w = g.integers(-128, 128, (rows, stride), dtype=np.int8)
    zx, zw = int(g.integers(-128, 128)), int(g.integers(-128, 128))
    rc1, y1 = oracle.matvec_i8(x, w, rows, cols, stride, zx, zw)
    rc2, y2 = ref.matvec_i8(x, w, rows, cols, stride, zx, zw)
    assert rc1 == rc2 == 0
    np.testing.assert_array_equal(y1, y2)


@needs_ref
def test_int32_wraparound_matches_reference(oracle):
    """K large enough that (x - zx)(w - zw) sums overflow int32."""
    ref = O.RefLib("generic")
    cols = 40000
    x = np.full(cols, 127, np.int8)
    w = np.full((2, cols), -128, np.int8)
    rc1, y1 = oracle.matvec_i8(x, w, 2, cols, cols, -128, 127)
    rc2, y2 = ref.matvec_i8(x, w, 2, cols, cols, -128, 127)
    assert rc1 == rc2 == 0
    np.testing.assert_array_equal(y1, y2)
    exact = cols * (127 + 128) * (-128 - 127)
    assert int(y1[0]) == ((exact + 2**31) % 2**32) - 2**31


@needs_ref
def test_bad_scale_row_semantics_match_reference(oracle):
    """A bad scale in row r: -1, rows < r written, rows >= r untouched."""
    ref = O.RefLib("generic")
    g = np.random.default_rng(7)
    rows, cols, group = 6, 64, 16
    x = g.integers(-128, 128, cols, dtype=np.int8)
    w = g.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    for bad in (0.0, -1.0, np.inf, np.nan):
        s = g.uniform(0.1, 1.0, (rows, cols // group)).astype(np.float32)
        s[3, 2] = bad
        o1 = np.full(rows, 7.0, np.float32)
        o2 = np.full(rows, 7.0, np.float32)
        rc1, _ = oracle.matvec_w4a8(x, w, cols // 2, s, cols // group, rows, cols, group, 0.5, out=o1)
        rc2, _ = ref.matvec_w4a8(x, w, cols // 2, s, cols // group, rows, cols, group, 0.5, out=o2)
        assert rc1 == rc2 == -1
        np.testing.assert_array_equal(o1.view(np.uint32), o2.view(np.uint32))
        assert (o1[3:] == 7.0).all()


def test_f16_scales_equal_widened_f32(oracle):
    g = np.random.default_rng(11)
    rows, cols, group = 12, 256, 32
    x = g.integers(-128, 128, cols, dtype=np.int8)
    w = g.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    s16 = g.uniform(1e-3, 1e-2, (rows, cols // group)).astype(np.float16)
    rc1, y1 = oracle.matvec_w4a8_f16(x, w, cols // 2, s16.view(np.uint16), cols // group, rows, cols, group, 0.02)
    rc2, y2 = oracle.matvec_w4a8(x, w, cols // 2, s16.astype(np.float32), cols // group, rows, cols, group, 0.02)
    assert rc1 == rc2 == 0
    np.testing.assert_array_equal(y1.view(np.uint32), y2.view(np.uint32))


def test_f16_conversion_exhaustive(oracle):
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.lib.kso_f16_to_f32(int(b)) for b in bits[::37]], np.float32)
    w = want[::37]
    same = (got.view(np.uint32) == w.view(np.uint32)) | (np.isnan(got) & np.isnan(w))
    assert same.all()


def test_pack_unpack_roundtrip():
    g = np.random.default_rng(3)
    v = g.integers(-8, 8, (5, 33), dtype=np.int8)
    np.testing.assert_array_equal(O.unpack_int4(O.pack_int4(v), 33), v)


def test_tolerance_rule():
    y = np.array([1.0, -2.0, 1e-9], np.float32)
    ok, worst = O.w4a8_tolerance_ok(y, y)
    assert ok and worst == 0.0
    ok, _ = O.w4a8_tolerance_ok(y * (1 + 1e-3), y)
    assert not ok
