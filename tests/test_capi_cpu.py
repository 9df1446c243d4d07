"""CPU-only checks of the libkernelsmith (B200) C ABI: the library loads,
exports every function the headers declare, reports the B200 profile, and
rejects invalid arguments with the reference's codes without touching a GPU.
On a host without a GPU a valid compute call must fail with KS_ERR_DEVICE:
there is no CPU fallback."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
INCLUDE = ROOT / "include"


def header_functions() -> set[str]:
    names = set()
    for h in INCLUDE.rglob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(ks_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_headers_declare_the_reference_abi():
    names = header_functions()
    reference_abi = {
        "ks_dot_i8", "ks_matvec_i8", "ks_dot_w4a8", "ks_matvec_w4a8",
        "ks_dot_i8_workspace", "ks_matvec_i8_workspace", "ks_dot_w4a8_workspace",
        "ks_matvec_w4a8_workspace", "ks_quantized_alignment", "ks_w4a8_packed_row_bytes",
        "ks_w4a8_scale_groups", "ks_target_name", "ks_simd_width_f32",
    }
    assert reference_abi <= names


def test_library_exports_every_declared_function(ks):
    L = ks.lib()
    missing = [n for n in sorted(header_functions()) if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_every_declared_function(ks):
    assert header_functions() <= set(ks.SIGNATURES)


def test_only_ks_symbols_exported():
    so = ROOT / "ulir-kernels_b200" / "lib" / "libkernelsmith.so"
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True, check=True).stdout
    syms = [line.split()[-1] for line in out.splitlines() if line.strip()]
    assert syms and all(s.startswith("ks_") for s in syms), [s for s in syms if not s.startswith("ks_")]


def test_static_archive_has_the_abi():
    ar = ROOT / "ulir-kernels_b200" / "lib" / "libkernelsmith.a"
    out = subprocess.run(["nm", "--defined-only", str(ar)], capture_output=True, text=True, check=True).stdout
    for name in ("ks_matvec_w4a8", "ks_matvec_i8", "ks_dot_w4a8", "ks_dot_i8", "ks_target_name"):
        assert re.search(rf"\bT {name}\b", out), name


def test_profile_queries(ks):
    L = ks.lib()
    assert L.ks_target_name() == b"b200-sm100a"
    assert L.ks_simd_width_f32() == 32
    assert L.ks_quantized_alignment() == 16
    assert L.ks_b200_version().decode().endswith("sm_100a")


def test_workspace_and_helpers(ks):
    # reference tests/capi/test_quantized.c:69-83 and :128-141
    L = ks.lib()
    assert L.ks_w4a8_packed_row_bytes(5) == 3
    assert L.ks_w4a8_scale_groups(17, 8) == 3
    assert L.ks_w4a8_scale_groups(17, 0) == 0
    assert L.ks_dot_i8_workspace(16) == 0
    assert L.ks_matvec_i8_workspace(4, 16) == 0
    assert L.ks_dot_w4a8_workspace(16, 8) == 0
    assert L.ks_matvec_w4a8_workspace(4, 16, 8) == 0


def _bufs():
    return (np.array([1], np.int8), np.array([1], np.int8), np.array([0], np.uint8),
            np.array([1.0], np.float32), np.zeros(1, np.int32), np.zeros(1, np.float32))


def test_reference_error_cases(ks):
    """reference tests/capi/test_quantized.c:143-171, plus the other checks of
    ks_quantized.c in their order; all fail before any device access."""
    L = ks.lib()
    x, w, packed, scale, i32, f32 = _bufs()
    p = ks.addr
    E = ks.KS_ERR_INVALID_ARG
    assert L.ks_dot_i8(None, p(w), 1, 0, 0, p(i32), None, 0) == E
    assert L.ks_dot_i8(p(x), p(w), 1, 129, 0, p(i32), None, 0) == E
    assert L.ks_matvec_i8(p(x), p(w), 0, p(i32), 1, 1, 0, 0, None, 0) == E
    assert L.ks_dot_w4a8(p(x), p(packed), p(scale), 1, 0, 1.0, 0, 0, p(f32), None, 0) == E
    assert L.ks_dot_w4a8(p(x), p(packed), p(scale), 1, 1, -1.0, 0, 0, p(f32), None, 0) == E
    assert L.ks_dot_w4a8(p(x), p(packed), p(scale), 1, 1, 1.0, 0, 8, p(f32), None, 0) == E
    # ks_matvec_i8: rows/cols zero, zero point range
    assert L.ks_matvec_i8(p(x), p(w), 1, p(i32), 0, 1, 0, 0, None, 0) == E
    assert L.ks_matvec_i8(p(x), p(w), 1, p(i32), 1, 0, 0, 0, None, 0) == E
    assert L.ks_matvec_i8(p(x), p(w), 1, p(i32), 1, 1, 0, -129, None, 0) == E
    # ks_matvec_w4a8: NULLs, zero sizes, strides, input scale, zero points
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, None, 1, p(f32), 1, 1, 1, 1.0, 0, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 1, p(f32), 1, 1, 0, 1.0, 0, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 1, p(f32), 1, 3, 1, 1.0, 0, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 0, p(f32), 1, 1, 1, 1.0, 0, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 1, p(f32), 1, 1, 1, float("nan"), 0, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 1, p(f32), 1, 1, 1, float("inf"), 0, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 1, p(f32), 1, 1, 1, 1.0, 128, 0, None, 0) == E
    assert L.ks_matvec_w4a8(p(x), p(packed), 1, p(scale), 1, p(f32), 1, 1, 1, 1.0, 0, -9, None, 0) == E
    # extensions
    assert L.ks_b200_matvec_i8_dequant(p(x), p(w), 1, None, 1.0, p(f32), 1, 1, 0, 0) == E
    assert L.ks_b200_matvec_w4a8_async(p(x), p(packed), 1, p(scale), 7, 1, p(f32), 1, 1, 1, 1.0, 0, 0,
                                       None, None) == E
    assert "scale_type" in ks.last_error()


def test_zero_length_dots_do_not_need_a_device(ks):
    """ks_dot_* with k == 0 write 0 (reference ks_quantized.c:57-64, :116-126)."""
    L = ks.lib()
    x, w, packed, scale, i32, f32 = _bufs()
    i32[0] = 99
    f32[0] = 99.0
    assert L.ks_dot_i8(ks.addr(x), ks.addr(w), 0, 0, 0, ks.addr(i32), None, 0) == ks.KS_OK
    assert L.ks_dot_w4a8(ks.addr(x), ks.addr(packed), ks.addr(scale), 0, 4, 1.0, 0, 0, ks.addr(f32),
                         None, 0) == ks.KS_OK
    assert i32[0] == 0 and f32[0] == 0.0


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback(ks):
    L = ks.lib()
    x = np.ones(64, np.int8)
    w = np.ones((2, 32), np.uint8)
    s = np.ones((2, 2), np.float32)
    y = np.zeros(2, np.float32)
    rc = L.ks_matvec_w4a8(ks.addr(x), ks.addr(w), 32, ks.addr(s), 2, ks.addr(y), 2, 64, 32, 1.0, 0, 0, None, 0)
    assert rc == ks.KS_ERR_DEVICE
    assert "CUDA" in ks.last_error() or "device" in ks.last_error()
    assert (y == 0).all()
    yi = np.zeros(2, np.int32)
    rc = L.ks_matvec_i8(ks.addr(x), ks.addr(x), 32, ks.addr(yi), 2, 32, 0, 0, None, 0)
    assert rc == ks.KS_ERR_DEVICE


def test_layout_version_and_importer_argument_checks(ks):
    """KS_QUANT_LAYOUT_VERSION in the header equals the library's, and the
    importer rejects bad arguments before touching any device."""
    import re

    hdr = (ROOT / "include" / "ks_b200.h").read_text()
    m = re.search(r"#define KS_QUANT_LAYOUT_VERSION (\d+)", hdr)
    assert m and int(m.group(1)) == ks.lib().ks_b200_quant_layout_version() == 1
    buf = np.zeros(64, np.uint8)
    L, E = ks.lib(), ks.KS_ERR_INVALID_ARG
    a = ks.addr(buf)
    assert L.ks_b200_import_ggml_q4_0_async(None, 18, 1, 32, 32, a, 32, a, 0, 1, None) == E
    assert L.ks_b200_import_ggml_q4_0_async(a, 18, 1, 48, 32, a, 32, a, 0, 1, None) == E
    assert L.ks_b200_import_ggml_q4_0_async(a, 18, 1, 32, 48, a, 32, a, 0, 1, None) == E
    assert L.ks_b200_import_ggml_q4_0_async(a, 10, 1, 32, 32, a, 32, a, 0, 1, None) == E
    assert L.ks_b200_import_ggml_q4_0_async(a, 18, 1, 32, 32, a, 8, a, 0, 1, None) == E
    assert L.ks_b200_import_ggml_q4_0_async(a, 18, 1, 32, 32, a, 32, a, 5, 1, None) == E


def test_wait_and_status_check_argument_checks(ks):
    """The bounded peer wait and the status check reject bad arguments on the
    host, before any CUDA call."""
    L = ks.lib()
    assert ks.KS_QUANT_LAYOUT_VERSION == L.ks_b200_quant_layout_version()
    buf = np.zeros(64, np.uint32)
    a = ks.addr(buf)
    assert L.ks_b200_peer_arrival_wait_ranks_async(None, 2, a, 1, 0, None, None) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_peer_arrival_wait_ranks_async(a, 2, None, 1, 0, None, None) == ks.KS_ERR_INVALID_ARG
    for nranks in (0, 9, -1):
        assert L.ks_b200_peer_arrival_wait_ranks_async(a, nranks, a + 128, 1, 0, None, None) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_peer_arrival_wait_ranks_async(a, 2, a + 128, 1, 10_000_000_001, None, None) == \
        ks.KS_ERR_INVALID_ARG
    assert "10 s" in ks.last_error()
    assert L.ks_b200_peer_arrival_wait_async(None, a, 1, None, None) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_status_check(None, None) == ks.KS_ERR_INVALID_ARG


def test_decode_layers_argument_checks(ks):
    """The layer-chain entry point checks its arguments on the host, in the
    single-layer call's order, and needs the larger workspace."""
    import ctypes

    L = ks.lib()
    h, i = 4096, 11008
    one = L.ks_b200_decode_layer_workspace(h, i)
    assert L.ks_b200_decode_layers_workspace(h, i) == one + 2 * 16384
    buf = np.zeros(64, np.float32)
    a = ks.addr(buf)
    ptrs = (ctypes.c_void_p * 10)(*([a] * 10))
    norms = (ctypes.c_void_p * 2)(a, a)
    args = [norms, norms, 1e-5, ptrs, ptrs, h, i, 32, a]
    assert L.ks_b200_decode_layers_w4a8_async(0, a, a, *args, one + 32768, None, None) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_decode_layers_w4a8_async(2, a, a, *args, one, None, None) == ks.KS_ERR_WORKSPACE
    bad = (ctypes.c_void_p * 10)(*([a] * 9 + [None]))
    assert L.ks_b200_decode_layers_w4a8_async(2, a, a, norms, norms, 1e-5, bad, ptrs, h, i, 32, a, one + 32768,
                                              None, None) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_decode_layers_w4a8_async(2, a, a, norms, norms, 0.0, ptrs, ptrs, h, i, 32, a, one + 32768,
                                              None, None) == ks.KS_ERR_INVALID_ARG


def test_resident_weights_argument_checks(ks):
    """Registration refuses a layout version other than the library's, and
    bad shapes, before touching a GPU."""
    import ctypes

    L = ks.lib()
    w = np.zeros((4, 16), np.uint8)
    s = np.zeros((4, 1), np.float32)
    h = ctypes.c_void_p()
    args = (ks.addr(w), 16, ks.addr(s), ks.SCALE_F32, 1, 4, 32, 32)
    assert L.ks_b200_w4a8_register(*args, 0, 4, 2, ctypes.byref(h)) == ks.KS_ERR_UNSUPPORTED
    assert "version 2" in ks.last_error() and h.value is None
    assert L.ks_b200_w4a8_register(*args, 3, 2, 1, ctypes.byref(h)) == ks.KS_ERR_INVALID_ARG  # rows 3..4 beyond 4
    assert L.ks_b200_w4a8_register(*args, 0, 0, 1, ctypes.byref(h)) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_w4a8_register(ks.addr(w), 8, ks.addr(s), ks.SCALE_F32, 1, 4, 32, 32, 0, 4, 1,
                                   ctypes.byref(h)) == ks.KS_ERR_INVALID_ARG  # stride < 16 bytes
    assert L.ks_b200_w4a8_register(*args, 0, 4, 1, None) == ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_w4a8_release(None) == ks.KS_OK
