"""CPU checks of the GGML MUL_MAT(Q4_0, f32) adapter (include/ks_b200_ggml.h)
and the two entry points it is built on (ks_b200_matvec_w4a8_f32in_async,
ks_b200_quantize_per_token_async): argument checks in order, no CPU fallback
(KS_ERR_DEVICE without a GPU), the invocation report, and -- on the oracle --
the conversion claims the adapter documents: Q4_0 -> native group 32 with
f16 scales loses nothing for blocks with a positive d (else at most half a
native step), and the
W4A8 product stays within the quantisation error of GGML's f32 reference
(the reference's integration design asks for reconstruction error and
output impact, docs/design/DES-016-known-runtime-first-transformer-integration.md:130-134)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle as O

KS_OK, KS_ERR_INVALID_ARG, KS_ERR_UNSUPPORTED, KS_ERR_DEVICE = 0, -1, -3, -4


def _no_gpu():
    import torch

    return not torch.cuda.is_available()


def test_create_argument_checks(ks):
    L = ks.lib()
    h = ctypes.c_void_p()
    blocks = np.zeros((4, 8 * 18), np.uint8)
    assert L.ks_b200_ggml_q4_0_create(None, 8 * 18, 4, 256, None, ctypes.byref(h)) == KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18, 4, 256, None, None) == KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18, 0, 256, None, ctypes.byref(h)) == KS_ERR_INVALID_ARG
    # not a whole Q4_0 block, and not a whole 16-byte scale row
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18, 4, 250, None, ctypes.byref(h)) == KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18, 4, 224, None, ctypes.byref(h)) == KS_ERR_UNSUPPORTED
    # row stride too short, odd stride, odd address
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18 - 2, 4, 256, None, ctypes.byref(h)) == \
        KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18 + 1, 4, 256, None, ctypes.byref(h)) == \
        KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data + 1, 8 * 18, 3, 256, None, ctypes.byref(h)) == \
        KS_ERR_INVALID_ARG
    assert h.value is None


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU behaviour")
def test_create_without_gpu_fails_loudly(ks):
    L = ks.lib()
    h = ctypes.c_void_p()
    blocks = np.zeros((4, 8 * 18), np.uint8)
    assert L.ks_b200_ggml_q4_0_create(blocks.ctypes.data, 8 * 18, 4, 256, None, ctypes.byref(h)) == KS_ERR_DEVICE
    assert h.value is None


def test_mul_mat_argument_checks(ks):
    L = ks.lib()
    x = np.zeros(256, np.float32)
    y = np.zeros(4, np.float32)
    assert L.ks_b200_ggml_mul_mat_q4_0_async(None, x.ctypes.data, 256, y.ctypes.data, 4, 1, None, None) == \
        KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_destroy(None) == KS_ERR_INVALID_ARG
    assert L.ks_b200_ggml_q4_0_native(None, None, None, None, None) == KS_ERR_INVALID_ARG


def test_report_counts_and_resets(ks):
    ks.lib().ks_b200_ggml_report_reset()
    r = ks.ggml_report()
    assert r == {"conversions": 0, "mul_mat_calls": 0, "tokens": 0, "gemv_launches": 0, "gemm_launches": 0}


def test_f32in_and_quantize_argument_checks(ks):
    L = ks.lib()
    x = np.zeros(256, np.float32)
    w = np.zeros((4, 128), np.uint8)
    s = np.zeros((4, 8), np.float16)
    y = np.zeros(4, np.float32)
    q = np.zeros(256, np.int8)
    sc = np.zeros(1, np.float32)
    args = [x.ctypes.data, w.ctypes.data, 128, s.ctypes.data, ks.SCALE_F16, 8, y.ctypes.data, 4, 256, 32,
            None, None, None, None]
    bad = list(args)
    bad[0] = None
    assert L.ks_b200_matvec_w4a8_f32in_async(*bad) == KS_ERR_INVALID_ARG
    bad = list(args)
    bad[2] = 127  # packed stride < cols / 2
    assert L.ks_b200_matvec_w4a8_f32in_async(*bad) == KS_ERR_INVALID_ARG
    bad = list(args)
    bad[4] = 7  # scale type
    assert L.ks_b200_matvec_w4a8_f32in_async(*bad) == KS_ERR_INVALID_ARG
    assert L.ks_b200_quantize_per_token_async(None, 256, 1, 256, q.ctypes.data, 256, sc.ctypes.data, None) == \
        KS_ERR_INVALID_ARG
    assert L.ks_b200_quantize_per_token_async(x.ctypes.data, 255, 1, 256, q.ctypes.data, 256, sc.ctypes.data,
                                              None) == KS_ERR_INVALID_ARG
    assert L.ks_b200_quantize_per_token_async(x.ctypes.data, 256, 0, 256, q.ctypes.data, 256, sc.ctypes.data,
                                              None) == KS_ERR_INVALID_ARG
    if _no_gpu():
        assert L.ks_b200_matvec_w4a8_f32in_async(*args) == KS_ERR_DEVICE
        assert L.ks_b200_quantize_per_token_async(x.ctypes.data, 256, 1, 256, q.ctypes.data, 256, sc.ctypes.data,
                                                  None) == KS_ERR_DEVICE


def test_q4_0_to_native_group32_reconstruction():
    """Native group 32 with f16 scales against GGML's own dequantisation.  A
    block with d > 0 holds (n - 8) * d in [-8d, 7d]: its native scale is d and
    its codes are the nibbles minus 8, so it converts without loss.  With d < 0
    (GGML's encoder gives that when the largest-magnitude value is positive)
    the block reaches +8|d|, which a positive native scale represents only as
    7 * (8|d| / 7): the error stays within half a native step."""
    rows, cols = 16, 512
    vals = O.rng(41, 0).standard_normal((rows, cols)).astype(np.float32)
    blocks = O.q4_0_encode(vals)
    ggml = O.q4_0_decode(blocks, rows, cols).reshape(rows, cols // 32, 32)
    packed, s16 = O.q4_0_import(blocks, rows, cols, 32, True)
    scale = s16.view(np.float16).astype(np.float32)
    q = O.unpack_int4(packed, cols).astype(np.float32).reshape(rows, cols // 32, 32)
    native = q * scale[:, :, None]
    d = np.ascontiguousarray(blocks.reshape(rows, cols // 32, 18)[:, :, 0:2]).view(np.float16)[:, :, 0]
    pos = d.astype(np.float32) > 0
    assert pos.any() and (~pos).any()
    np.testing.assert_array_equal(native[pos], ggml[pos])
    err = np.abs(native - ggml).max(axis=2)
    assert np.all(err <= 0.5 * scale * 1.01)


def test_w4a8_mul_mat_error_against_ggml_f32(oracle):
    """Output impact of the adapter's arithmetic (int8 activations per token,
    int4 weights with f16 group scales) against GGML's f32 reference of the
    same Q4_0 tensor: within the bound of the two quantisation errors, the
    activations' (|x - s*q| <= s/2 per element) and the weights' conversion
    error (|W_native - W_ggml|, zero for blocks with d > 0)."""
    rows, cols = 64, 512
    g = O.rng(42, 0)
    blocks = O.q4_0_encode(g.standard_normal((rows, cols)).astype(np.float32))
    W = O.q4_0_decode(blocks, rows, cols).astype(np.float64)
    packed, s16 = O.q4_0_import(blocks, rows, cols, 32, True)
    scale = s16.view(np.float16).astype(np.float64)
    Wn = (O.unpack_int4(packed, cols).astype(np.float64).reshape(rows, cols // 32, 32) * scale[:, :, None])
    Wn = Wn.reshape(rows, cols)
    rel = []
    for t in range(4):
        x = g.standard_normal(cols).astype(np.float32)
        rc, q, s = oracle.quantize_per_token(x)
        assert rc == 0
        rc, y = oracle.matvec_w4a8_f16(q, packed, cols // 2, s16, cols // 32, rows, cols, 32, s)
        assert rc == 0
        ref = W @ x.astype(np.float64)
        bound = 0.5 * s * np.abs(Wn).sum(axis=1) + np.abs(Wn - W) @ np.abs(x) + 1e-4 * np.abs(ref).max()
        assert np.all(np.abs(y - ref) <= bound)
        rel.append(np.linalg.norm(y - ref) / np.linalg.norm(ref))
    assert max(rel) < 0.1  # output impact: a few percent of the output's norm
