"""GGML Q4_0 -> native W4A8 importer: the oracle (numpy, f32 steps of the
reference's design, DES-015:148-179) against a per-element restatement, and
the properties the design asks importer tests to check (dequantised error)."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

F32 = np.float32


def _blocks(rows, cols, seed, d_range=(-2.0, 2.0)):
    g = np.random.default_rng(seed)
    nb = cols // 32
    b = np.zeros((rows, nb, 18), np.uint8)
    d = g.uniform(*d_range, (rows, nb)).astype(np.float16)
    b[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    b[:, :, 2:] = g.integers(0, 256, (rows, nb, 16), dtype=np.uint8)
    return b.reshape(rows, nb * 18)


def _import_scalar(blocks, rows, cols, group, f16):
    """One element at a time, float32 scalars: the design's pseudo-code."""
    packed = np.zeros((rows, cols // 2), np.uint8)
    scales = np.zeros((rows, cols // group), np.uint16 if f16 else np.float32)
    for r in range(rows):
        dec = []
        for b in range(cols // 32):
            blk = blocks[r, 18 * b: 18 * b + 18]
            d = F32(np.frombuffer(blk[:2].tobytes(), np.float16)[0])
            lo = [F32(int(blk[2 + j] & 0x0F) - 8) * d for j in range(16)]
            hi = [F32(int(blk[2 + j] >> 4) - 8) * d for j in range(16)]
            dec += lo + hi
        for g in range(cols // group):
            vals = dec[g * group:(g + 1) * group]
            lo_v, hi_v = min(vals), max(vals)
            s = max(F32(hi_v / F32(7)), F32(-lo_v * F32(0.125)))
            if s == 0:
                s = F32(1)
            if f16:
                h = np.float16(s)
                if not h > 0:
                    h = np.uint16(1).view(np.float16)
                if np.isinf(h):
                    h = np.float16(65504)
                scales[r, g] = h.view(np.uint16)
                s = F32(h)
            else:
                scales[r, g] = s
            for k, v in enumerate(vals):
                q = int(min(max(np.rint(F32(v / s)), -8), 7))
                kk = g * group + k
                packed[r, kk // 2] |= (q & 0xF) << (4 * (kk % 2))
    return packed, scales


def test_decode_known_block():
    blk = np.zeros((1, 18), np.uint8)
    blk[0, 0:2] = np.array([0.5], np.float16).view(np.uint8)
    blk[0, 2:] = np.array([j | ((15 - j) << 4) for j in range(16)], np.uint8)
    v = O.q4_0_decode(blk, 1, 32)[0]
    np.testing.assert_array_equal(v[:16], (np.arange(16) - 8) * 0.5)
    np.testing.assert_array_equal(v[16:], (7 - np.arange(16)) * 0.5)


@pytest.mark.parametrize("group,f16", [(32, False), (32, True), (64, False), (128, True)])
def test_oracle_matches_elementwise_restatement(group, f16):
    rows, cols = 3, 128
    blocks = _blocks(rows, cols, 5 + group)
    blocks[1, 0:18] = 0  # a zero block (d = 0)
    p1, s1 = O.q4_0_import(blocks, rows, cols, group, f16)
    p2, s2 = _import_scalar(blocks, rows, cols, group, f16)
    np.testing.assert_array_equal(p1, p2)
    np.testing.assert_array_equal(np.asarray(s1).view(np.uint32 if not f16 else np.uint16),
                                  np.asarray(s2).view(np.uint32 if not f16 else np.uint16))


@pytest.mark.parametrize("group", [32, 64, 128, 256])
def test_dequantised_error_within_half_step(group):
    rows, cols = 64, 1024
    blocks = _blocks(rows, cols, 11 + group)
    v = O.q4_0_decode(blocks, rows, cols)
    packed, s = O.q4_0_import(blocks, rows, cols, group, False)
    assert (s > 0).all()
    q = O.unpack_int4(packed, cols).astype(np.float32)
    deq = q * np.repeat(s, group, axis=1)
    err = np.abs(deq - v)
    bound = np.repeat(s, group, axis=1) * 0.5 * (1 + 1e-6)
    assert (err <= bound).all()
    if group == 32:
        # one GGML block per group: negative d is re-expressed with a positive
        # scale; the reconstruction stays within half a step
        assert (O.q4_0_decode(blocks, rows, cols).reshape(rows, -1, 32).max(axis=2) > 0).any()


def test_zero_and_tiny_blocks():
    rows, cols = 2, 64
    blocks = np.zeros((rows, 36), np.uint8)
    tiny = np.array([6e-8], np.float16)  # f16 subnormal
    blocks[1, 0:2] = tiny.view(np.uint8)
    blocks[1, 2:18] = 0xF0  # elements 16..31 = 7 * d, elements 0..15 = -8 * d
    p32, s32 = O.q4_0_import(blocks, rows, cols, 32, False)
    assert s32[0, 0] == 1 and s32[0, 1] == 1 and (p32[0] == 0).all()
    p16, s16 = O.q4_0_import(blocks, rows, cols, 32, True)
    assert (s16.view(np.float16) > 0).all()
