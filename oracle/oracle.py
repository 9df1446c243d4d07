"""CPU oracle for the quantized GEMV path -- TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, always as the checker or the timed CPU reference, never as the product.

Two CPU implementations are exposed:
  * `Oracle`  -- our C restatement (oracle/ks_oracle.c -> libks_oracle.so);
  * `RefLib`  -- the reference's own C sources compiled unmodified
                 (oracle/_ref/libks_ref_{generic,avx2}.so, built by
                 `make -C oracle ref` from the reference tree).

plus numpy helpers that follow the reference's golden-vector conventions
(tests/golden/generate.py in the reference: `default_rng(seed + idx*1009)`,
inclusive integer bounds via integers(low, high + 1), int4 packed low nibble
first).
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int32, c_size_t, c_void_p
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_LIB = ORACLE_DIR / "libks_oracle.so"
REF_DIR = ORACLE_DIR / "_ref"

_vp, _sz, _i32, _f = c_void_p, c_size_t, c_int32, c_float


def _p(a):
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------------ numpy --
def rng(seed: int, idx: int = 0) -> np.random.Generator:
    """The reference generator convention: default_rng(seed + idx * 1009)."""
    return np.random.default_rng(seed + idx * 1009)


def pack_int4(values: np.ndarray) -> np.ndarray:
    """[rows, cols] int values in [-8, 7] -> [rows, ceil(cols/2)] uint8, low nibble = even k."""
    v = np.asarray(values, dtype=np.int8)
    if v.ndim == 1:
        v = v[None, :]
    rows, cols = v.shape
    if cols % 2:
        v = np.concatenate([v, np.zeros((rows, 1), np.int8)], axis=1)
    nib = (v.astype(np.uint8) & 0x0F)
    return (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray, cols: int) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    if p.ndim == 1:
        p = p[None, :]
    lo = (p & 0x0F).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    out = np.empty((p.shape[0], p.shape[1] * 2), np.int16)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    out = np.where(out >= 8, out - 16, out).astype(np.int8)
    return out[:, :cols]


def f16_bits(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float16).view(np.uint16)


# ---------------------------------------------------------------- C libs --
class _CLib:
    def __init__(self, path: Path):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (make -C oracle)")
        self.path = path
        self.lib = ctypes.CDLL(str(path))


class Oracle(_CLib):
    """Our C restatement (oracle/ks_oracle.c)."""

    def __init__(self, path: Path = ORACLE_LIB):
        super().__init__(path)
        L = self.lib
        sig = {
            "kso_dot_i8": [_vp, _vp, _sz, _i32, _i32, _vp],
            "kso_matvec_i8": [_vp, _vp, _sz, _vp, _sz, _sz, _i32, _i32],
            "kso_matvec_i8_dequant": [_vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _i32, _i32],
            "kso_dot_w4a8": [_vp, _vp, _vp, _sz, _sz, _f, _i32, _i32, _vp],
            "kso_matvec_w4a8": [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32],
            "kso_matvec_w4a8_f16": [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32, _vp],
            "kso_gemm_i8_requant": [_vp, _sz, _vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _sz, _sz, _vp],
            "kso_rms_norm_f32": [_vp, _vp, _vp, _sz, _sz, _f],
            "kso_silu_f32": [_vp, _vp, _sz],
            "kso_mul_f32": [_vp, _vp, _vp, _sz],
            "kso_quantize_per_token": [_vp, _sz, _vp, _vp],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = c_int
        for name in ("kso_w4a8_packed_row_bytes",):
            getattr(L, name).argtypes = [_sz]
            getattr(L, name).restype = _sz
        L.kso_w4a8_scale_groups.argtypes = [_sz, _sz]
        L.kso_w4a8_scale_groups.restype = _sz
        L.kso_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.kso_f16_to_f32.restype = c_float

    # Each wrapper returns (rc, result).
    def dot_i8(self, x, w, zx=0, zw=0):
        out = np.zeros(1, np.int32)
        rc = self.lib.kso_dot_i8(_p(x), _p(w), x.size, zx, zw, _p(out))
        return rc, int(out[0])

    def matvec_i8(self, x, w, rows, cols, stride, zx=0, zw=0, out=None):
        out = np.zeros(rows, np.int32) if out is None else out
        rc = self.lib.kso_matvec_i8(_p(x), _p(w), stride, _p(out), rows, cols, zx, zw)
        return rc, out

    def matvec_i8_dequant(self, x, w, rows, cols, stride, ws, sa, zx=0, zw=0):
        out = np.zeros(rows, np.float32)
        rc = self.lib.kso_matvec_i8_dequant(_p(x), _p(w), stride, _p(ws), sa, _p(out), rows, cols, zx, zw)
        return rc, out

    def dot_w4a8(self, x, pw, scales, k, group, sx, zx=0, zw=0):
        out = np.zeros(1, np.float32)
        rc = self.lib.kso_dot_w4a8(_p(x), _p(pw), _p(scales), k, group, sx, zx, zw, _p(out))
        return rc, float(out[0])

    def matvec_w4a8(self, x, pw, pstride, scales, sstride, rows, cols, group, sx, zx=0, zw=0, out=None):
        out = np.zeros(rows, np.float32) if out is None else out
        rc = self.lib.kso_matvec_w4a8(_p(x), _p(pw), pstride, _p(scales), sstride, _p(out), rows, cols,
                                      group, sx, zx, zw)
        return rc, out

    def matvec_w4a8_f16(self, x, pw, pstride, scales16, sstride, rows, cols, group, sx, zx=0, zw=0, out=None):
        out = np.zeros(rows, np.float32) if out is None else out
        scratch = np.zeros(max(1, -(-cols // group)), np.float32)
        rc = self.lib.kso_matvec_w4a8_f16(_p(x), _p(pw), pstride, _p(scales16), sstride, _p(out), rows,
                                          cols, group, sx, zx, zw, _p(scratch))
        return rc, out

    def gemm_i8_requant(self, a, sa, w, ws, out_scale, want_acc=False):
        m, k = a.shape
        n = w.shape[0]
        out = np.zeros((m, n), np.int8)
        acc = np.zeros((m, n), np.int32) if want_acc else None
        rc = self.lib.kso_gemm_i8_requant(_p(a), a.strides[0], _p(sa), _p(w), w.strides[0], _p(ws),
                                          out_scale, _p(out), n, m, n, k, _p(acc))
        return (rc, out, acc) if want_acc else (rc, out)

    def rms_norm(self, x, w, eps):
        out = np.zeros_like(x, dtype=np.float32)
        rc = self.lib.kso_rms_norm_f32(_p(x), _p(w), _p(out), 1 if x.ndim == 1 else x.shape[0],
                                       x.shape[-1], eps)
        return rc, out

    def silu(self, x):
        out = np.zeros_like(x, dtype=np.float32)
        rc = self.lib.kso_silu_f32(_p(x), _p(out), x.size)
        return rc, out

    def mul(self, a, b):
        out = np.zeros_like(a, dtype=np.float32)
        rc = self.lib.kso_mul_f32(_p(a), _p(b), _p(out), a.size)
        return rc, out

    def quantize_per_token(self, x):
        q = np.zeros(x.size, np.int8)
        s = np.zeros(1, np.float32)
        rc = self.lib.kso_quantize_per_token(_p(x), x.size, _p(q), _p(s))
        return rc, q, float(s[0])


class RefLib(_CLib):
    """The reference libkernelsmith's C sources, compiled unmodified."""

    def __init__(self, profile: str = "generic"):
        super().__init__(REF_DIR / f"libks_ref_{profile}.so")
        L = self.lib
        L.ks_matvec_i8.argtypes = [_vp, _vp, _sz, _vp, _sz, _sz, _i32, _i32, _vp, _sz]
        L.ks_matvec_i8.restype = c_int
        L.ks_matvec_w4a8.argtypes = [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32, _vp, _sz]
        L.ks_matvec_w4a8.restype = c_int
        L.ks_dot_i8.argtypes = [_vp, _vp, _sz, _i32, _i32, _vp, _vp, _sz]
        L.ks_dot_i8.restype = c_int
        L.ks_dot_w4a8.argtypes = [_vp, _vp, _vp, _sz, _sz, _f, _i32, _i32, _vp, _vp, _sz]
        L.ks_dot_w4a8.restype = c_int
        L.ks_target_name.restype = ctypes.c_char_p

    def matvec_i8(self, x, w, rows, cols, stride, zx=0, zw=0, out=None):
        out = np.zeros(rows, np.int32) if out is None else out
        rc = self.lib.ks_matvec_i8(_p(x), _p(w), stride, _p(out), rows, cols, zx, zw, None, 0)
        return rc, out

    def matvec_w4a8(self, x, pw, pstride, scales, sstride, rows, cols, group, sx, zx=0, zw=0, out=None):
        out = np.zeros(rows, np.float32) if out is None else out
        rc = self.lib.ks_matvec_w4a8(_p(x), _p(pw), pstride, _p(scales), sstride, _p(out), rows, cols,
                                     group, sx, zx, zw, None, 0)
        return rc, out

    def matvec_w4a8_rows(self, out_addr: int, x, pw_addr: int, pstride, s_addr: int, sstride, rows, cols,
                         group, sx, zx=0, zw=0):
        """Raw-address form used by the threaded CPU baseline (row slices)."""
        return self.lib.ks_matvec_w4a8(_p(x), pw_addr, pstride, s_addr, sstride, out_addr, rows, cols,
                                       group, sx, zx, zw, None, 0)

    def matvec_i8_rows(self, out_addr: int, x, w_addr: int, stride, rows, cols, zx=0, zw=0):
        return self.lib.ks_matvec_i8(_p(x), w_addr, stride, out_addr, rows, cols, zx, zw, None, 0)


def ref_available(profile: str = "generic") -> bool:
    return (REF_DIR / f"libks_ref_{profile}.so").exists()


# ---------------------------------------------------------- parity rules --
def w4a8_tolerance_ok(y: np.ndarray, y_ref: np.ndarray, rel: float = 1e-4) -> tuple[bool, float]:
    """|y - y_ref| <= rel * max(|y_ref[n]|, rms(y_ref)) for every n.

    The reference sums W4A8 products one element at a time in f32; any other
    summation order differs on rows whose terms cancel, so the bound is
    floored at the output's RMS.  Returns (ok, worst ratio err / bound).
    """
    y = np.asarray(y, np.float64)
    r = np.asarray(y_ref, np.float64)
    rms = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    bound = rel * np.maximum(np.abs(r), rms)
    bound = np.where(bound > 0, bound, 1e-30)
    ratio = np.abs(y - r) / bound
    worst = float(ratio.max()) if ratio.size else 0.0
    return worst <= 1.0, worst


# ------------------------------------------------ decode layer (config 4) --
def decode_layer_stages(orc: Oracle, h, norm1, norm2, eps, W, S16, hidden, inter, group):
    """The quantised decode layer composed from the oracle's pieces, every
    intermediate returned.  W[k] packed int4 rows, S16[k] f16 scale bits, for
    k = qkv, o, gate, up, down (see include/ks_b200.h for the formulas)."""
    out = {}

    def gemv(k, q, s, rows, cols):
        rc, y = orc.matvec_w4a8_f16(q, W[k], cols // 2, S16[k], cols // group, rows, cols, group, s)
        assert rc == 0
        return y

    _, x1 = orc.rms_norm(h, norm1, eps)
    _, out["q1"], out["s1"] = orc.quantize_per_token(x1)
    out["qkv"] = gemv(0, out["q1"], out["s1"], 3 * hidden, hidden)
    v = np.ascontiguousarray(out["qkv"][2 * hidden:])
    _, out["q2"], out["s2"] = orc.quantize_per_token(v)
    o = gemv(1, out["q2"], out["s2"], hidden, hidden)
    out["h2"] = (h + o).astype(np.float32)
    _, x3 = orc.rms_norm(out["h2"], norm2, eps)
    _, out["q3"], out["s3"] = orc.quantize_per_token(x3)
    out["gate"] = gemv(2, out["q3"], out["s3"], inter, hidden)
    out["up"] = gemv(3, out["q3"], out["s3"], inter, hidden)
    _, sg = orc.silu(out["gate"])
    _, out["act"] = orc.mul(sg, out["up"])
    _, out["q4"], out["s4"] = orc.quantize_per_token(out["act"])
    d = gemv(4, out["q4"], out["s4"], hidden, inter)
    out["h_out"] = (out["h2"] + d).astype(np.float32)
    return out


# ---- GGML Q4_0 -> native W4A8 (the reference's offline conversion) ----------
Q4_0_BLOCK_BYTES = 18  # f16 d + 16 bytes of nibbles, 32 elements


def q4_0_decode(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """GGML Q4_0 blocks [rows, cols/32 * 18] -> f32 [rows, cols], as the
    reference's design restates GGML's dequantisation
    (docs/design/DES-015-quantized-layout-abi-and-integration-conversion-paths.md:155-160):
    element j < 16 is ((qs[j] & 0x0F) - 8) * d, element j + 16 is ((qs[j] >> 4) - 8) * d."""
    nb = cols // 32
    b = np.ascontiguousarray(blocks[:, : nb * Q4_0_BLOCK_BYTES]).reshape(rows, nb, Q4_0_BLOCK_BYTES)
    d = np.ascontiguousarray(b[:, :, 0:2]).view(np.float16).reshape(rows, nb).astype(np.float32)
    qs = b[:, :, 2:]
    lo = (qs & 0x0F).astype(np.int32) - 8
    hi = (qs >> 4).astype(np.int32) - 8
    vals = np.concatenate([lo, hi], axis=2).astype(np.float32) * d[:, :, None]
    return vals.reshape(rows, cols).astype(np.float32)


def q4_0_import(blocks: np.ndarray, rows: int, cols: int, group: int, f16_scales: bool):
    """Q4_0 -> native W4A8 following DES-015:162-174 step by step in f32:
    per native group scale = max(max(v) / 7, -min(v) / 8), 1 if 0;
    q = clamp(round_half_even(v / scale), -8, 7); value k in byte k/2, low
    nibble for even k.  With f16 scales the scale is rounded to f16 first (kept
    positive and finite) and the codes use that value.  Returns (packed uint8
    [rows, cols/2], scales f32 or f16-bits uint16 [rows, cols/group])."""
    v = q4_0_decode(blocks, rows, cols).reshape(rows, cols // group, group)
    with np.errstate(invalid="ignore"):
        lo = np.fmin.reduce(v, axis=2)
        hi = np.fmax.reduce(v, axis=2)
    scale = np.fmax(hi / np.float32(7), -lo * np.float32(0.125)).astype(np.float32)
    scale[scale == 0] = np.float32(1)
    if f16_scales:
        s16 = scale.astype(np.float16)
        s16[~(s16 > 0)] = np.uint16(1).view(np.float16)  # smallest positive f16
        s16[np.isinf(s16)] = np.float16(65504)
        scale = s16.astype(np.float32)
    q = np.clip(np.rint(v / scale[:, :, None]), -8, 7).astype(np.int8).reshape(rows, cols)
    packed = pack_int4(q)
    return packed, (s16.view(np.uint16) if f16_scales else scale)


def q4_0_encode(values: np.ndarray, rng_: np.random.Generator | None = None) -> np.ndarray:
    """f32 [rows, cols] -> Q4_0 blocks, a test-input generator: GGML's scale
    convention (d = the block's signed absolute maximum / -8, so d may be
    negative), nibble = clamp(round(v / d) + 8, 0, 15)."""
    rows, cols = values.shape
    nb = cols // 32
    v = values.reshape(rows, nb, 32).astype(np.float32)
    idx = np.argmax(np.abs(v), axis=2)
    mx = np.take_along_axis(v, idx[:, :, None], axis=2)[:, :, 0]
    d = (mx / np.float32(-8)).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df != 0, np.float32(1) / np.where(df != 0, df, np.float32(1)), np.float32(0))
    q = np.clip(np.round(v * inv[:, :, None]) + 8, 0, 15).astype(np.uint8)
    qs = (q[:, :, :16] & 0x0F) | ((q[:, :, 16:] & 0x0F) << 4)
    out = np.zeros((rows, nb, Q4_0_BLOCK_BYTES), np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = qs
    return out.reshape(rows, nb * Q4_0_BLOCK_BYTES)
