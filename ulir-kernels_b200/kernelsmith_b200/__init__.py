"""ctypes binding of libkernelsmith (B200).

The product is the C library (ulir-kernels_b200/lib/libkernelsmith.so) and
its headers (include/kernelsmith/*.h, include/ks_b200.h).  This module binds
every exported symbol with its C signature so Python callers -- the tests,
bench.py and the multi-GPU host logic -- go through exactly the entry points
a C caller of the reference libkernelsmith would use.

Buffers are passed as raw addresses: `addr(t)` accepts a torch tensor (device
or host), a numpy array, an int or None.

There is no Python or CPU implementation of any kernel here; if the library
is missing, `lib()` raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_size_t, c_uint16, c_uint32, c_void_p
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
# the in-tree build; KS_B200_LIBRARY names another build of the same library
LIB_PATH = Path(os.environ.get("KS_B200_LIBRARY") or (PKG_DIR / "lib" / "libkernelsmith.so"))

KS_OK = 0
KS_ERR_INVALID_ARG = -1
KS_ERR_WORKSPACE = -2
KS_ERR_UNSUPPORTED = -3
KS_ERR_DEVICE = -4

SCALE_F32 = 0
SCALE_F16 = 1
STATUS_WORDS = 2
STATUS_BAD_SCALE = 0
STATUS_TIMEOUT = 1
IPC_HANDLE_BYTES = 64
KS_QUANT_LAYOUT_VERSION = 1  # include/ks_b200.h; lib().ks_b200_quant_layout_version() returns the built value

_vp = c_void_p
_sz = c_size_t
_i32 = c_int32
_f = c_float

# name -> (restype, argtypes); the C declarations are in include/.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    # ks_common.h
    "ks_target_name": (c_char_p, []),
    "ks_simd_width_f32": (_sz, []),
    # ks_quantized.h
    "ks_dot_i8": (c_int, [_vp, _vp, _sz, _i32, _i32, _vp, _vp, _sz]),
    "ks_matvec_i8": (c_int, [_vp, _vp, _sz, _vp, _sz, _sz, _i32, _i32, _vp, _sz]),
    "ks_dot_w4a8": (c_int, [_vp, _vp, _vp, _sz, _sz, _f, _i32, _i32, _vp, _vp, _sz]),
    "ks_matvec_w4a8": (
        c_int,
        [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32, _vp, _sz],
    ),
    "ks_dot_i8_workspace": (_sz, [_sz]),
    "ks_matvec_i8_workspace": (_sz, [_sz, _sz]),
    "ks_dot_w4a8_workspace": (_sz, [_sz, _sz]),
    "ks_matvec_w4a8_workspace": (_sz, [_sz, _sz, _sz]),
    "ks_quantized_alignment": (_sz, []),
    "ks_w4a8_packed_row_bytes": (_sz, [_sz]),
    "ks_w4a8_scale_groups": (_sz, [_sz, _sz]),
    # ks_b200.h
    "ks_b200_version": (c_char_p, []),
    "ks_b200_last_error": (c_char_p, []),
    "ks_b200_device_count": (c_int, []),
    "ks_b200_matvec_w4a8_f16": (
        c_int,
        [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32],
    ),
    "ks_b200_matvec_w4a8_f16_noalloc": (
        c_int,
        [_vp, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32],
    ),
    "ks_b200_matvec_i8_dequant": (c_int, [_vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _i32, _i32]),
    "ks_b200_matvec_w4a8_async": (
        c_int,
        [_vp, _vp, _sz, _vp, c_int, _sz, _vp, _sz, _sz, _sz, _f, _i32, _i32, _vp, _vp],
    ),
    "ks_b200_matvec_i8_async": (c_int, [_vp, _vp, _sz, _vp, _sz, _sz, _i32, _i32, _vp]),
    "ks_b200_matvec_i8_dequant_async": (
        c_int,
        [_vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _i32, _i32, _vp],
    ),
    "ks_b200_matvec_w4a8_batch_async": (
        c_int,
        [c_int, _vp, _vp, _vp, _vp, _sz, c_int, _sz, _sz, _sz, _sz, _f, _i32, _i32, _vp, _vp],
    ),
    "ks_b200_matvec_i8_batch_async": (c_int, [c_int, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _i32, _i32, _f, _vp]),
    "ks_b200_ipc_get_handle": (c_int, [_vp, _vp, _vp]),
    "ks_b200_ipc_open_handle": (c_int, [_vp, _sz, _vp]),
    "ks_b200_ipc_close_handle": (c_int, [_vp, _sz]),
    "ks_b200_matvec_w4a8_batch_gather_async": (
        c_int,
        [c_int, _vp, _vp, _vp, c_int, _vp, _vp, _sz, _sz, _sz, c_int, _sz, _sz, _sz, _sz, _f, _i32, _i32, _vp,
         _vp, _vp],
    ),
    "ks_b200_peer_arrival_wait_async": (c_int, [_vp, _vp, c_uint32, _vp, _vp]),
    "ks_b200_peer_arrival_wait_ranks_async": (c_int, [_vp, c_int, _vp, c_uint32, ctypes.c_uint64, _vp, _vp]),
    "ks_b200_status_check": (c_int, [_vp, _vp]),
    "ks_b200_decode_layer_workspace": (_sz, [_sz, _sz]),
    "ks_b200_decode_layers_workspace": (_sz, [_sz, _sz]),
    "ks_b200_decode_layers_w4a8_async": (
        c_int,
        [_sz, _vp, _vp, _vp, _vp, _f, _vp, _vp, _sz, _sz, _sz, _vp, _sz, _vp, _vp],
    ),
    "ks_b200_decode_layer_offsets": (c_int, [_sz, _sz, _vp]),
    "ks_b200_decode_layer_w4a8_async": (
        c_int,
        [_vp, _vp, _vp, _vp, _f, _vp, _vp, _sz, _sz, _sz, _vp, _sz, _vp, _vp],
    ),
    "ks_b200_gemm_i8_requant": (c_int, [_vp, _sz, _vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _sz, _sz]),
    "ks_b200_gemm_i8_requant_async": (
        c_int,
        [_vp, _sz, _vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp],
    ),
    "ks_b200_gemm_i8_kernel_path": (c_int, [_vp, _sz, _vp, _sz, _sz, _sz, _sz]),
    "ks_b200_gemm_i8_requant_batch_async": (
        c_int,
        [c_int, _vp, _sz, _vp, _vp, _sz, _vp, _f, _vp, _sz, _sz, _sz, _sz, _vp, _vp],
    ),
    "ks_b200_quant_layout_version": (c_int, []),
    "ks_b200_w4a8_register": (c_int, [_vp, _sz, _vp, c_int, _sz, _sz, _sz, _sz, _sz, _sz, c_int, _vp]),
    "ks_b200_w4a8_weights_info": (c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ks_b200_w4a8_matvec_registered_async": (c_int, [_vp, _vp, _f, _i32, _i32, _vp, _vp, _vp]),
    "ks_b200_w4a8_release": (c_int, [_vp]),
    "ks_b200_gemm_w4a8_async": (
        c_int,
        [_vp, _sz, _vp, _vp, _sz, _vp, c_int, _sz, _vp, _sz, _sz, _sz, _sz, _sz, _vp, _vp],
    ),
    "ks_b200_import_ggml_q4_0_async": (c_int, [_vp, _sz, _sz, _sz, _sz, _vp, _sz, _vp, c_int, _sz, _vp]),
    "ks_b200_w4a8_kernel_path": (c_int, [_vp, _vp, _sz, _vp, c_int, _sz, _sz, _sz, _sz]),
    "ks_b200_i8_kernel_path": (c_int, [_vp, _vp, _sz, _sz, _sz]),
    "ks_b200_matvec_w4a8_f32in_async": (
        c_int,
        [_vp, _vp, _sz, _vp, c_int, _sz, _vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp],
    ),
    "ks_b200_quantize_per_token_async": (c_int, [_vp, _sz, _sz, _sz, _vp, _sz, _vp, _vp]),
    "ks_b200_decode_layer_launches": (c_int, [_sz, _sz, _sz]),
    # include/ks_b200_ggml.h: the GGML MUL_MAT(Q4_0, f32) adapter
    "ks_b200_ggml_q4_0_create": (c_int, [_vp, _sz, _sz, _sz, _vp, _vp]),
    "ks_b200_ggml_q4_0_destroy": (c_int, [_vp]),
    "ks_b200_ggml_q4_0_native": (c_int, [_vp, _vp, _vp, _vp, _vp]),
    "ks_b200_ggml_mul_mat_q4_0_async": (c_int, [_vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp]),
    "ks_b200_ggml_report_get": (None, [_vp]),
    "ks_b200_ggml_report_reset": (None, []),
}

_lib: ctypes.CDLL | None = None


class KernelSmithError(RuntimeError):
    def __init__(self, rc: int, msg: str):
        super().__init__(f"libkernelsmith returned {rc}: {msg}")
        self.rc = rc


def lib() -> ctypes.CDLL:
    """Load libkernelsmith (B200) once and bind every signature."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"libkernelsmith (B200) is not built at {LIB_PATH}; run "
                "`python ulir-kernels_b200/build.py` (or __graft_entry__.build())"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def addr(obj) -> int | None:
    """Raw address of a torch tensor, numpy array, int or None."""
    if obj is None:
        return None
    if isinstance(obj, int):
        return obj
    if hasattr(obj, "data_ptr"):
        return obj.data_ptr()
    if hasattr(obj, "ctypes"):
        return obj.ctypes.data
    raise TypeError(f"cannot take the address of {type(obj)!r}")


def last_error() -> str:
    return lib().ks_b200_last_error().decode()


def check(rc: int) -> None:
    if rc != KS_OK:
        raise KernelSmithError(rc, last_error())


def stream_handle(stream) -> int | None:
    """cudaStream_t of a torch.cuda.Stream (None -> legacy default stream)."""
    if stream is None:
        return None
    return int(stream.cuda_stream)


def matvec_w4a8_async(x, w, w_stride, s, s_stride, y, rows, cols, group, sx, zx=0, zw=0,
                      scale_type=SCALE_F16, status=None, stream=None) -> None:
    """Queue one W4A8 GEMV on `stream` (device buffers); raises on a bad argument."""
    check(
        lib().ks_b200_matvec_w4a8_async(
            addr(x), addr(w), w_stride, addr(s), scale_type, s_stride, addr(y), rows, cols,
            group, sx, zx, zw, addr(status), stream_handle(stream),
        )
    )


def matvec_i8_dequant_async(x, w, w_stride, ws, sa, y, rows, cols, zx=0, zw=0, stream=None) -> None:
    check(
        lib().ks_b200_matvec_i8_dequant_async(
            addr(x), addr(w), w_stride, addr(ws), sa, addr(y), rows, cols, zx, zw,
            stream_handle(stream),
        )
    )


def matvec_i8_async(x, w, w_stride, y, rows, cols, zx=0, zw=0, stream=None) -> None:
    check(
        lib().ks_b200_matvec_i8_async(
            addr(x), addr(w), w_stride, addr(y), rows, cols, zx, zw, stream_handle(stream)
        )
    )


def gemm_i8_requant_async(a, sa, w, ws, out_scale, out, m, n, k, lda=None, ldw=None, ldo=None,
                          acc_out=None, status=None, stream=None) -> None:
    check(
        lib().ks_b200_gemm_i8_requant_async(
            addr(a), lda or k, addr(sa), addr(w), ldw or k, addr(ws), out_scale, addr(out), ldo or n, m, n, k,
            addr(acc_out), addr(status), stream_handle(stream),
        )
    )


def gemm_i8_requant_batch_async(a, sa, w, ws, out_scale, out, m, n, k, lda=None, ldw=None, ldo=None,
                                status=None, stream=None) -> None:
    """count independent INT8 GEMMs with requantisation (lists of device tensors)."""
    count = len(w)
    if not (len(a) == len(sa) == len(ws) == len(out) == count):
        raise ValueError("batch lists differ in length")
    check(
        lib().ks_b200_gemm_i8_requant_batch_async(
            count, _ptr_array(a), lda or k, _ptr_array(sa), _ptr_array(w), ldw or k, _ptr_array(ws), out_scale,
            _ptr_array(out), ldo or n, m, n, k,
            addr(status), stream_handle(stream),
        )
    )


def gemm_w4a8_async(a, sx, w, s, out, m, n, k, group, lda=None, w_stride=None, s_stride=None, ldo=None,
                    scale_type=SCALE_F16, status=None, stream=None) -> None:
    """Batched W4A8 GEMM: out[m, n] = sx[m] * sum_g acc_g * s[n, g] (device buffers)."""
    check(
        lib().ks_b200_gemm_w4a8_async(
            addr(a), lda or k, addr(sx), addr(w), w_stride or (k + 1) // 2, addr(s), scale_type,
            s_stride or -(-k // group), addr(out), ldo or n, m, n, k, group, addr(status), stream_handle(stream),
        )
    )


def import_ggml_q4_0_async(blocks, block_row_stride, rows, cols, group, packed, packed_stride, scales,
                           scale_type=SCALE_F16, scale_stride=None, stream=None) -> None:
    """GGML Q4_0 blocks (device) -> packed int4 + positive group scales (device)."""
    check(
        lib().ks_b200_import_ggml_q4_0_async(
            addr(blocks), block_row_stride, rows, cols, group, addr(packed), packed_stride, addr(scales),
            scale_type, scale_stride or cols // group, stream_handle(stream),
        )
    )


def matvec_w4a8_f32in_async(x, w, w_stride, s, s_stride, y, rows, cols, group, scale_type=SCALE_F16, xq=None,
                            xs=None, status=None, stream=None) -> None:
    """W4A8 GEMV on f32 activations, quantised per token on the device."""
    check(
        lib().ks_b200_matvec_w4a8_f32in_async(
            addr(x), addr(w), w_stride, addr(s), scale_type, s_stride, addr(y), rows, cols, group, addr(xq),
            addr(xs), addr(status), stream_handle(stream),
        )
    )


def quantize_per_token_async(x, ldx, n_tokens, cols, q, ldq, scales, stream=None) -> None:
    """int8 per-token quantisation (s = max|x| / 127, round half to even)."""
    check(lib().ks_b200_quantize_per_token_async(addr(x), ldx, n_tokens, cols, addr(q), ldq, addr(scales),
                                                 stream_handle(stream)))


class GgmlReport(ctypes.Structure):
    """ks_b200_ggml_report (include/ks_b200_ggml.h)."""

    _fields_ = [("conversions", ctypes.c_uint64), ("mul_mat_calls", ctypes.c_uint64), ("tokens", ctypes.c_uint64),
                ("gemv_launches", ctypes.c_uint64), ("gemm_launches", ctypes.c_uint64)]


def ggml_report() -> dict:
    r = GgmlReport()
    lib().ks_b200_ggml_report_get(ctypes.byref(r))
    return {name: int(getattr(r, name)) for name, _ in GgmlReport._fields_}


class GgmlQ4_0:
    """A GGML Q4_0 weight converted once to the native W4A8 layout (device-resident),
    multiplied through ks_b200_ggml_mul_mat_q4_0_async."""

    def __init__(self, blocks, block_row_stride, rows, cols, stream=None):
        h = c_void_p()
        check(lib().ks_b200_ggml_q4_0_create(addr(blocks), block_row_stride, rows, cols, stream_handle(stream),
                                             ctypes.byref(h)))
        self.handle, self.rows, self.cols = h, rows, cols

    def mul_mat_async(self, src1, src1_stride, dst, dst_stride, n_tokens, status=None, stream=None) -> None:
        check(lib().ks_b200_ggml_mul_mat_q4_0_async(self.handle, addr(src1), src1_stride, addr(dst), dst_stride,
                                                    n_tokens, addr(status), stream_handle(stream)))

    def native(self):
        p, s = c_void_p(), c_void_p()
        check(lib().ks_b200_ggml_q4_0_native(self.handle, ctypes.byref(p), ctypes.byref(s), None, None))
        return p.value, s.value

    def close(self) -> None:
        if self.handle:
            check(lib().ks_b200_ggml_q4_0_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr_array(objs):
    arr = (c_void_p * len(objs))(*[addr(o) for o in objs])
    return arr


def matvec_w4a8_batch_async(xs, ws, ss, ys, w_stride, s_stride, rows, cols, group, sx, zx=0, zw=0,
                            scale_type=SCALE_F16, status=None, stream=None) -> None:
    """Queue len(xs) independent W4A8 GEMVs of one shape as one launch."""
    n = len(xs)
    assert len(ws) == len(ss) == len(ys) == n
    check(
        lib().ks_b200_matvec_w4a8_batch_async(
            n, _ptr_array(xs), _ptr_array(ws), _ptr_array(ss), _ptr_array(ys), w_stride, scale_type, s_stride,
            rows, cols, group, sx, zx, zw, addr(status), stream_handle(stream),
        )
    )


def matvec_i8_batch_async(xs, ws, ys, w_stride, rows, cols, zx=0, zw=0, w_scales=None, sa=1.0,
                          stream=None) -> None:
    n = len(xs)
    check(
        lib().ks_b200_matvec_i8_batch_async(
            n, _ptr_array(xs), _ptr_array(ws), _ptr_array(w_scales) if w_scales is not None else None,
            _ptr_array(ys), w_stride, rows, cols, zx, zw, sa, stream_handle(stream),
        )
    )


__all__ = [name for name in dir() if not name.startswith("_")]
