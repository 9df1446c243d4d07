"""GPU checks of the GGML MUL_MAT(Q4_0, f32) adapter (include/ks_b200_ggml.h)
and the entry points under it, against the oracle:

* ks_b200_quantize_per_token_async: bit-exact per-token int8 codes and scales;
* ks_b200_matvec_w4a8_f32in_async: its quantised input bit-exact, its output
  within the W4A8 tolerance of the oracle GEMV on those codes;
* the adapter: the resident native copy bit-exact to the oracle's Q4_0 import,
  MUL_MAT for 1..70 tokens (GEMV and GEMM paths) within the W4A8 tolerance,
  the invocation report, and greedy token parity on a small seeded Llama-style
  decoder whose matrices are Q4_0 (the reference's integration design:
  invocation counter plus deterministic token parity,
  docs/design/DES-016-known-runtime-first-transformer-integration.md:78-90).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _dev_q4_0(torch, dev, rows, cols, seed):
    vals = O.rng(seed, 0).standard_normal((rows, cols)).astype(np.float32)
    blocks = O.q4_0_encode(vals)
    return blocks, torch.from_numpy(blocks).to(dev)


def test_quantize_per_token_bit_exact(ks, oracle, cuda):
    import torch

    n, cols, ld = 5, 1000, 1024
    x = O.rng(51, 0).standard_normal((n, ld)).astype(np.float32) * 3
    x[2] = 0.0  # an all-zero token: scale 1
    x[3, :cols] = np.linspace(-2.5, 2.5, cols).astype(np.float32) * (127 / 2.5)  # exact ties
    dx = torch.from_numpy(x).to(cuda)
    q = torch.zeros((n, ld), dtype=torch.int8, device=cuda)
    s = torch.zeros(n, dtype=torch.float32, device=cuda)
    ks.quantize_per_token_async(dx, ld, n, cols, q, ld, s)
    torch.cuda.synchronize()
    for t in range(n):
        rc, qr, sr = oracle.quantize_per_token(np.ascontiguousarray(x[t, :cols]))
        assert rc == 0
        np.testing.assert_array_equal(q[t, :cols].cpu().numpy(), qr)
        assert s[t].item() == np.float32(sr)


@pytest.mark.parametrize("rows,cols", [(1024, 4096), (4096, 11008), (300, 512)])
def test_f32in_gemv_matches_oracle(ks, oracle, cuda, rows, cols):
    import torch

    g = O.rng(52, rows)
    x = g.standard_normal(cols).astype(np.float32)
    w = O.pack_int4(g.integers(-8, 8, (rows, cols), dtype=np.int8))
    s16 = g.uniform(1e-3, 1e-2, (rows, cols // 32)).astype(np.float16)
    dx, dw, ds = (torch.from_numpy(a).to(cuda) for a in (x, w, s16.view(np.uint16)))
    y = torch.zeros(rows, dtype=torch.float32, device=cuda)
    xq = torch.zeros(cols, dtype=torch.int8, device=cuda)
    xs = torch.zeros(1, dtype=torch.float32, device=cuda)
    st = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
    ks.matvec_w4a8_f32in_async(dx, dw, cols // 2, ds, cols // 32, y, rows, cols, 32, xq=xq, xs=xs, status=st)
    torch.cuda.synchronize()
    assert st.tolist() == [0, 0]
    rc, q, sx = oracle.quantize_per_token(x)
    np.testing.assert_array_equal(xq.cpu().numpy(), q)
    assert xs.item() == np.float32(sx)
    rc, yr = oracle.matvec_w4a8_f16(q, w, cols // 2, s16.view(np.uint16), cols // 32, rows, cols, 32, sx)
    ok, err = O.w4a8_tolerance_ok(y.cpu().numpy(), yr)
    assert ok, err


class _DeviceView:
    """A device buffer the library owns, seen by torch through the CUDA array
    interface (only read here)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


def _oracle_mul_mat(oracle, packed, s16, rows, cols, x):
    out = np.zeros((x.shape[0], rows), np.float32)
    for t in range(x.shape[0]):
        rc, q, s = oracle.quantize_per_token(np.ascontiguousarray(x[t]))
        assert rc == 0
        rc, out[t] = oracle.matvec_w4a8_f16(q, packed, cols // 2, s16, cols // 32, rows, cols, 32, s)
        assert rc == 0
    return out


@pytest.mark.parametrize("from_host", [False, True])
def test_adapter_native_copy_and_mul_mat(ks, oracle, cuda, from_host):
    import torch

    rows, cols = 768, 1024
    blocks, dblocks = _dev_q4_0(torch, cuda, rows, cols, 53)
    ks.lib().ks_b200_ggml_report_reset()
    W = ks.GgmlQ4_0(blocks if from_host else dblocks, cols // 32 * 18, rows, cols)
    try:
        packed_ref, s16_ref = O.q4_0_import(blocks, rows, cols, 32, True)
        p, s = W.native()
        got_p = torch.as_tensor(_DeviceView(p, (rows, cols // 2), "|u1"), device=cuda).cpu().numpy()
        got_s = torch.as_tensor(_DeviceView(s, (rows, cols // 32), "<i2"), device=cuda).cpu().numpy()
        np.testing.assert_array_equal(got_p, packed_ref)
        np.testing.assert_array_equal(got_s.view(np.uint16), s16_ref)
        st = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)
        for n in (1, 3, 64, 70):
            x = O.rng(54, n).standard_normal((n, cols)).astype(np.float32)
            dx = torch.from_numpy(x).to(cuda)
            y = torch.zeros((n, rows), dtype=torch.float32, device=cuda)
            W.mul_mat_async(dx, cols, y, rows, n, status=st)
            torch.cuda.synchronize()
            assert st.tolist() == [0, 0]
            ref = _oracle_mul_mat(oracle, packed_ref, s16_ref, rows, cols, x)
            got = y.cpu().numpy()
            for t in range(n):
                ok, err = O.w4a8_tolerance_ok(got[t], ref[t])
                assert ok, (n, t, err)
        r = ks.ggml_report()
        assert r["conversions"] == 1 and r["mul_mat_calls"] == 4 and r["tokens"] == 1 + 3 + 64 + 70
        assert r["gemv_launches"] >= 1 and r["gemm_launches"] >= 3
    finally:
        W.close()


def test_adapter_token_parity_small_decoder(ks, oracle, cuda):
    """Greedy decoding of a seeded two-layer Llama-style decoder (vocab 512,
    hidden 256, MLP 512; attention at one position is V) whose matrices are
    Q4_0 tensors: every MUL_MAT through the adapter on the GPU, or through the
    oracle (Q4_0 import, per-token quantisation, W4A8 GEMV); RMSNorm, SiLU and
    the residual adds on the host for both.  The tokens must be identical, and
    the adapter must have run."""
    import torch

    V, d, f, L = 512, 256, 512, 2
    g = O.rng(55, 0)
    emb = g.standard_normal((V, d)).astype(np.float32)
    norms = (g.uniform(0.5, 1.5, (2 * L + 1, d))).astype(np.float32)
    shapes = []
    for _ in range(L):
        shapes += [(d, d), (d, d), (f, d), (f, d), (d, f)]  # v, o, gate, up, down
    shapes.append((V, d))  # output head
    blocks = [O.q4_0_encode((g.standard_normal(s) * (1.0 / np.sqrt(s[1]))).astype(np.float32)) for s in shapes]
    ks.lib().ks_b200_ggml_report_reset()
    gpu_w = [ks.GgmlQ4_0(torch.from_numpy(b).to(cuda), s[1] // 32 * 18, s[0], s[1]) for b, s in zip(blocks, shapes)]
    ora_w = [O.q4_0_import(b, s[0], s[1], 32, True) for b, s in zip(blocks, shapes)]
    st = torch.zeros(ks.STATUS_WORDS, dtype=torch.int32, device=cuda)

    def mm_gpu(k, x):
        rows, cols = shapes[k]
        dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(cuda)
        y = torch.zeros(rows, dtype=torch.float32, device=cuda)
        gpu_w[k].mul_mat_async(dx, cols, y, rows, 1, status=st)
        return y.cpu().numpy()

    def mm_oracle(k, x):
        rows, cols = shapes[k]
        return _oracle_mul_mat(oracle, ora_w[k][0], ora_w[k][1], rows, cols, x[None, :])[0]

    def decode(mm, steps=12, tok=7):
        toks = []
        for _ in range(steps):
            h = emb[tok].copy()
            for l in range(L):
                b = 5 * l
                _, x = oracle.rms_norm(h, norms[2 * l], 1e-5)
                h = (h + mm(b + 1, mm(b + 0, x))).astype(np.float32)
                _, x = oracle.rms_norm(h, norms[2 * l + 1], 1e-5)
                _, sg = oracle.silu(mm(b + 2, x))
                _, a = oracle.mul(sg, mm(b + 3, x))
                h = (h + mm(b + 4, a)).astype(np.float32)
            _, x = oracle.rms_norm(h, norms[2 * L], 1e-5)
            tok = int(np.argmax(mm(5 * L, x)))
            toks.append(tok)
        return toks

    try:
        got = decode(mm_gpu)
        assert st.tolist() == [0, 0]
        want = decode(mm_oracle)
        assert got == want
        r = ks.ggml_report()
        assert r["conversions"] == len(shapes)
        assert r["mul_mat_calls"] == 12 * (5 * L + 1) and r["gemv_launches"] == r["mul_mat_calls"]
    finally:
        for w in gpu_w:
            w.close()
