"""Skinny INT8 GEMM with requantisation (tcgen05 kind::i8, TMEM accumulators)
against the oracle: int32 accumulators and requantised int8 outputs must be
bit-exact."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _case(seed, m, n, k):
    a = O.rng(seed, 0).integers(-127, 128, (m, k), dtype=np.int8)
    w = O.rng(seed, 1).integers(-127, 128, (n, k), dtype=np.int8)
    sa = O.rng(seed, 2).uniform(1e-3, 1e-2, m).astype(np.float32)
    ws = O.rng(seed, 3).uniform(1e-3, 1e-2, n).astype(np.float32)
    return a, w, sa, ws


def _run_async(ks, torch, cuda, a, w, sa, ws, out_scale, lda=None, ldw=None):
    m, k = a.shape
    n = w.shape[0]
    da, dw = torch.from_numpy(a).to(cuda), torch.from_numpy(w).to(cuda)
    dsa, dws = torch.from_numpy(sa).to(cuda), torch.from_numpy(ws).to(cuda)
    out = torch.zeros((m, n), dtype=torch.int8, device=cuda)
    acc = torch.zeros((m, n), dtype=torch.int32, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    ks.gemm_i8_requant_async(da, dsa, dw, dws, out_scale, out, m, n, k, acc_out=acc, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    return out.cpu().numpy(), acc.cpu().numpy()


@pytest.mark.parametrize("m", [8, 16, 32, 64])
def test_gemm_config_shapes(ks, cuda, oracle, m):
    """M x 4096 x 14336, output scale 0.05 (the skinny batched-decode configuration)."""
    import torch

    n, k = 14336, 4096
    a, w, sa, ws = _case(30 + m, m, n, k)
    assert ks.lib().ks_b200_gemm_i8_kernel_path(ks.addr(a), k, ks.addr(w), k, m, n, k) in (0, 1)
    out, acc = _run_async(ks, torch, cuda, a, w, sa, ws, 0.05)
    # oracle on a row sample of W (row independence), full M
    rows = np.unique(np.concatenate([np.arange(0, 256), np.arange(n - 256, n),
                                     np.random.default_rng(m).choice(n, 512, replace=False)]))
    rc, out_ref, acc_ref = oracle.gemm_i8_requant(a, sa, np.ascontiguousarray(w[rows]), ws[rows], 0.05, want_acc=True)
    assert rc == 0
    np.testing.assert_array_equal(acc[:, rows], acc_ref)
    np.testing.assert_array_equal(out[:, rows], out_ref)
    # requantised values use the whole int8 range (the test is not vacuous)
    assert out.min() == -128 and out.max() == 127


def test_gemm_tc_path_selected(ks, cuda):
    import torch

    a = torch.zeros((64, 4096), dtype=torch.int8, device=cuda)
    w = torch.zeros((14336, 4096), dtype=torch.int8, device=cuda)
    assert ks.lib().ks_b200_gemm_i8_kernel_path(a.data_ptr(), 4096, w.data_ptr(), 4096, 64, 14336, 4096) == 1


@pytest.mark.parametrize("shape", [(1, 128, 128), (5, 200, 320), (17, 1000, 1040), (48, 384, 4224),
                                   (256, 256, 512), (3, 129, 48)])
def test_gemm_ragged_shapes_bit_exact(ks, cuda, oracle, shape):
    """Tokens not a multiple of 16, weight rows not a multiple of 128, K not a
    multiple of 128: out-of-range tiles are zero-filled and masked."""
    import torch

    m, n, k = shape
    a, w, sa, ws = _case(sum(shape), m, n, k)
    out, acc = _run_async(ks, torch, cuda, a, w, sa, ws, 0.01)
    rc, out_ref, acc_ref = oracle.gemm_i8_requant(a, sa, w, ws, 0.01, want_acc=True)
    np.testing.assert_array_equal(acc, acc_ref)
    np.testing.assert_array_equal(out, out_ref)


def test_gemm_generic_path_strided_host(ks, cuda, oracle):
    """Unaligned leading dimensions take the generic kernel; host buffers via the
    synchronous entry point; the gaps of a strided output stay untouched."""
    m, n, k = 7, 300, 200
    lda, ldw, ldo = 203, 201, 310
    g = np.random.default_rng(5)
    abuf = g.integers(-127, 128, m * lda, dtype=np.int8)
    wbuf = g.integers(-127, 128, n * ldw, dtype=np.int8)
    sa = g.uniform(1e-3, 1e-2, m).astype(np.float32)
    ws = g.uniform(1e-3, 1e-2, n).astype(np.float32)
    out = np.full(m * ldo, 99, np.int8)
    L = ks.lib()
    assert L.ks_b200_gemm_i8_kernel_path(ks.addr(abuf), lda, ks.addr(wbuf), ldw, m, n, k) == 0
    rc = L.ks_b200_gemm_i8_requant(ks.addr(abuf), lda, ks.addr(sa), ks.addr(wbuf), ldw, ks.addr(ws), 0.02,
                                   ks.addr(out), ldo, m, n, k)
    assert rc == 0, ks.last_error()
    a = np.lib.stride_tricks.as_strided(abuf, (m, k), (lda, 1)).copy()
    w = np.lib.stride_tricks.as_strided(wbuf, (n, k), (ldw, 1)).copy()
    rc, out_ref = oracle.gemm_i8_requant(a, sa, w, ws, 0.02)
    o = out.reshape(m, ldo)
    np.testing.assert_array_equal(o[:, :n], out_ref)
    assert (o[:, n:] == 99).all()


def test_gemm_sync_device_matches_async(ks, cuda):
    import torch

    m, n, k = 16, 2048, 1024
    a, w, sa, ws = _case(77, m, n, k)
    out_async, _ = _run_async(ks, torch, cuda, a, w, sa, ws, 0.05)
    da, dw = torch.from_numpy(a).to(cuda), torch.from_numpy(w).to(cuda)
    dsa, dws = torch.from_numpy(sa).to(cuda), torch.from_numpy(ws).to(cuda)
    out = torch.zeros((m, n), dtype=torch.int8, device=cuda)
    rc = ks.lib().ks_b200_gemm_i8_requant(da.data_ptr(), k, dsa.data_ptr(), dw.data_ptr(), k, dws.data_ptr(), 0.05,
                                          out.data_ptr(), n, m, n, k)
    assert rc == 0, ks.last_error()
    np.testing.assert_array_equal(out.cpu().numpy(), out_async)


def test_gemm_rejects_bad_args(ks):
    L = ks.lib()
    a = np.zeros(64, np.int8)
    s = np.ones(4, np.float32)
    o = np.zeros(64, np.int8)
    E = ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_gemm_i8_requant(ks.addr(a), 8, ks.addr(s), ks.addr(a), 8, ks.addr(s), 0.0, ks.addr(o), 4, 2, 4,
                                     8) == E
    assert L.ks_b200_gemm_i8_requant(ks.addr(a), 4, ks.addr(s), ks.addr(a), 8, ks.addr(s), 1.0, ks.addr(o), 4, 2, 4,
                                     8) == E
    assert L.ks_b200_gemm_i8_requant(None, 8, ks.addr(s), ks.addr(a), 8, ks.addr(s), 1.0, ks.addr(o), 4, 2, 4,
                                     8) == E


def test_gemm_chain_on_side_stream(ks, cuda, oracle):
    """Three GEMMs queued back to back on a non-default stream (programmatic
    dependent launch on), each one's int8 output the next one's activations:
    every stage must equal the oracle chain bit for bit, so no CTA may read its
    activations or scales before the previous grid has finished."""
    import torch

    m, k = 16, 4096
    g = np.random.default_rng(123)
    a0 = g.integers(-127, 128, (m, k), dtype=np.int8)
    ws_list = [g.integers(-127, 128, (k, k), dtype=np.int8) for _ in range(3)]
    sws = [g.uniform(1e-3, 1e-2, k).astype(np.float32) for _ in range(3)]
    sa = np.full(m, 1.1e-3, np.float32)  # keeps every stage's outputs mostly unsaturated
    out_scale = 0.05
    stream = torch.cuda.Stream(device=cuda)
    dev = lambda x: torch.from_numpy(x).to(cuda)
    da, dsa = dev(a0), dev(sa)
    dws, dsws = [dev(w) for w in ws_list], [dev(s) for s in sws]
    outs = [torch.zeros((m, k), dtype=torch.int8, device=cuda) for _ in range(3)]
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        src = da
        for i in range(3):
            ks.gemm_i8_requant_async(src, dsa, dws[i], dsws[i], out_scale, outs[i], m, k, k, status=status,
                                     stream=stream)
            src = outs[i]
    stream.synchronize()
    assert status.cpu().tolist() == [0, 0]
    ref = a0
    for i in range(3):
        rc, ref = oracle.gemm_i8_requant(ref, sa, ws_list[i], sws[i], out_scale)
        assert rc == 0
        got = outs[i].cpu().numpy()
        np.testing.assert_array_equal(got, ref)
        assert len(np.unique(ref)) > 20  # the chain carries information


@pytest.mark.parametrize("out_scale", [2.0, 6.0, 0.4])
def test_gemm_requant_exact_ties(ks, cuda, oracle, out_scale):
    """Unit scales and small integers make t = acc exactly, so acc / out_scale
    (rounded to f32) falls exactly on half-integers (round half to even) for
    many outputs, and 1 / 6 and 1 / 0.4 are not exact in f32: the
    division-free epilogue must still agree with the divided result everywhere."""
    import torch

    m, n, k = 16, 640, 64
    g = np.random.default_rng(int(out_scale * 8))
    a = g.integers(-3, 4, (m, k), dtype=np.int8)
    w = g.integers(-3, 4, (n, k), dtype=np.int8)
    sa = np.ones(m, np.float32)
    ws = np.ones(n, np.float32)
    out, acc = _run_async(ks, torch, cuda, a, w, sa, ws, out_scale)
    rc, out_ref, acc_ref = oracle.gemm_i8_requant(a, sa, w, ws, out_scale, want_acc=True)
    np.testing.assert_array_equal(acc, acc_ref)
    np.testing.assert_array_equal(out, out_ref)
    q = acc_ref.astype(np.float32) / np.float32(out_scale)
    assert (q - np.floor(q) == np.float32(0.5)).sum() > 100  # exact ties are present


def _batch_inputs(torch, cuda, seed, count, m, n, k, shared_a=False):
    dev = lambda x: torch.from_numpy(x).to(cuda)
    cases = [_case(seed + 7 * i, m, n, k) for i in range(count)]
    if shared_a:
        cases = [(cases[0][0], w, cases[0][2], ws) for _, w, _, ws in cases]
    A = [dev(c[0]) for c in cases]
    W = [dev(c[1]) for c in cases]
    SA = [dev(c[2]) for c in cases]
    WS = [dev(c[3]) for c in cases]
    return cases, A, W, SA, WS


@pytest.mark.parametrize("m", [8, 16, 32, 64])
def test_gemm_batch_matches_single_and_oracle(ks, cuda, oracle, m):
    """Four GEMMs M x 4096 x 14336 in one batched launch: each output equals the
    single-GEMM launch bit for bit and the oracle on a sample of weight rows."""
    import torch

    n, k, count = 14336, 4096, 4
    cases, A, W, SA, WS = _batch_inputs(torch, cuda, 500 + m, count, m, n, k)
    outs = [torch.zeros((m, n), dtype=torch.int8, device=cuda) for _ in range(count)]
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    ks.gemm_i8_requant_batch_async(A, SA, W, WS, 0.05, outs, m, n, k, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    rows = np.unique(np.concatenate([np.arange(0, 128), np.arange(n - 128, n),
                                     np.random.default_rng(m).choice(n, 256, replace=False)]))
    for i, (a, w, sa, ws) in enumerate(cases):
        single, _ = _run_async(ks, torch, cuda, a, w, sa, ws, 0.05)
        got = outs[i].cpu().numpy()
        np.testing.assert_array_equal(got, single)
        rc, out_ref = oracle.gemm_i8_requant(a, sa, np.ascontiguousarray(w[rows]), ws[rows], 0.05)
        assert rc == 0
        np.testing.assert_array_equal(got[:, rows], out_ref)


@pytest.mark.parametrize("shape,count", [((1, 128, 128), 3), ((5, 200, 320), 5), ((17, 1000, 1040), 2),
                                         ((48, 384, 4224), 3), ((3, 129, 48), 18), ((64, 2000, 256), 17)])
def test_gemm_batch_ragged_bit_exact(ks, cuda, oracle, shape, count):
    """Ragged M, N and K; counts above 16 take more than one launch."""
    import torch

    m, n, k = shape
    cases, A, W, SA, WS = _batch_inputs(torch, cuda, sum(shape) + count, count, m, n, k, shared_a=count % 2 == 1)
    outs = [torch.zeros((m, n), dtype=torch.int8, device=cuda) for _ in range(count)]
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    ks.gemm_i8_requant_batch_async(A, SA, W, WS, 0.01, outs, m, n, k, status=status)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    for i, (a, w, sa, ws) in enumerate(cases):
        rc, out_ref = oracle.gemm_i8_requant(a, sa, w, ws, 0.01)
        assert rc == 0
        np.testing.assert_array_equal(outs[i].cpu().numpy(), out_ref)


def test_gemm_batch_unaligned_output_and_strides(ks, cuda, oracle):
    """An output row stride that is not a multiple of 16 takes the direct-store
    epilogue; strided outputs keep their gaps."""
    import torch

    m, n, k, count, ldo = 9, 520, 512, 3, 530
    cases, A, W, SA, WS = _batch_inputs(torch, cuda, 901, count, m, n, k)
    bufs = [torch.full((m * ldo,), 99, dtype=torch.int8, device=cuda) for _ in range(count)]
    ks.gemm_i8_requant_batch_async(A, SA, W, WS, 0.03, bufs, m, n, k, ldo=ldo)
    torch.cuda.synchronize()
    for i, (a, w, sa, ws) in enumerate(cases):
        rc, out_ref = oracle.gemm_i8_requant(a, sa, w, ws, 0.03)
        o = bufs[i].cpu().numpy().reshape(m, ldo)
        np.testing.assert_array_equal(o[:, :n], out_ref)
        assert (o[:, n:] == 99).all()


def test_gemm_batch_chain_on_side_stream(ks, cuda, oracle):
    """Two batched launches on one stream, the second reading the first's int8
    outputs as its activations (programmatic dependent launch on)."""
    import torch

    m, k, count = 16, 2048, 3
    g = np.random.default_rng(321)
    a0 = [g.integers(-127, 128, (m, k), dtype=np.int8) for _ in range(count)]
    w1 = [g.integers(-127, 128, (k, k), dtype=np.int8) for _ in range(count)]
    w2 = [g.integers(-127, 128, (k, k), dtype=np.int8) for _ in range(count)]
    ws = [g.uniform(1e-3, 1e-2, k).astype(np.float32) for _ in range(count)]
    sa = np.full(m, 1.1e-3, np.float32)
    dev = lambda x: torch.from_numpy(x).to(cuda)
    stream = torch.cuda.Stream(device=cuda)
    mid = [torch.zeros((m, k), dtype=torch.int8, device=cuda) for _ in range(count)]
    fin = [torch.zeros((m, k), dtype=torch.int8, device=cuda) for _ in range(count)]
    DA, DW1, DW2, DWS = [dev(x) for x in a0], [dev(x) for x in w1], [dev(x) for x in w2], [dev(x) for x in ws]
    DSA = [dev(sa) for _ in range(count)]
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ks.gemm_i8_requant_batch_async(DA, DSA, DW1, DWS, 0.05, mid, m, k, k, stream=stream)
        ks.gemm_i8_requant_batch_async(mid, DSA, DW2, DWS, 0.05, fin, m, k, k, stream=stream)
    stream.synchronize()
    for i in range(count):
        rc, r1 = oracle.gemm_i8_requant(a0[i], sa, w1[i], ws[i], 0.05)
        rc, r2 = oracle.gemm_i8_requant(r1, sa, w2[i], ws[i], 0.05)
        np.testing.assert_array_equal(fin[i].cpu().numpy(), r2)
        assert len(np.unique(r2)) > 20


def test_gemm_batch_rejects_bad_args(ks, cuda):
    import torch

    L = ks.lib()
    a = torch.zeros((4, 64), dtype=torch.int8, device=cuda)
    s = torch.ones(64, dtype=torch.float32, device=cuda)
    o = torch.zeros((4, 64), dtype=torch.int8, device=cuda)
    arr = lambda *t: ks._ptr_array(list(t))
    E = ks.KS_ERR_INVALID_ARG
    assert L.ks_b200_gemm_i8_requant_batch_async(-1, None, 64, None, None, 64, None, 1.0, None, 64, 4, 64, 64,
                                                 None, None) == E
    assert L.ks_b200_gemm_i8_requant_batch_async(2, arr(a, a), 64, arr(s, s), arr(a, a), 64, arr(s, s), 0.0,
                                                 arr(o, o), 64, 4, 64, 64, None, None) == E
    assert L.ks_b200_gemm_i8_requant_batch_async(2, arr(a, a), 64, arr(s, s), arr(a, None), 64, arr(s, s), 1.0,
                                                 arr(o, o), 64, 4, 64, 64, None, None) == E
    assert L.ks_b200_gemm_i8_requant_batch_async(0, None, 64, None, None, 64, None, 1.0, None, 64, 4, 64, 64,
                                                 None, None) == ks.KS_OK
