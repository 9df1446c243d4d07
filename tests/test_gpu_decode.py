"""The fused W4A8 decode layer (hidden 4096, inter
11008, group 32, f16 scales) against the oracle.

Stage by stage, each oracle stage is fed the GPU's own previous intermediate,
so every GEMV is checked on identical int8 activations (W4A8 tolerance) and
every quantisation on identical f32 inputs (bit-exact where the inputs are
identical; RMSNorm's sum order differs from the reference's serial loop, so
its quantised outputs may flip by one step on a few elements, counted).
End to end, the layer's output is compared with the oracle's own chain."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
H, I, G, EPS = 4096, 11008, 32, 1e-5
W4A8_REL_TOL = 1e-4


@pytest.fixture(scope="module", params=["persistent", "four_launches"])
def layer(request, cuda, ks):
    """One layer run twice on one workspace, by the persistent cooperative
    kernel (the default) or by the four chained launches (its fallback)."""
    import os

    import torch

    g = np.random.default_rng(4242)
    shapes = [(3 * H, H), (H, H), (I, H), (I, H), (H, I)]
    W = [g.integers(0, 256, (r, c // 2), dtype=np.uint8) for r, c in shapes]
    S = [g.uniform(1e-3, 1e-2, (r, c // G)).astype(np.float16).view(np.uint16) for r, c in shapes]
    h = g.uniform(-1, 1, H).astype(np.float32)
    n1 = g.uniform(0.5, 1.5, H).astype(np.float32)
    n2 = g.uniform(0.5, 1.5, H).astype(np.float32)
    dW = [torch.from_numpy(w).to(cuda) for w in W]
    dS = [torch.from_numpy(s).to(cuda) for s in S]
    dh, dn1, dn2 = (torch.from_numpy(a).to(cuda) for a in (h, n1, n2))
    L = ks.lib()
    ws_bytes = L.ks_b200_decode_layer_workspace(H, I)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
    out = torch.zeros(H, dtype=torch.float32, device=cuda)
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    import ctypes

    wptr = (ctypes.c_void_p * 5)(*[t.data_ptr() for t in dW])
    sptr = (ctypes.c_void_p * 5)(*[t.data_ptr() for t in dS])
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())  # inputs and the zeroed workspace first

    def run():
        old = os.environ.get("KS_B200_DECODE_PERSISTENT")
        os.environ["KS_B200_DECODE_PERSISTENT"] = "1" if request.param == "persistent" else "0"
        try:
            ks.check(L.ks_b200_decode_layer_w4a8_async(dh.data_ptr(), out.data_ptr(), dn1.data_ptr(),
                                                       dn2.data_ptr(), EPS, wptr, sptr, H, I, G, ws.data_ptr(),
                                                       ws_bytes, status.data_ptr(), ks.stream_handle(stream)))
            stream.synchronize()
            launches.append(L.ks_b200_decode_layer_launches(H, I, G))
        finally:
            if old is None:
                del os.environ["KS_B200_DECODE_PERSISTENT"]
            else:
                os.environ["KS_B200_DECODE_PERSISTENT"] = old
        return out.cpu().numpy().copy(), ws.cpu().numpy().copy()

    launches = []
    y1, w1 = run()
    y2, w2 = run()
    offs = (ctypes.c_size_t * 12)()
    ks.check(L.ks_b200_decode_layer_offsets(H, I, offs))
    o = list(offs)

    def region(k, dtype, n):
        return w1[o[k]:o[k] + n * np.dtype(dtype).itemsize].view(dtype)

    gpu = {"qkv": region(0, np.float32, 3 * H), "h2": region(1, np.float32, H), "gate": region(2, np.float32, I),
           "up": region(3, np.float32, I), "act": region(4, np.float32, I), "s": region(5, np.float32, 4),
           "amax": region(6, np.uint32, 1), "q1": region(7, np.int8, H), "q2": region(8, np.int8, H),
           "q3": region(9, np.int8, H), "q4": region(10, np.int8, I), "h_out": y1}
    # bytes 128..255 of the max|act| region are the persistent kernel's grid
    # barrier words (a generation counter that advances every call)
    for w in (w1, w2):
        w[o[6] + 128:o[6] + 256] = 0
    return dict(W=W, S=S, h=h, n1=n1, n2=n2, gpu=gpu, y2=y2, w2=w2, w1=w1, status=status.cpu().tolist(),
                launches=launches, path=request.param)


def _close(y, ref, what):
    ok, worst = O.w4a8_tolerance_ok(y, ref, W4A8_REL_TOL)
    assert ok, f"{what}: worst err/bound {worst:.3g}"


def _gemv(oracle, layer, k, q, s, rows, cols):
    rc, y = oracle.matvec_w4a8_f16(q, layer["W"][k], cols // 2, layer["S"][k], cols // G, rows, cols, G, s)
    assert rc == 0
    return y


def test_status_and_determinism(layer):
    assert layer["status"] == [0, 0]
    # the path query agrees with the path the fixture forced
    assert layer["launches"] == [1, 1] if layer["path"] == "persistent" else layer["launches"] == [4, 4]
    np.testing.assert_array_equal(layer["gpu"]["h_out"].view(np.uint32), layer["y2"].view(np.uint32))
    np.testing.assert_array_equal(layer["w1"], layer["w2"])


def test_stagewise_against_oracle(layer, oracle):
    g = layer["gpu"]
    s = g["s"]
    # 1. RMSNorm + quantise (sum order differs from the reference's serial loop)
    _, x1 = oracle.rms_norm(layer["h"], layer["n1"], EPS)
    _, q1, s1 = oracle.quantize_per_token(x1)
    assert abs(s[0] - s1) <= 1e-6 * s1
    flips = np.abs(q1.astype(int) - g["q1"].astype(int))
    assert flips.max() <= 1 and flips.sum() <= H // 1000 + 2, flips.sum()
    # 2. QKV GEMV on the GPU's own activations
    _close(g["qkv"], _gemv(oracle, layer, 0, g["q1"], float(s[0]), 3 * H, H), "qkv")
    # 3. V quantise: identical input -> identical output
    _, q2, s2 = oracle.quantize_per_token(np.ascontiguousarray(g["qkv"][2 * H:]))
    assert s2 == s[1]
    np.testing.assert_array_equal(q2, g["q2"])
    # 4. O GEMV + residual
    _close(g["h2"], layer["h"] + _gemv(oracle, layer, 1, g["q2"], float(s[1]), H, H), "h2")
    # 5. RMSNorm + quantise of h2
    _, x3 = oracle.rms_norm(g["h2"], layer["n2"], EPS)
    _, q3, s3 = oracle.quantize_per_token(x3)
    assert abs(s[2] - s3) <= 1e-6 * s3
    flips = np.abs(q3.astype(int) - g["q3"].astype(int))
    assert flips.max() <= 1 and flips.sum() <= H // 1000 + 2, flips.sum()
    # 6. gate / up GEMVs
    _close(g["gate"], _gemv(oracle, layer, 2, g["q3"], float(s[2]), I, H), "gate")
    _close(g["up"], _gemv(oracle, layer, 3, g["q3"], float(s[2]), I, H), "up")
    # 7. SiLU * up (the GPU's expf and the C library's differ by ULPs)
    _, sg = oracle.silu(g["gate"])
    _, act = oracle.mul(sg, g["up"])
    np.testing.assert_allclose(g["act"], act, rtol=2e-6, atol=1e-30)
    assert g["amax"][0] == np.abs(g["act"]).max().view(np.uint32)
    # 8. quantise act with its max: identical input -> identical output
    _, q4, s4 = oracle.quantize_per_token(g["act"])
    assert s4 == s[3]
    np.testing.assert_array_equal(q4, g["q4"])
    # 9. down GEMV + residual
    _close(g["h_out"], g["h2"] + _gemv(oracle, layer, 4, g["q4"], float(s[3]), H, I), "h_out")


def test_end_to_end_against_oracle_chain(layer, oracle):
    ref = O.decode_layer_stages(oracle, layer["h"], layer["n1"], layer["n2"], EPS, layer["W"], layer["S"], H, I, G)
    y = layer["gpu"]["h_out"]
    # The few one-step quantisation flips at the two RMSNorms propagate; the
    # layer output stays within 1e-4 of max(|y|, rms(y)).
    _close(y, ref["h_out"], "h_out end to end")


@pytest.mark.parametrize("path", ["persistent", "four_launches"])
@pytest.mark.parametrize("n_layers", [3, 33])
def test_layer_chain_bitwise_equals_single_layer_calls(ks, cuda, path, n_layers, monkeypatch):
    """ks_b200_decode_layers_w4a8_async runs n layers (33 crosses the
    32-layers-per-launch split) and must give bitwise the output of n
    single-layer calls, each fed the previous one's output."""
    import ctypes

    import torch

    monkeypatch.setenv("KS_B200_DECODE_PERSISTENT", "1" if path == "persistent" else "0")
    L = ks.lib()
    gen = torch.Generator(device=cuda)
    gen.manual_seed(777)
    shapes = [(3 * H, H), (H, H), (I, H), (I, H), (H, I)]
    # three distinct weight sets, cycled over the layers; distinct norms per layer
    sets = [([torch.randint(0, 256, (r, c // 2), dtype=torch.uint8, device=cuda, generator=gen) for r, c in shapes],
             [(torch.rand((r, c // G), device=cuda, generator=gen) * 9e-3 + 1e-3).half() for r, c in shapes])
            for _ in range(3)]
    norms = torch.rand((n_layers, 2, H), device=cuda, generator=gen) + 0.5
    h0 = torch.rand(H, device=cuda, generator=gen) * 2 - 1
    wl = [sets[l % 3][0][k].data_ptr() for l in range(n_layers) for k in range(5)]
    sl = [sets[l % 3][1][k].data_ptr() for l in range(n_layers) for k in range(5)]
    status = torch.zeros(2, dtype=torch.int32, device=cuda)
    # the chain in one call
    ws_bytes = L.ks_b200_decode_layers_workspace(H, I)
    assert ws_bytes >= L.ks_b200_decode_layer_workspace(H, I) + 2 * H * 4
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
    out = torch.zeros(H, dtype=torch.float32, device=cuda)
    torch.cuda.synchronize()
    ks.check(L.ks_b200_decode_layers_w4a8_async(
        n_layers, h0.data_ptr(), out.data_ptr(), (ctypes.c_void_p * n_layers)(*[norms[l, 0].data_ptr() for l in
                                                                                 range(n_layers)]),
        (ctypes.c_void_p * n_layers)(*[norms[l, 1].data_ptr() for l in range(n_layers)]), EPS,
        (ctypes.c_void_p * (5 * n_layers))(*wl), (ctypes.c_void_p * (5 * n_layers))(*sl), H, I, G, ws.data_ptr(),
        ws_bytes, status.data_ptr(), None))
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    # the same layers one call each
    ws1 = torch.zeros(L.ks_b200_decode_layer_workspace(H, I), dtype=torch.uint8, device=cuda)
    acts = torch.zeros((n_layers + 1, H), dtype=torch.float32, device=cuda)
    acts[0] = h0
    for l in range(n_layers):
        ks.check(L.ks_b200_decode_layer_w4a8_async(
            acts[l].data_ptr(), acts[l + 1].data_ptr(), norms[l, 0].data_ptr(), norms[l, 1].data_ptr(), EPS,
            (ctypes.c_void_p * 5)(*wl[5 * l:5 * l + 5]), (ctypes.c_void_p * 5)(*sl[5 * l:5 * l + 5]), H, I, G,
            ws1.data_ptr(), ws1.numel(), status.data_ptr(), None))
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0, 0]
    assert torch.isfinite(out).all() and out.abs().max() > 0
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), acts[n_layers].cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("ahead", ["0", "1", "6"])
def test_chain_l2_lookahead_inert(cuda, ks, monkeypatch, ahead):
    """The persistent kernel's L2 lookahead (slots prefetched while the ring
    is full, KS_B200_DECODE_L2_AHEAD, default 3) only moves weights into L2
    early: a four-layer chain gives bitwise the same output and intermediates
    with any lookahead as with the default."""
    import ctypes

    import torch

    monkeypatch.setenv("KS_B200_DECODE_PERSISTENT", "1")
    L = ks.lib()
    n = 4
    gen = torch.Generator(device=cuda)
    gen.manual_seed(901)
    shapes = [(3 * H, H), (H, H), (I, H), (I, H), (H, I)]
    W = [[torch.randint(0, 256, (r, c // 2), dtype=torch.uint8, device=cuda, generator=gen) for r, c in shapes]
         for _ in range(n)]
    S = [[(torch.rand((r, c // G), device=cuda, generator=gen) * 9e-3 + 1e-3).half() for r, c in shapes]
         for _ in range(n)]
    norms = torch.rand((n, 2, H), device=cuda, generator=gen) + 0.5
    h0 = torch.rand(H, device=cuda, generator=gen) * 2 - 1
    wl = (ctypes.c_void_p * (5 * n))(*[t.data_ptr() for Wl in W for t in Wl])
    sl = (ctypes.c_void_p * (5 * n))(*[t.data_ptr() for Sl in S for t in Sl])
    n1 = (ctypes.c_void_p * n)(*[norms[l, 0].data_ptr() for l in range(n)])
    n2 = (ctypes.c_void_p * n)(*[norms[l, 1].data_ptr() for l in range(n)])
    ws_bytes = L.ks_b200_decode_layers_workspace(H, I)
    offs = (ctypes.c_size_t * 12)()
    ks.check(L.ks_b200_decode_layer_offsets(H, I, offs))

    def run(env):
        if env is None:
            monkeypatch.delenv("KS_B200_DECODE_L2_AHEAD", raising=False)
        else:
            monkeypatch.setenv("KS_B200_DECODE_L2_AHEAD", env)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
        out = torch.zeros(H, dtype=torch.float32, device=cuda)
        status = torch.zeros(2, dtype=torch.int32, device=cuda)
        torch.cuda.synchronize()
        ks.check(L.ks_b200_decode_layers_w4a8_async(n, h0.data_ptr(), out.data_ptr(), n1, n2, EPS, wl, sl, H, I, G,
                                                    ws.data_ptr(), ws_bytes, status.data_ptr(), None))
        torch.cuda.synchronize()
        assert status.cpu().tolist() == [0, 0]
        w = ws.cpu().numpy()
        w[offs[6] + 128:offs[6] + 256] = 0  # the grid-barrier counter advances every call
        return out.cpu().numpy().view(np.uint32), w

    y_def, w_def = run(None)
    y, w = run(ahead)
    np.testing.assert_array_equal(y, y_def)
    np.testing.assert_array_equal(w, w_def)
