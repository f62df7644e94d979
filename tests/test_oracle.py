"""The CPU oracle pinned against golden vectors and checked for the semantics it restates.

Pins: Q4_K / Q6_K decoding bit-exact against gguf-py's decoder (tests/golden/kquant_golden.npz).
Semantics (hoard call sites in each test): Q8_K activation quantisation, integer sub-block dots,
softmax-before-top-k, renorm with clamp, combine order and the shared-expert gate.
"""
import os

import numpy as np
import pytest
import torch

from hoard_b200 import quant
from oracle import oracle as orc
from tests.moe_fixtures import LayerSpec, make_layer, make_x, oracle_layer, rel_l2

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kquant_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name,qt", [("q4k", quant.Q4_K), ("q6k", quant.Q6_K)])
def test_dequant_bitexact_vs_golden(golden, name, qt):
    blocks = golden[f"{name}_blocks"]
    want = golden[f"{name}_values"]
    got = orc.dequant(qt, blocks).reshape(want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name,qt,tol", [("q4k", quant.Q4_K, 0.10), ("q6k", quant.Q6_K, 0.03)])
def test_encoder_roundtrip(golden, name, qt, tol):
    """Our encoder's bytes decode (by the golden decoder) close to the source rows."""
    src = golden[f"{name}_source_row"]
    nenc = src.size // 256
    dec = golden[f"{name}_values"][:nenc].reshape(src.shape)
    assert rel_l2(dec, src) < tol
    again = quant.quantize(torch.from_numpy(src), qt).numpy().reshape(-1, quant.BLOCK_BYTES[qt])
    assert np.array_equal(again, golden[f"{name}_blocks"][:nenc])


def test_fp16_decode_special_values():
    assert orc.fp16_to_fp32(0x0000) == 0.0
    assert orc.fp16_to_fp32(0x3C00) == 1.0
    assert orc.fp16_to_fp32(0xBC00) == -1.0
    assert orc.fp16_to_fp32(0x0001) == np.float32(2.0 ** -24)
    assert orc.fp16_to_fp32(0x7BFF) == 65504.0
    for h in range(0, 0x7C00, 97):
        assert orc.fp16_to_fp32(h) == float(np.array([h], np.uint16).view(np.float16)[0])


def test_q8k_quantisation_rules():
    """ggml Q8_K: d = 1/(-127/max), q = rne(x * -127/max) (max = signed largest-magnitude value)."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal(1024).astype(np.float32)
    x[256:512] = 0.0                                      # all-zero segment -> d = 0, q = 0
    x[600] = -7.5                                          # negative maximum
    x[700] = 0.5 * (x[700] // 0.5)                         # exercise ties
    d, q, bs = orc.quantize_q8k(x)
    assert d[1] == 0 and not q[256:512].any() and not bs[16:32].any()
    for b in (0, 2, 3):
        seg = x[256 * b:256 * (b + 1)]
        mx = seg[np.argmax(np.abs(seg))]
        iscale = np.float32(-127.0) / np.float32(mx)
        want = np.minimum(127, np.rint(iscale * seg).astype(np.int32))
        assert np.array_equal(q[256 * b:256 * (b + 1)], want)
        assert d[b] == np.float32(1.0) / iscale
        assert np.abs(q[256 * b:256 * (b + 1)]).max() == 127
    assert np.array_equal(bs, q.astype(np.int32).reshape(-1, 16).sum(1))


@pytest.mark.parametrize("qt", [quant.Q4_K, quant.Q6_K])
def test_integer_dot_equals_dequantised_dot(qt):
    """ggml-mode matvec == sum(dequant(w) * dequant(q8(x))) up to f32 rounding."""
    g = torch.Generator().manual_seed(3)
    N, K = 16, 1024
    W = quant.quantize(torch.randn(N, K, generator=g) * 0.02, qt).numpy()
    x = torch.randn(K, generator=g).numpy()
    y = orc.matvec(qt, W, N, K, x, orc.MODE_GGML)
    wd = orc.dequant(qt, W).reshape(N, K).astype(np.float64)
    d, q, _ = orc.quantize_q8k(x)
    xq = (q.reshape(-1, 256).astype(np.float64) * d[:, None].astype(np.float64)).reshape(-1)
    ref = wd @ xq
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-6)
    y_exact = orc.matvec(qt, W, N, K, x, orc.MODE_EXACT)
    assert np.allclose(y_exact, wd @ x.astype(np.float64), rtol=1e-6, atol=1e-7)
    assert rel_l2(y, y_exact) < 2e-2


def test_router_softmax_before_topk_and_renorm():
    """src/run_moe_stream.cpp:352-373: softmax over all E, top-k of probs, renorm with clamp."""
    spec = LayerSpec(H=256, E=16, k=4, I=256)
    L = make_layer(spec, seed=5)
    x = make_x(3, spec.H, seed=5)
    for renorm in (False, True):
        fx, probs, sel, w = orc.route(x, L.w_norm, L.w_router, spec.k, renorm, spec.eps)
        xd = x.astype(np.float64)
        rms = np.sqrt((xd * xd).mean(1, keepdims=True) + spec.eps)
        assert np.allclose(fx, xd / rms * L.w_norm, rtol=1e-5)
        logits = fx.astype(np.float64) @ L.w_router.astype(np.float64).T
        p = np.exp(logits - logits.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        assert np.allclose(probs, p, rtol=1e-5)
        order = np.argsort(-probs, axis=1, kind="stable")[:, :spec.k]
        assert np.array_equal(sel, order)
        ww = np.take_along_axis(probs, sel.astype(np.int64), 1)
        if renorm:
            ww = ww / ww.sum(1, keepdims=True)
            assert np.allclose(w.sum(1), 1.0, atol=1e-6)
        assert np.allclose(w, ww, rtol=1e-6)


def test_renorm_clamp_and_tie_order():
    probs = np.zeros((1, 8), np.float32)
    probs[0, [1, 3, 5]] = 1e-6       # tiny, tied: clamp at 6.103515625e-5 applies, ties -> lower id
    probs[0, 7] = 1e-6
    sel = np.empty((1, 3), np.int32)
    w = np.empty((1, 3), np.float32)
    import ctypes
    orc.lib().orc_topk(probs.ctypes.data_as(ctypes.c_void_p), 8, 3, 1, sel.ctypes.data_as(ctypes.c_void_p),
                       w.ctypes.data_as(ctypes.c_void_p))
    assert sel.tolist() == [[1, 3, 5]]
    assert np.allclose(w, np.float32(1e-6) / np.float32(6.103515625e-5))


@pytest.mark.parametrize("types,renorm,shared", [((quant.Q4_K, quant.Q4_K, quant.Q6_K), True, False),
                                                 ((quant.Q4_K, quant.Q4_K, quant.Q4_K), False, False),
                                                 ((quant.Q4_K, quant.Q4_K, quant.Q6_K), True, True)])
def test_layer_matches_direct_composition(types, renorm, shared):
    """orc_moe_layer == route, then per token sum_j w_j*FFN_j (+ gated shared) + x, j ascending."""
    spec = LayerSpec(H=512, E=8, k=3, I=256, types=types, renorm=renorm, shared=shared)
    L = make_layer(spec, seed=11)
    x = make_x(4, spec.H, seed=11)
    out, sel, w, fx, _ = oracle_layer(L, x, orc.MODE_EXACT)
    gsz = L.gate.shape[1] * L.gate.shape[2]
    for t in range(x.shape[0]):
        acc = np.zeros(spec.H, np.float32)
        for j in range(spec.k):
            e = sel[t, j]
            gl = orc.matvec(types[0], L.gate[e], spec.I, spec.H, fx[t], orc.MODE_EXACT)
            ul = orc.matvec(types[1], L.up[e], spec.I, spec.H, fx[t], orc.MODE_EXACT)
            hh = (gl / (np.float32(1) + np.exp(-gl))) * ul
            y = orc.matvec(types[2], L.down[e], spec.H, spec.I, hh.astype(np.float32), orc.MODE_EXACT)
            acc = acc + w[t, j] * y
        if shared:
            sh = L.shared
            gl = orc.matvec(sh["gate_type"], sh["gate"], spec.I, spec.H, fx[t], orc.MODE_EXACT)
            ul = orc.matvec(sh["up_type"], sh["up"], spec.I, spec.H, fx[t], orc.MODE_EXACT)
            hh = (gl / (np.float32(1) + np.exp(-gl))) * ul
            y = orc.matvec(sh["down_type"], sh["down"], spec.H, spec.I, hh.astype(np.float32), orc.MODE_EXACT)
            sg = 1.0 / (1.0 + np.exp(-np.dot(sh["gate_inp"].astype(np.float64), fx[t].astype(np.float64))))
            acc = acc + y * np.float32(sg)
        assert rel_l2(out[t] - x[t], acc) < 1e-4
    assert gsz > 0


def test_ggml_mode_vs_exact_mode_within_tolerance():
    """Q8_K activation quantisation moves the MoE delta by well under the 2e-2 rel-L2 budget."""
    spec = LayerSpec(H=1024, E=16, k=4, I=512)
    L = make_layer(spec, seed=21)
    x = make_x(8, spec.H, seed=21)
    a = oracle_layer(L, x, orc.MODE_GGML)
    b = oracle_layer(L, x, orc.MODE_EXACT)
    assert np.array_equal(a[1], b[1])
    assert rel_l2(a[0] - x, b[0] - x) < 2e-2


def test_invalid_expert_id_rejected():
    spec = LayerSpec(H=256, E=4, k=2, I=256)
    L = make_layer(spec, seed=2)
    x = make_x(1, spec.H, seed=2)
    sel = np.array([[0, 4]], np.int32)
    with pytest.raises(ValueError):
        orc.experts(spec.H, spec.E, spec.k, spec.I, spec.types, L.gate, L.up, L.down, x, x, sel,
                    np.ones((1, 2), np.float32))
