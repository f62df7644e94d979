"""Greedy decode through the device driver (hoard_b200.harness: embedding, attention with QK norm and
NEOX RoPE over an f16 KV cache, the MoE layers through the C ABI, lm-head, argmax) against the CPU
restatement of hoard's schedule (oracle/harness_oracle.py) on seeded models of both attention
variants: OLMoE-like (MHA, QK norm over the whole projection, no top-k renorm) and Qwen3-like (GQA,
per-head QK norm, renorm), 64 generated tokens after a 16-token prompt.

The two sides agree to ~1e-7 until an activation lands within rounding noise of a Q8_K
quantisation boundary (both quantise every matmul input to int8, as ggml does; the float steps
around them -- RoPE, attention sums -- round differently in the last bit on the two sides). Such a
flip moves one int8 value by one step; through the KV cache the difference reaches every later
position, where it triggers further flips, so the two sides settle ~1e-2 apart (relative L2 of
the logits). Teacher forced on the oracle's tokens: median and first step within 2e-2, every step
within 5e-2, and the chosen token must match wherever the oracle's top two logits differ by at
least GAP; free running, the tokens must match up to the first step with a smaller gap. The
operations themselves are checked one by one on identical inputs (test_ops_match_oracle), where
the two sides agree to rounding. The model also goes through a GGUF file (written, then loaded by
hoard_b200.gguf_io) on one of the variants."""
import numpy as np
import pytest
import torch

from hoard_b200 import harness as hx
from tests.moe_fixtures import rel_l2

pytestmark = pytest.mark.gpu

OLMOE_S = hx.ModelConfig("olmoe", 3, 512, 4, 4, 128, 16, 4, 256, 2048, 1e4, 1e-5, "full", False)
QWEN_S = hx.ModelConfig("qwen3moe", 3, 512, 4, 2, 128, 16, 4, 256, 2048, 1e6, 1e-6, "head", True)
N_PROMPT, N_GEN = 16, 64
GAP = 0.05            # logit gap above which one Q8_K rounding flip cannot change the argmax here


def _host(tensors):
    return {k: (ty, ne, t.detach().cpu().numpy()) for k, (ty, ne, t) in tensors.items()}


@pytest.mark.parametrize("cfg,via_gguf", [(OLMOE_S, False), (QWEN_S, True)])
def test_greedy_decode_matches_oracle(tmp_path, cfg, via_gguf):
    from oracle.harness_oracle import OracleDecoder
    dev = torch.device("cuda", 0)
    tensors = hx.seeded_tensors(cfg, seed=11, device=dev)
    host = _host(tensors)
    if via_gguf:
        p = str(tmp_path / "m.gguf")
        hx.write_gguf(p, cfg, tensors)
        model = hx.DecodeModel.from_gguf(p, device=0, max_ctx=128)
        assert model.cfg.qk_norm == cfg.qk_norm and model.cfg.norm_topk == cfg.norm_topk
    else:
        model = hx.DecodeModel(cfg, tensors, device=0, max_ctx=128)
    try:
        rng = np.random.default_rng(5)
        prompt = rng.integers(0, cfg.n_vocab, N_PROMPT).tolist()
        logits = torch.empty(N_GEN, cfg.n_vocab, device=dev)
        got = model.generate(prompt, N_GEN, logits_out=logits)
        want, want_logits = OracleDecoder(cfg, host, max_ctx=128).generate(prompt, N_GEN)
        lg = logits.cpu().numpy()
        # free running: identical tokens up to the first step whose oracle top-2 gap is below GAP
        n_free = 0
        for i in range(N_GEN):
            if got[i] != want[i]:
                top2 = np.sort(want_logits[i])[-2:]
                assert top2[1] - top2[0] < GAP, (i, got[i], want[i], top2)
                break
            n_free += 1
        # teacher forced on the oracle's 64 tokens
        forced = model.score(prompt + want, N_PROMPT).cpu().numpy()
        rel = np.array([rel_l2(forced[i], want_logits[i]) for i in range(N_GEN)])
        assert rel[0] < 2e-2 and np.median(rel) < 2e-2 and rel.max() < 5e-2, rel
        for i in range(N_GEN):
            srt = np.sort(want_logits[i])
            if srt[-1] - srt[-2] >= GAP:
                assert int(np.argmax(forced[i])) == want[i], (i, int(np.argmax(forced[i])), want[i])
        print(f"free-running match {n_free}/{N_GEN}; teacher-forced rel-L2 median {np.median(rel):.1e} max {rel.max():.1e}")
        # one captured CUDA graph per step, position in device memory: the same tokens
        assert model.generate_graphed(prompt, N_GEN) == got
    finally:
        model.close()


def test_ops_match_oracle():
    """Each device operation of the decode step on identical inputs: embedding rows and the quantised
    GEMV (Q8_K activation, integer block dots) against the oracle, RMSNorm, NEOX RoPE + f16 KV store
    and single-query attention against numpy, argmax exactly."""
    from oracle import oracle as orc
    from oracle.harness_oracle import rms_norm, rope_neox
    from hoard_b200 import quant
    from hoard_b200.moe import _ptr, _stream
    dev = torch.device("cuda", 0)
    L, s = hx._hx(), _stream(None)
    g = torch.Generator(device=dev).manual_seed(3)
    H, N = 1024, 384
    # embedding rows of Q4_K and Q6_K tables
    for qt in (hx.Q4_K, hx.Q6_K):
        tab = quant.quantize(torch.randn(50, H, generator=g, device=dev) * 0.02, qt)
        tok = torch.tensor([37], dtype=torch.int32, device=dev)
        x = torch.empty(H, device=dev)
        assert L.hoard_hx_embed(qt, _ptr(tab), H, 50, _ptr(tok), _ptr(x), s) == 0
        want = orc.dequant(qt, tab[37].cpu().numpy())
        assert np.array_equal(x.cpu().numpy(), want), qt
    # GEMV: plane layout, Q8_K activation; plus the residual
    xv = torch.randn(H, generator=g, device=dev)
    q8 = torch.empty(int(L.hoard_hx_q8_bytes(H)), dtype=torch.uint8, device=dev)
    assert L.hoard_hx_quant_q8(_ptr(xv), H, _ptr(q8), s) == 0
    for qt in (hx.Q4_K, hx.Q6_K):
        W = quant.quantize(torch.randn(N, H, generator=g, device=dev) * 0.02, qt)
        Wp = torch.empty_like(W)
        assert L.hoard_hx_repack(qt, _ptr(W), _ptr(Wp), W.numel() // quant.row_bytes(qt, 256), s) == 0
        res = torch.randn(N, generator=g, device=dev)
        y = torch.empty(N, device=dev)
        assert L.hoard_hx_gemv(qt, _ptr(Wp), N, H, _ptr(q8), _ptr(res), _ptr(y), s) == 0
        want = orc.matvec(qt, W.cpu().numpy(), N, H, xv.cpu().numpy(), orc.MODE_GGML) + res.cpu().numpy()
        np.testing.assert_allclose(y.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    # RMSNorm per head
    hd, nh, nkv = 128, 8, 2
    qv = torch.randn(nh * hd, generator=g, device=dev)
    w = (1 + 0.1 * torch.randn(hd, generator=g, device=dev)).float()
    out = torch.empty_like(qv)
    assert L.hoard_hx_rmsnorm(_ptr(qv), nh, hd, 1e-6, _ptr(w), _ptr(out), s) == 0
    np.testing.assert_allclose(out.cpu().numpy(), rms_norm(qv.cpu().numpy(), w.cpu().numpy(), nh, hd, 1e-6),
                               rtol=2e-6, atol=1e-6)
    # RoPE + store, then attention over 37 positions of random cache
    n_pos, pos = 37, 36
    kc = (torch.randn(64, nkv * hd, generator=g, device=dev) * 0.5).half()
    vc = (torch.randn(64, nkv * hd, generator=g, device=dev) * 0.5).half()
    q = torch.randn(nh * hd, generator=g, device=dev)
    k = torch.randn(nkv * hd, generator=g, device=dev)
    v = torch.randn(nkv * hd, generator=g, device=dev)
    q0, k0 = q.cpu().numpy().copy(), k.cpu().numpy().copy()
    assert L.hoard_hx_rope_store(_ptr(q), _ptr(k), _ptr(v), nh, nkv, hd, pos, 1e6, _ptr(kc), _ptr(vc), 1, s) == 0
    np.testing.assert_allclose(q.cpu().numpy(), rope_neox(q0, nh, hd, pos, 1e6), rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(k.cpu().numpy(), rope_neox(k0, nkv, hd, pos, 1e6), rtol=1e-5, atol=2e-5)
    assert np.array_equal(kc[pos].cpu().numpy(), k.cpu().numpy().astype(np.float16))
    assert np.array_equal(vc[pos].cpu().numpy(), v.cpu().numpy().astype(np.float16))
    att = torch.empty(nh * hd, device=dev)
    sc = 1.0 / np.sqrt(hd)
    assert L.hoard_hx_attention(_ptr(q), _ptr(kc), _ptr(vc), nh, nkv, hd, n_pos, sc, _ptr(att), 1, s) == 0
    K = kc[:n_pos].float().cpu().numpy().reshape(n_pos, nkv, hd)
    V = vc[:n_pos].float().cpu().numpy().reshape(n_pos, nkv, hd)
    qh = q.cpu().numpy().reshape(nh, hd)
    for h in range(nh):
        sco = K[:, h // (nh // nkv)] @ qh[h] * sc
        p = np.exp(sco - sco.max())
        p /= p.sum()
        np.testing.assert_allclose(att[h * hd:(h + 1) * hd].cpu().numpy(), p @ V[:, h // (nh // nkv)],
                                   rtol=1e-4, atol=1e-5)
    # argmax: the first index of the maximum
    vals = torch.randn(5000, generator=g, device=dev)
    vals[4000] = 9.0
    vals[123] = 9.0
    idx = torch.empty(1, dtype=torch.int32, device=dev)
    assert L.hoard_hx_argmax(_ptr(vals), 5000, _ptr(idx), s) == 0
    assert int(idx.item()) == 123


def test_speculative_loop_is_lossless():
    """Draft with the top-1 expert, verify k tokens in one batched forward (MoE at T = k), accept the
    matching prefix: the tokens equal plain greedy decoding's."""
    cfg = QWEN_S
    dev = torch.device("cuda", 0)
    model = hx.DecodeModel(cfg, hx.seeded_tensors(cfg, seed=12, device=dev), device=0, max_ctx=128)
    try:
        prompt = np.random.default_rng(6).integers(0, cfg.n_vocab, N_PROMPT).tolist()
        want = model.generate(prompt, 48)
        got, st = model.speculative_generate(prompt, 48, k_draft=4)
        assert got == want
        assert st["rounds"] > 0 and 0 <= st["accepted"] <= st["proposed"]
        assert model.generate(prompt, 48) == want          # the top-k override was restored
    finally:
        model.close()


def test_fused_ops_match_unfused():
    """rmsnorm_q8 == rmsnorm then quant_q8 (up to the order of the squares' sum), gemv_multi == three
    gemv calls exactly, qknorm_rope_store == rmsnorm + rope_store (both norm modes)."""
    from hoard_b200 import quant
    from hoard_b200.moe import _ptr, _stream
    dev = torch.device("cuda", 0)
    L, s = hx._hx(), _stream(None)
    g = torch.Generator(device=dev).manual_seed(9)
    H = 2048
    x = torch.randn(H, generator=g, device=dev)
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).float()
    nq = int(L.hoard_hx_q8_bytes(H))
    qa, qb = torch.zeros(nq, dtype=torch.uint8, device=dev), torch.zeros(nq, dtype=torch.uint8, device=dev)
    cur = torch.empty(H, device=dev)
    assert L.hoard_hx_rmsnorm_q8(_ptr(x), H, 1e-5, _ptr(w), _ptr(qa), s) == 0
    assert L.hoard_hx_rmsnorm(_ptr(x), 1, H, 1e-5, _ptr(w), _ptr(cur), s) == 0
    assert L.hoard_hx_quant_q8(_ptr(cur), H, _ptr(qb), s) == 0
    a8, b8 = qa[:H].view(torch.int8).int(), qb[:H].view(torch.int8).int()
    assert int((a8 - b8).abs().max()) <= 1 and float((a8 != b8).float().mean()) < 1e-2
    # three projections in one launch
    Ws, Wp, ys = [], [], []
    for qt, n in ((hx.Q4_K, 512), (hx.Q4_K, 256), (hx.Q6_K, 256)):
        W = quant.quantize(torch.randn(n, H, generator=g, device=dev) * 0.02, qt)
        P = torch.empty_like(W)
        assert L.hoard_hx_repack(qt, _ptr(W), _ptr(P), W.numel() // quant.row_bytes(qt, 256), s) == 0
        Wp.append((qt, P, n))
    outs = [torch.empty(n, device=dev) for _, _, n in Wp]
    rc = L.hoard_hx_gemv_multi(3, hx._iarr([t for t, _, _ in Wp]), hx._parr([p.data_ptr() for _, p, _ in Wp]),
                               hx._iarr([n for _, _, n in Wp]), H, _ptr(qb), None, hx._parr([o.data_ptr() for o in outs]), s)
    assert rc == 0
    for (qt, P, n), o in zip(Wp, outs):
        y = torch.empty(n, device=dev)
        assert L.hoard_hx_gemv(qt, _ptr(P), n, H, _ptr(qb), None, _ptr(y), s) == 0
        assert torch.equal(o, y)
    # fused QK norm + rope + store against rmsnorm + rope_store
    nh, nkv, hd, pos = 8, 2, 128, 11
    for mode in (1, 2):
        q = torch.randn(nh * hd, generator=g, device=dev)
        k = torch.randn(nkv * hd, generator=g, device=dev)
        v = torch.randn(nkv * hd, generator=g, device=dev)
        qn = (1 + 0.1 * torch.randn(nh * hd if mode == 1 else hd, generator=g, device=dev)).float()
        kn = (1 + 0.1 * torch.randn(nkv * hd if mode == 1 else hd, generator=g, device=dev)).float()
        kc1, vc1 = torch.zeros(16, nkv * hd, dtype=torch.float16, device=dev), torch.zeros(16, nkv * hd, dtype=torch.float16, device=dev)
        kc2, vc2 = kc1.clone(), vc1.clone()
        qo = torch.empty_like(q)
        assert L.hoard_hx_qknorm_rope_store(_ptr(q), _ptr(k), _ptr(v), _ptr(qn), _ptr(kn), mode, 1e-6, nh, nkv, hd, pos,
                                            1e6, _ptr(qo), _ptr(kc1), _ptr(vc1), 1, s) == 0
        q2, k2 = q.clone(), k.clone()
        rows_q, cols_q = (1, nh * hd) if mode == 1 else (nh, hd)
        rows_k, cols_k = (1, nkv * hd) if mode == 1 else (nkv, hd)
        assert L.hoard_hx_rmsnorm(_ptr(q2), rows_q, cols_q, 1e-6, _ptr(qn), _ptr(q2), s) == 0
        assert L.hoard_hx_rmsnorm(_ptr(k2), rows_k, cols_k, 1e-6, _ptr(kn), _ptr(k2), s) == 0
        assert L.hoard_hx_rope_store(_ptr(q2), _ptr(k2), _ptr(v), nh, nkv, hd, pos, 1e6, _ptr(kc2), _ptr(vc2), 1, s) == 0
        torch.testing.assert_close(qo, q2, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(kc1.float(), kc2.float(), rtol=2e-3, atol=2e-3)
        assert torch.equal(vc1, vc2)


def test_bf16_kv_ops_and_qwen3_attention_decode():
    """The KV cache in bf16 (config C3): rope_store writes the rotated k and v rounded to bf16 and
    attention reads them back (checked against numpy on the same rounded values); then greedy decode
    at the Qwen3-30B-A3B attention shapes (GQA 32/4 x 128, per-head QK norm, theta 1e6, vocab 151936,
    E 128 top-8 + renorm, I 768; 2 layers) against the oracle decoder with a bf16 cache, with the
    criteria of test_greedy_decode_matches_oracle."""
    from oracle.harness_oracle import OracleDecoder, bf16_round, rope_neox
    from hoard_b200.moe import _ptr, _stream
    dev = torch.device("cuda", 0)
    L, s = hx._hx(), _stream(None)
    g = torch.Generator(device=dev).manual_seed(21)
    nh, nkv, hd, pos, n_pos = 32, 4, 128, 9, 10
    q = torch.randn(nh * hd, generator=g, device=dev)
    k = torch.randn(nkv * hd, generator=g, device=dev)
    v = torch.randn(nkv * hd, generator=g, device=dev)
    q0, k0, v0 = q.cpu().numpy().copy(), k.cpu().numpy().copy(), v.cpu().numpy().copy()
    kc = torch.randn(16, nkv * hd, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(16, nkv * hd, generator=g, device=dev).to(torch.bfloat16)
    assert L.hoard_hx_rope_store(_ptr(q), _ptr(k), _ptr(v), nh, nkv, hd, pos, 1e6, _ptr(kc), _ptr(vc), 30, s) == 0
    np.testing.assert_allclose(k.cpu().numpy(), rope_neox(k0, nkv, hd, pos, 1e6), rtol=1e-5, atol=2e-5)
    assert np.array_equal(kc[pos].float().cpu().numpy(), bf16_round(k.cpu().numpy()))
    assert np.array_equal(vc[pos].float().cpu().numpy(), bf16_round(v0))
    att = torch.empty(nh * hd, device=dev)
    sc = 1.0 / np.sqrt(hd)
    assert L.hoard_hx_attention(_ptr(q), _ptr(kc), _ptr(vc), nh, nkv, hd, n_pos, sc, _ptr(att), 30, s) == 0
    K = kc[:n_pos].float().cpu().numpy().reshape(n_pos, nkv, hd)
    V = vc[:n_pos].float().cpu().numpy().reshape(n_pos, nkv, hd)
    qh = q.cpu().numpy().reshape(nh, hd)
    for h in range(nh):
        sco = K[:, h // (nh // nkv)] @ qh[h] * sc
        p = np.exp(sco - sco.max())
        p /= p.sum()
        np.testing.assert_allclose(att[h * hd:(h + 1) * hd].cpu().numpy(), p @ V[:, h // (nh // nkv)],
                                   rtol=1e-4, atol=1e-5)
    # decode at the Qwen3 attention shapes, bf16 cache
    cfg = hx.ModelConfig("qwen3moe", 2, 2048, 32, 4, 128, 128, 8, 768, 151936, 1e6, 1e-6, "head", True)
    tensors = hx.seeded_tensors(cfg, seed=23, device=dev)
    model = hx.DecodeModel(cfg, tensors, device=0, max_ctx=64, kv_dtype=torch.bfloat16)
    try:
        prompt = np.random.default_rng(8).integers(0, cfg.n_vocab, N_PROMPT).tolist()
        n_gen = 16
        logits = torch.empty(n_gen, cfg.n_vocab, device=dev)
        got = model.generate(prompt, n_gen, logits_out=logits)
        host = _host(tensors)
        want, want_logits = OracleDecoder(cfg, host, max_ctx=64, kv="bf16").generate(prompt, n_gen)
        n_free = 0
        for i in range(n_gen):
            if got[i] != want[i]:
                top2 = np.sort(want_logits[i])[-2:]
                assert top2[1] - top2[0] < GAP, (i, got[i], want[i], top2)
                break
            n_free += 1
        forced = model.score(prompt + want, N_PROMPT).cpu().numpy()
        rel = np.array([rel_l2(forced[i], want_logits[i]) for i in range(n_gen)])
        assert rel[0] < 2e-2 and np.median(rel) < 2e-2 and rel.max() < 5e-2, rel
        for i in range(n_gen):
            srt = np.sort(want_logits[i])
            if srt[-1] - srt[-2] >= GAP:
                assert int(np.argmax(forced[i])) == want[i], (i, int(np.argmax(forced[i])), want[i])
        print(f"Qwen3 attention shapes, bf16 KV: free-running match {n_free}/{n_gen}; teacher-forced rel-L2 "
              f"median {np.median(rel):.1e} max {rel.max():.1e}")
        assert model.generate_graphed(prompt, n_gen) == got
    finally:
        model.close()
