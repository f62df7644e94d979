"""The hybrid (Qwen3-Next, config C5) layer kinds through the device driver against the CPU oracle
(oracle/harness_oracle.py): the gated delta-net step (causal conv over the last inputs, L2-normalised
q/k, the delta-rule state update, gated RMSNorm) over a sequence of tokens, the gated full attention
pieces (fused q + gate rows, per-head QK norm, NEOX RoPE on the first 64 of 256 values, sigmoid output
gate), and greedy decode of a reduced-depth C5-shape model (3 delta-net layers + 1 gated attention
layer; E 512, top-10 + renorm, I 512, gated shared expert; vocab 151936): the first token's logits to
rounding, tokens equal wherever the oracle's top-2 gap is clear, and the teacher-forced drift of
Q8_K rounding flips carried by the recurrent state bounded. The oracle restates the published gated
delta-net recurrence (ggml's fused kernel is not in the reference), so these checks pin the
implementation to that restatement."""
import numpy as np
import pytest
import torch

from hoard_b200 import harness as hx
from tests.moe_fixtures import rel_l2

pytestmark = pytest.mark.gpu

N_PROMPT, GAP = 16, 0.05


def _host(tensors):
    return {k: (ty, ne, t.detach().cpu().numpy()) for k, (ty, ne, t) in tensors.items()}


def test_gdn_step_sequence_matches_oracle():
    from oracle.harness_oracle import gdn_step
    from hoard_b200.moe import _ptr, _stream
    dev = torch.device("cuda", 0)
    L, s = hx._hx(), _stream(None)
    g = torch.Generator(device=dev).manual_seed(31)
    Hk, Hv, D, dc, eps = 4, 8, 128, 4, 1e-6
    cd = (2 * Hk + Hv) * D
    conv_w = (torch.randn(cd, dc, generator=g, device=dev) * 0.3).float()
    dt_bias = (torch.randn(Hv, generator=g, device=dev) * 0.5).float()
    ssm_a = (-torch.exp(torch.rand(Hv, generator=g, device=dev) * 2.7)).float()
    norm_w = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).float()
    ring = torch.full((dc, cd), 7.0, device=dev)          # stale contents: position 0 must not read them
    state = torch.zeros(Hv, D, D, device=dev)
    out = torch.empty(Hv * D, device=dev)
    S_ref = np.zeros((Hv, D, D), np.float32)
    hist = []
    pos_dev = torch.zeros(1, dtype=torch.int32, device=dev)
    for pos in range(7):
        qkv = torch.randn(cd, generator=g, device=dev)
        z = torch.randn(Hv * D, generator=g, device=dev)
        ba = torch.randn(2 * Hv, generator=g, device=dev)
        pos_dev.fill_(pos)
        pd = _ptr(pos_dev) if pos % 2 else None            # both position forms
        assert L.hoard_hx_gdn_step(_ptr(qkv), _ptr(z), _ptr(ba), _ptr(conv_w), _ptr(ring), _ptr(dt_bias),
                                   _ptr(ssm_a), _ptr(norm_w), _ptr(state), Hv, Hk, D, dc, eps, pos, pd, _ptr(out),
                                   s) == 0
        q_np = qkv.cpu().numpy()
        want = gdn_step(q_np, z.cpu().numpy(), ba.cpu().numpy(), conv_w.cpu().numpy().reshape(-1), hist,
                        dt_bias.cpu().numpy(), ssm_a.cpu().numpy(), norm_w.cpu().numpy(), S_ref, Hv, Hk, D, dc, eps)
        hist.append(q_np)
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=2e-4, atol=2e-5)
        np.testing.assert_allclose(state.cpu().numpy(), S_ref, rtol=2e-4, atol=2e-6)
    # argument errors
    assert L.hoard_hx_gdn_step(_ptr(qkv), _ptr(z), _ptr(ba), _ptr(conv_w), _ptr(ring), _ptr(dt_bias), _ptr(ssm_a),
                               _ptr(norm_w), _ptr(state), Hv, 3, D, dc, eps, 0, None, _ptr(out), s) != 0
    assert L.hoard_hx_gdn_step(_ptr(qkv), _ptr(z), _ptr(ba), _ptr(conv_w), _ptr(ring), _ptr(dt_bias), _ptr(ssm_a),
                               _ptr(norm_w), _ptr(state), Hv, Hk, 64, dc, eps, 0, None, _ptr(out), s) != 0


def test_gated_attention_ops_match_numpy():
    from oracle.harness_oracle import rms_norm, rope_neox, sigmoid
    from hoard_b200.moe import _ptr, _stream
    dev = torch.device("cuda", 0)
    L, s = hx._hx(), _stream(None)
    g = torch.Generator(device=dev).manual_seed(37)
    nh, nkv, hd, n_rot, pos, base, eps = 16, 2, 256, 64, 11, 1e7, 1e-6
    qg = torch.randn(nh * 2 * hd, generator=g, device=dev)          # [q | gate] per head
    k = torch.randn(nkv * hd, generator=g, device=dev)
    v = torch.randn(nkv * hd, generator=g, device=dev)
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device=dev)).float()
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device=dev)).float()
    kc = torch.randn(32, nkv * hd, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(32, nkv * hd, generator=g, device=dev).to(torch.bfloat16)
    q_out = torch.empty(nh * hd, device=dev)
    assert L.hoard_hx_qknorm_rope_store_ex(_ptr(qg), _ptr(k), _ptr(v), _ptr(qn), _ptr(kn), 2, eps, nh, nkv, hd, 2 * hd,
                                           n_rot, pos, None, 32, base, _ptr(q_out), _ptr(kc), _ptr(vc), 30, s) == 0
    qg_np = qg.cpu().numpy().reshape(nh, 2, hd)
    q_want = rope_neox(rms_norm(qg_np[:, 0].reshape(-1), qn.cpu().numpy(), nh, hd, eps), nh, hd, pos, base, n_rot)
    k_want = rope_neox(rms_norm(k.cpu().numpy(), kn.cpu().numpy(), nkv, hd, eps), nkv, hd, pos, base, n_rot)
    np.testing.assert_allclose(q_out.cpu().numpy(), q_want, rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(kc[pos].float().cpu().numpy(), k_want, rtol=1e-2, atol=1e-2)   # bf16 store
    n_pos = pos + 1
    att = torch.empty(nh * hd, device=dev)
    sc = 1.0 / np.sqrt(hd)
    assert L.hoard_hx_attention_ex(_ptr(q_out), _ptr(kc), _ptr(vc), nh, nkv, hd, n_pos, None, sc,
                                   _ptr(qg) + 4 * hd, 2 * hd, _ptr(att), 30, s) == 0
    K = kc[:n_pos].float().cpu().numpy().reshape(n_pos, nkv, hd)
    V = vc[:n_pos].float().cpu().numpy().reshape(n_pos, nkv, hd)
    qh = q_out.cpu().numpy().reshape(nh, hd)
    for h in range(nh):
        sco = K[:, h // (nh // nkv)] @ qh[h] * sc
        p = np.exp(sco - sco.max())
        p /= p.sum()
        np.testing.assert_allclose(att[h * hd:(h + 1) * hd].cpu().numpy(),
                                   (p @ V[:, h // (nh // nkv)]) * sigmoid(qg_np[h, 1]), rtol=1e-4, atol=1e-5)


def test_c5_shape_decode_matches_oracle():
    from oracle.harness_oracle import OracleDecoder
    dev = torch.device("cuda", 0)
    c5 = hx.C5_QWEN3NEXT
    cfg = hx.ModelConfig(c5.arch, 4, c5.n_embd, c5.n_head, c5.n_head_kv, c5.head_dim, c5.n_expert, c5.n_expert_used,
                         c5.n_ff, c5.n_vocab, c5.freq_base, c5.eps, c5.qk_norm, c5.norm_topk, n_ff_shexp=c5.n_ff_shexp,
                         full_attn_interval=c5.full_attn_interval, attn_gate=c5.attn_gate, rope_dim=c5.rope_dim,
                         ssm_d_state=c5.ssm_d_state, ssm_n_group=c5.ssm_n_group, ssm_dt_rank=c5.ssm_dt_rank,
                         ssm_d_conv=c5.ssm_d_conv)
    tensors = hx.seeded_tensors(cfg, seed=41, device=dev)
    model = hx.DecodeModel(cfg, tensors, device=0, max_ctx=64, kv_dtype=torch.bfloat16)
    try:
        prompt = np.random.default_rng(9).integers(0, cfg.n_vocab, N_PROMPT).tolist()
        n_gen = 16
        logits = torch.empty(n_gen, cfg.n_vocab, device=dev)
        got = model.generate(prompt, n_gen, logits_out=logits)
        want, want_logits = OracleDecoder(cfg, _host(tensors), max_ctx=64, kv="bf16").generate(prompt, n_gen)
        n_free = 0
        for i in range(n_gen):
            if got[i] != want[i]:
                top2 = np.sort(want_logits[i])[-2:]
                assert top2[1] - top2[0] < GAP, (i, got[i], want[i], top2)
                break
            n_free += 1
        # the first token (no state, no cache history yet): the two sides agree to rounding
        first = model.score(prompt[:2], 1).cpu().numpy()[0]
        first_want = OracleDecoder(cfg, _host(tensors), max_ctx=64, kv="bf16").step(prompt[0], 0)
        rel0 = rel_l2(first, first_want)
        assert rel0 < 1e-3, rel0
        # teacher forced: a Q8_K rounding flip (an int8 value one step apart) enters the delta-net state
        # and the KV cache and is carried to every later token, so the sides drift further apart than on
        # the attention-only models (median 3e-2 measured over 16 tokens after a 16-token prompt)
        forced = model.score(prompt + want, N_PROMPT).cpu().numpy()
        rel = np.array([rel_l2(forced[i], want_logits[i]) for i in range(n_gen)])
        assert rel[0] < 2e-2 and np.median(rel) < 5e-2 and rel.max() < 1e-1, rel
        for i in range(n_gen):
            srt = np.sort(want_logits[i])
            if srt[-1] - srt[-2] >= GAP:
                assert int(np.argmax(forced[i])) == want[i], (i, int(np.argmax(forced[i])), want[i])
        print(f"C5 shape (3 delta-net + 1 gated attention layers): first-token logits rel-L2 {rel0:.1e}; "
              f"free-running match {n_free}/{n_gen}; teacher-forced rel-L2 median {np.median(rel):.1e} "
              f"max {rel.max():.1e}")
        # the captured per-token graph (positions in device memory) gives the same tokens
        assert model.generate_graphed(prompt, n_gen) == got
    finally:
        model.close()
