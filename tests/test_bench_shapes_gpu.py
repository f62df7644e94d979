"""GPU parity at the shapes the benchmark times, against the CPU oracle.

* The tensor-core expert path on the isolated Qwen3-30B-A3B-shape layer (E 128, top-8 + renorm,
  I 768, down Q6_K) at T = 512 and T = 4096, the batched `mul_mat_id` form of hoard
  (src/run_specloop.cpp:125-140). Token rows are independent, so the oracle checks a seeded sample
  of 256 rows of each batch, with the tensor-core tolerances (batch rel-L2 <= 1e-2 against the
  ggml-mode oracle, every token <= 3e-2, <= 3e-2 against exact mode).
* The persistent decode kernel over the benchmark's 48-layer stack (E 128, top-8 + renorm, I 768,
  down Q6_K on even and Q4_K on odd layers) against oracle layers (hoard's per-layer decode form,
  src/run_moe_stream.cpp:352-447): every layer on its own GPU input (teacher forced, the strict
  per-layer tolerances, far inside the north star's 2e-2 per layer), the one-launch stack against
  the chain of single-layer launches, and the free-running oracle chain (reported). Expert ids
  must agree wherever the k-th/(k+1)-th log-probability gap exceeds 1e-3; at a smaller gap both
  selections are correct answers and the comparison continues with the GPU's. Along a free-running
  chain single Q8_K rounding flips of h (an f32 summation-order effect, ~2e-3 on the layer where
  one happens) make the two sides' inputs drift apart and the random model amplifies the drift
  (measured: 1e-2 to 2.5e-2 rel-L2 after 48 layers), which is why the teacher-forced check is the
  per-layer gate.
* C1 whole-model greedy decode (OLMoE shape: 16 layers, H 2048, MHA 16 x 128, 64 experts top-8,
  I 1024, vocab 50304) through the device driver against the oracle decoder: 64 tokens after a
  16-token prompt. As hoard's reference generator does (src/ref_gen.cpp:52-56), every position
  whose top-2 logit gap is below GAP is reported as a near tie; free-running tokens must match up to
  the first near tie, and teacher forced (on the oracle's tokens, and on a random continuation,
  since greedy decoding of a random model repeats one token) the choice must match at every
  position with a clear gap.
"""
import numpy as np
import pytest
import torch

from hoard_b200 import moe, quant
from oracle import oracle as orc
from tests.moe_fixtures import LayerSpec, load_context, make_layer, make_x, near_tie_mask, oracle_layer, rel_l2, Q4_K, Q6_K

pytestmark = pytest.mark.gpu

DEV = 0
H, E, K, I, NL = 2048, 128, 8, 768, 48
N_REPEAT = 1000


@pytest.fixture(scope="module")
def c2_layer():
    spec = LayerSpec(H=H, E=E, k=K, I=I)
    L = make_layer(spec, seed=4401, device=f"cuda:{DEV}")
    ctx = moe.MoEContext(n_embd=H, n_expert=E, n_expert_used=K, n_ff=I, n_layer=1, norm_topk=True, eps=spec.eps,
                         resid_dtype=torch.float32, gate_types=[Q4_K], up_types=[Q4_K], down_types=[Q6_K],
                         max_tokens=4096, device=DEV)
    ctx.set_gemm_min_tokens(64)
    load_context(ctx, 0, L)
    yield spec, L, ctx
    ctx.close()


@pytest.mark.parametrize("T", [512, 4096])
def test_tc_path_at_c2_shape(c2_layer, T):
    spec, L, ctx = c2_layer
    x = make_x(T, H, seed=9000 + T)
    xd = torch.from_numpy(x).cuda(DEV)
    sel = torch.empty(T, K, dtype=torch.int32, device=xd.device)
    w = torch.empty(T, K, device=xd.device)
    ctx.layer(0, xd, sel, w)
    ctx.sync_status()
    out, sel = xd.cpu().numpy(), sel.cpu().numpy()
    rows = np.sort(np.random.default_rng(T).choice(T, 256, replace=False))
    xs = x[rows]
    ref_out, ref_sel, _, _, ref_probs = oracle_layer(L, xs, orc.MODE_GGML)
    ok = ~near_tie_mask(ref_probs, ref_sel, K)
    assert ok.mean() > 0.8
    assert np.array_equal(np.sort(sel[rows][ok], 1), np.sort(ref_sel[ok], 1))
    d, r = out[rows][ok] - xs[ok], ref_out[ok] - xs[ok]
    per_tok = np.array([rel_l2(d[i], r[i]) for i in range(d.shape[0])])
    err = rel_l2(d, r)
    exact = oracle_layer(L, xs, orc.MODE_EXACT)[0]
    err_exact = rel_l2(d, exact[ok] - xs[ok])
    print(f"T={T}: rel-L2 of the MoE delta vs ggml mode {err:.2e} (max token {per_tok.max():.2e}), "
          f"vs exact mode {err_exact:.2e}, on {ok.sum()} sampled rows")
    assert err < 1e-2 and per_tok.max() < 3e-2 and err_exact < 3e-2


def _build_stack(dev):
    """The benchmark's 48 seeded layers: a context holding them plus their raw GGUF bytes (on the
    device, for the oracle's per-layer expert slices) and router weights (host)."""
    ctx = moe.MoEContext(n_embd=H, n_expert=E, n_expert_used=K, n_ff=I, n_layer=NL, norm_topk=True, eps=1e-6,
                         resid_dtype=torch.float32, gate_types=[Q4_K] * NL, up_types=[Q4_K] * NL,
                         down_types=[Q6_K if l % 2 == 0 else Q4_K for l in range(NL)], max_tokens=4, device=DEV)
    g = torch.Generator(device=dev)
    layers = []
    for l in range(NL):
        g.manual_seed(7700 + 31 * l)
        wr = torch.randn(E, H, generator=g, device=dev) * 0.02
        wn = 1.0 + 0.1 * torch.randn(H, generator=g, device=dev)
        dt = Q6_K if l % 2 == 0 else Q4_K
        gate = quant.quantize_q4k(torch.randn(E, I, H, generator=g, device=dev) * 0.02)
        up = quant.quantize_q4k(torch.randn(E, I, H, generator=g, device=dev) * 0.02)
        down = quant.quantize(torch.randn(E, H, I, generator=g, device=dev) * 0.02, dt)
        ctx.set_router(l, wr, wn)
        for e in range(E):
            ctx.upload_expert(l, e, gate[e], up[e], down[e])
        layers.append(dict(wr=wr.cpu().numpy(), wn=wn.float().cpu().numpy(), gate=gate, up=up, down=down, dt=dt))
    torch.cuda.synchronize(dev)
    return ctx, layers


def _oracle_step(Ld, x, force_sel=None, force_w=None):
    """One oracle layer on x [H]: routing, then the experts of the given (or its own) selection,
    computed from the selected experts' raw bytes only."""
    fx, probs, sel_o, w_o = orc.route(x[None], Ld["wn"], Ld["wr"], K, True, 1e-6)
    use_sel = sel_o[0] if force_sel is None else force_sel
    use_w = w_o[0] if force_w is None else force_w
    idx = torch.from_numpy(use_sel.astype(np.int64)).to(Ld["gate"].device)
    g8, u8, d8 = (Ld[m].index_select(0, idx).cpu().numpy() for m in ("gate", "up", "down"))
    out = orc.experts(H, K, K, I, (Q4_K, Q4_K, Ld["dt"]), g8, u8, d8, fx, x[None],
                      np.arange(K, dtype=np.int32)[None], use_w[None].astype(np.float32), orc.MODE_GGML)[0]
    return out, probs, sel_o[0], w_o[0]


def test_decode_stack_48_layers_vs_oracle():
    """(0) 1000 repeated one-launch runs are bit-identical (fixed-point router sums). (1) Teacher
    forced: each of the 48 layers, run by the persistent kernel on its own input,
    against the oracle layer on that same input (ids where the gap is clear, weights within 1e-5,
    the MoE delta of >= 90 % of layers within 1e-5 and of every layer within 5e-3). (2) The whole
    stack in one launch against the chain of 48 single-layer launches, within 2e-2 (reported). (3) The free-running oracle chain is reported against the
    one-launch result (bounded at 1e-1 against gross errors), with the layers where its drifted
    input selects other experts than the GPU did; there it continues with the GPU's choice."""
    dev = torch.device("cuda", DEV)
    ctx, layers = _build_stack(dev)
    try:
        x0 = make_x(2, H, seed=4242)
        layer_err, ties, chain, modes = [], 0, [], []
        for t in range(2):
            # one launch for the whole stack
            xd = torch.from_numpy(x0[t:t + 1].copy()).cuda(DEV)
            sel48 = torch.empty(NL, 1, K, dtype=torch.int32, device=dev)
            w48 = torch.empty(NL, 1, K, device=dev)
            n0 = ctx.launch_count
            ctx.layers(0, NL, xd, sel48, w48)
            ctx.sync_status()
            assert ctx.launch_count - n0 == 1
            x48, sel48, w48 = xd.cpu().numpy()[0], sel48.cpu().numpy()[:, 0], w48.cpu().numpy()[:, 0]
            # bit-reproducible: the router sums are integer (fixed-point) adds, so the order in which
            # the CTAs add them cannot change a bit of the routing or of the result (hoard's
            # invariant that repeated runs are bit-identical, notes/STATUS.md:96)
            x_ref, s_ref, w_ref = xd.clone(), torch.from_numpy(sel48).cuda(DEV), torch.from_numpy(w48).cuda(DEV)
            xr = torch.empty_like(xd)
            sr = torch.empty(NL, 1, K, dtype=torch.int32, device=dev)
            wr_ = torch.empty(NL, 1, K, device=dev)
            for _ in range(N_REPEAT if t == 0 else 10):
                xr.copy_(torch.from_numpy(x0[t:t + 1].copy()))
                ctx.layers(0, NL, xr, sr, wr_)
                assert torch.equal(xr, x_ref) and torch.equal(sr[:, 0], s_ref) and torch.equal(wr_[:, 0], w_ref)
            # one launch per layer, keeping every layer's input
            xl = torch.from_numpy(x0[t:t + 1].copy()).cuda(DEV)
            xs, sels, ws = [], [], []
            for l in range(NL):
                xs.append(xl.cpu().numpy()[0])
                s1 = torch.empty(1, K, dtype=torch.int32, device=dev)
                w1 = torch.empty(1, K, device=dev)
                ctx.layers(l, 1, xl, s1, w1)
                sels.append(s1.cpu().numpy()[0])
                ws.append(w1.cpu().numpy()[0])
            ctx.sync_status()
            x_chain = xl.cpu().numpy()[0]
            # the two launch modes scale the fixed-point router sums by different norms (the previous
            # layer's in one launch, the layer's own in a single-layer launch), so a routing weight
            # can differ in its last bit; through Q8_K rounding flips that grows over 48 layers
            modes.append((rel_l2(x48 - x0[t], x_chain - x0[t]), int((np.asarray(sels) != sel48).any(1).sum())))
            assert modes[-1][0] < 2e-2
            # (1) every layer against the oracle on the GPU's input of that layer
            for l, Ld in enumerate(layers):
                x_out = xs[l + 1] if l + 1 < NL else x_chain
                ref, probs, sel_o, w_o = _oracle_step(Ld, xs[l])
                if near_tie_mask(probs, sel_o[None], K)[0]:
                    ties += 1
                    ref = _oracle_step(Ld, xs[l], sels[l], ws[l])[0]
                else:
                    assert np.array_equal(np.sort(sels[l]), np.sort(sel_o)), (t, l)
                    assert np.allclose(np.sort(ws[l]), np.sort(w_o), rtol=1e-5, atol=1e-7), (t, l)
                layer_err.append(rel_l2(x_out - xs[l], ref - xs[l]))
            # (3) free-running oracle chain; where the drifted oracle input selects other experts
            #     than the GPU did, the chain records the layer and continues with the GPU's choice
            x = x0[t].copy()
            diverged = []
            for l, Ld in enumerate(layers):
                fx, probs, sel_o, w_o = orc.route(x[None], Ld["wn"], Ld["wr"], K, True, 1e-6)
                if not np.array_equal(np.sort(sel48[l]), np.sort(sel_o[0])):
                    diverged.append(l)
                    x = _oracle_step(Ld, x, sel48[l], w48[l])[0]
                else:
                    x = _oracle_step(Ld, x)[0]
            chain.append((rel_l2(x48 - x0[t], x - x0[t]), diverged))
        layer_err = np.asarray(layer_err)
        print(f"48-layer stack: per-layer rel-L2 vs oracle median {np.median(layer_err):.1e}, max "
              f"{layer_err.max():.1e} ({(layer_err < 1e-5).mean():.0%} within 1e-5, {ties} near-tie layers); "
              f"{N_REPEAT} repeated launches bit-identical; one launch vs single-layer launches: " +
              ", ".join(f"{e:.1e} ({n} layers routed differently)" for e, n in modes) + "; "
              f"free-running oracle chain vs one launch: " +
              ", ".join(f"{e:.1e} (other experts selected at layers {d})" for e, d in chain))
        assert (layer_err < 1e-5).mean() >= 0.9 and layer_err.max() < 5e-3
        # the north star's 2e-2 is a per-layer bound (checked above, teacher forced); over 48 chained
        # layers of a random model tiny differences grow, so the free-running figure is reported
        # and only bounded against gross errors
        assert max(e for e, _ in chain) < 1e-1
    finally:
        ctx.close()


C1_PROMPT_SEED = 1717
GAP = 0.05


def test_c1_greedy_decode_64_tokens_vs_oracle():
    from hoard_b200 import harness as hx
    from oracle.harness_oracle import OracleDecoder
    cfg = hx.C1_OLMOE
    dev = torch.device("cuda", DEV)
    tensors = hx.seeded_tensors(cfg, seed=31, device=dev)
    host = {k: (ty, ne, t.detach().cpu().numpy()) for k, (ty, ne, t) in tensors.items()}
    model = hx.DecodeModel(cfg, tensors, device=DEV, max_ctx=96)
    try:
        prompt = np.random.default_rng(C1_PROMPT_SEED).integers(0, cfg.n_vocab, 16).tolist()
        got = model.generate_graphed(prompt, 64)
        want, want_logits = OracleDecoder(cfg, host, max_ctx=96).generate(prompt, 64)
        srt = np.sort(want_logits, axis=1)
        gaps = srt[:, -1] - srt[:, -2]
        near = [i for i in range(64) if gaps[i] < GAP]
        n_free = 0
        for i in range(64):
            if got[i] != want[i]:
                break
            n_free += 1
        print(f"C1 greedy: {n_free}/64 tokens identical free-running; {len(set(want))} distinct tokens; "
              f"near ties (oracle top-2 gap < {GAP}) at {near}")
        assert n_free == 64 or (near and n_free >= near[0]), (n_free, near)
        forced = model.score(prompt + want, 16).cpu().numpy()
        for i in range(64):
            if gaps[i] >= GAP:
                assert int(np.argmax(forced[i])) == want[i], (i, int(np.argmax(forced[i])), want[i])
        rel = np.array([rel_l2(forced[i], want_logits[i]) for i in range(64)])
        assert np.median(rel) < 2e-2 and rel.max() < 5e-2, rel
        # Greedy decoding of a random model settles on a repeated token (its final state barely
        # depends on the input), so the positions above see few distinct inputs. Teacher forced on
        # a random 64-token continuation every position sees a different token: the choice must
        # match the oracle's wherever its top-2 gap is clear.
        cont = np.random.default_rng(C1_PROMPT_SEED + 1).integers(0, cfg.n_vocab, 64).tolist()
        seq = prompt + cont
        orc_dec = OracleDecoder(cfg, host, max_ctx=96)
        ref = np.stack([orc_dec.step(seq[p], p) for p in range(len(seq) - 1)])[15:]
        got_l = model.score(seq, 16).cpu().numpy()
        srt = np.sort(ref, axis=1)
        gaps_r = srt[:, -1] - srt[:, -2]
        clear = gaps_r >= GAP
        agree = np.argmax(got_l, 1) == np.argmax(ref, 1)
        rel_r = np.array([rel_l2(got_l[i], ref[i]) for i in range(64)])
        print(f"C1 teacher forced on a random continuation: {len(set(np.argmax(ref, 1).tolist()))} distinct "
              f"oracle choices, argmax agreement {agree.mean():.0%} ({clear.sum()} clear positions all "
              f"required), logits rel-L2 median {np.median(rel_r):.1e} max {rel_r.max():.1e}")
        assert agree[clear].all()
        assert np.median(rel_r) < 2e-2 and rel_r.max() < 5e-2
    finally:
        model.close()


def _shared_stack(spec, n_layer, max_tokens, seed):
    Ls = [make_layer(LayerSpec(H=spec.H, E=spec.E, k=spec.k, I=spec.I, shared=True,
                               types=(Q4_K, Q4_K, Q6_K if l % 2 == 0 else Q4_K)), seed=seed + l, device=f"cuda:{DEV}")
          for l in range(n_layer)]
    ctx = moe.MoEContext(n_embd=spec.H, n_expert=spec.E, n_expert_used=spec.k, n_ff=spec.I, n_layer=n_layer,
                         norm_topk=True, eps=spec.eps, resid_dtype=torch.float32, gate_types=[Q4_K] * n_layer,
                         up_types=[Q4_K] * n_layer, down_types=[L.spec.types[2] for L in Ls], n_ff_shexp=spec.I,
                         shexp_types=spec.sh_types, max_tokens=max_tokens, device=DEV)
    for l, L in enumerate(Ls):
        load_context(ctx, l, L)
    return Ls, ctx


@pytest.mark.parametrize("E,k,I", [(64, 8, 768), (512, 10, 512)])
def test_decode_with_shared_expert(E, k, I):
    """T = 1 with a gated shared expert (src/run_qwen35.cpp:659-676) through the persistent decode kernel
    (one launch for the stack) against the grouped kernels and a chain of oracle layers; (512, 10, 512)
    is the Qwen3-Next-80B-A3B MoE shape (E 512, top-10, I 512, shared expert I 512)."""
    spec = LayerSpec(H=H, E=E, k=k, I=I, shared=True)
    Ls, ctx = _shared_stack(spec, 2, 4, seed=6100 + E)
    try:
        x0 = make_x(1, H, seed=61)
        outs = {}
        for impl in (1, 0):
            ctx.set_decode_impl(impl)
            x = torch.from_numpy(x0.copy()).cuda(DEV)
            sel = torch.empty(2, 1, k, dtype=torch.int32, device=x.device)
            w = torch.empty(2, 1, k, device=x.device)
            n0 = ctx.launch_count
            ctx.layers(0, 2, x, sel, w)
            ctx.sync_status()
            if impl == 1:
                assert ctx.launch_count - n0 == 1                  # the persistent kernel ran the stack
            outs[impl] = (x.cpu().numpy(), sel.cpu().numpy(), w.cpu().numpy())
        assert np.array_equal(outs[0][1], outs[1][1])
        assert np.allclose(outs[0][2], outs[1][2], rtol=1e-5, atol=1e-7)
        assert rel_l2(outs[1][0] - x0, outs[0][0] - x0) < 1e-3
        ref = x0
        for l, L in enumerate(Ls):
            ref_l, ref_sel, _, _, probs = oracle_layer(L, ref, orc.MODE_GGML)
            if not near_tie_mask(probs, ref_sel, k)[0]:
                assert np.array_equal(np.sort(ref_sel, 1), np.sort(outs[1][1][l], 1))
            ref = ref_l
        err = rel_l2(outs[1][0] - x0, ref - x0)
        print(f"E={E} k={k} I={I} + shared expert, decode kernel vs oracle: rel-L2 {err:.1e}")
        assert err < 1e-3
    finally:
        ctx.close()


def test_tc_path_c5_shape():
    """Batched tokens at the Qwen3-Next MoE shape (E 512, top-10, I 512, shared expert) on the tensor-core
    path against the oracle, tensor-core tolerances."""
    spec = LayerSpec(H=H, E=512, k=10, I=512, shared=True)
    Ls, ctx = _shared_stack(spec, 1, 512, seed=6300)
    try:
        ctx.set_gemm_min_tokens(64)
        T = 512
        x = make_x(T, H, seed=63)
        xd = torch.from_numpy(x).cuda(DEV)
        ctx.layer(0, xd)
        ctx.sync_status()
        out = xd.cpu().numpy()
        rows = np.sort(np.random.default_rng(5).choice(T, 128, replace=False))
        xs = x[rows]
        ref_out, ref_sel, _, _, probs = oracle_layer(Ls[0], xs, orc.MODE_GGML)
        ok = ~near_tie_mask(probs, ref_sel, 10)
        d, r = out[rows][ok] - xs[ok], ref_out[ok] - xs[ok]
        err = rel_l2(d, r)
        per_tok = max(rel_l2(d[i], r[i]) for i in range(d.shape[0]))
        print(f"C5 shape, T={T}, tensor-core path: rel-L2 vs ggml mode {err:.1e} (max token {per_tok:.1e})")
        assert err < 1e-2 and per_tok < 3e-2
    finally:
        ctx.close()
