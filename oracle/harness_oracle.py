"""CPU restatement of hoard's per-token decode schedule -- TEST INFRASTRUCTURE ONLY (the checker of
hoard_b200.harness; never imported by the library).

Follows src/run_moe_stream.cpp:295-472 step by step:
  graph E   embedding row (ggml_get_rows of a Q4_K / Q6_K table: dequantised)          :302-312
  graph A   RMSNorm(x) * attn_norm                                                   :322
            q, k, v = ggml_mul_mat(W, cur): Q8_K activation, integer block dots      :323-325
            QK RMSNorm over the whole projection (OLMoE) or per head (Qwen3)         :326-331
            NEOX RoPE, theta_i = p * base^(-2i/head_dim) by repeated multiplication :332-333
            KV cache store, single-query attention, scale 1/sqrt(head_dim),
            softmax with the max subtracted and a double sum                         :334-347
            ffn_inp = Wo att + x                                                     :348-349
  MoE       x = ffn_inp + sum_j w_j FFN_j(RMSNorm(ffn_inp) * ffn_norm) (oracle.moe_layer)
  head      RMSNorm(x) * output_norm, lm-head, argmax (first maximum)                :452-472
Two choices follow the configuration rather than the reference (which keeps an f32 cache): the
KV cache holds f16 (config C1 asks for an fp16 KV cache) or bf16 (config C3), and every position,
the current one included, is read back from it.

Hybrid models (Qwen3-Next, src/run_qwen35.cpp:472-553) add two layer kinds:
  gated full attention  q projection rows [q | gate] per head, per-head QK RMSNorm, NEOX RoPE on
                        the first rope_dim values of a head, att * sigmoid(gate)           :472-507
  gated delta-net       qkv / z / ba projections; causal conv1d (kernel d_conv) over the last
                        inputs, silu; q, k L2-normalised, key heads repeated to the value
                        heads; beta = sigmoid(b), decay = exp(softplus(a + dt_bias) * ssm_a);
                        the delta rule S <- decay S; S <- S + k (beta (v - S^T k))^T; o = S^T q
                        (q scaled by 1/sqrt(d), the published recurrent form of gated delta-net);
                        RMSNorm(o) * ssm_norm * silu(z); ssm_out                            :508-553
ggml's fused gated_delta_net / ssm_conv kernels are not vendored in the reference, so this
restatement of their published algorithm is not pinned against ggml output.
"""
from __future__ import annotations

import ctypes

import numpy as np

from oracle import oracle as orc


def rms_norm(x: np.ndarray, w: np.ndarray, rows: int, cols: int, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(rows, cols)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    wb = np.broadcast_to(w, (cols,)).copy() if w.size == cols else w
    orc.lib().orc_rms_norm(orc._p(x), orc._p(wb), ctypes.c_int(rows), ctypes.c_int(cols), ctypes.c_float(eps),
                           orc._p(out))
    return out.reshape(-1)


def rope_neox(x: np.ndarray, n_heads: int, hd: int, pos: int, freq_base: float, n_rot: int = 0) -> np.ndarray:
    """NEOX RoPE of the first n_rot (default: all hd) values of each head; the rest pass through."""
    n_rot = n_rot or hd
    x = x.reshape(n_heads, hd).astype(np.float32).copy()
    theta_scale = np.float32(np.float32(freq_base) ** np.float32(-2.0 / n_rot))
    half = n_rot // 2
    theta = np.empty(half, np.float32)
    t = np.float32(pos)
    for i in range(half):
        theta[i] = t
        t = np.float32(t * theta_scale)
    c, s = np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)
    x0, x1 = x[:, :half].copy(), x[:, half:n_rot].copy()
    x[:, :half] = x0 * c - x1 * s
    x[:, half:n_rot] = x0 * s + x1 * c
    return x.reshape(-1)


def silu(x):
    x = np.asarray(x, np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def sigmoid(x):
    x = np.asarray(x, np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gdn_step(qkv, z, ba, conv_w, hist, dt_bias, ssm_a, norm_w, S, Hv: int, Hk: int, D: int, d_conv: int, eps: float):
    """One token through a gated delta-net block (see the module docstring). hist: the previous inputs
    (newest last, at most d_conv - 1 used); S [Hv][D key][D value] f32 is updated in place.
    Returns out [Hv*D] (before the output projection)."""
    cd = qkv.size
    W = np.asarray(conv_w, np.float32).reshape(cd, d_conv)
    acc = (qkv * W[:, d_conv - 1]).astype(np.float32)
    prev = hist[-(d_conv - 1):] if d_conv > 1 else []
    for u in range(d_conv - 1):                    # tap u: position pos - (d_conv - 1) + u
        j = u - (d_conv - 1 - len(prev))
        if j >= 0:
            acc = (acc + prev[j] * W[:, u]).astype(np.float32)
    x = silu(acc)
    vpg = Hv // Hk
    out = np.empty(Hv * D, np.float32)
    for h in range(Hv):
        g, r = h // vpg, h % vpg
        q = x[g * D:(g + 1) * D]
        k = x[Hk * D + g * D:Hk * D + (g + 1) * D]
        v = x[2 * Hk * D + h * D:2 * Hk * D + (h + 1) * D]
        qs = np.float32(1.0 / max(np.sqrt(np.float32((q.astype(np.float64) ** 2).sum())), eps)) * np.float32(1.0 / np.sqrt(D))
        ks = np.float32(1.0 / max(np.sqrt(np.float32((k.astype(np.float64) ** 2).sum())), eps))
        beta = sigmoid(ba[g * 2 * vpg + r])
        a = np.float32(ba[g * 2 * vpg + vpg + r] + dt_bias[h])
        sp = a if a > 20 else np.float32(np.log1p(np.exp(a)))
        decay = np.float32(np.exp(np.float32(sp * ssm_a[h])))
        kn, qn = (k * ks).astype(np.float32), (q * qs).astype(np.float32)
        Sh = (S[h] * decay).astype(np.float32)
        kv = (Sh * kn[:, None]).sum(0, dtype=np.float32)
        delta = (beta * (v - kv)).astype(np.float32)
        Sh = (Sh + kn[:, None] * delta[None, :]).astype(np.float32)
        S[h] = Sh
        o = (Sh * qn[:, None]).sum(0, dtype=np.float32)
        rs = np.float32(1.0 / np.sqrt(np.float32((o.astype(np.float64) ** 2).sum() / D) + np.float32(eps)))
        out[h * D:(h + 1) * D] = ((o * rs) * norm_w) * silu(z[h * D:(h + 1) * D])
    return out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 values rounded to the nearest bf16 (ties to even), returned as f32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


class OracleDecoder:
    def __init__(self, cfg, tensors: dict, max_ctx: int, kv: str = "f16"):
        """tensors: name -> (ggml type, ne, numpy raw bytes / f32 values), as the harness takes them;
        kv: "f16" or "bf16" elements of the KV cache."""
        self.cfg = cfg
        self.t = {k: (ty, ne, np.asarray(v)) for k, (ty, ne, v) in tensors.items()}
        hd = cfg.head_dim
        self.nq, self.nkv = cfg.n_head * hd, cfg.n_head_kv * hd
        if kv not in ("f16", "bf16"):
            raise ValueError("kv must be f16 or bf16")
        self.kv = kv
        self.kc = np.zeros((cfg.n_layer, max_ctx, self.nkv), np.float16 if kv == "f16" else np.float32)
        self.vc = np.zeros_like(self.kc)
        hybrid = getattr(cfg, "full_attn_interval", 0) > 0
        self.hist = {il: [] for il in range(cfg.n_layer)} if hybrid else {}
        self.S = {il: np.zeros((cfg.ssm_dt_rank, cfg.ssm_d_state, cfg.ssm_d_state), np.float32)
                  for il in range(cfg.n_layer) if hybrid and cfg.is_recurrent(il)}

    def _mv(self, name, n_out, k_in, x):
        ty, _, w = self.t[name]
        return orc.matvec(ty, w.reshape(-1), n_out, k_in, x, orc.MODE_GGML)

    def _f(self, name):
        return self.t[name][2].reshape(-1).view(np.float32) if self.t[name][2].dtype == np.uint8 else \
            self.t[name][2].astype(np.float32).reshape(-1)

    def step(self, token: int, pos: int) -> np.ndarray:
        c = self.cfg
        H, hd = c.n_embd, c.head_dim
        ty, _, table = self.t["token_embd.weight"]
        rb = table.reshape(-1).size // c.n_vocab
        x = orc.dequant(ty, table.reshape(-1)[token * rb:(token + 1) * rb]) if ty in (12, 14) else \
            table.reshape(c.n_vocab, H)[token].astype(np.float32)
        hybrid = getattr(c, "full_attn_interval", 0) > 0
        for il in range(c.n_layer):
            b = f"blk.{il}."
            cur = rms_norm(x, self._f(b + "attn_norm.weight"), 1, H, c.eps)
            if hybrid and c.is_recurrent(il):
                D, Hk, Hv = c.ssm_d_state, c.ssm_n_group, c.ssm_dt_rank
                qkv = self._mv(b + "attn_qkv.weight", c.conv_dim, H, cur)
                zz = self._mv(b + "attn_gate.weight", Hv * D, H, cur)
                bav = self._mv(b + "ssm_ba.weight", 2 * Hv, H, cur)
                o = gdn_step(qkv, zz, bav, self._f(b + "ssm_conv1d.weight"), self.hist[il], self._f(b + "ssm_dt.bias"),
                             self._f(b + "ssm_a"), self._f(b + "ssm_norm.weight"), self.S[il], Hv, Hk, D, c.ssm_d_conv,
                             c.eps)
                self.hist[il].append(qkv.astype(np.float32))
                ffn_inp = (self._mv(b + "ssm_out.weight", H, Hv * D, o) + x).astype(np.float32)
            else:
                gated = getattr(c, "attn_gate", False)
                qg = self._mv(b + "attn_q.weight", 2 * self.nq if gated else self.nq, H, cur)
                if gated:
                    qg2 = qg.reshape(c.n_head, 2, hd)
                    q, gate = qg2[:, 0, :].reshape(-1).copy(), qg2[:, 1, :].reshape(-1).copy()
                else:
                    q, gate = qg, None
                k = self._mv(b + "attn_k.weight", self.nkv, H, cur)
                v = self._mv(b + "attn_v.weight", self.nkv, H, cur)
                if c.qk_norm == "full":
                    q = rms_norm(q, self._f(b + "attn_q_norm.weight"), 1, self.nq, c.eps)
                    k = rms_norm(k, self._f(b + "attn_k_norm.weight"), 1, self.nkv, c.eps)
                elif c.qk_norm == "head":
                    q = rms_norm(q, self._f(b + "attn_q_norm.weight"), c.n_head, hd, c.eps)
                    k = rms_norm(k, self._f(b + "attn_k_norm.weight"), c.n_head_kv, hd, c.eps)
                n_rot = getattr(c, "rope_dim", 0) or hd
                q = rope_neox(q, c.n_head, hd, pos, c.freq_base, n_rot)
                k = rope_neox(k, c.n_head_kv, hd, pos, c.freq_base, n_rot)
                if self.kv == "f16":
                    self.kc[il, pos] = k.astype(np.float16)
                    self.vc[il, pos] = v.astype(np.float16)
                else:
                    self.kc[il, pos] = bf16_round(k)
                    self.vc[il, pos] = bf16_round(v)
                K = self.kc[il, :pos + 1].astype(np.float32).reshape(pos + 1, c.n_head_kv, hd)
                V = self.vc[il, :pos + 1].astype(np.float32).reshape(pos + 1, c.n_head_kv, hd)
                att = np.empty((c.n_head, hd), np.float32)
                qh = q.reshape(c.n_head, hd)
                scale = np.float32(1.0 / np.sqrt(hd))
                grp = c.n_head // c.n_head_kv
                for h in range(c.n_head):
                    s = (K[:, h // grp, :] @ qh[h]).astype(np.float32) * scale
                    e = np.exp(s - s.max()).astype(np.float32)
                    inv = np.float32(1.0 / e.astype(np.float64).sum())
                    att[h] = ((e * inv)[:, None] * V[:, h // grp, :]).sum(0, dtype=np.float32)
                    if gate is not None:
                        att[h] = att[h] * sigmoid(gate[h * hd:(h + 1) * hd])
                ffn_inp = (self._mv(b + "attn_output.weight", H, self.nq, att.reshape(-1)) + x).astype(np.float32)
            gty = self.t[b + "ffn_gate_exps.weight"][0]
            uty = self.t[b + "ffn_up_exps.weight"][0]
            dty = self.t[b + "ffn_down_exps.weight"][0]
            shared = None
            if getattr(c, "n_ff_shexp", 0):
                shared = {"I": c.n_ff_shexp, "gate_type": self.t[b + "ffn_gate_shexp.weight"][0],
                          "up_type": self.t[b + "ffn_up_shexp.weight"][0],
                          "down_type": self.t[b + "ffn_down_shexp.weight"][0],
                          "gate": self.t[b + "ffn_gate_shexp.weight"][2].reshape(-1),
                          "up": self.t[b + "ffn_up_shexp.weight"][2].reshape(-1),
                          "down": self.t[b + "ffn_down_shexp.weight"][2].reshape(-1),
                          "gate_inp": self._f(b + "ffn_gate_inp_shexp.weight")}
            norm_name = c.ffn_norm_name() if hasattr(c, "ffn_norm_name") else "ffn_norm.weight"
            out, _, _, _, _ = orc.moe_layer(ffn_inp.reshape(1, H), self._f(b + norm_name),
                                            self._f(b + "ffn_gate_inp.weight").reshape(c.n_expert, H),
                                            self.t[b + "ffn_gate_exps.weight"][2].reshape(c.n_expert, -1),
                                            self.t[b + "ffn_up_exps.weight"][2].reshape(c.n_expert, -1),
                                            self.t[b + "ffn_down_exps.weight"][2].reshape(c.n_expert, -1),
                                            H=H, E=c.n_expert, k=c.n_expert_used, I=c.n_ff, types=(gty, uty, dty),
                                            renorm=c.norm_topk, eps=c.eps, shared=shared)
            x = out.reshape(-1)
        r = rms_norm(x, self._f("output_norm.weight"), 1, H, c.eps)
        return self._mv("output.weight", c.n_vocab, H, r)

    def generate(self, prompt, n_gen: int):
        """Greedy ids and the logits each was chosen from."""
        toks, logits = [], []
        seq = list(prompt)
        for p in range(len(prompt) + n_gen - 1):
            lg = self.step(seq[p], p)
            if p >= len(prompt) - 1:
                nxt = int(np.argmax(lg))
                toks.append(nxt)
                logits.append(lg)
                seq.append(nxt)
        return toks, np.stack(logits)
