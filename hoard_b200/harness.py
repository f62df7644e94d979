"""A minimal decode driver around the MoE path: hoard's per-token schedule (src/run_moe_stream.cpp:
295-472) with every step on the device.

    graph E   x = token_embd[token]                                            (hoard_hx_embed)
    per layer (graph A, attention part; then the MoE layer):
              cur = RMSNorm(x) * attn_norm
              q, k, v = Wq cur, Wk cur, Wv cur          (Q4_K / Q6_K . Q8_K(cur), hoard_hx_gemv)
              QK RMSNorm: over the whole projection (OLMoE) or per head (Qwen3)
              NEOX RoPE of q, k at position p; k, v into the f16/bf16 KV cache (hoard_hx_rope_store)
              att = softmax(q k^T / sqrt(head_dim)) v over positions 0..p     (hoard_hx_attention)
              ffn_inp = Wo att + x
              x = ffn_inp + sum_j w_j FFN_j(RMSNorm(ffn_inp) * ffn_norm)       (hoard_moe_layers)
    head      logits = W_out (RMSNorm(x) * output_norm); next = argmax         (hoard_hx_argmax)

Prompt tokens run through the same step one at a time, as in hoard; generation starts from the
logits of the last prompt token. Models come from a GGUF file (`DecodeModel.from_gguf`) or from
seeded tensors generated on the device (`seeded_tensors`, the benchmark configurations' weights:
N(0, 0.02), Q4_K_M types). The MoE layers use all experts HBM-resident (T = 1: the persistent
decode kernel)."""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch

from hoard_b200 import moe, quant
from hoard_b200.moe import HoardError, _ptr, _stream, lib

Q4_K, Q6_K, F32 = quant.Q4_K, quant.Q6_K, 0
KV_TYPES = {torch.float16: 1, torch.bfloat16: 30}     # KV cache element -> HOARD_TYPE_F16 / HOARD_TYPE_BF16
MAX_BATCH = 16          # tokens of one batched (verify) forward
QK_MODE = {"": 0, "full": 1, "head": 2}


def _iarr(vals):
    return (ctypes.c_int * len(vals))(*vals)


def _parr(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)

_bound = False


def _hx():
    global _bound
    L = lib()
    if not _bound:
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        L.hoard_hx_repack.argtypes = [i32, vp, vp, i64, vp]
        L.hoard_hx_embed.argtypes = [i32, vp, i32, i64, vp, vp, vp]
        L.hoard_hx_rmsnorm.argtypes = [vp, i32, i32, f32, vp, vp, vp]
        L.hoard_hx_q8_bytes.argtypes = [i32]
        L.hoard_hx_q8_bytes.restype = i64
        L.hoard_hx_quant_q8.argtypes = [vp, i32, vp, vp]
        L.hoard_hx_gemv.argtypes = [i32, vp, i32, i32, vp, vp, vp, vp]
        L.hoard_hx_rope_store.argtypes = [vp, vp, vp, i32, i32, i32, i32, f32, vp, vp, i32, vp]
        L.hoard_hx_attention.argtypes = [vp, vp, vp, i32, i32, i32, i32, f32, vp, i32, vp]
        L.hoard_hx_argmax.argtypes = [vp, i32, vp, vp]
        L.hoard_hx_embed_at.argtypes = [i32, vp, i32, i64, vp, vp, vp, vp]
        L.hoard_hx_rope_store_at.argtypes = [vp, vp, vp, i32, i32, i32, vp, i32, f32, vp, vp, i32, vp]
        L.hoard_hx_attention_at.argtypes = [vp, vp, vp, i32, i32, i32, vp, i32, f32, vp, i32, vp]
        L.hoard_hx_argmax_at.argtypes = [vp, i32, vp, vp, i32, vp]
        L.hoard_hx_rmsnorm_q8.argtypes = [vp, i32, f32, vp, vp, vp]
        L.hoard_hx_gemv_multi.argtypes = [i32, vp, vp, vp, i32, vp, vp, vp, vp]
        L.hoard_hx_qknorm_rope_store.argtypes = [vp, vp, vp, vp, vp, i32, f32, i32, i32, i32, i32, f32, vp, vp, vp, i32,
                                                 vp]
        L.hoard_hx_qknorm_rope_store_at.argtypes = [vp, vp, vp, vp, vp, i32, f32, i32, i32, i32, vp, i32, f32, vp, vp,
                                                   vp, i32, vp]
        L.hoard_hx_qknorm_rope_store_ex.argtypes = [vp, vp, vp, vp, vp, i32, f32, i32, i32, i32, i32, i32, i32, vp, i32,
                                                   f32, vp, vp, vp, i32, vp]
        L.hoard_hx_attention_ex.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp, f32, vp, i32, vp, i32, vp]
        L.hoard_hx_gdn_step.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, i32, vp, vp, vp]
        _bound = True
    return L


def _ok(rc: int, what: str):
    if rc != 0:
        raise HoardError(rc, f"{what} failed ({lib().hoard_strerror(rc).decode()})")


@dataclass
class ModelConfig:
    """Hyper-parameters and GGUF tensor types of a seeded model (Q4_K_M: attn q/k/o and the
    embedding Q4_K, attn v and the lm-head Q6_K, expert gate/up Q4_K, expert down Q6_K on even and
    Q4_K on odd layers)."""
    arch: str
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_expert: int
    n_expert_used: int
    n_ff: int
    n_vocab: int
    freq_base: float
    eps: float
    qk_norm: str            # "full" (OLMoE: over the whole projection), "head" (Qwen3) or ""
    norm_topk: bool
    # hybrid models (Qwen3-Next, src/run_qwen35.cpp:472-553): every full_attn_interval-th layer is gated
    # full attention (fused q + sigmoid output gate, NEOX RoPE on the first rope_dim values of a head),
    # the others gated delta-net; a gated shared expert of n_ff_shexp
    n_ff_shexp: int = 0
    full_attn_interval: int = 0     # 0: every layer is full attention
    attn_gate: bool = False
    rope_dim: int = 0               # 0: head_dim
    ssm_d_state: int = 0            # delta-net head dim (key = value)
    ssm_n_group: int = 0            # key heads
    ssm_dt_rank: int = 0            # value heads
    ssm_d_conv: int = 0             # causal conv taps

    def down_type(self, il: int) -> int:
        return Q6_K if il % 2 == 0 else Q4_K

    def is_recurrent(self, il: int) -> bool:
        return self.full_attn_interval > 0 and (il + 1) % self.full_attn_interval != 0

    def ffn_norm_name(self) -> str:
        return "post_attention_norm.weight" if self.full_attn_interval > 0 else "ffn_norm.weight"

    @property
    def n_rot(self) -> int:
        return self.rope_dim or self.head_dim

    @property
    def conv_dim(self) -> int:
        return (2 * self.ssm_n_group + self.ssm_dt_rank) * self.ssm_d_state


C1_OLMOE = ModelConfig("olmoe", 16, 2048, 16, 16, 128, 64, 8, 1024, 50304, 1e4, 1e-5, "full", False)
C3_QWEN3 = ModelConfig("qwen3moe", 48, 2048, 32, 4, 128, 128, 8, 768, 151936, 1e6, 1e-6, "head", True)
C5_QWEN3NEXT = ModelConfig("qwen3next", 48, 2048, 16, 2, 256, 512, 10, 512, 151936, 1e7, 1e-6, "head", True,
                           n_ff_shexp=512, full_attn_interval=4, attn_gate=True, rope_dim=64, ssm_d_state=128,
                           ssm_n_group=16, ssm_dt_rank=32, ssm_d_conv=4)


def seeded_tensors(cfg: ModelConfig, seed: int, device) -> dict:
    """Every tensor of a seeded model, named as in hoard's GGUFs, on `device`:
    name -> (ggml type, ne (GGUF order), tensor: uint8 raw blocks or f32)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, hd, E, I = cfg.n_embd, cfg.head_dim, cfg.n_expert, cfg.n_ff
    nq, nkv = cfg.n_head * hd, cfg.n_head_kv * hd

    def w(n_out, k_in, qt):
        return quant.quantize(torch.randn(n_out, k_in, generator=g, device=device) * 0.02, qt)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).float()

    t = {"token_embd.weight": (Q4_K, (H, cfg.n_vocab), w(cfg.n_vocab, H, Q4_K)),
         "output_norm.weight": (F32, (H,), norm(H)),
         "output.weight": (Q6_K, (H, cfg.n_vocab), w(cfg.n_vocab, H, Q6_K))}
    for il in range(cfg.n_layer):
        b = f"blk.{il}."
        t[b + "attn_norm.weight"] = (F32, (H,), norm(H))
        if cfg.is_recurrent(il):
            D, Hk, Hv = cfg.ssm_d_state, cfg.ssm_n_group, cfg.ssm_dt_rank
            cd, vd = cfg.conv_dim, Hv * D
            t[b + "attn_qkv.weight"] = (Q4_K, (H, cd), w(cd, H, Q4_K))
            t[b + "attn_gate.weight"] = (Q4_K, (H, vd), w(vd, H, Q4_K))
            t[b + "ssm_ba.weight"] = (Q4_K, (H, 2 * Hv), w(2 * Hv, H, Q4_K))
            t[b + "ssm_conv1d.weight"] = (F32, (cfg.ssm_d_conv, cd),
                                          (torch.randn(cd, cfg.ssm_d_conv, generator=g, device=device) * 0.3).float())
            t[b + "ssm_dt.bias"] = (F32, (Hv,), (torch.randn(Hv, generator=g, device=device) * 0.5).float())
            # ssm_a = -exp(A_log), A_log ~ U(0, log 16)
            t[b + "ssm_a"] = (F32, (Hv,), (-torch.exp(torch.rand(Hv, generator=g, device=device) * math.log(16.0))).float())
            t[b + "ssm_norm.weight"] = (F32, (D,), norm(D))
            t[b + "ssm_out.weight"] = (Q4_K, (vd, H), w(H, vd, Q4_K))
        else:
            nqp = 2 * nq if cfg.attn_gate else nq
            t[b + "attn_q.weight"] = (Q4_K, (H, nqp), w(nqp, H, Q4_K))
            t[b + "attn_k.weight"] = (Q4_K, (H, nkv), w(nkv, H, Q4_K))
            t[b + "attn_v.weight"] = (Q6_K, (H, nkv), w(nkv, H, Q6_K))
            t[b + "attn_output.weight"] = (Q4_K, (nq, H), w(H, nq, Q4_K))
            if cfg.qk_norm == "full":
                t[b + "attn_q_norm.weight"] = (F32, (nq,), norm(nq))
                t[b + "attn_k_norm.weight"] = (F32, (nkv,), norm(nkv))
            elif cfg.qk_norm == "head":
                t[b + "attn_q_norm.weight"] = (F32, (hd,), norm(hd))
                t[b + "attn_k_norm.weight"] = (F32, (hd,), norm(hd))
        t[b + cfg.ffn_norm_name()] = (F32, (H,), norm(H))
        t[b + "ffn_gate_inp.weight"] = (F32, (H, E), (torch.randn(E, H, generator=g, device=device) * 0.02).float())
        dt = cfg.down_type(il)
        t[b + "ffn_gate_exps.weight"] = (Q4_K, (H, I, E), quant.synth_experts(E, I, H, Q4_K, seed * 1000 + 3 * il, device))
        t[b + "ffn_up_exps.weight"] = (Q4_K, (H, I, E), quant.synth_experts(E, I, H, Q4_K, seed * 1000 + 3 * il + 1, device))
        t[b + "ffn_down_exps.weight"] = (dt, (I, H, E), quant.synth_experts(E, H, I, dt, seed * 1000 + 3 * il + 2, device))
        if cfg.n_ff_shexp:
            Is = cfg.n_ff_shexp
            t[b + "ffn_gate_shexp.weight"] = (Q4_K, (H, Is), w(Is, H, Q4_K))
            t[b + "ffn_up_shexp.weight"] = (Q4_K, (H, Is), w(Is, H, Q4_K))
            t[b + "ffn_down_shexp.weight"] = (Q6_K, (Is, H), w(H, Is, Q6_K))
            t[b + "ffn_gate_inp_shexp.weight"] = (F32, (H,), (torch.randn(H, generator=g, device=device) * 0.02).float())
    return t


def write_gguf(path: str, cfg: ModelConfig, tensors: dict):
    from hoard_b200 import gguf_io as gi
    w = gi.GGUFWriter(cfg.arch)
    a = cfg.arch
    w.add(f"{a}.block_count", cfg.n_layer)
    w.add(f"{a}.embedding_length", cfg.n_embd)
    w.add(f"{a}.attention.head_count", cfg.n_head)
    w.add(f"{a}.attention.head_count_kv", cfg.n_head_kv)
    w.add(f"{a}.attention.key_length", cfg.head_dim)
    w.add(f"{a}.expert_feed_forward_length", cfg.n_ff)
    w.add(f"{a}.expert_count", cfg.n_expert)
    w.add(f"{a}.expert_used_count", cfg.n_expert_used)
    w.add(f"{a}.rope.freq_base", float(cfg.freq_base))
    w.add(f"{a}.attention.layer_norm_rms_epsilon", float(cfg.eps))
    for name, (ty, ne, data) in tensors.items():
        w.add_tensor(name, ne, ty, data.detach().cpu().numpy())
    w.write(path)


def config_from_hparams(hp) -> ModelConfig:
    return ModelConfig(hp.arch, hp.n_layer, hp.n_embd, hp.n_head, hp.n_head_kv, hp.head_dim, hp.n_expert,
                       hp.n_expert_used, hp.n_ff, hp.n_vocab, hp.freq_base, hp.eps,
                       "" if not hp.has_qk_norm else ("head" if hp.qk_perhead else "full"), hp.norm_topk)


class DecodeModel:
    def __init__(self, cfg: ModelConfig, tensors: dict, device: int = 0, max_ctx: int = 512, eos_id: int = -1,
                 kv_dtype=torch.float16):
        """tensors: name -> (ggml type, ne, array or tensor of raw bytes / f32 values), host or device.
        kv_dtype: torch.float16 or torch.bfloat16 elements of the KV cache."""
        if kv_dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("kv_dtype must be torch.float16 or torch.bfloat16")
        self.cfg, self.device, self.max_ctx, self.eos_id = cfg, device, max_ctx, eos_id
        self.kv_type = KV_TYPES[kv_dtype]
        dev = self.dev = torch.device("cuda", device)
        _hx()
        H, hd = cfg.n_embd, cfg.head_dim
        self.nq, self.nkv = cfg.n_head * hd, cfg.n_head_kv * hd

        def raw(name):
            ty, ne, data = tensors[name]
            t = torch.as_tensor(np.asarray(data)) if not isinstance(data, torch.Tensor) else data
            return ty, t.contiguous().to(dev)

        def plane(name):
            ty, t = raw(name)
            out = torch.empty_like(t, dtype=torch.uint8)
            nblk = t.numel() // quant.row_bytes(ty, 256)
            _ok(_hx().hoard_hx_repack(ty, _ptr(t), _ptr(out), nblk, _stream(None)), "repack")
            return ty, out

        def f32(name):
            ty, t = raw(name)
            assert ty == F32
            return t.view(torch.float32) if t.dtype == torch.uint8 else t.float()

        self.embd_type, self.embd = raw("token_embd.weight")
        self.out_norm = f32("output_norm.weight")
        self.out_type, self.out_w = plane("output.weight")
        self.nqp = 2 * self.nq if cfg.attn_gate else self.nq      # q projection rows (+ the output gate)
        hybrid = cfg.full_attn_interval > 0
        self.gdn_vd = cfg.ssm_dt_rank * cfg.ssm_d_state
        self.layers = []
        for il in range(cfg.n_layer):
            b = f"blk.{il}."
            L = {"attn_norm": f32(b + "attn_norm.weight"), "recurrent": cfg.is_recurrent(il)}
            if L["recurrent"]:
                L.update({"qkv": plane(b + "attn_qkv.weight"), "z": plane(b + "attn_gate.weight"),
                          "ba": plane(b + "ssm_ba.weight"), "conv_w": f32(b + "ssm_conv1d.weight"),
                          "dt_bias": f32(b + "ssm_dt.bias"), "ssm_a": f32(b + "ssm_a"),
                          "ssm_norm": f32(b + "ssm_norm.weight"), "o": plane(b + "ssm_out.weight")})
                L["qkv_types"] = _iarr([L[m][0] for m in ("qkv", "z", "ba")])
                L["qkv_w"] = _parr([L[m][1].data_ptr() for m in ("qkv", "z", "ba")])
            else:
                L.update({"q": plane(b + "attn_q.weight"), "k": plane(b + "attn_k.weight"),
                          "v": plane(b + "attn_v.weight"), "o": plane(b + "attn_output.weight")})
                if cfg.qk_norm:
                    L["q_norm"], L["k_norm"] = f32(b + "attn_q_norm.weight"), f32(b + "attn_k_norm.weight")
                L["qkv_types"] = _iarr([L[m][0] for m in ("q", "k", "v")])
                L["qkv_w"] = _parr([L[m][1].data_ptr() for m in ("q", "k", "v")])
            self.layers.append(L)
        # the MoE layers: all experts resident, T = 1
        types = [tuple(tensors[f"blk.{il}.ffn_{m}_exps.weight"][0] for m in ("gate", "up", "down"))
                 for il in range(cfg.n_layer)]
        sh_types = (Q4_K, Q4_K, Q6_K)
        if cfg.n_ff_shexp:
            sh_types = tuple(tensors[f"blk.0.ffn_{m}_shexp.weight"][0] for m in ("gate", "up", "down"))
        self.moe = moe.MoEContext(n_embd=H, n_expert=cfg.n_expert, n_expert_used=cfg.n_expert_used, n_ff=cfg.n_ff,
                                  n_layer=cfg.n_layer, norm_topk=cfg.norm_topk, eps=cfg.eps,
                                  gate_types=[t[0] for t in types], up_types=[t[1] for t in types],
                                  down_types=[t[2] for t in types], n_ff_shexp=cfg.n_ff_shexp, shexp_types=sh_types,
                                  max_tokens=MAX_BATCH, device=device)
        for il in range(cfg.n_layer):
            b = f"blk.{il}."
            self.moe.set_router(il, f32(b + "ffn_gate_inp.weight").view(cfg.n_expert, H), f32(b + cfg.ffn_norm_name()))
            mats = [raw(b + f"ffn_{m}_exps.weight")[1].view(cfg.n_expert, -1) for m in ("gate", "up", "down")]
            for e in range(cfg.n_expert):
                self.moe.upload_expert(il, e, mats[0][e], mats[1][e], mats[2][e])
            if cfg.n_ff_shexp:
                self.moe.set_shared(il, *(raw(b + f"ffn_{m}_shexp.weight")[1] for m in ("gate", "up", "down")),
                                    f32(b + "ffn_gate_inp_shexp.weight"))
        # activations, Q8_K workspaces, KV caches, delta-net states, token sequence
        z = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)
        self.x, self.x2, self.cur = z(H), z(H), z(H)
        self.q, self.k, self.v, self.att = z(self.nqp), z(self.nkv), z(self.nkv), z(self.nq)
        self.logits = z(cfg.n_vocab)
        self.q_rot = z(self.nq)
        self.qkv_N = _iarr([self.nqp, self.nkv, self.nkv])
        self.qkv_y = _parr([self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr()])
        kq = max(H, self.nq, self.gdn_vd)
        self.q8 = torch.zeros(int(_hx().hoard_hx_q8_bytes(kq)), dtype=torch.uint8, device=dev)
        n_full = sum(1 for L in self.layers if not L["recurrent"])
        self.kv_index = {}
        for il, L in enumerate(self.layers):
            if not L["recurrent"]:
                self.kv_index[il] = len(self.kv_index)
        self.kc = torch.zeros(max(1, n_full), max_ctx, self.nkv, dtype=kv_dtype, device=dev)
        self.vc = torch.zeros_like(self.kc)
        if hybrid:
            n_rec = cfg.n_layer - n_full
            self.gdn_qkv, self.gdn_z, self.gdn_ba = z(cfg.conv_dim), z(self.gdn_vd), z(2 * cfg.ssm_dt_rank)
            self.gdn_out = z(self.gdn_vd)
            self.gdn_N = _iarr([cfg.conv_dim, self.gdn_vd, 2 * cfg.ssm_dt_rank])
            self.gdn_y = _parr([self.gdn_qkv.data_ptr(), self.gdn_z.data_ptr(), self.gdn_ba.data_ptr()])
            self.gdn_ring = torch.zeros(n_rec, cfg.ssm_d_conv, cfg.conv_dim, dtype=torch.float32, device=dev)
            self.gdn_state = torch.zeros(n_rec, cfg.ssm_dt_rank, cfg.ssm_d_state, cfg.ssm_d_state, dtype=torch.float32,
                                         device=dev)
            self.rec_index = {il: i for i, il in enumerate(j for j, L in enumerate(self.layers) if L["recurrent"])}
        self.seq = torch.zeros(max_ctx + 1, dtype=torch.int32, device=dev)
        self.scratch_tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self._graph = None
        torch.cuda.synchronize(dev)

    @classmethod
    def from_gguf(cls, path: str, device: int = 0, max_ctx: int = 512, kv_dtype=torch.float16):
        from hoard_b200 import gguf_io as gi
        g = gi.GGUFFile(path)
        hp = gi.read_hparams(g)
        tensors = {}
        for name, t in g.tensors.items():
            data = g.array(name) if t.type == F32 else g.data(name)
            tensors[name] = (t.type, t.ne, np.array(data))
        g.close()
        return cls(config_from_hparams(hp), tensors, device=device, max_ctx=max_ctx, eos_id=hp.eos_id,
                   kv_dtype=kv_dtype)

    def close(self):
        self.moe.close()

    # ---- one token: logits of position pos for token seq[pos]; argmax into `next_tok` ----
    def step(self, pos: int, next_tok: torch.Tensor, stream=None):
        c, hx, s = self.cfg, _hx(), _stream(stream)
        H = c.n_embd
        x, x2 = self.x, self.x2
        _ok(hx.hoard_hx_embed(self.embd_type, _ptr(self.embd), H, c.n_vocab, _ptr(self.seq[pos:pos + 1]), _ptr(x), s),
            "embed")
        for il, L in enumerate(self.layers):
            self._layer_attention(il, L, x, x2, hx, s, pos)
            self.moe.layers(il, 1, x2.view(1, H), stream=stream)
            x, x2 = x2, x
        _ok(hx.hoard_hx_rmsnorm_q8(_ptr(x), H, c.eps, _ptr(self.out_norm), _ptr(self.q8), s), "rmsnorm_q8")
        _ok(hx.hoard_hx_gemv(self.out_type, _ptr(self.out_w), c.n_vocab, H, _ptr(self.q8), None, _ptr(self.logits), s),
            "gemv")
        _ok(hx.hoard_hx_argmax(_ptr(self.logits), c.n_vocab, _ptr(next_tok), s), "argmax")

    def _layer_attention(self, il, L, x, x2, hx, s, pos=None, bufs=None):
        """Graph A's attention part of layer il: x2 = Wo att + x (or the delta-net block's output
        projection + x). pos None: the device position. bufs: (q, k, v, q_rot, att, qkv_y) of one token of
        a batch (default: the step's own)."""
        c = self.cfg
        H, hd = c.n_embd, c.head_dim
        if L["recurrent"]:
            self._layer_gdn(il, L, x, x2, hx, s, pos)
            return
        q, k, v, q_rot, att, qkv_y = bufs or (self.q, self.k, self.v, self.q_rot, self.att, self.qkv_y)
        kc, vc = self.kc[self.kv_index[il]], self.vc[self.kv_index[il]]
        _ok(hx.hoard_hx_rmsnorm_q8(_ptr(x), H, c.eps, _ptr(L["attn_norm"]), _ptr(self.q8), s), "rmsnorm_q8")
        _ok(hx.hoard_hx_gemv_multi(3, L["qkv_types"], L["qkv_w"], self.qkv_N, H, _ptr(self.q8), None, qkv_y, s),
            "gemv qkv")
        mode = QK_MODE[c.qk_norm]
        qn, kn = (L["q_norm"], L["k_norm"]) if mode else (None, None)
        scale = 1.0 / math.sqrt(hd)
        if c.attn_gate or c.n_rot != hd:
            # fused q + gate rows ([q | gate] per head), partial rotary dims
            qs = 2 * hd if c.attn_gate else hd
            pd = None if pos is not None else _ptr(self.pos_dev)
            p0 = pos if pos is not None else 0
            _ok(hx.hoard_hx_qknorm_rope_store_ex(_ptr(q), _ptr(k), _ptr(v), _ptr(qn), _ptr(kn), mode, c.eps, c.n_head,
                                                 c.n_head_kv, hd, qs, c.n_rot, p0, pd, self.max_ctx, c.freq_base,
                                                 _ptr(q_rot), _ptr(kc), _ptr(vc), self.kv_type, s), "qk rope")
            n_pos = pos + 1 if pos is not None else self.max_ctx
            gate = _ptr(q) + 4 * hd if c.attn_gate else None
            _ok(hx.hoard_hx_attention_ex(_ptr(q_rot), _ptr(kc), _ptr(vc), c.n_head, c.n_head_kv, hd, n_pos, pd, scale,
                                         gate, qs, _ptr(att), self.kv_type, s), "attention")
        elif pos is None:
            _ok(hx.hoard_hx_qknorm_rope_store_at(_ptr(q), _ptr(k), _ptr(v), _ptr(qn), _ptr(kn), mode, c.eps, c.n_head,
                                                 c.n_head_kv, hd, _ptr(self.pos_dev), self.max_ctx, c.freq_base,
                                                 _ptr(q_rot), _ptr(kc), _ptr(vc), self.kv_type, s), "qk rope")
            _ok(hx.hoard_hx_attention_at(_ptr(q_rot), _ptr(kc), _ptr(vc), c.n_head, c.n_head_kv, hd,
                                         _ptr(self.pos_dev), self.max_ctx, scale, _ptr(att), self.kv_type, s),
                "attention")
        else:
            _ok(hx.hoard_hx_qknorm_rope_store(_ptr(q), _ptr(k), _ptr(v), _ptr(qn), _ptr(kn), mode, c.eps, c.n_head,
                                              c.n_head_kv, hd, pos, c.freq_base, _ptr(q_rot), _ptr(kc), _ptr(vc),
                                              self.kv_type, s), "qk rope")
            _ok(hx.hoard_hx_attention(_ptr(q_rot), _ptr(kc), _ptr(vc), c.n_head, c.n_head_kv, hd, pos + 1, scale,
                                      _ptr(att), self.kv_type, s), "attention")
        _ok(hx.hoard_hx_quant_q8(_ptr(att), self.nq, _ptr(self.q8), s), "quant")
        ty, wo = L["o"]
        _ok(hx.hoard_hx_gemv(ty, _ptr(wo), H, self.nq, _ptr(self.q8), _ptr(x), _ptr(x2), s), "gemv")

    def _layer_gdn(self, il, L, x, x2, hx, s, pos=None):
        """A gated delta-net block (src/run_qwen35.cpp:508-553): x2 = W_out gdn(RMSNorm(x) * attn_norm) + x."""
        c = self.cfg
        H, r = c.n_embd, self.rec_index[il]
        _ok(hx.hoard_hx_rmsnorm_q8(_ptr(x), H, c.eps, _ptr(L["attn_norm"]), _ptr(self.q8), s), "rmsnorm_q8")
        _ok(hx.hoard_hx_gemv_multi(3, L["qkv_types"], L["qkv_w"], self.gdn_N, H, _ptr(self.q8), None, self.gdn_y, s),
            "gemv qkv z ba")
        _ok(hx.hoard_hx_gdn_step(_ptr(self.gdn_qkv), _ptr(self.gdn_z), _ptr(self.gdn_ba), _ptr(L["conv_w"]),
                                 _ptr(self.gdn_ring[r]), _ptr(L["dt_bias"]), _ptr(L["ssm_a"]), _ptr(L["ssm_norm"]),
                                 _ptr(self.gdn_state[r]), c.ssm_dt_rank, c.ssm_n_group, c.ssm_d_state, c.ssm_d_conv,
                                 c.eps, pos if pos is not None else 0, None if pos is not None else _ptr(self.pos_dev),
                                 _ptr(self.gdn_out), s), "gdn step")
        _ok(hx.hoard_hx_quant_q8(_ptr(self.gdn_out), self.gdn_vd, _ptr(self.q8), s), "quant")
        ty, wo = L["o"]
        _ok(hx.hoard_hx_gemv(ty, _ptr(wo), H, self.gdn_vd, _ptr(self.q8), _ptr(x), _ptr(x2), s), "gemv")

    def reset_state(self):
        """Zeroes the delta-net states (the start of a sequence; src/run_qwen35.cpp:366-373)."""
        if hasattr(self, "gdn_state"):
            self.gdn_state.zero_()

    def _step_at(self, stream=None):
        """One decode step at the device position: token seq[pos] -> seq[pos + 1], pos += 1."""
        c, hx, s = self.cfg, _hx(), _stream(stream)
        H = c.n_embd
        x, x2 = self.x, self.x2
        _ok(hx.hoard_hx_embed_at(self.embd_type, _ptr(self.embd), H, c.n_vocab, _ptr(self.seq), _ptr(self.pos_dev),
                                 _ptr(x), s), "embed")
        for il, L in enumerate(self.layers):
            self._layer_attention(il, L, x, x2, hx, s)
            self.moe.layers(il, 1, x2.view(1, H), stream=stream)
            x, x2 = x2, x
        _ok(hx.hoard_hx_rmsnorm_q8(_ptr(x), H, c.eps, _ptr(self.out_norm), _ptr(self.q8), s), "rmsnorm_q8")
        _ok(hx.hoard_hx_gemv(self.out_type, _ptr(self.out_w), c.n_vocab, H, _ptr(self.q8), None, _ptr(self.logits), s),
            "gemv")
        _ok(hx.hoard_hx_argmax_at(_ptr(self.logits), c.n_vocab, _ptr(self.seq), _ptr(self.pos_dev), self.seq.numel(), s),
            "argmax")

    def prefill(self, prompt, stream=None):
        """Runs the prompt tokens but the last through the step (their KV entries), then sets the
        device position to the last prompt token."""
        T = len(prompt)
        self.reset_state()
        self.seq[:T].copy_(torch.tensor(prompt, dtype=torch.int32))
        for p in range(T - 1):
            self.step(p, self.scratch_tok, stream)
        self.pos_dev.fill_(T - 1)

    def capture(self):
        """Captures one decode step (position in device memory) as a CUDA graph."""
        if self._graph is None:
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._step_at()
            self._graph = g
        return self._graph

    def generate_graphed(self, prompt, n_gen: int):
        """Greedy decode like generate(), each generated token one replay of the captured step."""
        T = len(prompt)
        if T < 1 or T + n_gen > self.max_ctx:
            raise ValueError("prompt + n_gen must fit max_ctx")
        g = self.capture()
        self.prefill(prompt)
        for _ in range(n_gen):
            g.replay()
        torch.cuda.synchronize(self.dev)
        self.moe.sync_status()
        return self.seq[T:T + n_gen].tolist()

    def forward_batch(self, tokens, base: int, stream=None) -> torch.Tensor:
        """One forward over m <= MAX_BATCH consecutive tokens at positions base .. base+m-1 (causal:
        token i attends to positions <= base+i; K/V stored for all m), the MoE layers batched (T = m).
        Returns the logits [m][vocab]; row i predicts position base+i+1. hoard's verify pass,
        src/run_specloop.cpp:76-150."""
        c, hx, s = self.cfg, _hx(), _stream(stream)
        m, H, hd = len(tokens), c.n_embd, c.head_dim
        if c.full_attn_interval > 0:
            raise ValueError("batched forward of a hybrid (delta-net) model is not supported: its state is sequential")
        if not 1 <= m <= MAX_BATCH or base + m > self.max_ctx:
            raise ValueError("batch must be 1..MAX_BATCH tokens inside max_ctx")
        self.seq[base:base + m].copy_(torch.tensor(tokens, dtype=torch.int32))
        if not hasattr(self, "_xb"):
            z = lambda *sh: torch.zeros(*sh, dtype=torch.float32, device=self.dev)
            self._xb, self._x2b, self._curb = z(MAX_BATCH, H), z(MAX_BATCH, H), z(MAX_BATCH, H)
            self._qb, self._kb, self._vb = z(MAX_BATCH, self.nq), z(MAX_BATCH, self.nkv), z(MAX_BATCH, self.nkv)
            self._attb, self._lgb = z(MAX_BATCH, self.nq), z(MAX_BATCH, c.n_vocab)
        xb, x2b, cur = self._xb, self._x2b, self._curb
        for i in range(m):
            _ok(hx.hoard_hx_embed(self.embd_type, _ptr(self.embd), H, c.n_vocab, _ptr(self.seq[base + i:base + i + 1]),
                                  _ptr(xb[i]), s), "embed")
        if not hasattr(self, "_qrb"):
            self._qrb = torch.zeros(MAX_BATCH, self.nq, dtype=torch.float32, device=self.dev)
            self._qkv_yb = [_parr([self._qb[i].data_ptr(), self._kb[i].data_ptr(), self._vb[i].data_ptr()])
                            for i in range(MAX_BATCH)]
        for il, L in enumerate(self.layers):
            for i in range(m):
                bufs = (self._qb[i], self._kb[i], self._vb[i], self._qrb[i], self._attb[i], self._qkv_yb[i])
                self._layer_attention(il, L, xb[i], x2b[i], hx, s, base + i, bufs)
            self.moe.layers(il, 1, x2b[:m], stream=stream)
            xb, x2b = x2b, xb
        for i in range(m):
            _ok(hx.hoard_hx_rmsnorm_q8(_ptr(xb[i]), H, c.eps, _ptr(self.out_norm), _ptr(self.q8), s), "rmsnorm_q8")
            _ok(hx.hoard_hx_gemv(self.out_type, _ptr(self.out_w), c.n_vocab, H, _ptr(self.q8), None,
                                 _ptr(self._lgb[i]), s), "gemv")
        return self._lgb[:m].clone()

    def speculative_generate(self, prompt, n_gen: int, k_draft: int = 4):
        """hoard's speculative loop (src/run_specloop.cpp:189-210): draft k tokens greedily with the same
        model routed to its top-1 expert, verify them in one batched forward with the full top-k,
        accept the matching prefix, then run the corrected token. Greedy and lossless: the result
        equals generate()'s. Returns (tokens, {"rounds", "proposed", "accepted"})."""
        T, k_full = len(prompt), self.cfg.n_expert_used
        if T < 1 or T + n_gen + k_draft + 1 > self.max_ctx or not 1 <= k_draft <= MAX_BATCH:
            raise ValueError("prompt + n_gen + k_draft must fit max_ctx, 1 <= k_draft <= MAX_BATCH")
        self.seq[:T].copy_(torch.tensor(prompt, dtype=torch.int32))
        for p in range(T):
            self.step(p, self.scratch_tok)
        pred = self.logits.clone()
        cur, out, stats = T, [], {"rounds": 0, "proposed": 0, "accepted": 0}
        while len(out) < n_gen:
            draft, lg, dpos = [], pred, cur
            self.moe.set_top_k(1)
            try:
                for _ in range(k_draft):
                    d = int(torch.argmax(lg).item())
                    draft.append(d)
                    self.seq[dpos] = d
                    self.step(dpos, self.scratch_tok)
                    lg = self.logits.clone()
                    dpos += 1
            finally:
                self.moe.set_top_k(k_full)
            V = self.forward_batch(draft, cur)
            n, last = 0, pred
            for j in range(k_draft):
                tgt_l = pred if j == 0 else V[j - 1]
                if draft[j] == int(torch.argmax(tgt_l).item()):
                    n += 1
                    if j == k_draft - 1:
                        last = V[k_draft - 1]
                else:
                    last = tgt_l
                    break
            stats["rounds"] += 1
            stats["proposed"] += k_draft
            stats["accepted"] += n
            out += draft[:n]
            cur += n
            if len(out) >= n_gen:
                break
            corrected = int(torch.argmax(last).item())
            out.append(corrected)
            self.seq[cur] = corrected
            self.step(cur, self.scratch_tok)
            pred = self.logits.clone()
            cur += 1
        self.moe.sync_status()
        return out[:n_gen], stats

    def score(self, tokens, first: int, stream=None) -> torch.Tensor:
        """Teacher-forced logits: runs tokens[0 .. n-2] through the decode step and returns the logits
        that predict tokens[first .. n-1] ([n - first][vocab])."""
        n = len(tokens)
        if not 1 <= first < n or n > self.max_ctx:
            raise ValueError("need 1 <= first < len(tokens) <= max_ctx")
        self.reset_state()
        self.seq[:n].copy_(torch.tensor(tokens, dtype=torch.int32))
        out = torch.empty(n - first, self.cfg.n_vocab, dtype=torch.float32, device=self.dev)
        for p in range(n - 1):
            self.step(p, self.scratch_tok, stream)
            if p >= first - 1:
                out[p - (first - 1)].copy_(self.logits)
        self.moe.sync_status(stream)
        return out

    def generate(self, prompt, n_gen: int, stop_at_eos: bool = False, logits_out: torch.Tensor | None = None,
                 stream=None):
        """Greedy decode of n_gen tokens after `prompt` (a list of ids). logits_out [n_gen][vocab], if given,
        receives the logits each generated token was chosen from. Returns the generated ids."""
        T = len(prompt)
        if T < 1 or T + n_gen > self.max_ctx:
            raise ValueError("prompt + n_gen must fit max_ctx")
        self.reset_state()
        self.seq[:T].copy_(torch.tensor(prompt, dtype=torch.int32))
        for p in range(T + n_gen - 1):
            out = self.seq[p + 1:p + 2] if p >= T - 1 else self.scratch_tok
            self.step(p, out, stream)
            if p >= T - 1 and logits_out is not None:
                logits_out[p - (T - 1)].copy_(self.logits)
            if stop_at_eos and p >= T - 1 and int(self.seq[p + 1].item()) == self.eos_id:
                return self.seq[T:p + 2].tolist()
        self.moe.sync_status(stream)
        return self.seq[T:T + n_gen].tolist()
