"""GGUF v3 reader / writer and a loader that fills a MoEContext from a GGUF model file.

hoard reads its models with ggml's gguf API (src/run_moe_stream.cpp:118-186): hyper-parameters from
the architecture-prefixed metadata keys, expert tensors `blk.N.ffn_{gate,up,down}_exps.weight`
left on disk as (file offset, per-expert stride = nbytes / n_expert, type) per layer, and every
other tensor loaded to the device. This module is that step for this library, written from the
GGUF v3 format definition:

    "GGUF" | u32 version | u64 n_tensors | u64 n_kv | kv pairs | tensor infos | pad | data
    kv:     string key | u32 value type | value        (string = u64 length + bytes)
    tensor: string name | u32 n_dims | u64 ne[n_dims] | u32 ggml type | u64 offset from data start

The data section and every tensor start on `general.alignment` (default 32). A tensor with
ne = [K_in, N_out, E] stores E experts of N_out rows of K_in elements, quantised along K_in.

`GGUFFile` maps the file read-only (numpy memmap) and hands out views; `read_hparams` applies
hoard's rules (renormalised top-k except for OLMoE, head_dim from `attention.key_length` or the
q projection, per-head QK norm when its length equals head_dim); `GGUFWriter` emits the seeded
models; `load_moe_context` creates a MoEContext and uploads routers, norms, experts (all resident,
or a subset into fewer slots) and shared experts.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
DEFAULT_ALIGNMENT = 32

# metadata value types
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, T_UINT64, T_INT64, \
    T_FLOAT64 = range(13)
_SCALAR = {T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I", T_INT32: "<i",
           T_FLOAT32: "<f", T_BOOL: "<?", T_UINT64: "<Q", T_INT64: "<q", T_FLOAT64: "<d"}

# ggml tensor types this library reads or writes: (elements per block, bytes per block)
GGML_F32, GGML_F16, GGML_Q4_K, GGML_Q6_K, GGML_BF16 = 0, 1, 12, 14, 30
GGML_BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210), GGML_BF16: (1, 2)}


class GGUFError(ValueError):
    pass


def tensor_nbytes(ne, ggml_type: int) -> int:
    if ggml_type not in GGML_BLOCK:
        raise GGUFError(f"unsupported ggml type {ggml_type}")
    per, nb = GGML_BLOCK[ggml_type]
    if ne[0] % per:
        raise GGUFError(f"ne[0] = {ne[0]} is not a multiple of the block size {per}")
    n = 1
    for d in ne:
        n *= int(d)
    return n // per * nb


@dataclass
class TensorInfo:
    name: str
    ne: tuple                # ggml order: ne[0] is the contiguous (K_in) dimension
    type: int
    offset: int              # absolute file offset of the data
    nbytes: int


@dataclass
class GGUFFile:
    path: str
    version: int = 0
    kv: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    alignment: int = DEFAULT_ALIGNMENT
    data_offset: int = 0

    def __post_init__(self):
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        self._parse()

    # -- parsing --
    def _parse(self):
        buf = self._map
        pos = 0

        def take(n):
            nonlocal pos
            if pos + n > buf.size:
                raise GGUFError("truncated GGUF file")
            b = bytes(buf[pos:pos + n])
            pos += n
            return b

        def u32():
            return struct.unpack("<I", take(4))[0]

        def u64():
            return struct.unpack("<Q", take(8))[0]

        def string():
            n = u64()
            return take(n).decode("utf-8")

        def value(vt):
            if vt in _SCALAR:
                f = _SCALAR[vt]
                return struct.unpack(f, take(struct.calcsize(f)))[0]
            if vt == T_STRING:
                return string()
            if vt == T_ARRAY:
                et, n = u32(), u64()
                return [value(et) for _ in range(n)]
            raise GGUFError(f"unknown metadata value type {vt}")

        if take(4) != GGUF_MAGIC:
            raise GGUFError("not a GGUF file")
        self.version = u32()
        if self.version not in (2, 3):
            raise GGUFError(f"unsupported GGUF version {self.version}")
        n_tensors, n_kv = u64(), u64()
        for _ in range(n_kv):
            key = string()
            self.kv[key] = value(u32())
        self.alignment = int(self.kv.get("general.alignment", DEFAULT_ALIGNMENT))
        infos = []
        for _ in range(n_tensors):
            name = string()
            nd = u32()
            ne = tuple(u64() for _ in range(nd))
            ty = u32()
            off = u64()
            infos.append((name, ne, ty, off))
        self.data_offset = (pos + self.alignment - 1) // self.alignment * self.alignment
        for name, ne, ty, off in infos:
            nb = tensor_nbytes(ne, ty) if ty in GGML_BLOCK else -1
            abs_off = self.data_offset + off
            if nb >= 0 and abs_off + nb > buf.size:
                raise GGUFError(f"tensor {name} extends past the end of the file")
            self.tensors[name] = TensorInfo(name, ne, ty, abs_off, nb)

    # -- access --
    def data(self, name: str) -> np.ndarray:
        """Raw bytes of a tensor (a read-only view of the mapping)."""
        t = self.tensors[name]
        if t.nbytes < 0:
            raise GGUFError(f"tensor {name} has a type this library does not read ({t.type})")
        return self._map[t.offset:t.offset + t.nbytes]

    def array(self, name: str) -> np.ndarray:
        """An f32 / f16 / bf16 tensor as a numpy array shaped [ne[-1], ..., ne[0]] (f32 for bf16)."""
        t = self.tensors[name]
        raw = self.data(name)
        shape = tuple(reversed(t.ne))
        if t.type == GGML_F32:
            return raw.view(np.float32).reshape(shape)
        if t.type == GGML_F16:
            return raw.view(np.float16).reshape(shape)
        if t.type == GGML_BF16:
            return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(shape)
        raise GGUFError(f"tensor {name} is quantised (type {t.type}); use data() / expert()")

    def expert(self, name: str, e: int) -> np.ndarray:
        """Raw bytes of expert e of a [K_in, N_out, E] tensor: per-expert stride nbytes / E."""
        t = self.tensors[name]
        if len(t.ne) != 3:
            raise GGUFError(f"{name} is not an expert tensor")
        n_exp = int(t.ne[2])
        if not 0 <= e < n_exp:
            raise GGUFError(f"expert {e} out of range (0..{n_exp - 1})")
        stride = t.nbytes // n_exp
        return self._map[t.offset + e * stride:t.offset + (e + 1) * stride]

    def close(self):
        m = getattr(self, "_map", None)
        if m is not None and hasattr(m, "_mmap") and m._mmap is not None:
            m._mmap.close()
        self._map = None


@dataclass
class HParams:
    arch: str
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_ff: int
    n_expert: int
    n_expert_used: int
    n_ctx: int
    freq_base: float
    eps: float
    n_vocab: int
    has_qk_norm: bool
    qk_perhead: bool
    norm_topk: bool
    eos_id: int
    n_ff_shexp: int = 0


def read_hparams(g: GGUFFile) -> HParams:
    """hoard's hyper-parameter rules (src/run_moe_stream.cpp:125-150)."""
    arch = str(g.kv.get("general.architecture", ""))

    def key(s, default):
        return g.kv.get(f"{arch}.{s}", default)

    n_layer = int(key("block_count", 0))
    n_embd = int(key("embedding_length", 0))
    n_head = int(key("attention.head_count", 0))
    n_head_kv = int(key("attention.head_count_kv", n_head))
    n_ff = int(key("feed_forward_length", 0))
    n_ff = int(key("expert_feed_forward_length", n_ff))
    n_expert = int(key("expert_count", 0))
    n_used = int(key("expert_used_count", 0))
    n_ctx = int(key("context_length", 4096))
    freq_base = float(key("rope.freq_base", 10000.0))
    eps = float(key("attention.layer_norm_rms_epsilon", 1e-5))
    n_vocab, q_out, qk_norm_dim = 0, 0, 0
    if "token_embd.weight" in g.tensors:
        n_vocab = int(g.tensors["token_embd.weight"].ne[1])
    if "blk.0.attn_q.weight" in g.tensors:
        q_out = int(g.tensors["blk.0.attn_q.weight"].ne[1])
    has_qk = "blk.0.attn_q_norm.weight" in g.tensors
    if has_qk:
        qk_norm_dim = int(g.tensors["blk.0.attn_q_norm.weight"].ne[0])
    derived = q_out // n_head if (n_head and q_out) else (n_embd // n_head if n_head else 0)
    head_dim = int(key("attention.key_length", derived))
    n_ff_sh = int(key("expert_shared_feed_forward_length", 0))
    if not n_ff_sh:
        sh = [t for n, t in g.tensors.items() if n.endswith(".ffn_gate_shexp.weight")]
        n_ff_sh = int(sh[0].ne[1]) if sh else 0
    if n_layer <= 0 or n_embd <= 0 or n_expert <= 0:
        raise GGUFError("unsupported or missing hyper-parameters (block_count, embedding_length, expert_count)")
    return HParams(arch=arch, n_layer=n_layer, n_embd=n_embd, n_head=n_head, n_head_kv=n_head_kv, head_dim=head_dim,
                   n_ff=n_ff, n_expert=n_expert, n_expert_used=n_used, n_ctx=n_ctx, freq_base=freq_base, eps=eps,
                   n_vocab=n_vocab, has_qk_norm=has_qk, qk_perhead=has_qk and qk_norm_dim == head_dim,
                   norm_topk=arch != "olmoe", eos_id=int(g.kv.get("tokenizer.ggml.eos_token_id", 50279)),
                   n_ff_shexp=n_ff_sh)


class GGUFWriter:
    """Writes a GGUF v3 file: metadata, then tensors in the order added, each aligned."""

    def __init__(self, arch: str, alignment: int = DEFAULT_ALIGNMENT):
        self.kv: list[tuple[str, int, object]] = []
        self.tensors: list[tuple[str, tuple, int, np.ndarray]] = []
        self.alignment = alignment
        self.add("general.architecture", arch, T_STRING)
        if alignment != DEFAULT_ALIGNMENT:
            self.add("general.alignment", alignment, T_UINT32)

    def add(self, key: str, value, vtype: int | None = None, elem_type: int | None = None):
        if vtype is None:
            if isinstance(value, bool):
                vtype = T_BOOL
            elif isinstance(value, int):
                vtype = T_UINT32 if 0 <= value < 2 ** 32 else T_INT64
            elif isinstance(value, float):
                vtype = T_FLOAT32
            elif isinstance(value, str):
                vtype = T_STRING
            elif isinstance(value, (list, tuple)):
                vtype = T_ARRAY
            else:
                raise GGUFError(f"cannot infer the GGUF type of {key}")
        if vtype == T_ARRAY and elem_type is None:
            v0 = value[0] if len(value) else 0
            elem_type = T_STRING if isinstance(v0, str) else T_FLOAT32 if isinstance(v0, float) else T_INT32
        self.kv.append((key, vtype, (elem_type, list(value)) if vtype == T_ARRAY else value))

    def add_tensor(self, name: str, ne, ggml_type: int, data):
        """data: raw bytes (uint8 array) or an f32/f16 array whose element count matches ne."""
        ne = tuple(int(d) for d in ne)
        raw = np.ascontiguousarray(data).reshape(-1).view(np.uint8)
        if raw.size != tensor_nbytes(ne, ggml_type):
            raise GGUFError(f"{name}: {raw.size} bytes for ne={ne} type {ggml_type} "
                            f"(expected {tensor_nbytes(ne, ggml_type)})")
        self.tensors.append((name, ne, ggml_type, raw))

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _value(self, vtype, value) -> bytes:
        if vtype in _SCALAR:
            return struct.pack(_SCALAR[vtype], value)
        if vtype == T_STRING:
            return self._str(value)
        if vtype == T_ARRAY:
            et, items = value
            return struct.pack("<IQ", et, len(items)) + b"".join(self._value(et, v) for v in items)
        raise GGUFError(f"unknown value type {vtype}")

    def write(self, path: str):
        al = self.alignment
        head = bytearray(GGUF_MAGIC + struct.pack("<IQQ", GGUF_VERSION, len(self.tensors), len(self.kv)))
        for key, vt, val in self.kv:
            head += self._str(key) + struct.pack("<I", vt) + self._value(vt, val)
        off = 0
        offsets = []
        for name, ne, ty, raw in self.tensors:
            offsets.append(off)
            head += self._str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
            head += struct.pack("<IQ", ty, off)
            off = (off + raw.size + al - 1) // al * al
        pad = (-len(head)) % al
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            f.write(head)
            f.write(b"\0" * pad)
            for (name, ne, ty, raw), o in zip(self.tensors, offsets):
                f.write(raw.tobytes())
                f.write(b"\0" * ((-raw.size) % al))
        os.replace(tmp, path)


def add_moe_layer(w: GGUFWriter, il: int, w_router: np.ndarray, w_norm: np.ndarray, gate: np.ndarray,
                  up: np.ndarray, down: np.ndarray, types: tuple, shared: dict | None = None):
    """One MoE layer in hoard's tensor names: router f32 ne=[H, E], ffn_norm f32 [H], experts
    [K_in, N_out, E] with the expert index outermost (gate/up: K_in = H, N_out = I; down: K_in = I,
    N_out = H). gate/up/down are uint8 [E, N_out, row bytes]."""
    E, H = w_router.shape
    I = gate.shape[1]
    w.add_tensor(f"blk.{il}.ffn_gate_inp.weight", (H, E), GGML_F32, w_router.astype(np.float32))
    w.add_tensor(f"blk.{il}.ffn_norm.weight", (H,), GGML_F32, w_norm.astype(np.float32))
    w.add_tensor(f"blk.{il}.ffn_gate_exps.weight", (H, I, E), types[0], gate)
    w.add_tensor(f"blk.{il}.ffn_up_exps.weight", (H, I, E), types[1], up)
    w.add_tensor(f"blk.{il}.ffn_down_exps.weight", (I, H, E), types[2], down)
    if shared is not None:
        Ish = shared["gate"].shape[0]
        w.add_tensor(f"blk.{il}.ffn_gate_shexp.weight", (H, Ish), shared["gate_type"], shared["gate"])
        w.add_tensor(f"blk.{il}.ffn_up_shexp.weight", (H, Ish), shared["up_type"], shared["up"])
        w.add_tensor(f"blk.{il}.ffn_down_shexp.weight", (Ish, H), shared["down_type"], shared["down"])
        w.add_tensor(f"blk.{il}.ffn_gate_inp_shexp.weight", (H,), GGML_F32, shared["gate_inp"].astype(np.float32))


def load_moe_context(path: str, device: int = 0, max_tokens: int = 1, n_slots: int | None = None,
                     experts: dict | None = None, resid_dtype=None, layers=None):
    """Creates a MoEContext for the MoE layers of a GGUF model and uploads them.

    experts: None uploads every expert into slot = expert id (all resident; n_slots defaults to
    n_expert); or {layer: {expert: slot}} for a partial pool of n_slots slots (the residency layer
    fills the rest). layers: restrict to these layer indices (default all). Returns (ctx, hparams,
    gguf_file); the file stays mapped for RAM-tier registration."""
    import torch
    from hoard_b200 import moe

    g = GGUFFile(path)
    hp = read_hparams(g)
    layer_ids = list(range(hp.n_layer)) if layers is None else list(layers)
    types = []
    for il in layer_ids:
        t = tuple(g.tensors[f"blk.{il}.ffn_{m}_exps.weight"].type for m in ("gate", "up", "down"))
        types.append(t)
    has_sh = [f"blk.{il}.ffn_gate_shexp.weight" in g.tensors for il in layer_ids]
    if any(has_sh) and not all(has_sh):
        raise GGUFError("a shared expert in some MoE layers but not in others is not supported")
    sh = all(has_sh)
    kw = {}
    if resid_dtype is not None:
        kw["resid_dtype"] = resid_dtype
    if sh:
        sh_types = {tuple(g.tensors[f"blk.{il}.ffn_{m}_shexp.weight"].type for m in ("gate", "up", "down"))
                    for il in layer_ids}
        if len(sh_types) != 1:
            raise GGUFError("shared experts of different types across layers are not supported")
        kw.update(n_ff_shexp=int(g.tensors[f"blk.{layer_ids[0]}.ffn_gate_shexp.weight"].ne[1]),
                  shexp_types=sh_types.pop())
    ctx = moe.MoEContext(n_embd=hp.n_embd, n_expert=hp.n_expert, n_expert_used=hp.n_expert_used, n_ff=hp.n_ff,
                         n_layer=len(layer_ids), n_slots=n_slots or hp.n_expert, norm_topk=hp.norm_topk, eps=hp.eps,
                         gate_types=[t[0] for t in types], up_types=[t[1] for t in types],
                         down_types=[t[2] for t in types], max_tokens=max_tokens, device=device, **kw)
    dev = torch.device("cuda", device)

    def to_dev(a):
        return torch.from_numpy(np.array(a)).to(dev)

    for li, il in enumerate(layer_ids):
        ctx.set_router(li, to_dev(g.array(f"blk.{il}.ffn_gate_inp.weight")), to_dev(g.array(f"blk.{il}.ffn_norm.weight")))
        chosen = ({e: e for e in range(hp.n_expert)} if experts is None else experts.get(il, {}))
        names = [f"blk.{il}.ffn_{m}_exps.weight" for m in ("gate", "up", "down")]
        for e, slot in chosen.items():
            ctx.upload_expert(li, slot, *(to_dev(g.expert(n, e)) for n in names))
        if sh:
            ctx.set_shared(li, to_dev(g.data(f"blk.{il}.ffn_gate_shexp.weight")),
                           to_dev(g.data(f"blk.{il}.ffn_up_shexp.weight")),
                           to_dev(g.data(f"blk.{il}.ffn_down_shexp.weight")),
                           to_dev(g.array(f"blk.{il}.ffn_gate_inp_shexp.weight")))
    torch.cuda.synchronize(dev)
    return ctx, hp, g
