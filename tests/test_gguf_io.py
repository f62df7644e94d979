"""GGUF reader / writer (hoard_b200.gguf_io) on the CPU: round trip of metadata and tensors,
per-expert stride views, hoard's hyper-parameter rules, malformed files, and a cross-check in both
directions against the `gguf` Python package (a test dependency, not used by the library)."""
import numpy as np
import pytest

from hoard_b200 import gguf_io as gi
from tests.moe_fixtures import LayerSpec, make_layer, Q4_K, Q6_K

SPECS = [LayerSpec(H=512, E=8, k=2, I=256, types=(Q4_K, Q4_K, Q6_K), shared=True),
         LayerSpec(H=512, E=8, k=2, I=256, types=(Q4_K, Q4_K, Q4_K), shared=True)]


def write_model(path, arch="qwen3moe", layers=None, extra=None):
    layers = layers or [make_layer(s, seed=70 + i) for i, s in enumerate(SPECS)]
    w = gi.GGUFWriter(arch)
    w.add(f"{arch}.block_count", len(layers))
    w.add(f"{arch}.embedding_length", 512)
    w.add(f"{arch}.attention.head_count", 4)
    w.add(f"{arch}.attention.head_count_kv", 2)
    w.add(f"{arch}.expert_feed_forward_length", 256)
    w.add(f"{arch}.expert_count", 8)
    w.add(f"{arch}.expert_used_count", 2)
    w.add(f"{arch}.rope.freq_base", 1e6)
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)
    w.add("tokenizer.ggml.eos_token_id", 7)
    w.add("general.name", "seeded")
    w.add("test.list", [1, 2, 3], gi.T_ARRAY, gi.T_INT32)
    for k, v in (extra or {}).items():
        w.add(k, v)
    for il, L in enumerate(layers):
        gi.add_moe_layer(w, il, L.w_router, L.w_norm, L.gate, L.up, L.down, L.spec.types, L.shared)
    w.write(str(path))
    return layers


def test_round_trip(tmp_path):
    p = tmp_path / "m.gguf"
    layers = write_model(p)
    g = gi.GGUFFile(str(p))
    assert g.version == 3 and g.kv["general.architecture"] == "qwen3moe"
    assert g.kv["qwen3moe.block_count"] == 2 and g.kv["test.list"] == [1, 2, 3]
    assert abs(g.kv["qwen3moe.rope.freq_base"] - 1e6) < 1 and g.kv["general.name"] == "seeded"
    for il, L in enumerate(layers):
        t = g.tensors[f"blk.{il}.ffn_down_exps.weight"]
        assert t.ne == (256, 512, 8) and t.type == L.spec.types[2] and t.offset % 32 == 0
        assert np.array_equal(g.array(f"blk.{il}.ffn_gate_inp.weight"), L.w_router)
        assert np.array_equal(g.array(f"blk.{il}.ffn_norm.weight"), L.w_norm)
        for e in range(8):
            assert np.array_equal(g.expert(f"blk.{il}.ffn_gate_exps.weight", e), L.gate[e].reshape(-1))
            assert np.array_equal(g.expert(f"blk.{il}.ffn_down_exps.weight", e), L.down[e].reshape(-1))
    sh = layers[1].shared
    assert np.array_equal(g.data("blk.1.ffn_down_shexp.weight"), sh["down"].reshape(-1))
    with pytest.raises(gi.GGUFError):
        g.expert("blk.0.ffn_gate_exps.weight", 8)
    g.close()


def test_hparams_rules(tmp_path):
    p = tmp_path / "q.gguf"
    write_model(p, extra={"qwen3moe.attention.key_length": 128})
    hp = gi.read_hparams(gi.GGUFFile(str(p)))
    assert (hp.n_layer, hp.n_embd, hp.n_expert, hp.n_expert_used, hp.n_ff) == (2, 512, 8, 2, 256)
    assert hp.norm_topk and hp.head_dim == 128 and hp.n_head_kv == 2 and hp.eos_id == 7
    assert hp.n_ff_shexp == 256 and abs(hp.eps - 1e-6) < 1e-12
    p2 = tmp_path / "o.gguf"
    write_model(p2, arch="olmoe")
    hp2 = gi.read_hparams(gi.GGUFFile(str(p2)))
    assert not hp2.norm_topk                   # OLMoE keeps the softmax weights of its top-k
    assert hp2.head_dim == 512 // 4            # n_embd / n_head without key_length or a q projection


def test_malformed(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUX" + b"\0" * 64)
    with pytest.raises(gi.GGUFError):
        gi.GGUFFile(str(p))
    good = tmp_path / "m.gguf"
    write_model(good)
    raw = good.read_bytes()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(raw[:len(raw) // 2])
    with pytest.raises(gi.GGUFError):
        gi.GGUFFile(str(cut))
    w = gi.GGUFWriter("x")
    with pytest.raises(gi.GGUFError):
        w.add_tensor("t", (512, 2), Q4_K, np.zeros(100, np.uint8))


def test_gguf_package_reads_our_file(tmp_path):
    gguf = pytest.importorskip("gguf")
    p = tmp_path / "m.gguf"
    layers = write_model(p)
    r = gguf.GGUFReader(str(p))
    by = {t.name: t for t in r.tensors}
    t = by["blk.0.ffn_gate_exps.weight"]
    assert int(t.tensor_type) == Q4_K and [int(d) for d in t.shape] == [512, 256, 8]
    assert np.array_equal(np.asarray(t.data).reshape(-1).view(np.uint8), layers[0].gate.reshape(-1))
    assert np.array_equal(np.asarray(by["blk.1.ffn_gate_inp.weight"].data).reshape(8, 512), layers[1].w_router)


def test_we_read_gguf_package_file(tmp_path):
    gguf = pytest.importorskip("gguf")
    L = make_layer(SPECS[0], seed=5)
    p = tmp_path / "pkg.gguf"
    w = gguf.GGUFWriter(str(p), "qwen3moe")
    w.add_uint32("qwen3moe.block_count", 1)
    w.add_uint32("qwen3moe.embedding_length", 512)
    w.add_uint32("qwen3moe.expert_count", 8)
    w.add_uint32("qwen3moe.expert_used_count", 2)
    w.add_tensor("blk.0.ffn_gate_inp.weight", L.w_router)
    w.add_tensor("blk.0.ffn_gate_exps.weight", L.gate, raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = gi.GGUFFile(str(p))
    assert g.tensors["blk.0.ffn_gate_exps.weight"].ne == (512, 256, 8)
    assert np.array_equal(g.array("blk.0.ffn_gate_inp.weight"), L.w_router)
    for e in (0, 5, 7):
        assert np.array_equal(g.expert("blk.0.ffn_gate_exps.weight", e), L.gate[e].reshape(-1))
    hp = gi.read_hparams(g)
    assert hp.n_expert == 8 and hp.n_embd == 512
