"""The C-ABI library loads without a GPU, exports every entry point include/hoard_moe.h declares,
and rejects malformed descriptors before touching CUDA."""
import ctypes
import os
import re

import pytest

from hoard_b200 import moe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hoard_moe.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(hoard_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for want in ("hoard_moe_create", "hoard_moe_destroy", "hoard_moe_upload_expert", "hoard_moe_set_router",
                 "hoard_moe_route", "hoard_moe_experts", "hoard_moe_layer"):
        assert want in names


def test_library_exports_every_declared_symbol():
    L = moe.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    assert sorted(moe.EXPORTED) == sorted(declared_functions())


def test_strerror():
    L = moe.lib()
    assert L.hoard_strerror(0) == b"ok"
    assert L.hoard_strerror(-1) == b"invalid argument"
    assert L.hoard_strerror(-4) == b"device wait timed out"


def _desc(**kw):
    base = dict(n_embd=2048, n_expert=128, n_expert_used=8, n_ff=768, n_layer=1, n_slots=128, norm_topk=1,
                eps=1e-6, resid_type=0, gate_types=None, up_types=None, down_types=None, n_ff_shexp=0,
                shexp_gate_type=12, shexp_up_type=12, shexp_down_type=14, max_tokens=16, device=0)
    base.update(kw)
    return moe.Desc(**base)


@pytest.mark.parametrize("bad", [dict(n_embd=2000), dict(n_ff=700), dict(n_expert_used=0), dict(n_expert_used=17),
                                 dict(n_expert=0), dict(n_expert=2048), dict(n_expert_used=9, n_expert=8),
                                 dict(max_tokens=0), dict(resid_type=1), dict(n_slots=0),
                                 dict(n_ff_shexp=512), dict(n_ff_shexp=768, shexp_down_type=3)])
def test_create_rejects_bad_descriptor(bad):
    L = moe.lib()
    h = ctypes.c_void_p()
    assert L.hoard_moe_create(ctypes.byref(_desc(**bad)), ctypes.byref(h)) == moe.HOARD_EINVAL
    assert not h.value


def test_create_rejects_bad_layer_types():
    L = moe.lib()
    h = ctypes.c_void_p()
    types = (ctypes.c_int * 2)(12, 13)
    d = _desc(n_layer=2, down_types=types)
    assert L.hoard_moe_create(ctypes.byref(d), ctypes.byref(h)) == moe.HOARD_EINVAL


def test_null_context_is_rejected():
    L = moe.lib()
    assert L.hoard_moe_destroy(None) == moe.HOARD_EINVAL
    assert L.hoard_moe_route(None, 0, None, 1, None, None, None) == moe.HOARD_EINVAL
    assert L.hoard_moe_layers(None, 0, 1, None, 1, None, None, None) == moe.HOARD_EINVAL
    assert L.hoard_moe_expert_bytes(None, 0) == -1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(moe, "_lib", None)
    monkeypatch.setattr(moe, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError):
        moe.lib()


HARNESS_HEADER = os.path.join(ROOT, "include", "hoard_harness.h")


def test_harness_header_symbols_exported():
    src = re.sub(r"/\*.*?\*/", "", open(HARNESS_HEADER).read(), flags=re.S)
    names = sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(hoard_\w+)\s*\(", src, flags=re.M)))
    assert "hoard_hx_gemv" in names and "hoard_hx_attention" in names
    L = moe.lib()
    assert not [n for n in names if not hasattr(L, n)]


def test_harness_rejects_bad_arguments():
    from hoard_b200 import harness as hx
    L = hx._hx()
    assert L.hoard_hx_q8_bytes(300) == -1 and L.hoard_hx_q8_bytes(0) == -1
    assert L.hoard_hx_q8_bytes(2048) == 2048 + 256 + 512
    one = ctypes.c_void_p(16)                      # never dereferenced: the checks come first
    assert L.hoard_hx_gemv(3, one, 8, 512, one, None, one, None) == moe.HOARD_EINVAL          # type
    assert L.hoard_hx_gemv(12, one, 8, 500, one, None, one, None) == moe.HOARD_EINVAL         # K % 256
    assert L.hoard_hx_rope_store(one, one, one, 4, 4, 127, 0, 1e4, one, one, 1, None) == moe.HOARD_EINVAL
    assert L.hoard_hx_rope_store(one, one, one, 4, 4, 128, 0, 1e4, one, one, 0, None) == moe.HOARD_EINVAL  # f32 cache
    assert L.hoard_hx_attention(one, one, one, 6, 4, 128, 5, 0.1, one, 1, None) == moe.HOARD_EINVAL
    assert L.hoard_hx_attention(one, one, one, 4, 4, 128, 0, 0.1, one, 30, None) == moe.HOARD_EINVAL
    assert L.hoard_hx_rmsnorm(one, 1, 9000, 1e-6, one, one, None) == moe.HOARD_EINVAL
    assert L.hoard_hx_embed(13, one, 512, 10, one, one, None) == moe.HOARD_EINVAL
    assert L.hoard_hx_argmax(None, 10, one, None) == moe.HOARD_EINVAL
