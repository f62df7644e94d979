"""hoard_moe_decode_noalloc: decode with the library's static device scratch, for callers that cannot
allocate device memory when they run a step (all device memory handed out by their own arena, or a
step loop that must not call cudaMalloc). Its output must match the regular fused
decode entry point (hoard_moe_layers) on the same context, call after call.

This file is collected last on purpose: it exercises a process-wide device array, and a failure here
should not stop a `-x` run before every other test has run. It builds its own fixtures, so it also
passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from hoard_b200 import moe
from tests.moe_fixtures import LayerSpec, load_context, make_layer, make_x, rel_l2, Q4_K, Q6_K

pytestmark = pytest.mark.gpu

DEV = 0
N_LAYER = 2


@pytest.fixture(scope="module")
def model():
    spec = LayerSpec(H=2048, E=64, k=8, I=768)
    down = [Q6_K, Q4_K]
    layers = [make_layer(LayerSpec(H=2048, E=64, k=8, I=768, types=(Q4_K, Q4_K, t)), seed=900 + i)
              for i, t in enumerate(down)]
    ctx = moe.MoEContext(n_embd=spec.H, n_expert=spec.E, n_expert_used=spec.k, n_ff=spec.I, n_layer=N_LAYER,
                         norm_topk=True, eps=spec.eps, gate_types=[Q4_K] * N_LAYER, up_types=[Q4_K] * N_LAYER,
                         down_types=down, max_tokens=1, device=DEV)
    for i, L in enumerate(layers):
        load_context(ctx, i, L)
    yield spec, ctx
    ctx.close()


def run(ctx, fn, x_np):
    x = torch.from_numpy(x_np).cuda(DEV)
    sel = torch.empty(N_LAYER, 1, ctx.k, dtype=torch.int32, device=x.device)
    w = torch.empty(N_LAYER, 1, ctx.k, device=x.device)
    fn(0, N_LAYER, x, sel, w)
    torch.cuda.synchronize(DEV)
    return x.cpu().numpy(), sel.cpu().numpy(), w.cpu().numpy()


def test_noalloc_matches_layers_on_consecutive_calls(model):
    spec, ctx = model
    for call in range(2):
        x_np = make_x(1, spec.H, seed=4000 + call)
        ref, ref_sel, ref_w = run(ctx, ctx.layers, x_np)
        out, sel, w = run(ctx, ctx.decode_noalloc, x_np)
        assert np.array_equal(sel, ref_sel), call
        assert np.allclose(w, ref_w, rtol=1e-5, atol=1e-7), call
        # the same kernel and arithmetic with integer (fixed-point) router sums: the same bits
        assert rel_l2(out - x_np, ref - x_np) < 1e-5, call
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), call
    ctx.sync_status()


def test_noalloc_calls_allocate_no_device_memory(model):
    """The entry point's promise: after the first call, further calls change neither the device's free
    memory nor torch's allocations."""
    spec, ctx = model
    x = torch.from_numpy(make_x(1, spec.H, seed=4100)).cuda(DEV)
    ctx.decode_noalloc(0, N_LAYER, x)
    torch.cuda.synchronize(DEV)
    free0, _ = torch.cuda.mem_get_info(DEV)
    alloc0 = torch.cuda.memory_allocated(DEV)
    for _ in range(5):
        ctx.decode_noalloc(0, N_LAYER, x)
    ctx.decode_noalloc_status()            # the static array's error word: clear, read without allocating
    torch.cuda.synchronize(DEV)
    free1, _ = torch.cuda.mem_get_info(DEV)
    assert free1 == free0 and torch.cuda.memory_allocated(DEV) == alloc0
    ctx.sync_status()


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    ctx = moe.MoEContext(n_embd=2048, n_expert=16, n_expert_used=2, n_ff=1280, n_layer=1, max_tokens=1, device=DEV)
    x = torch.zeros(1, 2048, device=f"cuda:{DEV}")
    with pytest.raises(moe.HoardError) as ei:
        ctx.decode_noalloc(0, 1, x)
    assert ei.value.status == moe.HOARD_EINVAL
    assert "static decode scratch" in str(ei.value)
    ctx.close()
