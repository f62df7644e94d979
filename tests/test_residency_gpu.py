"""Residency layer on the GPU: a per-layer LRU slot pool smaller than the expert count, filled from a
RAM tier by hoard_moe_ensure on the library's upload stream (hoard's to_vram / fetch and
LRU, src/run_moe_stream.cpp:279-284, :380-421).

hoard's invariant "LRU cache == naive == all-resident, bit-identical" must hold: a decode sequence
through route -> host readback of sel -> ensure -> experts(slot_of_sel) equals the all-resident
context's route -> experts, bit for bit, while slots are evicted and re-filled."""
import numpy as np
import pytest
import torch

from hoard_b200 import moe
from tests.moe_fixtures import LayerSpec, make_layer, make_x

pytestmark = pytest.mark.gpu

DEV = 0
SPEC = LayerSpec(H=512, E=16, k=4, I=256)
N_LAYER = 2


def make_ctx(n_slots):
    ctx = moe.MoEContext(n_embd=SPEC.H, n_expert=SPEC.E, n_expert_used=SPEC.k, n_ff=SPEC.I, n_layer=N_LAYER,
                         n_slots=n_slots, norm_topk=True, eps=SPEC.eps, gate_types=[SPEC.types[0]] * N_LAYER,
                         up_types=[SPEC.types[1]] * N_LAYER, down_types=[SPEC.types[2]] * N_LAYER, max_tokens=4,
                         device=DEV)
    ctx.set_decode_impl(0)
    ctx.set_gemm_min_tokens(0)
    return ctx


@pytest.fixture(scope="module", params=["pinned", "pageable"])
def contexts(request):
    """Pinned RAM-tier bytes are re-laid in place over PCIe; pageable ones go through the staging buffer."""
    dev = torch.device("cuda", DEV)
    layers = [make_layer(SPEC, seed=700 + i) for i in range(N_LAYER)]
    full = make_ctx(SPEC.E)
    lru = make_ctx(6)
    host = []                                        # pinned RAM tier, kept alive for the contexts
    for il, L in enumerate(layers):
        for ctx in (full, lru):
            ctx.set_router(il, torch.from_numpy(L.w_router).to(dev), torch.from_numpy(L.w_norm).to(dev))
        for e in range(SPEC.E):
            full.upload_expert(il, e, torch.from_numpy(L.gate[e]).to(dev), torch.from_numpy(L.up[e]).to(dev),
                               torch.from_numpy(L.down[e]).to(dev))
            g, u, d = (torch.from_numpy(np.ascontiguousarray(a[e])) for a in (L.gate, L.up, L.down))
            if request.param == "pinned":
                g, u, d = g.pin_memory(), u.pin_memory(), d.pin_memory()
            host.append((g, u, d))
            lru.ram_tier(il, e, g, u, d)
    torch.cuda.synchronize(dev)
    yield full, lru, host
    full.close()
    lru.close()


def test_lru_decode_equals_all_resident(contexts):
    full, lru, _ = contexts
    before = lru.residency_stats()
    steps = 24
    for step in range(steps):
        x_np = make_x(1, SPEC.H, seed=50 + step)
        xf = torch.from_numpy(x_np).cuda(DEV)
        xl = torch.from_numpy(x_np).cuda(DEV)
        for il in range(N_LAYER):
            sel_f, w_f = full.route(il, xf)
            full.experts(il, sel_f, w_f, xf)
            sel, w = lru.route(il, xl)
            slots = lru.ensure(il, sel.cpu().numpy())               # the host readback hoard does
            lru.experts(il, sel, w, xl, slot_of_sel=torch.from_numpy(slots).cuda(DEV))
            assert np.array_equal(sel.cpu().numpy(), sel_f.cpu().numpy())
        torch.cuda.synchronize(DEV)
        assert np.array_equal(xl.cpu().numpy().view(np.uint32), xf.cpu().numpy().view(np.uint32)), step
    lru.sync_status()
    st = lru.residency_stats()
    lookups = st["hits"] + st["misses"] - before["hits"] - before["misses"]
    assert lookups == steps * N_LAYER * SPEC.k
    assert st["misses"] - before["misses"] >= 6 * N_LAYER                    # every slot filled at least once
    assert st["bytes_uploaded"] == st["misses"] * lru.expert_bytes(0)


def test_ensure_errors(contexts):
    full, lru, _ = contexts
    with pytest.raises(moe.HoardError) as ei:
        lru.ensure(0, np.arange(7, dtype=np.int32))                          # 7 experts, 6 slots
    assert ei.value.status == moe.HOARD_EINVAL
    with pytest.raises(moe.HoardError) as ei:
        lru.ensure(0, np.array([SPEC.E], dtype=np.int32))
    assert ei.value.status == moe.HOARD_EINVAL
    other = make_ctx(6)
    with pytest.raises(moe.HoardError) as ei:
        other.ensure(0, np.array([3], dtype=np.int32))                       # nothing registered
    assert ei.value.status == moe.HOARD_ESTATE
    other.close()
