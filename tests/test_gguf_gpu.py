"""A MoE model read from a GGUF file (hoard_b200.gguf_io.load_moe_context) computes exactly what the
same layers uploaded directly compute, for batched tokens and for decode."""
import numpy as np
import pytest
import torch

from hoard_b200 import gguf_io as gi, moe
from tests.moe_fixtures import load_context, make_x
from tests.test_gguf_io import SPECS, write_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 80])
def test_gguf_model_equals_direct_upload(tmp_path, T):
    p = tmp_path / "m.gguf"
    layers = write_model(p)
    ctx, hp, g = gi.load_moe_context(str(p), device=0, max_tokens=128)
    s = SPECS[0]
    ref = moe.MoEContext(n_embd=s.H, n_expert=s.E, n_expert_used=s.k, n_ff=s.I, n_layer=2, norm_topk=True,
                         eps=s.eps, gate_types=[L.spec.types[0] for L in layers],
                         up_types=[L.spec.types[1] for L in layers], down_types=[L.spec.types[2] for L in layers],
                         n_ff_shexp=s.I, shexp_types=s.sh_types, max_tokens=128, device=0)
    try:
        for il, L in enumerate(layers):
            load_context(ref, il, L)
        x_np = make_x(T, s.H, seed=T)
        xa = torch.from_numpy(x_np).cuda()
        xb = torch.from_numpy(x_np).cuda()
        ctx.layers(0, 2, xa)
        ref.layers(0, 2, xb)
        ctx.sync_status()
        ref.sync_status()
        assert np.array_equal(xa.cpu().numpy().view(np.uint32), xb.cpu().numpy().view(np.uint32))
        assert hp.n_ff_shexp == s.I and hp.norm_topk
    finally:
        ctx.close()
        ref.close()
        g.close()
