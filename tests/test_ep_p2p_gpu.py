"""Expert parallelism over NVLink peer memory (hoard_moe_p2p_*) on the GPU.

The send kernel stores each entry's row into its destination rank's receive region, the down-GEMM
epilogue stores each output row into its source rank's y_back, and bounded device barriers order the
steps. Every row's arithmetic is the single-rank tensor-core path's, so the layer must equal
hoard_moe_layers on one GPU bit for bit:
  * G ranks emulated as G contexts of one process on one GPU (hoard_moe_p2p_attach), the three steps
    issued rank by rank on one stream so that every wait finds its signals already written; pools
    holding only the rank's own experts and pools holding all of them; ranks with different T;
  * a wait that nobody signals: HOARD_ETIMEOUT after the bound, and the context stays usable;
  * two ranks on two GPUs (CUDA IPC handles all-gathered over NCCL) when the box has them.
"""
import os
import socket

import numpy as np
import pytest
import torch

from hoard_b200 import moe
from tests.moe_fixtures import LayerSpec, load_context, make_layer, make_x, Q4_K, Q6_K

pytestmark = pytest.mark.gpu

DEV = 0
SPECS = [LayerSpec(H=2048, E=32, k=8, I=768, types=(Q4_K, Q4_K, Q6_K)),
         LayerSpec(H=2048, E=32, k=8, I=768, types=(Q4_K, Q4_K, Q4_K))]
H, E, K = 2048, 32, 8
MAX_T = 640


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_ctx(n_slots, device=DEV):
    ctx = moe.MoEContext(n_embd=H, n_expert=E, n_expert_used=K, n_ff=768, n_layer=2, n_slots=n_slots,
                         norm_topk=True, eps=SPECS[0].eps, gate_types=[Q4_K, Q4_K], up_types=[Q4_K, Q4_K],
                         down_types=[s.types[2] for s in SPECS], max_tokens=MAX_T, device=device)
    ctx.set_gemm_min_tokens(1)
    ctx.set_decode_impl(0)
    return ctx


def load_rank(ctx, layers, g, epr, own_pool):
    for il, L in enumerate(layers):
        if own_pool:
            load_context(ctx, il, L, {e: e - g * epr for e in range(g * epr, min(E, (g + 1) * epr))})
        else:
            load_context(ctx, il, L)


@pytest.fixture(scope="module")
def setup():
    layers = [make_layer(s, seed=5201 + i) for i, s in enumerate(SPECS)]
    ref = make_ctx(E)
    load_rank(ref, layers, 0, E, False)
    yield layers, ref
    ref.close()


def reference(ref, x_np):
    x = torch.from_numpy(x_np).cuda(DEV)
    ref.layers(0, 2, x)
    ref.sync_status()
    return x.cpu().numpy()


@pytest.mark.parametrize("G,own_pool,Ts", [(1, False, [517]), (2, True, [640, 333]), (3, False, [200, 1, 611]),
                                           (4, True, [96, 640, 130, 257])])
def test_emulated_group_equals_local(setup, G, own_pool, Ts):
    layers, ref = setup
    epr = (E + G - 1) // G
    ctxs = []
    try:
        for g in range(G):
            c = make_ctx(epr if own_pool else E)
            load_rank(c, layers, g, epr, own_pool)
            c.p2p_init(G, g, epr, 0 if own_pool else g * epr)
            ctxs.append(c)
        for c in ctxs:
            c.p2p_attach(ctxs)
        x_np = [make_x(T, H, seed=60 + 7 * g + G) for g, T in enumerate(Ts)]
        xs = [torch.from_numpy(a).cuda(DEV) for a in x_np]
        sels = [torch.empty(2, T, K, dtype=torch.int32, device=xs[0].device) for T in Ts]
        for layer in range(2):
            for g in range(G):
                ctxs[g].p2p_send(layer, xs[g], sel_out=sels[g][layer])
            for g in range(G):
                ctxs[g].p2p_compute()
            for g in range(G):
                ctxs[g].p2p_finish(xs[g])
        for c in ctxs:
            c.sync_status()
        for g in range(G):
            want = reference(ref, x_np[g])
            assert np.array_equal(xs[g].cpu().numpy().view(np.uint32), want.view(np.uint32)), g
            assert ((sels[g] >= 0) & (sels[g] < E)).all()
    finally:
        for c in ctxs:
            c.close()


def test_steps_out_of_order_are_rejected(setup):
    layers, ref = setup
    c = make_ctx(E)
    try:
        x = torch.from_numpy(make_x(8, H, seed=3)).cuda(DEV)
        with pytest.raises(moe.HoardError) as ei:
            c.p2p_send(0, x)                               # not initialised
        assert ei.value.status == moe.HOARD_ESTATE
        c.p2p_init(1, 0, E, 0)
        with pytest.raises(moe.HoardError) as ei:
            c.p2p_send(0, x)                               # not connected
        assert ei.value.status == moe.HOARD_ESTATE
        c.p2p_attach([c])
        with pytest.raises(moe.HoardError) as ei:
            c.p2p_compute()                                # send first
        assert ei.value.status == moe.HOARD_ESTATE
        with pytest.raises(moe.HoardError) as ei:
            c.p2p_init(1, 0, E, 0)                         # twice
        assert ei.value.status == moe.HOARD_ESTATE
    finally:
        c.close()


def test_unsignalled_wait_times_out_and_context_stays_usable(setup):
    layers, ref = setup
    ctxs = [make_ctx(E), make_ctx(E)]
    try:
        for g, c in enumerate(ctxs):
            load_rank(c, layers, g, E // 2, False)
            c.p2p_init(2, g, E // 2, g * (E // 2))
        for c in ctxs:
            c.p2p_attach(ctxs)
        c0 = ctxs[0]
        c0.p2p_set_timeout(0.2)
        x = torch.from_numpy(make_x(64, H, seed=4)).cuda(DEV)
        c0.p2p_send(0, x)                                  # rank 1 never sends: the wait must give up
        c0.p2p_compute()
        c0.p2p_finish(x)
        with pytest.raises(moe.HoardError) as ei:
            c0.sync_status()
        assert ei.value.status == moe.HOARD_ETIMEOUT
        x_np = make_x(100, H, seed=5)                      # the context still computes correctly
        xl = torch.from_numpy(x_np).cuda(DEV)
        c0.layers(0, 2, xl)
        c0.sync_status()
        assert np.array_equal(xl.cpu().numpy().view(np.uint32), reference(ref, x_np).view(np.uint32))
    finally:
        for c in ctxs:
            c.close()


def _two_gpu_rank(rank, world, port, out_dir, Ts):
    import torch.distributed as dist
    from hoard_b200.ep import ExpertParallel
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        layers = [make_layer(s, seed=5201 + i) for i, s in enumerate(SPECS)]
        ctx = make_ctx(E, device=rank)
        load_rank(ctx, layers, rank, E, False)
        x_np = make_x(Ts[rank], H, seed=900 + rank)
        ref = torch.from_numpy(x_np).cuda(rank)
        ctx.layers(0, 2, ref)
        ctx.sync_status()
        x = torch.from_numpy(x_np).cuda(rank)
        ep = ExpertParallel(ctx, experts_per_rank=E // world, slot_base=rank * (E // world), transport="p2p")
        ep.layers(0, 2, x)
        ctx.sync_status()
        x2 = torch.from_numpy(x_np).cuda(rank)           # a second pass through the same buffers
        ep.layers(0, 2, x2)
        ctx.sync_status()
        np.savez(os.path.join(out_dir, f"p{rank}.npz"), ref=ref.cpu().numpy(), ep=x.cpu().numpy(),
                 ep2=x2.cpu().numpy())
        ep.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_p2p_equals_local(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_two_gpu_rank, args=(2, _free_port(), str(tmp_path), [512, 301]), nprocs=2, join=True)
    for r in range(2):
        d = np.load(tmp_path / f"p{r}.npz")
        assert np.array_equal(d["ep"].view(np.uint32), d["ref"].view(np.uint32)), r
        assert np.array_equal(d["ep2"].view(np.uint32), d["ref"].view(np.uint32)), r
