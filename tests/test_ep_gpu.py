"""Expert parallelism on the GPU through the C ABI (hoard_moe_ep_pack / _experts / _combine).

Every row's arithmetic is independent of the rows it shares a tile with and the outputs travel in the
same f16 form the single-rank path stores, so the expert-parallel layer must equal the single-rank
tensor-core layer bit for bit:
  * one rank over a real NCCL process group (all-to-all of one rank);
  * four destination ranks emulated in one process (each destination's rows through ep_experts
    separately), which exercises the pack's partition on one GPU;
  * two ranks on two GPUs (NCCL all-to-all over NVLink) when the box has them.
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
SPEC = LayerSpec(H=2048, E=32, k=8, I=768, types=(Q4_K, Q4_K, Q6_K))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_ctx(max_tokens, device=DEV):
    ctx = moe.MoEContext(n_embd=SPEC.H, n_expert=SPEC.E, n_expert_used=SPEC.k, n_ff=SPEC.I, n_layer=1,
                         norm_topk=True, eps=SPEC.eps, gate_types=[SPEC.types[0]], up_types=[SPEC.types[1]],
                         down_types=[SPEC.types[2]], max_tokens=max_tokens, device=device)
    ctx.set_gemm_min_tokens(1)
    ctx.set_decode_impl(0)
    return ctx


@pytest.fixture(scope="module")
def layer_ctx():
    L = make_layer(SPEC, seed=4101)
    ctx = make_ctx(1024)
    load_context(ctx, 0, L)
    ctx.ep_reserve(1024 * SPEC.k)
    yield L, ctx
    ctx.close()


def local_layer(ctx, x_np):
    x = torch.from_numpy(x_np).cuda(DEV)
    ctx.layer(0, x)
    ctx.sync_status()
    return x.cpu().numpy()


def test_pack_partitions_entries(layer_ctx):
    L, ctx = layer_ctx
    T, G = 300, 4
    x = torch.from_numpy(make_x(T, SPEC.H, seed=11)).cuda(DEV)
    sel, w = ctx.route(0, x)
    counts, pos, expert, rows = ctx.ep_pack(0, sel, G, SPEC.E // G)
    ctx.sync_status()
    c, p, ex = counts.cpu().numpy(), pos.cpu().numpy(), expert.cpu().numpy()
    assert c.sum() == T * SPEC.k
    assert np.array_equal(np.sort(p), np.arange(T * SPEC.k))
    starts = np.concatenate([[0], np.cumsum(c)])
    for r in range(G):
        assert (ex[starts[r]:starts[r + 1]] // (SPEC.E // G) == r).all()
    assert np.array_equal(ex[p], sel.cpu().numpy().reshape(-1))
    # the k send rows of a token are copies of its Q8_K row
    by_entry = rows.float().cpu().numpy()[p].reshape(T, SPEC.k, SPEC.H)
    assert (by_entry == by_entry[:, :1]).all()


@pytest.mark.parametrize("G", [1, 4])
def test_emulated_ranks_equal_local_layer(layer_ctx, G):
    L, ctx = layer_ctx
    T = 517
    x_np = make_x(T, SPEC.H, seed=12 + G)
    ref = local_layer(ctx, x_np)
    x = torch.from_numpy(x_np).cuda(DEV)
    sel, w = ctx.route(0, x)
    counts, pos, expert, rows = ctx.ep_pack(0, sel, G, SPEC.E // G)
    c = counts.cpu().tolist()
    y_back = torch.empty(T * SPEC.k, SPEC.H, dtype=torch.float16, device=x.device)
    off = 0
    for r in range(G):             # destination r's rows through its own ep_experts call
        if c[r]:
            y_back[off:off + c[r]] = ctx.ep_experts(0, rows[off:off + c[r]], expert[off:off + c[r]])
        off += c[r]
    ctx.ep_combine(w, pos, y_back, x)
    ctx.sync_status()
    assert np.array_equal(x.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("chunks", [1, 3])
def test_single_rank_process_group_equals_local_layer(layer_ctx, chunks):
    import torch.distributed as dist
    from hoard_b200.ep import ExpertParallel
    L, ctx = layer_ctx
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            device_id=torch.device("cuda", DEV))
    try:
        T = 640
        x_np = make_x(T, SPEC.H, seed=31)
        ref = local_layer(ctx, x_np)
        x = torch.from_numpy(x_np).cuda(DEV)
        ep = ExpertParallel(ctx, experts_per_rank=SPEC.E, slot_base=0, chunks=chunks)
        ep.layers(0, 1, x)
        ctx.sync_status()
        assert np.array_equal(x.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ctas", [1, 37, 132])
def test_reduced_gemm_grid_is_bit_exact(layer_ctx, ctas):
    """The tensor-core GEMMs on fewer CTAs than SMs (room for a concurrent all-to-all) compute the same
    rows: the work list is strided over whatever grid runs it."""
    L, ctx = layer_ctx
    x_np = make_x(700, SPEC.H, seed=32)
    ref = local_layer(ctx, x_np)
    ctx.set_gemm_ctas(ctas)
    try:
        got = local_layer(ctx, x_np)
    finally:
        ctx.set_gemm_ctas(0)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_ep_reserve_bounds_received_rows(layer_ctx):
    L, ctx = layer_ctx
    rows = torch.zeros(1024 * SPEC.k + 1, SPEC.H, dtype=torch.float16, device=f"cuda:{DEV}")
    slots = torch.zeros(rows.shape[0], dtype=torch.int32, device=rows.device)
    with pytest.raises(moe.HoardError) as ei:
        ctx.ep_experts(0, rows, slots)
    assert ei.value.status == moe.HOARD_EINVAL


def _two_gpu_rank(rank, world, port, out_dir, chunks=1):
    import torch.distributed as dist
    from hoard_b200.ep import ExpertParallel
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        L = make_layer(SPEC, seed=4101)
        ctx = make_ctx(512, device=rank)
        load_context(ctx, 0, L)
        x_np = make_x(512, SPEC.H, seed=900 + rank)
        ref = torch.from_numpy(x_np).cuda(rank)
        ctx.layer(0, ref)
        ctx.sync_status()
        x = torch.from_numpy(x_np).cuda(rank)
        ep = ExpertParallel(ctx, experts_per_rank=SPEC.E // world, slot_base=rank * (SPEC.E // world),
                            max_rows=512 * SPEC.k * world, chunks=chunks)
        if chunks > 1:
            ctx.set_gemm_ctas(132)
        ep.layers(0, 1, x)
        ctx.sync_status()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ref=ref.cpu().numpy(), ep=x.cpu().numpy(),
                 recv=ep.last_recv_rows)
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("chunks", [1, 2])
def test_two_gpus_equal_local_layer(tmp_path, chunks):
    import torch.multiprocessing as mp
    mp.spawn(_two_gpu_rank, args=(2, _free_port(), str(tmp_path), chunks), nprocs=2, join=True)
    recv = 0
    for r in range(2):
        d = np.load(tmp_path / f"r{r}.npz")
        assert np.array_equal(d["ep"].view(np.uint32), d["ref"].view(np.uint32)), r
        recv += int(d["recv"])
    assert recv == 2 * 512 * SPEC.k
