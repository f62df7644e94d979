"""Expert parallelism on gloo ranks (CPU): the orchestration of hoard_b200.ep.ExpertParallel (pack
counts, split sizes, the send-order map, combine order) over 2 and 3 ranks reproduces the single-process
layer bit for bit. The kernels are numpy stand-ins (tests/ep_fake.py); the GPU kernels are tested
against the single-rank path in tests/test_ep_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.moe_fixtures import LayerSpec, make_layer, make_x, Q4_K, Q6_K

SPEC = LayerSpec(H=256, E=8, k=3, I=256, types=(Q4_K, Q4_K, Q6_K))
T_RANK = 9


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, chunks=1):
    import torch.distributed as dist
    from hoard_b200.ep import ExpertParallel
    from tests.ep_fake import FakeContext
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        L = make_layer(SPEC, seed=77)
        ctx = FakeContext(L, shuffle_seed=rank + 1)
        x = torch.from_numpy(make_x(T_RANK, SPEC.H, seed=200 + rank))
        epr = (SPEC.E + world - 1) // world
        ep = ExpertParallel(ctx, experts_per_rank=epr, slot_base=rank * epr, chunks=chunks)
        if chunks > 1:
            sel, w = ctx.route(0, x.clone())
            out = ep.layer_pipelined(0, x)
        else:
            out, sel, w = ep.layer(0, x)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out.numpy(), sel=sel.numpy(), w=w.numpy(),
                 recv=ep.last_recv_rows)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,chunks", [(2, 1), (3, 1), (2, 3)])
def test_expert_parallel_equals_single_process(tmp_path, world, chunks):
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path), chunks), nprocs=world, join=True)
    from tests.ep_fake import FakeContext
    L = make_layer(SPEC, seed=77)
    total_recv = 0
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npz")
        ref_ctx = FakeContext(L)
        x = torch.from_numpy(make_x(T_RANK, SPEC.H, seed=200 + rank))
        ref, sel, w = ref_ctx.reference_layer(x)
        assert np.array_equal(got["sel"], sel.numpy())
        assert np.array_equal(got["out"].view(np.uint32), ref.numpy().view(np.uint32)), rank
        total_recv += int(got["recv"])
    assert total_recv == world * T_RANK * SPEC.k      # every entry went to exactly one rank


def test_pack_partitions_entries_by_rank():
    from tests.ep_fake import FakeContext
    L = make_layer(SPEC, seed=78)
    ctx = FakeContext(L, shuffle_seed=3)
    x = torch.from_numpy(make_x(T_RANK, SPEC.H, seed=5))
    sel, w = ctx.route(0, x)
    counts, pos, expert, rows = ctx.ep_pack(0, sel, 3, 3)
    c, p, ex = counts.numpy(), pos.numpy(), expert.numpy()
    assert c.sum() == T_RANK * SPEC.k
    assert sorted(p.tolist()) == list(range(T_RANK * SPEC.k))          # a permutation
    starts = np.concatenate([[0], np.cumsum(c)])
    for r in range(3):
        assert (ex[starts[r]:starts[r + 1]] // 3 == r).all()           # rank r's run holds its experts
    assert np.array_equal(ex[p], sel.numpy().reshape(-1))


class _HandleStub:
    """Records what ExpertParallel(transport="p2p") hands the context: init arguments, the gathered
    peer handles (rank order) and the close."""
    E = SPEC.E

    def __init__(self):
        self.init_args = None
        self.opened = None
        self.closed = False

    def p2p_init(self, n_ranks, rank, experts_per_rank, slot_base):
        self.init_args = (n_ranks, rank, experts_per_rank, slot_base)

    def p2p_handle(self):
        return bytes([self.init_args[1]] * 8 + [0xA5] * 120)

    def p2p_open(self, handles):
        self.opened = handles

    def p2p_close(self):
        self.closed = True


def _p2p_handles_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from hoard_b200.ep import ExpertParallel
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ctx = _HandleStub()
        ep = ExpertParallel(ctx, transport="p2p", slot_base=0)
        ep.close()
        np.savez(os.path.join(out_dir, f"h{rank}.npz"), init=np.array(ctx.init_args),
                 opened=np.frombuffer(b"".join(ctx.opened), np.uint8), closed=ctx.closed)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_p2p_transport_exchanges_handles_in_rank_order(tmp_path, world):
    mp.spawn(_p2p_handles_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    epr = (SPEC.E + world - 1) // world
    for rank in range(world):
        d = np.load(tmp_path / f"h{rank}.npz")
        assert tuple(d["init"]) == (world, rank, epr, 0)
        opened = d["opened"].reshape(world, 128)
        for s in range(world):
            assert (opened[s, :8] == s).all() and (opened[s, 8:] == 0xA5).all()
        assert bool(d["closed"])
