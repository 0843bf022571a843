"""Host logic of the sharded layer and the communication layer, on CPU:
the routing plan (every edge sent once, received where the destination
reads it), a real gloo all-to-allv of byte buffers laid out by the plan
(world sizes 2 and 4), DistributedComm in mock and gloo modes, and the
var-len codec (the reference's tests/test_var_len_msg.py and
tests/test_smoke.py restated)."""
from __future__ import annotations

import multiprocessing as pymp
import random

import pytest
import torch

from dcc_kv_b200.comm import DistributedComm, VarLenMessage
from dcc_kv_b200.dist_layer import DistPlan
from dcc_kv_b200.var_len_msg import (EdgeLayout, mock_all_to_allv, pack_var_len_messages,
                                     unpack_var_len_messages)

import dist_workers


def _spawn(target, world, *args):
    ctx = pymp.get_context("spawn")
    errq = ctx.Queue()
    port = random.randint(20000, 40000)
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (errq,)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_routes_every_edge_once(world):
    """Every (edge, KV head) unit is written once on its source's rank and
    read once on the rank that attends with it; the heads of one edge that
    a rank reads are contiguous (one KV segment)."""
    budgets = {(s, r): [256, 512, 1024, 2048][(s * 3 + r) % 4] for r in range(8) for s in range(r)}
    plan = DistPlan(8, world, 16384, 8, 128, budgets)
    units = {(s, r, g) for (s, r) in budgets for g in range(8)}
    sent, received = {}, {}
    for rank in range(world):
        for u, loc in plan.send_offsets(rank).items():
            assert plan.owner(u[0]) == rank and u not in sent
            sent[u] = (rank, loc)
        recv = plan.recv_offsets(rank)
        for u, loc in recv.items():
            assert plan.consumer(u) == rank and u not in received
            received[u] = (rank, loc)
        # byte ranges of one buffer never overlap
        for offsets in (plan.send_offsets(rank), recv):
            spans = sorted((buf, off, off + plan.layout[(u[0], u[1])].head_bytes) for u, (buf, off) in offsets.items())
            for a, b in zip(spans, spans[1:]):
                assert a[0] != b[0] or a[2] <= b[1]
        for e in budgets:
            lo, hi = plan.heads_on(rank, e)
            for g in range(lo + 1, hi):
                buf, off = recv[(e[0], e[1], g)]
                assert recv[(e[0], e[1], g - 1)] == (buf, off - plan.layout[e].head_bytes)
    assert set(sent) == set(received) == units
    for i in range(world):
        for j in range(world):
            assert plan.send_splits(i)[j] == plan.recv_splits(j)[i]
    # every block sits on exactly one rank, and the local index is its
    # position among the rank's blocks
    assert sorted(b for r in range(world) for b in plan.local_blocks(r)) == list(range(8))
    for b in range(8):
        assert plan.local_blocks(plan.owner(b))[plan.local_index(b)] == b


@pytest.mark.parametrize("world", [1, 2, 4])
def test_snake_mapping_balances_compact_and_build_work(world):
    """Block r attends to r compact blocks and block s builds 7 - s edges:
    with 8 blocks on 1, 2 or 4 ranks the snake order gives every rank the
    same amount of both (on 8 ranks each rank holds one block)."""
    from dcc_kv_b200.dist_layer import local_blocks_of
    parts = [local_blocks_of(8, world, r) for r in range(world)]
    assert sorted(b for p in parts for b in p) == list(range(8))
    assert len({sum(p) for p in parts}) == 1
    assert len({sum(7 - b for b in p) for p in parts}) == 1


def test_plan_hands_kv_heads_of_heavy_blocks_to_their_mirror():
    """One block per rank (the 128K layer on 8 GPUs): the cost model hands
    the compact attention of the first 3 / 2 / 1 KV heads of blocks 7 / 6 /
    5 to the ranks of their mirrors 0 / 1 / 2, which evens out the
    estimated per-rank work (local attention, builds, compact attention and
    the hand-off transfers)."""
    plan = DistPlan(8, 8, 16384, 8, 128, 1024)
    assert plan.help == {7: 3, 6: 2, 5: 1}
    assert plan.helped_by(0) == [7] and plan.helped_by(1) == [6] and plan.helped_by(7) == []
    assert plan.consumer((2, 7, 2)) == 0 and plan.consumer((2, 7, 3)) == 7
    assert plan.heads_on(0, (4, 7)) == (0, 3) and plan.heads_on(7, (4, 7)) == (3, 8)
    assert plan.heads_on(3, (4, 7)) == (0, 0)
    # several blocks per rank: no hand-off; a forced one is refused
    assert DistPlan(8, 4, 16384, 8, 128, 1024).help == {}
    with pytest.raises(ValueError):
        DistPlan(8, 4, 16384, 8, 128, 1024, help_heads={7: 2})
    with pytest.raises(ValueError):
        DistPlan(8, 8, 16384, 8, 128, 1024, help_heads={7: 8})  # all heads: nothing left on the owner
    # the 1M layer (variable budgets): block 7 only; a small layer: none (the transfers would
    # cost more than they save)
    from dcc_kv_b200.workloads import variable_budgets
    assert DistPlan(8, 8, 131072, 8, 128, variable_budgets(8)).help == {7: 3}
    assert DistPlan(4, 4, 512, 2, 128, 96).help == {}
    # a forced hand-off on two ranks (the 2-GPU test's setting)
    plan2 = DistPlan(2, 2, 512, 2, 128, 64, help_heads={1: 1})
    assert plan2.consumer((0, 1, 0)) == 0 and plan2.consumer((0, 1, 1)) == 1 and plan2.helped_by(0) == [1]


def test_plan_rejects_uneven_split():
    with pytest.raises(ValueError):
        DistPlan(8, 3, 128, 2, 16, 64)


def test_edge_layout_alignment():
    """KV-head-major blocks: every head starts 256-byte aligned, its keys,
    values and bias 16-byte aligned, and a run of heads is one byte range."""
    for rows in (1, 45, 64, 1024):
        lay = EdgeLayout(3, rows, 128, 2)
        assert lay.head_bytes % 256 == 0 and lay.nbytes == 3 * lay.head_bytes
        assert lay.values_off % 16 == 0 and lay.bias_off % 16 == 0
        buf = torch.zeros(lay.nbytes * 2, dtype=torch.uint8)
        k, v, b = lay.views(buf, lay.nbytes, torch.bfloat16)
        assert k.shape == (3, rows, 128) and b.shape == (3, rows)
        k[2].fill_(1.0)
        v[1].fill_(2.0)
        b[0].fill_(3.0)
        k1, v1, b1 = lay.views(buf, lay.nbytes + lay.head_bytes, torch.bfloat16, n_heads=2)
        assert torch.all(k1[1] == 1.0) and torch.all(v1[0] == 2.0) and torch.all(b1 == 0.0)
        with pytest.raises(ValueError):
            lay.views(buf, 128, torch.bfloat16)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gloo_exchange_by_plan(world):
    """8 ranks: one block per rank, so the plan also hands KV heads of
    blocks 5-7 to their mirrors' ranks (unit routing and the point-to-point
    transfers of queries and partial states)."""
    budgets = {(s, r): [17, 64, 100][(s + r) % 3] for r in range(8) for s in range(r)}
    _spawn(dist_workers.exchange_worker, world, 8, budgets)


def test_gloo_distributed_comm_all_to_all_v():
    _spawn(dist_workers.comm_worker, 2)


# ---- DistributedComm, mock mode and errors (reference tests/test_smoke.py:67-157, :306-340)
def test_comm_mock_lifecycle_and_shapes():
    comm = DistributedComm(backend="gloo", mock=True)
    assert not comm.initialized
    comm.init(rank=0, world_size=2)
    assert comm.initialized and comm.rank == 0 and comm.world_size == 2
    recv = comm.all_to_all_single(torch.tensor([1.0, 2.0, 3.0, 4.0]), send_counts=[2, 2], recv_counts=[2, 2])
    assert recv.shape == (4,) and torch.all(recv == 0)
    msgs = [VarLenMessage(payload=torch.tensor([1.0, 2.0])), VarLenMessage(payload=torch.tensor([3.0, 4.0, 5.0]))]
    res = comm.all_to_all_v(msgs, send_sizes=[2, 3], recv_sizes=[3, 2])
    assert [r.payload.shape for r in res] == [(3,), (2,)]
    assert res[0].metadata["src_rank"] == 0 and res[1].metadata["src_rank"] == 1
    t = torch.tensor([1.0])
    assert torch.equal(comm.all_reduce(t), t)
    comm.cleanup()
    assert not comm.initialized


def test_comm_errors():
    with pytest.raises(ValueError):
        DistributedComm(backend="tcp")
    comm = DistributedComm(mock=True)
    with pytest.raises(RuntimeError):
        comm.all_to_all_v([], recv_sizes=[])
    comm.init(0, 2)
    with pytest.raises(ValueError):
        comm.all_to_all_v([VarLenMessage(torch.zeros(1))], recv_sizes=[1, 1])
    with pytest.raises(ValueError):
        comm.all_to_all_v([VarLenMessage(torch.zeros(1))] * 2, recv_sizes=None)
    with pytest.raises(ValueError):
        comm.all_to_all_v([VarLenMessage(torch.zeros(1))] * 2, send_sizes=[2, 1], recv_sizes=[1, 1])
    with pytest.raises(ValueError):
        comm.all_to_all_single(torch.zeros(5), send_counts=[2, 2])
    real = DistributedComm(backend="gloo", mock=False)
    with pytest.raises(RuntimeError):
        real.init(0, 2)  # torch.distributed not initialised


# ---- var-len codec (reference tests/test_var_len_msg.py:23-97)
def test_var_len_round_trips():
    msgs = [torch.tensor([1.0, 2.0]), torch.tensor([3.0]), torch.tensor([4.0, 5.0, 6.0])]
    packed, offsets = pack_var_len_messages(msgs, [2, 1, 3])
    assert packed.shape == (6,) and offsets == [0, 2, 3, 6]
    for a, b in zip(msgs, unpack_var_len_messages(packed, [2, 1, 3])):
        assert torch.equal(a, b)
    msgs2 = [torch.randn(2, 64), torch.randn(3, 64), torch.randn(5, 64)]
    packed2, offsets2 = pack_var_len_messages(msgs2, [2, 3, 5])
    assert packed2.shape == (10, 64) and offsets2 == [0, 2, 5, 10]
    with pytest.raises(AssertionError):
        pack_var_len_messages([torch.tensor([1.0, 2.0]), torch.tensor([3.0])], sizes=[2, 3])


def test_mock_all_to_allv_two_ranks():
    m00, m01 = torch.tensor([1.0, 2.0]), torch.tensor([10.0, 11.0, 12.0])
    m10, m11 = torch.tensor([100.0, 101.0, 102.0]), torch.tensor([200.0, 201.0])
    p0, _ = pack_var_len_messages([m00, m01], [2, 3])
    p1, _ = pack_var_len_messages([m10, m11], [3, 2])
    r0 = mock_all_to_allv(0, 2, [m00, m01], [2, 3], {1: (p1, [3, 2])})
    r1 = mock_all_to_allv(1, 2, [m10, m11], [3, 2], {0: (p0, [2, 3])})
    assert torch.equal(r0[0], m00) and torch.equal(r0[1], m10)
    assert torch.equal(r1[0], m01) and torch.equal(r1[1], m11)
    with pytest.raises(ValueError):
        mock_all_to_allv(0, 2, [m00, m01], [2, 3], {})
