"""Worker functions for the multi-process (gloo, CPU) tests; a module of its
own so spawned children can import them."""
from __future__ import annotations

import os
import traceback

import torch
import torch.distributed as dist


def _init(rank: int, world: int, port: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _pattern(unit, nbytes: int) -> torch.Tensor:
    s, r, g = unit
    return ((torch.arange(nbytes, dtype=torch.int64) * 7 + 31 * s + 131 * r + 17 * g) % 251).to(torch.uint8)


def exchange_worker(rank: int, world: int, port: int, n_blocks: int, budgets, errq) -> None:
    """Fill the send/local buffers per DistPlan, exchange with the plan's
    splits, check every incoming (edge, KV head) unit lands where
    recv_offsets says."""
    try:
        from dcc_kv_b200.dist_layer import DistPlan
        _init(rank, world, port)
        plan = DistPlan(n_blocks, world, 512, 2, 16, budgets,
                        help_heads={7: 1, 6: 1, 5: 1} if world == n_blocks else None)
        send = torch.zeros(max(sum(plan.send_splits(rank)), 1), dtype=torch.uint8)
        local = torch.zeros(max(plan.bytes_ij[(rank, rank)], 1), dtype=torch.uint8)
        bufs = {"send": send, "local": local}
        for u, (buf, off) in plan.send_offsets(rank).items():
            n = plan.layout[(u[0], u[1])].head_bytes
            bufs[buf][off:off + n] = _pattern(u, n)
        recv = torch.zeros(max(sum(plan.recv_splits(rank)), 1), dtype=torch.uint8)
        ss, rs = plan.send_splits(rank), plan.recv_splits(rank)
        dist.all_to_all_single(recv[:sum(rs)], send[:sum(ss)], output_split_sizes=rs, input_split_sizes=ss)
        bufs["recv"] = recv
        for u, (buf, off) in plan.recv_offsets(rank).items():
            n = plan.layout[(u[0], u[1])].head_bytes
            assert plan.consumer(u) == rank
            if not torch.equal(bufs[buf][off:off + n], _pattern(u, n)):
                raise AssertionError(f"rank {rank}: unit {u} wrong at {buf}+{off}")
        # the compact-attention hand-off (one block per rank), in the layer's
        # order: helped blocks' queries to their helpers, then each helper's
        # partial state back to the helped block's rank
        mine = plan.local_blocks(rank)
        helped = [r for r in mine if r in plan.help]
        helping = plan.helped_by(rank)
        q_in = {r: torch.zeros(64) for r in helping}
        ops = [dist.P2POp(dist.isend, torch.full((64,), float(r)), plan.helper(r)) for r in helped]
        ops += [dist.P2POp(dist.irecv, q_in[r], plan.owner(r)) for r in helping]
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for r in helping:
            assert torch.equal(q_in[r], torch.full((64,), float(r))), f"rank {rank}: queries of block {r}"
        part_in = {r: torch.zeros(32) for r in helped}
        ops = [dist.P2POp(dist.isend, torch.full((32,), 1000.0 + r), plan.owner(r)) for r in helping]
        ops += [dist.P2POp(dist.irecv, part_in[r], plan.helper(r)) for r in helped]
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for r in helped:
            assert torch.equal(part_in[r], torch.full((32,), 1000.0 + r)), f"rank {rank}: partial of block {r}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(traceback.format_exc())


def comm_worker(rank: int, world: int, port: int, errq) -> None:
    """DistributedComm.all_to_all_v contents over gloo (reference
    tests/test_smoke.py:237-285 restated)."""
    try:
        from dcc_kv_b200.comm import DistributedComm, VarLenMessage
        _init(rank, world, port)
        comm = DistributedComm(backend="gloo")
        comm.init(rank, world)
        # rank i sends (i + 1) * (j + 1) rows of value 100 * i + j to rank j
        msgs = [VarLenMessage(payload=torch.full(((rank + 1) * (j + 1), 3), float(100 * rank + j)))
                for j in range(world)]
        recv_sizes = [(i + 1) * (rank + 1) for i in range(world)]
        for trust in (False, True):
            out = comm.all_to_all_v(msgs, recv_sizes=recv_sizes, trust_recv_sizes=trust)
            for i, m in enumerate(out):
                assert m.metadata["src_rank"] == i
                assert m.payload.shape == (recv_sizes[i], 3)
                assert torch.all(m.payload == float(100 * i + rank))
        # the layer's form: payloads as views of one packed send buffer, sizes
        # trusted, received into a caller buffer
        packed = torch.cat([m.payload for m in msgs])
        offs = [sum(m.numel() for m in msgs[:j]) for j in range(world)]
        views = [VarLenMessage(payload=packed[o:o + m.numel()]) for o, m in zip(offs, msgs)]
        recv = torch.full((sum(recv_sizes), 3), -1.0)
        out = comm.all_to_all_v(views, recv_sizes=recv_sizes, trust_recv_sizes=True, out=recv, packed=packed)
        for i, m in enumerate(out):
            assert m.payload.data_ptr() == recv[sum(recv_sizes[:i]):].data_ptr()
            assert torch.all(m.payload == float(100 * i + rank))
        # the same exchange on an explicit process group (the layer passes its own)
        sub = dist.new_group(ranks=list(range(world)))
        gcomm = DistributedComm(backend="gloo", group=sub)
        gcomm.init(rank, world)
        out = gcomm.all_to_all_v(msgs, recv_sizes=recv_sizes, trust_recv_sizes=True)
        for i, m in enumerate(out):
            assert torch.all(m.payload == float(100 * i + rank))
        t = torch.tensor([float(rank + 1)])
        assert gcomm.all_reduce(t.clone()).item() == sum(range(1, world + 1))
        assert comm.all_reduce(t).item() == sum(range(1, world + 1))
        g = comm.gather(torch.tensor([rank]), dst=0)
        if rank == 0:
            assert [x.item() for x in g] == list(range(world))
        comm.barrier()
        comm.cleanup()
        dist.destroy_process_group()
    except Exception:
        errq.put(traceback.format_exc())
