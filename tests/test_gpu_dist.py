"""The sharded layer on 2+ GPUs (one process per GPU, NCCL) against the
single-GPU layer on the same inputs: every rank's blocks agree within the
bf16 bar (2e-2); the two differ only in how the compact blocks are split
into KV tiles.  The host-buffer call must reproduce the device call bit for
bit.  The single-rank case runs the same code on one GPU; the others are
skipped on a box with fewer GPUs."""
from __future__ import annotations

import multiprocessing as pymp
import os
import random
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

NB, L, HQ, HKV, D = 4, 512, 8, 2, 128
BUDGETS = {(s, r): [64, 96, 128][(s + 2 * r) % 3] for r in range(NB) for s in range(r)}


def _worker(rank, world, port, errq):
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        import dcc_kv_b200 as dk
        from dcc_kv_b200.dist_layer import DistributedDccKvLayer
        from dcc_kv_b200.workloads import layer_inputs
        q, k, v = layer_inputs(NB, L, HQ, HKV, D, device="cpu", first_seed=11)
        from dcc_kv_b200.dist_layer import local_blocks_of
        mine = local_blocks_of(NB, world, rank)
        layer = DistributedDccKvLayer(NB, L, HQ, HKV, D, BUDGETS, window=128, device=dev)
        out = None
        for _ in range(2):  # second call reuses every buffer
            out = layer(q[mine].contiguous().to(dev), k[mine].contiguous().to(dev), v[mine].contiguous().to(dev))
        torch.cuda.synchronize()
        ref = dk.DccKvSyncLayer(NB, L, HQ, HKV, D, BUDGETS, window=128, device=dev)(q.to(dev), k.to(dev), v.to(dev))
        torch.cuda.synchronize()
        for li, b in enumerate(mine):
            err = ((out[li].float() - ref[b].float()).abs().max() / ref[b].float().abs().max()).item()
            assert err < 2e-2, f"block {b}: {err}"
        # host buffers: copies pipelined with the compute, same kernels, same
        # result; three calls alternating two inputs (consecutive calls use
        # alternate device staging sets and overlap one another)
        want = [out.cpu()]
        q2, k2, v2 = layer_inputs(NB, L, HQ, HKV, D, device="cpu", first_seed=29)
        want.append(layer(q2[mine].contiguous().to(dev), k2[mine].contiguous().to(dev),
                          v2[mine].contiguous().to(dev)).cpu())
        hosts = [tuple(t[mine].contiguous().pin_memory() for t in x) for x in ((q, k, v), (q2, k2, v2))]
        host_outs = [torch.empty(want[0].shape, dtype=want[0].dtype).pin_memory() for _ in range(3)]
        for c in range(3):
            layer(*hosts[c % 2], out=host_outs[c])
        torch.cuda.synchronize()
        for c in range(3):
            assert torch.equal(host_outs[c], want[c % 2]), c
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(traceback.format_exc())


@pytest.mark.parametrize("world", [1, 2])
def test_distributed_layer_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = pymp.get_context("spawn")
    errq = ctx.Queue()
    port = random.randint(20000, 40000)
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)


def _stack_worker(rank, world, port, errq):
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from dcc_kv_b200.dist_layer import DistributedDccKvLayer, DistributedDccKvStack
        from dcc_kv_b200.workloads import layer_inputs
        from dcc_kv_b200.dist_layer import local_blocks_of
        mine = local_blocks_of(NB, world, rank)
        inputs = []
        for seed in (11, 29, 47):
            q, k, v = layer_inputs(NB, L, HQ, HKV, D, device="cpu", first_seed=seed)
            inputs.append(tuple(t[mine].contiguous().to(dev) for t in (q, k, v)))
        layer = DistributedDccKvLayer(NB, L, HQ, HKV, D, BUDGETS, window=128, device=dev)
        want = [layer(*x).clone() for x in inputs]
        # no communication-computation overlap: same kernels, same outputs
        layer.overlap_exchange = False
        for x, w in zip(inputs, want):
            assert torch.equal(layer(*x), w)
        # exchange of layer l + 1 overlapped with the attention of layer l
        stack = DistributedDccKvStack(NB, L, HQ, HKV, D, BUDGETS, window=128, device=dev)
        for _ in range(2):  # second call reuses every buffer
            outs = stack(inputs)
            torch.cuda.synchronize()
            for li, (o, w) in enumerate(zip(outs, want)):
                assert torch.equal(o, w), f"layer {li}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(traceback.format_exc())


@pytest.mark.parametrize("world", [1, 2])
def test_layer_stack_double_buffered_exchange_matches_layer_by_layer(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = pymp.get_context("spawn")
    errq = ctx.Queue()
    port = random.randint(20000, 40000)
    procs = [ctx.Process(target=_stack_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)


def _help_worker(rank, world, port, errq):
    """One block per rank: part of the last blocks' compact attention is
    computed on their mirror's rank and merged back."""
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        import dcc_kv_b200 as dk
        from dcc_kv_b200.dist_layer import DistributedDccKvLayer, local_blocks_of
        from dcc_kv_b200.workloads import layer_inputs
        nb = world
        budgets = {(s, r): [64, 96, 128][(s + 2 * r) % 3] for r in range(nb) for s in range(r)}
        help_sources = {1: 1} if world == 2 else None  # 4 ranks: the default hand-off {3: 1}
        q, k, v = layer_inputs(nb, L, HQ, HKV, D, device="cpu", first_seed=13)
        mine = local_blocks_of(nb, world, rank)
        layer = DistributedDccKvLayer(nb, L, HQ, HKV, D, budgets, window=128, device=dev, help_sources=help_sources)
        assert layer.plan.help, "no hand-off configured"
        out = None
        for _ in range(2):
            out = layer(q[mine].contiguous().to(dev), k[mine].contiguous().to(dev), v[mine].contiguous().to(dev))
        torch.cuda.synchronize()
        ref = dk.DccKvSyncLayer(nb, L, HQ, HKV, D, budgets, window=128, device=dev)(q.to(dev), k.to(dev), v.to(dev))
        torch.cuda.synchronize()
        for li, b in enumerate(mine):
            err = ((out[li].float() - ref[b].float()).abs().max() / ref[b].float().abs().max()).item()
            assert err < 2e-2, f"block {b}: {err}"
        want = out.cpu()
        hosts = tuple(t[mine].contiguous().pin_memory() for t in (q, k, v))
        host_outs = [torch.empty(want.shape, dtype=want.dtype).pin_memory() for _ in range(2)]
        for c in range(2):
            layer(*hosts, out=host_outs[c])
        torch.cuda.synchronize()
        for c in range(2):
            assert torch.equal(host_outs[c], want), c
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(traceback.format_exc())


@pytest.mark.parametrize("world", [2, 4])
def test_compact_attention_handed_to_mirror_rank(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = pymp.get_context("spawn")
    errq = ctx.Queue()
    port = random.randint(20000, 40000)
    procs = [ctx.Process(target=_help_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)


def _ring_worker(rank, world, port, errq):
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from dcc_kv_b200 import baselines as bl
        g = torch.Generator().manual_seed(5)
        T, d = 256 * world, 128
        q, k, v = (torch.randn(T, d, generator=g).to(torch.bfloat16) for _ in range(3))
        c = T // world
        lo, hi = rank * c, (rank + 1) * c
        for causal in (True, False):
            got = bl.dist_ring_attention(q[lo:hi].to(dev), k[lo:hi].to(dev), v[lo:hi].to(dev), causal=causal)
            want = bl.ring_attention(q.to(dev), [k.to(dev)], [v.to(dev)], causal=causal)[lo:hi]
            torch.cuda.synchronize()
            err = ((got.float() - want.float()).abs().max() / want.float().abs().max()).item()
            assert err < 2e-2, f"rank {rank} causal {causal}: {err}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(traceback.format_exc())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ring_attention_over_nccl_matches_single_gpu():
    world = 2
    ctx = pymp.get_context("spawn")
    errq = ctx.Queue()
    port = random.randint(20000, 40000)
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)
