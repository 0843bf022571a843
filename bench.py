"""DCC-KV layer prefill benchmark: tokens/s of the full 128K-context layer.

Workload: 131072 tokens as 8 blocks of 16384, 32 query / 8 KV heads,
head_dim 128, bf16, compact budget 1024 per (source, destination) edge,
destination window 2048 queries per query head, M = 64 representative
queries, d_p = 32.  A step is one forward of the layer over the whole
context: pooling + 28 x 8 compact builds + local causal attention +
compact attention with logit bias + online-softmax merge.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

N = 1 runs the 8 logical blocks on one GPU.  ``--impl reference`` times the
FP64 CPU oracle (a restatement of the reference path) on a bounded sample
of the same workload and extrapolates to the full layer.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_BLOCKS, BLOCK_LEN, HQ, HKV, D = 8, 16384, 32, 8, 128
BUDGET, WINDOW, M_REPR, DP = 1024, 2048, 64, 32
TOKENS = N_BLOCKS * BLOCK_LEN
METRIC = "DCC-KV layer prefill tokens/s at 128K ctx"
WORKLOAD = {"workload": "dcc_kv_sync_layer_128k", "context_tokens": TOKENS, "blocks": N_BLOCKS,
            "block_len": BLOCK_LEN, "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "budget": BUDGET,
            "window": WINDOW, "repr_queries": M_REPR, "projection_dim": DP,
            "l2": "inputs larger than L2 (q 1 GiB, k/v 256 MiB each)"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


def causal_attention_flops():
    """Algorithmic FLOPs of one step's attention: local causal (L(L+1)/2 pairs
    per head and block) and compact (block r sees r * BUDGET keys), 4 d per pair."""
    local = N_BLOCKS * HQ * (BLOCK_LEN * (BLOCK_LEN + 1) // 2) * 4 * D
    compact = sum(HQ * BLOCK_LEN * r * BUDGET * 4 * D for r in range(N_BLOCKS))
    return local, compact


def attention_bytes(blocks_compact_rows):
    """Algorithmic HBM bytes of one attention launch over the given blocks:
    (read, write).  Per block: Q, local K and V read once, its compact K, V
    (bf16) and bias (fp32) read once, O written once."""
    read = write = 0
    for rows in blocks_compact_rows:
        read += (HQ + 2 * HKV) * BLOCK_LEN * D * 2 + HKV * rows * (2 * D * 2 + 4)
        write += HQ * BLOCK_LEN * D * 2
    return read, write


# DRAM bytes of one ncu capture of the --profile-attention launch (the last
# destination block: 16384 causal keys + 7 x 1024 compact keys per KV head):
# dram__bytes_read.sum / dram__bytes_write.sum.  Its reads are 1.001 x the
# algorithmic read bytes (no re-reads past L2).  Its writes are lower than the
# output size because the tail of the output is still in L2 when the launch
# ends; a full launch writes ~1 GiB, far beyond L2, so its writes are taken
# at the algorithmic figure.
PROFILED_DRAM_READ = 231_221_248


def attention_traffic():
    """Estimated DRAM bytes of the full single-GPU attention launch: reads
    scaled from the profiled block by algorithmic read bytes, writes at the
    algorithmic output size."""
    prof_read, _ = attention_bytes([7 * BUDGET])
    read, write = attention_bytes([r * BUDGET for r in range(N_BLOCKS)])
    return int(read * PROFILED_DRAM_READ / prof_read + write)


class ClockSampler:
    """SM clock and clock-event reasons of this GPU, read through NVML every
    millisecond on a host thread for the whole timed region (read-only
    queries; falls back to nvidia-smi at 200 ms when NVML is unavailable)."""

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.max_mhz = None
        self.thread = None
        self.stop = None
        self.proc = None
        self.path = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.index).uuid)
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.stop = threading.Event()

            def run():
                while not self.stop.is_set():
                    try:
                        mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.rows.append((float(mhz), int(mask)))
                    except Exception:
                        pass
                    self.stop.wait(0.001)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            except OSError:
                self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.thread is not None:
            if not self.rows:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "source": "nvml"}
            reasons = sorted({name for _, mask in self.rows for bit, name in self.REASONS.items() if mask & bit})
            return {"sm_mhz": statistics.median(m for m, _ in self.rows), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.rows), "source": "nvml"}
        rows = []
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except (OSError, TypeError):
            pass
        finally:
            if self.path:
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the FP64 oracle on a bounded sample
# ---------------------------------------------------------------------------
_CPU_INPUTS = None


def _cpu_inputs():
    """Block 0 (source) and the destination window of block 1, drawn once."""
    global _CPU_INPUTS
    if _CPU_INPUTS is None:
        import numpy as np
        from dcc_kv_b200.workloads import gqa_block
        q, k, v = gqa_block(HQ, HKV, BLOCK_LEN, D, seed=1000, device="cpu")
        q1, _, _ = gqa_block(HQ, HKV, BLOCK_LEN, D, seed=1001, device="cpu")
        dq = np.concatenate([q1[j, :WINDOW].double().numpy() for j in range(4)])
        _CPU_INPUTS = (q, k[0].double().numpy(), v[0].double().numpy(), dq)
    return _CPU_INPUTS


def cpu_sample():
    """Time the oracle on (a) one full-size edge build for one KV head and
    (b) attention of sampled query rows against full-size blocks, then
    extrapolate to the layer: 28 edges x 8 KV heads of builds and every
    (query row, visible key) pair of the local and compact attention."""
    import numpy as np
    from oracle import dcc_kv_oracle as orc

    q, k64, v64, dq = _cpu_inputs()
    t0 = time.perf_counter()
    qh, _ = orc.select_representative_queries(dq, M_REPR, DP)
    t_pool = time.perf_counter() - t0
    t0 = time.perf_counter()
    c = orc.build_compact_kv_from_repr(k64, v64, qh, BUDGET)
    t_build = time.perf_counter() - t0
    rows = 64
    qs = q[0, -rows:].double().numpy()
    t0 = time.perf_counter()
    orc.attention_partial(qs, k64, v64, positions=np.arange(BLOCK_LEN - rows, BLOCK_LEN))
    orc.attention_partial(qs, c.keys, c.values, bias=c.logit_bias)
    t_attn = time.perf_counter() - t0
    pairs_sample = rows * (BLOCK_LEN + BUDGET)
    local_pairs = N_BLOCKS * HQ * BLOCK_LEN * (BLOCK_LEN + 1) // 2
    compact_pairs = sum(HQ * BLOCK_LEN * r * BUDGET for r in range(N_BLOCKS))
    n_edges = N_BLOCKS * (N_BLOCKS - 1) // 2
    total = ((N_BLOCKS - 1) * HKV * t_pool + n_edges * HKV * t_build
             + (local_pairs + compact_pairs) * t_attn / pairs_sample)
    sample = (f"one KV head: FPS over {4 * WINDOW} queries ({t_pool:.2f}s) + one edge build "
              f"L_s={BLOCK_LEN} B={BUDGET} ({t_build:.2f}s) + {rows} query rows x {BLOCK_LEN + BUDGET} keys "
              f"({t_attn:.2f}s); extrapolated to {n_edges * HKV} builds and "
              f"{local_pairs + compact_pairs:.3e} (row, key) pairs")
    return total, sample


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    for _ in range(args.warmup):
        cpu_sample()
    times, sample = [], ""
    for _ in range(args.steps):
        t, sample = cpu_sample()
        times.append(t)
    mean_t = sum(times) / len(times)
    value = TOKENS / mean_t
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": mean_t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded, bf16-valued inputs)",
            "config": dict(WORKLOAD, parallelism="cpu"), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
_HOST_CPUS = None


def bind_near_gpu(index: int) -> None:
    """Run this process on the host cores nearest GPU ``index`` (NVML's
    read-only CPU-affinity mask), so the pinned host buffers it allocates
    afterwards sit in that socket's memory and the host <-> device copies
    of the end-to-end leg do not cross the socket interconnect."""
    global _HOST_CPUS
    _HOST_CPUS = os.sched_getaffinity(0)
    try:
        nv, h = ClockSampler(index)._nvml_handle()
        words = ((os.cpu_count() or 1) + 63) // 64
        mask = nv.nvmlDeviceGetCpuAffinity(h, words)
        cpus = {w * 64 + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
    except Exception:
        pass


def _setup_dist():
    import datetime
    import torch.distributed as dist
    ws, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    bind_near_gpu(local)
    if ws > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    return ws, rank, dev


def _max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(ws: int) -> None:
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def run_gpu(args):
    import dcc_kv_b200 as dk
    from dcc_kv_b200.workloads import gqa_block, layer_inputs

    ws, rank, dev = _setup_dist()
    if ws == 1:
        q, k, v = layer_inputs(N_BLOCKS, BLOCK_LEN, HQ, HKV, D, device="cuda")
        layer = dk.DccKvSyncLayer(N_BLOCKS, BLOCK_LEN, HQ, HKV, D, BUDGET, WINDOW, M_REPR, DP, device=dev)
        layer.schedule = args.schedule
        parallelism = f"single GPU, 8 logical blocks, {args.schedule} schedule"
    else:
        from dcc_kv_b200.dist_layer import DistributedDccKvLayer
        from dcc_kv_b200.dist_layer import local_blocks_of
        blocks = local_blocks_of(N_BLOCKS, ws, rank)
        parts = [gqa_block(HQ, HKV, BLOCK_LEN, D, 1000 + b, device="cuda") for b in blocks]
        q, k, v = (torch.stack([p_[i] for p_ in parts]) for i in range(3))
        layer = DistributedDccKvLayer(N_BLOCKS, BLOCK_LEN, HQ, HKV, D, BUDGET, WINDOW, M_REPR, DP, device=dev)
        parallelism = (f"context parallel over {ws} GPUs (blocks dealt to ranks in snake order), "
                       "NCCL all-to-allv of compacts")
    stream = torch.cuda.current_stream(dev)
    warmup = max(args.warmup, 3)
    for _ in range(warmup):
        layer(q, k, v)
    _barrier(ws)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    attn_ev = [[] for _ in range(args.steps)]  # (start, end) around each attention launch
    layer.timing_events = attn_ev
    with ClockSampler(dev.index) as clk:
        _barrier(ws)
        for i in range(args.steps):
            ev[i][0].record(stream)
            layer.timing_index = i
            layer(q, k, v)
            ev[i][1].record(stream)
        _barrier(ws)
    layer.timing_events = None
    ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / args.steps, ws)
    a_ms = sum(a.elapsed_time(b) for step in attn_ev for a, b in step) / args.steps
    a_launches = len(attn_ev[0])
    clocks = clk.summary()
    # end to end through the public layer call: pinned host inputs in, output
    # back to host; the layers pipeline the copies with the compute
    hq_, hk_, hv_ = (t.cpu().pin_memory() for t in (q, k, v))
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()

    def e2e_step():
        layer(hq_, hk_, hv_, out=out_host)

    for _ in range(warmup):
        e2e_step()
    torch.cuda.synchronize(dev)
    _barrier(ws)
    e2e_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    # the device is idle here, so no copy of the first timed step starts before this event
    e2e_ev[0].record(stream)
    for _ in range(args.steps):
        e2e_step()
    e2e_ev[1].record(stream)
    torch.cuda.synchronize(dev)
    _barrier(ws)
    e2e_ms = _max_over_ranks(e2e_ev[0].elapsed_time(e2e_ev[1]) / args.steps, ws)
    h2d = _max_over_ranks(float(sum(t.numel() * t.element_size() for t in (q, k, v))), ws) * ws
    d2h = float(out_host.numel() * out_host.element_size()) * ws
    launches = layer.launches_per_forward() * args.steps
    if rank != 0:
        _teardown(ws)
        return
    hbm, tf_burst, tf_sust, src = peaks()
    n_local = q.shape[0]
    if ws == 1:
        # every block's causal local segment plus its compact segment
        kflops = sum(causal_attention_flops())
        kname = (f"attention: causal local + compact with logit bias, all 8 blocks, {a_launches} launch(es) "
                 "per step (flops-weighted)")
    else:
        kflops = n_local * HQ * (BLOCK_LEN * (BLOCK_LEN + 1) // 2) * 4 * D
        kname = f"local causal attention ({n_local} block(s) per GPU, one launch, rank 0)"
    achieved = kflops / (a_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": TOKENS / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
        "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1), 4 outlier channels x8 per KV head)",
        "config": dict(WORKLOAD, parallelism=parallelism),
        "e2e": {"value": TOKENS / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches,
        "roofline": {"kernel": kname, "bound": "tensor", "achieved": achieved, "peak": tf_sust,
                     "unit": "TFLOP/s", "frac": achieved / tf_sust, "peak_source": f"{src} bf16 sustained",
                     "traffic": attention_traffic() / a_launches if ws == 1 else None,
                     "traffic_source": "ncu DRAM bytes of one block (--profile-attention), reads scaled to "
                                       "8 blocks by algorithmic read bytes, writes = output size; "
                                       "averaged over the step's launches",
                     "algorithmic_bytes": sum(attention_bytes([r * BUDGET for r in range(N_BLOCKS)])) / a_launches
                     if ws == 1 else None,
                     "algorithmic_flops": kflops, "launches": a_launches,
                     "ms_per_launch": a_ms / max(a_launches, 1), "ms_per_step": a_ms},
        "clocks": clocks,
    }
    if args.cpu_baseline and ws == 1:
        if _HOST_CPUS:
            os.sched_setaffinity(0, _HOST_CPUS)  # the CPU baseline uses every host core
        cores = len(os.sched_getaffinity(0))
        torch.set_num_threads(cores)
        t, sample = cpu_sample()
        line["cpu_baseline"] = {"value": TOKENS / t, "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": sample}
    print(json.dumps(line), flush=True)
    _teardown(ws)


def _teardown(ws: int) -> None:
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def profile_attention(args):
    """One fused attention launch of the last destination block (16384 causal
    local keys + 7 x 1024 compact keys with bias, 32/8 heads, d 128, bf16;
    ~250 MB on the device) after one warm-up launch: the small case for ncu."""
    import math as _m
    from dcc_kv_b200.attention import attn_problem, kv_segment, run_attention
    from dcc_kv_b200.workloads import gqa_block
    dev = torch.device("cuda", 0)
    q, k, v = gqa_block(HQ, HKV, BLOCK_LEN, D, 1007, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    ck = torch.randn(HKV, 7 * BUDGET, D, generator=g, device="cuda").to(torch.bfloat16)
    cv = torch.randn(HKV, 7 * BUDGET, D, generator=g, device="cuda").to(torch.bfloat16)
    cb = torch.randn(HKV, 7 * BUDGET, generator=g, device="cuda")
    o = torch.empty_like(q)
    prob = attn_problem(q, o, None, [kv_segment(k, v), kv_segment(ck, cv, cb)], causal=True)
    for _ in range(2):
        run_attention([prob], HQ, HKV, D, 1.0 / _m.sqrt(D), 1, dev)
    torch.cuda.synchronize()
    print("profiled attention launch done", flush=True)


def exchange_study(args):
    """Communication-computation overlap of the compact-KV exchange (the
    reference's sync-vs-async question, tests/gpu/test_async_overlap.py):
    per-layer time with the pooling, builds and all-to-allv on the main stream
    before any attention (sync), on the side stream under the local attention
    (async, the default), and for ``--layers`` layers in a row with the
    exchange double buffered across layers (stack).  Not the bench line."""
    from dcc_kv_b200.dist_layer import DistributedDccKvLayer, DistributedDccKvStack
    from dcc_kv_b200.workloads import gqa_block
    ws, rank, dev = _setup_dist()
    if ws < 2:
        print(json.dumps({"study": "exchange overlap", "unavailable": "needs 2+ GPUs under torchrun"}))
        return
    from dcc_kv_b200.dist_layer import local_blocks_of
    blocks = local_blocks_of(N_BLOCKS, ws, rank)
    inputs = []
    for layer_i in range(args.layers):
        parts = [gqa_block(HQ, HKV, BLOCK_LEN, D, 1000 * (layer_i + 1) + b, device="cuda") for b in blocks]
        inputs.append(tuple(torch.stack([p_[i] for p_ in parts]) for i in range(3)))
    kw = dict(device=dev)
    layer = DistributedDccKvLayer(N_BLOCKS, BLOCK_LEN, HQ, HKV, D, BUDGET, WINDOW, M_REPR, DP, **kw)
    stack = DistributedDccKvStack(N_BLOCKS, BLOCK_LEN, HQ, HKV, D, BUDGET, WINDOW, M_REPR, DP, **kw)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        _barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        _barrier(ws)
        return _max_over_ranks(e0.elapsed_time(e1) / args.steps / args.layers, ws)

    def layer_by_layer():
        for x in inputs:
            layer(*x)

    layer.overlap_exchange = False
    t_sync = timed(layer_by_layer)
    layer.overlap_exchange = True
    t_async = timed(layer_by_layer)
    t_stack = timed(lambda: stack(inputs))
    plan = layer.plan
    if rank == 0:
        print(json.dumps({
            "study": "exchange overlap", "n_gpus": ws, "layers": args.layers, "steps": args.steps,
            "config": dict(WORKLOAD, parallelism=f"context parallel over {ws} GPUs"),
            "exchange_bytes_per_rank_per_layer": max(sum(plan.send_splits(r)) for r in range(ws)),
            "ms_per_layer": {"sync": t_sync, "async": t_async, "stack": t_stack},
            "speedup_async_vs_sync": t_sync / t_async, "speedup_stack_vs_sync": t_sync / t_stack,
        }), flush=True)
    del stack, layer
    _teardown(ws)


def phase_study(args):
    """Under torchrun (N >= 2): per rank, the mean time from the start of a
    forward to the end of each phase (pooling, gather, builds, exchange on
    the side stream; local attention, the wait for the exchange, compact
    attention, hand-off transfers, helper attention, merge on the main
    stream), CUDA events on each phase's stream.  One JSON line on rank 0
    with every rank's figures; not the bench line."""
    from dcc_kv_b200.dist_layer import DistributedDccKvLayer, local_blocks_of
    from dcc_kv_b200.workloads import gqa_block
    import torch.distributed as dist
    ws, rank, dev = _setup_dist()
    if ws < 2:
        print(json.dumps({"study": "phase times", "unavailable": "needs 2+ GPUs under torchrun"}))
        return
    blocks = local_blocks_of(N_BLOCKS, ws, rank)
    parts = [gqa_block(HQ, HKV, BLOCK_LEN, D, 1000 + b, device="cuda") for b in blocks]
    q, k, v = (torch.stack([p_[i] for p_ in parts]) for i in range(3))
    layer = DistributedDccKvLayer(N_BLOCKS, BLOCK_LEN, HQ, HKV, D, BUDGET, WINDOW, M_REPR, DP, device=dev)
    for _ in range(max(args.warmup, 3)):
        layer(q, k, v)
    _barrier(ws)
    layer.phase_events = []
    for _ in range(args.steps):
        layer(q, k, v)
    _barrier(ws)
    mine = {"rank": rank, "blocks": blocks, "helped": layer.helped, "helping": layer.helping,
            "build_problems": len(layer.build), "ms": layer.phase_times(layer.phase_events)}
    layer.phase_events = None
    everyone = [None] * ws
    dist.all_gather_object(everyone, mine)
    if rank == 0:
        print(json.dumps({"study": "phase times", "n_gpus": ws, "steps": args.steps,
                          "config": dict(WORKLOAD, parallelism=f"context parallel over {ws} GPUs"),
                          "ranks": everyone}), flush=True)
    del layer
    _teardown(ws)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--schedule", choices=("pipelined", "batched"), default="batched",
                    help="single-GPU layer schedule: builds then one attention launch (default), or builds "
                         "overlapped with per-block attention")
    ap.add_argument("--profile-attention", action="store_true",
                    help="run two attention launches of one block (small case for ncu) and exit")
    ap.add_argument("--exchange-study", action="store_true",
                    help="under torchrun, N >= 2: time the compact exchange synchronous, overlapped, and "
                         "double buffered across --layers layers, and exit")
    ap.add_argument("--layers", type=int, default=4, help="layers in a row for --exchange-study")
    ap.add_argument("--phase-times", action="store_true",
                    help="under torchrun, N >= 2: per-rank times of each phase of the sharded layer, and exit")
    args = ap.parse_args()
    if args.exchange_study:
        exchange_study(args)
    elif args.phase_times:
        phase_study(args)
    elif args.profile_attention:
        profile_attention(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
