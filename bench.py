"""DCC-KV benchmark: tokens/s of the full DCC-KV layer, plus the secondary
configurations of the hot path.

Default workload (``--config cfg4``): the 128K-context layer -- 131072 tokens
as 8 blocks of 16384, 32 query / 8 KV heads, head_dim 128, bf16, compact
budget 1024 per (source, destination) edge, destination window 2048 queries
per query head, M = 64 representative queries, d_p = 32.  A step is one
forward of the layer over the whole context: pooling + 28 x 8 compact builds
+ local causal attention + compact attention with logit bias +
online-softmax merge.

Other configurations (one JSON line each, same keys):
  cfg2  online-softmax merge microbench: 8 partial outputs [32, 4096, 128]
        bf16 + fp32 LSE merged into one (HBM-bound; GB/s);
  cfg3  batched GQA build_compact_kv: 8 KV heads, L_s 16384, 4 x 2048
        destination queries per KV head, budget 512 (edge builds/s);
  cfg5  the 1M-context layer: 8 blocks of 131072, budgets drawn from
        {256, 512, 1024, 2048} with seed 1 (tokens/s).

    python bench.py [--config cfgN] [--gpus N --steps K --warmup W] [--impl reference]

N = 1 runs the 8 logical blocks on one GPU; under torchrun the layers are
sharded by block (cfg2 / cfg3 run one replica per GPU).  ``--impl reference``
times the FP64 CPU oracle (a restatement of the reference path) on a bounded
sample of the same workload.
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
from dataclasses import dataclass, field
from typing import Dict, Tuple

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HQ, HKV, D = 32, 8, 128
WINDOW, M_REPR, DP = 2048, 64, 32


@dataclass
class LayerWorkload:
    """One DCC-KV layer configuration (block geometry and per-edge budgets)."""
    name: str
    metric: str
    blocks: int
    block_len: int
    budgets: Dict[Tuple[int, int], int] = field(repr=False)
    l2: str = ""
    budget_desc: object = None

    @property
    def tokens(self) -> int:
        return self.blocks * self.block_len

    def compact_rows(self, r: int) -> int:
        return sum(min(self.budgets[(s, r)], self.block_len) for s in range(r))

    def config(self, **extra) -> dict:
        return dict({"workload": self.name, "context_tokens": self.tokens, "blocks": self.blocks,
                     "block_len": self.block_len, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                     "budget": self.budget_desc, "window": WINDOW, "repr_queries": M_REPR,
                     "projection_dim": DP, "l2": self.l2}, **extra)


def _layer_128k() -> LayerWorkload:
    nb, L = 8, 16384
    return LayerWorkload("dcc_kv_sync_layer_128k", "DCC-KV layer prefill tokens/s at 128K ctx", nb, L,
                         {(s, r): 1024 for r in range(nb) for s in range(r)},
                         "inputs larger than L2 (q 1 GiB, k/v 256 MiB each)", 1024)


def _layer_1m() -> LayerWorkload:
    from dcc_kv_b200.workloads import variable_budgets
    nb, L = 8, 131072
    return LayerWorkload("dcc_kv_sync_layer_1m", "DCC-KV layer prefill tokens/s at 1M ctx", nb, L,
                         variable_budgets(nb), "inputs larger than L2 (q 8 GiB, k/v 2 GiB each)",
                         "per edge from {256, 512, 1024, 2048}, seed 1")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


def causal_attention_flops(wl: LayerWorkload):
    """Algorithmic FLOPs of one step's attention: local causal (L(L+1)/2 pairs
    per head and block) and compact (block r sees its compact rows), 4 d per pair."""
    L = wl.block_len
    local = wl.blocks * HQ * (L * (L + 1) // 2) * 4 * D
    compact = sum(HQ * L * wl.compact_rows(r) * 4 * D for r in range(wl.blocks))
    return local, compact


def attention_bytes(wl: LayerWorkload, blocks_compact_rows):
    """Algorithmic HBM bytes of one attention launch over the given blocks:
    (read, write).  Per block: Q, local K and V read once, its compact K, V
    (bf16) and bias (fp32) read once, O written once."""
    read = write = 0
    for rows in blocks_compact_rows:
        read += (HQ + 2 * HKV) * wl.block_len * D * 2 + HKV * rows * (2 * D * 2 + 4)
        write += HQ * wl.block_len * D * 2
    return read, write


# DRAM bytes of one ncu capture of the --profile-attention launch (the last
# destination block of the 128K layer: 16384 causal keys + 7 x 1024 compact
# keys per KV head): dram__bytes_read.sum.  Its reads are 1.001 x the
# algorithmic read bytes (no re-reads past L2).  Its writes are lower than the
# output size because the tail of the output is still in L2 when the launch
# ends; a full launch writes ~1 GiB, far beyond L2, so its writes are taken
# at the algorithmic figure.
PROFILED_DRAM_READ = 231_221_248


def attention_traffic(wl: LayerWorkload):
    """Estimated DRAM bytes of the full single-GPU attention launch of the
    128K layer: reads scaled from the profiled block by algorithmic read
    bytes, writes at the algorithmic output size (None for other layers:
    nothing profiled there)."""
    if wl.block_len != 16384:
        return None
    prof_read, _ = attention_bytes(wl, [7 * 1024])
    read, write = attention_bytes(wl, [wl.compact_rows(r) for r in range(wl.blocks)])
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
_CPU_INPUTS = {}


def _cpu_layer_inputs(wl: LayerWorkload):
    """Block 0 (source) and the destination window of block 1 of one KV head
    and its 4 query heads (the timed sample reads nothing else), drawn once
    with the layer's value distribution."""
    if wl.name not in _CPU_INPUTS:
        import numpy as np
        from dcc_kv_b200.workloads import gqa_block
        q, k, v = gqa_block(HQ // HKV, 1, wl.block_len, D, seed=1000, device="cpu")
        q1, _, _ = gqa_block(HQ // HKV, 1, wl.block_len, D, seed=1001, device="cpu")
        dq = np.concatenate([q1[j, :WINDOW].double().numpy() for j in range(4)])
        _CPU_INPUTS[wl.name] = (q, k[0].double().numpy(), v[0].double().numpy(), dq)
    return _CPU_INPUTS[wl.name]


def cpu_sample(wl: LayerWorkload):
    """Time the oracle on (a) one full-size edge build for one KV head and
    (b) attention of sampled query rows against full-size blocks, then
    extrapolate to the layer: every edge x 8 KV heads of builds (each at the
    sampled build's cost) and every (query row, visible key) pair of the
    local and compact attention.  Returns (extrapolated seconds per layer,
    seconds this sample took, description).  The oracle's streaming
    farthest-point sampling is faster than the reference's N x N form, so
    this overstates the reference's CPU speed rather than understating it."""
    import numpy as np
    from oracle import dcc_kv_oracle as orc

    t_start = time.perf_counter()
    L = wl.block_len
    budget = 1024
    q, k64, v64, dq = _cpu_layer_inputs(wl)
    t0 = time.perf_counter()
    qh, _ = orc.select_representative_queries(dq, M_REPR, DP)
    t_pool = time.perf_counter() - t0
    t0 = time.perf_counter()
    c = orc.build_compact_kv_from_repr(k64, v64, qh, budget)
    t_build = time.perf_counter() - t0
    rows = 64
    qs = q[0, -rows:].double().numpy()
    t0 = time.perf_counter()
    orc.attention_partial(qs, k64, v64, positions=np.arange(L - rows, L))
    orc.attention_partial(qs, c.keys, c.values, bias=c.logit_bias)
    t_attn = time.perf_counter() - t0
    pairs_sample = rows * (L + budget)
    local_pairs = wl.blocks * HQ * L * (L + 1) // 2
    compact_pairs = sum(HQ * L * wl.compact_rows(r) for r in range(wl.blocks))
    n_edges = len(wl.budgets)
    total = ((wl.blocks - 1) * HKV * t_pool + n_edges * HKV * t_build
             + (local_pairs + compact_pairs) * t_attn / pairs_sample)
    sample = (f"one KV head: FPS over {4 * WINDOW} queries ({t_pool:.2f}s) + one edge build "
              f"L_s={L} B={budget} ({t_build:.2f}s) + {rows} query rows x {L + budget} keys "
              f"({t_attn:.2f}s); extrapolated to {n_edges * HKV} builds and "
              f"{local_pairs + compact_pairs:.3e} (row, key) pairs")
    return total, time.perf_counter() - t_start, sample


MERGE_PARTS, MERGE_HEADS, MERGE_ROWS = 8, 32, 4096
MERGE_BYTES = (MERGE_PARTS * MERGE_HEADS * MERGE_ROWS * (D * 2 + 4)   # partial O (bf16) and LSE (fp32) read
               + MERGE_HEADS * MERGE_ROWS * (D * 2 + 4))               # merged O (bf16) and LSE (fp32) written


def cpu_merge_sample():
    """The whole merge microbench on the oracle (FP64 fold of
    online_softmax.py:92-111), one head at a time.  Returns (seconds, seconds,
    description): nothing is extrapolated."""
    from oracle import dcc_kv_oracle as orc
    from dcc_kv_b200.workloads import merge_inputs
    if "merge" not in _CPU_INPUTS:
        outs, lses = merge_inputs(MERGE_PARTS, MERGE_HEADS, MERGE_ROWS, D, seed=0, device="cpu")
        _CPU_INPUTS["merge"] = ([o.float().numpy() for o in outs], [x.numpy() for x in lses])
    outs, lses = _CPU_INPUTS["merge"]
    t0 = time.perf_counter()
    for h in range(MERGE_HEADS):
        orc.merge_lse([o[h] for o in outs], [x[h] for x in lses])
    t = time.perf_counter() - t0
    return t, t, f"all {MERGE_HEADS} heads x {MERGE_ROWS} rows x {MERGE_PARTS} parts, FP64 numpy, one head at a time"


BUILD_LS, BUILD_LR, BUILD_BUDGET = 16384, 2048, 512


def _build_bytes():
    """Algorithmic HBM bytes of one cfg3 edge build (all 8 KV heads): K and V
    read once, the destination queries (4 x 2048 per KV head) read once,
    the compact keys / values (bf16), bias (fp32) and indices (int64) written."""
    kv = 2 * HKV * BUILD_LS * D * 2
    qw = HQ * BUILD_LR * D * 2
    out = HKV * BUILD_BUDGET * (2 * D * 2 + 4 + 8)
    return kv + qw + out


def cpu_build_sample():
    """cfg3 on the oracle: pooling and the build of every KV head (nothing
    extrapolated)."""
    import numpy as np
    from oracle import dcc_kv_oracle as orc
    from dcc_kv_b200.workloads import gqa_block
    if "build" not in _CPU_INPUTS:
        q, k, v = gqa_block(HQ, HKV, BUILD_LS, D, seed=0, q_len=BUILD_LR, device="cpu")
        _CPU_INPUTS["build"] = (q, k, v)
    q, k, v = _CPU_INPUTS["build"]
    t0 = time.perf_counter()
    for h in range(HKV):
        dq = np.concatenate([q[4 * h + j].double().numpy() for j in range(4)])
        orc.build_compact_kv(k[h].double().numpy(), v[h].double().numpy(), dq, BUILD_BUDGET)
    t = time.perf_counter() - t0
    return t, t, f"one edge, all {HKV} KV heads: pooling + build (L_s={BUILD_LS}, B={BUILD_BUDGET}), FP64 numpy"


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    if args.config == "cfg2":
        sample_fn, unit, per = cpu_merge_sample, "GB/s", lambda t: MERGE_BYTES / t / 1e9
        metric, config = MERGE_METRIC, MERGE_CONFIG
    elif args.config == "cfg3":
        sample_fn, unit, per = cpu_build_sample, "edge builds/s", lambda t: 1.0 / t
        metric, config = BUILD_METRIC, BUILD_CONFIG
    else:
        wl = _layer_1m() if args.config == "cfg5" else _layer_128k()
        sample_fn, unit, per = (lambda: cpu_sample(wl)), "tokens/s", lambda t: wl.tokens / t
        metric, config = wl.metric, wl.config()
    for _ in range(args.warmup):
        sample_fn()
    times, spent, sample = [], [], ""
    for _ in range(args.steps):
        t, t_sample, sample = sample_fn()
        times.append(t)
        spent.append(t_sample)
    mean_t = sum(times) / len(times)
    value = per(mean_t)
    # ms_per_step is the time one bounded sample took (what this run spent);
    # value is the whole workload's rate (extrapolated from the sample where
    # the sample is smaller than the workload)
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sum(spent) / len(spent) * 1e3,
            "extrapolated_ms_per_step": mean_t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded, bf16-valued inputs)",
            "config": dict(config, parallelism="cpu"), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": sample,
                             "port_vs_reference": PORT_VS_REFERENCE},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ncu dram__bytes_read.sum + dram__bytes_write.sum of one merge launch
# (272,643,072 read = the algorithmic read bytes; 14,579,456 written: the rest
# of the 34 MB output is still in L2 when the launch ends)
MERGE_PROFILED_DRAM = 272_643_072 + 14_579_456

# The oracle port against the reference's own torch code on the same CPU (not
# measured in this run: the reference is not installed where the bench runs).
PORT_VS_REFERENCE = ("one cfg3 edge-head build (L_s 16384, 8192 destination queries): the reference's torch code "
                     "(FP64, its N x N farthest-point sampling) 0.74 s, this oracle port 0.11 s, same 8-thread "
                     "container; the port's timings overstate the reference's CPU speed")

MERGE_METRIC = "online-softmax LSE merge bandwidth, 8 partials of [32, 4096, 128]"
MERGE_CONFIG = {"workload": "online_softmax_merge_8way", "parts": MERGE_PARTS, "heads": MERGE_HEADS,
                "queries": MERGE_ROWS, "head_dim": D, "o_dtype": "bf16", "lse_dtype": "f32",
                "algorithmic_bytes": MERGE_BYTES, "l2": "inputs larger than L2 (276 MB read per step)"}
BUILD_METRIC = "batched GQA build_compact_kv edge builds/s (8 KV heads, L_s 16384, B 512)"
BUILD_CONFIG = {"workload": "build_compact_kv_gqa_edge", "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                "source_len": BUILD_LS, "window": BUILD_LR, "budget": BUILD_BUDGET, "repr_queries": M_REPR,
                "projection_dim": DP, "algorithmic_bytes": _build_bytes(),
                "l2": "L2 flushed between steps (a 256 MiB write; inputs are 84 MB)"}


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


def run_gpu(args, wl: LayerWorkload):
    import dcc_kv_b200 as dk
    from dcc_kv_b200.workloads import gqa_block, layer_inputs

    ws, rank, dev = _setup_dist()
    nb, L = wl.blocks, wl.block_len
    if ws == 1:
        q, k, v = layer_inputs(nb, L, HQ, HKV, D, device="cuda")
        layer = dk.DccKvSyncLayer(nb, L, HQ, HKV, D, wl.budgets, WINDOW, M_REPR, DP, device=dev)
        layer.schedule = args.schedule
        parallelism = f"single GPU, {nb} logical blocks, {args.schedule} schedule"
    else:
        from dcc_kv_b200.dist_layer import DistributedDccKvLayer
        from dcc_kv_b200.dist_layer import local_blocks_of
        blocks = local_blocks_of(nb, ws, rank)
        parts = [gqa_block(HQ, HKV, L, D, 1000 + b, device="cuda") for b in blocks]
        q, k, v = (torch.stack([p_[i] for p_ in parts]) for i in range(3))
        del parts
        layer = DistributedDccKvLayer(nb, L, HQ, HKV, D, wl.budgets, WINDOW, M_REPR, DP, device=dev)
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
    layer.check()  # no bounded device wait gave up during the timed steps
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
    layer.check()
    e2e_ms = _max_over_ranks(e2e_ev[0].elapsed_time(e2e_ev[1]) / args.steps, ws)
    h2d = _max_over_ranks(float(sum(t.numel() * t.element_size() for t in (q, k, v))), ws) * ws
    d2h = float(out_host.numel() * out_host.element_size()) * ws
    launches = layer.launches_per_forward() * args.steps
    if rank != 0:
        _teardown(ws)
        return
    hbm, tf_burst, tf_sust, src = peaks()
    n_local = q.shape[0]
    traffic = alg_bytes = None
    if ws == 1:
        # every block's causal local segment plus its compact segment
        kflops = sum(causal_attention_flops(wl))
        kname = (f"attention: causal local + compact with logit bias, all {nb} blocks, {a_launches} launch(es) "
                 "per step (flops-weighted)")
        t_all = attention_traffic(wl)
        traffic = None if t_all is None else t_all / a_launches
        alg_bytes = sum(attention_bytes(wl, [wl.compact_rows(r) for r in range(nb)])) / a_launches
    else:
        kflops = n_local * HQ * (L * (L + 1) // 2) * 4 * D
        kname = f"local causal attention ({n_local} block(s) per GPU, one launch, rank 0)"
    achieved = kflops / (a_ms * 1e-3) / 1e12
    layer_flops = sum(causal_attention_flops(wl))
    line = {
        "metric": wl.metric, "value": wl.tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1), 4 outlier channels x8 per KV head)",
        "config": wl.config(parallelism=parallelism),
        "e2e": {"value": wl.tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches,
        "roofline": {"kernel": kname, "bound": "tensor", "achieved": achieved, "peak": tf_sust,
                     "unit": "TFLOP/s", "frac": achieved / tf_sust, "peak_source": f"{src} bf16 sustained",
                     "traffic": traffic,
                     "traffic_source": "ncu DRAM bytes of one 128K-layer block (--profile-attention), reads "
                                       "scaled to all blocks by algorithmic read bytes, writes = output size; "
                                       "averaged over the step's launches" if traffic is not None else None,
                     "algorithmic_bytes": alg_bytes,
                     "algorithmic_flops": kflops, "launches": a_launches,
                     "ms_per_launch": a_ms / max(a_launches, 1), "ms_per_step": a_ms},
        # the whole layer against the whole job's tensor peak: every block's
        # attention FLOPs (local + compact, the bulk of the layer's work) over
        # n_gpus x the measured sustained peak x the step time
        "layer_roofline": {"flops": layer_flops, "achieved": layer_flops / (ms * 1e-3) / 1e12,
                           "peak": ws * tf_sust, "unit": "TFLOP/s",
                           "frac": layer_flops / (ms * 1e-3) / 1e12 / (ws * tf_sust)},
        "clocks": clocks,
    }
    if args.cpu_baseline and ws == 1:
        if _HOST_CPUS:
            os.sched_setaffinity(0, _HOST_CPUS)  # the CPU baseline uses every host core
        cores = len(os.sched_getaffinity(0))
        torch.set_num_threads(cores)
        t, _, sample = cpu_sample(wl)
        line["cpu_baseline"] = {"value": wl.tokens / t, "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": sample, "port_vs_reference": PORT_VS_REFERENCE}
    print(json.dumps(line), flush=True)
    _teardown(ws)


def _time_steps(step, steps: int, warmup: int, stream, flush=None):
    """CUDA-event time of each of ``steps`` calls of ``step`` after
    ``warmup`` untimed ones; ``flush`` (untimed) runs before every step."""
    for _ in range(warmup):
        if flush is not None:
            flush()
        step()
    torch.cuda.synchronize()
    total = 0.0
    evs = []
    for _ in range(steps):
        if flush is not None:
            flush()
        e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        e[0].record(stream)
        step()
        e[1].record(stream)
        evs.append(e)
    torch.cuda.synchronize()
    for a, b in evs:
        total += a.elapsed_time(b)
    return total / steps


def _cpu_baseline_line(sample_fn, per, unit):
    if _HOST_CPUS:
        os.sched_setaffinity(0, _HOST_CPUS)
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    t, _, sample = sample_fn()
    return {"value": per(t), "unit": unit, "cores": cores, "kind": "port", "sample": sample}


def run_merge(args):
    """cfg2: the P-way LSE merge kernel (dcc_merge_lse) on 8 partials of
    [32, 4096, 128] bf16 + fp32 LSE; one launch per step, HBM-bound.  Under
    torchrun every rank merges its own partials (replicas)."""
    import dcc_kv_b200 as dk
    from dcc_kv_b200.workloads import merge_inputs
    ws, rank, dev = _setup_dist()
    outs, lses = merge_inputs(MERGE_PARTS, MERGE_HEADS, MERGE_ROWS, D, seed=rank, device="cuda")
    out = torch.empty_like(outs[0])
    lse = torch.empty(MERGE_HEADS, MERGE_ROWS, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    warmup = max(args.warmup, 3)
    _barrier(ws)
    with ClockSampler(dev.index) as clk:
        ms = _time_steps(lambda: dk.merge_lse(outs, lses, out=out, lse_out=lse), args.steps, warmup, stream)
    ms = _max_over_ranks(ms, ws)
    # end to end: the 8 partials and LSEs from pinned host memory, merged,
    # the merged output and LSE back to pinned host memory, every step
    h_outs = [o.cpu().pin_memory() for o in outs]
    h_lses = [x.cpu().pin_memory() for x in lses]
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h_lse = torch.empty(lse.shape, dtype=lse.dtype).pin_memory()

    def e2e_step():
        for d_, h_ in zip(outs + lses, h_outs + h_lses):
            d_.copy_(h_, non_blocking=True)
        dk.merge_lse(outs, lses, out=out, lse_out=lse)
        h_out.copy_(out, non_blocking=True)
        h_lse.copy_(lse, non_blocking=True)

    e2e_ms = _max_over_ranks(_time_steps(e2e_step, args.steps, warmup, stream), ws)
    h2d = sum(t.numel() * t.element_size() for t in h_outs + h_lses) * ws
    d2h = (h_out.numel() * h_out.element_size() + h_lse.numel() * h_lse.element_size()) * ws
    if rank != 0:
        _teardown(ws)
        return
    hbm, _, _, src = peaks()
    gbs = MERGE_BYTES * ws / (ms * 1e-3) / 1e9
    per_gpu = MERGE_BYTES / (ms * 1e-3) / 1e9
    line = {"metric": MERGE_METRIC, "value": gbs, "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded: O ~ N(0,1) bf16, LSE ~ N(0,1) x 4 fp32)",
            "config": dict(MERGE_CONFIG, parallelism="one GPU" if ws == 1 else f"{ws} replicas"),
            "e2e": {"value": MERGE_BYTES * ws / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": args.steps,
            "roofline": {"kernel": "merge_lse_vec_kernel<bf16, 8 parts> (the whole step)", "bound": "hbm",
                         "achieved": per_gpu, "peak": hbm, "unit": "GB/s", "frac": per_gpu / hbm,
                         "peak_source": f"{src} HBM copy", "traffic": MERGE_PROFILED_DRAM,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch",
                         "algorithmic_bytes": MERGE_BYTES, "launches": 1, "ms_per_launch": ms},
            "clocks": clk.summary()}
    if args.cpu_baseline and ws == 1:
        line["cpu_baseline"] = _cpu_baseline_line(cpu_merge_sample, lambda t: MERGE_BYTES / t / 1e9, "GB/s")
    print(json.dumps(line), flush=True)
    _teardown(ws)


def run_build(args):
    """cfg3: one edge of the batched GQA build -- pooling of the 8 destination
    query sets (4 x 2048 queries per KV head) and the build of all 8 KV heads
    (L_s 16384, budget 512).  The inputs (84 MB) fit in L2, so a 256 MiB
    write flushes it before every step (untimed).  Under torchrun every rank
    builds its own edge (replicas)."""
    import dcc_kv_b200 as dk
    from dcc_kv_b200 import _lib as L
    from dcc_kv_b200.compact_kv import build_launch_count, build_problem, run_build_problems
    from dcc_kv_b200.representative_query import query_set, select_query_sets
    from dcc_kv_b200.workloads import gqa_block
    ws, rank, dev = _setup_dist()
    q, k, v = gqa_block(HQ, HKV, BUILD_LS, D, seed=rank, q_len=BUILD_LR, device="cuda")
    g = HQ // HKV
    rep = torch.empty(HKV, M_REPR, D, dtype=q.dtype, device=dev)
    ridx = torch.empty(HKV, M_REPR, dtype=torch.int64, device=dev)
    ok = torch.empty(HKV, BUILD_BUDGET, D, dtype=q.dtype, device=dev)
    ov = torch.empty_like(ok)
    ob = torch.empty(HKV, BUILD_BUDGET, dtype=torch.float32, device=dev)
    oi = torch.empty(HKV, BUILD_BUDGET, dtype=torch.int64, device=dev)

    def descriptors(q_, k_, v_):
        sets = [query_set(q_[g * h], rep[h], ridx[h], n_seg=g, seg_rows=BUILD_LR, seg_stride=q_.stride(0),
                          row_stride=q_.stride(1)) for h in range(HKV)]
        build = [build_problem(k_[h], v_[h], rep[h], BUILD_BUDGET, ok[h], ov[h], ob[h], oi[h], num_repr=M_REPR)
                 for h in range(HKV)]
        return sets, build

    sets, build = descriptors(q, k, v)
    arr = (L.dcc_build_problem * len(build))(*build)
    wsb = L.workspace(L.lib().dcc_build_compact_kv_workspace_bytes(arr, len(build), D, D, L.DCC_BF16), dev)

    def step(sets=sets, build=build):
        select_query_sets(sets, D, M_REPR, DP, 42, L.DCC_BF16, dev)
        run_build_problems(build, D, D, 1e-3, 1e-3, L.DCC_BF16, dev, wsb)

    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    warmup = max(args.warmup, 3)
    _barrier(ws)
    with ClockSampler(dev.index) as clk:
        ms = _time_steps(step, args.steps, warmup, stream, flush=lambda: flush_buf.zero_())
    ms = _max_over_ranks(ms, ws)
    # end to end: K, V and the destination query windows from pinned host
    # memory, the compact keys / values / bias / indices back, every step
    hq_, hk_, hv_ = (t.cpu().pin_memory() for t in (q, k, v))
    h_outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (ok, ov, ob, oi)]

    def e2e_step():
        q.copy_(hq_, non_blocking=True)
        k.copy_(hk_, non_blocking=True)
        v.copy_(hv_, non_blocking=True)
        step()
        for h_, d_ in zip(h_outs, (ok, ov, ob, oi)):
            h_.copy_(d_, non_blocking=True)

    e2e_ms = _max_over_ranks(_time_steps(e2e_step, args.steps, warmup, stream), ws)
    h2d = sum(t.numel() * t.element_size() for t in (hq_, hk_, hv_)) * ws
    d2h = sum(t.numel() * t.element_size() for t in h_outs) * ws
    launches = (1 + 1 + build_launch_count(len(build), L.DCC_BF16, D)) * args.steps
    if rank != 0:
        _teardown(ws)
        return
    hbm, _, _, src = peaks()
    per_gpu = _build_bytes() / (ms * 1e-3) / 1e9
    line = {"metric": BUILD_METRIC, "value": ws / (ms * 1e-3), "unit": "edge builds/s", "n_gpus": ws,
            "steps": args.steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), 4 outlier channels x8 per KV head; Q ~ N(0,1)/sqrt(128))",
            "config": dict(BUILD_CONFIG, parallelism="one GPU" if ws == 1 else f"{ws} replicas"),
            "e2e": {"value": ws / (e2e_ms * 1e-3), "unit": "edge builds/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": launches,
            "roofline": {"kernel": "the whole build step (pooling, two tcgen05 scoring passes, top-k, three FP64 "
                                   "calibration launches) against HBM: latency-bound, see profiles/",
                         "bound": "hbm", "achieved": per_gpu, "peak": hbm, "unit": "GB/s", "frac": per_gpu / hbm,
                         "peak_source": f"{src} HBM copy", "traffic": None,
                         "algorithmic_bytes": _build_bytes(), "launches": launches // args.steps,
                         "ms_per_step": ms},
            "clocks": clk.summary()}
    if args.cpu_baseline and ws == 1:
        line["cpu_baseline"] = _cpu_baseline_line(cpu_build_sample, lambda t: 1.0 / t, "edge builds/s")
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
    q, k, v = gqa_block(HQ, HKV, 16384, D, 1007, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    ck = torch.randn(HKV, 7 * 1024, D, generator=g, device="cuda").to(torch.bfloat16)
    cv = torch.randn(HKV, 7 * 1024, D, generator=g, device="cuda").to(torch.bfloat16)
    cb = torch.randn(HKV, 7 * 1024, generator=g, device="cuda")
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
    wl = _layer_128k()
    blocks = local_blocks_of(wl.blocks, ws, rank)
    inputs = []
    for layer_i in range(args.layers):
        parts = [gqa_block(HQ, HKV, wl.block_len, D, 1000 * (layer_i + 1) + b, device="cuda") for b in blocks]
        inputs.append(tuple(torch.stack([p_[i] for p_ in parts]) for i in range(3)))
    kw = dict(device=dev)
    layer = DistributedDccKvLayer(wl.blocks, wl.block_len, HQ, HKV, D, wl.budgets, WINDOW, M_REPR, DP, **kw)
    stack = DistributedDccKvStack(wl.blocks, wl.block_len, HQ, HKV, D, wl.budgets, WINDOW, M_REPR, DP, **kw)
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
            "config": wl.config(parallelism=f"context parallel over {ws} GPUs"),
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
    wl = _layer_1m() if args.config == "cfg5" else _layer_128k()
    blocks = local_blocks_of(wl.blocks, ws, rank)
    parts = [gqa_block(HQ, HKV, wl.block_len, D, 1000 + b, device="cuda") for b in blocks]
    q, k, v = (torch.stack([p_[i] for p_ in parts]) for i in range(3))
    del parts
    layer = DistributedDccKvLayer(wl.blocks, wl.block_len, HQ, HKV, D, wl.budgets, WINDOW, M_REPR, DP, device=dev)
    if args.pool_first is not None:
        layer.pool_first = args.pool_first
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
        print(json.dumps({"study": "phase times", "n_gpus": ws, "steps": args.steps, "pool_first": layer.pool_first,
                          "config": wl.config(parallelism=f"context parallel over {ws} GPUs"),
                          "ranks": everyone}), flush=True)
    del layer
    _teardown(ws)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg4", choices=["cfg2", "cfg3", "cfg4", "cfg5"],
                    help="cfg4: the 128K layer (default, the headline); cfg2: 8-way merge microbench; "
                         "cfg3: batched GQA build of one edge; cfg5: the 1M layer with variable budgets")
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
    ap.add_argument("--pool-first", dest="pool_first", action="store_true", default=None,
                    help="--phase-times: the local attention waits for the pooling (default: only with one "
                         "block per rank)")
    ap.add_argument("--no-pool-first", dest="pool_first", action="store_false",
                    help="--phase-times: let the local attention start before the pooling finishes")
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
    elif args.config == "cfg2":
        run_merge(args)
    elif args.config == "cfg3":
        run_build(args)
    else:
        run_gpu(args, _layer_1m() if args.config == "cfg5" else _layer_128k())


if __name__ == "__main__":
    main()
