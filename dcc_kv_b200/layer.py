"""The DCC-KV sync layer on one GPU (all logical blocks resident).

Semantics (dcc_kv_sync_cpu.py:22-84 and compact_kv.py:50-118, in the
north-star direction): the context is split into ``n_blocks`` contiguous
blocks; block r attends causally to its own keys and, for every earlier
block s < r, to the compact KV C_{s->r} built from s's keys and values and
r's destination queries (per KV head: the first ``window`` queries of each
of its query heads, concatenated head by head), with the compact logit bias
added at full weight; the partial outputs are merged by online softmax.

Layout (HBM): block-major, head-major, contiguous --
    q [n_blocks, H_q, L, d], k / v [n_blocks, H_kv, L, d], out like q.
All buffers and kernel descriptors are built once per shape; ``forward``
on device inputs only enqueues kernels on the current stream:
    1 projection + 1 FPS launch       (all (destination, KV head) sets)
    6 build launches per <=128 edges  (score stats, score probs, top-k, three
                                       calibration launches)
    1 attention launch: per block its causal local segment followed by its
      compact segment with the logit bias, one online softmax over both (the
      merge of dcc_kv_sync_cpu.py:81-84 happens inside the kernel)
On host inputs the same kernels run block by block, pipelined with the
host <-> device copies (``_forward_host``).
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple, Union

import torch

from . import _lib as L
from .attention import attn_problem, kv_segment, run_attention
from .calibration import side_dtype
from .compact_kv import build_launch_count, build_problem, run_build_problems
from .representative_query import query_set, select_query_sets

Budgets = Union[int, Dict[Tuple[int, int], int]]


def budget_table(n_blocks: int, budgets: Budgets) -> Dict[Tuple[int, int], int]:
    if isinstance(budgets, int):
        return {(s, r): budgets for r in range(n_blocks) for s in range(r)}
    return {(s, r): int(budgets[(s, r)]) for r in range(n_blocks) for s in range(r)}


class DccKvSyncLayer:
    """One DCC-KV layer over ``n_blocks`` logical blocks on a single device."""

    def __init__(self, n_blocks: int, block_len: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                 budgets: Budgets, window: int, num_representative_queries: int = 64,
                 projection_dim: int = 32, lambda_beta: float = 1e-3, lambda_value: float = 1e-3,
                 seed: int = 42, dtype: torch.dtype = torch.bfloat16,
                 device: Union[str, torch.device] = "cuda"):
        if n_q_heads % n_kv_heads:
            raise ValueError("n_q_heads must be a multiple of n_kv_heads")
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("the layer runs in float32 (parity path) or bfloat16")
        self.nb, self.L, self.hq, self.hkv, self.d = n_blocks, block_len, n_q_heads, n_kv_heads, head_dim
        self.group = n_q_heads // n_kv_heads
        self.window = min(window, block_len)
        self.M = num_representative_queries
        self.m_eff = min(self.M, self.group * self.window)
        self.dp = projection_dim
        self.lb, self.lv, self.seed = lambda_beta, lambda_value, seed
        self.dtype = dtype
        self.code = L.dtype_code(torch.empty(0, dtype=dtype))
        self.device = torch.device(device)
        self.budgets = budget_table(n_blocks, budgets)
        dev, d = self.device, head_dim
        self.repr = torch.empty(n_blocks, n_kv_heads, self.m_eff, d, dtype=dtype, device=dev)
        self.repr_idx = torch.empty(n_blocks, n_kv_heads, self.m_eff, dtype=torch.int64, device=dev)
        # compact KV per destination r: the sources s < r concatenated, B' = min(B, L) rows each
        self.offsets: Dict[Tuple[int, int], int] = {}
        self.total = [0] * n_blocks
        for r in range(n_blocks):
            off = 0
            for s in range(r):
                self.offsets[(s, r)] = off
                off += min(self.budgets[(s, r)], block_len)
            self.total[r] = off
        sd = side_dtype(torch.empty(0, dtype=dtype))
        self.ck = [torch.empty(n_kv_heads, t, d, dtype=dtype, device=dev) for t in self.total]
        self.cv = [torch.empty(n_kv_heads, t, d, dtype=dtype, device=dev) for t in self.total]
        self.cb = [torch.empty(n_kv_heads, t, dtype=sd, device=dev) for t in self.total]
        self.ci = [torch.empty(n_kv_heads, t, dtype=torch.int64, device=dev) for t in self.total]
        self.out = torch.empty(n_blocks, n_q_heads, block_len, d, dtype=dtype, device=dev)
        self._bound = None
        self._bindings: Dict[Tuple[int, int, int, int], tuple] = {}
        self._ws, self._ws_bytes = None, 0
        self._ws2, self._ws2_bytes = None, 0
        self._host_out = None
        self._staging = None
        self._host_stream = None
        self._last_call_host = False
        self._streams = None
        # "batched" (default): pooling, the builds (two halves on two streams),
        # then one attention launch; "pipelined": builds on a side stream
        # overlapped with per-block attention (same results; on B200 the
        # batched order is ~1 % faster, as the build kernels hold the SMs
        # they run on either way)
        self.schedule = "batched"
        # optional per-step lists that collect (start, end) CUDA events around
        # each attention launch
        self.timing_events = None
        self.timing_index = 0
        self._errors = L.DeviceErrorWatch()

    # -- descriptors (rebuilt only when the input tensors change) ------------
    def _bind(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: Optional[torch.Tensor] = None) -> None:
        """Point the kernel descriptors at q, k, v and the device output
        ``out`` (default: the internal buffer ``self.out``).  Descriptor sets
        are cached per buffers (the host-buffer path alternates between two
        device staging sets), and the build workspaces are shared: they only
        grow."""
        out = self.out if out is None else out
        key = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr())
        if self._bound == key:
            return
        bound = self._bindings.get(key)
        if bound is None:
            bound = self._make_binding(q, k, v, out)
            if len(self._bindings) >= 4:
                self._bindings.pop(next(iter(self._bindings)))
            self._bindings[key] = bound
        (self.sets, self.sets_of, self.build, self.build_of, self.build_halves, self.attn_problems,
         (need, need2)) = bound
        if need > self._ws_bytes or need2 > self._ws2_bytes:
            if self._streams is not None:
                # the workspaces may still be in use by the side stream
                torch.cuda.current_stream(self.device).wait_stream(self._streams[1])
            if need > self._ws_bytes:
                self._ws, self._ws_bytes = L.workspace(need, self.device), need
            if need2 > self._ws2_bytes:
                self._ws2, self._ws2_bytes = L.workspace(need2, self.device), need2
        self._bound = key

    def _make_binding(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor):
        g = self.group
        sets = []
        # per destination block r: its query sets and the edges s -> r, as
        # slices of the batched lists (the host-buffer path runs them block by block)
        sets_of = [slice(0, 0)]
        build_of = [slice(0, 0)]
        for r in range(1, self.nb):
            sets_of.append(slice(len(sets), len(sets) + self.hkv))
            for h in range(self.hkv):
                sets.append(query_set(q[r, h * g], self.repr[r, h], self.repr_idx[r, h], n_seg=g,
                                      seg_rows=self.window, seg_stride=q.stride(1), row_stride=q.stride(2)))
        build = []
        for r in range(1, self.nb):
            build_of.append(slice(len(build), len(build) + r * self.hkv))
            for s in range(r):
                b = self.budgets[(s, r)]
                bp = min(b, self.L)
                o = self.offsets[(s, r)]
                for h in range(self.hkv):
                    build.append(build_problem(
                        k[s, h], v[s, h], self.repr[r, h], b, self.ck[r][h, o:o + bp], self.cv[r][h, o:o + bp],
                        self.cb[r][h, o:o + bp], self.ci[r][h, o:o + bp], num_repr=self.m_eff))
        # batched schedule: the edges split in two halves (by destination block)
        # that run on two streams, so the latency-bound calibration launches of
        # one half overlap those of the other
        half = len(build) // 2
        cut = min((sl.stop for sl in build_of[1:]), key=lambda e: abs(e - half), default=0)
        build_halves = [slice(0, cut), slice(cut, len(build))]

        def ws_bytes(probs):
            if not probs:
                return 0
            arr = (L.dcc_build_problem * len(probs))(*probs)
            return L.lib().dcc_build_compact_kv_workspace_bytes(arr, len(probs), self.d, self.d, self.code)

        need = max([ws_bytes(build[part]) for part in [slice(0, len(build)), build_halves[0]] + build_of[1:]] + [0])
        need2 = ws_bytes(build[build_halves[1]])
        # one attention problem per block: its causal local segment, then (for r >= 1)
        # the concatenated compact blocks with their logit bias -- the online softmax
        # runs over both in one pass, so no separate merge is needed
        attn_problems = []
        for b in range(self.nb):
            segs = [kv_segment(k[b], v[b])]
            if b > 0 and self.total[b] > 0:
                segs.append(kv_segment(self.ck[b], self.cv[b], self.cb[b]))
            attn_problems.append(attn_problem(q[b], out[b], None, segs, causal=True))
        return sets, sets_of, build, build_of, build_halves, attn_problems, (need, need2)

    def check_inputs(self, q, k, v):
        L.require_cuda(q, k, v)
        exp_q = (self.nb, self.hq, self.L, self.d)
        exp_kv = (self.nb, self.hkv, self.L, self.d)
        if tuple(q.shape) != exp_q or tuple(k.shape) != exp_kv or tuple(v.shape) != exp_kv:
            raise ValueError(f"expected q {exp_q}, k/v {exp_kv}; got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
        for t in (q, k, v):
            if t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError(f"inputs must be contiguous {self.dtype}")

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """q [nb, H_q, L, d], k / v [nb, H_kv, L, d] -> out [nb, H_q, L, d].

        Device inputs: the returned tensor is an internal buffer, reused by
        the next call.  Host inputs (CPU tensors, pinned for overlap): the
        call streams them in block by block and returns ``out`` (or an
        internal pinned host buffer); like a ``non_blocking`` copy it is
        complete once the current stream is synchronized."""
        self._errors.poll()
        if not q.is_cuda:
            out = self._forward_host(q, k, v, out)
            self._errors.record(self._host_stream)
            return out
        self.check_inputs(q, k, v)
        if self._host_stream is not None and self._last_call_host:
            # the internal buffers were last used by the host-buffer path's stream
            torch.cuda.current_stream(self.device).wait_stream(self._host_stream)
        self._last_call_host = False
        self._bind(q, k, v)
        if self.schedule == "batched":
            self._forward_batched()
        else:
            self._ensure_streams()
            self._run_blocks(pool_all=True)
        self._errors.record(torch.cuda.current_stream(self.device))
        return self.out

    __call__ = forward

    def check(self) -> None:
        """Synchronise the device and raise ``DccError(DCC_ERR_TIMEOUT)`` if a
        bounded device wait of any forward so far gave up (each forward
        checks the ones before it without synchronising)."""
        self._errors.check(self.device)

    def _attention(self, problems) -> None:
        dev = self.device
        main = torch.cuda.current_stream(dev)
        ev = None
        if self.timing_events:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.timing_events[self.timing_index].append(ev)
            ev[0].record(main)
        run_attention(problems, self.hq, self.hkv, self.d, 1.0 / math.sqrt(self.d), self.code, dev)
        if ev is not None:
            ev[1].record(main)

    def _forward_batched(self) -> None:
        """All pooling, all builds (two halves on two streams), then one
        attention launch over every block."""
        dev = self.device
        select_query_sets(self.sets, self.d, self.M, self.dp, self.seed, self.code, dev)
        first, second = (self.build[part] for part in self.build_halves)
        if second:
            self._ensure_streams()
            main, aux = torch.cuda.current_stream(dev), self._streams[1]
            aux.wait_stream(main)  # representative queries ready
            with torch.cuda.stream(aux):
                run_build_problems(second, self.d, self.d, self.lb, self.lv, self.code, dev, self._ws2)
            run_build_problems(first, self.d, self.d, self.lb, self.lv, self.code, dev, self._ws)
            main.wait_stream(aux)
        else:
            run_build_problems(first, self.d, self.d, self.lb, self.lv, self.code, dev, self._ws)
        self._attention(self.attn_problems)

    def _ensure_streams(self) -> None:
        if self._streams is None:
            dev = self.device
            lo, hi = torch.cuda.Stream.priority_range()
            # copy-in, builds (high priority: their few CTAs are dispatched ahead
            # of the attention CTAs that fill the GPU), copy-out
            self._streams = tuple(torch.cuda.Stream(device=dev, priority=p) for p in (0, hi, 0))
            self._events = [[torch.cuda.Event() for _ in range(self.nb)] for _ in range(4)]

    def _run_blocks(self, pool_all: bool, copy_in=None, copy_out=None, inputs_free=None,
                    inputs_done=None, drained=None) -> None:
        """Per-block schedule.  Side stream (high priority): pooling, then for
        b = 1 .. nb-1 the builds s -> b; current stream: attention of block b
        as soon as its compacts are built (block 0 needs none and starts at
        once), so the latency-bound pooling / build kernels share the GPU
        with attention instead of running before it.  ``copy_in(b)`` /
        ``copy_out(b)``, when given, run on the copy-in / copy-out streams;
        the copy-in waits for ``inputs_free`` (the last compute that read the
        staging buffers), ``inputs_done`` is recorded once this call's
        compute no longer reads them, and ``drained[b]`` (waited before block
        b's attention overwrites its output, recorded after its copy-out)
        belongs to the device output buffer in use."""
        dev = self.device
        h2d, side, d2h = self._streams
        copied, built, attended = self._events[:3]
        main = torch.cuda.current_stream(dev)
        if copy_in is not None:
            if inputs_free is not None:
                h2d.wait_event(inputs_free)
            with torch.cuda.stream(h2d):
                for b in range(self.nb):
                    copy_in(b)
                    copied[b].record(h2d)
        side.wait_stream(main)
        if pool_all:
            with torch.cuda.stream(side):
                select_query_sets(self.sets, self.d, self.M, self.dp, self.seed, self.code, dev)
        for b in range(self.nb):
            if b > 0:
                with torch.cuda.stream(side):
                    if copy_in is not None:
                        side.wait_event(copied[b])
                    if not pool_all:
                        select_query_sets(self.sets[self.sets_of[b]], self.d, self.M, self.dp, self.seed,
                                          self.code, dev)
                    run_build_problems(self.build[self.build_of[b]], self.d, self.d, self.lb, self.lv,
                                       self.code, dev, self._ws)
                    built[b].record(side)
                main.wait_event(built[b])
            if copy_in is not None:
                main.wait_event(copied[b])
            if copy_out is not None:
                main.wait_event(drained[b])  # the last copy-out from this output buffer
            self._attention([self.attn_problems[b]])
            if copy_out is not None:
                attended[b].record(main)
                d2h.wait_event(attended[b])
                with torch.cuda.stream(d2h):
                    copy_out(b)
                    drained[b].record(d2h)
        if self.nb == 1:
            main.wait_stream(side)
        if inputs_done is not None:
            inputs_done.record(main)

    def _forward_host(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      out: Optional[torch.Tensor]) -> torch.Tensor:
        """Host buffers in and out, pipelined per block over four streams:
        copy-in of block b (h2d) || pooling of b + builds s -> b (high-priority
        side stream) || attention of b (current stream) || copy-out of block
        b (d2h).  Block b's builds only need the keys / values of blocks
        s < b, which arrived earlier, so the copies hide behind the compute.
        Consecutive calls alternate between two device staging sets, so the
        copy-in of one call overlaps the compute of the previous one."""
        exp_q = (self.nb, self.hq, self.L, self.d)
        exp_kv = (self.nb, self.hkv, self.L, self.d)
        for t, shp in ((q, exp_q), (k, exp_kv), (v, exp_kv)):
            if t.is_cuda or tuple(t.shape) != shp or t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError(f"host inputs must be contiguous CPU {self.dtype} tensors of shape "
                                 f"q {exp_q}, k/v {exp_kv}")
        if out is None:
            if self._host_out is None:
                self._host_out = torch.empty(exp_q, dtype=self.dtype).pin_memory()
            out = self._host_out
        elif out.is_cuda or tuple(out.shape) != exp_q or out.dtype != self.dtype or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous CPU {self.dtype} tensor of shape {exp_q}")
        dev = self.device
        if self._staging is None:
            # two device staging sets (inputs and output), alternated by
            # consecutive calls
            self._staging = [(torch.empty(exp_q, dtype=self.dtype, device=dev),
                              torch.empty(exp_kv, dtype=self.dtype, device=dev),
                              torch.empty(exp_kv, dtype=self.dtype, device=dev),
                              torch.empty(exp_q, dtype=self.dtype, device=dev)) for _ in range(2)]
            # recorded once a call's compute no longer reads staging set i
            self._staging_done = [None, None]
            # per set and block: recorded after the copy-out of that block
            self._drained = [[torch.cuda.Event() for _ in range(self.nb)] for _ in range(2)]
            self._host_calls = 0
            self._host_stream = torch.cuda.Stream(device=dev)
        self._ensure_streams()
        caller = torch.cuda.current_stream(dev)
        if not self._last_call_host:
            # device-path work on the caller's stream may still use the internal buffers
            self._host_stream.wait_stream(caller)
        self._last_call_host = True
        i = self._host_calls % 2
        self._host_calls += 1
        dq, dk_, dv, dout = self._staging[i]
        self._bind(dq, dk_, dv, dout)
        free = self._staging_done[i]
        self._staging_done[i] = torch.cuda.Event()

        def copy_in(b):
            dq[b].copy_(q[b], non_blocking=True)
            dk_[b].copy_(k[b], non_blocking=True)
            dv[b].copy_(v[b], non_blocking=True)

        def copy_out(b):
            out[b].copy_(dout[b], non_blocking=True)

        # the compute runs on an internal stream that does not wait for the
        # copy-out, so the next call's compute can start under this call's
        # last copies; the caller's stream waits for the output
        with torch.cuda.stream(self._host_stream):
            self._run_blocks(pool_all=False, copy_in=copy_in, copy_out=copy_out, inputs_free=free,
                             inputs_done=self._staging_done[i], drained=self._drained[i])
        caller.wait_stream(self._streams[2])
        return out

    def launches_per_forward(self) -> int:
        """Kernel launches one device-input forward enqueues (batch caps of
        the C library: 64 query sets, 128 build edges, 8 tcgen05 attention
        problems per launch)."""
        sets = len(self.sets)
        pool = 0 if sets == 0 else (2 if self.m_eff < self.group * self.window else 1) * -(-sets // 64)
        if self.schedule == "batched":
            build = sum(build_launch_count(len(self.build[part]), self.code, self.d) for part in self.build_halves)
            attn = -(-len(self.attn_problems) // 8)
        else:
            build = sum(build_launch_count(len(self.build[part]), self.code, self.d) for part in self.build_of)
            attn = len(self.attn_problems)
        return pool + build + attn + 1  # + the error-flag report

    def compact(self, s: int, r: int, h: int):
        """The CompactKV C_{s->r} of KV head h from the last forward."""
        from .compact_kv import CompactKV
        o = self.offsets[(s, r)]
        bp = min(self.budgets[(s, r)], self.L)
        return CompactKV(self.ck[r][h, o:o + bp], self.cb[r][h, o:o + bp], self.cv[r][h, o:o + bp],
                         self.ci[r][h, o:o + bp])
