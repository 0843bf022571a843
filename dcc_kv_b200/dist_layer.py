"""The DCC-KV sync layer sharded by sequence block over one process per GPU.

Logical blocks are dealt to ranks in snake order (0, 1, .., G-1, G-1, ..,
1, 0, 0, 1, ..): block r attends to r compact blocks and block s builds
n_blocks - 1 - s edges, so pairing block b with its mirror n_blocks - 1 - b
on one rank balances both (for 8 blocks on 4 ranks every rank gets 7 compact
blocks; round-robin would give 4 to 10).  One forward on every rank:

  0. pooling: representative queries of the local destination blocks
     (FP64 FPS), then ``all_gather`` of the [n_local, H_kv, M, d] tensors
     (the only collective before the exchange; ~128 KB per rank);
     steps 0-2 run on a high-priority side stream;
  1. builds: every local source s builds C_{s->r} for every r > s, written
     straight into the wire layout (var_len_msg.EdgeLayout) of a
     per-destination-rank send buffer (edges between co-resident blocks go
     to a local buffer and never touch NCCL);
  2. exchange: one NCCL all-to-allv of the byte buffers on a side stream,
     through ``DistributedComm.all_to_all_v`` (the reference's interface),
     sizes known from the shared budget table (no size round trip);
  3. local causal attention on the main stream from the start, overlapped
     with (0)-(2);
  4. compact attention with logit bias, one KV segment per source edge,
     read in place from the receive / local buffers, continuing each
     block's online softmax from the local (O, LSE) in place -- the merge
     (online_softmax.py:92-111) happens inside that launch;
  5. with one block per rank only (``default_help``): the compact attention
     of a heavy block's first KV heads runs on its mirror block's rank -- the
     query heads of those KV heads go there once (point-to-point on a
     communicator of their own, so the transfer waits only for the inputs),
     the builds route those KV heads of every source edge there, that rank
     attends with them, and the partial (O, LSE) comes back and is merged.

``DistPlan`` is the pure host-side routing (offsets and split sizes),
identical on every rank and testable without a GPU.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from .attention import attn_problem, kv_segment, run_attention
from .comm import DistributedComm, VarLenMessage
from .compact_kv import build_launch_count, build_problem, run_build_problems
from .layer import Budgets, budget_table
from .online_softmax import merge_lse
from .representative_query import query_set, select_query_sets
from .var_len_msg import EdgeLayout


def block_owner(b: int, world: int) -> int:
    """Rank of logical block b: snake order over the ranks."""
    m = b % (2 * world)
    return m if m < world else 2 * world - 1 - m


def local_blocks_of(n_blocks: int, world: int, rank: int) -> List[int]:
    """The logical blocks of ``rank`` in ascending order -- the order of the
    local block dimension of its inputs and outputs."""
    return [b for b in range(n_blocks) if block_owner(b, world) == rank]


# Cost model of the hand-off, in FLOP-equivalents of attention work (measured
# on B200 with the 128K layer at one block per GPU): a build problem (one
# edge and KV head) slows the attention it shares the GPU with by ~7.9e9
# FLOP-equivalents per 16384 source keys; a byte handed to or from the
# helper costs ~3.7e3 (NCCL point-to-point ~270 GB/s against ~1e15 FLOP/s
# of attention).
BUILD_FLOP_PER_16K_KEYS = 7.9e9
HANDOFF_FLOP_PER_BYTE = 3.7e3


def default_help(n_blocks: int, world: int, block_len: int, n_kv_heads: int, q_per_kv: int, head_dim: int,
                 budgets, elem_bytes: int = 2) -> Dict[int, int]:
    """With one block per rank the compact attention is unbalanced (block r
    attends to r compact blocks, and block s builds n_blocks - 1 - s edges).
    Block r > its mirror p = n_blocks - 1 - r hands the compact attention of
    its first k KV heads (their q_per_kv query heads each) to p's rank; k
    minimises the larger of the two ranks' estimated work (local causal
    attention + builds + compact attention + the return of the helper's
    partial output; the query transfer runs under the local attention).
    Returns {r: k} for the hand-offs that save at least 2 %."""
    if world != n_blocks:
        return {}
    table = budget_table(n_blocks, budgets)
    L, hq = block_len, n_kv_heads * q_per_kv
    pair = 4.0 * head_dim  # FLOPs per (query row, key) per query head
    local = L * (L + 1) / 2 * hq * pair
    build = BUILD_FLOP_PER_16K_KEYS * L / 16384.0

    def compact(b):
        return L * hq * pair * sum(min(table[(s, b)], L) for s in range(b))

    def builds(b):
        return (n_blocks - 1 - b) * n_kv_heads * build

    help_ = {}
    for r in range(n_blocks):
        p = n_blocks - 1 - r
        if r <= p:
            continue
        best_k, best_t = 0, None
        for k in range(n_kv_heads):
            f = k / n_kv_heads
            # the partial output comes back after the helper's attention; the
            # query transfer runs under the local attention and is not counted
            xfer = k * q_per_kv * L * head_dim * elem_bytes * HANDOFF_FLOP_PER_BYTE
            t_owner = local + builds(r) + (1 - f) * compact(r)
            t_helper = local + builds(p) + compact(p) + f * compact(r) + xfer
            t = max(t_owner, t_helper)
            if best_t is None or t < best_t:
                best_k, best_t = k, t
        # a hand-off that saves under 2 % is not worth its transfers and merge
        t_none = max(local + builds(r) + compact(r), local + builds(p) + compact(p))
        if best_k > 0 and best_t < 0.98 * t_none:
            help_[r] = best_k
    return help_


class DistPlan:
    """Routing of every compact-KV edge (s -> r, s < r) for G ranks, per KV
    head: head g of edge (s, r) goes to the rank that attends with it -- the
    owner of r, or, for the first ``help[r]`` KV heads of a helped block r,
    the owner of r's mirror block.  Units (s, r, g) sit in a buffer in
    (r, s, g) order, so the heads of one edge on one rank are contiguous."""

    def __init__(self, n_blocks: int, world: int, block_len: int, n_kv_heads: int, head_dim: int,
                 budgets: Budgets, elem_bytes: int = 2, help_heads: Optional[Dict[int, int]] = None,
                 q_per_kv: int = 4):
        if n_blocks % world:
            raise ValueError(f"{n_blocks} blocks do not split evenly over {world} ranks")
        self.nb, self.world, self.L, self.hkv = n_blocks, world, block_len, n_kv_heads
        self.n_local = n_blocks // world
        self.budgets = budget_table(n_blocks, budgets)
        self.layout = {e: EdgeLayout(n_kv_heads, min(b, block_len), head_dim, elem_bytes)
                       for e, b in self.budgets.items()}
        if help_heads is None:
            help_heads = default_help(n_blocks, world, block_len, n_kv_heads, q_per_kv, head_dim,
                                      self.budgets, elem_bytes)
        self.help = {r: k for r, k in help_heads.items() if k > 0}
        for r, k in self.help.items():
            if not (0 < k < n_kv_heads) or not (0 < r < n_blocks) or self.helper(r) == self.owner(r) \
                    or self.n_local != 1:
                raise ValueError(f"block {r}: cannot hand {k} KV heads to rank {self.helper(r)}")
        units = sorted(((s, r, g) for (s, r) in self.budgets for g in range(n_kv_heads)),
                       key=lambda u: (u[1], u[0], u[2]))
        # units from rank i to rank j, in (r, s, g) order
        self.units_ij = {(i, j): [] for i in range(world) for j in range(world)}
        for u in units:
            self.units_ij[(self.owner(u[0]), self.consumer(u))].append(u)
        self.bytes_ij = {ij: sum(self.layout[(u[0], u[1])].head_bytes for u in us)
                         for ij, us in self.units_ij.items()}

    def owner(self, b: int) -> int:
        return block_owner(b, self.world)

    def helper(self, r: int) -> int:
        """Rank that takes part of block r's compact attention (its mirror's owner)."""
        return self.owner(self.nb - 1 - r)

    def consumer(self, u: Tuple[int, ...]) -> int:
        """Rank whose attention reads KV head g of edge (s, r), u = (s, r, g)."""
        s, r, g = u
        return self.helper(r) if g < self.help.get(r, 0) else self.owner(r)

    def heads_on(self, rank: int, e: Tuple[int, int]) -> Tuple[int, int]:
        """KV heads [lo, hi) of edge e that ``rank`` attends with (lo == hi: none)."""
        s, r = e
        k = self.help.get(r, 0)
        if rank == self.owner(r):
            return (k, self.hkv)
        if k > 0 and rank == self.helper(r):
            return (0, k)
        return (0, 0)

    def helped_by(self, rank: int) -> List[int]:
        """Blocks of other ranks part of whose compact attention ``rank`` computes."""
        return [r for r in sorted(self.help) if self.helper(r) == rank]

    def local_index(self, b: int) -> int:
        return self.local_blocks(self.owner(b)).index(b)

    def local_blocks(self, rank: int) -> List[int]:
        return local_blocks_of(self.nb, self.world, rank)

    def send_splits(self, rank: int) -> List[int]:
        return [0 if j == rank else self.bytes_ij[(rank, j)] for j in range(self.world)]

    def recv_splits(self, rank: int) -> List[int]:
        return [0 if i == rank else self.bytes_ij[(i, rank)] for i in range(self.world)]

    def _place(self, units, buf, out, off=0):
        for u in units:
            out[u] = (buf, off)
            off += self.layout[(u[0], u[1])].head_bytes
        return off

    def send_offsets(self, rank: int) -> Dict[Tuple[int, int, int], Tuple[str, int]]:
        """Where rank's builds write each outgoing unit (s, r, g): ("send"|"local", byte offset)."""
        out, off = {}, 0
        for j in range(self.world):
            if j != rank:
                off = self._place(self.units_ij[(rank, j)], "send", out, off)
        self._place(self.units_ij[(rank, rank)], "local", out)
        return out

    def recv_offsets(self, rank: int) -> Dict[Tuple[int, int, int], Tuple[str, int]]:
        """Where each unit that rank attends with sits: ("recv"|"local", byte offset)."""
        out, off = {}, 0
        for i in range(self.world):
            if i != rank:
                off = self._place(self.units_ij[(i, rank)], "recv", out, off)
        self._place(self.units_ij[(rank, rank)], "local", out)
        return out


class DistributedDccKvLayer:
    """One process per GPU; block-major local inputs
    q [n_local, H_q, L, d], k / v [n_local, H_kv, L, d] for the blocks
    ``local_blocks_of(n_blocks, G, rank)`` of the context, ascending."""

    def __init__(self, n_blocks: int, block_len: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                 budgets: Budgets, window: int, num_representative_queries: int = 64, projection_dim: int = 32,
                 lambda_beta: float = 1e-3, lambda_value: float = 1e-3, seed: int = 42,
                 dtype: torch.dtype = torch.bfloat16, device=None, group=None,
                 help_heads: Optional[Dict[int, int]] = None, p2p_group=None):
        """``help_heads`` ({block: KV heads}) overrides the default hand-off
        of compact attention from heavy blocks to their mirror's rank (see
        ``default_help``; only with one block per rank).

        Communicators: with ``group`` None every rank creates two of its own
        here (collective calls), both with high-priority NCCL streams, so
        their kernels are dispatched ahead of the attention that fills the
        GPU: one for the exchange (all-gather and all-to-allv) and one for
        the hand-off's point-to-point transfers.  NCCL runs the operations
        of one communicator in issue order on one internal stream, so on a
        shared one the query transfer would queue behind the all-to-allv,
        which waits for the builds.  With a sub-``group`` the exchange runs
        on it, and the transfers on ``p2p_group`` if given, else on it too."""
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.nb, self.L, self.hq, self.hkv, self.d = n_blocks, block_len, n_q_heads, n_kv_heads, head_dim
        self.qgroup = n_q_heads // n_kv_heads
        self.window = min(window, block_len)
        self.M = num_representative_queries
        self.m_eff = min(self.M, self.qgroup * self.window)
        self.dp, self.lb, self.lv, self.seed = projection_dim, lambda_beta, lambda_value, seed
        self.dtype = dtype
        self.code = L.dtype_code(torch.empty(0, dtype=dtype))
        self.plan = DistPlan(n_blocks, self.world, block_len, n_kv_heads, head_dim, budgets,
                             torch.empty(0, dtype=dtype).element_size(), help_heads, self.qgroup)
        self.n_local = self.plan.n_local
        self.local_blocks = self.plan.local_blocks(self.rank)
        dev = self.device
        self.repr_local = torch.zeros(self.n_local, n_kv_heads, self.m_eff, head_dim, dtype=dtype, device=dev)
        self.repr_idx = torch.empty(self.n_local, n_kv_heads, self.m_eff, dtype=torch.int64, device=dev)
        self.repr_all = torch.empty(self.world, self.n_local, n_kv_heads, self.m_eff, head_dim, dtype=dtype,
                                    device=dev)
        send_splits = self.plan.send_splits(self.rank)
        recv_splits = self.plan.recv_splits(self.rank)
        self.send_splits, self.recv_splits = send_splits, recv_splits
        local_bytes = self.plan.bytes_ij[(self.rank, self.rank)]
        self.send_buf = torch.empty(max(sum(send_splits), 256), dtype=torch.uint8, device=dev)
        self.recv_buf = torch.empty(max(sum(recv_splits), 256), dtype=torch.uint8, device=dev)
        self.local_buf = torch.empty(max(local_bytes, 256), dtype=torch.uint8, device=dev)
        self.bufs = {"send": self.send_buf, "recv": self.recv_buf, "local": self.local_buf}
        # per-edge selected indices stay on the source rank
        self.sel_idx = {e: torch.empty(n_kv_heads, self.plan.layout[e].rows, dtype=torch.int64, device=dev)
                        for e in sorted({(s, r) for (s, r, g) in self.plan.send_offsets(self.rank)})}
        self.o_loc = torch.empty(self.n_local, n_q_heads, block_len, head_dim, dtype=dtype, device=dev)
        self.lse_loc = torch.empty(self.n_local, n_q_heads, block_len, dtype=torch.float32, device=dev)
        # compact attention handed between mirror ranks (one block per rank):
        # the query heads of a helped block's first KV heads go to the
        # helper, which attends with those heads of every compact source; its
        # partial (O, LSE) for them comes back and is merged
        self.helped = [r for r in self.local_blocks if r in self.plan.help]
        self.helping = self.plan.helped_by(self.rank)
        g = self.qgroup

        def qshape(r):
            return (self.plan.help[r] * g, block_len, head_dim)

        self.q_help = {r: torch.empty(qshape(r), dtype=dtype, device=dev) for r in self.helping}
        self.o_help = {r: torch.empty(qshape(r), dtype=dtype, device=dev) for r in self.helping}
        self.lse_help = {r: torch.empty(qshape(r)[:2], dtype=torch.float32, device=dev) for r in self.helping}
        self.o_from = {r: torch.empty(qshape(r), dtype=dtype, device=dev) for r in self.helped}
        self.lse_from = {r: torch.empty(qshape(r)[:2], dtype=torch.float32, device=dev) for r in self.helped}
        self.p2p_stream = torch.cuda.Stream(device=dev)
        self.xgroup, self.p2p_group = group, p2p_group
        if group is None and self.world > 1 and dist.get_backend() == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
            ranks = list(range(self.world))
            self.xgroup = dist.new_group(ranks=ranks, pg_options=opts)
            if self.plan.help and p2p_group is None:
                self.p2p_group = dist.new_group(ranks=ranks, pg_options=opts)
                # the first operation on a communicator must involve all of
                # its ranks; the hand-off transfers involve only some
                dist.barrier(group=self.p2p_group)
        if self.p2p_group is None:
            self.p2p_group = self.xgroup
        # the exchange goes through the reference-interface wrapper
        # (comm.py:174-280): sizes from the shared budget table (no size round
        # trip), payloads already back to back in the send buffer, received
        # in place
        self.comm = DistributedComm(backend=dist.get_backend(self.xgroup), group=self.xgroup)
        self.comm.init(self.rank, self.world)
        offs = [sum(send_splits[:j]) for j in range(self.world)]
        self._messages = [VarLenMessage(payload=self.send_buf[o:o + n]) for o, n in zip(offs, send_splits)]
        # pooling, the gather, the builds and the exchange run on a high-priority
        # side stream, so their kernels are dispatched ahead of the local
        # attention that fills the GPU meanwhile on the main stream
        lo, hi = torch.cuda.Stream.priority_range()
        self.comm_stream = torch.cuda.Stream(device=dev, priority=hi)
        # False: pooling, builds and exchange on the main stream before any
        # attention (no communication-computation overlap; same outputs)
        self.overlap_exchange = True
        # True: the local attention waits for the pooling, which then runs on
        # an idle GPU (its farthest-point-sampling clusters need several free
        # SMs of one GPC at once; behind the attention CTAs they wait for
        # them), so the gather, the builds and the exchange start sooner.  On
        # by default with one block per rank, where the exchange is on the
        # critical path; with several blocks per rank the local attention is
        # long enough to hide it, and the wait would only delay the attention
        self.pool_first = self.n_local == 1
        self._bound = None
        self._bindings = {}
        self._host_stream = None
        self._last_call_host = False
        self._ws, self._ws_bytes = None, 0
        self.timing_events = None
        self.timing_index = 0
        # optional list that collects, per forward, {phase: CUDA event}
        # recorded on the stream that runs the phase (phase_times())
        self.phase_events = None
        self._errors = L.DeviceErrorWatch()

    def _mark(self, name: str, stream) -> None:
        if self.phase_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            self.phase_events[-1][name] = ev

    @staticmethod
    def phase_times(log) -> Dict[str, float]:
        """Mean milliseconds from the start of a forward to each recorded
        phase end, over the forwards in ``log`` (a ``phase_events`` list)."""
        acc: Dict[str, float] = {}
        for step in log:
            t0 = step["start"]
            for name, ev in step.items():
                if name != "start":
                    acc[name] = acc.get(name, 0.0) + t0.elapsed_time(ev) / len(log)
        return acc

    def _bind(self, q, k, v, o=None, lse=None):
        """Point the kernel descriptors at q, k, v and the device output /
        LSE buffers (default: the internal ``o_loc`` / ``lse_loc``);
        descriptor sets are cached per buffers (the host-buffer path
        alternates between two device staging sets) and the build workspace
        only grows."""
        o = self.o_loc if o is None else o
        lse = self.lse_loc if lse is None else lse
        key = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr())
        if self._bound == key:
            return
        bound = self._bindings.get(key)
        if bound is None:
            bound = self._make_binding(q, k, v, o, lse)
            if len(self._bindings) >= 8:
                self._bindings.pop(next(iter(self._bindings)))
            self._bindings[key] = bound
        (self.sets, self.build, self.local_problems, self.compact_calls, self.helper_calls, self.merges,
         need) = bound
        if need > self._ws_bytes:
            # the workspace may still be in use by the side stream
            torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
            self._ws, self._ws_bytes = L.workspace(need, self.device), need
        self._bound = key

    def _make_binding(self, q, k, v, o, lse):
        g = self.qgroup
        sets = [query_set(q[li, h * g], self.repr_local[li, h], self.repr_idx[li, h], n_seg=g,
                               seg_rows=self.window, seg_stride=q.stride(1), row_stride=q.stride(2))
                for li, b in enumerate(self.local_blocks) if b > 0 for h in range(self.hkv)]
        send_off = self.plan.send_offsets(self.rank)
        build = []
        for (s, r, h), (buf, off) in sorted(send_off.items()):
            lay = self.plan.layout[(s, r)]
            ko, vo, bo = lay.views(self.bufs[buf], off, self.dtype, n_heads=1)
            rep = self.repr_all[self.plan.owner(r), self.plan.local_index(r)]
            ls = self.plan.local_index(s)
            build.append(build_problem(k[ls, h], v[ls, h], rep[h], self.plan.budgets[(s, r)], ko[0], vo[0],
                                       bo[0], self.sel_idx[(s, r)][h], num_repr=self.m_eff))
        need = 0
        if build:
            arr = (L.dcc_build_problem * len(build))(*build)
            need = L.lib().dcc_build_compact_kv_workspace_bytes(arr, len(build), self.d, self.d, self.code)
        local_problems = [attn_problem(q[li], o[li], lse[li], [kv_segment(k[li], v[li])],
                                       causal=True) for li in range(self.n_local)]
        recv_off = self.plan.recv_offsets(self.rank)

        def consumed_segments(r):
            """This rank's KV heads [lo, hi) of every compact source of block r."""
            segs, heads = [], None
            for s in range(r):
                lo, hi = self.plan.heads_on(self.rank, (s, r))
                if lo == hi:
                    continue
                heads = (lo, hi)
                buf, off = recv_off[(s, r, lo)]
                ko, vo, bo = self.plan.layout[(s, r)].views(self.bufs[buf], off, self.dtype, n_heads=hi - lo)
                segs.append(kv_segment(ko, vo, bo))
            return segs, heads

        # the compact blocks continue each local block's online softmax from
        # its (O, LSE), in place: the merge needs no separate pass.  Launches
        # are grouped by head range: (problems, first query head, query heads).
        compact_calls, merges = [], []
        plain = []
        for li, r in enumerate(self.local_blocks):
            segs, heads = consumed_segments(r)
            if r in self.helped:
                # this rank attends with KV heads [k, H_kv) (query heads [k g, H_q));
                # the helper's partial for query heads [0, k g) is merged afterwards
                kq = self.plan.help[r] * g
                if segs:
                    compact_calls.append(([attn_problem(q[li, kq:], o[li, kq:], None, segs,
                                                        o_init=o[li, kq:], lse_init=lse[li, kq:])],
                                          self.hq - kq, self.hkv - kq // g))
                merges.append((q[li, :kq], o[li, :kq], lse[li, :kq], r))
            elif segs:
                plain.append(attn_problem(q[li], o[li], None, segs, o_init=o[li], lse_init=lse[li]))
        if plain:
            compact_calls.insert(0, (plain, self.hq, self.hkv))
        # this rank's part of other ranks' blocks: their first query heads over
        # those KV heads of every source
        helper_calls = []
        for r in self.helping:
            segs, _ = consumed_segments(r)
            kq = self.plan.help[r] * g
            helper_calls.append(([attn_problem(self.q_help[r], self.o_help[r], self.lse_help[r], segs)], kq, kq // g))
        return sets, build, local_problems, compact_calls, helper_calls, merges, need

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
        """Local blocks q [n_local, H_q, L, d], k / v [n_local, H_kv, L, d] ->
        their outputs.  Device inputs: returns an internal buffer.  Host
        inputs (CPU, pinned for overlap): the copies are pipelined with the
        compute and ``out`` (or an internal pinned buffer) is returned,
        complete once the current stream is synchronized."""
        exp_q = (self.n_local, self.hq, self.L, self.d)
        exp_kv = (self.n_local, self.hkv, self.L, self.d)
        if tuple(q.shape) != exp_q or tuple(k.shape) != exp_kv or tuple(v.shape) != exp_kv:
            raise ValueError(f"expected local q {exp_q}, k/v {exp_kv}")
        self._errors.poll()
        host = not q.is_cuda
        for t in (q, k, v):
            if t.dtype != self.dtype or not t.is_contiguous() or (not host and t.device != self.device) or \
                    (host and t.is_cuda):
                raise ValueError(f"inputs must be contiguous {self.dtype}, all on {self.device} or all on the host")
        if host:
            out = self._forward_host(q, k, v, out)
            self._errors.record(self._host_stream)
            return out
        if self._host_stream is not None and self._last_call_host:
            # the internal buffers were last used by the host-buffer path's stream
            torch.cuda.current_stream(self.device).wait_stream(self._host_stream)
        self._last_call_host = False
        self._bind(q, k, v)
        self._run()
        self._errors.record(torch.cuda.current_stream(self.device))
        return self.o_loc

    __call__ = forward

    def check(self) -> None:
        """Synchronise the device and raise ``DccError(DCC_ERR_TIMEOUT)`` if a
        bounded device wait of any forward so far gave up on this rank."""
        self._errors.check(self.device)

    def _peer(self, group_rank: int) -> int:
        return group_rank if self.group is None else dist.get_global_rank(self.group, group_rank)

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

    def _run(self, windows_ready=None, kv_ready=None, q_ready=None, merged=None, side_waits=None,
             done=None) -> None:
        """One forward on bound buffers.  The optional per-phase events gate
        the work on host-to-device copies (pooling on the query windows,
        builds on K / V, local attention of block li on its queries) and
        ``merged[li]`` is recorded once block li's output is final.  The side
        stream waits for the main stream (inputs written, the previous
        forward done with the exchange buffers) unless ``side_waits`` names
        the events to wait for instead; ``done`` is recorded after the
        compact attention, the last reader of the exchange buffers.  With
        ``overlap_exchange`` off, the pooling, builds and exchange run on the
        main stream before any attention (the synchronous baseline)."""
        dev = self.device
        main = torch.cuda.current_stream(dev)
        side = self.comm_stream if self.overlap_exchange else main
        if self.phase_events is not None:
            self.phase_events.append({})
            self._mark("start", main)
        if side is not main:
            if side_waits is None:
                side.wait_stream(main)  # inputs written, previous step's buffers released
            else:
                for e in side_waits:
                    side.wait_event(e)
        with torch.cuda.stream(side):
            if windows_ready is not None:
                side.wait_event(windows_ready)
            select_query_sets(self.sets, self.d, self.M, self.dp, self.seed, self.code, dev)
            self._mark("pooling", side)
            if self.pool_first and side is not main and self.sets:
                pooled = torch.cuda.Event()
                pooled.record(side)
                main.wait_event(pooled)
            dist.all_gather_into_tensor(self.repr_all, self.repr_local, group=self.xgroup)
            self._mark("gather", side)
            if kv_ready is not None:
                side.wait_event(kv_ready)
            run_build_problems(self.build, self.d, self.d, self.lb, self.lv, self.code, dev, self._ws)
            self._mark("builds", side)
            ns, nr = sum(self.send_splits), sum(self.recv_splits)
            self.comm.all_to_all_v(self._messages, send_sizes=self.send_splits, recv_sizes=self.recv_splits,
                                   trust_recv_sizes=True, out=self.recv_buf[:nr], packed=self.send_buf[:ns])
            self._mark("exchange", side)
        # helped blocks' queries to their helpers (after the collectives in
        # issue order, on a stream that waits only for the inputs)
        q_reqs = []
        if self.helped or self.helping:
            p2p = self.p2p_stream
            p2p.wait_stream(main)  # inputs written, the previous helper attention done with q_help
            if q_ready is not None:
                for li in range(self.n_local):
                    p2p.wait_event(q_ready[li])
            ops = [dist.P2POp(dist.isend, q_send, self._peer(self.plan.helper(r)), self.p2p_group)
                   for (q_send, _, _, r) in self.merges]
            ops += [dist.P2POp(dist.irecv, self.q_help[r], self._peer(self.plan.owner(r)), self.p2p_group)
                    for r in self.helping]
            with torch.cuda.stream(p2p):
                q_reqs = dist.batch_isend_irecv(ops)
                if self.phase_events is not None:
                    for req in q_reqs:
                        req.wait()
                    self._mark("query_handoff", p2p)
        # local causal attention meanwhile, on the main stream
        if q_ready is None:
            self._attention(self.local_problems)
        else:
            main.wait_event(kv_ready)
            for li in range(self.n_local):
                main.wait_event(q_ready[li])
                self._attention([self.local_problems[li]])
        self._mark("local_attention", main)
        main.wait_stream(side)
        self._mark("exchange_wait", main)
        scale = 1.0 / math.sqrt(self.d)
        for probs, hq, hkv in self.compact_calls:
            run_attention(probs, hq, hkv, self.d, scale, self.code, dev)
        self._mark("compact_attention", main)
        if self.helped or self.helping:
            for req in q_reqs:
                req.wait()  # the main stream waits for the query transfers
            if self.helping:
                for probs, hq, hkv in self.helper_calls:
                    run_attention(probs, hq, hkv, self.d, scale, self.code, dev)
                self._mark("helper_attention", main)
            # partial states back to the helped blocks' ranks, merged there
            ops = []
            for r in self.helping:
                dst = self._peer(self.plan.owner(r))
                ops += [dist.P2POp(dist.isend, self.o_help[r], dst, self.p2p_group),
                        dist.P2POp(dist.isend, self.lse_help[r], dst, self.p2p_group)]
            for (_, _, _, r) in self.merges:
                src = self._peer(self.plan.helper(r))
                ops += [dist.P2POp(dist.irecv, self.o_from[r], src, self.p2p_group),
                        dist.P2POp(dist.irecv, self.lse_from[r], src, self.p2p_group)]
            for req in dist.batch_isend_irecv(ops):
                req.wait()
            self._mark("partial_return", main)
            for (_, o_li, lse_li, r) in self.merges:
                merge_lse([o_li, self.o_from[r]], [lse_li, self.lse_from[r]], out=o_li, want_lse=False)
        self._mark("end", main)
        if done is not None:
            done.record(main)
        if merged is not None:
            for li in range(self.n_local):
                merged[li].record(main)

    def _forward_host(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out) -> torch.Tensor:
        """Host buffers in and out.  Copy-in order: the destination windows of
        every local block (pooling starts on them), then K and V (the builds),
        then the remaining query rows block by block (local attention of a
        block starts when its queries are in); each block's output is copied
        out as soon as its merge is done."""
        exp_q = (self.n_local, self.hq, self.L, self.d)
        if out is None:
            if getattr(self, "_host_out", None) is None:
                self._host_out = torch.empty(exp_q, dtype=self.dtype).pin_memory()
            out = self._host_out
        elif out.is_cuda or tuple(out.shape) != exp_q or out.dtype != self.dtype or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous CPU {self.dtype} tensor of shape {exp_q}")
        dev = self.device
        if getattr(self, "_staging", None) is None:
            # two device staging sets (inputs, output, LSE), alternated by
            # consecutive calls, so the copy-in of one call overlaps the
            # compute of the previous one
            self._staging = [(torch.empty_like(q, device=dev), torch.empty_like(k, device=dev),
                              torch.empty_like(v, device=dev), torch.empty_like(self.o_loc),
                              torch.empty_like(self.lse_loc)) for _ in range(2)]
            self._staging_done = [None, None]
            self._host_calls = 0
            self._host_stream = torch.cuda.Stream(device=dev)
            self._h2d = torch.cuda.Stream(device=dev)
            self._d2h = torch.cuda.Stream(device=dev)
            self._ev_win, self._ev_kv = torch.cuda.Event(), torch.cuda.Event()
            self._ev_q = [torch.cuda.Event() for _ in range(self.n_local)]
            self._ev_merged = [torch.cuda.Event() for _ in range(self.n_local)]
            # per staging set and local block: recorded after its copy-out
            self._ev_drained = [[torch.cuda.Event() for _ in range(self.n_local)] for _ in range(2)]
        caller = torch.cuda.current_stream(dev)
        if not self._last_call_host:
            # device-path work on the caller's stream may still use the internal buffers
            self._host_stream.wait_stream(caller)
        self._last_call_host = True
        i = self._host_calls % 2
        self._host_calls += 1
        dq, dk_, dv, do, dlse = self._staging[i]
        self._bind(dq, dk_, dv, do, dlse)
        # the compute runs on an internal stream that does not wait for the
        # copy-out, so the next call's compute can start under this call's
        # last copies; the caller's stream waits for the output
        main = self._host_stream
        h2d, d2h = self._h2d, self._d2h
        W = self.window
        # the kernels of the call before the previous one must be done with
        # this staging set, and the previous call's copy-out with the outputs
        if self._staging_done[i] is None:
            h2d.wait_stream(main)
        else:
            h2d.wait_event(self._staging_done[i])
        self._staging_done[i] = torch.cuda.Event()
        for li in range(self.n_local):
            main.wait_event(self._ev_drained[i][li])
        with torch.cuda.stream(h2d):
            for li in range(self.n_local):
                for h in range(self.hq):
                    dq[li, h, :W].copy_(q[li, h, :W], non_blocking=True)
            self._ev_win.record(h2d)
            dk_.copy_(k, non_blocking=True)
            dv.copy_(v, non_blocking=True)
            self._ev_kv.record(h2d)
            for li in range(self.n_local):
                if W < self.L:
                    for h in range(self.hq):
                        dq[li, h, W:].copy_(q[li, h, W:], non_blocking=True)
                self._ev_q[li].record(h2d)
        with torch.cuda.stream(main):
            self._run(self._ev_win, self._ev_kv, self._ev_q, self._ev_merged)
        self._staging_done[i].record(main)
        with torch.cuda.stream(d2h):
            for li in range(self.n_local):
                d2h.wait_event(self._ev_merged[li])
                out[li].copy_(do[li], non_blocking=True)
                self._ev_drained[i][li].record(d2h)
        caller.wait_stream(d2h)
        return out

    def launches_per_forward(self) -> int:
        sets = len(self.sets)
        pool = 0 if sets == 0 else 2 * -(-sets // 64)
        # the last launch reports the bounded-wait error flags to the host
        return (pool + build_launch_count(len(self.build), self.code, self.d) + -(-len(self.local_problems) // 8)
                + sum(-(-len(c[0]) // 8) for c in self.compact_calls + self.helper_calls) + len(self.merges) + 1)


class DistributedDccKvStack:
    """Several DCC-KV sync layers in a row (one process per GPU, each layer
    with its own local q / k / v, as ``DistributedDccKvLayer``), with the
    compact-KV exchange double buffered across layers: two layer slots, each
    with its own compact, receive, representative-query and workspace
    buffers, take the layers in turn, and a slot's pooling, builds and
    all-to-allv (its high-priority side stream) wait only for the inputs and
    for the compact attention of the layer two back.  So layer l + 1's
    exchange runs while layer l's attention runs (the reference's
    asynchronous-exchange pipeline, tests/gpu/test_async_overlap.py:43-98).
    Every layer writes its own output buffer; outputs equal those of the
    layers called one at a time, bit for bit."""

    def __init__(self, *args, **kwargs):
        self.slots = [DistributedDccKvLayer(*args, **kwargs) for _ in range(2)]
        self._outs: List[torch.Tensor] = []
        self._done = [None, None]

    def forward(self, inputs) -> List[torch.Tensor]:
        """inputs: a sequence of (q, k, v) device tensors per layer, shaped
        as for ``DistributedDccKvLayer``.  Returns one output per layer
        (internal buffers, reused by the next call); complete once the
        current stream is synchronized."""
        first = self.slots[0]
        first._errors.poll()
        dev = first.device
        main = torch.cuda.current_stream(dev)
        exp_q = (first.n_local, first.hq, first.L, first.d)
        exp_kv = (first.n_local, first.hkv, first.L, first.d)
        while len(self._outs) < len(inputs):
            self._outs.append(torch.empty(exp_q, dtype=first.dtype, device=dev))
        ready = torch.cuda.Event()
        ready.record(main)  # every layer's inputs are written
        for li, (q, k, v) in enumerate(inputs):
            if tuple(q.shape) != exp_q or tuple(k.shape) != exp_kv or tuple(v.shape) != exp_kv:
                raise ValueError(f"layer {li}: expected local q {exp_q}, k/v {exp_kv}")
            for t in (q, k, v):
                if t.dtype != first.dtype or not t.is_contiguous() or t.device != dev:
                    raise ValueError(f"layer {li}: inputs must be contiguous {first.dtype} on {dev}")
            slot = self.slots[li % 2]
            if slot._host_stream is not None and slot._last_call_host:
                main.wait_stream(slot._host_stream)
            slot._last_call_host = False
            slot._bind(q, k, v, self._outs[li], slot.lse_loc)
            prev = self._done[li % 2]
            waits = [ready] + ([prev] if prev is not None else [])
            done = torch.cuda.Event()
            slot._run(side_waits=waits, done=done)
            self._done[li % 2] = done
        first._errors.record(main)
        return self._outs[:len(inputs)]

    __call__ = forward
