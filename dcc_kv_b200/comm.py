"""Communication layer with the reference's interface (src/distributed/comm.py).

``DistributedComm`` wraps ``torch.distributed`` (NCCL on GPUs, gloo on CPU)
with the reference's lifecycle, argument checks and exceptions.  The
var-len all-to-allv keeps the reference's contract (comm.py:174-280):
``messages[i]`` goes to rank i, result ``[i]`` came from rank i, and
``recv_sizes`` is required.  By default the sizes are exchanged and used as
the reference does; ``trust_recv_sizes=True`` skips that round trip and its
device-to-host synchronisation when every rank derives the sizes from the
shared budget configuration (the DCC-KV layer does).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)


@dataclass
class VarLenMessage:
    """comm.py:29-42: a payload [N, ...] with optional metadata."""
    payload: torch.Tensor
    metadata: Optional[dict] = field(default_factory=dict)

    def numel(self) -> int:
        return self.payload.shape[0] if self.payload.dim() > 0 else 1


class DistributedComm:
    """comm.py:48-339 (backend gloo / nccl / mpi; mock mode without torch.distributed)."""

    def __init__(self, backend: str = "gloo", mock: bool = False, group=None):
        """``group`` (an addition to the reference's signature): the process
        group every collective runs on; None is the default group."""
        if backend not in ("gloo", "nccl", "mpi"):
            raise ValueError(f"Unknown backend: {backend}; choose gloo/nccl/mpi")
        self.backend = backend
        self.mock = mock
        self.group = group
        self.rank = 0
        self.world_size = 1
        self.initialized = False

    def init(self, rank: int, world_size: int) -> None:
        if self.initialized:
            logger.warning("DistributedComm already initialized; skipping reinit")
            return
        self.rank = rank
        self.world_size = world_size
        if not self.mock:
            if not dist.is_initialized():
                raise RuntimeError("torch.distributed not initialized; call setup_distributed() first")
            g = self.group
            if dist.get_rank(g) != rank or dist.get_world_size(g) != world_size:
                raise ValueError(f"Comm init rank/ws mismatch: requested ({rank}/{world_size}), "
                                 f"actual ({dist.get_rank(g)}/{dist.get_world_size(g)})")
        self.initialized = True

    def cleanup(self) -> None:
        self.initialized = False

    def __enter__(self):
        if not self.initialized:
            raise RuntimeError("DistributedComm not initialized")
        return self

    def __exit__(self, *args):
        self.cleanup()

    def _check_init(self) -> None:
        if not self.initialized:
            raise RuntimeError("DistributedComm not initialized; call init() first")

    def all_to_all_single(self, send_tensor: torch.Tensor, send_counts: Optional[List[int]] = None,
                          recv_counts: Optional[List[int]] = None) -> torch.Tensor:
        """comm.py:127-172."""
        self._check_init()
        if send_counts is None:
            send_counts = [send_tensor.shape[0] // self.world_size] * self.world_size
        if recv_counts is None:
            recv_counts = send_counts
        if sum(send_counts) != send_tensor.shape[0]:
            raise ValueError(f"send_counts sum ({sum(send_counts)}) != send_tensor.shape[0] ({send_tensor.shape[0]})")
        if self.mock:
            shape = list(send_tensor.shape)
            shape[0] = sum(recv_counts)
            return torch.zeros(shape, dtype=send_tensor.dtype, device=send_tensor.device)
        recv = torch.empty((sum(recv_counts),) + tuple(send_tensor.shape[1:]), dtype=send_tensor.dtype,
                           device=send_tensor.device)
        dist.all_to_all_single(recv, send_tensor, output_split_sizes=list(recv_counts),
                               input_split_sizes=list(send_counts), group=self.group)
        return recv

    def all_to_all_v(self, messages: List[VarLenMessage], send_sizes: Optional[List[int]] = None,
                     recv_sizes: Optional[List[int]] = None, trust_recv_sizes: bool = False,
                     out: Optional[torch.Tensor] = None,
                     packed: Optional[torch.Tensor] = None) -> List[VarLenMessage]:
        """comm.py:174-280: variable-length all-to-all; ``out`` optionally
        supplies the receive buffer [sum(recv_sizes), ...] and ``packed`` the
        send buffer when the payloads already lie in it back to back (as
        views, message i at offset sum(send_sizes[:i])), so no concatenation
        copy is made."""
        self._check_init()
        if len(messages) != self.world_size:
            raise ValueError(f"messages length ({len(messages)}) != world_size ({self.world_size})")
        if send_sizes is None:
            send_sizes = [m.numel() for m in messages]
        if any(m.numel() != s for m, s in zip(messages, send_sizes)):
            raise ValueError(f"send_sizes inconsistent with messages: sizes={send_sizes}, "
                             f"actual={[m.numel() for m in messages]}")
        if recv_sizes is None:
            raise ValueError("recv_sizes is required for all_to_all_v "
                             "(DCC-KV must share budget config across ranks)")
        if len(recv_sizes) != self.world_size:
            raise ValueError(f"recv_sizes length ({len(recv_sizes)}) != world_size ({self.world_size})")
        first = messages[0].payload
        if self.mock:
            return [VarLenMessage(payload=torch.zeros((s,) + tuple(first.shape[1:]), dtype=first.dtype,
                                                      device=first.device),
                                  metadata={"src_rank": i, "mock": True}) for i, s in enumerate(recv_sizes)]
        if trust_recv_sizes:
            actual = [int(s) for s in recv_sizes]
        else:
            st = torch.tensor(send_sizes, dtype=torch.long, device=first.device)
            rt = torch.empty_like(st)
            dist.all_to_all_single(rt, st, output_split_sizes=[1] * self.world_size,
                                   input_split_sizes=[1] * self.world_size, group=self.group)
            actual = rt.tolist()
        if packed is not None:
            if packed.shape[0] != sum(send_sizes):
                raise ValueError(f"packed holds {packed.shape[0]} rows, send_sizes sum to {sum(send_sizes)}")
            send = packed
        else:
            send = torch.cat([m.payload for m in messages], dim=0)
        recv = out if out is not None else torch.empty((sum(actual),) + tuple(first.shape[1:]), dtype=first.dtype,
                                                       device=first.device)
        dist.all_to_all_single(recv, send, output_split_sizes=actual, input_split_sizes=list(send_sizes),
                               group=self.group)
        res, off = [], 0
        for i, s in enumerate(actual):
            res.append(VarLenMessage(payload=recv[off:off + s], metadata={"src_rank": i, "size": s}))
            off += s
        return res

    def all_reduce(self, tensor: torch.Tensor, op=dist.ReduceOp.SUM) -> torch.Tensor:
        self._check_init()
        if self.mock:
            return tensor.clone()
        dist.all_reduce(tensor, op=op, group=self.group)
        return tensor

    def broadcast(self, tensor: torch.Tensor, src: int = 0) -> torch.Tensor:
        self._check_init()
        if self.mock:
            return tensor.clone()
        dist.broadcast(tensor, src=src, group=self.group)
        return tensor

    def barrier(self) -> None:
        if not self.mock and dist.is_initialized():
            dist.barrier(group=self.group)

    def gather(self, tensor: torch.Tensor, dst: int = 0) -> Optional[List[torch.Tensor]]:
        self._check_init()
        if self.mock:
            return [tensor.clone() for _ in range(self.world_size)]
        if self.rank == dst:
            out = [torch.empty_like(tensor) for _ in range(self.world_size)]
            dist.gather(tensor, out, dst=dst, group=self.group)
            return out
        dist.gather(tensor, None, dst=dst, group=self.group)
        return None

    def __repr__(self) -> str:
        return (f"DistributedComm(backend={self.backend}, mock={self.mock}, "
                f"rank={self.rank}/{self.world_size}, initialized={self.initialized})")
