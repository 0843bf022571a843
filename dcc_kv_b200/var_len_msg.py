"""Variable-length message codec (src/distributed/var_len_msg.py) and the
CompactKV wire format used by the distributed layer.

``pack_var_len_messages`` / ``unpack_var_len_messages`` / ``mock_all_to_allv``
keep the reference's signatures and assertions.  The wire format of one
edge's compact KV is KV-head-major: per KV head a byte block

    keys   [B', d]  (input dtype)
    values [B', d]  (input dtype)
    bias   [B']     float32
    padding to a multiple of 256 bytes

so every keys / values / bias block starts 16-byte aligned (TMA operands),
a destination attends to it in place (one KV segment per edge, head stride
= the block size), and any run of consecutive KV heads of an edge is one
contiguous byte range -- an edge can be split by KV heads between two
consuming ranks without a copy.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch


def pack_var_len_messages(messages: List[torch.Tensor], sizes: List[int]) -> Tuple[torch.Tensor, List[int]]:
    """var_len_msg.py:16-37: concatenate [n_i, ...] messages; offsets [0, n_0, n_0+n_1, ...]."""
    assert len(messages) == len(sizes)
    for m, s in zip(messages, sizes):
        assert m.shape[0] == s, f"message size {m.shape[0]} != expected {s}"
    packed = torch.cat(messages, dim=0)
    offsets = [0]
    for s in sizes:
        offsets.append(offsets[-1] + s)
    return packed, offsets


def unpack_var_len_messages(packed: torch.Tensor, sizes: List[int]) -> List[torch.Tensor]:
    """var_len_msg.py:40-59: split [sum(sizes), ...] into views."""
    assert packed.shape[0] == sum(sizes), f"packed size {packed.shape[0]} != sum {sum(sizes)}"
    out, off = [], 0
    for s in sizes:
        out.append(packed[off:off + s])
        off += s
    return out


def mock_all_to_allv(rank: int, world_size: int, send_messages: List[torch.Tensor], send_sizes: List[int],
                     peer_send_data: dict) -> List[torch.Tensor]:
    """var_len_msg.py:62-98: single-process all-to-allv from {src: (packed, sizes)}."""
    assert len(send_messages) == world_size
    assert len(send_sizes) == world_size
    recv = []
    for src in range(world_size):
        if src == rank:
            recv.append(send_messages[rank])
        else:
            if src not in peer_send_data:
                raise ValueError(f"Missing mock data for src={src}")
            packed, sizes = peer_send_data[src]
            recv.append(unpack_var_len_messages(packed, sizes)[rank])
    return recv


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


@dataclass(frozen=True)
class EdgeLayout:
    """Byte layout of one edge's compact KV block (KV-head-major)."""
    n_kv_heads: int
    rows: int        # B' = min(budget, L_s)
    head_dim: int
    elem: int        # bytes per key / value element

    @property
    def kv_bytes(self) -> int:
        """Bytes of one head's keys (or values)."""
        return self.rows * self.head_dim * self.elem

    @property
    def keys_off(self) -> int:
        return 0

    @property
    def values_off(self) -> int:
        return self.kv_bytes

    @property
    def bias_off(self) -> int:
        return 2 * self.kv_bytes

    @property
    def head_bytes(self) -> int:
        return _align(2 * self.kv_bytes + self.rows * 4)

    @property
    def nbytes(self) -> int:
        return self.n_kv_heads * self.head_bytes

    def views(self, buf: torch.Tensor, offset: int, dtype: torch.dtype, n_heads: int = None):
        """(keys [n, B', d], values [n, B', d], bias [n, B']) views of ``n``
        consecutive head blocks (default: all heads) of ``buf`` (uint8, a
        multiple of 256 bytes long) starting at byte ``offset``."""
        n = self.n_kv_heads if n_heads is None else n_heads
        b, d, hb = self.rows, self.head_dim, self.head_bytes
        if offset % 256 or buf.numel() % 256 or offset + n * hb > buf.numel():
            raise ValueError("edge views need 256-byte aligned offsets inside the buffer")
        elem = torch.empty(0, dtype=dtype).element_size()
        typed = buf.view(dtype)
        base = typed.storage_offset() + offset // elem
        k = typed.as_strided((n, b, d), (hb // elem, d, 1), base + self.keys_off // elem)
        v = typed.as_strided((n, b, d), (hb // elem, d, 1), base + self.values_off // elem)
        fl = buf.view(torch.float32)
        bias = fl.as_strided((n, b), (hb // 4, 1), fl.storage_offset() + (offset + self.bias_off) // 4)
        return k, v, bias
