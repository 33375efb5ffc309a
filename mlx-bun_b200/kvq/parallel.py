"""Multi-GPU partitioning of quantized-KV decode (one process per GPU).

mlx-bun is single-device; this module adds the two partitionings its
quantized-KV attention admits on one 8-GPU node:

* Shard by kv head or by sequence (``shard_plan``): every rank owns whole
  (sequence, kv-head) caches and computes their query heads' outputs with no
  communication at all.  kv heads split evenly when ``Hkv % world == 0``;
  otherwise sequences are bin-packed by length (longest first onto the
  least-loaded rank).
* Split one long context (``ContextSplitDecode``): rank r owns the
  contiguous key range ``context_ranges(N, world)[r]`` of the sequence;
  each rank computes log-sum-exp partials (m, l, o) of its range with
  ``kvq_sdpa_decode_partial`` into one packed buffer (rows * (D + 2) floats),
  the partials move to every rank, and every rank merges them in rank order
  (deterministic, identical on all ranks).  Two transports:
    - "peer" (GPUs): ``kvq_peer_exchange_merge`` stores the packed partial
      into every rank's exchange buffer over peer memory (CUDA IPC, NVLink)
      and merges once all have arrived — one kernel, no NCCL call and no
      host synchronisation per step, so a step can live in a CUDA graph;
    - "collective": ``all_gather_into_tensor`` through torch.distributed
      (NCCL, or gloo in the CPU tests) followed by ``kvq_sdpa_merge``.

The process group is used for set-up (exchanging the IPC handles) in the
peer transport, and for the data in the collective one.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class ShardPlan:
    """Work owned by one rank."""
    rank: int
    kv_heads: tuple  # (first, last + 1) kv-head range, all of them when sharding by sequence
    sequences: list = field(default_factory=list)  # sequence indices owned
    load: int = 0    # key rows x kv heads owned (for balance checks)


def shard_plan(seq_lens, kv_heads: int, world: int, prefer_heads: bool = True):
    """Plans for all ranks; the union covers every (sequence, kv head) once."""
    if world <= 0:
        raise ValueError("world must be positive")
    n = len(seq_lens)
    if prefer_heads and kv_heads % world == 0:
        per = kv_heads // world
        total = int(sum(seq_lens))
        return [ShardPlan(r, (r * per, (r + 1) * per), list(range(n)), total * per)
                for r in range(world)]
    plans = [ShardPlan(r, (0, kv_heads), [], 0) for r in range(world)]
    order = sorted(range(n), key=lambda i: (-int(seq_lens[i]), i))
    for i in order:
        tgt = min(plans, key=lambda p: (p.load, p.rank))
        tgt.sequences.append(i)
        tgt.load += int(seq_lens[i]) * kv_heads
    for p in plans:
        p.sequences.sort()
    return plans


def context_ranges(N: int, world: int, align: int = 16):
    """Contiguous [start, end) key ranges, one per rank, covering [0, N)
    exactly; inner boundaries sit at r*N/world rounded down to `align` rows."""
    if world <= 0:
        raise ValueError("world must be positive")
    cuts = [0] + [min(N, (r * N // world) // align * align) for r in range(1, world)] + [N]
    for i in range(1, len(cuts)):
        cuts[i] = max(cuts[i], cuts[i - 1])
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def gather_partials(packed, group=None):
    """all_gather of this rank's packed partials [rows * (D + 2)] (float32)
    into a [world, rows * (D + 2)] tensor in rank order."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = packed.contiguous().view(-1)
    out = torch.empty(world * flat.numel(), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    return out.view((world,) + tuple(packed.shape))


def _stream_ctx(stream):
    """`with` context making `stream` (a torch.cuda.Stream, or None for the
    current stream) current, so partial, exchange and merge share one
    stream and run in order."""
    import contextlib
    import torch
    return torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()


class PeerGroup:
    """This rank's side of a peer-memory exchange among the ranks of
    `group` (one per GPU of one node) for partial sets of `rows` x
    `head_dim` (kvq_peer_group_* in include/kvq.h)."""

    def __init__(self, rows: int, head_dim: int, group=None):
        import ctypes
        import torch.distributed as dist
        from ._lib import check, lib
        self.rows, self.head_dim = rows, head_dim
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        handle = (ctypes.c_uint8 * 64)()
        h = ctypes.c_void_p()
        check(lib().kvq_peer_group_create(rank, world, rows, head_dim, handle, ctypes.byref(h)))
        self._h = h
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        blob = b"".join(handles)
        check(lib().kvq_peer_group_connect(h, blob))
        dist.barrier(group=group)  # every rank mapped every buffer

    def exchange_merge(self, packed, dtype, out, stream_handle):
        from ._lib import check, lib
        from .cache import dtype_code
        check(lib().kvq_peer_exchange_merge(self._h, packed.data_ptr(), dtype_code(dtype),
                                            out.data_ptr(), stream_handle))

    def check(self, stream_handle=None):
        """Synchronize the device and raise if a step gave up waiting for a rank."""
        import torch
        from ._lib import check, lib
        torch.cuda.synchronize()
        check(lib().kvq_peer_group_check(self._h, stream_handle))

    def close(self):
        """Free after every rank's last step (callers barrier first)."""
        from ._lib import check, lib
        if self._h:
            h, self._h = self._h, None
            check(lib().kvq_peer_group_free(h))


class ContextSplitDecode:
    """Decode of one very long sequence whose K/V is split across ranks.

    Each rank holds a kvq cache with its own key range; ``step(q)`` returns
    the full attention output on every rank.  Only the partials cross
    NVLink: B * Hq * (D + 2) floats per rank per step.  `transport` is
    "peer" (peer-memory exchange kernel) or "collective" (all-gather through
    torch.distributed, then merge)."""

    def __init__(self, group=None, transport: str = "peer"):
        if transport not in ("peer", "collective"):
            raise ValueError("transport must be 'peer' or 'collective'")
        self.group = group
        self.transport = transport
        self._packed = None
        self._gathered = None
        self._peer = None
        self._out = None

    def _buffers(self, q, R, D):
        import torch
        import torch.distributed as dist
        if self._packed is None or self._packed.numel() != R * (D + 2) or \
                self._packed.device != q.device:
            world = dist.get_world_size(self.group)
            self._packed = torch.empty(R * (D + 2), dtype=torch.float32, device=q.device)
            if self.transport == "collective":
                self._gathered = torch.empty(world * R * (D + 2), dtype=torch.float32,
                                             device=q.device)
            else:
                if self._peer is not None:
                    self._peer.close()
                self._peer = PeerGroup(R, D, self.group)
        if self._out is None or self._out.shape != (R, D) or self._out.dtype != q.dtype or \
                self._out.device != q.device:
            self._out = torch.empty(R, D, dtype=q.dtype, device=q.device)

    def step(self, q, keys, values, scale: float, stream=None):
        """One decode step.  `stream`: a torch.cuda.Stream to run on (None:
        the current stream); partial, exchange and merge are all issued on
        it, in order.  Returns [B, Hq, 1, D] (a buffer reused by the next
        step)."""
        import torch
        import torch.distributed as dist
        from . import sdpa
        B, Hq, _, D = q.shape
        R = B * Hq
        self._buffers(q, R, D)
        with _stream_ctx(stream):
            cur = torch.cuda.current_stream(q.device)
            sdpa.sdpa_decode_partial(q, keys, values, scale, packed_out=self._packed,
                                     stream=cur.cuda_stream)
            if self.transport == "peer":
                self._peer.exchange_merge(self._packed, q.dtype, self._out, cur.cuda_stream)
            else:
                dist.all_gather_into_tensor(self._gathered, self._packed, group=self.group)
                sdpa.sdpa_merge_packed(self._gathered.view(-1, R * (D + 2)), R, D, q.dtype,
                                       out=self._out, stream=cur.cuda_stream)
        return self._out.view(B, Hq, 1, D)

    def check(self, stream=None):
        """Raise if a peer exchange gave up waiting for a rank (peer transport)."""
        if self._peer is not None:
            self._peer.check(stream.cuda_stream if stream is not None else None)

    def close(self):
        if self._peer is not None:
            self._peer.close()
            self._peer = None
