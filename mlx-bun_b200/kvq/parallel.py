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
  ``kvq_sdpa_decode_partial``, one ``all_gather_into_tensor`` exchanges the
  packed partials (rows * (D + 2) floats per rank), and every rank merges
  them in rank order with ``kvq_sdpa_merge`` (deterministic).

The collectives go through ``torch.distributed`` (NCCL on GPUs; the host
logic is exercised with gloo on CPU in the tests).
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


class ContextSplitDecode:
    """Decode of one very long sequence whose K/V is split across ranks.

    Each rank holds a kvq cache with its own key range; ``step(q)`` returns
    the full attention output on every rank.  Only the partials cross
    NVLink: B * Hq * (D + 2) floats per rank per step."""

    def __init__(self, group=None):
        self.group = group
        self._packed = None
        self._gathered = None

    def step(self, q, keys, values, scale: float, stream=None):
        import torch
        import torch.distributed as dist
        from . import sdpa
        B, Hq, _, D = q.shape
        R = B * Hq
        if self._packed is None or self._packed.numel() != R * (D + 2) or \
                self._packed.device != q.device:
            world = dist.get_world_size(self.group)
            self._packed = torch.empty(R * (D + 2), dtype=torch.float32, device=q.device)
            self._gathered = torch.empty(world * R * (D + 2), dtype=torch.float32,
                                         device=q.device)
        sdpa.sdpa_decode_partial(q, keys, values, scale, packed_out=self._packed, stream=stream)
        dist.all_gather_into_tensor(self._gathered, self._packed, group=self.group)
        out = sdpa.sdpa_merge_packed(self._gathered.view(-1, R * (D + 2)), R, D, q.dtype,
                                     stream=stream)
        return out.view(B, Hq, 1, D)
