"""Multi-GPU host logic on CPU: shard plans, context ranges and the (m, l, o)
all-gather + merge, run as world_size-2 gloo process groups.

The per-rank partials are computed with a numpy restatement of the
log-sum-exp split (from the oracle's dequantized K/V) so the test checks the
host orchestration — ranges, packing layout, rank order of the gather,
merge arithmetic — against the single-process oracle output.
"""
import os
import socket

import numpy as np
import pytest

from kvq.parallel import context_ranges, shard_plan


def test_shard_plan_by_heads_and_sequences():
    lens = [1024, 32768, 5000, 20000, 7, 16000, 9000, 3000]
    plans = shard_plan(lens, 8, 4)
    assert [p.kv_heads for p in plans] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert all(p.sequences == list(range(8)) for p in plans)
    plans = shard_plan(lens, 8, 3)  # 8 % 3 != 0 -> by sequence, LPT packing
    owned = sorted(i for p in plans for i in p.sequences)
    assert owned == list(range(8))
    loads = [p.load for p in plans]
    assert max(loads) - min(loads) <= max(lens) * 8
    plans = shard_plan(lens, 8, 2, prefer_heads=False)
    assert sorted(i for p in plans for i in p.sequences) == list(range(8))


@pytest.mark.parametrize("N,world", [(131072, 8), (1000, 3), (17, 4), (256, 1), (3, 8)])
def test_context_ranges_cover(N, world):
    r = context_ranges(N, world)
    assert len(r) == world
    assert r[0][0] == 0 and r[-1][1] == N
    for (a, b), (c, d) in zip(r[:-1], r[1:]):
        assert b == c and a <= b
    assert all(a % 16 == 0 or a == N for a, _ in r)
    sizes = [b - a for a, b in r]
    if N >= 16 * world:
        assert max(sizes) - min(sizes) <= 16 + N // world - (N // world) // 16 * 16 + 16


def _partials_np(q, kd, vd):
    """q [R, D] f32, kd/vd [R, n, D] f32 -> m, l, o (LSE partials)."""
    s = np.einsum("rd,rnd->rn", q, kd)
    m = s.max(axis=1) if s.shape[1] else np.full(q.shape[0], -1e30, np.float32)
    e = np.exp(s - m[:, None])
    return m.astype(np.float32), e.sum(1).astype(np.float32), np.einsum("rn,rnd->rd", e, vd).astype(np.float32)


def _worker(rank, world, port, q, kd, vd, want, errq):
    try:
        import torch
        import torch.distributed as dist
        from kvq.parallel import gather_partials
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        N = kd.shape[1]
        a, b = context_ranges(N, world, align=16)[rank]
        m, l, o = _partials_np(q, kd[:, a:b], vd[:, a:b])
        R, D = o.shape
        packed = torch.from_numpy(np.concatenate([m, l, o.reshape(-1)]))
        g = gather_partials(packed).numpy()
        assert g.shape == (world, R * (D + 2))
        M = g[:, :R].max(0)
        w = np.exp(g[:, :R] - M)
        L = (g[:, R:2 * R] * w).sum(0)
        O = (g[:, 2 * R:].reshape(world, R, D) * w[:, :, None]).sum(0) / L[:, None]
        err = float(np.abs(O - want).max())
        assert err < 1e-4, err
        dist.destroy_process_group()
    except Exception as e:  # report to the parent
        errq.put(f"rank {rank}: {e!r}")


def test_context_split_gather_merge_gloo():
    import multiprocessing as mp
    rng = np.random.default_rng(0)
    R, N, D = 6, 300, 32
    q = rng.standard_normal((R, D)).astype(np.float32) * 0.2
    kd = rng.standard_normal((R, N, D)).astype(np.float32)
    vd = rng.standard_normal((R, N, D)).astype(np.float32)
    m, l, o = _partials_np(q, kd, vd)
    want = o / l[:, None]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, kd, vd, want, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs)
