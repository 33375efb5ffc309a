"""Multi-GPU paths on real GPUs over NCCL (skipped with fewer than two GPUs).

* Context split: one long sequence's keys are split into contiguous ranges,
  one per rank; each rank computes (m, l, o) partials of its range, the
  partials are all-gathered over NCCL and merged.  Every rank's result must
  match the single-GPU decode over all keys within the decode tolerance
  (2e-3 on fp16 outputs), and rank 0's must match the oracle.
* Sharding by kv head: each rank decodes its own kv heads with no
  communication; the concatenated outputs must match the oracle.

Ranks run as spawned processes (one per GPU) with a short process-group
timeout, so a rank that fails ends the others' collectives with an error.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port):
    for p in (os.path.join(ROOT, "tests"), ROOT, os.path.join(ROOT, "mlx-bun_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def _context_split_worker(rank, world, port, out_dir):
    _setup(rank, world, port)
    import torch
    import torch.distributed as dist
    import kvq
    from helpers import F16, as_qtensor, from_torch, max_abs, quantized_inputs, to_torch_bits, \
        upload_triple
    from kvq.parallel import ContextSplitDecode, context_ranges
    from oracle import oracle as O
    try:
        B, Hq, Hkv, N, D, gs, bits = 1, 32, 8, 40000, 128, 64, 4
        rng = np.random.default_rng(21)  # the same inputs on every rank
        q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, F16)
        scale = 1.0 / np.sqrt(D)
        a, b = context_ranges(N, world)[rank]
        sk = tuple(np.ascontiguousarray(x[:, :, a:b]) for x in kq)
        sv = tuple(np.ascontiguousarray(x[:, :, a:b]) for x in vq)
        K = as_qtensor(*upload_triple(*sk, gs, bits)[:3], b - a, gs, bits, F16)
        V = as_qtensor(*upload_triple(*sv, gs, bits)[:3], b - a, gs, bits, F16)
        qt = to_torch_bits(q, F16)
        split = ContextSplitDecode()
        out = split.step(qt, K, V, scale)
        out = split.step(qt, K, V, scale)  # second step reuses the gather buffers
        torch.cuda.synchronize()
        got = from_torch(out, F16)
        Kf = as_qtensor(*upload_triple(*kq, gs, bits)[:3], N, gs, bits, F16)
        Vf = as_qtensor(*upload_triple(*vq, gs, bits)[:3], N, gs, bits, F16)
        full = from_torch(kvq.sdpa_decode(qt, Kf, Vf, scale), F16)
        err_full = max_abs(got, full, F16)
        err_oracle = -1.0
        if rank == 0:
            want = O.sdpa_unfused(q, kq, vq, scale, gs, bits, F16)
            err_oracle = max_abs(got, want, F16)
        np.save(os.path.join(out_dir, f"ctx_{rank}.npy"), np.array([err_full, err_oracle]))
    finally:
        dist.destroy_process_group()


def _kv_head_shard_worker(rank, world, port, out_dir):
    _setup(rank, world, port)
    import torch
    import torch.distributed as dist
    import kvq
    from helpers import F16, as_qtensor, from_torch, quantized_inputs, to_torch_bits, upload_triple
    from kvq.parallel import shard_plan
    try:
        B, Hq, Hkv, D, gs, bits = 4, 32, 8, 128, 64, 4
        lens = [3000, 1200, 2048, 17]
        N = max(lens)
        rng = np.random.default_rng(22)
        q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, F16)
        plan = shard_plan(lens, Hkv, world)[rank]
        h0, h1 = plan.kv_heads
        nrep = Hq // Hkv
        sk = tuple(np.ascontiguousarray(x[:, h0:h1]) for x in kq)
        sv = tuple(np.ascontiguousarray(x[:, h0:h1]) for x in vq)
        K = as_qtensor(*upload_triple(*sk, gs, bits)[:3], N, gs, bits, F16)
        V = as_qtensor(*upload_triple(*sv, gs, bits)[:3], N, gs, bits, F16)
        qs = np.ascontiguousarray(q[:, h0 * nrep:h1 * nrep])
        sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
        out = kvq.sdpa_decode(to_torch_bits(qs, F16), K, V, 1.0 / np.sqrt(D), seq_lens=sl)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"heads_{rank}.npy"), from_torch(out, F16))
        np.save(os.path.join(out_dir, f"heads_lens.npy"), np.array(lens))
    finally:
        dist.destroy_process_group()


def _spawn(fn, world, tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(fn, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")


@pytest.mark.timeout(600)
def test_context_split_nccl(tmp_path):
    import torch
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = min(world, 8)
    _spawn(_context_split_worker, world, tmp_path)
    for r in range(world):
        err_full, err_oracle = np.load(tmp_path / f"ctx_{r}.npy")
        assert err_full <= TOL, (r, err_full)
        if r == 0:
            assert err_oracle <= TOL, err_oracle


@pytest.mark.timeout(600)
def test_kv_head_shards_nccl(tmp_path):
    import torch
    from helpers import F16, max_abs, quantized_inputs
    from oracle import oracle as O
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = 2 if 8 % world else min(world, 8)
    _spawn(_kv_head_shard_worker, world, tmp_path)
    B, Hq, Hkv, D, gs, bits = 4, 32, 8, 128, 64, 4
    lens = [3000, 1200, 2048, 17]
    rng = np.random.default_rng(22)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, max(lens), D, gs, bits, F16)
    want = O.sdpa_unfused(q, kq, vq, 1.0 / np.sqrt(D), gs, bits, F16, seq_lens=lens)
    got = np.concatenate([np.load(tmp_path / f"heads_{r}.npy") for r in range(world)], axis=1)
    assert max_abs(got, want, F16) <= TOL
