"""Multi-GPU paths on real GPUs over NCCL (skipped with fewer than two GPUs).

* Context split: one 131,072-key sequence is split into contiguous ranges,
  one per rank; each rank computes (m, l, o) partials of its range, the
  partials move to every rank — over peer memory (the exchange kernel) or
  through an NCCL all-gather — and are merged.  Every rank's result must
  match the single-GPU decode over all keys within the decode tolerance
  (2e-3 on fp16 outputs), in eager steps and in CUDA-graph replays, and
  rank 0's must match the oracle.
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


def _context_split_worker(rank, world, port, out_dir, transport):
    _setup(rank, world, port)
    import torch
    import torch.distributed as dist
    import kvq
    from helpers import F16, from_torch, max_abs
    from kvq.parallel import ContextSplitDecode, context_ranges
    from oracle import oracle as O
    split = None
    try:
        # the full-size sequence of config 5: 131,072 keys, drawn on the GPU
        # from the same seed on every rank; rank r attends its own range
        B, Hq, Hkv, N, D, gs, bits = 1, 32, 8, 131072, 128, 64, 4
        g = torch.Generator(device="cuda")
        g.manual_seed(61)
        cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=N)
        for s0 in range(0, N, 8192):
            k = torch.randn(B, Hkv, 8192, D, generator=g, device="cuda").half()
            v = torch.randn(B, Hkv, 8192, D, generator=g, device="cuda").half()
            Kf, Vf = cache.update_and_fetch_quantized(k, v)
        q = torch.randn(B, Hq, 1, D, generator=g, device="cuda").half()
        scale = 1.0 / np.sqrt(D)
        a, b = context_ranges(N, world)[rank]
        K, V = Kf.slice_rows(a, b), Vf.slice_rows(a, b)
        split = ContextSplitDecode(transport=transport)
        outs = [split.step(q, K, V, scale).clone() for _ in range(2)]  # buffers reused
        # the same step recorded once in a CUDA graph and replayed twice
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            gout = split.step(q, K, V, scale)
        for _ in range(2):
            graph.replay()
            torch.cuda.synchronize()
            outs.append(gout.clone())
        split.check()
        full = kvq.sdpa_decode(q, Kf, Vf, scale)
        torch.cuda.synchronize()
        errs = [max_abs(from_torch(o, F16), from_torch(full, F16), F16) for o in outs]
        err_oracle = -1.0
        if rank == 0:
            trip = []
            for t in (Kf, Vf):
                trip.append(tuple(
                    x.contiguous().view(torch.int32 if x.dtype == torch.int32 else torch.int16)
                    .cpu().numpy().view(np.uint32 if x.dtype == torch.int32 else np.uint16)
                    for x in (t.packed, t.scales, t.biases)))
            want = O.sdpa_unfused(from_torch(q, F16), trip[0], trip[1], scale, gs, bits, F16)
            err_oracle = max_abs(from_torch(outs[-1], F16), want, F16)
        same = all(torch.equal(outs[0], o) for o in outs[1:])
        np.save(os.path.join(out_dir, f"ctx_{rank}.npy"),
                np.array([max(errs), err_oracle, float(same)]))
        del graph
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        if split is not None:
            split.close()
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


def _spawn(fn, world, tmp_path, *extra):
    import torch.multiprocessing as mp
    mp.start_processes(fn, args=(world, _free_port(), str(tmp_path)) + extra, nprocs=world,
                       join=True, start_method="spawn")


@pytest.mark.timeout(900)
@pytest.mark.parametrize("transport", ["peer", "collective"])
def test_context_split_131072_keys(tmp_path, transport):
    """Every rank's output equals the one-GPU decode over all keys (2e-3) in
    eager steps and in graph replays, identically across steps; rank 0's
    equals the oracle's."""
    import torch
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs two or more GPUs")
    world = min(world, 8)
    _spawn(_context_split_worker, world, tmp_path, transport)
    for r in range(world):
        err_full, err_oracle, same = np.load(tmp_path / f"ctx_{r}.npy")
        assert err_full <= TOL, (r, err_full)
        assert same == 1.0, r
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
