#!/usr/bin/env python
"""Benchmark of the quantized-KV decode hot path.

The line the driver reads (default `--workload decode`), at N = 1, 2, 4, 8
GPUs (one process per GPU, torchrun for N > 1):

value      config 5, long-context serving: B = 64 sequences with ragged
           lengths U[1024, 32768] (numpy seed 5), Hq 32, Hkv 8, D 128, kv4
           group 64, decoded with per-sequence key counts (seq_lens).  The 8
           kv heads are sharded over the N GPUs (8/N each, with their GQA
           query heads): strong scaling, no collective on the data path.
           One step = one decode of all 64 sequences on every rank; steps
           cycle through NL distinct layer caches (more than 3x the 126 MB
           L2 per GPU), replayed from CUDA graphs, timed with
           CUDA events over exactly K steps, max over ranks.  Aggregate
           algorithmic HBM GB/s = K/V codes + scales + biases of every
           sequence's keys, plus q and output, over all ranks.  The timed
           region replays one graph per pass over the NL layers (K // NL
           times, consecutive steps chained by programmatic dependent
           launch) and one graph per layer for the K mod NL left over.
e2e        the same step through the public Python API (kvq.sdpa_decode with
           seq_lens), with each step's q copied from pinned host memory and
           the output copied back inside the timed region; the copies run on
           two copy streams, double-buffered over the layers, so they
           overlap the neighbouring steps' decodes as in a serving loop.
roofline   the decode launch pair of one rank (attn_bal_kernel +
           attn_bal_merge_kernel, the whole step): its algorithmic bytes per
           launch / its CUDA-event time, against the measured HBM copy
           bandwidth.
config2    nested: batched kv4 decode with quantize-on-append (B 8, Hq 32,
           Hkv 8, D 128, 8,193 keys, key outliers), one replica per GPU,
           with its own decode roofline (a CUDA graph per pass over the
           layers).
context_split
           nested: one 131,072-key sequence split along the context over the
           N ranks, partials exchanged over peer memory and merged (a CUDA
           graph per pass over the layers), us per step and the exchange's
           share of it.
kv_projection
           nested: the fused Q/K/V projection + RMSNorms + RoPE + quantize-
           on-append of one decode token through 48 Gemma-4-12B sliding-layer
           weight sets (hidden 3840 -> 16 query + 2 x 8 kv heads of 256,
           4-bit), one replica per GPU, with its HBM roofline; and a
           512-token prefill chunk.
cpu_baseline / --impl reference
           the CPU oracle (C restatement of mlx-bun's unfused op graph) with
           every host core, on a bounded sample of config 5's (sequence, kv
           head) pairs.

Other workloads print their own line: `--workload prefill` (config 4,
tensor-core chunked prefill), `prefill-kv4`, `config1`, `config3` and
`kv-projection`.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mlx-bun_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

L2_BYTES = 126e6
FALLBACK_HBM = 6650.0
UNIT = "GB/s"

CFG5 = dict(B=64, Hq=32, Hkv=8, D=128, bits=4, gs=64, lo=1024, hi=32768, seed=5)
METRIC = ("quantized-KV decode SDPA achieved HBM GB/s (config 5: B64 ragged lengths "
          "U[1024, 32768], Hq32 Hkv8 D128 kv4 gs64, kv heads sharded over the GPUs)")
WORKLOAD = "config5-kv4-ragged-decode-kvhead-shards"

CFG2 = dict(B=8, Hq=32, Hkv=8, D=128, N_prior=8192, bits=4, gs=64, outliers=4)


def kv_row_bytes(c):
    """K and V bytes of one key row of one kv head: codes + scales + biases."""
    return 2 * (c["D"] * c["bits"] // 8 + 2 * (c["D"] // c["gs"]) * 2)


def config5_lens():
    import numpy as np
    c = CFG5
    return np.random.default_rng(c["seed"]).integers(c["lo"], c["hi"] + 1, size=c["B"])


def config5_rank_bytes(lens, hk):
    """Algorithmic bytes of one decode step on a rank owning `hk` kv heads."""
    c = CFG5
    nrep = c["Hq"] // c["Hkv"]
    return int(lens.sum()) * hk * kv_row_bytes(c) + 2 * c["B"] * hk * nrep * c["D"] * 2


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def traffic_ratio(name):
    """DRAM bytes per algorithmic byte of a decode launch, from the committed
    ncu summary profiles/<name> ("traffic_ratio:" line), or None."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.strip().startswith("traffic_ratio:"):
                return float(line.split(":")[1].split()[0])
    except Exception:
        pass
    return None


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.06)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        mhz = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


class Timed:
    """Barrier + synchronize on both sides of a CUDA-event-timed region on
    `stream`; `ms` is the maximum over ranks."""

    def __init__(self, stream, world, device, clocks=None):
        import torch
        self.stream, self.world, self.device, self.clocks = stream, world, device, clocks
        self.e0 = torch.cuda.Event(enable_timing=True)
        self.e1 = torch.cuda.Event(enable_timing=True)
        self.clk = None
        self.ms = None

    def __enter__(self):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if self.clocks:
            self.clocks.start()
            time.sleep(0.1)
        self.e0.record(self.stream)
        return self

    def __exit__(self, *exc):
        import torch
        import torch.distributed as dist
        self.e1.record(self.stream)
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier()
        if self.clocks:
            self.clk = self.clocks.stop()
        t = torch.tensor([self.e0.elapsed_time(self.e1)], device=self.device, dtype=torch.float64)
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        self.ms = float(t.item())
        return False


# ------------------------------------------------------------ CPU oracle --

def cpu_oracle_config5(max_calls, budget_s, threads, seed=0):
    """Time the C oracle on (sequence, kv-head) pairs of config 5 with
    `threads` OpenMP threads.  One call covers `threads` pairs (the first
    `threads` sequences' lengths, one kv head and its 4 query heads each);
    at most `max_calls` calls and about `budget_s` seconds are timed.
    Returns (GB/s, description, calls, seconds)."""
    import numpy as np
    from oracle import oracle as O
    c = CFG5
    D, nrep = c["D"], c["Hq"] // c["Hkv"]
    lens = config5_lens()
    P = max(1, threads)
    sl = np.array([int(lens[i % len(lens)]) for i in range(P)], np.int32)
    Nmax = int(sl.max())
    rng = np.random.default_rng(seed)
    kb = O.to_dtype_bits(rng.standard_normal((1, 1, Nmax, D)).astype(np.float32), O.F16)
    vb = O.to_dtype_bits(rng.standard_normal((1, 1, Nmax, D)).astype(np.float32), O.F16)
    kq = O.quantize(kb, c["gs"], c["bits"], O.F16)
    vq = O.quantize(vb, c["gs"], c["bits"], O.F16)
    kqP = tuple(np.ascontiguousarray(np.broadcast_to(a, (P,) + a.shape[1:])) for a in kq)
    vqP = tuple(np.ascontiguousarray(np.broadcast_to(a, (P,) + a.shape[1:])) for a in vq)
    q = O.to_dtype_bits(rng.standard_normal((P, nrep, 1, D)).astype(np.float32), O.F16)
    scale = 1.0 / np.sqrt(D)

    def call():
        O.sdpa_unfused(q, kqP, vqP, scale, c["gs"], c["bits"], O.F16, seq_lens=sl,
                       threads=threads)

    call()  # warm
    t0 = time.perf_counter()
    call()
    t_call = time.perf_counter() - t0
    calls = max(1, min(max_calls, int(budget_s / max(t_call, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(calls):
        call()
    el = time.perf_counter() - t0
    by = calls * (int(sl.sum()) * kv_row_bytes(c) + 2 * P * nrep * D * 2)
    desc = (f"{calls} calls x {P} (sequence, kv-head) pairs of config 5 (the first {P} "
            f"sequences' lengths, mean {sl.mean():.0f} keys, 4 query heads each), C oracle of "
            f"the unfused op graph, {threads} threads")
    return by / el / 1e9, desc, calls, el


# ------------------------------------------------------- config 5 (main) --

def _fill(cache, B, H, N, D, g, device, chunk):
    """Append N seeded fp16 rows to `cache` in chunks; return the last views."""
    import torch
    views = None
    for s0 in range(0, N, chunk):
        S = min(chunk, N - s0)
        k = torch.randn(B, H, S, D, generator=g, device=device).half()
        v = torch.randn(B, H, S, D, generator=g, device=device).half()
        views = cache.update_and_fetch_quantized(k, v)
        del k, v
    return views


def run_config5(args, rank, world, local_rank):
    import numpy as np
    import torch
    import kvq
    c = CFG5
    B, Hq, Hkv, D = c["B"], c["Hq"], c["Hkv"], c["D"]
    if Hkv % world:
        raise SystemExit("config 5 shards 8 kv heads: run on 1, 2, 4 or 8 GPUs")
    device = torch.device("cuda", local_rank)
    hk = Hkv // world
    nrep = Hq // Hkv
    scale = 1.0 / np.sqrt(D)
    lens = config5_lens()
    Nmax = int(lens.max())
    rank_bytes = config5_rank_bytes(lens, hk)
    total_bytes = config5_rank_bytes(lens, Hkv)
    NL = min(16, max(2, math.ceil(3 * L2_BYTES / rank_bytes)))
    g = torch.Generator(device=device)
    g.manual_seed(5000 + rank)
    sl = torch.tensor(lens, dtype=torch.int32, device=device)
    layers = []
    for _ in range(NL):
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=(Nmax + 255) // 256 * 256)
        K, V = _fill(cache, B, hk, Nmax, D, g, device, 2048)
        q = torch.randn(B, hk * nrep, 1, D, generator=g, device=device).half()
        layers.append(dict(cache=cache, K=K, V=V, q=q, out=torch.empty_like(q)))
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device)

    def step(Ly):
        kvq.sdpa_decode(Ly["q"], Ly["K"], Ly["V"], scale, seq_lens=sl, out=Ly["out"])

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(layers[i % NL])
    stream.synchronize()
    # one graph per pass over the NL layers (consecutive steps chain by
    # programmatic dependent launch inside it), and one per layer for the
    # K mod NL steps left over: exactly K steps are timed
    graphs = []
    for Ly in layers:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            step(Ly)
        graphs.append(gr)
    gpass = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gpass, stream=stream):
        for Ly in layers:
            step(Ly)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            graphs[i % NL].replay()
        gpass.replay()
    torch.cuda.synchronize()

    K = args.steps
    with torch.cuda.stream(stream):
        with Timed(stream, world, device, Clocks(local_rank) if rank == 0 else None) as tm:
            for _ in range(K // NL):
                gpass.replay()
            for i in range(K % NL):
                graphs[i].replay()
    ms = tm.ms

    # e2e through the public API, host buffers, copies inside the timed
    # region: every step uploads its query rows from pinned host memory and
    # downloads its output to pinned host memory, as a serving loop does —
    # the uploads on one copy stream, the downloads on another, so step
    # i + 1's upload and step i - 1's download overlap step i's decode.
    # Layer j's device buffers are reused only after the step that last
    # used them is done with them (its decode for q, its download for out).
    hq = [torch.empty_like(Ly["q"], device="cpu").pin_memory() for Ly in layers]
    ho = [torch.empty_like(Ly["q"], device="cpu").pin_memory() for Ly in layers]
    for j, Ly in enumerate(layers):
        hq[j].copy_(Ly["q"])
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    up = [torch.cuda.Event() for _ in layers]
    dec = [torch.cuda.Event() for _ in layers]
    down = [torch.cuda.Event() for _ in layers]
    K2 = min(K, 200)
    with torch.cuda.stream(stream):
        with Timed(stream, world, device) as te:
            h2d.wait_stream(stream)
            d2h.wait_stream(stream)
            for i in range(K2):
                j = i % NL
                Ly = layers[j]
                if i >= NL:
                    h2d.wait_event(dec[j])       # the last decode that read q_j
                with torch.cuda.stream(h2d):
                    Ly["q"].copy_(hq[j], non_blocking=True)
                    up[j].record(h2d)
                stream.wait_event(up[j])
                if i >= NL:
                    stream.wait_event(down[j])   # the last download of out_j
                step(Ly)
                dec[j].record(stream)
                d2h.wait_event(dec[j])
                with torch.cuda.stream(d2h):
                    ho[j].copy_(Ly["out"], non_blocking=True)
                    down[j].record(d2h)
            stream.wait_stream(d2h)
    e2e_ms = te.ms
    if not torch.isfinite(layers[0]["out"].float()).all():
        raise RuntimeError("non-finite decode output")
    if not all(torch.equal(ho[j], Ly["out"].cpu()) for j, Ly in enumerate(layers)):
        raise RuntimeError("a downloaded output differs from the device's")
    del graphs, gpass

    value = total_bytes * K / (ms / 1e3) / 1e9
    kern_s = ms / 1e3 / K
    achieved = rank_bytes / kern_s / 1e9
    peak, peak_kind = peaks()
    ratio = traffic_ratio("attn_decode_config5.md")
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": K, "warmup": args.warmup, "ms_per_step": round(ms / K, 5),
        "us_per_step": round(1e3 * ms / K, 3),
        "tokens_per_s": round(B * K / (ms / 1e3), 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u4 codes/f16",
        "data": "synthetic (seeded torch.randn K/V/q; lengths numpy PCG64 seed 5)",
        "config": {"workload": WORKLOAD, "batch": B, "Hq": Hq, "Hkv": Hkv, "head_dim": D,
                   "bits": c["bits"], "group_size": c["gs"],
                   "lengths": f"U[{c['lo']}, {c['hi']}] seed {c['seed']}, sum {int(lens.sum())}",
                   "parallelism": f"kv-head shards: {hk} kv head(s) x 64 sequences per GPU, "
                                  f"{world} GPU(s), no collective",
                   "layers_cycled": NL,
                   "l2": f"inputs larger than L2: {NL} distinct layer caches, "
                         f"{NL * rank_bytes / 1e6:.0f} MB per GPU cycled",
                   "timing": "a CUDA graph per pass over the layers (K // NL replays) and "
                             "one per layer (K % NL replays): exactly K steps, CUDA events, "
                             "barrier + synchronize on both sides, max over ranks"},
        "bytes_per_step": total_bytes,
        "e2e": {"value": round(total_bytes * K2 / (e2e_ms / 1e3) / 1e9, 1), "unit": UNIT,
                "h2d_bytes_per_step": int(hq[0].numel() * 2) * world,
                "d2h_bytes_per_step": int(ho[0].numel() * 2) * world,
                "us_per_step": round(1e3 * e2e_ms / K2, 3), "steps": K2,
                "path": "kvq.sdpa_decode per step (eager), q from pinned host memory, output "
                        "back to pinned host memory, every rank; uploads and downloads on two "
                        "copy streams, overlapped with the neighbouring steps' decodes"},
        "gpu_launches": 2 * K,  # per step: attn_bal_kernel + attn_bal_merge_kernel
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "kernel": "decode = attn_bal_kernel<4,128,64,1> (seq_lens) + "
                               "attn_bal_merge_kernel",
                     "kernel_us": round(kern_s * 1e6, 3), "bytes_per_launch": rank_bytes,
                     "traffic": int(ratio * rank_bytes) if ratio else None,
                     "traffic_note": "ncu DRAM bytes per algorithmic byte of a 16-sequence "
                                     "capture, scaled to this launch",
                     "timing": "CUDA events over the K timed graph replays (the step is the "
                               "decode launch pair), max over ranks"},
        "clocks": tm.clk,
    }
    for Ly in layers:
        Ly["cache"].dispose()
    return res


# -------------------------------------------------- config 2 (nested) --

def run_config2(args, rank, world, local_rank):
    """Batched kv4 decode with quantize-on-append, one replica per GPU."""
    import numpy as np
    import torch
    import kvq
    c = CFG2
    device = torch.device("cuda", local_rank)
    B, Hq, Hkv, D, Np = c["B"], c["Hq"], c["Hkv"], c["D"], c["N_prior"]
    scale = 1.0 / np.sqrt(D)
    N = Np + 1
    layer_bytes = B * Hkv * N * kv_row_bytes(c)
    step_bytes = layer_bytes + 2 * B * Hq * D * 2 + B * Hkv * D * 2 * 2
    launch_bytes = layer_bytes + 2 * B * Hq * D * 2
    NL = max(4, math.ceil(3 * L2_BYTES / layer_bytes))
    g = torch.Generator(device=device)
    g.manual_seed(1000 + rank)
    layers = []
    for _ in range(NL):
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=(N + 255) // 256 * 256)
        k = torch.randn(B, Hkv, Np, D, generator=g, device=device)
        k[..., :c["outliers"]] *= 8.0
        v = torch.randn(B, Hkv, Np, D, generator=g, device=device)
        cache.update_and_fetch_quantized(k.half(), v.half())
        del k, v
        kn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
        kn[..., :c["outliers"]] *= 8.0
        vn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
        q = torch.randn(B, Hq, 1, D, generator=g, device=device).half()
        layers.append(dict(cache=cache, kn=kn, vn=vn, q=q, out=torch.empty_like(q)))
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)

    def step(L):
        qk, qv = L["cache"].update_and_fetch_quantized(L["kn"], L["vn"])
        kvq.sdpa_decode(L["q"], qk, qv, scale, out=L["out"])
        L["cache"].trim(1)  # host bookkeeping: every replay does the same work

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(layers[i % NL])
    stream.synchronize()
    # one graph per pass over the layers (a replay is NL steps), and a
    # decode-only graph of the same layers (the roofline's kernel time)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for L in layers:
            step(L)
    views = []
    for L in layers:
        views.append(L["cache"].update_and_fetch_quantized(L["kn"], L["vn"]))
    dec = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dec, stream=stream):
        for L, (qk, qv) in zip(layers, views):
            kvq.sdpa_decode(L["q"], qk, qv, scale, out=L["out"])
    for L in layers:
        L["cache"].trim(1)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
            dec.replay()
    torch.cuda.synchronize()
    reps = max(1, math.ceil(args.steps / NL))
    K = reps * NL
    with torch.cuda.stream(stream):
        with Timed(stream, world, device) as t1:
            for _ in range(reps):
                graph.replay()
        with Timed(stream, world, device) as t2:
            for _ in range(reps):
                dec.replay()
    kern_s = t2.ms / 1e3 / K
    achieved = launch_bytes / kern_s / 1e9
    peak, peak_kind = peaks()
    ratio = traffic_ratio("attn_decode_config2.md")
    out = {
        "workload": "config2-kv4-decode-append: B8 Hq32 Hkv8 D128, 8192 prior keys + 1 appended "
                    "per step, kv4 gs64, key outliers; one replica per GPU (weak)",
        "value": round(world * step_bytes * K / (t1.ms / 1e3) / 1e9, 1), "unit": UNIT,
        "steps": K, "us_per_step": round(1e3 * t1.ms / K, 3), "bytes_per_step": step_bytes,
        "layers_cycled": NL, "timing": "a CUDA graph per pass over the layers, CUDA events",
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "kernel": "decode = attn_bal_kernel<4,128,64,1> + attn_bal_merge_kernel",
                     "kernel_us": round(kern_s * 1e6, 3), "bytes_per_launch": launch_bytes,
                     "traffic": int(ratio * launch_bytes) if ratio else None,
                     "timing": "decode-only graph replays of the same layers, CUDA events"},
    }
    del graph, dec
    for L in layers:
        L["cache"].dispose()
    return out


# ------------------------------------------- context split (nested) --

def run_context_split(args, rank, world, local_rank):
    """Config 5's single 131,072-key sequence split along the context."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import kvq
    from kvq.parallel import ContextSplitDecode, context_ranges
    Hq, Hkv, D, bits, gs, N = 32, 8, 128, 4, 64, 131072
    c = dict(D=D, bits=bits, gs=gs)
    device = torch.device("cuda", local_rank)
    scale = 1.0 / np.sqrt(D)
    a, b = context_ranges(N, world)[rank]
    rank_bytes = (b - a) * Hkv * kv_row_bytes(c) + 2 * Hq * D * 2
    NL = min(32, max(2, math.ceil(3 * L2_BYTES / rank_bytes)))
    g = torch.Generator(device=device)
    g.manual_seed(7000 + rank)
    gq = torch.Generator(device=device)
    gq.manual_seed(77)  # the same queries on every rank
    layers = []
    for _ in range(NL):
        cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=(b - a + 255) // 256 * 256)
        K, V = _fill(cache, 1, Hkv, b - a, D, g, device, 8192)
        q = torch.randn(1, Hq, 1, D, generator=gq, device=device).half()
        layers.append(dict(cache=cache, K=K, V=V, q=q, out=torch.empty_like(q)))
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)
    split = ContextSplitDecode(transport="peer") if world > 1 else None
    R = Hq
    packed = torch.empty(R * (D + 2), dtype=torch.float32, device=device)

    def step(Ly):
        if split is None:
            kvq.sdpa_decode(Ly["q"], Ly["K"], Ly["V"], scale, out=Ly["out"])
        else:
            Ly["out"].copy_(split.step(Ly["q"], Ly["K"], Ly["V"], scale))

    def partial_only(Ly):
        kvq.sdpa_decode_partial(Ly["q"], Ly["K"], Ly["V"], scale, packed_out=packed)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(layers[i % NL])
    stream.synchronize()
    # one graph per pass over the layers (a replay is NL steps); the same
    # pass with the partial decode alone, for the exchange's share
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for Ly in layers:
            step(Ly)
    pgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(pgraph, stream=stream):
        for Ly in layers:
            partial_only(Ly)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
            pgraph.replay()
    torch.cuda.synchronize()
    reps = max(1, math.ceil(args.steps / NL))
    K = reps * NL
    with torch.cuda.stream(stream):
        with Timed(stream, world, device) as t1:
            for _ in range(reps):
                graph.replay()
        with Timed(stream, world, device) as t2:
            for _ in range(reps):
                pgraph.replay()
    if split is not None:
        split.check(stream)
    if not torch.isfinite(layers[0]["out"].float()).all():
        raise RuntimeError("non-finite context-split output")
    del graph, pgraph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # every rank's last exchange is done before the buffers go
    if split is not None:
        split.close()
    for Ly in layers:
        Ly["cache"].dispose()
    total = N * Hkv * kv_row_bytes(c) + 2 * Hq * D * 2 * world
    us = 1e3 * t1.ms / K
    out = {
        "workload": "one 131072-key sequence, Hq32 Hkv8 D128 kv4 gs64, split along the context "
                    f"over {world} GPU(s); partials exchanged over peer memory (CUDA IPC, "
                    "plain stores + flags) and merged in one kernel; a CUDA graph per pass "
                    "over the layers",
        "us_per_step": round(us, 3), "value": round(total * K / (t1.ms / 1e3) / 1e9, 1),
        "unit": UNIT, "steps": K, "layers_cycled": NL,
        "partial_us_per_step": round(1e3 * t2.ms / K, 3),
    }
    if world > 1:
        out["exchange_share"] = round(max(0.0, 1.0 - t2.ms / t1.ms), 4)
        out["exchange_note"] = ("share of the step not spent in the partial decode: the "
                                "exchange-and-merge kernel and its wait for the slowest rank")
    return out


# ----------------------------------------------------- other workloads --

CFG4 = dict(B=1, Hq=32, Hkv=8, D=128, N_prior=16384, L=512, bits=8, gs=64, outliers=4)


def prefill_flops(c):
    """Causal chunk of L rows after N_prior keys: 4 * Hq * L * D * (N_prior + (L + 1) / 2)."""
    return 4 * c["Hq"] * c["L"] * c["D"] * (c["N_prior"] + (c["L"] + 1) / 2)


def run_prefill(args, bits=8):
    """Config 4: chunked prefill of 512 query rows (causal in the chunk) over a
    kv8 cache of 16,384 prior rows plus the chunk, appended first (with
    bits=4, the same shape over a kv4 cache: the warp-specialised kernel).  One step =
    append of the 512 K/V rows + prefill attention; both timed with CUDA
    events over graph replays of NL distinct layers; the attention alone
    (the tensor-core kernel and the merge of units cut between its CTAs) is
    timed the same way for the tensor-core roofline."""
    import numpy as np
    import torch
    import kvq
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    c = dict(CFG4, bits=bits)
    B, Hq, Hkv, D, Np, L = c["B"], c["Hq"], c["Hkv"], c["D"], c["N_prior"], c["L"]
    scale = 1.0 / np.sqrt(D)
    NL = 4 if bits == 8 else 8  # 147 MB of K/V cycled per replay: above L2
    g = torch.Generator(device=device)
    g.manual_seed(11)
    layers = []
    for _ in range(NL):
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=(Np + L + 255) // 256 * 256)
        k = torch.randn(B, Hkv, Np, D, generator=g, device=device)
        k[..., :c["outliers"]] *= 8.0
        v = torch.randn(B, Hkv, Np, D, generator=g, device=device)
        cache.update_and_fetch_quantized(k.half(), v.half())
        kn = torch.randn(B, Hkv, L, D, generator=g, device=device)
        kn[..., :c["outliers"]] *= 8.0
        layers.append(dict(cache=cache, kn=kn.half(),
                           vn=torch.randn(B, Hkv, L, D, generator=g, device=device).half(),
                           q=torch.randn(B, Hq, L, D, generator=g, device=device).half()))
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()

    def step(Ly):
        qk, qv = Ly["cache"].update_and_fetch_quantized(Ly["kn"], Ly["vn"])
        Ly["out"] = kvq.quantized_sdpa(Ly["q"], qk, qv, scale, Ly["cache"].make_mask(L, None))
        Ly["cache"].trim(L)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            for Ly in layers:
                step(Ly)
        torch.cuda.synchronize()
        g_step = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step, stream=stream):
            for Ly in layers:
                step(Ly)
        views, masks = [], []
        for Ly in layers:
            views.append(Ly["cache"].update_and_fetch_quantized(Ly["kn"], Ly["vn"]))
            masks.append(Ly["cache"].make_mask(L, None))
        g_att = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_att, stream=stream):
            for Ly, (qk, qv), m in zip(layers, views, masks):
                kvq.quantized_sdpa(Ly["q"], qk, qv, scale, m)
        for Ly in layers:
            Ly["cache"].trim(L)
        for _ in range(3):
            g_step.replay()
            g_att.replay()
        torch.cuda.synchronize()
    reps = max(1, args.steps // NL)
    with torch.cuda.stream(stream):
        with Timed(stream, 1, device, Clocks(0)) as t1:
            for _ in range(reps):
                g_step.replay()
        with Timed(stream, 1, device) as t2:
            for _ in range(reps):
                g_att.replay()
    step_ms = t1.ms / (reps * NL)
    att_ms = t2.ms / (reps * NL)
    fl = prefill_flops(c)
    try:
        peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
        pk = "measured (bf16 dense burst; fp16 runs at the same rate)"
    except Exception:
        peak, pk = 1590.0, "fallback"
    att_tf = fl / (att_ms / 1e3) / 1e12
    kern = ("prefill_tc_kernel (tcgen05 UMMA, TMEM accumulators) + prefill_tc_merge_kernel"
            if bits == 8 else
            "prefill_tc2_kernel (warp-specialised tcgen05, K as fp16 hi + lo) + "
            "prefill_tc_merge_kernel")
    print(json.dumps({
        "metric": f"quantized-KV chunked prefill TFLOP/s (config 4: B1 Hq32 Hkv8 D128, 16384 "
                  f"prior + 512-row causal chunk, kv{bits} gs64)",
        "value": round(fl / (step_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": reps * NL, "warmup": args.warmup, "ms_per_step": round(step_ms, 5),
        "higher_is_better": True, "dtype": f"u{bits} codes/f16", "data": "synthetic (seeded torch.randn)",
        "config": {"workload": f"config4-kv{bits}-prefill-append", "flops_per_step": fl,
                   "layers_cycled": NL, "l2": f"{NL} distinct layers (147 MB of K/V) per replay"},
        "roofline": {"bound": "tensor", "achieved": round(att_tf, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(att_tf / peak, 4), "peak_kind": pk,
                     "kernel": kern, "kernel_us": round(att_ms * 1e3, 3)},
        "gpu_launches": 3 * reps * NL, "clocks": t1.clk}))


# ------------------------------------------- fused Q/K/V projection --

# Gemma-4-12B sliding-attention layer, query and K/V sides: hidden 3840 ->
# 16 query heads and 8 kv heads of 256, 4-bit group-64 weights with biases,
# bf16 activations, Q and K RMSNorm with weights, V RMSNorm without, default
# RoPE (base 10000) on all 256 dims of Q and K, a kv4 group-64 cache; 48
# layers, as the model has.
CFGP = dict(hidden=3840, Hq=16, Hkv=8, D=256, wbits=4, wgs=64, bits=4, gs=64, layers=48,
            chunk=512)


def projection_out_features(c):
    """Output features of one call: Q, K and V."""
    return (c["Hq"] + 2 * c["Hkv"]) * c["D"]


def projection_bytes(c, rows):
    """Algorithmic HBM bytes of one fused call over `rows` token rows: the
    Q, K and V weight triples (packed codes + bf16 scales and biases), the
    bf16 input rows, the bf16 query rows written out and the quantized K/V
    rows written to the cache."""
    out, inn = projection_out_features(c), c["hidden"]
    w = out * inn * c["wbits"] // 8 + 2 * out * (inn // c["wgs"]) * 2
    x = rows * inn * 2
    q = rows * c["Hq"] * c["D"] * 2
    row = c["D"] * c["bits"] // 8 + 2 * (c["D"] // c["gs"]) * 2
    return w + x + q + 2 * rows * c["Hkv"] * row


def projection_layers(c, n, device, g):
    """`n` layers of random 4-bit Q/K/V projection weights (codes uniform,
    scales U[0.001, 0.005], biases -7.5 x scale: outputs of order one) with
    their growing kv caches."""
    import torch
    import kvq
    H, D, hid = c["Hkv"], c["D"], c["hidden"]

    def qlinear(out_f):
        words = hid * c["wbits"] // 32
        packed = torch.randint(-2 ** 31, 2 ** 31 - 1, (out_f, words), generator=g,
                               device=device, dtype=torch.int32)
        sc = (torch.rand(out_f, hid // c["wgs"], generator=g, device=device) * 0.004 + 0.001)
        bi = -7.5 * sc
        return kvq.QuantizedLinear(packed, sc.bfloat16(), bi.bfloat16(), c["wgs"], c["wbits"])

    def norm_w():
        return (torch.rand(D, generator=g, device=device) + 0.5).bfloat16()

    layers = []
    for _ in range(n):
        proj = kvq.KvProjection(qlinear(H * D), qlinear(H * D), D, k_norm_weight=norm_w(),
                                rope_dims=D, rope_base=10000.0, q_proj=qlinear(c["Hq"] * D),
                                q_heads=c["Hq"], q_norm_weight=norm_w())
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=2048)
        layers.append(dict(proj=proj, cache=cache))
    return layers


def projection_q_out(c, tokens, device):
    """The query rows' buffer of one call over `tokens` tokens."""
    import torch
    return torch.empty(1, c["Hq"], tokens, c["D"], dtype=torch.bfloat16, device=device)


def run_kv_projection(args, rank, world, local_rank):
    """Fused Q/K/V projection + norms + RoPE + quantize-on-append
    (kvq_append_projected), one replica per GPU.  Decode: one token per
    step through each of the 48 layers (a CUDA graph per pass over the
    layers; 850 MB of weights cycled, above L2), timed with CUDA events.
    Prefill: one 512-token chunk through one layer, timed the same way
    (FLOPs: 2 x tokens x hidden x (Q + K + V output features))."""
    import torch
    c = CFGP
    device = torch.device("cuda", local_rank)
    hid = c["hidden"]
    out_f = projection_out_features(c)
    g = torch.Generator(device=device)
    g.manual_seed(2000 + rank)
    layers = projection_layers(c, c["layers"], device, g)
    x1 = torch.randn(1, 1, hid, generator=g, device=device).bfloat16()
    xc = torch.randn(1, c["chunk"], hid, generator=g, device=device).bfloat16()
    q1, qc, q0 = (projection_q_out(c, n, device) for n in (1, c["chunk"], 1000))
    # every cache starts at offset 1000 (positions in range of a real decode)
    for Ly in layers:
        Ly["cache"].update_and_fetch_projected(torch.zeros(1, 1000, hid, device=device,
                                                           dtype=torch.bfloat16), Ly["proj"],
                                               q_out=q0)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)

    def step(Ly, x):
        Ly["cache"].update_and_fetch_projected(x, Ly["proj"], q_out=q1 if x.shape[1] == 1 else qc)
        Ly["cache"].trim(x.shape[1])  # host bookkeeping: every replay writes the same rows

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            for Ly in layers:
                step(Ly, x1)
            step(layers[0], xc)
        torch.cuda.synchronize()
        g_dec = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_dec, stream=stream):
            for Ly in layers:
                step(Ly, x1)
        g_pre = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_pre, stream=stream):
            step(layers[0], xc)
        for _ in range(3):
            g_dec.replay()
            g_pre.replay()
        torch.cuda.synchronize()
    NL = c["layers"]
    reps = max(1, math.ceil(args.steps / NL))
    with torch.cuda.stream(stream):
        with Timed(stream, world, device) as t1:
            for _ in range(reps):
                g_dec.replay()
        preps = max(3, min(50, args.steps // 8))
        with Timed(stream, world, device) as t2:
            for _ in range(preps):
                g_pre.replay()
    dec_s = t1.ms / 1e3 / (reps * NL)
    pre_s = t2.ms / 1e3 / preps
    nb = projection_bytes(c, 1)
    achieved = nb / dec_s / 1e9
    peak, peak_kind = peaks()
    flops = 2 * c["chunk"] * hid * out_f
    ratio = traffic_ratio("kv_projection_decode.md")
    res = {
        "workload": "gemma4-12b-sliding-qkv-projection: hidden 3840 -> Hq16 + Hkv8 + Hkv8 x "
                    "D256, 4-bit gs64 weights, Q and K RMSNorm+RoPE, V RMSNorm, kv4 gs64 "
                    "cache; one replica per GPU (weak)",
        "decode": {"us_per_layer": round(dec_s * 1e6, 3), "layers_cycled": NL,
                   "steps": reps * NL, "bytes_per_layer": nb,
                   "value": round(world * nb / dec_s / 1e9, 1), "unit": UNIT,
                   "timing": "a CUDA graph per pass over the 48 layers, CUDA events"},
        "prefill_chunk": {"tokens": c["chunk"], "us_per_layer": round(pre_s * 1e6, 2),
                          "tflops": round(flops / pre_s / 1e12, 2),
                          "kernels": "proj_xprep_kernel + proj_mma_kernel (mma.sync, codes as "
                                     "exact fp16 operands) + proj_epilogue_warp_kernel"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "kernel": "proj_cluster_kernel<4,4,bf16,1,8> (one launch per layer)",
                     "kernel_us": round(dec_s * 1e6, 3), "bytes_per_launch": nb,
                     "traffic": int(ratio * nb) if ratio else None},
        "gpu_launches": reps * NL,
    }
    del g_dec, g_pre
    for Ly in layers:
        Ly["cache"].dispose()
    return res


def print_kv_projection(args):
    import torch
    torch.cuda.set_device(0)
    r = run_kv_projection(args, 0, 1, 0)
    print(json.dumps({
        "metric": "fused Q/K/V projection + norms + RoPE + quantize-on-append achieved HBM GB/s "
                  "(decode, Gemma-4-12B sliding-layer shapes)",
        "value": r["decode"]["value"], "unit": UNIT, "n_gpus": 1, "steps": r["decode"]["steps"],
        "warmup": args.warmup, "ms_per_step": round(r["decode"]["us_per_layer"] / 1e3, 6),
        "higher_is_better": True, "dtype": "u4 weights/bf16", "data": "synthetic (seeded torch)",
        "config": {"workload": r["workload"], "l2": "48 distinct layers (850 MB of weights) "
                   "per replay"},
        "roofline": r["roofline"], "prefill_chunk": r["prefill_chunk"],
        "gpu_launches": r["gpu_launches"]}))


CONFIG_DESC = {
    "config1": "single decode step: B1 Hq16 Hkv4 D128 N2048 kv8 gs64, 64 distinct layers cycled",
    "config3": "Gemma-style window: B4 Hq8 Hkv4 D256 kv8 gs64; per step 5 rotating layers (window "
               "1024, 4096 tokens written) + 1 global layer (4096), append + decode each",
}


def run_config(args):
    """Secondary lines for configs 1 and 3 on one GPU (graph of one pass)."""
    import numpy as np
    import torch
    import kvq
    w = args.workload
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device)
    g.manual_seed(3000)
    steps, keep = [], []
    nbytes = 0
    if w == "config1":
        B, Hq, Hkv, D, N, bits, gs = 1, 16, 4, 128, 2048, 8, 64
        rb = kv_row_bytes(dict(D=D, bits=bits, gs=gs))
        scale = 1.0 / np.sqrt(D)
        for _ in range(64):
            cache = kvq.QuantizedKVCache(gs, bits)
            kq, vq = _fill(cache, B, Hkv, N, D, g, device, N)
            q = torch.randn(B, Hq, 1, D, generator=g, device=device).half()
            out = torch.empty_like(q)
            keep.append((cache, kq, vq, q, out))
            steps.append(lambda kq=kq, vq=vq, q=q, out=out:
                         kvq.sdpa_decode(q, kq, vq, scale, out=out))
            nbytes += B * Hkv * N * rb + 2 * B * Hq * D * 2
    else:
        B, Hq, Hkv, D, bits, gs, win = 4, 8, 4, 256, 8, 64, 1024
        rb = kv_row_bytes(dict(D=D, bits=bits, gs=gs))
        scale = 1.0 / 16.0
        for _ in range(3):  # 3 x (5 + 1) layers: 241 MB cycled, above L2
            for li in range(6):
                local = li < 5
                cache = kvq.RotatingQuantizedKVCache(win, gs, bits) if local else \
                    kvq.QuantizedKVCache(gs, bits, reserve_rows=4352)
                _fill(cache, B, Hkv, 4096, D, g, device, win)
                kn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
                vn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
                q = torch.randn(B, Hq, 1, D, generator=g, device=device).half()
                out = torch.empty_like(q)
                kq, vq = cache.update_and_fetch_quantized(kn, vn)  # steady-state length
                n = kq.shape[2]
                if not local:
                    cache.trim(1)
                keep.append((cache, kn, vn, q, out))

                def st(cache=cache, kn=kn, vn=vn, q=q, out=out, local=local):
                    k2, v2 = cache.update_and_fetch_quantized(kn, vn)
                    kvq.sdpa_decode(q, k2, v2, scale, out=out)
                    if not local:
                        cache.trim(1)  # host bookkeeping: every replay the same work
                steps.append(st)
                nbytes += B * Hkv * n * rb + 2 * B * Hq * D * 2 + B * Hkv * D * 2 * 2
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            for s in steps:
                s()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for s in steps:
            s()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    reps = max(1, (args.steps + len(steps) - 1) // len(steps))
    with torch.cuda.stream(stream):
        with Timed(stream, 1, device, Clocks(0)) as tm:
            for _ in range(reps):
                graph.replay()
    K = reps * len(steps)
    gbs = nbytes * reps / (tm.ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    print(json.dumps({
        "metric": f"quantized-KV decode SDPA achieved HBM GB/s ({w})", "value": round(gbs, 1),
        "unit": UNIT, "n_gpus": 1, "steps": K, "warmup": args.warmup,
        "ms_per_step": round(tm.ms / K, 5), "us_per_step": round(1e3 * tm.ms / K, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 codes/f16",
        "data": "synthetic (seeded torch.randn)",
        "config": {"workload": w, "description": CONFIG_DESC[w], "bytes_per_pass": int(nbytes),
                   "steps_per_pass": len(steps),
                   "timing": "CUDA graph of one pass, CUDA events"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": UNIT,
                     "frac": round(gbs / peak, 4), "peak_kind": peak_kind,
                     "note": "whole step (append included where the config appends)"},
        "clocks": tm.clk}))


def profile_run(args):
    """Fixed small workloads for ncu (no timing): `--steps` launches of one
    kernel.  decode / append: 3 config-2 layers (227 MB, above L2), cycled;
    config5: the first 16 sequences of config 5, all 8 kv heads (315 MB);
    projection: one-token fused K/V projection appends through 24 layers of
    Gemma-4-12B sliding-layer weights (213 MB), cycled; projection-prefill:
    512-token chunks through 2 such layers."""
    import numpy as np
    import torch
    import kvq
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device)
    g.manual_seed(7)
    if args.profile == "projection":
        c = CFGP
        layers = projection_layers(c, 24, device, g)  # 425 MB of weights, above L2
        x1 = torch.randn(1, 1, c["hidden"], generator=g, device=device).bfloat16()
        q1 = projection_q_out(c, 1, device)
        for i in range(args.steps):
            Ly = layers[i % 24]
            Ly["cache"].update_and_fetch_projected(x1, Ly["proj"], q_out=q1)
            Ly["cache"].trim(1)
        torch.cuda.synchronize()
        print(json.dumps({"profile": "projection", "launches": args.steps,
                          "algorithmic_bytes_per_launch": projection_bytes(c, 1)}))
        return
    if args.profile == "projection-prefill":
        c = CFGP
        layers = projection_layers(c, 2, device, g)
        xc = torch.randn(1, c["chunk"], c["hidden"], generator=g, device=device).bfloat16()
        qc = projection_q_out(c, c["chunk"], device)
        for i in range(args.steps):
            Ly = layers[i % 2]
            Ly["cache"].update_and_fetch_projected(xc, Ly["proj"], q_out=qc)
            Ly["cache"].trim(c["chunk"])
        torch.cuda.synchronize()
        print(json.dumps({"profile": "projection-prefill", "launches": args.steps,
                          "flops_per_launch": 2 * c["chunk"] * c["hidden"] *
                          projection_out_features(c)}))
        return
    if args.profile == "config5":
        c = CFG5
        lens = config5_lens()[:16]
        Nmax = int(lens.max())
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=(Nmax + 255) // 256 * 256)
        K, V = _fill(cache, 16, c["Hkv"], Nmax, c["D"], g, device, 2048)
        q = torch.randn(16, c["Hq"], 1, c["D"], generator=g, device=device).half()
        sl = torch.tensor(lens, dtype=torch.int32, device=device)
        for _ in range(args.steps):
            out = kvq.sdpa_decode(q, K, V, 1.0 / np.sqrt(c["D"]), seq_lens=sl)
        torch.cuda.synchronize()
        print(json.dumps({"profile": "config5", "launches": args.steps,
                          "algorithmic_bytes_per_launch":
                              int(lens.sum()) * c["Hkv"] * kv_row_bytes(c) + 2 * 16 * c["Hq"] *
                              c["D"] * 2,
                          "out_mean_abs": float(out.float().abs().mean())}))
        return
    c = CFG2
    B, Hq, Hkv, D, Np = c["B"], c["Hq"], c["Hkv"], c["D"], c["N_prior"]
    layers = []
    for _ in range(3):
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=(Np + 256) // 256 * 256)
        k = torch.randn(B, Hkv, Np, D, generator=g, device=device)
        k[..., :c["outliers"]] *= 8.0
        cache.update_and_fetch_quantized(k.half(), torch.randn(B, Hkv, Np, D, generator=g,
                                                               device=device).half())
        kn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
        vn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
        q = torch.randn(B, Hq, 1, D, generator=g, device=device).half()
        layers.append(dict(cache=cache, kn=kn, vn=vn, q=q, out=torch.empty_like(q)))
    scale = 1.0 / np.sqrt(D)
    views = []
    for L in layers:
        views.append(L["cache"].update_and_fetch_quantized(L["kn"], L["vn"]))
        L["cache"].trim(1)
    for i in range(args.steps):
        L = layers[i % 3]
        if args.profile == "decode":
            kvq.sdpa_decode(L["q"], views[i % 3][0], views[i % 3][1], scale, out=L["out"])
        else:
            L["cache"].update_and_fetch_quantized(L["kn"], L["vn"])
            L["cache"].trim(1)
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.profile, "launches": args.steps,
                      "out_mean_abs": float(layers[0]["out"].float().abs().mean())}))


# ----------------------------------------------------------------- main --

def reference_arm(args, rank):
    """mlx-bun's own CPU path cannot run here (Bun + MLX, macOS arm64 only);
    its op graph restated in C is timed on every host core, rank 0 only."""
    if rank != 0:
        return
    threads = host_cores()
    K = max(1, args.steps)
    gbs, desc, calls, el = cpu_oracle_config5(K, 60.0, threads)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": calls, "steps_requested": K, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u4 codes/f16", "data": "synthetic (seeded numpy)",
        "config": {"workload": WORKLOAD},
        "cpu_baseline": {"value": round(gbs, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(gbs, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "mlx-bun's own CPU path (MLX CPU stream under Bun) cannot run on this box; the C "
                "restatement of its op graph is timed with an explicit thread count of every "
                "host core (torchrun's OMP_NUM_THREADS=1 does not apply); each step is one "
                "oracle call, at most ~60 s of them"}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="kvq", choices=["kvq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-nested", action="store_true",
                    help="skip the nested config-2 and context-split measurements")
    ap.add_argument("--workload", choices=["decode", "prefill", "prefill-kv4", "config1", "config3",
                                           "kv-projection"],
                    default="decode",
                    help="decode: the config-5 line the driver reads (default); prefill: "
                         "config 4 chunked prefill (kv8); prefill-kv4: the same shape in kv4; "
                         "config1 / config3: their own lines; kv-projection: the fused K/V "
                         "projection + append alone")
    ap.add_argument("--profile", choices=["decode", "append", "config5", "projection",
                                          "projection-prefill"],
                    default=None,
                    help="run only the named kernel on a small fixed workload, `--steps` "
                         "launches, no timing (for ncu captures)")
    args = ap.parse_args()
    if args.profile:
        return profile_run(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "prefill-kv4":
        return run_prefill(args, bits=4)
    if args.workload in CONFIG_DESC:
        return run_config(args)
    if args.workload == "kv-projection":
        return print_kv_projection(args)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        res = run_config5(args, rank, world, local_rank)
        if not args.no_nested:
            c2 = run_config2(args, rank, world, local_rank)
            ctx = run_context_split(args, rank, world, local_rank)
            kp = run_kv_projection(args, rank, world, local_rank)
            if res is not None:
                res["config2"] = c2
                res["context_split"] = ctx
                res["kv_projection"] = kp
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                threads = host_cores()
                gbs, desc, _, _ = cpu_oracle_config5(10 ** 6, 15.0, threads)
                res["cpu_baseline"] = {"value": round(gbs, 4), "unit": UNIT, "cores": threads,
                                       "kind": "port", "sample": desc}
            print(json.dumps(res))
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
