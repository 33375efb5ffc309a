#!/usr/bin/env python
"""Benchmark of the quantized-KV decode hot path.

One step = one attention layer of batched kv4 decode: quantize-on-append of
one new K/V row per sequence into the layer's cache, then flash-decoding SDPA
of 32 query heads (8 kv heads, GQA 4) over the 8193-row cache, for B = 8
sequences (D 128, group 64, fp16, keys with 4 outlier channels x8).  Steps
cycle through NL distinct layer caches whose total size (NL x 75.5 MB)
exceeds twice the 126 MB L2, so every step streams its K/V from HBM; after
each step the layer is trimmed by one token (host bookkeeping only) so every
step does identical work.

value      aggregate algorithmic HBM GB/s over all ranks (K/V packed codes +
           scales + biases of 8193 rows, q, output, appended rows) for K steps
           replayed from CUDA graphs, timed with CUDA events, max over ranks.
e2e        the same metric through the public Python API per step, with the
           step's q and new K/V rows copied from pinned host memory and the
           output copied back inside the timed region.
roofline   the decode kernel alone: algorithmic bytes per launch / its mean
           CUDA-event duration inside the timed graphs, against the measured
           HBM copy bandwidth.
cpu_baseline / --impl reference
           the CPU oracle (C restatement of mlx-bun's unfused op graph, all
           host threads) on a bounded sample of the same workload.

Multi-GPU (torchrun): each rank owns its own shard of sequences (weak
scaling, no communication on the data path).
"""
import argparse
import json
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

CFG = dict(B=8, Hq=32, Hkv=8, D=128, N_prior=8192, bits=4, gs=64, outliers=4)
METRIC = "quantized-KV decode SDPA achieved HBM GB/s (config 2: B8 Hq32 Hkv8 D128 N8193 kv4 gs64, append+decode per step)"
UNIT = "GB/s"
WORKLOAD = "config2-kv4-decode-append"
FALLBACK_HBM = 6650.0


def kv_row_bytes(c):
    return 2 * (c["D"] * c["bits"] // 8 + 2 * (c["D"] // c["gs"]) * 2)


def step_bytes(c):
    N = c["N_prior"] + 1
    kv = c["B"] * c["Hkv"] * N * kv_row_bytes(c)
    q = c["B"] * c["Hq"] * c["D"] * 2
    app = c["B"] * c["Hkv"] * c["D"] * 2 * 2
    return kv + 2 * q + app


def decode_launch_bytes(c):
    N = c["N_prior"] + 1
    return c["B"] * c["Hkv"] * N * kv_row_bytes(c) + 2 * c["B"] * c["Hq"] * c["D"] * 2


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def traffic_from_profiles():
    """dram bytes of the decode's attention launch from the committed ncu summary
    (the merge reads the partials from L2), or None."""
    p = os.path.join(ROOT, "profiles", "attn_decode_config2.md")
    try:
        for line in open(p):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip().split()[0])
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


# ------------------------------------------------------------ CPU oracle --

def cpu_oracle_sample(K_steps, budget_s, seed=0):
    """Time the C oracle on (sequence, kv-head) pairs of config 2.

    Returns (GB/s, threads, description).  Each timed call covers `pairs`
    of the 64 (b, kv-head) pairs of one step (N = 8193 rows, 4 query heads
    each), sized so K_steps calls take about `budget_s` seconds."""
    import numpy as np
    from oracle import oracle as O
    c = CFG
    N, D, nrep = c["N_prior"] + 1, c["D"], c["Hq"] // c["Hkv"]
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((1, 1, N, D)).astype(np.float32)
    k[..., :c["outliers"]] *= 8.0
    kb = O.to_dtype_bits(k, O.F16)
    vb = O.to_dtype_bits(rng.standard_normal((1, 1, N, D)).astype(np.float32), O.F16)
    kq = O.quantize(kb, c["gs"], c["bits"], O.F16)
    vq = O.quantize(vb, c["gs"], c["bits"], O.F16)
    threads = O.max_threads()
    # one pair per thread per call: [threads, 1, N, *] replicated pair data
    P = max(1, threads)
    kqP = tuple(np.ascontiguousarray(np.broadcast_to(a, (P,) + a.shape[1:])) for a in kq)
    vqP = tuple(np.ascontiguousarray(np.broadcast_to(a, (P,) + a.shape[1:])) for a in vq)
    q = O.to_dtype_bits(rng.standard_normal((P, nrep, 1, D)).astype(np.float32), O.F16)
    scale = 1.0 / np.sqrt(D)
    O.sdpa_unfused(q, kqP, vqP, scale, c["gs"], c["bits"], O.F16)  # warm
    t0 = time.perf_counter()
    O.sdpa_unfused(q, kqP, vqP, scale, c["gs"], c["bits"], O.F16)
    t_call = time.perf_counter() - t0
    # time at most K_steps calls, and no more than budget_s of work
    steps = max(1, min(K_steps, int(budget_s / max(t_call, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        O.sdpa_unfused(q, kqP, vqP, scale, c["gs"], c["bits"], O.F16)
    el = time.perf_counter() - t0
    pairs = P * steps
    by = pairs * (N * kv_row_bytes(c) + 2 * nrep * D * 2)
    desc = (f"{pairs} (sequence, kv-head) pairs of config 2 (N=8193, 4 query heads each, "
            f"{pairs / 64:.2f} layer-steps), C oracle of the unfused op graph, {threads} threads")
    return by / el / 1e9, threads, desc, el


# ------------------------------------------------------------- GPU arm --

def setup_layers(c, NL, device, seed):
    import torch
    import kvq
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    B, Hq, Hkv, D, Np = c["B"], c["Hq"], c["Hkv"], c["D"], c["N_prior"]
    reserve = (Np + 1 + 255) // 256 * 256
    layers = []
    for _ in range(NL):
        cache = kvq.QuantizedKVCache(c["gs"], c["bits"], reserve_rows=reserve)
        k = torch.randn(B, Hkv, Np, D, generator=g, device=device, dtype=torch.float32)
        k[..., :c["outliers"]] *= 8.0
        v = torch.randn(B, Hkv, Np, D, generator=g, device=device, dtype=torch.float32)
        cache.update_and_fetch_quantized(k.half(), v.half())
        del k, v
        kn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
        kn[..., :c["outliers"]] *= 8.0
        vn = torch.randn(B, Hkv, 1, D, generator=g, device=device).half()
        q = torch.randn(B, Hq, 1, D, generator=g, device=device).half()
        layers.append(dict(cache=cache, kn=kn, vn=vn, q=q, out=torch.empty_like(q)))
    torch.cuda.synchronize()
    return layers


def gpu_step(L, scale):
    import kvq
    qk, qv = L["cache"].update_and_fetch_quantized(L["kn"], L["vn"])
    kvq.sdpa_decode(L["q"], qk, qv, scale, out=L["out"])
    L["cache"].trim(1)


def run_gpu(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    import kvq

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    c = CFG
    scale = 1.0 / np.sqrt(c["D"])
    layer_bytes = c["B"] * c["Hkv"] * (c["N_prior"] + 1) * kv_row_bytes(c)
    NL = max(4, int(np.ceil(2 * 126e6 * 1.5 / layer_bytes)))
    layers = setup_layers(c, NL, device, seed=1000 + rank)
    stream = torch.cuda.Stream(device)
    # warm-up (also sizes the library-managed workspace before capture)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            gpu_step(layers[i % NL], scale)
    stream.synchronize()

    # ---- graphs: one replay = NL steps (one pass over the layers)
    per_graph = NL
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for j in range(per_graph):
            gpu_step(layers[j], scale)
    # decode-only graph over the same layers (kernel timing for the roofline)
    views = []
    for L in layers:
        L["cache"].update_and_fetch_quantized(L["kn"], L["vn"])  # leave row 8192 written
        views.append(L["cache"].fetch())
    g_dec = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_dec, stream=stream):
        for j in range(per_graph):
            kvq.sdpa_decode(layers[j]["q"], views[j][0], views[j][1], scale, out=layers[j]["out"])
    for L in layers:
        L["cache"].trim(1)
    for _ in range(3):
        graph.replay()
        g_dec.replay()
    torch.cuda.synchronize()

    K = args.steps
    reps = max(1, (K + per_graph - 1) // per_graph)
    K = reps * per_graph
    clocks = Clocks(local_rank) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.start()
        time.sleep(0.1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        for r in range(reps):
            graph.replay()
        e1.record()
        # the decode kernel alone, same layers, same stream, right after
        e2.record()
        for r in range(reps):
            g_dec.replay()
        e3.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = e0.elapsed_time(e1)
    kern_ms = [e2.elapsed_time(e3) / (reps * per_graph)]
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # ---- e2e through the public API with host buffers
    import kvq as _k  # noqa: F401
    hq = [torch.empty_like(L["q"], device="cpu").pin_memory() for L in layers]
    hk = [torch.empty_like(L["kn"], device="cpu").pin_memory() for L in layers]
    hv = [torch.empty_like(L["vn"], device="cpu").pin_memory() for L in layers]
    ho = [torch.empty_like(L["q"], device="cpu").pin_memory() for L in layers]
    for j, L in enumerate(layers):
        hq[j].copy_(L["q"])
        hk[j].copy_(L["kn"])
        hv[j].copy_(L["vn"])
    K2 = min(K, max(200, NL * 50))
    K2 = (K2 + NL - 1) // NL * NL
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record()
        for i in range(K2):
            j = i % NL
            L = layers[j]
            L["q"].copy_(hq[j], non_blocking=True)
            L["kn"].copy_(hk[j], non_blocking=True)
            L["vn"].copy_(hv[j], non_blocking=True)
            qk, qv = L["cache"].update_and_fetch_quantized(L["kn"], L["vn"])
            kvq.sdpa_decode(L["q"], qk, qv, scale, out=L["out"])
            L["cache"].trim(1)
            ho[j].copy_(L["out"], non_blocking=True)
        f1.record()
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())

    # sanity: the benchmarked output is finite
    if not torch.isfinite(layers[0]["out"].float()).all():
        raise RuntimeError("non-finite decode output")

    sb = step_bytes(c)
    value = world * sb * K / (ms_max / 1e3) / 1e9
    e2e_value = world * sb * K2 / (e2e_ms / 1e3) / 1e9
    kmean = sum(kern_ms) / len(kern_ms)
    achieved = decode_launch_bytes(c) / (kmean / 1e3) / 1e9
    peak, peak_kind = peaks()
    res = None
    if rank == 0:
        res = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_max / K, 5),
            "us_per_step": round(1e3 * ms_max / K, 3),
            "tokens_per_s": round(world * c["B"] * K / (ms_max / 1e3), 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes/f16",
            "data": "synthetic (seeded torch.randn; keys with 4 outlier channels x8)",
            "config": {"workload": WORKLOAD, "B_per_gpu": c["B"], "Hq": c["Hq"], "Hkv": c["Hkv"],
                       "head_dim": c["D"], "context": c["N_prior"] + 1, "bits": c["bits"],
                       "group_size": c["gs"], "layers_cycled": NL,
                       "l2": f"inputs larger than L2: {NL} distinct layer caches, "
                             f"{NL * layer_bytes / 1e6:.0f} MB cycled",
                       "parallelism": f"shard by sequence, {world} GPU(s), no collective",
                       "timing": "CUDA graphs of NL steps, CUDA events, max over ranks"},
            "bytes_per_step": sb,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT,
                    "h2d_bytes_per_step": int(hq[0].numel() * 2 + hk[0].numel() * 2 + hv[0].numel() * 2),
                    "d2h_bytes_per_step": int(ho[0].numel() * 2),
                    "us_per_step": round(1e3 * e2e_ms / K2, 3), "steps": K2,
                    "path": "kvq Python API per step (eager), pinned host buffers"},
            "gpu_launches": 3 * K,  # per step: fused K/V append, attention, merge of partials
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind,
                         "kernel": "decode = attn_bal_kernel<4,128,64,1> + attn_bal_merge_kernel",
                         "kernel_us": round(kmean * 1e3, 3),
                         "bytes_per_launch": decode_launch_bytes(c),
                         "traffic": traffic_from_profiles(),
                         "timing": "CUDA events around decode-only graph replays of the same "
                                   "layers, right after the timed steps, same stream"},
            "clocks": clk,
        }
    return res


CFG4 = dict(B=1, Hq=32, Hkv=8, D=128, N_prior=16384, L=512, bits=8, gs=64, outliers=4)


def prefill_flops(c):
    """Causal chunk of L rows after N_prior keys: 4 * Hq * L * D * (N_prior + (L + 1) / 2)."""
    return 4 * c["Hq"] * c["L"] * c["D"] * (c["N_prior"] + (c["L"] + 1) / 2)


def run_prefill(args):
    """Config 4: chunked prefill of 512 query rows (causal in the chunk) over a
    kv8 cache of 16,384 prior rows plus the chunk, appended first.  One step =
    append of the 512 K/V rows + prefill attention; both timed with CUDA
    events over graph replays of NL distinct layers; the attention alone
    (the tensor-core kernel and the merge of units cut between its CTAs) is
    timed the same way for the tensor-core roofline."""
    import numpy as np
    import torch
    import kvq
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    c = CFG4
    B, Hq, Hkv, D, Np, L = c["B"], c["Hq"], c["Hkv"], c["D"], c["N_prior"], c["L"]
    scale = 1.0 / np.sqrt(D)
    NL = 4  # 4 x 36.8 MB of K/V: above L2 across a replay
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
    mask = None

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
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(stream)
        for _ in range(reps):
            g_step.replay()
        ev[1].record(stream)
        for _ in range(reps):
            g_att.replay()
        ev[2].record(stream)
        ev[2].synchronize()
    step_ms = ev[0].elapsed_time(ev[1]) / (reps * NL)
    att_ms = ev[1].elapsed_time(ev[2]) / (reps * NL)
    fl = prefill_flops(c)
    try:
        peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
        pk = "measured (bf16 dense burst; fp16 runs at the same rate)"
    except Exception:
        peak, pk = 1590.0, "fallback"
    att_tf = fl / (att_ms / 1e3) / 1e12
    print(json.dumps({
        "metric": "quantized-KV chunked prefill TFLOP/s (config 4: B1 Hq32 Hkv8 D128, 16384 prior + 512-row causal chunk, kv8 gs64)",
        "value": round(fl / (step_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": reps * NL, "warmup": args.warmup, "ms_per_step": round(step_ms, 5),
        "higher_is_better": True, "dtype": "u8 codes/f16", "data": "synthetic (seeded torch.randn)",
        "config": {"workload": "config4-kv8-prefill-append", "flops_per_step": fl,
                   "layers_cycled": NL, "l2": "4 distinct layers (147 MB of K/V) per replay"},
        "roofline": {"bound": "tensor", "achieved": round(att_tf, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(att_tf / peak, 4), "peak_kind": pk,
                     "kernel": "prefill_tc_kernel (tcgen05 UMMA, TMEM accumulators) + prefill_tc_merge_kernel",
                     "kernel_us": round(att_ms * 1e3, 3)},
        "gpu_launches": 3 * reps * NL}))


# ------------------------------------------------------ other configs --
#
# Secondary measurement lines for the other BASELINE configs (one JSON line
# each, not read by the driver): config 1 (one small decode step, many
# distinct layers so the working set exceeds L2), config 3 (Gemma-style
# rotating window: 5 window layers + 1 global layer per step, append and
# decode), config 5 (ragged batch of 64 sequences decoded with seq_lens, kv
# heads sharded over ranks with no communication) and config 5's single
# 131,072-token sequence split along the context (partials all-gathered over
# NCCL and merged).  Synthetic seeded data of the named shapes.

CONFIG_DESC = {
    "config1": "single decode step: B1 Hq16 Hkv4 D128 N2048 kv8 gs64, 64 distinct layers cycled",
    "config3": "Gemma-style window: B4 Hq8 Hkv4 D256 kv8 gs64; per step 5 rotating layers (window "
               "1024, 4096 tokens written) + 1 global layer (4096), append + decode each",
    "config5": "ragged serving: B64 lengths U[1024, 32768] (seed 5), Hq32 Hkv8 D128 kv4 gs64, "
               "decode with seq_lens; kv heads sharded over ranks, no collective",
    "config5-ctx": "one 131072-token sequence, Hq32 Hkv8 D128 kv4 gs64, context split over ranks; "
                   "(m, l, o) partials all-gathered over NCCL and merged",
}


def _fill_cache(cache, B, H, N, D, g, device, chunk):
    """Append N seeded rows (fp16) to `cache` in chunks; returns the last views."""
    import torch
    views = None
    for s0 in range(0, N, chunk):
        S = min(chunk, N - s0)
        k = torch.randn(B, H, S, D, generator=g, device=device).half()
        v = torch.randn(B, H, S, D, generator=g, device=device).half()
        views = cache.update_and_fetch_quantized(k, v)
        del k, v
    return views


def run_config(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    import kvq
    from kvq.parallel import ContextSplitDecode, context_ranges

    w = args.workload
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device)
    g.manual_seed(3000 + rank)
    steps, keep = [], []
    nbytes = 0  # algorithmic bytes of this rank per pass over `steps`
    dt = "u8 codes/f16"
    scaling = "weak"
    graph_ok = True
    if w == "config1":
        B, Hq, Hkv, D, N, bits, gs = 1, 16, 4, 128, 2048, 8, 64
        rb = 2 * (D * bits // 8 + 2 * (D // gs) * 2)
        scale = 1.0 / np.sqrt(D)
        for _ in range(64):
            cache = kvq.QuantizedKVCache(gs, bits)
            kq, vq = _fill_cache(cache, B, Hkv, N, D, g, device, N)
            q = torch.randn(B, Hq, 1, D, generator=g, device=device).half()
            out = torch.empty_like(q)
            keep.append((cache, kq, vq, q, out))
            steps.append(lambda kq=kq, vq=vq, q=q, out=out:
                         kvq.sdpa_decode(q, kq, vq, scale, out=out))
            nbytes += B * Hkv * N * rb + 2 * B * Hq * D * 2
    elif w == "config3":
        B, Hq, Hkv, D, bits, gs, win = 4, 8, 4, 256, 8, 64, 1024
        rb = 2 * (D * bits // 8 + 2 * (D // gs) * 2)
        scale = 1.0 / 16.0
        for _ in range(3):  # 3 x (5 + 1) layers: 241 MB cycled, above L2
            for li in range(6):
                local = li < 5
                cache = kvq.RotatingQuantizedKVCache(win, gs, bits) if local else \
                    kvq.QuantizedKVCache(gs, bits, reserve_rows=4352)
                _fill_cache(cache, B, Hkv, 4096, D, g, device, win)
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
    elif w == "config5":
        B, Hq, Hkv, D, bits, gs = 64, 32, 8, 128, 4, 64
        if Hkv % world:
            raise SystemExit("config5 shards 8 kv heads: use 1, 2, 4 or 8 GPUs")
        rb = 2 * (D * bits // 8 + 2 * (D // gs) * 2)
        scale = 1.0 / np.sqrt(D)
        lens = np.random.default_rng(5).integers(1024, 32769, size=B)
        hk = Hkv // world
        Nmax = int(lens.max())
        cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=(Nmax + 255) // 256 * 256)
        kq, vq = _fill_cache(cache, B, hk, Nmax, D, g, device, 1024)
        q = torch.randn(B, hk * (Hq // Hkv), 1, D, generator=g, device=device).half()
        out = torch.empty_like(q)
        sl = torch.tensor(lens, dtype=torch.int32, device=device)
        keep.append((cache, kq, vq, q, out, sl))
        steps.append(lambda: kvq.sdpa_decode(q, kq, vq, scale, seq_lens=sl, out=out))
        nbytes = int(lens.sum()) * hk * rb + 2 * B * hk * (Hq // Hkv) * D * 2
        dt = "u4 codes/f16"
        scaling = "strong"
    elif w == "config5-ctx":
        Hq, Hkv, D, bits, gs, N = 32, 8, 128, 4, 64, 131072
        rb = 2 * (D * bits // 8 + 2 * (D // gs) * 2)
        scale = 1.0 / np.sqrt(D)
        a, b = context_ranges(N, world)[rank]
        cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=(b - a + 255) // 256 * 256)
        kq, vq = _fill_cache(cache, 1, Hkv, b - a, D, g, device, 4096)
        gq = torch.Generator(device=device)
        gq.manual_seed(77)  # the same query on every rank
        q = torch.randn(1, Hq, 1, D, generator=gq, device=device).half()
        out = torch.empty_like(q)
        keep.append((cache, kq, vq, q, out))
        if world > 1:
            split = ContextSplitDecode()
            steps.append(lambda: out.copy_(split.step(q, kq, vq, scale)))
            graph_ok = False  # the all-gather runs eagerly
        else:
            steps.append(lambda: kvq.sdpa_decode(q, kq, vq, scale, out=out))
        nbytes = (b - a) * Hkv * rb + 2 * Hq * D * 2
        dt = "u4 codes/f16"
        scaling = "strong"
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            for s in steps:
                s()
    stream.synchronize()
    graph = None
    if graph_ok:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for s in steps:
                s()
        for _ in range(3):
            graph.replay()
    torch.cuda.synchronize()
    reps = max(1, (args.steps + len(steps) - 1) // len(steps))
    clocks = Clocks(local_rank) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.start()
        time.sleep(0.1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        for _ in range(reps):
            if graph is not None:
                graph.replay()
            else:
                for s in steps:
                    s()
        e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    t = torch.tensor([e0.elapsed_time(e1), float(nbytes)], device=device, dtype=torch.float64)
    if world > 1:
        tt = t.clone()
        dist.all_reduce(t[0:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tt[1:2], op=dist.ReduceOp.SUM)
        t[1] = tt[1]
    ms, total_bytes = float(t[0].item()), float(t[1].item())
    if not torch.isfinite(keep[0][-2 if w == "config5" else -1].float()).all():
        raise RuntimeError("non-finite decode output")
    if rank != 0:
        return None
    K = reps * len(steps)
    gbs = total_bytes * reps / (ms / 1e3) / 1e9
    per_gpu = gbs / world
    peak, peak_kind = peaks()
    return {
        "metric": f"quantized-KV decode SDPA achieved HBM GB/s ({w})", "value": round(gbs, 1),
        "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": round(ms / K, 5), "us_per_step": round(1e3 * ms / K, 3),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": dt,
        "data": "synthetic (seeded torch.randn / numpy lengths)",
        "config": {"workload": w, "description": CONFIG_DESC[w],
                   "bytes_per_pass_all_ranks": int(total_bytes), "steps_per_pass": len(steps),
                   "timing": ("CUDA graph of one pass" if graph is not None else
                              "eager steps (NCCL all-gather inside)") +
                             ", CUDA events, max over ranks"},
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu / peak, 4), "peak_kind": peak_kind,
                     "note": "whole step per GPU (append included where the config appends)"},
        "clocks": clk,
    }


def profile_run(args):
    """Fixed small workload for ncu: 3 config-2 layers (227 MB, above L2),
    `--steps` launches of one kernel, cycling layers."""
    import numpy as np
    import torch
    import kvq
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    layers = setup_layers(CFG, 3, device, seed=7)
    scale = 1.0 / np.sqrt(CFG["D"])
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="kvq", choices=["kvq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["decode", "prefill", "config1", "config3", "config5",
                                           "config5-ctx"], default="decode",
                    help="decode: the config-2 step the driver reads (default); prefill: "
                         "config 4 chunked prefill; config1/3/5/5-ctx: the other BASELINE "
                         "configs (separate JSON lines)")
    ap.add_argument("--profile", choices=["decode", "append"], default=None,
                    help="run only the named kernel over 3 config-2 layers, `--steps` "
                         "launches, no timing (a small, fixed workload for ncu captures)")
    args = ap.parse_args()
    if args.profile:
        return profile_run(args)
    if args.workload == "prefill":
        return run_prefill(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        K = max(1, args.steps)
        budget = 60.0
        gbs, threads, desc, el = cpu_oracle_sample(K, budget)
        line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": UNIT,
                "n_gpus": args.gpus, "steps": K, "warmup": args.warmup,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "u4 codes/f16", "data": "synthetic (seeded numpy)",
                "config": {"workload": WORKLOAD},
                "cpu_baseline": {"value": round(gbs, 4), "unit": UNIT, "cores": threads,
                                 "kind": "port", "sample": desc},
                "e2e": {"value": round(gbs, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "note": "mlx-bun's own CPU path (MLX CPU stream under Bun) cannot run on "
                        "this box; the C restatement of its op graph is timed instead"}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.workload in CONFIG_DESC:
        try:
            res = run_config(args, rank, world, local_rank)
            if rank == 0:
                print(json.dumps(res))
        finally:
            if world > 1:
                dist.destroy_process_group()
        return
    try:
        res = run_gpu(args, rank, world, local_rank)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                gbs, threads, desc, el = cpu_oracle_sample(4, 12.0)
                res["cpu_baseline"] = {"value": round(gbs, 4), "unit": UNIT, "cores": threads,
                                       "kind": "port", "sample": desc}
            print(json.dumps(res))
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
