#!/usr/bin/env python
"""Benchmark of the packed decode-attention hot path (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1|2|4] [--impl b200|reference]

A *step* is one decode step of attention for every layer of the model over a
batch of sequences: for each of the L layers, K2 (split-K GQA decode over the
packed history, residual page and new token) and K3 (split merge).  This is
the metric the reference's ``packed`` backend would be measured on
(``scripts/evaluate.py:1-6``): decode tokens/s = batch / step time, plus the
HBM bandwidth it implies over the algorithmic bytes of the packed layout.

Workload (default): Qwen2-7B geometry, 28 layers, 28 q /
4 KV heads, head_dim 128, batch 16 per GPU, 8192-token packed history plus a
seeded U{0..127}-token bf16 residual per sequence, synthetic K/V with 5 %
outlier Key channels, seeded policy at target_bit 2.5 (Key mean 3.0 bit).
Per-GPU work is fixed as N grows (``scaling: weak``): every rank holds its own
16 sequences, no collective on the data path.

Timing: W untimed warm-up steps, then K timed steps replayed from a CUDA graph
of the L per-layer K2+K3 launches, bracketed by barrier + synchronize, timed
with CUDA events on the launching stream, max over ranks.  The step's working
set (~1.5 GB) is far larger than the 126 MB L2, so no flush is needed.
``--impl reference`` times the reference algorithm on the host CPU instead
(the numpy restatement in ``oracle/``; the reference itself is Python and
cannot travel to the GPU box), on all host cores, one bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "packed decode-attn tok/s & HBM GB/s (% of peak) at 8k/32k ctx, 1–8 GPUs"
CONFIGS = {
    1: dict(name="config1", layers=28, batch=16, n_q=28, n_kv=4, head_dim=128, history=8192,
            target_bit=2.5, seed=1),
    2: dict(name="config2", layers=28, batch=8, n_q=28, n_kv=4, head_dim=128, history=32768,
            target_bit=3.0, seed=2),
    4: dict(name="config4", layers=64, batch=64, n_q=40, n_kv=8, head_dim=128, history=16384,
            target_bit=2.5, seed=4),
}
FALLBACK_HBM_GBS = 6650.0


def measured_peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(config_id: int):
    """DRAM bytes (read + write) of one K2 launch for this config, from the
    committed ncu capture summary (profiles/k2_decode_traffic.txt), or None."""
    try:
        for line in (ROOT / "profiles" / "k2_decode_traffic.txt").read_text().splitlines():
            parts = line.split()
            if len(parts) == 2 and parts[0] == f"config{config_id}":
                return int(parts[1])
    except (OSError, ValueError):
        return None
    return None


def max_over_ranks(value: float, device) -> float:
    """Max of a per-rank time over the default process group (the value
    itself without one): every multi-GPU time is the slowest rank's."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def tails_for(cfg: dict, rank: int):
    import numpy as np

    rng = np.random.default_rng([cfg["seed"], 31337, rank])
    return rng.integers(0, 128, size=cfg["batch"]).tolist()


# ----------------------------------------------------------- byte model ----
def algorithmic_bytes(widths_words, hist_tokens, tails, n_q, n_kv, head_dim, page=128,
                      q_bytes=2, out_bytes=2, resid_bytes=2):
    """Bytes one decode step must move for one layer, in the reference layout
    (payload + scale/min + padding to the tier width + residual + q/out).

    ``widths_words`` = (w2, w4, w8, w16, words2, words4, words8) of the layer.
    Returns (k2_bytes, total_bytes)."""
    w2, w4, w8, w16, n2, n4, n8 = widths_words
    gq = n_q // n_kv
    k2 = 0
    for t_hist, tail in zip(hist_tokens, tails):
        groups = t_hist // page
        per_head = (t_hist * 4 * (n2 + n4 + n8)              # K codes
                    + groups * 2 * 2 * (w2 + w4 + w8)         # K scale/min
                    + t_hist * 2 * w16                        # FP16 Key tier
                    + t_hist * 4 * (head_dim * 2 // 32)       # V codes
                    + t_hist * 2 * 2                          # V scale/min
                    + (tail + 1) * head_dim * resid_bytes * 2  # residual K/V + new token
                    + gq * head_dim * q_bytes)                # query group
        k2 += per_head * n_kv
    out = len(hist_tokens) * n_q * head_dim * out_bytes
    return k2, k2 + out


# ------------------------------------------------------------- clocks -------
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = ROOT / "gpurun_out" / f"clocks_gpu{index}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        import statistics

        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        under_load = [x for x in sm if smax and x > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(under_load) if under_load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU legs ------
def _cpu_sample_worker(args):
    """Time the reference algorithm (oracle port) on one (sequence, layer) of the workload."""
    cfg, layer, tail, budget_s = args
    import numpy as np

    from oracle import packed_ref as orc
    from logitfill_b200.synthetic import synthetic_kv, synthetic_levels

    D, H = cfg["head_dim"], cfg["n_kv"]
    levels = synthetic_levels(cfg["layers"], H, D, cfg["target_bit"], seed=cfg["seed"])[layer]
    n = cfg["history"] + tail
    k, v = synthetic_kv(1, H, n + 1, D, seed=cfg["seed"], layer=layer, device="cpu")
    k, v = k[0].float().numpy(), v[0].float().numpy()
    store = orc.OracleLayer(levels, 128, 128, 128, 2)
    store.append(k[:, :n], v[:, :n])
    rng = np.random.default_rng(layer)
    q = rng.standard_normal((cfg["n_q"], 1, D)).astype(np.float32)
    from threadpoolctl import threadpool_limits

    threadpool_limits(1)  # one core per worker: `cores` counts workers
    orc.reference_attention(store, q, k[:, n:n + 1], v[:, n:n + 1], D ** -0.5)  # untimed first touch
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        orc.reference_attention(store, q, k[:, n:n + 1], v[:, n:n + 1], D ** -0.5)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    return times


def cpu_decode_rate(cfg: dict, budget_s: float, workers: int) -> dict:
    """Decode tok/s of the reference algorithm on the host: one (seq, layer)
    attention call takes t seconds, a step needs batch x layers of them."""
    import multiprocessing as mp

    tails = tails_for(cfg, 0)
    jobs = [(cfg, (i * 7) % cfg["layers"], tails[i % len(tails)], budget_s) for i in range(workers)]
    if workers == 1:
        results = [_cpu_sample_worker(jobs[0])]
    else:
        with mp.get_context("spawn").Pool(workers) as pool:
            results = pool.map(_cpu_sample_worker, jobs)
    calls = sum(len(r) for r in results)
    per_call = sum(sum(r) for r in results) / calls
    # `workers` calls run concurrently: throughput = workers / per_call (seq, layer) calls/s.
    calls_per_s = workers / per_call
    tok_s = calls_per_s / cfg["layers"]   # one token per sequence needs `layers` calls
    return {"value": tok_s, "unit": "tok/s", "cores": workers, "calls": calls,
            "sec_per_call": per_call,
            "sample": f"{calls} reference_attention calls (oracle port) on (seq, layer) samples of "
                      f"{cfg['name']} ({cfg['history']}-token packed history + bf16 tail), "
                      f"{workers} process(es), extrapolated to tok/s = {workers}/(t_call x {cfg['layers']} layers)"}


def run_reference(args, cfg) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    workers = max(1, os.cpu_count() or 1)
    budget = max(1.0, min(20.0, 60.0 / max(1, args.steps + args.warmup)))
    values = []
    for i in range(args.warmup + args.steps):
        res = cpu_decode_rate(cfg, budget, workers)
        if i >= args.warmup:
            values.append(res)
    tok_s = sum(r["value"] for r in values) / len(values)
    ms = cfg["batch"] / tok_s * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(cfg, args.gpus),
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": workers, "kind": "port",
                         "sample": values[-1]["sample"]},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_k1(cache, k, v, T: int, dev) -> dict:
    """K1 (page quantize + pack) on layer 0's prefill: every full page of every
    sequence re-packed into the slot it already occupies (the output bytes do
    not change).  Algorithmic bytes: the pages' Key and Value in their dtype
    plus the packed rows and meta rows written."""
    import ctypes

    import numpy as np
    import torch

    from logitfill_b200 import _lib
    from logitfill_b200.packed.layout import pack_pages

    layer, P = cache.layers[0], cache.page_size
    pages = T // P
    jobs = [(b, p * P, b, p) for b in range(cache.batch) for p in range(pages)]
    lay = layer.layout
    moved = len(jobs) * cache.n_kv * (2 * P * cache.head_dim * k.element_size()
                                      + P * lay.row_words * 4 + lay.meta_halves * 2)
    pack_pages(lay, layer.rows, layer.kmeta, k, v, jobs)  # validates the jobs once
    jobs_dev = torch.tensor(jobs, dtype=torch.int32, device=dev)
    so = _lib.lib()

    def launch():  # the kernel alone: jobs already on the device
        _lib.check(so.lf_pack_pages(
            ctypes.byref(lay.c), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(k.dtype), k.stride(0), k.stride(1),
            k.stride(2), _lib.ptr(jobs_dev), len(jobs), cache.batch, _lib.ptr(lay.chan_code), _lib.ptr(layer.rows),
            _lib.ptr(layer.kmeta), _lib.ptr(cache.status), _lib.stream_handle(dev)), "lf_pack_pages")

    launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    cache.check_status()
    ms = float(np.median(times))
    return {"kernel": "lf_pack_pages (K1)", "bound": "hbm", "unit": "GB/s", "pages_per_launch": len(jobs) * cache.n_kv,
            "bytes_per_launch": moved, "avg_launch_ms": ms, "achieved": moved / (ms * 1e-3) / 1e9}


def workload_config(cfg: dict, n_gpus: int) -> dict:
    return {
        "workload": f"{cfg['name']}: {cfg['layers']} layers, {cfg['n_q']} q / {cfg['n_kv']} kv heads, "
                    f"head_dim {cfg['head_dim']}, batch {cfg['batch']} per GPU, {cfg['history']}-token packed "
                    f"history + U{{0..127}} bf16 residual + 1 new token, target_bit {cfg['target_bit']}",
        "layers": cfg["layers"], "batch_per_gpu": cfg["batch"], "global_batch": cfg["batch"] * n_gpus,
        "history_tokens": cfg["history"], "n_q": cfg["n_q"], "n_kv": cfg["n_kv"], "head_dim": cfg["head_dim"],
        "page_size": 128, "target_bit": cfg["target_bit"], "bit_v": 2,
        "l2": "no flush: per-step working set > 126 MB L2",
        "parallelism": f"dp{n_gpus} (sequences sharded, no collective)",
    }


# ------------------------------------------------------------- GPU leg ------
def run_b200(args, cfg) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from logitfill_b200.packed import PackedKVCache
    from logitfill_b200.packed.attention import DecodeCall
    from logitfill_b200.synthetic import mean_key_bits, synthetic_kv, synthetic_levels

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    L, B, NQ, H, D = cfg["layers"], cfg["batch"], cfg["n_q"], cfg["n_kv"], cfg["head_dim"]
    T = cfg["history"]
    levels = synthetic_levels(L, H, D, cfg["target_bit"], seed=cfg["seed"])
    tails = tails_for(cfg, rank)
    lengths = [T + t for t in tails]
    cache = PackedKVCache(list(levels), B, NQ, H, D, device=dev, capacity=T + 128)
    for layer in range(L):
        k, v = synthetic_kv(B, H, T + 128, D, seed=cfg["seed"] * 1000 + rank, layer=layer, device=dev)
        cache.prefill(layer, k, v, lengths)
        if layer == 0:
            k1_src = (k, v)  # kept for the K1 timing below
        del k, v
    torch.cuda.synchronize()
    k1 = time_k1(cache, *k1_src, T, dev)
    del k1_src
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    q = torch.randn(L, B, NQ, D, generator=gen, device=dev).to(torch.bfloat16)
    kn = torch.randn(L, B, H, D, generator=gen, device=dev).to(torch.bfloat16)
    vn = torch.randn(L, B, H, D, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty(L, B, NQ, D, device=dev, dtype=torch.bfloat16)
    scaling = D ** -0.5
    calls = [DecodeCall(cache, l, q[l], kn[l], vn[l], scaling, out[l], pps=args.pps) for l in range(L)]

    def step():
        for c in calls:
            c.launch()

    # Warm-up (also configures kernels before capture).
    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, dev)

    # K2 launch durations over the same kind of timed steps (eager launches, events per K2).
    k2_ms = []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    for _ in range(args.steps):
        for (a, b), c in zip(ev, calls):
            a.record(stream)
            c.launch_partial()
            b.record(stream)
            c.launch_merge()
        torch.cuda.synchronize()
        k2_ms.extend(a.elapsed_time(b) for a, b in ev)
    k2_avg_ms = max_over_ranks(sum(k2_ms) / len(k2_ms), dev)

    # End to end: every step uploads its inputs from pinned host memory and reads
    # its outputs back.  Two device buffer sets (and a graph bound to each) let
    # step i+1's upload and step i's read-back run on a copy stream while the
    # GPU computes; every copy is inside the timed region.
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, kn, vn))
    q2, kn2, vn2, out2 = (torch.empty_like(x) for x in (q, kn, vn, out))
    calls2 = [DecodeCall(cache, l, q2[l], kn2[l], vn2[l], scaling, out2[l], pps=args.pps) for l in range(L)]
    graph2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph2, capture_error_mode="thread_local"):
        for c in calls2:
            c.launch()
    sets = [(q, kn, vn, out, graph), (q2, kn2, vn2, out2, graph2)]
    houts = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    cs = torch.cuda.Stream(dev)
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        b = i % 2
        with torch.cuda.stream(cs):
            if i >= 2:
                cs.wait_event(computed[b])  # the step that last read this set has finished
            for dst, src in zip(sets[b][:3], (hq, hk, hv)):
                dst.copy_(src, non_blocking=True)
            uploaded[b].record(cs)

    for i in range(2):  # one untimed pass over both sets
        upload(i)
        stream.wait_event(uploaded[i])
        sets[i][4].replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    upload(0)
    for i in range(args.steps):
        b = i % 2
        stream.wait_event(uploaded[b])
        sets[b][4].replay()
        computed[b].record(stream)
        if i + 1 < args.steps:
            upload(i + 1)
        with torch.cuda.stream(cs):
            cs.wait_event(computed[b])
            houts[b].copy_(sets[b][3], non_blocking=True)
    read_back = torch.cuda.Event()
    read_back.record(cs)
    stream.wait_event(read_back)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
    d2h = houts[0].numel() * houts[0].element_size()
    assert torch.equal(houts[(args.steps - 1) % 2], out.cpu() if (args.steps - 1) % 2 == 0 else out2.cpu())

    # Algorithmic bytes (reference layout) per step and per K2 launch.
    k2_bytes = []
    step_bytes = 0
    for layer in cache.layers:
        c = layer.layout.c
        ww = (c.width[0], c.width[1], c.width[2], c.width[3], c.words[0], c.words[1], c.words[2])
        kb, tb = algorithmic_bytes(ww, layer.hist_len.tolist(), layer.tail_len.tolist(), NQ, H, D)
        k2_bytes.append(kb)
        step_bytes += tb
    k2_bytes_avg = sum(k2_bytes) / len(k2_bytes)
    peak, peak_kind = measured_peak_hbm()
    achieved = k2_bytes_avg / (k2_avg_ms * 1e-3) / 1e9
    step_gbs = step_bytes / (ms * 1e-3) / 1e9

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu_res = cpu_decode_rate(cfg, budget_s=10.0, workers=1)
            cpu = {"value": cpu_res["value"], "unit": "tok/s", "cores": 1, "kind": "port",
                   "sample": cpu_res["sample"]}
        line = {
            "metric": METRIC, "value": world * B / (ms_max * 1e-3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(cfg, world),
            "hbm_gbs": step_gbs * world, "hbm_frac_of_peak_per_gpu": step_gbs / peak,
            "key_mean_bits": mean_key_bits(levels),
            "pages_per_split": calls[0].pps,
            "roofline": {"kernel": "lf_decode_partial (K2)", "bound": "hbm", "achieved": achieved,
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": ncu_traffic(args.config) if args.target_bit is None else None,
                         "traffic_source": f"ncu --set full, profiles/k2_decode_config{args.config}_ncu.md",
                         "bytes_per_launch": k2_bytes_avg, "avg_launch_ms": k2_avg_ms},
            "k1": dict(k1, peak=peak, frac=k1["achieved"] / peak),
            "e2e": {"value": world * B / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * L * 2,
        }
        print(json.dumps(line), flush=True)
    del graph, graph2
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_model_decode(args) -> None:
    """Model-level decode loop (a DeepSeek-R1-Distill-Qwen-7B-shaped Qwen2 with
    random weights, batch 1): prefill ``--context`` tokens through the adapter,
    then time greedy decode steps eagerly (the reference's sampling loop,
    benchmarks/generate.py:28-57) and replayed from a CUDA graph
    (GraphDecoder).  Prints one JSON line; not the driver's bench line."""
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from logitfill_b200.adapter import DeepSeekQwenKVAdapter
    from logitfill_b200.graph_decode import GraphDecoder
    from logitfill_b200.synthetic import synthetic_levels

    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                      num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=32768,
                      rope_theta=10000.0, attention_dropout=0.0)
    cfg._attn_implementation = "sdpa"
    with torch.device("cuda"):
        model = Qwen2ForCausalLM(cfg).to(torch.bfloat16).eval()
    levels = list(synthetic_levels(28, 4, 128, 2.5, seed=1))
    ctx, n = args.context, args.steps
    prompt = torch.randint(0, cfg.vocab_size, (1, ctx), generator=torch.Generator().manual_seed(1)).cuda()
    adapter = DeepSeekQwenKVAdapter(model).attach()
    adapter.set_k_levels(levels)

    def timed(fn, count):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(count):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / count

    # Eager loop (the adapter on every layer, host-side commits).
    cache = adapter.make_cache()
    cache.reset()
    state = {}
    with torch.inference_mode():
        out = model(input_ids=prompt, use_cache=True, past_key_values=cache)
        state["tok"] = out.logits[:, -1].argmax(-1, keepdim=True)

        def eager():
            o = model(input_ids=state["tok"], use_cache=True, past_key_values=cache)
            state["tok"] = o.logits[:, -1].argmax(-1, keepdim=True)

        for _ in range(args.warmup):
            eager()
        eager_ms = timed(eager, n)
    # Graph loop.
    adapter.set_k_levels(levels)
    g = GraphDecoder(model, adapter, max_tokens=ctx + args.warmup + n + 8)
    with torch.inference_mode():
        state["tok"] = g.prefill(prompt).argmax(-1, keepdim=True)

        def graphed():
            state["tok"] = g.step(state["tok"]).argmax(-1, keepdim=True)

        for _ in range(args.warmup):
            graphed()
        graph_ms = timed(graphed, n)
    g.release()
    print(json.dumps({
        "mode": "model_decode", "model": "Qwen2, DeepSeek-R1-Distill-Qwen-7B shape, random bf16 weights",
        "batch": 1, "context": ctx, "steps": n, "warmup": args.warmup, "policy_target_bit": 2.5,
        "eager_ms_per_token": eager_ms, "graph_ms_per_token": graph_ms, "speedup": eager_ms / graph_ms,
        "data": "synthetic"}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--target-bit", type=float, default=None,
                    help="override the config's Key policy budget (config 2 sweep: 2.25, 2.5, 3.0, 4.0)")
    ap.add_argument("--pps", type=int, default=None,
                    help="pages per K2 work item (default: the occupancy-aware planner)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the config's sequences per GPU (small cases for profiling)")
    ap.add_argument("--model-decode", action="store_true",
                    help="time the model-level decode loop, eager vs CUDA graph (not the driver's bench line)")
    ap.add_argument("--context", type=int, default=8192, help="prompt length for --model-decode")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.target_bit is not None:
        cfg["target_bit"] = args.target_bit
    if args.batch is not None:
        cfg["batch"] = args.batch
    if args.model_decode:
        run_model_decode(args)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
