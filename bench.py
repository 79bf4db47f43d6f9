#!/usr/bin/env python
"""Benchmark of the packed decode-attention hot path (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1|2|4]
                    [--shard weak|batch|kv] [--k2 auto|tc|simt] [--impl b200|reference]

A *step* is one decode step of attention for every layer of the model over a
batch of sequences: for each of the L layers, K2 (split-K GQA decode over the
packed history, residual page and new token) and K3 (split merge).  This is
the metric the reference's ``packed`` backend would be measured on
(``scripts/evaluate.py:1-6``): decode tokens/s = batch / step time, plus the
HBM bandwidth it implies over the algorithmic bytes of the packed layout.

Main line (default): Qwen2-7B geometry, 28 layers, 28 q /
4 KV heads, head_dim 128, batch 16 per GPU, 8192-token packed history plus a
seeded U{0..127}-token bf16 residual per sequence, synthetic K/V with 5 %
outlier Key channels, seeded policy at target_bit 2.5 (Key mean 3.0 bit).
Per-GPU work is fixed as N grows (``scaling: weak``): every rank holds its own
16 sequences, no collective on the data path.  The line also carries:

* ``config2`` (N = 1): config 2, 32768-token histories, batch 8, target_bit 3.0
  (the north star's >= 70 % HBM target is stated there), with its own
  ``ms_per_step``, ``roofline`` and ``e2e``;
* ``config1_chunk16`` (N = 1): config 1's cache with a 16-token query chunk per
  sequence (chunked prefill / scoring through ``lf_decode_multi``);
* ``config3`` (N = 1): config 3, the page compression path: the 28-layer
  prefill of a 4096-token prompt per sequence (batch 16) packed through the
  public API and, separately, its K1 launches alone (HBM roofline fraction);
  then 256 decode steps, each one CUDA-graph replay of every layer's attention
  and device-side token commit, with a page flush every 128 tokens;
* ``config4_kv``: config 4 (64 layers, 40 q / 8 KV heads, batch 64, 16384-token
  histories, target_bit 2.5) sharded by KV head over the N ranks (strong
  scaling: the total work is fixed).  Each layer's split merge stores the
  rank's output heads into every rank's gathered buffer over NVLink and
  signals it; a bounded wait per layer completes the gather, inside the timed
  step;
* ``config4_kv_nccl`` (N > 1): the same with each layer's output gathered by
  an NCCL all-gather instead of the fused merge-gather (the collective
  baseline);
* ``config4_batch`` (N > 1): config 4 sharded by sequence (strong, no collective).

Timing: W untimed warm-up steps, then K timed steps replayed from a CUDA graph
of the per-layer launches, bracketed by barrier + synchronize, timed with CUDA
events on the launching stream, max over ranks.  Every step's working set
(>= 1.5 GB) is far larger than the 126 MB L2, so no flush is needed.  K2's
average launch duration comes from a second CUDA graph holding only the L K2
launches (same programmatic launches, K3 left out), event-timed and divided
by L, so it always fits inside the step.  ``e2e`` repeats the step through
the public API with every step's query / new K/V uploaded from pinned host
memory and the outputs read back, the copies inside the timed region and
overlapped with the previous step's attention (a pipelined attention-only
loop, not a model step).  ``cpu_baseline`` times the reference's algorithm on
the host cores: a torch restatement of its dense packed path and the numpy
oracle, one process per core (``oracle/``; the reference itself is Python and
does not exist on the GPU box).  ``--impl reference`` times the torch
restatement alone, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
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
    """nvidia-smi clock / throttle-reason samples during the timed region
    (written to a temporary file, read back by ``summary``)."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"lf_bench_clocks_gpu{index}_{os.getpid()}.csv"

    def __enter__(self):
        try:
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
        try:
            self.path.unlink()
        except OSError:
            pass
        under_load = [x for x in sm if smax and x > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(under_load) if under_load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU legs ------
def host_cores() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def _cpu_sample_worker(args):
    """Time the reference algorithm on one (sequence, layer) of the workload:
    ``kind`` "torch" (restatement of the reference's torch path) or "numpy"
    (the oracle).  One core per worker."""
    cfg, layer, tail, budget_s, kind, n_steps = args
    import numpy as np
    import torch

    torch.set_num_threads(1)
    from threadpoolctl import threadpool_limits

    threadpool_limits(1)
    from logitfill_b200.synthetic import synthetic_kv, synthetic_levels
    from oracle import packed_ref as orc
    from oracle import packed_ref_torch as orct

    D, H = cfg["head_dim"], cfg["n_kv"]
    levels = synthetic_levels(cfg["layers"], H, D, cfg["target_bit"], seed=cfg["seed"])[layer]
    n = cfg["history"] + tail
    k, v = synthetic_kv(1, H, n + 1, D, seed=cfg["seed"], layer=layer, device="cpu")
    k, v = k[0].float().numpy(), v[0].float().numpy()
    store = orc.OracleLayer(levels, 128, 128, 128, 2)
    store.append(k[:, :n], v[:, :n])
    rng = np.random.default_rng(layer)
    q = rng.standard_normal((cfg["n_q"], 1, D)).astype(np.float32)
    fn = orct.reference_attention if kind == "torch" else orc.reference_attention
    args = (store, q, k[:, n:n + 1], v[:, n:n + 1], D ** -0.5)
    fn(*args)  # untimed first touch
    per_step = []
    for _ in range(n_steps):
        times = []
        t_end = time.perf_counter() + budget_s
        while True:
            t0 = time.perf_counter()
            fn(*args)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() > t_end:
                break
        per_step.append(times)
    return per_step


def cpu_decode_rates(cfg: dict, budget_s: float, workers: int, kind: str, n_steps: int = 1) -> list[dict]:
    """Decode tok/s of the reference algorithm on the host, per step: every
    worker process (one core each) times its own (sequence, layer) attention
    calls for ``budget_s``; the host completes ``workers / t_call`` calls per
    second and one token per sequence needs ``layers`` of them."""
    import multiprocessing as mp

    tails = tails_for(cfg, 0)
    jobs = [(cfg, (i * 7) % cfg["layers"], tails[i % len(tails)], budget_s, kind, n_steps) for i in range(workers)]
    with mp.get_context("spawn").Pool(workers) as pool:
        results = pool.map(_cpu_sample_worker, jobs)
    label = {"torch": "torch restatement of reference.py:30-56", "numpy": "numpy oracle"}[kind]
    out = []
    for s in range(n_steps):
        calls = sum(len(r[s]) for r in results)
        per_call = sum(sum(r[s]) for r in results) / calls
        tok_s = workers / per_call / cfg["layers"]
        out.append({"value": tok_s, "unit": "tok/s", "cores": workers, "kind": "port", "calls": calls,
                    "sec_per_call": per_call,
                    "sample": f"{calls} reference_attention calls ({label}) on {workers} (sequence, layer) samples "
                              f"of {cfg['name']} ({cfg['history']}-token packed history + bf16 tail), one process "
                              f"per core for {budget_s:.0f} s; tok/s = {workers} / (t_call x {cfg['layers']} layers)"})
    return out


def run_reference(args, cfg) -> None:
    """The reference's algorithm on the host CPU (rank 0 only): the torch
    restatement of its dense packed path, one process per core."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    workers = host_cores()
    n = args.warmup + args.steps
    budget = max(1.0, min(10.0, 120.0 / n))
    rates = cpu_decode_rates(cfg, budget, workers, "torch", n_steps=n)[args.warmup:]
    tok_s = sum(r["value"] for r in rates) / len(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": cfg["batch"] / tok_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(cfg, args.gpus, "weak"),
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": workers, "kind": "port",
                         "sample": rates[-1]["sample"] + f"; {args.steps} timed steps after {args.warmup} warm-up"},
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


CONFIG3 = dict(name="config3", layers=28, batch=16, n_q=28, n_kv=4, head_dim=128, prompt=4096, decode_steps=256,
               target_bit=2.5, seed=3)


def run_config3(steps: int, warmup: int, dev, peak: float) -> dict:
    """BASELINE config 3, the page compression path, on one GPU.

    * prefill: every layer's 4096-token bf16 prompt of all 16 sequences packed
      into 32 pages per sequence and KV head through ``PackedKVCache.commit``
      (host job lists, one K1 launch per layer), inputs resident in HBM;
      ``steps`` timed repetitions, each from an empty cache, median kept;
    * prefill_k1: the same 28 K1 launches alone (jobs already on the device):
      the kernel's HBM roofline fraction;
    * decode: 256 decode steps after a fresh prefill, each step a CUDA-graph
      replay of the 28 layers' attention (K2 + K3) and ``lf_commit_token``
      (append to the residual page, pack it when it fills), so every sequence
      flushes a page at steps 128 and 256 inside the timed region."""
    import ctypes

    import numpy as np
    import torch

    from logitfill_b200 import _lib
    from logitfill_b200.packed import PackedKVCache
    from logitfill_b200.packed.attention import DecodeCall
    from logitfill_b200.packed.layout import pack_pages
    from logitfill_b200.synthetic import mean_key_bits, synthetic_kv, synthetic_levels

    cfg = CONFIG3
    L, B, NQ, H, D, T = cfg["layers"], cfg["batch"], cfg["n_q"], cfg["n_kv"], cfg["head_dim"], cfg["prompt"]
    n_dec = cfg["decode_steps"]
    levels = list(synthetic_levels(L, H, D, cfg["target_bit"], seed=cfg["seed"]))
    cache = PackedKVCache(levels, B, NQ, H, D, device=dev, capacity=T + n_dec + 128)
    P = cache.page_size
    kv = [synthetic_kv(B, H, T, D, seed=cfg["seed"] * 1000, layer=l, device=dev) for l in range(L)]
    moved = 0
    for l in range(L):
        lay = cache.layers[l].layout
        moved += B * (T // P) * H * (2 * P * D * 2 + P * lay.row_words * 4 + lay.meta_halves * 2)

    def prefill():
        for l in range(L):
            cache.commit(l, kv[l][0], kv[l][1])

    def timed(fn, reps, before=None):
        out = []
        for _ in range(reps):
            if before is not None:
                before()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            out.append(a.elapsed_time(b))
        return float(np.median(out))

    reps = max(3, min(steps, 5))
    timed(prefill, warmup, before=cache.reset)
    cache.check_status()
    ms_prefill = timed(prefill, reps, before=cache.reset)
    cache.check_status()

    # The K1 launches alone: the same jobs, already on the device.
    so = _lib.lib()
    jobs = [(b, p * P, b, p) for b in range(B) for p in range(T // P)]
    jobs_dev = torch.tensor(jobs, dtype=torch.int32, device=dev)
    pack_pages(cache.layers[0].layout, cache.layers[0].rows, cache.layers[0].kmeta, kv[0][0], kv[0][1], jobs)

    def k1_all():
        for l in range(L):
            layer, (k, v) = cache.layers[l], kv[l]
            _lib.check(so.lf_pack_pages(
                ctypes.byref(layer.layout.c), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(k.dtype), k.stride(0),
                k.stride(1), k.stride(2), _lib.ptr(jobs_dev), len(jobs), B, _lib.ptr(layer.layout.chan_code),
                _lib.ptr(layer.rows), _lib.ptr(layer.kmeta), _lib.ptr(cache.status), _lib.stream_handle(dev)),
                "lf_pack_pages")

    timed(k1_all, warmup)
    ms_k1 = timed(k1_all, reps)
    cache.check_status()

    # Decode with page flushes.
    gen = torch.Generator(device=dev).manual_seed(4321)
    q = torch.randn(L, B, NQ, D, generator=gen, device=dev).to(torch.bfloat16)
    kn = torch.randn(L, B, H, D, generator=gen, device=dev).to(torch.bfloat16)
    vn = torch.randn(L, B, H, D, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    cache.reset()
    prefill()
    torch.cuda.synchronize()
    calls = [DecodeCall(cache, l, q[l], kn[l], vn[l], D ** -0.5, out[l]) for l in range(L)]

    def step():
        for l in range(L):
            calls[l].launch()
            cache.layers[l].commit_token_device(kn[l], vn[l])

    graph = _graph(step)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    cache.check_status()
    cache.reset()
    prefill()

    def decode():
        for _ in range(n_dec):
            graph.replay()

    ms_dec = timed(decode, 1)
    cache.check_status()
    lengths = int(cache.layers[0].dev_hist[0].item()) + int(cache.layers[-1].dev_tail[0].item())
    del graph
    return {
        "workload": f"config3: {L} layers, {NQ} q / {H} kv heads, head_dim {D}, batch {B}, bf16 prefill of a "
                    f"{T}-token prompt per sequence packed into {T // P} pages per layer, then {n_dec} decode steps "
                    f"with a page flush every {P} tokens, target_bit {cfg['target_bit']}",
        "key_mean_bits": mean_key_bits(levels),
        "prefill": {"tokens_per_s": B * T / (ms_prefill * 1e-3), "ms": ms_prefill, "bytes": moved,
                    "gbs": moved / (ms_prefill * 1e-3) / 1e9, "frac": moved / (ms_prefill * 1e-3) / 1e9 / peak,
                    "reps": reps,
                    "method": "PackedKVCache.commit for every layer (host job lists + one K1 launch per layer), "
                              "CUDA events, median"},
        "prefill_k1": {"kernel": "lf_pack_pages (K1)", "bound": "hbm", "launches": L, "ms": ms_k1,
                       "gbs": moved / (ms_k1 * 1e-3) / 1e9, "frac": moved / (ms_k1 * 1e-3) / 1e9 / peak,
                       "peak": peak, "unit": "GB/s"},
        "decode": {"value": B * n_dec / (ms_dec * 1e-3), "unit": "tok/s", "steps": n_dec,
                   "ms_per_step": ms_dec / n_dec, "flush_steps": n_dec // P, "final_length": lengths,
                   "method": "CUDA graph of one step (per layer K2 + K3, then lf_commit_token), replayed "
                             f"{n_dec} times after a fresh prefill, CUDA events"},
    }


def run_chunk(w, q_len: int, steps: int, warmup: int, peak: float) -> dict:
    """A chunk of ``q_len`` query tokens per sequence over ``w``'s cache (a
    chunked prefill or scoring step): every layer's ``lf_decode_multi`` (K2 over
    virtual heads = q-heads x query tokens, in chunks of 8 per CTA, then K3),
    replayed from a CUDA graph.  Each chunk reads the pages again, so the
    unique history bytes / time understates the bytes the kernels fetch."""
    import torch

    from logitfill_b200.packed.attention import DecodeCall

    gen = torch.Generator(device=w.dev).manual_seed(99)
    L, B, NQ, H, D = w.L, w.B, w.NQ, w.H, w.D
    q = torch.randn(L, B, NQ, q_len, D, generator=gen, device=w.dev).to(torch.bfloat16)
    kn = torch.randn(L, B, H, q_len, D, generator=gen, device=w.dev).to(torch.bfloat16)
    vn = torch.randn(L, B, H, q_len, D, generator=gen, device=w.dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    calls = [DecodeCall(w.cache, l, q[l], kn[l], vn[l], D ** -0.5, out[l]) for l in range(L)]
    for _ in range(warmup):
        for c in calls:
            c.launch()
    torch.cuda.synchronize()
    w.cache.check_status()
    g = _graph(lambda: [c.launch() for c in calls])
    for _ in range(warmup):
        g.replay()
    ms = _timed_replays(g, steps, torch.cuda.current_stream(), lambda: None)
    w.cache.check_status()
    del g
    kb, _ = w.bytes_per_step()
    chunks = -(-(NQ // H) * q_len // 8)
    return {"q_len": q_len, "value": B * q_len / (ms * 1e-3), "unit": "query tok/s", "ms_per_step": ms,
            "steps": steps, "virtual_head_chunks_per_kv_head": chunks,
            "unique_history_gbs": kb * L / (ms * 1e-3) / 1e9,
            "unique_history_frac": kb * L / (ms * 1e-3) / 1e9 / peak,
            "method": "CUDA graph of the L lf_decode_multi calls (K2 + K3 each), CUDA events"}


def workload_config(cfg: dict, n_gpus: int, shard: str, kv_gather: str = "p2p") -> dict:
    per_gpu = cfg["batch"] if shard in ("weak", "kv") else cfg["batch"] // n_gpus
    par = {"weak": f"dp{n_gpus} (sequences sharded, {cfg['batch']} per GPU, no collective)",
           "batch": f"dp{n_gpus} ({cfg['batch']} sequences split over the GPUs, no collective)",
           "kv": f"kv{n_gpus} ({cfg['n_kv']} KV heads split over the GPUs; each layer's output gathered "
                 + ("by the split merge storing into every GPU's buffer over NVLink (lf_decode_merge_gather) "
                    "and a bounded wait per layer)" if kv_gather == "p2p" else "with an NCCL all-gather)")}[shard]
    return {
        "workload": f"{cfg['name']}: {cfg['layers']} layers, {cfg['n_q']} q / {cfg['n_kv']} kv heads, "
                    f"head_dim {cfg['head_dim']}, batch {cfg['batch']}"
                    + (" per GPU" if shard == "weak" else "") + f", {cfg['history']}-token packed "
                    f"history + U{{0..127}} bf16 residual + 1 new token, target_bit {cfg['target_bit']}",
        "layers": cfg["layers"], "batch_per_gpu": per_gpu,
        "global_batch": cfg["batch"] * n_gpus if shard == "weak" else cfg["batch"],
        "history_tokens": cfg["history"], "n_q": cfg["n_q"], "n_kv": cfg["n_kv"], "head_dim": cfg["head_dim"],
        "page_size": 128, "target_bit": cfg["target_bit"], "bit_v": 2,
        "l2": "no flush: per-step working set > 126 MB L2",
        "parallelism": par,
    }


# ------------------------------------------------------------- GPU leg ------
class Workload:
    """One rank's share of a config: the packed caches of every layer,
    per-step inputs, outputs and the per-layer decode calls."""

    def __init__(self, cfg: dict, rank: int, world: int, shard: str, dev, pps=None, with_k1=False,
                 kv_gather: str = "p2p"):
        import torch

        from logitfill_b200.packed import PackedKVCache
        from logitfill_b200.packed.attention import DecodeCall
        from logitfill_b200.sharding import kv_head_range, shard_levels
        from logitfill_b200.synthetic import synthetic_kv, synthetic_levels

        self.cfg, self.rank, self.world, self.shard, self.dev = cfg, rank, world, shard, dev
        L, D, T = cfg["layers"], cfg["head_dim"], cfg["history"]
        H, NQ, B = cfg["n_kv"], cfg["n_q"], cfg["batch"]
        levels = list(synthetic_levels(L, H, D, cfg["target_bit"], seed=cfg["seed"]))
        tails = tails_for(cfg, rank if shard == "weak" else 0)
        if shard == "kv":
            h0, h1, q0, q1 = kv_head_range(H, NQ, world, rank)
            levels = shard_levels(levels, H, world, rank)
            H, NQ = h1 - h0, q1 - q0
        elif shard == "batch":
            if B % world:
                raise ValueError(f"batch {B} does not split over {world} GPUs")
            per = B // world
            tails = tails[rank * per:(rank + 1) * per]
            B = per
        self.L, self.B, self.NQ, self.H, self.D = L, B, NQ, H, D
        self.levels = levels
        lengths = [T + t for t in tails]
        cache = PackedKVCache(levels, B, NQ, H, D, device=dev, capacity=T + 128)
        self.k1 = None
        for layer in range(L):
            k, v = synthetic_kv(B, H, T + 128, D, seed=cfg["seed"] * 1000 + rank, layer=layer, device=dev)
            cache.prefill(layer, k, v, lengths)
            if layer == 0 and with_k1:
                torch.cuda.synchronize()
                self.k1 = time_k1(cache, k, v, T, dev)
            del k, v
        torch.cuda.synchronize()
        cache.check_status()
        self.cache = cache
        gen = torch.Generator(device=dev).manual_seed(1234 + rank)
        self.q = torch.randn(L, B, NQ, D, generator=gen, device=dev).to(torch.bfloat16)
        self.kn = torch.randn(L, B, H, D, generator=gen, device=dev).to(torch.bfloat16)
        self.vn = torch.randn(L, B, H, D, generator=gen, device=dev).to(torch.bfloat16)
        self.out = torch.empty(L, B, NQ, D, device=dev, dtype=torch.bfloat16)
        self.gathered = None
        self.peer = None
        self.kv_gather = kv_gather
        if shard == "kv" and world > 1:
            if kv_gather == "p2p":
                from logitfill_b200.sharding import PeerGather

                self.peer = PeerGather(L, B, NQ, D, torch.bfloat16, dev)
                self.gathered = self.peer.gathered
            else:
                self.gathered = torch.empty(L, world, B, NQ, D, device=dev, dtype=torch.bfloat16)
        self.scaling = D ** -0.5
        self.calls = [DecodeCall(cache, l, self.q[l], self.kn[l], self.vn[l], self.scaling, self.out[l], pps=pps)
                      for l in range(L)]

    def step(self, calls=None, out=None, gathered=None):
        from logitfill_b200.sharding import gather_heads

        calls = calls or self.calls
        out = self.out if out is None else out
        gathered = self.gathered if gathered is None else gathered
        for l, c in enumerate(calls):
            if self.peer is not None and calls is self.calls:
                # K2, then the split merge storing this rank's heads into every
                # rank's buffer over NVLink, then the bounded wait for the layer.
                c.launch_partial()
                self.peer.merge(c, l)
                self.peer.wait(l)
                continue
            c.launch()
            if self.shard == "kv" and self.world > 1:
                gather_heads(out[l], gathered[l])

    def close(self) -> None:
        """Collective when the outputs are gathered through peer memory."""
        if self.peer is not None:
            self.peer.check_status()
            self.peer.close()
            self.peer = None

    def bytes_per_step(self):
        k2_bytes, total = [], 0
        for layer in self.cache.layers:
            c = layer.layout.c
            ww = (c.width[0], c.width[1], c.width[2], c.width[3], c.words[0], c.words[1], c.words[2])
            kb, tb = algorithmic_bytes(ww, layer.hist_len.tolist(), layer.tail_len.tolist(), self.NQ, self.H, self.D)
            k2_bytes.append(kb)
            total += tb
        return sum(k2_bytes) / len(k2_bytes), total


def _graph(fn):
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        fn()
    return g


def _timed_replays(graph, steps: int, stream, barrier, clocks=None) -> float:
    """ms per replay of ``graph`` over ``steps`` replays (CUDA events on the
    launching stream, barrier + synchronize on both sides)."""
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps


def measure(w: Workload, steps: int, warmup: int, barrier, clocks_index=None, e2e=True) -> dict:
    """Step time (graph replay), K2-only graph time, e2e, bytes and roofline
    of one workload on this rank; times are maxima over ranks."""
    import torch

    dev = w.dev
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(warmup, 1)):  # eager warm-up (also configures the kernels before capture)
        w.step()
    torch.cuda.synchronize()
    graph = _graph(w.step)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    clocks = None
    if clocks_index is not None:
        with ClockSampler(clocks_index) as cs:
            ms = _timed_replays(graph, steps, stream, barrier)
        clocks = cs.summary()
    else:
        ms = _timed_replays(graph, steps, stream, barrier)
    ms_max = max_over_ranks(ms, dev)

    # K2 alone: a graph of the L K2 launches (programmatic launches as in the step).
    k2_graph = _graph(lambda: [c.launch_partial() for c in w.calls])
    for _ in range(warmup):
        k2_graph.replay()
    k2_step_ms = max_over_ranks(_timed_replays(k2_graph, steps, stream, barrier), dev)
    k2_avg_ms = k2_step_ms / w.L
    del k2_graph

    res = {"ms": ms_max, "ms_rank": ms, "k2_avg_ms": k2_avg_ms, "k2_graph_ms": k2_step_ms, "clocks": clocks}
    if e2e:
        res.update(measure_e2e(w, steps, barrier, graph))
    del graph
    k2_bytes_avg, step_bytes = w.bytes_per_step()
    res["k2_bytes"], res["step_bytes"] = k2_bytes_avg, step_bytes
    return res


def measure_e2e(w: Workload, steps: int, barrier, graph) -> dict:
    """The step through the public API with host buffers: every step uploads
    its inputs from pinned host memory and reads its outputs back.  Two device
    buffer sets (and a graph bound to each) let step i+1's upload and step i's
    read-back run on a copy stream while the GPU computes; every copy is
    inside the timed region."""
    import torch

    from logitfill_b200.packed.attention import DecodeCall

    dev = w.dev
    stream = torch.cuda.current_stream(dev)
    q, kn, vn = w.q, w.kn, w.vn
    result = w.gathered if w.gathered is not None else w.out
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, kn, vn))
    q2, kn2, vn2, out2 = (torch.empty_like(x) for x in (q, kn, vn, w.out))
    g2 = torch.empty_like(w.gathered) if w.gathered is not None else None
    calls2 = [DecodeCall(w.cache, l, q2[l], kn2[l], vn2[l], w.scaling, out2[l], pps=w.calls[l].pps)
              for l in range(w.L)]
    graph2 = _graph(lambda: w.step(calls2, out2, g2))
    res2 = g2 if g2 is not None else out2
    sets = [(q, kn, vn, result, graph), (q2, kn2, vn2, res2, graph2)]
    houts = [torch.empty(result.shape, dtype=result.dtype, pin_memory=True) for _ in range(2)]
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
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    upload(0)
    for i in range(steps):
        b = i % 2
        stream.wait_event(uploaded[b])
        sets[b][4].replay()
        computed[b].record(stream)
        if i + 1 < steps:
            upload(i + 1)
        with torch.cuda.stream(cs):
            cs.wait_event(computed[b])
            houts[b].copy_(sets[b][3], non_blocking=True)
    read_back = torch.cuda.Event()
    read_back.record(cs)
    stream.wait_event(read_back)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps, dev)
    last = (steps - 1) % 2
    assert torch.equal(houts[last], sets[last][3].cpu())
    del graph2
    return {"e2e_ms": e2e_ms, "h2d": sum(x.numel() * x.element_size() for x in (hq, hk, hv)),
            "d2h": houts[0].numel() * houts[0].element_size()}


def block(w: Workload, m: dict, config_id: int, traffic_ok: bool) -> dict:
    """JSON fields of one measured workload (whole job over all ranks)."""
    peak, peak_kind = measured_peak_hbm()
    cfg, world = w.cfg, w.world
    seqs = cfg["batch"] * world if w.shard == "weak" else cfg["batch"]
    achieved = m["k2_bytes"] / (m["k2_avg_ms"] * 1e-3) / 1e9
    step_gbs = m["step_bytes"] / (m["ms"] * 1e-3) / 1e9
    out = {
        "value": seqs / (m["ms"] * 1e-3), "unit": "tok/s", "ms_per_step": m["ms"], "n_gpus": world,
        "scaling": "weak" if w.shard == "weak" else "strong",
        "config": workload_config(cfg, world, w.shard, w.kv_gather),
        "hbm_gbs": step_gbs * world, "hbm_frac_of_peak_per_gpu": step_gbs / peak,
        "pages_per_split": w.calls[0].pps,
        "roofline": {"kernel": "lf_decode_partial (K2)", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": ncu_traffic(config_id) if traffic_ok else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one K2 launch, "
                                       "same config (committed capture summary)",
                     "bytes_per_launch": m["k2_bytes"], "avg_launch_ms": m["k2_avg_ms"],
                     "avg_launch_method": "CUDA graph of the L K2 launches alone (programmatic launches), "
                                          "event-timed, divided by L",
                     "k2_share_of_step": m["k2_graph_ms"] / m["ms"]},
        "gpu_launches_per_step": w.L * 2,
    }
    if "e2e_ms" in m:
        out["e2e"] = {"value": seqs / (m["e2e_ms"] * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": m["h2d"] * world,
                      "d2h_bytes_per_step": m["d2h"] * world, "ms_per_step": m["e2e_ms"],
                      "method": "pipelined attention-only loop: step i+1's inputs uploaded and step i's outputs read "
                                "back on a copy stream while step i computes"}
    if m.get("clocks") is not None:
        out["clocks"] = m["clocks"]
    return out


def run_b200(args, cfg) -> None:
    import gc

    import torch
    import torch.distributed as dist

    if args.k2 != "auto":
        os.environ["LF_K2_KERNEL"] = args.k2
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cpu_rates = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # Host baselines first: their worker pools start (spawn) before this
        # process's GPU work, and the GPU is idle meanwhile.
        cores = host_cores()
        cpu_rates = {kind: cpu_decode_rates(cfg, 10.0, cores, kind)[0] for kind in ("torch", "numpy")}
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from logitfill_b200.synthetic import mean_key_bits

    w = Workload(cfg, rank, world, args.shard, dev, pps=args.pps, with_k1=True)
    m = measure(w, args.steps, args.warmup, barrier, clocks_index=local)
    main = block(w, m, args.config, traffic_ok=args.target_bit is None and args.batch is None and world == 1
                 and args.shard == "weak" and args.k2 != "simt")
    chunk = None
    if not args.no_blocks and args.config == 1 and args.shard == "weak" and world == 1:
        chunk = run_chunk(w, 16, max(3, min(args.steps, 10)), args.warmup, main["roofline"]["peak"])
    k1 = w.k1
    key_bits = mean_key_bits(w.levels if args.shard != "kv" else [lv.numpy() for lv in w.levels])
    launches = args.steps * w.L * 2
    del w
    gc.collect()
    torch.cuda.empty_cache()

    extra = {}
    if chunk is not None:
        extra["config1_chunk16"] = chunk
    if not args.no_blocks and args.config == 1 and args.shard == "weak":
        if world == 1:
            w2 = Workload(CONFIGS[2], rank, world, "weak", dev)
            extra["config2"] = block(w2, measure(w2, args.steps, args.warmup, barrier), 2,
                                     traffic_ok=args.k2 != "simt")
            del w2
            gc.collect()
            torch.cuda.empty_cache()
            extra["config3"] = run_config3(args.steps, args.warmup, dev, main["roofline"]["peak"])
            gc.collect()
            torch.cuda.empty_cache()
        steps4 = max(3, min(args.steps, 10))
        shards = [("kv", "p2p")] + ([("kv", "nccl"), ("batch", None)] if world > 1 else [])
        for shard, gather in shards:
            w4 = Workload(CONFIGS[4], rank, world, shard, dev, kv_gather=gather or "p2p")
            b4 = block(w4, measure(w4, steps4, args.warmup, barrier, e2e=False), 4, traffic_ok=False)
            b4["steps"] = steps4
            extra["config4_kv_nccl" if gather == "nccl" else f"config4_{shard}"] = b4
            w4.close()
            del w4
            gc.collect()
            torch.cuda.empty_cache()

    if rank == 0:
        line = {
            "metric": METRIC, "value": main["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "higher_is_better": True,
            "scaling": main["scaling"], "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": main["config"], "hbm_gbs": main["hbm_gbs"],
            "hbm_frac_of_peak_per_gpu": main["hbm_frac_of_peak_per_gpu"], "key_mean_bits": key_bits,
            "pages_per_split": main["pages_per_split"], "k2_kernel": args.k2,
            "roofline": main["roofline"],
            "k1": dict(k1, peak=main["roofline"]["peak"], frac=k1["achieved"] / main["roofline"]["peak"]),
            "e2e": main["e2e"],
            "cpu_baseline": None,
            "clocks": main.get("clocks"),
            "gpu_launches": launches,
        }
        if cpu_rates is not None:
            best = max(cpu_rates.values(), key=lambda r: r["value"])
            line["cpu_baseline"] = {k: best[k] for k in ("value", "unit", "cores", "kind", "sample")}
            line["cpu_baselines"] = {kind: {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
                                     for kind, r in cpu_rates.items()}
        line.update(extra)
        print(json.dumps(line), flush=True)
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
    ap.add_argument("--shard", default="weak", choices=["weak", "batch", "kv"],
                    help="weak: every GPU holds the config's batch; batch / kv: the config is split over the GPUs "
                         "by sequence / by KV head (kv gathers each layer's output over NCCL)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--k2", default="auto", choices=["auto", "tc", "simt"],
                    help="K2 kernel: auto/tc = tensor-core kernel where the geometry allows, simt = CUDA-core kernel")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-blocks", action="store_true", help="only the main line (no config2 / config4 blocks)")
    ap.add_argument("--target-bit", type=float, default=None,
                    help="override the config's Key policy budget (config 2 sweep: 2.25, 2.5, 3.0, 4.0)")
    ap.add_argument("--pps", type=int, default=None,
                    help="pages per K2 work item (default: the occupancy-aware planner)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the config's sequences per GPU (small cases for profiling)")
    ap.add_argument("--config3-only", action="store_true",
                    help="print only the config-3 block (page compression path), one GPU")
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
    if args.config3_only:
        import torch

        torch.cuda.set_device(0)
        peak, _ = measured_peak_hbm()
        print(json.dumps({"config3": run_config3(args.steps, args.warmup, torch.device("cuda", 0), peak)}), flush=True)
    elif args.model_decode:
        run_model_decode(args)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
