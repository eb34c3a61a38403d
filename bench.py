#!/usr/bin/env python
"""Headline benchmark: sparse-decode µs/layer @ 32K context, 1K budget.

Workload (the headline "32K ctx, B=1024" configuration with outlier-key inputs): one
request, 32 heads MHA, head_dim 128, fp16 paged KV with page_size 16, context
32768 tokens (N = 2048 pages), budget 1024 tokens (64 pages: 63 selected +
the last page), AOA-KV value-aware scoring; K ~ N(0,1) * LogNormal(0,1)
per-channel scale, q, V ~ N(0,1), seed 1; synthetic data.

A "step" is one decode token through L = 32 layers (each layer has its own
KV cache, metadata and v_log_norm): per layer the library appends the token
and runs estimate -> top-k -> sparse decode. The 32 layers touch
32 x 50.5 MB > L2 (126 MB) per step, so no layer finds its data in L2.

  value     device time per layer-step, whole job: max-over-ranks time of K
            CUDA-graph replays of the 32-layer step / (K * 32 * n_gpus)
  e2e       the same through InferenceController.decode_step, with the
            step's q, k, v copied from pinned host memory and its outputs
            copied back inside the timed region, no graph
  roofline  the step kernel (one fused launch per layer): algorithmic bytes
            of a layer-step / its average duration inside the timed graph;
            estimate_roofline: the stand-alone page scorer timed the same way

With --gpus N (torchrun, one process per GPU) every rank serves its own
request (request sharding, no collective): scaling "weak".
--mode longctx instead splits ONE 128K-context request (budget 4096) by page
range over the GPUs, with two NCCL all_gathers per layer: scaling "strong".
--mode batched runs 32 requests of 4K-16K tokens (config 4), balanced over
the GPUs by bytes, no collective: scaling "strong". --mode model times a
32-layer Llama-2-7B-shaped decode step with this attention (config 3).
--impl reference times the reference's CPU simulation path (the numpy port
in oracle/sim.py of filter_util.py + quest_attention.py) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "sparse-decode µs/layer @32K ctx, 1K budget; % of B200 HBM roofline"
# DRAM bytes (read + write) of one fused step launch at the headline shape,
# from the ncu capture summarised under profiles/ (dram__bytes_read.sum +
# dram__bytes_write.sum, one layer, caches flushed)
STEP_TRAFFIC_BYTES = 52_328_448
H, D, P = 32, 128, 16


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["headline", "longctx", "batched", "model"],
                    default="headline",
                    help="headline: 32K ctx, 1K budget, one request per GPU; longctx: one "
                         "128K-context request split by page range over the GPUs; batched: "
                         "--requests requests of 4K-16K tokens balanced over the GPUs; "
                         "model: a 32-layer Llama-2-7B-shaped decode step (random weights)")
    ap.add_argument("--requests", type=int, default=32, help="batched: requests in the batch")
    ap.add_argument("--streams", type=int, default=8,
                    help="batched: requests' steps run side by side on this many streams, each "
                         "step's fused kernel capped to its share of the GPU (1 = one after "
                         "another on the whole GPU)")
    ap.add_argument("--layers", type=int, default=None, help="default 32 (headline), 4 (longctx)")
    ap.add_argument("--ctx", type=int, default=None, help="default 32768 (headline), 131072 (longctx)")
    ap.add_argument("--budget", type=int, default=None,
                    help="token budget; default 1024 (headline), 4096 (longctx)")
    ap.add_argument("--method", choices=["aoakv", "quest"], default="aoakv")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="CPU-baseline sample budget (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--soak-seconds", type=float, default=1.0,
                    help="graph replays before the timed region so the clock sampler sees load")
    ap.add_argument("--no-graph", action="store_true", help="longctx: launch without a CUDA graph")
    a = ap.parse_args()
    long = a.mode == "longctx"
    a.layers = a.layers or (4 if a.mode != "headline" else 32)
    a.ctx = a.ctx or (131072 if long else 32768)
    a.budget = a.budget or (4096 if long else 1024)
    return a


def lib_md5() -> str:
    """md5 of the loaded libaoakv.so (the reference's latency CSV records the
    kernel build per row the same way, bench_latency.py:42-46)."""
    import hashlib
    from aoa_kv_b200 import _lib
    try:
        return hashlib.md5(Path(_lib.LIB_PATH).read_bytes()).hexdigest()
    except OSError:
        return "unknown"


def workload_config(a, n_gpus):
    n_pages = (a.ctx + P - 1) // P
    return {
        "workload": f"1 request/GPU, {a.layers}-layer decode step, ctx {a.ctx}, budget {a.budget}",
        "context_tokens": a.ctx, "token_budget": a.budget, "page_size": P, "num_heads": H,
        "head_dim": D, "layers_per_step": a.layers, "score_mode": a.method, "sink_first_page": False,
        "pages_scored": n_pages - 1, "pages_attended": min(a.budget // P, n_pages),
        "inputs": "K~N(0,1)*LogNormal(0,1)[h,d], q,V~N(0,1), seed %d" % a.seed,
        "l2": "inputs larger than L2: %d layers x %.1f MB touched per step" % (
            a.layers, step_bytes(a) / 1e6),
        "accumulate": "fp32", "parallelism": f"request-sharded x{n_gpus}, no collective",
    }


def step_bytes(a) -> int:
    """Algorithmic bytes of one layer-step: metadata of the
    N-1 scored pages, their v_log_norm (aoakv), the k attended pages' K and V,
    and q + o."""
    n = (a.ctx + P - 1) // P
    k = min(a.budget // P, n)
    b = (n - 1) * H * 2 * D * 2 + k * P * H * D * 2 * 2 + 2 * H * D * 2
    if a.method == "aoakv":
        b += (n - 1) * H * 2
    return b


def estimate_bytes(a) -> int:
    """Algorithmic bytes of one estimate launch: metadata + v_log_norm of the
    N-1 scored pages, q, and the fp32 scores written."""
    n = (a.ctx + P - 1) // P
    b = (n - 1) * H * 2 * D * 2 + H * D * 2 + (n - 1) * H * 4
    if a.method == "aoakv":
        b += (n - 1) * H * 2
    return b


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (100 ms) of the benchmark's GPU while it runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.samples = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except (OSError, ValueError):
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.monotonic(), parts))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [p for t, p in self.samples if t0 <= t <= t1] or [p for _, p in self.samples]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def gpu_query_id(dev_index: int) -> str:
    import torch
    try:
        p = torch.cuda.get_device_properties(dev_index)
        return "%08X:%02X:%02X.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
    except Exception:  # noqa: BLE001 - fall back to the ordinal
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[dev_index] if vis else str(dev_index)


# ------------------------------------------------------------- CPU baseline
def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:  # noqa: BLE001
        pass
    return os.cpu_count() or 1


def cpu_sim_setup(a):
    import numpy as np
    from oracle import sim
    g = np.random.default_rng(a.seed)
    S = a.ctx
    q = g.standard_normal((H, D), dtype=np.float32).astype(np.float16).astype(np.float32)
    scale = np.exp(g.standard_normal((H, D), dtype=np.float32))
    K = (g.standard_normal((H, S, D), dtype=np.float32) * scale[:, None]).astype(np.float16)
    V = g.standard_normal((H, S, D), dtype=np.float32).astype(np.float16)
    st = sim.SimLayerState(K[:, :-1].astype(np.float32), V[:, :-1].astype(np.float32), P)
    return st, q, K[:, -1].astype(np.float32), V[:, -1].astype(np.float32)


def cpu_sim_steps(a, n_steps, budget_s=None):
    """Times the reference simulation's decode step for one layer (one unit of
    the metric) on the host cores; returns per-step seconds."""
    import copy

    from oracle import sim
    st0, q, k, v = cpu_sim_setup(a)
    times = []
    t_start = time.perf_counter()
    for _ in range(n_steps):
        st = copy.copy(st0)  # decode_step rebinds arrays; the prefill state is reused
        t0 = time.perf_counter()
        sim.decode_step(st, q, k, v, a.budget, a.method, True, expand=True)
        times.append(time.perf_counter() - t0)
        if budget_s and time.perf_counter() - t_start > budget_s:
            break
    return times


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    n_gpus = int(os.environ.get("WORLD_SIZE", str(a.gpus)))
    if rank != 0:
        return
    for _ in range(max(0, min(a.warmup, 3))):
        cpu_sim_steps(a, 1)
    times = cpu_sim_steps(a, a.steps)
    us = statistics.median(times) * 1e6
    cores = cpu_threads()
    line = {
        "metric": METRIC, "value": round(us, 3), "unit": "us", "impl": "reference",
        "n_gpus": n_gpus, "steps": len(times), "warmup": a.warmup, "ms_per_step": round(us / 1e3, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(a, n_gpus),
        "cpu_baseline": {"value": round(us, 3), "unit": "us", "cores": cores, "kind": "port",
                         "sample": f"{len(times)} single-layer decode steps of the simulation "
                                   f"(oracle/sim.py restating filter_util.py + quest_attention.py), "
                                   f"ctx {a.ctx}, budget {a.budget}, {a.method}, fixed=True, median"},
        "e2e": {"value": round(us, 3), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm
def setup_layers(a, dev):
    import torch

    import aoa_kv_b200 as ak
    gen = torch.Generator(device=dev).manual_seed(a.seed)
    ctl = ak.InferenceController(a.layers, H, D, P, a.budget // P, a.ctx + P, torch.float16, dev,
                                 method=a.method)
    S = a.ctx
    ctl.prepare_metadata(S - 1)
    ctl.begin_forward(S - 1)
    news = []
    for layer in range(a.layers):
        scale = torch.exp(torch.randn(H, D, device=dev, generator=gen))
        K = (torch.randn(S, H, D, device=dev, generator=gen) * scale).half()
        V = torch.randn(S, H, D, device=dev, generator=gen).half()
        q = torch.randn(1, H, D, device=dev, generator=gen).half()
        ak.append_kv(K[:-1].contiguous(), V[:-1].contiguous(), ctl, layer)
        news.append((q, K[-1:].contiguous(), V[-1:].contiguous()))
        del K, V
    ctl.end_forward()
    ctl.prepare_metadata(1)
    ctl.begin_forward(1)
    torch.cuda.synchronize()
    return ctl, news


def run_ours(a):
    import torch
    import torch.distributed as dist

    import aoa_kv_b200 as ak
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ak._lib.load()

    ctl, news = setup_layers(a, dev)
    outs = [torch.empty(1, H, D, dtype=torch.float16, device=dev) for _ in range(a.layers)]
    import ctypes
    nk = ctypes.c_int32(0)
    ak._lib.call("aoakv_step_launches", H, D, P, len(ctl.kv_cache.indicies),
                 ctl.step_page_budget(), int(ctl.sink_first_page), 0, ctypes.byref(nk))
    kernels_per_layer = int(nk.value)

    def one_step():
        for layer, (q, k, v) in enumerate(news):
            ctl.decode_step(q, k, v, layer, out=outs[layer])

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        one_step()  # first calls set kernel attributes outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        one_step()
    torch.cuda.synchronize()
    ak.check_device()

    sampler = ClockSampler(gpu_query_id(local)) if rank == 0 else None
    t_soak = time.monotonic()
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()
    # keep the GPU busy so the clock sampler sees it under this load
    t_end = time.monotonic() + a.soak_seconds
    while time.monotonic() < t_end:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(a.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_timed_end = time.monotonic()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ak.check_device()
    us_layer_job = ms * 1e3 / (a.steps * a.layers * world)
    us_layer_gpu = ms * 1e3 / (a.steps * a.layers)

    # --- dominant kernel alone: the page-score estimate (fp32 scores)
    n = (a.ctx + P - 1) // P
    scores = torch.empty(H, n, dtype=torch.float32, device=dev)

    def est_all():
        for layer, (q, _, _) in enumerate(news):
            meta = ctl.metadata_cache.buf_layer(layer)
            ak._lib.call("aoakv_estimate_attn_score", q.data_ptr(), scores.data_ptr(), 1, n,
                         meta.data_ptr(), ctl.metadata_indices.data_ptr(),
                         len(ctl.metadata_cache.indicies), ctl.metadata_cache.last_page_len,
                         meta.shape[0], ctl.kv_indices_with_last.data_ptr(),
                         ctl.kv_cache.pool.capacity, ctl.v_log_norm_layer(layer).data_ptr(), H, D,
                         P, 0, ctl.score_mode, torch.cuda.current_stream().cuda_stream)
    with torch.cuda.stream(s):
        est_all()
    torch.cuda.synchronize()
    g_est = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_est):
        est_all()
    for _ in range(3):
        g_est.replay()
    reps = max(5, a.steps // 2)
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(reps):
        g_est.replay()
    ev1.record()
    torch.cuda.synchronize()
    est_us = ev0.elapsed_time(ev1) * 1e3 / (reps * a.layers)

    # --- e2e through the public API with host buffers
    e2e = None
    if not a.no_e2e:
        # the step's inputs (every layer's q, k, v) in one pinned host buffer,
        # copied in once per step; every layer's output read back once
        pin_qkv = torch.stack([torch.stack([t[0], t[1], t[2]]) for t in news]).cpu().pin_memory()
        dev_qkv = torch.empty_like(pin_qkv, device=dev)  # [L, 3, 1, H, D]
        o_all = torch.empty(a.layers, 1, H, D, dtype=torch.float16, device=dev)
        host_o = torch.empty(a.layers, 1, H, D, dtype=torch.float16).pin_memory()

        def e2e_step():
            dev_qkv.copy_(pin_qkv, non_blocking=True)
            for layer in range(a.layers):
                ctl.decode_step(dev_qkv[layer, 0], dev_qkv[layer, 1], dev_qkv[layer, 2], layer,
                                out=o_all[layer])
            host_o.copy_(o_all, non_blocking=True)
        for _ in range(a.warmup):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0.record()
        for _ in range(a.steps):
            e2e_step()
        ev1.record()
        torch.cuda.synchronize()
        ems = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([ems], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": round(ems * 1e3 / (a.steps * a.layers * world), 3), "unit": "us",
               "h2d_bytes_per_step": a.layers * 3 * H * D * 2,
               "d2h_bytes_per_step": a.layers * H * D * 2,
               "api": "InferenceController.decode_step per layer (ctypes -> aoakv_decode_step); "
                      "one H2D of the step's q/k/v and one D2H of its outputs; no graph"}

    if sampler:
        sampler.stop()
    clocks = sampler.summary(t_soak, t_timed_end) if sampler else None

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs") or 6650.0)
    peak_src = "measured" if peaks.get("hbm_gbs") else "fallback"
    eb = estimate_bytes(a)
    ach = eb / (est_us * 1e-6) / 1e9
    sb = step_bytes(a)
    step_ach = sb / (us_layer_gpu * 1e-6) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        times = cpu_sim_steps(a, 50, budget_s=a.cpu_seconds)
        cpu_us = statistics.median(times) * 1e6
        cpu = {"value": round(cpu_us, 1), "unit": "us", "cores": cpu_threads(), "kind": "port",
               "sample": f"{len(times)} single-layer decode steps of the reference simulation "
                         f"(oracle/sim.py: filter_util.py + quest_attention.py decode branch) at "
                         f"ctx {a.ctx}, budget {a.budget}, {a.method}, fixed=True; median"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(us_layer_job, 3), "unit": "us", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": workload_config(a, world),
            "per_gpu_us_per_layer": round(us_layer_gpu, 3),
            # the step kernel: one launch per layer (fused) or the chain of
            # kernels_per_layer launches; avg launch duration = timed graph
            # time / layers, gaps between launches included
            "roofline": {"bound": "hbm",
                         "kernel": "fused_step_kernel (append+estimate+top-k+decode)"
                         if kernels_per_layer == 1 else
                         f"step chain of {kernels_per_layer} kernels",
                         "achieved": round(step_ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(step_ach / peak, 4),
                         "traffic": STEP_TRAFFIC_BYTES if (kernels_per_layer == 1 and
                                                           a.ctx == 32768 and a.budget == 1024 and
                                                           a.method == "aoakv") else None,
                         "algorithmic_bytes": sb, "avg_launch_us": round(us_layer_gpu, 3),
                         "ideal_us": round(sb / (peak * 1e9) * 1e6, 3),
                         "peak_source": peak_src},
            "estimate_roofline": {"kernel": "estimate_attn_score stand-alone (page scorer)",
                                  "achieved": round(ach, 1), "unit": "GB/s",
                                  "frac": round(ach / peak, 4), "algorithmic_bytes": eb,
                                  "avg_launch_us": round(est_us, 3)},
            "e2e": e2e, "gpu_launches": kernels_per_layer * a.layers * a.steps,
            "step_kernels_per_layer": kernels_per_layer, "clocks": clocks,
            "library_md5": lib_md5(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph, g_est
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------ long context, sharded
LONG_METRIC = "sparse-decode µs/layer @128K ctx, 4K budget, page-range sharded"


class _SoloGroup:
    """The all_gather of a one-rank job."""

    @staticmethod
    def all_gather_stack(t):
        return t.unsqueeze(0)


def run_longctx(a):
    """One request of a.ctx tokens split by page range over the job's GPUs
    (aoa_kv_b200.sharded): per layer, the last rank appends, every rank
    scores and proposes its top-(k-1), all_gather, global top-(k-1), partial
    decode of the owned pages, all_gather, LSE merge. Strong scaling: the
    total work is one request whatever the GPU count."""
    import datetime

    import torch
    import torch.distributed as dist

    from aoa_kv_b200 import _lib, sharded
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD
    else:
        group = _SoloGroup()
    _lib.load()
    S = a.ctx
    n_total, last_len = S // P + 1, S % P + 1
    lo, hi = sharded.partition_pages(n_total, world, P)[rank]
    n_local = hi - lo
    owns = rank == world - 1
    cap = n_local + 1
    mcap = -(-cap // P)
    layers, news = [], []
    for layer in range(a.layers):
        g_layer = torch.Generator(device=dev).manual_seed(a.seed * 1000 + layer)
        scale = torch.exp(torch.randn(H, D, device=dev, generator=g_layer))
        q = torch.randn(H, D, device=dev, generator=g_layer).half()
        k_new = (torch.randn(H, D, device=dev, generator=g_layer) * scale).half()
        v_new = torch.randn(H, D, device=dev, generator=g_layer).half()
        g_rank = torch.Generator(device=dev).manual_seed(a.seed * 100000 + layer * 100 + rank)
        kv = torch.empty(cap, 2, P, H, D, dtype=torch.float16, device=dev)
        meta = torch.empty(mcap, 2, P, H, D, dtype=torch.float16, device=dev)
        vlog = torch.zeros(cap, H, dtype=torch.float16, device=dev)
        kv_idx = torch.arange(n_local, dtype=torch.int32, device=dev)
        meta_idx = torch.arange(mcap, dtype=torch.int32, device=dev)
        t0, t1 = lo * P, min(hi * P, S)
        if t1 > t0:
            Kc = (torch.randn(t1 - t0, H, D, device=dev, generator=g_rank) * scale).half()
            Vc = torch.randn(t1 - t0, H, D, device=dev, generator=g_rank).half()
            n_pref = -(-(t1 - t0) // P)
            _lib.call("aoakv_append_kv_cache_prefill", Kc.data_ptr(), Vc.data_ptr(), t1 - t0,
                      kv.data_ptr(), kv_idx.data_ptr(), n_pref, (t1 - t0 - 1) % P + 1, cap,
                      meta.data_ptr(), meta_idx.data_ptr(), -(-n_pref // P),
                      (n_pref - 1) % P + 1, mcap, vlog.data_ptr(), H, D, P, _lib.LAYOUT_NHD,
                      torch.cuda.current_stream().cuda_stream)
            del Kc, Vc
        layers.append(sharded.ShardLayer(kv=kv, meta=meta, vlog=vlog, kv_idx=kv_idx,
                                         meta_idx=meta_idx, page_lo=lo, n_local=n_local,
                                         n_total=n_total, last_len=last_len, owns_last=owns,
                                         last_phys=n_local - 1 if owns else -1))
        news.append((q, k_new, v_new))
    torch.cuda.synchronize()
    dec = sharded.ShardedDecoder(group, H, D, P, a.budget // P, a.method)

    def one_step():
        for lay, (q, k, v) in zip(layers, news):
            dec.step(lay, q, k, v)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        one_step()  # workspaces and kernel attributes outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = None
    if not a.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_step()
    def run():
        if graph is not None:
            graph.replay()
        else:
            one_step()

    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    _lib.check_device()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        run()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    _lib.check_device()
    us = ms * 1e3 / (a.steps * a.layers)
    sb = step_bytes(a)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs") or 6650.0)
    ach = sb / (us * 1e-6) / 1e9
    ks = min(a.budget // P, n_total) - 1
    if rank == 0:
        print(json.dumps({
            "metric": LONG_METRIC, "value": round(us, 3), "unit": "us", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": f"1 request, {a.layers}-layer decode step, ctx {S}, budget "
                                   f"{a.budget}, pages split by range over {world} GPU(s)",
                       "context_tokens": S, "token_budget": a.budget, "page_size": P,
                       "num_heads": H, "head_dim": D, "layers_per_step": a.layers,
                       "score_mode": a.method, "pages_per_gpu": n_local,
                       "exchange_bytes_per_layer_per_gpu": world * H * ks * 8 +
                       world * H * (D + 1) * 4,
                       "graph": graph is not None,
                       "parallelism": f"page-range x{world}, all_gather of candidates and "
                                      f"partial states (NCCL)" if world > 1 else "1 GPU"},
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak * world,
                         "unit": "GB/s", "frac": round(ach / (peak * world), 4),
                         "algorithmic_bytes": sb, "avg_layer_us": round(us, 3),
                         "note": "peak = measured HBM GB/s x GPUs"},
        }), flush=True)
    # a graph that holds NCCL calls must be released before the process
    # group, or the exit waits for ever
    graph = None
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------ batched decode
BATCH_METRIC = "sparse-decode µs/layer for a batch of 32 requests (4K-16K ctx, 1K budget)"


def run_batched(a):
    """Config 4: a.requests independent requests, context U[4096, 16384]
    tokens in whole pages (seed 3), budget a.budget, balanced over the job's
    GPUs by bytes (aoa_kv_b200.batching); each GPU runs its requests' steps
    (one fused launch per request and layer) in a CUDA graph. No collective
    on the data path; the total work is fixed: scaling "strong"."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    import aoa_kv_b200 as ak
    from aoa_kv_b200 import batching
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    ak._lib.load()
    g = np.random.default_rng(3)
    ctxs = [int(c) * P for c in g.integers(4096 // P, 16384 // P + 1, size=a.requests)]
    weights = [batching.step_bytes(c, a.budget, H, D, P, a.method) for c in ctxs]
    mine = batching.balance_requests(weights, world)[rank]
    reqs = []
    for r in mine:
        gen = torch.Generator(device=dev).manual_seed(3000 + r)
        S = ctxs[r]
        ctl = ak.InferenceController(a.layers, H, D, P, a.budget // P, S + P, torch.float16, dev,
                                     method=a.method)
        ctl.prepare_metadata(S - 1)
        ctl.begin_forward(S - 1)
        news = []
        for layer in range(a.layers):
            scale = torch.exp(torch.randn(H, D, device=dev, generator=gen))
            K = (torch.randn(S, H, D, device=dev, generator=gen) * scale).half()
            V = torch.randn(S, H, D, device=dev, generator=gen).half()
            q = torch.randn(1, H, D, device=dev, generator=gen).half()
            ak.append_kv(K[:-1].contiguous(), V[:-1].contiguous(), ctl, layer)
            news.append((q, K[-1:].contiguous(), V[-1:].contiguous(),
                         torch.empty(1, H, D, dtype=torch.float16, device=dev)))
            del K, V
        ctl.end_forward()
        ctl.prepare_metadata(1)
        ctl.begin_forward(1)
        reqs.append((ctl, news))
    torch.cuda.synchronize()

    n_streams = max(1, min(a.streams, len(reqs)))
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    cap = 0 if n_streams == 1 else max(64, (2 * sms // n_streams) // 2 * 2)
    lanes = [torch.cuda.Stream(device=dev) for _ in range(n_streams)]
    order = sorted(range(len(reqs)), key=lambda i: -weights[mine[i]])
    lane_of = {i: j % n_streams for j, i in enumerate(order)}

    def one_step():
        # fork: every lane waits for the issuing stream; join at the end
        main = torch.cuda.current_stream()
        for ln in lanes:
            ln.wait_stream(main)
        for layer in range(a.layers):
            for i, (ctl, news) in enumerate(reqs):
                q, k, v, o = news[layer]
                with torch.cuda.stream(lanes[lane_of[i]]):
                    ctl.decode_step(q, k, v, layer, out=o, max_ctas=cap)
        for ln in lanes:
            main.wait_stream(ln)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        one_step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        one_step()
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ak.check_device()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ak.check_device()
    us = ms * 1e3 / (a.steps * a.layers)
    total_bytes = sum(weights)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs") or 6650.0)
    ach = total_bytes / (us * 1e-6) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": BATCH_METRIC.replace("32 requests", f"{a.requests} requests"),
            "value": round(us, 3), "unit": "us", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{a.requests} requests, ctx U[4096,16384] tokens (seed 3), "
                                   f"budget {a.budget}, {a.layers}-layer step",
                       "requests_on_rank0": len(mine), "bytes_per_layer_step": total_bytes,
                       "streams": n_streams, "ctas_per_step": cap or "whole GPU",
                       "parallelism": f"request-sharded x{world} (greedy byte balance), "
                                      f"no collective"},
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak * world,
                         "unit": "GB/s", "frac": round(ach / (peak * world), 4),
                         "note": "peak = measured HBM GB/s x GPUs"},
        }), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------- Llama-2-7B-shaped decode step
MODEL_METRIC = "ms/token, 32-layer Llama-2-7B-shaped decode, sparse attention (layers 2-31)"


def run_model(a):
    """Config 3: one decode token through a 32-layer Llama-2-7B-shaped model
    with random fp16 weights (hidden 4096, 32 heads, head_dim 128, MLP 11008,
    vocab 32000): RMSNorm, q/k/v GEMVs, RoPE (aoakv_apply_rope_in_place),
    attention through
    InferenceController.decode_step (layers 0-1 dense, as in the reference's
    skip layers, llama.py:428-439; the rest with the token budget), o_proj,
    SwiGLU MLP, final norm, LM head and a device-side argmax, captured in one
    CUDA graph. The KV caches hold a.ctx synthetic tokens per layer. The
    GEMVs are torch (cuBLAS); the attention share is timed separately by
    replaying a graph of only the attention calls."""
    import torch

    import aoa_kv_b200 as ak
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    ak._lib.load()
    L, HID, FF, VOCAB = 32, 4096, 11008, 32000
    gen = torch.Generator(device=dev).manual_seed(a.seed)

    def w(*shape):
        return (torch.randn(*shape, device=dev, generator=gen) * 0.02).half()

    layers = [dict(ln1=torch.ones(HID, device=dev, dtype=torch.float16), wq=w(HID, HID),
                   wk=w(HID, HID), wv=w(HID, HID), wo=w(HID, HID),
                   ln2=torch.ones(HID, device=dev, dtype=torch.float16), wg=w(HID, FF),
                   wu=w(HID, FF), wd=w(FF, HID)) for _ in range(L)]
    emb, lm_head = w(VOCAB, HID), w(HID, VOCAB)
    norm_f = torch.ones(HID, device=dev, dtype=torch.float16)
    weight_bytes = sum(t.numel() * 2 for lw in layers for t in lw.values()) + \
        (emb.numel() + lm_head.numel() + norm_f.numel()) * 2

    S = a.ctx
    ctl = ak.InferenceController(L, H, D, P, a.budget // P, S + P, torch.float16, dev,
                                 method=a.method)
    ctl.prepare_metadata(S - 1)
    ctl.begin_forward(S - 1)
    for layer in range(L):
        scale = torch.exp(torch.randn(H, D, device=dev, generator=gen))
        K = (torch.randn(S - 1, H, D, device=dev, generator=gen) * scale).half()
        V = torch.randn(S - 1, H, D, device=dev, generator=gen).half()
        ak.append_kv(K, V, ctl, layer)
        del K, V
    ctl.end_forward()
    ctl.prepare_metadata(1)
    ctl.begin_forward(1)
    dense_budget = ctl.kv_cache.pool.capacity  # layers 0-1: every page
    sparse_budget = a.budget // P


    def rmsnorm(x, g):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).half() * g

    token = torch.zeros(1, dtype=torch.long, device=dev)
    q_buf = torch.empty(L, 1, H, D, dtype=torch.float16, device=dev)
    k_buf = torch.empty_like(q_buf)
    v_buf = torch.empty_like(q_buf)
    o_buf = torch.empty_like(q_buf)
    for layer in (0, 1):  # size the step workspace for the dense layers outside capture
        ctl.set_page_budget(dense_budget)
        ctl._ensure_step_workspace()
    ctl.set_page_budget(sparse_budget)

    def attention(layer):
        ctl.set_page_budget(dense_budget if layer < 2 else sparse_budget)
        ctl.decode_step(q_buf[layer], k_buf[layer], v_buf[layer], layer, out=o_buf[layer])

    def token_step():
        x = emb[token]  # [1, HID]
        for layer, lw in enumerate(layers):
            h = rmsnorm(x, lw["ln1"])
            q_buf[layer].copy_((h @ lw["wq"]).view(1, H, D))
            k_buf[layer].copy_((h @ lw["wk"]).view(1, H, D))
            v_buf[layer].copy_((h @ lw["wv"]).view(1, H, D))
            # RoPE at the new token's position (this library's kernel)
            ak.apply_rope_in_place(q_buf[layer], k_buf[layer], S - 1)
            attention(layer)
            x = x + o_buf[layer].view(1, HID) @ lw["wo"]
            h = rmsnorm(x, lw["ln2"])
            x = x + (torch.nn.functional.silu(h @ lw["wg"]) * (h @ lw["wu"])) @ lw["wd"]
        logits = rmsnorm(x, norm_f) @ lm_head
        token.copy_(logits.argmax(dim=-1))

    def attention_only():
        for layer in range(L):
            attention(layer)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        token_step()
        attention_only()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g_tok, g_att = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_tok):
        token_step()
    with torch.cuda.graph(g_att):
        attention_only()

    def timed(graph):
        for _ in range(a.warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps

    ms_tok = timed(g_tok)
    ms_att = timed(g_att)
    ak.check_device()
    print(json.dumps({
        "metric": MODEL_METRIC, "value": round(ms_tok, 4), "unit": "ms", "n_gpus": 1,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_tok, 4),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": f"Llama-2-7B-shaped decode, random weights, ctx {S}, "
                               f"budget {a.budget}, layers 0-1 dense",
                   "weight_bytes": weight_bytes, "context_tokens": S, "token_budget": a.budget},
        "attention_ms_per_token": round(ms_att, 4),
        "attention_share": round(ms_att / ms_tok, 4),
        "weights_ideal_ms": round(weight_bytes / (6452.2e9) * 1e3, 4),
    }), flush=True)
    del g_tok, g_att


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    elif a.mode == "longctx":
        run_longctx(a)
    elif a.mode == "batched":
        run_batched(a)
    elif a.mode == "model":
        run_model(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
