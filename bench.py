#!/usr/bin/env python
"""Headline benchmark: sparse-decode µs/layer @ 32K context, 1K budget.

Workload (the headline "32K ctx, B=1024" configuration with outlier-key
inputs): one request, 32 heads MHA, head_dim 128, fp16 paged KV with
page_size 16, context 32768 tokens (N = 2048 pages, the new token included),
budget 1024 tokens (64 pages: 63 selected + the last page), AOA-KV
value-aware scoring; K ~ N(0,1) * LogNormal(0,1) per-channel scale, q, V ~
N(0,1), seed 1; synthetic data.

A "step" is one decode token through L = 32 layers (each layer has its own
KV cache, metadata and v_log_norm): per layer the library appends the token
and runs estimate -> top-k -> sparse decode (one launch per layer). The 32
layers touch 32 x 50.5 MB > L2 (126 MB) per step, so no layer finds its data
in L2.

  value     device time per layer-step of one request on one GPU: the
            max-over-ranks time of K CUDA-graph replays of the 32-layer step
            / (K * 32). With --gpus N every GPU serves its own request (N
            replicas, no collective), so the value is per GPU ("weak").
  e2e       the same through InferenceController.decode_step, with the
            step's q, k, v copied from pinned host memory and its outputs
            copied back inside the timed region, no graph
  roofline  the step kernel: algorithmic bytes of a layer-step / its
            average duration inside the timed graph

Extra keys of the same line (each its own workload; see their "config"):
  longctx           config 5: ONE 131072-token request (budget 4096) split
                    by page range over the job's N GPUs (strong scaling),
                    two all_gathers per layer; at N = 1 the plain step
  batched           config 4: 32 requests of 4K-16K tokens balanced over the
                    GPUs by bytes, one launch per layer per GPU (strong)
  prefill_metadata  config 5's prefill: KV pages + key max/min + v_log_norm
                    for 131071 tokens in one pass (N = 1 only)
  config2           config 2 at 8192 tokens: each kernel alone and the step
                    as one launch and as the chain (N = 1 only)
  config3           config 3: a 32-layer Llama-2-7B-shaped decode token,
                    contexts 16K/32K x budgets 512-4096, attention share
                    (N = 1 only; --mode model prints it as its own line)
  gqa               the GQA step (32 query / 8 KV heads) at the headline's
                    context and budget (N = 1 only)
--impl reference times the reference's CPU simulation path (the numpy port
in oracle/sim.py of filter_util.py + quest_attention.py) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
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
H, D, P = 32, 128, 16
# DRAM bytes (read + write) of one cluster step launch at the headline shape:
# dram__bytes_read.sum + dram__bytes_write.sum from the ncu capture
# summarised in profiles/cluster_step_32k.md (not measured in this run)
STEP_TRAFFIC_BYTES = 57_103_000
STEP_TRAFFIC_SOURCE = "profiles/cluster_step_32k.md (ncu, not measured in this run)"


def parse():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["headline", "longctx", "batched", "model", "kernels"],
                    default="headline",
                    help="headline (default): the headline line with every extra key; "
                         "longctx / batched: that key alone; model: config 3; kernels: each "
                         "kernel of one headline layer alone, L2 flushed before every launch "
                         "(the workload of the per-kernel ncu summaries)")
    ap.add_argument("--extras",
                    default="longctx,batched,prefill_metadata,config2,config3,gqa,prefill_attn",
                    help="comma list of extra keys for the headline line ('' = none)")
    ap.add_argument("--layers", type=int, default=32, help="headline layers per step")
    ap.add_argument("--ctx", type=int, default=32768, help="headline context tokens")
    ap.add_argument("--budget", type=int, default=1024, help="headline token budget")
    ap.add_argument("--method", choices=["aoakv", "quest"], default="aoakv")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--long-ctx", type=int, default=131072)
    ap.add_argument("--long-budget", type=int, default=4096)
    ap.add_argument("--extra-layers", type=int, default=4,
                    help="layers per step of the longctx and batched keys")
    ap.add_argument("--requests", type=int, default=32, help="batched: requests")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="CPU-baseline sample budget (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--soak-seconds", type=float, default=1.0,
                    help="graph replays before the timed region so the clock sampler sees load")
    return ap.parse_args()


# ------------------------------------------------------------- plumbing
def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init_gpu(world, local):
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return dev


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_ints(vals, world, dev):
    """Every rank's list of ints (same length on every rank), rank order."""
    import torch
    t = torch.tensor(vals, device=dev, dtype=torch.int64)
    if world == 1:
        return [list(map(int, t.tolist()))]
    import torch.distributed as dist
    out = torch.empty(world * t.numel(), device=dev, dtype=torch.int64)
    dist.all_gather_into_tensor(out, t)
    return [list(map(int, r)) for r in out.view(world, -1).tolist()]


def time_replays(run, steps, warmup, world, dev) -> float:
    """ms of `steps` calls of run() on the current stream, CUDA events, after
    `warmup` calls, barrier + synchronize on both sides, max over ranks."""
    import torch
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1), world, dev)


def capture(fn, dev):
    """fn() once eagerly on a side stream (attributes and workspaces outside
    capture), then a CUDA graph of it."""
    import torch
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def load_peak():
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        peaks = {}
    if peaks.get("hbm_gbs"):
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback"


def roof(bytes_, us, peak, n_gpus=1):
    ach = bytes_ / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(ach, 1), "peak": round(peak * n_gpus, 1),
            "unit": "GB/s", "frac": round(ach / (peak * n_gpus), 4), "algorithmic_bytes": bytes_}


def lib_md5() -> str:
    """md5 of the loaded libaoakv.so (the reference's latency CSV records the
    kernel build per row the same way, bench_latency.py:42-46)."""
    import hashlib
    from aoa_kv_b200 import _lib
    try:
        return hashlib.md5(Path(_lib.LIB_PATH).read_bytes()).hexdigest()
    except OSError:
        return "unknown"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def step_bytes(ctx, budget, method="aoakv") -> int:
    """Algorithmic bytes of one layer-step: metadata (key max and min rows)
    of the N-1 scored pages, their v_log_norm (aoakv), the k attended pages'
    K and V, and q + o."""
    from aoa_kv_b200.batching import step_bytes as sb
    return sb(ctx, budget, H, D, P, method)


def estimate_bytes(ctx, method="aoakv") -> int:
    """Algorithmic bytes of one estimate launch: metadata + v_log_norm of the
    N-1 scored pages, q, and the fp32 scores written."""
    n = (ctx + P - 1) // P
    b = (n - 1) * H * 2 * D * 2 + H * D * 2 + (n - 1) * H * 4
    if method == "aoakv":
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


def reference_timing_here():
    """The reference's own filter_util.py step timed beside the port on the
    machine that has the reference checkout (tests/golden/time_cpu_reference.py)."""
    try:
        return json.loads((ROOT / "tests" / "golden" / "cpu_reference_timing.json").read_text())
    except (OSError, ValueError):
        return None


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


def cpu_baseline_entry(times, a):
    """The port's median step, and the same scaled by the filter_util / port
    ratio measured where the reference checkout exists (the reference
    itself cannot run here)."""
    us = statistics.median(times) * 1e6
    rt = reference_timing_here()
    ratio = rt["filter_util_over_port"] if rt else None
    return us, {
        "value": round(us * ratio if ratio else us, 1), "unit": "us", "cores": cpu_threads(),
        "cpu_model": cpu_model(), "kind": "port",
        "port_measured_us": round(us, 1),
        "filter_util_over_port": ratio,
        "filter_util_over_port_measured_on": rt and f"{rt['cpu_model']}, {rt['threads']} threads",
        "sample": f"{len(times)} single-layer decode steps of the reference simulation restated "
                  f"in oracle/sim.py (filter_util.py + quest_attention.py decode branch) at ctx "
                  f"{a.ctx}, budget {a.budget}, {a.method}, fixed=True (pages 0 and N-1 forced); "
                  f"median" + ("; value = port median x filter_util/port ratio" if ratio else ""),
    }


def run_reference(a):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    for _ in range(max(0, min(a.warmup, 3))):
        cpu_sim_steps(a, 1)
    times = cpu_sim_steps(a, a.steps)
    _, cpu = cpu_baseline_entry(times, a)
    us = cpu["value"]
    cfg = workload_config(a, world)
    cfg["sink_first_page"] = True  # the simulation's fixed=True
    cfg["parallelism"] = "host cores of rank 0's node (per-replica latency, not divided by N)"
    line = {
        "metric": METRIC, "value": us, "unit": "us", "impl": "reference",
        "n_gpus": world, "steps": len(times), "warmup": a.warmup,
        "ms_per_step": round(us / 1e3, 3), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
        "cpu_baseline": cpu,
        "e2e": {"value": us, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- headline
def workload_config(a, n_gpus):
    n_pages = (a.ctx + P - 1) // P
    return {
        "workload": f"1 request per GPU, {a.layers}-layer decode step, ctx {a.ctx}, "
                    f"budget {a.budget}",
        "context_tokens": a.ctx, "token_budget": a.budget, "page_size": P, "num_heads": H,
        "head_dim": D, "layers_per_step": a.layers, "score_mode": a.method,
        "sink_first_page": False, "pages_scored": n_pages - 1,
        "pages_attended": min(a.budget // P, n_pages),
        "inputs": "K~N(0,1)*LogNormal(0,1)[h,d], q,V~N(0,1), seed %d" % a.seed,
        "l2": "inputs larger than L2: %d layers x %.1f MB touched per step" % (
            a.layers, step_bytes(a.ctx, a.budget, a.method) / 1e6),
        "accumulate": "fp32",
        "parallelism": f"{n_gpus} replica(s), one request per GPU, no collective; value is "
                       f"per GPU (max over ranks), not divided by the GPU count",
    }


def setup_layers(ctx, layers, budget, seed, method, dev, outlier=True, spare_tokens=P):
    """An InferenceController holding `layers` layers of ctx-1 cached tokens,
    ready for the decode step of token ctx, with room for spare_tokens more;
    returns (ctl, [(q, k, v)])."""
    import torch

    import aoa_kv_b200 as ak
    gen = torch.Generator(device=dev).manual_seed(seed)
    ctl = ak.InferenceController(layers, H, D, P, budget // P, ctx + spare_tokens, torch.float16,
                                 dev, method=method)
    ctl.prepare_metadata(ctx - 1)
    ctl.begin_forward(ctx - 1)
    news = []
    for layer in range(layers):
        scale = torch.exp(torch.randn(H, D, device=dev, generator=gen)) if outlier else 1.0
        K = (torch.randn(ctx, H, D, device=dev, generator=gen) * scale).half()
        V = torch.randn(ctx, H, D, device=dev, generator=gen).half()
        q = torch.randn(1, H, D, device=dev, generator=gen).half()
        ak.append_kv(K[:-1].contiguous(), V[:-1].contiguous(), ctl, layer)
        news.append((q, K[-1:].contiguous(), V[-1:].contiguous()))
        del K, V
    ctl.end_forward()
    ctl.prepare_metadata(1)
    ctl.begin_forward(1)
    torch.cuda.synchronize()
    return ctl, news


def graph_token_e2e(a, ctl, pin_qkv, world, dev):
    """The decode loop through the device-resident page table: per token one
    H2D copy of every layer's q/k/v (pinned), one CUDA graph replay (device
    page-table append of the token + the 32 layers' aoakv_decode_step_table)
    and one D2H copy of every layer's output. The sequence really grows by one
    token per replay (the headline replays the same token); the page table is
    built over the headline's caches (a fresh device pool hands out the same
    page ids as the host pool did)."""
    import torch

    import aoa_kv_b200 as ak
    kv0, meta0 = ctl.kv_cache.buf_layer(0), ctl.metadata_cache.buf_layer(0)
    pt = ak.DevicePageTable(1, kv0.shape[0], kv0.shape[0], meta0.shape[0], P, dev)
    pt.append(a.ctx - 1)
    n = (a.ctx - 1 + P - 1) // P
    same = bool(torch.equal(pt.kv_indices(0)[:n], ctl.kv_indices_with_last[:n]))
    dev_qkv = torch.empty_like(pin_qkv, device=dev)  # [L, 3, 1, H, D]
    o_all = torch.empty(a.layers, 1, H, D, dtype=torch.float16, device=dev)
    host_o = torch.empty(a.layers, 1, H, D, dtype=torch.float16).pin_memory()
    dev_qkv.copy_(pin_qkv)

    def token():
        pt.append(1)
        for layer in range(a.layers):
            pt.decode_step(dev_qkv[layer, 0], dev_qkv[layer, 1], dev_qkv[layer, 2], o_all[layer],
                           ctl.kv_cache.buf_layer(layer), ctl.metadata_cache.buf_layer(layer),
                           ctl.v_log_norm_layer(layer), a.budget // P, ctl.score_mode, False)
    token()  # once outside capture (kernel attributes)
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        g.capture_begin()
        token()
        g.capture_end()
    torch.cuda.current_stream().wait_stream(side)

    def step():
        dev_qkv.copy_(pin_qkv, non_blocking=True)
        g.replay()
        host_o.copy_(o_all, non_blocking=True)
    ems = time_replays(step, a.steps, a.warmup, world, dev)
    dms = time_replays(g.replay, a.steps, 0, world, dev)
    ak.check_device()
    tokens = 1 + a.warmup + 2 * a.steps
    del g
    pt.close()
    return {"value": round(ems * 1e3 / (a.steps * a.layers), 3), "unit": "us",
            "device_only_us": round(dms * 1e3 / (a.steps * a.layers), 3),
            "h2d_bytes_per_step": a.layers * 3 * H * D * 2,
            "d2h_bytes_per_step": a.layers * H * D * 2,
            "context_tokens": f"{a.ctx} .. {a.ctx + tokens - 1} (one more per replay)",
            "page_ids_match_host_pool": same,
            "gpu_launches": (1 + a.layers) * a.steps,
            "api": "DevicePageTable (aoakv_page_table_append + aoakv_decode_step_table per "
                   "layer) captured once as a CUDA graph of the whole token; per token one H2D "
                   "of all layers' q/k/v, one replay, one D2H of all outputs"}


def run_headline(a):
    import ctypes

    import torch

    import aoa_kv_b200 as ak
    world, rank, local = dist_env()
    dev = init_gpu(world, local)
    ak._lib.load()
    peak, peak_src = load_peak()

    ctl, news = setup_layers(a.ctx, a.layers, a.budget, a.seed, a.method, dev, spare_tokens=256)
    outs = [torch.empty(1, H, D, dtype=torch.float16, device=dev) for _ in range(a.layers)]
    nk, ncl = ctypes.c_int32(0), ctypes.c_int32(0)
    ak._lib.call("aoakv_step_plan_info", ctl.step_plan(0)._h, len(ctl.kv_cache.indicies), 0,
                 ctypes.byref(nk), ctypes.byref(ncl))
    kernels_per_layer, cluster = int(nk.value), int(ncl.value)

    def one_step():
        for layer, (q, k, v) in enumerate(news):
            ctl.decode_step(q, k, v, layer, out=outs[layer])

    graph = capture(one_step, dev)
    ak.check_device()

    sampler = ClockSampler(gpu_query_id(local)) if rank == 0 else None
    t_soak = time.monotonic()
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()
    t_end = time.monotonic() + a.soak_seconds  # let the clock sampler see the load
    while time.monotonic() < t_end:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize()
    ms = time_replays(graph.replay, a.steps, 0, world, dev)
    t_timed_end = time.monotonic()
    ak.check_device()
    us_layer = ms * 1e3 / (a.steps * a.layers)

    # the page scorer alone (fp32 scores), the same layers
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
    g_est = capture(est_all, dev)
    est_us = time_replays(g_est.replay, max(5, a.steps // 2), 3, world, dev) * 1e3 / (
        max(5, a.steps // 2) * a.layers)

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
        ems = time_replays(e2e_step, a.steps, a.warmup, world, dev)
        e2e = {"value": round(ems * 1e3 / (a.steps * a.layers), 3), "unit": "us",
               "h2d_bytes_per_step": a.layers * 3 * H * D * 2,
               "d2h_bytes_per_step": a.layers * H * D * 2,
               "api": "InferenceController.decode_step per layer (ctypes -> "
                      "aoakv_step_plan_run); one H2D of the step's q/k/v and one D2H of its "
                      "outputs; no graph; per GPU"}

    e2e_graph = None
    if not a.no_e2e:
        e2e_graph = graph_token_e2e(a, ctl, pin_qkv, world, dev)

    if sampler:
        sampler.stop()
    clocks = sampler.summary(t_soak, t_timed_end) if sampler else None

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        _, cpu = cpu_baseline_entry(cpu_sim_steps(a, 50, budget_s=a.cpu_seconds), a)

    sb = step_bytes(a.ctx, a.budget, a.method)
    eb = estimate_bytes(a.ctx, a.method)
    r = roof(sb, us_layer, peak)
    r.update({"kernel": (f"cluster_step_kernel<{D},{cluster}> (append+estimate+top-k+decode, "
                         f"one launch)") if kernels_per_layer == 1 else
              f"step chain of {kernels_per_layer} kernels",
              "traffic": STEP_TRAFFIC_BYTES, "traffic_source": STEP_TRAFFIC_SOURCE,
              "avg_launch_us": round(us_layer, 3),
              "ideal_us": round(sb / (peak * 1e9) * 1e6, 3), "peak_source": peak_src,
              "timing": "CUDA events around K graph replays of the 32-layer step on the "
                        "launching stream; avg launch = time / (K * layers), gaps included"})
    er = roof(eb, est_us, peak)
    er.update({"kernel": "estimate_attn_score alone (page scorer)",
               "avg_launch_us": round(est_us, 3)})
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(us_layer, 3), "unit": "us", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": workload_config(a, world),
            "roofline": r, "estimate_roofline": er,
            "e2e": e2e, "e2e_graph_token": e2e_graph,
            "gpu_launches": kernels_per_layer * a.layers * a.steps,
            "step_kernels_per_layer": kernels_per_layer, "clocks": clocks,
            "library_md5": lib_md5(), "cpu_baseline": cpu,
        }
    del graph, g_est
    ctl.clean_states()
    del ctl, news, outs
    torch.cuda.empty_cache()

    extras = [x for x in a.extras.split(",") if x]
    for key in extras:
        fn = {"longctx": longctx_key, "batched": batched_key,
              "prefill_metadata": prefill_key, "config2": config2_key,
              "config3": lambda *x: model_key(*x, steps=5, warmup=2), "gqa": gqa_key,
              "prefill_attn": prefill_attn_key}.get(key)
        if fn is None:
            raise SystemExit(f"unknown extra key {key!r}")
        if key in ("prefill_metadata", "config2", "config3", "gqa", "prefill_attn") and world > 1:
            continue  # single-GPU workloads: reported at N = 1
        val = fn(a, world, rank, dev, peak)
        if line is not None:
            line[key] = val
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(line), flush=True)
    finish(world)


def finish(world):
    import gc

    import torch
    gc.collect()  # graphs that hold NCCL calls go before the process group
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------ long context, sharded
def _prefill(K, V, t0, t1, kv, kv_idx, meta, meta_idx, vlog, stream):
    """Tokens [t0, t1) of K, V [S, H, D] into pages 0.. of the given tables."""
    from aoa_kv_b200 import _lib
    n_tok = t1 - t0
    if n_tok <= 0:
        return
    n_pref = -(-n_tok // P)
    _lib.call("aoakv_append_kv_cache_prefill", K[t0:t1].data_ptr(), V[t0:t1].data_ptr(), n_tok,
              kv.data_ptr(), kv_idx.data_ptr(), n_pref, (n_tok - 1) % P + 1, kv.shape[0],
              meta.data_ptr(), meta_idx.data_ptr(), -(-n_pref // P), (n_pref - 1) % P + 1,
              meta.shape[0], vlog.data_ptr(), H, D, P, _lib.LAYOUT_NHD, stream)


def _pool(n_pages, dev):
    import torch
    cap = n_pages + 1
    mcap = -(-cap // P)
    kv = torch.empty(cap, 2, P, H, D, dtype=torch.float16, device=dev)
    meta = torch.empty(mcap, 2, P, H, D, dtype=torch.float16, device=dev)
    vlog = torch.zeros(cap, H, dtype=torch.float16, device=dev)
    kv_idx = torch.arange(n_pages, dtype=torch.int32, device=dev)
    meta_idx = torch.arange(mcap, dtype=torch.int32, device=dev)
    return kv, meta, vlog, kv_idx, meta_idx


def longctx_key(a, world, rank, dev, peak):
    """Config 5: one request of a.long_ctx tokens (the new one included),
    budget a.long_budget, q, K, V ~ N(0,1) (seed 4). N = 1: the plain step
    (StepPlan, one launch per layer), cross-checked against the sharded
    decoder run on one rank. N > 1: the page range is split over the ranks
    (aoa_kv_b200.sharded: local top-k, all_gather of candidates, global
    top-k, partial decode of the owned pages, all_gather of partial states,
    LSE merge), cross-checked on rank 0 against the plain step over the
    whole sequence."""
    import torch

    from aoa_kv_b200 import StepPlan, _lib, sharded
    S, budget, L = a.long_ctx, a.long_budget, a.extra_layers
    n_total, last_len = -(-S // P), (S - 1) % P + 1
    lo, hi = sharded.partition_pages(n_total, world, P)[rank]
    n_local, owns = hi - lo, rank == world - 1
    stream = torch.cuda.current_stream().cuda_stream
    kpages = budget // P
    layers, news, full0 = [], [], None
    for layer in range(L):
        g = torch.Generator(device=dev).manual_seed(4000 + layer)
        K = torch.randn(S, H, D, device=dev, generator=g).half()
        V = torch.randn(S, H, D, device=dev, generator=g).half()
        q = torch.randn(H, D, device=dev, generator=g).half()
        news.append((q, K[S - 1].clone(), V[S - 1].clone()))
        kv, meta, vlog, kv_idx, meta_idx = _pool(n_local, dev)
        _prefill(K, V, lo * P, min(hi * P, S - 1), kv, kv_idx, meta, meta_idx, vlog, stream)
        layers.append(sharded.ShardLayer(kv=kv, meta=meta, vlog=vlog, kv_idx=kv_idx,
                                         meta_idx=meta_idx, page_lo=lo, n_local=n_local,
                                         n_total=n_total, last_len=last_len, owns_last=owns,
                                         last_phys=n_local - 1 if owns else -1))
        if layer == 0 and rank == 0 and world > 1:  # the whole sequence, for the check
            full0 = _pool(n_total, dev)
            _prefill(K, V, 0, S - 1, full0[0], full0[3], full0[1], full0[4], full0[2], stream)
        del K, V
    torch.cuda.synchronize()
    mode = _lib.SCORE_AOAKV if a.method == "aoakv" else _lib.SCORE_QUEST
    o = torch.empty(L, H, D, dtype=torch.float16, device=dev)
    sel = torch.empty(L, H, kpages, dtype=torch.int32, device=dev)
    # the step's workspace (used only if a plan runs the four-kernel chain)
    ws = torch.zeros(_lib.size_query("aoakv_step_workspace_size", H, D, n_total, kpages),
                     dtype=torch.uint8, device=dev)
    if world == 1:
        plans = [StepPlan(lay.kv, lay.kv.shape[0], lay.meta, lay.meta.shape[0], lay.vlog, H, D, P,
                          kpages, mode, max_pages=n_total) for lay in layers]

        def one_step():
            for i, (lay, (q, k, v)) in enumerate(zip(layers, news)):
                plans[i].run(q, k, v, o[i], lay.kv_idx, n_total, last_len, lay.meta_idx,
                             None, ws, ws.numel(), torch.cuda.current_stream().cuda_stream)
        launches = plans[0].info(n_total)[0] * L
    steps = max(10, a.steps // 2)
    nccl_us = None
    if world == 1:
        graph = capture(one_step, dev)
        ms = time_replays(graph.replay, steps, a.warmup, world, dev)
    else:
        # both exchanges, the same data: NCCL all_gathers, then the kernels'
        # own peer stores (the value)
        for exchange in ("nccl", "p2p"):
            dec = sharded.ShardedDecoder(torch.distributed.group.WORLD, H, D, P, kpages,
                                         a.method, exchange=exchange, device=dev)

            def one_step():
                for i, (lay, (q, k, v)) in enumerate(zip(layers, news)):
                    o[i].copy_(dec.step(lay, q, k, v)[0])
            graph = capture(one_step, dev)
            ms = time_replays(graph.replay, steps, a.warmup, world, dev)
            if exchange == "nccl":
                nccl_us = ms * 1e3 / (steps * L)
                del graph
        launches = 3 * L
    _lib.check_device()
    us = ms * 1e3 / (steps * L)

    # check (layer 0): the other implementation on the same data
    err, sel_equal = None, None
    if world == 1:
        plans[0].run(news[0][0], news[0][1], news[0][2], o[0], layers[0].kv_idx, n_total,
                     last_len, layers[0].meta_idx, sel[0], ws, ws.numel(), stream)
        dec = sharded.ShardedDecoder(_SoloGroup(), H, D, P, kpages, a.method)
        o_x, sel_x = dec.step(layers[0], *news[0])
        torch.cuda.synchronize()
        err = float((o[0].float() - o_x.float()).abs().max())
        mine = torch.sort(sel[0][:, :kpages - 1], dim=1).values
        sel_equal = bool(torch.equal(mine, torch.sort(sel_x, dim=1).values))
        sel_global = sel[0][:, :kpages - 1]
    else:
        o_s, sel_s = dec.step(layers[0], *news[0])
        torch.cuda.synchronize()
        sel_global = sel_s
        if rank == 0:
            kv, meta, vlog, kv_idx, meta_idx = full0
            ref_plan = StepPlan(kv, kv.shape[0], meta, meta.shape[0], vlog, H, D, P, kpages, mode,
                                max_pages=n_total)
            o_ref = torch.empty(H, D, dtype=torch.float16, device=dev)
            sel_ref = torch.empty(H, kpages, dtype=torch.int32, device=dev)
            ref_plan.run(news[0][0], news[0][1], news[0][2], o_ref, kv_idx, n_total, last_len,
                         meta_idx, sel_ref, ws, ws.numel(), stream)
            torch.cuda.synchronize()
            err = float((o_s.float() - o_ref.float()).abs().max())
            sel_equal = bool(torch.equal(torch.sort(sel_ref[:, :kpages - 1], dim=1).values,
                                         torch.sort(sel_s, dim=1).values))
            del ref_plan
    # per-GPU algorithmic bytes of a layer-step: this rank's scored pages'
    # metadata (+ v_log_norm), its attended pages' K and V, q and o
    n_score = n_local - (1 if owns else 0)
    in_mine = ((sel_global >= lo) & (sel_global < hi)).sum().item() + (H if owns else 0)
    row = 2 * D * 2 + (2 if a.method == "aoakv" else 0)
    mine_bytes = n_score * H * row + in_mine * P * D * 2 * 2 + 2 * H * D * 2
    got = gather_ints([mine_bytes, in_mine], world, dev)
    per_gpu, pages_dec = [r[0] for r in got], [r[1] for r in got]
    del graph
    torch.cuda.synchronize()
    if world > 1 and dec.mailbox is not None:  # every rank past its last pass first
        barrier(world)
        dec.mailbox.close()
    if rank != 0:
        return None
    total = sum(per_gpu)
    out = {
        "metric": "sparse-decode µs/layer @128K ctx, 4K budget (config 5)",
        "value": round(us, 3), "unit": "us", "n_gpus": world, "scaling": "strong",
        "steps": steps, "layers_per_step": L,
        "roofline": roof(total, us, peak, world),
        "max_gpu_bytes": max(per_gpu), "per_gpu_bytes": per_gpu,
        "decode_head_pages_per_gpu": pages_dec,
        "max_abs_err": err, "selection_equal": sel_equal,
        "nccl_exchange_us": None if nccl_us is None else round(nccl_us, 3),
        "checked_against": ("the sharded decoder run as one rank (propose and finish passes, "
                            "packed merge) on the same data, layer 0" if world == 1 else
                            "the one-GPU step over the whole sequence on rank 0, layer 0"),
        "config": {"workload": f"1 request, ctx {S} (new token included), budget {budget}, "
                               f"{L}-layer step, q,K,V~N(0,1) seed 4",
                   "pages": n_total, "pages_per_gpu": n_local,
                   "parallelism": "1 GPU, one step launch per layer" if world == 1 else
                   f"page range x{world}; per layer: propose launch (stores its "
                   f"{H}x{kpages - 1}x8 B of candidates into every GPU's mailbox over NVLink), "
                   f"finish launch (waits for every GPU's flag; stores its {H}x{D + 1}x4 B "
                   f"partial state the same way), merge launch; no collective; one CUDA "
                   f"graph. nccl_exchange_us: the same with two NCCL all_gathers instead"},
    }
    if launches is not None:
        out["gpu_launches"] = launches * steps
    return out


class _SoloGroup:
    """The all_gather of a one-rank job."""

    @staticmethod
    def all_gather_stack(t):
        return t.unsqueeze(0)


# ------------------------------------------------------ batched decode
def batched_key(a, world, rank, dev, peak):
    """Config 4: a.requests requests, context U[4096, 16384] tokens in whole
    pages (seed 3), budget a.budget, balanced over the GPUs by bytes
    (aoa_kv_b200.batching); each GPU keeps its requests in one pool per
    layer and runs ONE aoakv_decode_step_batched launch per layer. No
    collective; fixed total work: strong scaling. Checked on rank 0 against
    one StepPlan run per request (layer 0)."""
    import numpy as np
    import torch

    from aoa_kv_b200 import StepPlan, _lib, batching
    L = a.extra_layers
    g = np.random.default_rng(3)
    ctxs = [int(c) * P for c in g.integers(4096 // P, 16384 // P + 1, size=a.requests)]
    weights = [batching.step_bytes(c, a.budget, H, D, P, a.method) for c in ctxs]
    mine = batching.balance_requests(weights, world)[rank]
    R = len(mine)
    pages = [-(-ctxs[r] // P) for r in mine]
    n_all = sum(pages)
    kv_indptr = np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)
    mp = [-(-n // P) for n in pages]
    meta_indptr = np.concatenate([[0], np.cumsum(mp)]).astype(np.int32)
    last = np.array([(ctxs[r] - 1) % P + 1 for r in mine], np.int32)
    stream = torch.cuda.current_stream().cuda_stream

    def dev_i32(x):
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.int32)).to(dev)
    kv_indptr_d, meta_indptr_d, last_d = dev_i32(kv_indptr), dev_i32(meta_indptr), dev_i32(last)
    kv_tab = torch.arange(n_all, dtype=torch.int32, device=dev)
    meta_tab = torch.arange(int(meta_indptr[-1]), dtype=torch.int32, device=dev)
    pools, qkv = [], []
    for layer in range(L):
        kv = torch.empty(n_all + 1, 2, P, H, D, dtype=torch.float16, device=dev)
        meta = torch.empty(int(meta_indptr[-1]) + 1, 2, P, H, D, dtype=torch.float16, device=dev)
        vlog = torch.zeros(n_all + 1, H, dtype=torch.float16, device=dev)
        q_l = torch.empty(R, H, D, dtype=torch.float16, device=dev)
        k_l, v_l = torch.empty_like(q_l), torch.empty_like(q_l)
        for i, r in enumerate(mine):
            gen = torch.Generator(device=dev).manual_seed(3000 + 100 * r + layer)
            S = ctxs[r]
            scale = torch.exp(torch.randn(H, D, device=dev, generator=gen))
            K = (torch.randn(S, H, D, device=dev, generator=gen) * scale).half()
            V = torch.randn(S, H, D, device=dev, generator=gen).half()
            q_l[i] = torch.randn(H, D, device=dev, generator=gen).half()
            k_l[i], v_l[i] = K[S - 1], V[S - 1]
            p0, m0 = int(kv_indptr[i]), int(meta_indptr[i])
            _prefill(K, V, 0, S - 1, kv, kv_tab[p0:], meta, meta_tab[m0:], vlog, stream)
            del K, V
        pools.append((kv, meta, vlog))
        qkv.append((q_l, k_l, v_l))
    torch.cuda.synchronize()
    o = torch.empty(L, R, H, D, dtype=torch.float16, device=dev)
    max_pages = max(pages) if pages else 1

    def one_step():
        for layer in range(L):
            kv, meta, vlog = pools[layer]
            q_l, k_l, v_l = qkv[layer]
            batching.decode_step_batched(q_l, k_l, v_l, o[layer], kv, kv_indptr_d, kv_tab, last_d,
                                         meta, meta_indptr_d, meta_tab, vlog, max_pages,
                                         a.budget // P, a.method)
    ms = 0.0
    steps = max(10, a.steps // 2)
    graph = None
    if R:
        graph = capture(one_step, dev)
        ms = time_replays(graph.replay, steps, a.warmup, world, dev)
    else:
        ms = time_replays(lambda: None, steps, 0, world, dev)
    _lib.check_device()
    us = ms * 1e3 / (steps * L)
    err = None
    if rank == 0 and R:
        kv, meta, vlog = pools[0]
        q_l, k_l, v_l = qkv[0]
        o_one = torch.empty(H, D, dtype=torch.float16, device=dev)
        mode = _lib.SCORE_AOAKV if a.method == "aoakv" else _lib.SCORE_QUEST
        plan = StepPlan(kv, kv.shape[0], meta, meta.shape[0], vlog, H, D, P, a.budget // P, mode,
                        max_pages=max_pages)
        err = 0.0
        for i in range(R):
            p0, m0 = int(kv_indptr[i]), int(meta_indptr[i])
            plan.run(q_l[i], k_l[i], v_l[i], o_one, kv_tab[p0:].data_ptr(), pages[i],
                     int(last[i]), meta_tab[m0:].data_ptr(), None, None, 0, stream)
            torch.cuda.synchronize()
            err = max(err, float((o_one.float() - o[0, i].float()).abs().max()))
        plan.close()
    mine_bytes = sum(weights[r] for r in mine)
    got = gather_ints([mine_bytes, R], world, dev)
    per_gpu, per_req = [x[0] for x in got], [x[1] for x in got]
    del graph
    torch.cuda.synchronize()
    if rank != 0:
        return None
    total = sum(weights)
    return {
        "metric": f"sparse-decode µs/layer for a batch of {a.requests} requests (4K-16K ctx, "
                  f"{a.budget} budget) (config 4)",
        "value": round(us, 3), "unit": "us", "n_gpus": world, "scaling": "strong",
        "steps": steps, "layers_per_step": L,
        "roofline": roof(total, us, peak, world),
        "max_gpu_bytes": max(per_gpu), "per_gpu_bytes": per_gpu, "requests_per_gpu": per_req,
        "max_abs_err": err,
        "checked_against": "one StepPlan step per request on the same pool (layer 0, rank 0)",
        "gpu_launches": L * steps,
        "config": {"workload": f"{a.requests} requests, ctx U[4096,16384] tokens in whole pages "
                               f"(seed 3), budget {a.budget}, {L}-layer step, outlier K",
                   "bytes_per_layer_step": total,
                   "parallelism": f"request-sharded x{world} (greedy byte balance), no "
                                  f"collective; one batched launch per layer per GPU"},
    }


# ------------------------------------------------- config 5 prefill build
def gqa_key(a, world, rank, dev, peak):
    """Grouped-query attention (a Llama-3-8B-like layer: 32 query heads over
    8 KV heads, head_dim 128), 32K context, budget 1024, outlier K (seed 1):
    aoakv_decode_step_gqa over 16 layers (16 x 12.6 MB > L2) in a CUDA graph,
    µs per layer-step. Bytes: the KV heads' metadata and K/V, the query
    heads' q and o."""
    import numpy as np
    import torch

    from aoa_kv_b200 import _lib
    Hq, Hk, ctx, budget, L = 32, 8, a.ctx, a.budget, 16
    n = (ctx + P - 1) // P
    kp = budget // P
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=dev).manual_seed(1)
    layers = []
    for _ in range(L):
        cap = n + 1
        kv = torch.empty(cap, 2, P, Hk, D, dtype=torch.float16, device=dev)
        meta = torch.empty(-(-cap // P), 2, P, Hk, D, dtype=torch.float16, device=dev)
        vlog = torch.zeros(cap, Hk, dtype=torch.float16, device=dev)
        idx = torch.arange(cap, dtype=torch.int32, device=dev)
        midx = torch.arange(meta.shape[0], dtype=torch.int32, device=dev)
        scale = torch.exp(torch.randn(Hk, D, device=dev, generator=g))
        K = (torch.randn(ctx, Hk, D, device=dev, generator=g) * scale).half()
        V = torch.randn(ctx, Hk, D, device=dev, generator=g).half()
        q = torch.randn(Hq, D, device=dev, generator=g).half()
        S = ctx - 1
        n0 = -(-S // P)
        _lib.call("aoakv_append_kv_cache_prefill", K.data_ptr(), V.data_ptr(), S, kv.data_ptr(),
                  idx.data_ptr(), n0, (S - 1) % P + 1, cap, meta.data_ptr(), midx.data_ptr(),
                  -(-n0 // P), (n0 - 1) % P + 1, meta.shape[0], vlog.data_ptr(), Hk, D, P, 0,
                  stream)
        layers.append((kv, meta, vlog, idx, midx, q, K[-1].clone(), V[-1].clone(),
                       torch.empty(Hq, D, dtype=torch.float16, device=dev)))
        del K, V
    ws_n = _lib.size_query("aoakv_step_workspace_size", Hq, D, n + 1, kp)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device=dev)
    mode = _lib.SCORE_AOAKV if a.method == "aoakv" else _lib.SCORE_QUEST

    def run():
        st = torch.cuda.current_stream().cuda_stream
        for kv, meta, vlog, idx, midx, q, k, v, o in layers:
            _lib.call("aoakv_decode_step_gqa", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                      o.data_ptr(), kv.data_ptr(), idx.data_ptr(), n, (ctx - 1) % P + 1,
                      kv.shape[0], meta.data_ptr(), midx.data_ptr(), meta.shape[0],
                      vlog.data_ptr(), Hq, Hk, D, P, kp, mode, 0, None, ws.data_ptr(), ws_n, st)
    graph = capture(run, dev)
    steps = max(10, a.steps // 2)
    ms = time_replays(graph.replay, steps, 3, world, dev)
    _lib.check_device()
    us = ms * 1e3 / (steps * L)
    b = ((n - 1) * Hk * (2 * D * 2 + (2 if a.method == "aoakv" else 0)) +
         kp * P * Hk * D * 2 * 2 + 2 * Hq * D * 2)
    del graph, layers
    return {"metric": f"GQA sparse-decode µs/layer @{ctx} ctx, {budget} budget, 32 query / 8 KV "
                      f"heads", "value": round(us, 3), "unit": "us", "roofline": roof(b, us, peak),
            "gpu_launches": 4 * L * steps,
            "config": {"workload": f"{L} layers, Hq 32, Hkv 8, head_dim 128, ctx {ctx}, budget "
                                   f"{budget}, outlier K seed 1; append, group scoring, top-k, "
                                   f"decode (four launches)"}}


def prefill_attn_key(a, world, rank, dev, peak):
    """Prefill attention of config 3's 32K prompt on one layer
    (aoakv_prefill_paged: causal, 32 heads, head_dim 128, page size 16, pages
    in a shuffled page table): ms per layer and TFLOP/s, 4 * D * H * S(S+1)/2
    flops, against the sustained bf16 tensor peak (a ~10 ms kernel). torch's
    scaled_dot_product_attention on the same q/K/V, contiguous, is timed beside
    it for context (a library kernel, not this library's)."""
    import torch

    from aoa_kv_b200 import _lib
    S = 32768
    n_pages = S // P
    cap = n_pages + 4
    g = torch.Generator(device=dev).manual_seed(6)
    kv = torch.randn(cap, 2, P, H, D, device=dev, generator=g).half()
    ids = torch.randperm(cap, device=dev, generator=g)[:n_pages].int()
    q = torch.randn(S, H, D, device=dev, generator=g).half()
    o = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream

    def run():
        _lib.call("aoakv_prefill_paged", q.data_ptr(), o.data_ptr(), None, kv.data_ptr(), cap,
                  ids.data_ptr(), n_pages, P, S, H, H, D, P, 0, 1, 0.0, stream)
    steps = 5
    ms = time_replays(run, steps, 2, world, dev) / steps
    _lib.check_device()
    flops = 4.0 * D * H * S * (S + 1) / 2
    tf = flops / (ms * 1e-3) / 1e12
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tpeak = float(peaks.get("bf16_tflops_sustained") or 1400.0)
    src = ("measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
           if peaks.get("bf16_tflops_sustained") else "fallback 1400 TFLOP/s sustained")
    kt = kv[ids.long(), 0].reshape(S, H, D).transpose(0, 1)[None].contiguous()
    vt = kv[ids.long(), 1].reshape(S, H, D).transpose(0, 1)[None].contiguous()
    qt = q.transpose(0, 1)[None].contiguous()
    sdpa = lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=True)
    ms_t = time_replays(sdpa, steps, 2, world, dev) / steps
    err = float((sdpa().transpose(1, 2)[0] - o).abs().max())
    del kv, kt, vt, qt
    return {"metric": "prefill attention ms/layer @32768 tokens (causal, 32 heads, head_dim 128)",
            "value": round(ms, 3), "unit": "ms", "tflops": round(tf, 1),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": tpeak,
                         "unit": "TFLOP/s", "frac": round(tf / tpeak, 4), "peak_source": src,
                         "flops": flops},
            "gpu_launches": steps,
            "torch_sdpa_ms": round(ms_t, 3), "max_abs_diff_vs_torch_sdpa": round(err, 5),
            "config": {"workload": "one layer, 32768-token causal prefill, q [S, 32, 128] fp16, "
                                   "KV in 16-token pages of a shuffled page table; tcgen05 MMAs, "
                                   "accumulators in tensor memory"}}


def prefill_key(a, world, rank, dev, peak):
    """Config 5's prefill: aoakv_append_kv_cache_prefill of a.long_ctx - 1
    tokens of one layer in one pass (KV pages, key max/min metadata of every
    page, v_log_norm of every full page). Bytes: K and V read and written
    once, the metadata and v_log_norm written."""
    import torch

    from aoa_kv_b200 import _lib
    S = a.long_ctx - 1
    n_pages = -(-S // P)
    g = torch.Generator(device=dev).manual_seed(4)
    K = torch.randn(S, H, D, device=dev, generator=g).half()
    V = torch.randn(S, H, D, device=dev, generator=g).half()
    kv, meta, vlog, kv_idx, meta_idx = _pool(n_pages, dev)

    def run():
        _prefill(K, V, 0, S, kv, kv_idx, meta, meta_idx, vlog,
                 torch.cuda.current_stream().cuda_stream)
    steps = 10
    ms = time_replays(run, steps, 3, world, dev)
    _lib.check_device()
    us = ms * 1e3 / steps
    kvb = S * H * D * 2 * 2
    b = 2 * kvb + n_pages * 2 * H * D * 2 + (S // P) * H * 2
    return {"metric": f"prefill page build µs for {S} tokens (config 5)", "value": round(us, 1),
            "unit": "us", "roofline": roof(b, us, peak), "gpu_launches": steps,
            "config": {"tokens": S, "pages": n_pages,
                       "bytes": "K,V read + KV pages written + key max/min metadata written + "
                                "v_log_norm written",
                       "inputs": "q,K,V~N(0,1) seed 4; 4.4 GB per call > L2"}}


# ------------------------------------------------------ config 2, 8192
def config2_key(a, world, rank, dev, peak):
    """Config 2 at 8192 tokens, budget 1024 (outlier K, seed 1): each kernel
    alone over 8 layers (8 x 25 MB > L2) and the step as one launch and as
    the four-kernel chain, µs per layer."""
    import torch

    from aoa_kv_b200 import StepPlan, _lib
    ctx, budget, L = 8192, 1024, 8
    ctl, news = setup_layers(ctx, L, budget, 1, a.method, dev)
    n = len(ctl.kv_cache.indicies)
    kp = budget // P
    o = torch.empty(L, H, D, dtype=torch.float16, device=dev)
    scores = torch.empty(L, H, n, dtype=torch.float32, device=dev)
    sel = torch.empty(L, H, kp - 1, dtype=torch.int32, device=dev)
    ws_n = _lib.size_query("aoakv_decode_workspace_size", H, D, kp - 1)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device=dev)
    sws = ctl._ensure_step_workspace()
    chain = []
    for layer in range(L):
        kv_p, kv_cap, meta_p, meta_cap, vlog_p = ctl._layer_buffers(layer)
        chain.append(StepPlan(kv_p, kv_cap, meta_p, meta_cap, vlog_p, H, D, P, kp,
                              ctl.score_mode, chain=True))

    def st():
        return torch.cuda.current_stream().cuda_stream

    def k_append():
        for layer, (q, k, v) in enumerate(news):
            kv_p, kv_cap, meta_p, meta_cap, vlog_p = ctl._layer_buffers(layer)
            _lib.call("aoakv_append_kv_cache_decode", k.data_ptr(), v.data_ptr(), kv_p,
                      ctl.kv_indices_with_last.data_ptr(), n, ctl.kv_cache.last_page_len, kv_cap,
                      meta_p, ctl.metadata_indices.data_ptr(), len(ctl.metadata_cache.indicies),
                      ctl.metadata_cache.last_page_len, meta_cap, vlog_p, H, D, P, 0, st())

    def k_estimate():
        for layer, (q, _, _) in enumerate(news):
            kv_p, kv_cap, meta_p, meta_cap, vlog_p = ctl._layer_buffers(layer)
            _lib.call("aoakv_estimate_attn_score", q.data_ptr(), scores[layer].data_ptr(), 1, n,
                      meta_p, ctl.metadata_indices.data_ptr(), len(ctl.metadata_cache.indicies),
                      ctl.metadata_cache.last_page_len, meta_cap,
                      ctl.kv_indices_with_last.data_ptr(), kv_cap, vlog_p, H, D, P, 0,
                      ctl.score_mode, st())

    def k_topk():
        for layer in range(L):
            _lib.call("aoakv_topk_filtering", scores[layer].data_ptr(), 1, n,
                      ctl.kv_indices_with_last.data_ptr(), 0, H, n - 1, kp - 1, None, 0,
                      sel[layer].data_ptr(), kp - 1, 0, st())

    def k_decode():
        for layer, (q, _, _) in enumerate(news):
            kv_p, kv_cap, _, _, _ = ctl._layer_buffers(layer)
            _lib.call("aoakv_sparse_decode", q.data_ptr(), o[layer].data_ptr(), kv_p, kv_cap,
                      sel[layer].data_ptr(), kp - 1, kp - 1, ctl.kv_cache.indicies[-1],
                      ctl.kv_cache.last_page_len, H, D, P, 0, 0.0, ws.data_ptr(), ws_n, st())

    def fused():
        for layer, (q, k, v) in enumerate(news):
            ctl.decode_step(q, k, v, layer, out=o[layer])

    def chained():
        for layer, (q, k, v) in enumerate(news):
            chain[layer].run(q, k, v, o[layer], ctl.kv_indices_with_last, n,
                             ctl.kv_cache.last_page_len, ctl.metadata_indices, None, sws,
                             sws.numel(), st())
    row = 2 * D * 2 + (2 if a.method == "aoakv" else 0)
    parts = {
        "append_decode": (k_append, 2 * H * D * 2 + 2 * H * D * 2 * 2),
        "estimate": (k_estimate, estimate_bytes(ctx, a.method)),
        "topk": (k_topk, H * (n - 1) * 4 + H * (kp - 1) * 4),
        "sparse_decode": (k_decode, kp * P * H * D * 2 * 2 + 2 * H * D * 2 + H * (kp - 1) * 4),
        "step_one_launch": (fused, step_bytes(ctx, budget, a.method)),
        "step_chain": (chained, step_bytes(ctx, budget, a.method)),
    }
    k_append()  # the token's page holds it before the timings (all idempotent)
    k_estimate()
    k_topk()
    out = {"metric": "µs per layer at 8192 ctx, 1K budget (config 2)",
           "config": {"workload": f"{L} layers x ctx {ctx}, budget {budget}, outlier K seed 1, "
                                  f"{a.method}; each launch over its layers in one CUDA graph",
                      "scored_bytes_per_page": H * row}}
    launches = 0
    steps = max(10, a.steps // 2)
    for name, (fn, b) in parts.items():
        g = capture(fn, dev)
        ms = time_replays(g.replay, steps, 3, world, dev)
        us = ms * 1e3 / (steps * L)
        out[name] = {"us": round(us, 3), **roof(b, us, peak)}
        launches += steps * L * (4 if name == "step_chain" else 1)
        del g
    _lib.check_device()
    out["gpu_launches"] = launches
    for p in chain:
        p.close()
    ctl.clean_states()
    return out


def run_single(a, key):
    world, rank, local = dist_env()
    dev = init_gpu(world, local)
    from aoa_kv_b200 import _lib
    _lib.load()
    peak, _ = load_peak()
    fn = longctx_key if key == "longctx" else batched_key
    val = fn(a, world, rank, dev, peak)
    if rank == 0:
        line = dict(val)
        line.update({"warmup": a.warmup, "higher_is_better": False, "vs_baseline": None,
                     "dtype": "f16", "data": "synthetic", "ms_per_step":
                     round(val["value"] * val["layers_per_step"] / 1e3, 4)})
        print(json.dumps(line), flush=True)
    finish(world)


# ------------------------------------------- Llama-2-7B-shaped decode step
MODEL_METRIC = "ms/token, 32-layer Llama-2-7B-shaped decode, sparse attention (layers 2-31)"


def model_key(a, world, rank, dev, peak, steps=None, warmup=None):
    """Config 3: one decode token through a 32-layer Llama-2-7B-shaped model
    with random fp16 weights (hidden 4096, 32 heads, head_dim 128, MLP 11008,
    vocab 32000): RMSNorm, q/k/v GEMVs, attention through
    InferenceController.decode_step with RoPE fused into the step (layers 0-1
    dense, as in the reference's skip layers, llama.py:428-439; the rest with
    the token budget), o_proj, SwiGLU MLP, final norm, LM head and a
    device-side argmax, captured in one CUDA graph; contexts 16384 and 32768
    x budgets 512/1024/2048/4096 (KV ~ N(0,1), seed 2). The GEMVs are torch
    (cuBLAS); the attention share is timed by replaying a graph of only the
    attention calls."""
    import torch

    import aoa_kv_b200 as ak
    steps = steps or a.steps
    warmup = warmup if warmup is not None else a.warmup
    L, HID, FF, VOCAB = 32, 4096, 11008, 32000
    gen = torch.Generator(device=dev).manual_seed(2)

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

    def rmsnorm(x, g):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).half() * g

    results = []
    for S in (16384, 32768):
        ctl = ak.InferenceController(L, H, D, P, 4096 // P, S + P, torch.float16, dev,
                                     method=a.method)
        ctl.prepare_metadata(S - 1)
        ctl.begin_forward(S - 1)
        for layer in range(L):
            K = torch.randn(S - 1, H, D, device=dev, generator=gen).half()
            V = torch.randn(S - 1, H, D, device=dev, generator=gen).half()
            ak.append_kv(K, V, ctl, layer)
            del K, V
        ctl.end_forward()
        ctl.prepare_metadata(1)
        ctl.begin_forward(1)
        ctl.fuse_rope(1.0, 1e4)
        dense_budget = ctl.kv_cache.pool.capacity  # layers 0-1: every page
        token = torch.zeros(1, dtype=torch.long, device=dev)
        q_buf = torch.empty(L, 1, H, D, dtype=torch.float16, device=dev)
        k_buf, v_buf, o_buf = (torch.empty_like(q_buf) for _ in range(3))
        for budget in (512, 1024, 2048, 4096):
            sparse_budget = budget // P
            ctl.set_page_budget(dense_budget)
            ctl._ensure_step_workspace()
            ctl.set_page_budget(sparse_budget)

            def attention(layer):
                ctl.set_page_budget(dense_budget if layer < 2 else sparse_budget)
                ctl.decode_step(q_buf[layer], k_buf[layer], v_buf[layer], layer,
                                out=o_buf[layer])

            def token_step():
                x = emb[token]  # [1, HID]
                for layer, lw in enumerate(layers):
                    h = rmsnorm(x, lw["ln1"])
                    q_buf[layer].copy_((h @ lw["wq"]).view(1, H, D))
                    k_buf[layer].copy_((h @ lw["wk"]).view(1, H, D))
                    v_buf[layer].copy_((h @ lw["wv"]).view(1, H, D))
                    attention(layer)  # RoPE at position S - 1 inside the step
                    x = x + o_buf[layer].view(1, HID) @ lw["wo"]
                    h = rmsnorm(x, lw["ln2"])
                    x = x + (torch.nn.functional.silu(h @ lw["wg"]) * (h @ lw["wu"])) @ lw["wd"]
                logits = rmsnorm(x, norm_f) @ lm_head
                token.copy_(logits.argmax(dim=-1))

            def attention_only():
                for layer in range(L):
                    attention(layer)
            g_tok, g_att = capture(token_step, dev), capture(attention_only, dev)
            ms_tok = time_replays(g_tok.replay, steps, warmup, 1, dev) / steps
            ms_att = time_replays(g_att.replay, steps, warmup, 1, dev) / steps
            ak.check_device()
            att_bytes = 2 * step_bytes(S, S) + (L - 2) * step_bytes(S, budget)
            results.append({"context": S, "budget": budget, "ms_per_token": round(ms_tok, 4),
                            "attention_ms_per_token": round(ms_att, 4),
                            "attention_share": round(ms_att / ms_tok, 4),
                            "attention_roofline": roof(att_bytes, ms_att * 1e3, peak)})
            del g_tok, g_att
        ctl.clean_states()
        del ctl
        torch.cuda.empty_cache()
    del layers, emb, lm_head
    torch.cuda.empty_cache()
    head = next(r for r in results if r["context"] == 32768 and r["budget"] == 1024)
    return {
        "metric": MODEL_METRIC, "value": head["ms_per_token"], "unit": "ms",
        "steps": steps, "warmup": warmup,
        "config": {"workload": "Llama-2-7B-shaped decode, random weights, KV~N(0,1) seed 2, "
                               "layers 0-1 dense, RoPE fused into the attention step; value "
                               "at ctx 32768, budget 1024",
                   "weight_bytes": weight_bytes},
        "sweep": results,
        "weights_ideal_ms": round(weight_bytes / (peak * 1e9) * 1e3, 4),
    }


def run_model(a):
    dev = init_gpu(1, int(os.environ.get("LOCAL_RANK", "0")))
    from aoa_kv_b200 import _lib
    _lib.load()
    peak, _ = load_peak()
    line = model_key(a, 1, 0, dev, peak)
    line.update({"n_gpus": 1, "ms_per_step": line["value"], "higher_is_better": False,
                 "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic"})
    print(json.dumps(line), flush=True)


# ----------------------------------------------- each kernel, one layer
def run_kernels(a):
    """One layer of the headline shape (ctx a.ctx, budget a.budget, outlier K,
    seed a.seed). Each kernel of the step runs alone, 5 times, with L2
    flushed (a 256 MB write) before every launch and CUDA events around the
    launch itself: the prefill append (once, in the setup, untimed), the
    decode append, the page scorer, the top-k, the sparse decode, the
    one-launch step and the four-kernel chain. Prints one JSON line: per
    kernel its mean launch time, algorithmic bytes and GB/s."""
    import torch

    from aoa_kv_b200 import StepPlan, _lib
    dev = init_gpu(1, int(os.environ.get("LOCAL_RANK", "0")))
    _lib.load()
    peak, peak_src = load_peak()
    ctl, news = setup_layers(a.ctx, 1, a.budget, a.seed, a.method, dev)
    n = len(ctl.kv_cache.indicies)
    kp = a.budget // P
    q, k, v = news[0]
    kv_p, kv_cap, meta_p, meta_cap, vlog_p = ctl._layer_buffers(0)
    scores = torch.empty(H, n, dtype=torch.float32, device=dev)
    sel = torch.empty(H, kp - 1, dtype=torch.int32, device=dev)
    o = torch.empty(H, D, dtype=torch.float16, device=dev)
    ws_n = _lib.size_query("aoakv_decode_workspace_size", H, D, kp - 1)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device=dev)
    sws = ctl._ensure_step_workspace()
    chain = StepPlan(kv_p, kv_cap, meta_p, meta_cap, vlog_p, H, D, P, kp, ctl.score_mode,
                     chain=True)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def st():
        return torch.cuda.current_stream().cuda_stream

    def append():
        _lib.call("aoakv_append_kv_cache_decode", k.data_ptr(), v.data_ptr(), kv_p,
                  ctl.kv_indices_with_last.data_ptr(), n, ctl.kv_cache.last_page_len, kv_cap,
                  meta_p, ctl.metadata_indices.data_ptr(), len(ctl.metadata_cache.indicies),
                  ctl.metadata_cache.last_page_len, meta_cap, vlog_p, H, D, P, 0, st())

    def estimate():
        _lib.call("aoakv_estimate_attn_score", q.data_ptr(), scores.data_ptr(), 1, n, meta_p,
                  ctl.metadata_indices.data_ptr(), len(ctl.metadata_cache.indicies),
                  ctl.metadata_cache.last_page_len, meta_cap,
                  ctl.kv_indices_with_last.data_ptr(), kv_cap, vlog_p, H, D, P, 0,
                  ctl.score_mode, st())

    def topk():
        _lib.call("aoakv_topk_filtering", scores.data_ptr(), 1, n,
                  ctl.kv_indices_with_last.data_ptr(), 0, H, n - 1, kp - 1, None, 0,
                  sel.data_ptr(), kp - 1, 0, st())

    def decode():
        _lib.call("aoakv_sparse_decode", q.data_ptr(), o.data_ptr(), kv_p, kv_cap,
                  sel.data_ptr(), kp - 1, kp - 1, ctl.kv_cache.indicies[-1],
                  ctl.kv_cache.last_page_len, H, D, P, 0, 0.0, ws.data_ptr(), ws_n, st())

    def step():
        ctl.decode_step(q, k, v, 0, out=o)

    def chained():
        chain.run(q, k, v, o, ctl.kv_indices_with_last, n, ctl.kv_cache.last_page_len,
                  ctl.metadata_indices, None, sws, sws.numel(), st())

    # prefill attention of an 8192-token prompt over this layer's first pages
    # (q 67 MB, the pages' K/V 134 MB: larger than L2)
    pf_s = 8192
    pf_q = torch.randn(pf_s, H, D, device=dev).half()
    pf_o = torch.empty_like(pf_q)

    def prefill_attn():
        _lib.call("aoakv_prefill_paged", pf_q.data_ptr(), pf_o.data_ptr(), None, kv_p, kv_cap,
                  ctl.kv_indices_with_last.data_ptr(), pf_s // P, P, pf_s, H, H, D, P, 0, 1,
                  0.0, st())
    sb = step_bytes(a.ctx, a.budget, a.method)
    cases = [
        ("append_decode", append, 2 * H * D * 2 * 2 + 2 * H * D * 2 * 2),
        ("estimate", estimate, estimate_bytes(a.ctx, a.method)),
        ("topk", topk, H * (n - 1) * 4 + H * (kp - 1) * 4),
        ("sparse_decode", decode, kp * P * H * D * 2 * 2 + 2 * H * D * 2 + H * (kp - 1) * 4),
        ("step_one_launch", step, sb),
        ("step_chain", chained, sb),
    ]
    out = {"metric": "per-kernel µs, one headline layer, L2 flushed before each launch",
           "config": {"workload": f"1 layer, ctx {a.ctx}, budget {a.budget}, {a.method}, "
                                  f"outlier K seed {a.seed}",
                      "timing": "CUDA events around each launch; mean of 5"},
           "peak_gbs": peak, "peak_source": peak_src, "kernels": {}}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for name, fn, b in cases:
        fn()  # attributes, tensor maps; every call leaves the same state
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            flush.fill_(1)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        us = statistics.mean(ts)
        out["kernels"][name] = {"us": round(us, 3), **roof(b, us, peak)}
    prefill_attn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        flush.fill_(1)
        e0.record()
        prefill_attn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    us = statistics.mean(ts)
    flops = 4.0 * D * H * pf_s * (pf_s + 1) / 2
    out["kernels"]["prefill_attn_8k"] = {"us": round(us, 3), "bound": "tensor",
                                         "tflops": round(flops / us / 1e6, 1), "flops": flops}
    _lib.check_device()
    chain.close()
    print(json.dumps(out), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    elif a.mode in ("longctx", "batched"):
        run_single(a, a.mode)
    elif a.mode == "model":
        run_model(a)
    elif a.mode == "kernels":
        run_kernels(a)
    else:
        run_headline(a)


if __name__ == "__main__":
    main()
