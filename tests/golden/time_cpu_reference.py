"""Times the reference's own CPU decode step (filtering/filter_util.py driven
by the decode branch of evaluation/quest_attention.py) beside this repo's
numpy restatement of it (oracle/sim.py), on the same inputs and host cores,
and writes tests/golden/cpu_reference_timing.json.

The reference checkout is needed (it is not available where the benchmark
runs), so the benchmark's CPU legs time the restatement and carry the ratio
measured here. Run where the checkout exists:
    python tests/golden/time_cpu_reference.py <reference checkout> [--ctx 32768]

Per step (one layer with layer_id >= 2, batch 1, MHA, fp32), both sides do
what quest_attention.py's decode branch does after the prefill (:249-356 for
aoakv): update the page V means (aoakv), append the token to K/V, the dense
q K^T, update the page key max/min filters, the selection weights, the
value-aware group-consistent top-k mask (fixed=True, the simulation's
default: pages 0 and N-1 forced), the masked softmax and p V.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(ROOT))


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def make_inputs(seed, H, S, D):
    """q, K, V as the benchmark's headline workload draws them on the host:
    K ~ N(0,1) * LogNormal(0,1) per (head, channel), q, V ~ N(0,1), fp16."""
    g = np.random.default_rng(seed)
    q = g.standard_normal((H, D), dtype=np.float32).astype(np.float16)
    scale = np.exp(g.standard_normal((H, D), dtype=np.float32))
    K = (g.standard_normal((H, S, D), dtype=np.float32) * scale[:, None]).astype(np.float16)
    V = g.standard_normal((H, S, D), dtype=np.float32).astype(np.float16)
    return q, K, V


def ref_step(fu, st, qt, cur_k, cur_v, P, budget, D, fixed=True):
    """One aoakv decode step with the reference's functions; st holds the
    prefill state (Kt, Vt [1, H, past, D], filters, vmean)."""
    past = st["Kt"].shape[2]
    S = past + 1
    vmean = fu.update_mean_page_filters(st["vmean"].unsqueeze(-2), cur_v, past, P).squeeze(-2)
    Kt = torch.cat([st["Kt"], cur_k], dim=2)
    Vt = torch.cat([st["Vt"], cur_v], dim=2)
    attn = torch.matmul(qt, Kt.transpose(2, 3)) / math.sqrt(D)
    filters = fu.update_page_filters(st["filters"], cur_k, past, P)
    w = fu.compute_attn_weights_for_selection(qt, filters, 1, P, S, math.ceil(S / P))
    mask = fu.local_heavy_hitter_mask_value_aware_group_consistent_sum(
        w, min(S, budget), P, vmean, 1, D, fixed)
    attn[~mask] = torch.tensor(torch.finfo(attn.dtype).min)
    p = torch.nn.functional.softmax(attn, dim=-1, dtype=torch.float32)
    return torch.matmul(p, Vt)[0, :, 0]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("reference", nargs="?", default=os.environ.get("AOAKV_REFERENCE"))
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--budget", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=8)
    a = ap.parse_args()
    if not a.reference or not (Path(a.reference) / "filtering" / "filter_util.py").is_file():
        sys.exit("usage: time_cpu_reference.py <reference checkout> (or set AOAKV_REFERENCE)")
    sys.path.insert(0, str(Path(a.reference).resolve()))
    from filtering import filter_util as fu  # noqa: E402

    from oracle import sim  # noqa: E402

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    H, D, P, S = 32, 128, 16, a.ctx
    q, K, V = make_inputs(1, H, S, D)
    past = S - 1
    # reference state after the prefill (qa:227-243)
    Kt = torch.from_numpy(K.astype(np.float32))[None]
    Vt = torch.from_numpy(V.astype(np.float32))[None]
    st = {"Kt": Kt[:, :, :past].contiguous(), "Vt": Vt[:, :, :past].contiguous()}
    st["filters"] = fu.get_max_min_filters(st["Kt"], P)
    st["vmean"] = fu.compute_page_v_mean(past, P, st["Vt"])
    qt = torch.from_numpy(q.astype(np.float32))[None, :, None, :]
    cur_k, cur_v = Kt[:, :, past:].contiguous(), Vt[:, :, past:].contiguous()
    port0 = sim.SimLayerState(K[:, :-1].astype(np.float32), V[:, :-1].astype(np.float32), P)
    qf, kf, vf = q.astype(np.float32), K[:, -1].astype(np.float32), V[:, -1].astype(np.float32)

    import copy
    ref_t, port_t = [], []
    out_r = out_p = None
    for i in range(a.steps + 1):  # the first of each is a warm-up
        t0 = time.perf_counter()
        out_r = ref_step(fu, st, qt, cur_k, cur_v, P, a.budget, D)
        t1 = time.perf_counter()
        pst = copy.copy(port0)
        t2 = time.perf_counter()
        out_p, _, _ = sim.decode_step(pst, qf, kf, vf, a.budget, "aoakv", True, expand=True)
        t3 = time.perf_counter()
        if i:
            ref_t.append(t1 - t0)
            port_t.append(t3 - t2)
    err = float(np.abs(out_r.numpy() - out_p).max())
    r_us, p_us = statistics.median(ref_t) * 1e6, statistics.median(port_t) * 1e6
    res = {
        "what": "one aoakv decode step (fixed=True), 32 heads, head_dim 128, page 16, "
                f"ctx {S}, budget {a.budget}; median of {a.steps} after one warm-up",
        "cpu_model": cpu_model(), "threads": threads, "torch": torch.__version__,
        "numpy": np.__version__,
        "filter_util_us": round(r_us, 1), "port_us": round(p_us, 1),
        "filter_util_over_port": round(r_us / p_us, 3),
        "max_abs_diff_outputs": err,
    }
    (HERE / "cpu_reference_timing.json").write_text(json.dumps(res, indent=1) + "\n")
    print(json.dumps(res))


if __name__ == "__main__":
    main()
