"""Writes the golden vectors in tests/golden/*.npz from the reference's OWN code.

Run where the reference checkout exists, giving its root as the first
argument or in AOAKV_REFERENCE:
    python tests/golden/make_golden.py <reference checkout>

Semantics A (``sim_*.npz``): the reference simulation — the real
filtering/filter_util.py functions (imported, not copied) driven by the decode
branch of evaluation/quest_attention.py (:249-356 aoakv, :90-167 quest), whose
~25 lines of glue are restated below because that module does not import under
the installed transformers. torch.Tensor.topk is wrapped for the duration of
the selection call to record the page scores the reference ranks.

Semantics B (``kt_*.npz``): the reference kernel tree's CPU test references,
imported from kernels/aoa_kv/quest/tests/ with a stub ``quest`` package (those
modules import the CUDA extension at top level but their reference functions
are plain torch):
  test_estimate.py:17-75                 _ref_cpu_estimate
  test_approx_attention.py:17-110        _ref_self_approx_attention
  test_v_log_norm_prefill_claude.py:28-66 compute_expected_v_log_norm_cpu

Page table (``pt_*.npz``): the reference's own host allocator, KvCache from
kernels/aoa_kv/quest/utils/kv_cache.py (imported with a stub quest.utils.utils
for its TensorLayout import), driven the way controller.py:82-87
prepare_metadata drives it (a KV cache plus a metadata cache that appends one
entry per new KV page); after every append the page lists and last-page
lengths are recorded.

Inputs come from tests/golden/gen.py (seeded, fp16); each file stores the
input digest, the case parameters and the reference outputs.

Prefill attention (``pf_*.npz``): the reference test's own CPU attention,
_ref_self_attention of kernels/aoa_kv/quest/tests/test_prefill_attention.py:
17-40 (causal, fp16 inputs, its softmax cast back to fp16 before P.V).

``--only page_table`` / ``--only prefill`` regenerate just those files.
"""
from __future__ import annotations

import importlib.util
import json
import math
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from gen import digest, gen_gqa, gen_qkv  # noqa: E402

REF: Path  # the reference checkout's root, set by main()
TESTS: Path  # its kernels/aoa_kv/quest/tests

SIM_CASES = [
    # name, seed, H, S, D, P, token_budget, method, fixed, dist
    ("sim_aoakv_fixed_ragged", 11, 4, 300, 128, 16, 128, "aoakv", True, "normal"),
    ("sim_quest_fixed_ragged", 11, 4, 300, 128, 16, 128, "quest", True, "normal"),
    ("sim_aoakv_nofix_ragged", 12, 4, 300, 128, 16, 128, "aoakv", False, "normal"),
    ("sim_quest_nofix_ragged", 12, 4, 300, 128, 16, 128, "quest", False, "normal"),
    ("sim_aoakv_fixed_newpage_outlier", 13, 4, 513, 128, 16, 160, "aoakv", True, "outlier"),
    ("sim_quest_fixed_newpage_outlier", 13, 4, 513, 128, 16, 160, "quest", True, "outlier"),
    ("sim_aoakv_fixed_pagefill", 14, 4, 256, 128, 16, 64, "aoakv", True, "normal"),
    ("sim_aoakv_fixed_short_dense", 15, 4, 40, 128, 16, 1024, "aoakv", True, "normal"),
    ("sim_quest_fixed_min3", 16, 4, 200, 128, 16, 32, "quest", True, "normal"),
    ("sim_aoakv_fixed_d64", 17, 8, 333, 64, 16, 96, "aoakv", True, "outlier"),
    ("sim_aoakv_fixed_h32", 18, 32, 1024, 128, 16, 256, "aoakv", True, "normal"),
    ("sim_quest_fixed_h32", 18, 32, 1024, 128, 16, 256, "quest", True, "normal"),
]

GQA_CASES = [
    # name, seed, Hq, Hkv, S, D, P, token_budget, method, fixed, dist
    ("sim_aoakv_fixed_gqa4", 19, 8, 2, 333, 128, 16, 96, "aoakv", True, "outlier"),
    ("sim_quest_fixed_gqa4", 19, 8, 2, 333, 128, 16, 96, "quest", True, "outlier"),
    ("sim_aoakv_fixed_gqa2_d64", 20, 8, 4, 500, 64, 16, 128, "aoakv", True, "normal"),
]

KT_EST_CASES = [  # name, seed, kv_len (test_estimate.py:77 parameter list)
    ("kt_est_27", 21, 27), ("kt_est_113", 22, 113), ("kt_est_577", 23, 577),
    ("kt_est_1541", 24, 1541),
]
KT_APPROX_CASES = [  # name, seed, kv_len, page_budget (test_approx_attention.py:112)
    ("kt_approx_61_7", 31, 61, 7), ("kt_approx_113_4", 32, 113, 4),
    ("kt_approx_577_15", 33, 577, 15), ("kt_approx_1011_31", 34, 1011, 31),
    ("kt_approx_1541_55", 35, 1541, 55), ("kt_approx_482_71", 36, 482, 71),
]
KT_VLOG_CASES = [("kt_vlog_128", 41, 128), ("kt_vlog_256", 42, 256), ("kt_vlog_200", 43, 200)]

PT_CASES = [  # name, page_size, max_seq_len, appends (prompt, then decode tokens)
    ("pt_prompt100_decode40", 16, 4096, [100] + [1] * 40),
    ("pt_pagefill_p16", 16, 4096, [16, 1, 15, 1, 16, 16, 1]),
    ("pt_many_pages_p8", 8, 8192, [1000, 1, 1, 7, 1, 300]),
    ("pt_meta_boundary", 16, 16384, [16 * 16, 1, 16 * 16 - 1, 1, 1]),
]


def load_ref_kv_cache():
    for mod in ("quest", "quest.utils", "quest.utils.utils"):
        sys.modules.setdefault(mod, types.ModuleType(mod))

    class TensorLayout:  # quest/utils/utils.py's enum, only NHD is read
        NHD = 0
        HND = 1
    sys.modules["quest.utils.utils"].TensorLayout = TensorLayout
    path = REF / "kernels" / "aoa_kv" / "quest" / "utils" / "kv_cache.py"
    spec = importlib.util.spec_from_file_location("_ref_kv_cache", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


PF_CASES = [  # name, seed, qo_len, kv_len, heads (test_prefill_attention.py:42 grid)
    ("pf_13_33", 51, 13, 33, 4), ("pf_77_400", 52, 77, 400, 2), ("pf_244_244", 53, 244, 244, 2),
    ("pf_311_1110", 54, 311, 1110, 1),
]


def make_prefill_goldens():
    t_pf = load_ref_test("test_prefill_attention")
    for name, seed, qo, kvl, heads in PF_CASES:
        g = np.random.default_rng(seed)
        q = g.standard_normal((qo, heads, 128), dtype=np.float32).astype(np.float16)
        k = g.standard_normal((kvl, heads, 128), dtype=np.float32).astype(np.float16)
        v = g.standard_normal((kvl, heads, 128), dtype=np.float32).astype(np.float16)
        o = t_pf._ref_self_attention(torch.from_numpy(q), torch.from_numpy(k),
                                     torch.from_numpy(v))
        save(name, dict(seed=seed, qo_len=qo, kv_len=kvl, heads=heads, D=128), q=q, k=k, v=v,
             out=o.numpy().astype(np.float16))
        print(name, tuple(o.shape))


def make_page_table_goldens():
    kvc = load_ref_kv_cache()
    for name, P, max_len, appends in PT_CASES:
        kv = kvc.KvCache(1, 1, 1, max_len, P, torch.float16, torch.device("cpu"))
        meta = kvc.KvCache(1, 1, 1, (max_len + P - 1) // P, P, torch.float16,
                           torch.device("cpu"))
        n_kv, n_meta = (max_len + P - 1) // P, (max_len + P * P - 1) // (P * P)
        kv_ids = np.full((len(appends), n_kv), -1, np.int32)
        meta_ids = np.full((len(appends), n_meta), -1, np.int32)
        last = np.zeros(len(appends), np.int32)
        for i, n in enumerate(appends):
            new_pages = kv.append_seq(n)  # controller.py:84-87
            meta.append_seq(new_pages)
            kv_ids[i, :len(kv.indicies)] = kv.indicies
            meta_ids[i, :len(meta.indicies)] = meta.indicies
            last[i] = kv.last_page_len
        save(name, dict(page_size=P, max_seq_len=max_len, appends=appends), kv_ids=kv_ids,
             meta_ids=meta_ids, last_page_len=last)
        print(name, kv_ids.shape, meta_ids.shape)


def load_filter_util():
    sys.path.insert(0, str(REF))
    from filtering import filter_util  # noqa: E402
    return filter_util


def load_ref_test(name: str):
    if "quest" not in sys.modules:
        quest = types.ModuleType("quest")
        quest.utils = types.ModuleType("quest.utils")
        sys.modules["quest"] = quest
        sys.modules["quest.utils"] = quest.utils
    spec = importlib.util.spec_from_file_location(f"_ref_{name}", TESTS / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ref_sim_decode(fu, q, K, V, P, budget, method, fixed):
    """Decode branch of quest_attention.py for one layer with layer_id >= 2,
    after a prefill of the first S-1 tokens (:227-243), batch 1, fp32; q may
    have more heads than K and V (GQA: query head h reads KV head h // g, the
    repeat_kv of the attention)."""
    S, H, D = K.shape
    groups = q.shape[0] // H
    past = S - 1
    Kt = torch.from_numpy(K.astype(np.float32)).permute(1, 0, 2)[None].contiguous()
    Vt = torch.from_numpy(V.astype(np.float32)).permute(1, 0, 2)[None].contiguous()
    qt = torch.from_numpy(q.astype(np.float32))[None, :, None, :]
    filters = fu.get_max_min_filters(Kt[:, :, :past], P)               # qa:238
    vmean = fu.compute_page_v_mean(past, P, Vt[:, :, :past])           # qa:239
    cur_k, cur_v = Kt[:, :, past:], Vt[:, :, past:]
    if method == "aoakv":                                              # qa:254-260
        vmean = fu.update_mean_page_filters(vmean.unsqueeze(-2), cur_v, past, P).squeeze(-2)
    Kr = Kt.repeat_interleave(groups, dim=1) if groups > 1 else Kt     # repeat_kv
    attn = torch.matmul(qt, Kr.transpose(2, 3)) / math.sqrt(D)         # qa:265-268
    filters = fu.update_page_filters(filters, cur_k, past, P)          # qa:291-293
    w = fu.compute_attn_weights_for_selection(qt, filters, groups, P, S, math.ceil(S / P))  # qa:297-300
    tb = min(S, budget)                                                # qa:326
    seen = {}
    orig_topk = torch.Tensor.topk

    def rec_topk(self, *a, **kw):
        seen["scores"] = self.detach().clone()
        return orig_topk(self, *a, **kw)

    torch.Tensor.topk = rec_topk
    try:
        if method == "aoakv":                                          # qa:328-332
            mask = fu.local_heavy_hitter_mask_value_aware_group_consistent_sum(
                w, tb, P, vmean, groups, D, fixed)
        else:                                                          # qa:139-143
            mask, _ = fu.local_heavy_hitter_mask_group_consistent_sum(w, tb, P, groups, fixed)
    finally:
        torch.Tensor.topk = orig_topk
    attn[~mask] = torch.tensor(torch.finfo(attn.dtype).min)            # qa:347
    p = torch.nn.functional.softmax(attn, dim=-1, dtype=torch.float32)  # qa:351
    Vr = Vt.repeat_interleave(groups, dim=1) if groups > 1 else Vt
    out = torch.matmul(p, Vr)[0, :, 0]                                 # qa:353-356
    N = math.ceil(S / P)
    pad = N * P - S
    page_sel = torch.cat([mask[0, ::groups, 0], torch.zeros(H, pad, dtype=torch.bool)], 1)
    page_sel = page_sel.reshape(H, N, P).any(-1)
    sel = np.stack([np.nonzero(r)[0] for r in page_sel.numpy()]).astype(np.int32)
    scores = seen["scores"].reshape(H, N).numpy().astype(np.float32)
    return out.numpy().astype(np.float32), sel, scores


def save(name, meta, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), **arrays)


def main():
    global REF, TESTS
    root = sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("--") else \
        os.environ.get("AOAKV_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py <reference checkout> (or set AOAKV_REFERENCE)")
    REF = Path(root).resolve()
    TESTS = REF / "kernels" / "aoa_kv" / "quest" / "tests"
    if not (REF / "filtering" / "filter_util.py").is_file():
        sys.exit(f"{REF}: no filtering/filter_util.py (not the reference checkout)")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only in (None, "page_table"):
        make_page_table_goldens()
    if only in (None, "prefill"):
        make_prefill_goldens()
    if only is not None:
        return
    fu = load_filter_util()
    for name, seed, H, S, D, P, budget, method, fixed, dist in SIM_CASES:
        q, K, V = gen_qkv(seed, H, S, D, dist)
        out, sel, scores = ref_sim_decode(fu, q, K, V, P, budget, method, fixed)
        meta = dict(seed=seed, H=H, S=S, D=D, P=P, token_budget=budget, method=method,
                    fixed=fixed, dist=dist, digest=digest(q, K, V))
        save(name, meta, out=out, sel=sel, scores=scores)
        print(name, sel.shape, out.shape)

    for name, seed, Hq, Hkv, S, D, P, budget, method, fixed, dist in GQA_CASES:
        q, K, V = gen_gqa(seed, Hq, Hkv, S, D, dist)
        out, sel, scores = ref_sim_decode(fu, q, K, V, P, budget, method, fixed)
        meta = dict(seed=seed, Hq=Hq, Hkv=Hkv, H=Hkv, S=S, D=D, P=P, token_budget=budget,
                    method=method, fixed=fixed, dist=dist, digest=digest(q, K, V))
        save(name, meta, out=out, sel=sel, scores=scores)
        print(name, sel.shape, out.shape)

    t_est = load_ref_test("test_estimate")
    for name, seed, kv_len in KT_EST_CASES:
        q, K, V = gen_qkv(seed, 32, kv_len, 128)
        est = t_est._ref_cpu_estimate(torch.from_numpy(q)[None], torch.from_numpy(K),
                                      torch.from_numpy(V), 16)
        meta = dict(seed=seed, H=32, S=kv_len, D=128, P=16, dist="normal", digest=digest(q, K, V))
        save(name, meta, est=est.numpy().astype(np.float16))
        print(name, tuple(est.shape), est.dtype)

    t_apx = load_ref_test("test_approx_attention")
    for name, seed, kv_len, budget in KT_APPROX_CASES:
        q, K, V = gen_qkv(seed, 32, kv_len, 128)
        o, idx = t_apx._ref_self_approx_attention(torch.from_numpy(q)[None], torch.from_numpy(K),
                                                  torch.from_numpy(V), 16, budget)
        meta = dict(seed=seed, H=32, S=kv_len, D=128, P=16, page_budget=budget, dist="normal",
                    digest=digest(q, K, V))
        arrays = dict(out=o[0].numpy().astype(np.float16))
        if idx is not None:
            arrays["topk"] = idx.numpy().astype(np.int32).reshape(32, -1)
        save(name, meta, **arrays)
        print(name, tuple(o.shape), None if idx is None else tuple(idx.shape))

    t_vl = load_ref_test("test_v_log_norm_prefill_claude")
    for name, seed, seq in KT_VLOG_CASES:
        q, K, V = gen_qkv(seed, 32, seq, 128)
        vl = t_vl.compute_expected_v_log_norm_cpu(torch.from_numpy(V), 16)
        meta = dict(seed=seed, H=32, S=seq, D=128, P=16, dist="normal", digest=digest(q, K, V))
        save(name, meta, vlog=vl.numpy().astype(np.float32))
        print(name, tuple(vl.shape))


if __name__ == "__main__":
    main()
