"""GPU parity of the whole per-layer step (append -> estimate -> top-k ->
sparse decode) against both oracles:
  * semantics B (kernel tree, sink_first_page=0) — oracle.kernel_tree.step;
  * semantics A (the reference simulation, fixed=True) — oracle.sim.decode_step
    with sink_first_page=1.
Selections must match exactly except for near-ties (1e-3 relative); the
attention output must be within max-abs 2e-3 of the oracle (fp16 output)."""
import math

import numpy as np
import pytest
import torch

from aoa_kv_b200 import StepPlan, _lib
from gen import gen_qkv
from gpu_util import GpuLayer, ptr, stream
from helpers import selection_mismatch
from oracle import kernel_tree as kt
from oracle import sim

pytestmark = pytest.mark.gpu


def run_step(lay, q, k, v, n, last, budget, mode, sink, impl=None):
    """One step through aoakv_decode_step, or through a StepPlan when impl
    is "cluster" (the default plan) or "chain" (AOAKV_PLAN_CHAIN)."""
    H, D, P = lay.H, lay.D, lay.P
    cols = max(3, budget) if sink else budget
    ws_n = _lib.size_query("aoakv_step_workspace_size", H, D, lay.cap, cols)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    sel = torch.full((H, cols), -9, dtype=torch.int32, device="cuda")
    o = torch.empty(H, D, dtype=torch.float16, device="cuda")
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    score = _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST
    if impl is None:
        _lib.call("aoakv_decode_step", ptr(qd), ptr(kd), ptr(vd), ptr(o), ptr(lay.kv),
                  ptr(lay.kv_idx), n, last, lay.cap, ptr(lay.meta), ptr(lay.meta_idx), lay.mcap,
                  ptr(lay.vlog), H, D, P, budget, score, int(sink), ptr(sel), ptr(ws), ws_n,
                  stream())
    else:
        plan = StepPlan(lay.kv, lay.cap, lay.meta, lay.mcap, lay.vlog, H, D, P, budget, score,
                        sink, chain=impl == "chain")
        kernels, cluster = plan.info(n)
        assert (cluster == 0) if impl == "chain" else (kernels == 1 and cluster >= 1)
        plan.run(qd, kd, vd, o, lay.kv_idx, n, last, lay.meta_idx, sel, ws, ws_n, stream())
    torch.cuda.synchronize()
    return o.float().cpu().numpy(), sel.cpu().numpy()


def logical(sel_phys, kv_idx, n):
    inv = {int(p): i for i, p in enumerate(kv_idx[:n])}
    return [sorted(inv[int(p)] for p in row if p >= 0) for row in sel_phys]


CASES_B = [(8192, 64, "outlier"), (32768, 64, "outlier"), (1000, 16, "normal"),
           (5000, 1, "normal"), (300, 64, "normal"), (4097, 2, "outlier"), (33, 64, "normal")]


@pytest.mark.parametrize("mode", ["aoakv", "quest"])
@pytest.mark.parametrize("S,budget,dist", CASES_B)
def test_step_matches_kernel_tree(cuda, mode, S, budget, dist):
    H, D, P = 32, 128, 16
    q, K, V = gen_qkv(S + budget, H, S, D, dist)
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 2, H, D, P, seed=S)
    lay.fill(K[:-1], V[:-1])
    torch.cuda.synchronize()
    ref = lay.snapshot()
    got_o, got_sel = run_step(lay, q, K[-1], V[-1], n, last, budget, mode, sink=False)
    want_o, want_sel = kt.step(q, K[-1], V[-1], ref, lay.kv_idx_np, lay.meta_idx_np, n, last,
                               budget, mode, sink=False)
    k = min(budget, n)
    assert all(len(r) == k for r in logical(got_sel, lay.kv_idx_np, n))
    assert np.all(got_sel[:, k:] == -1)
    assert np.all(got_sel[:, k - 1] == lay.kv_idx_np[n - 1])  # last page last
    g_log = np.array(logical(got_sel, lay.kv_idx_np, n))
    w_log = np.array(logical(want_sel, lay.kv_idx_np, n))
    if n > k and k > 1:
        scores = kt.estimate(q, ref, lay.meta_idx_np, lay.kv_idx_np, n, mode)
        scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
        assert not selection_mismatch(g_log, w_log, scores)
    else:
        assert np.array_equal(g_log, w_log)
    # output vs the oracle's decode over the pages the GPU chose
    phys = [[int(p) for p in row[: k - 1]] for row in got_sel]
    o_ref = kt.sparse_decode(q, ref, np.array(phys, dtype=np.int64).reshape(H, k - 1),
                             int(lay.kv_idx_np[n - 1]), last)
    assert np.abs(got_o - o_ref).max() < 2e-3
    if np.array_equal(g_log, w_log):
        assert np.abs(got_o - want_o).max() < 2e-3
    assert _lib.device_error() == 0


CASES_A = [(8192, 1024, "outlier"), (4096 + 7, 1024, "normal"), (2048, 256, "outlier"),
           (528, 64, "normal"), (40, 1024, "normal"), (3000, 32, "normal")]


@pytest.mark.parametrize("method", ["aoakv", "quest"])
@pytest.mark.parametrize("S,B,dist", CASES_A)
def test_step_sink_matches_reference_simulation(cuda, method, S, B, dist):
    H, D, P = 32, 128, 16
    q, K, V = gen_qkv(7 * S + B, H, S, D, dist)
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 2, H, D, P, seed=S + 1, permute=True)
    lay.fill(K[:-1], V[:-1])
    Kh, Vh = K.astype(np.float32).transpose(1, 0, 2), V.astype(np.float32).transpose(1, 0, 2)
    st = sim.SimLayerState(Kh[:, :-1], Vh[:, :-1], P)
    out_s, sel_s, sc_s = sim.decode_step(st, q.astype(np.float32), Kh[:, -1], Vh[:, -1], B,
                                         method, True, expand=False)
    budget_pages = min(S, B) // P
    got_o, got_sel = run_step(lay, q, K[-1], V[-1], n, last, budget_pages, method, sink=True)
    g_log = np.array(logical(got_sel, lay.kv_idx_np, n))
    assert g_log.shape == sel_s.shape
    assert not selection_mismatch(g_log, sel_s, sc_s)
    mask = sim.token_mask(g_log, S, P)
    o_ref = sim.masked_decode(q.astype(np.float32), st.K, st.V, mask)
    assert np.abs(got_o - o_ref).max() < 2e-3
    if np.array_equal(g_log, sel_s):
        assert np.abs(got_o - out_s).max() < 2e-3


@pytest.fixture(params=["cluster", "chain"])
def step_impl(request):
    """Runs a test through a StepPlan: the one cluster launch (the default)
    and the four-kernel chain (AOAKV_PLAN_CHAIN)."""
    return request.param


@pytest.mark.parametrize("mode,sink,S,budget", [
    (m, s, S, b) for m in ("aoakv", "quest") for s in (False, True)
    for S, b in ((32768, 64), (8192 + 9, 64), (3000, 5))] + [("aoakv", False, 131072, 256)])
def test_step_impls_agree_with_oracle(cuda, step_impl, mode, sink, S, budget):
    H, D, P = 32, 128, 16
    q, K, V = gen_qkv(S + 3 * budget, H, S, D, "outlier")
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 1, H, D, P, seed=S + 5)
    lay.fill(K[:-1], V[:-1])
    torch.cuda.synchronize()
    ref = lay.snapshot()
    got_o, got_sel = run_step(lay, q, K[-1], V[-1], n, last, budget, mode, sink, step_impl)
    kp = max(3, budget) if sink else budget
    k = min(kp, n)
    want_o, want_sel = kt.step(q, K[-1], V[-1], ref, lay.kv_idx_np, lay.meta_idx_np, n, last,
                               budget, mode, sink)
    g_log = np.array(logical(got_sel, lay.kv_idx_np, n))
    w_log = np.array(logical(want_sel, lay.kv_idx_np, n))
    scores = kt.estimate(q, ref, lay.meta_idx_np, lay.kv_idx_np, n, mode)
    scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
    if sink:
        scores[:, 0] = np.inf
    assert not selection_mismatch(g_log, w_log, scores)
    phys = np.array([[int(p) for p in row[: k - 1]] for row in got_sel], dtype=np.int64)
    o_ref = kt.sparse_decode(q, ref, phys.reshape(H, k - 1), int(lay.kv_idx_np[n - 1]), last)
    assert np.abs(got_o - o_ref).max() < 2e-3
    if np.array_equal(g_log, w_log):
        assert np.abs(got_o - want_o).max() < 2e-3
    # the appended token landed exactly as the oracle put it
    after = lay.snapshot()
    pid = int(lay.kv_idx_np[n - 1])
    assert np.array_equal(after.kv[pid], ref.kv[pid])
    assert np.array_equal(after.meta, ref.meta)
    assert _lib.device_error() == 0


def test_step_captured_in_cuda_graph(cuda, step_impl):
    """The planned step (cluster launch or PDL chain) captures into a CUDA
    graph and replays with the same result; the workspace stays clean."""
    H, D, P, B = 32, 128, 16, 64
    S = 8192
    q, K, V = gen_qkv(99, H, S, D, "outlier")
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 1, H, D, P, seed=4)
    lay.fill(K[:-1], V[:-1])
    ws_n = _lib.size_query("aoakv_step_workspace_size", H, D, lay.cap, B)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    o = torch.empty(H, D, dtype=torch.float16, device="cuda")
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, K[-1], V[-1]))

    plan = StepPlan(lay.kv, lay.cap, lay.meta, lay.mcap, lay.vlog, H, D, P, B, _lib.SCORE_AOAKV,
                    False, chain=step_impl == "chain")

    def call():
        plan.run(qd, kd, vd, o, lay.kv_idx, n, last, lay.meta_idx, None, ws, ws_n,
                 torch.cuda.current_stream().cuda_stream)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        call()
    torch.cuda.synchronize()
    eager = o.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    for _ in range(5):
        o.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(o, eager)
    assert int(ws[: H * 4].view(torch.int32).abs().sum()) == 0  # the decode tickets re-armed
    assert _lib.device_error() == 0


def test_step_repeated_calls_keep_workspace_clean(cuda):
    """Ten consecutive steps (tokens appended each time, one page boundary
    crossed) against the oracle: the tickets in the workspace re-arm."""
    H, D, P, B = 32, 128, 16, 16
    S0 = 2000
    q, K, V = gen_qkv(77, H, S0 + 10, D, "outlier")
    cap = (S0 + 10 + P - 1) // P + 1
    lay = GpuLayer(cap, H, D, P, seed=9)
    lay.fill(K[:S0], V[:S0])
    torch.cuda.synchronize()
    ref = lay.snapshot()
    ws_n = _lib.size_query("aoakv_step_workspace_size", H, D, cap, B)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    o = torch.empty(H, D, dtype=torch.float16, device="cuda")
    qd = torch.from_numpy(q).cuda()
    for t in range(S0, S0 + 10):
        S = t + 1
        n, last = (S + P - 1) // P, (S - 1) % P + 1
        kd, vd = torch.from_numpy(K[t]).cuda(), torch.from_numpy(V[t]).cuda()
        _lib.call("aoakv_decode_step", ptr(qd), ptr(kd), ptr(vd), ptr(o), ptr(lay.kv),
                  ptr(lay.kv_idx), n, last, cap, ptr(lay.meta), ptr(lay.meta_idx), lay.mcap,
                  ptr(lay.vlog), H, D, P, B, _lib.SCORE_AOAKV, 0, None, ptr(ws), ws_n, stream())
        want_o, _ = kt.step(q, K[t], V[t], ref, lay.kv_idx_np, lay.meta_idx_np, n, last, B,
                            "aoakv", False)
        torch.cuda.synchronize()
        assert np.abs(o.float().cpu().numpy() - want_o).max() < 2e-3, t
    cnt = ws[: H * 4].view(torch.int32)
    assert int(cnt.abs().sum()) == 0


@pytest.mark.parametrize("max_ctas", [64, 74, 148])
def test_step_grid_capped_matches_oracle(cuda, max_ctas):
    """aoakv_decode_step_grid: the step on a fraction of the GPU (the cluster
    launch with fewer CTAs per head) gives the oracle's selection and output."""
    H, D, P, budget, S, mode = 32, 128, 16, 64, 8192 + 5, "aoakv"
    q, K, V = gen_qkv(S + max_ctas, H, S, D, "outlier")
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 1, H, D, P, seed=S + max_ctas)
    lay.fill(K[:-1], V[:-1])
    torch.cuda.synchronize()
    ref = lay.snapshot()
    ws_n = _lib.size_query("aoakv_step_workspace_size", H, D, lay.cap, budget)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    sel = torch.full((H, budget), -9, dtype=torch.int32, device="cuda")
    o = torch.empty(H, D, dtype=torch.float16, device="cuda")
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, K[-1], V[-1]))
    _lib.call("aoakv_decode_step_grid", ptr(qd), ptr(kd), ptr(vd), ptr(o), ptr(lay.kv),
              ptr(lay.kv_idx), n, last, lay.cap, ptr(lay.meta), ptr(lay.meta_idx), lay.mcap,
              ptr(lay.vlog), H, D, P, budget, _lib.SCORE_AOAKV, 0, ptr(sel), ptr(ws), ws_n,
              max_ctas, stream())
    torch.cuda.synchronize()
    want_o, want_sel = kt.step(q, K[-1], V[-1], ref, lay.kv_idx_np, lay.meta_idx_np, n, last,
                               budget, mode, False)
    got_sel = sel.cpu().numpy()
    g_log = np.array(logical(got_sel, lay.kv_idx_np, n))
    w_log = np.array(logical(want_sel, lay.kv_idx_np, n))
    scores = kt.estimate(q, ref, lay.meta_idx_np, lay.kv_idx_np, n, mode)
    scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
    assert not selection_mismatch(g_log, w_log, scores)
    if np.array_equal(g_log, w_log):
        assert np.abs(o.float().cpu().numpy() - want_o).max() < 2e-3
    assert _lib.device_error() == 0


@pytest.mark.parametrize("start_pages,budget,mode,sink", [
    (41, 16, "aoakv", False), (300, 64, "aoakv", True), (590, 32, "quest", False)])
def test_step_back_to_back_same_layer(cuda, start_pages, budget, mode, sink):
    """Twenty steps of ONE layer issued back to back on one stream with
    nothing between them (no copy, no synchronisation): every step reads the
    page metadata, v_log_norm and KV rows that the previous step's append
    wrote, across two page fills and two new pages, while under programmatic
    dependent launch it may start before the previous step ends. Every
    output and selection is checked against the oracle run step by step."""
    H, D, P, T = 32, 128, 16, 20
    S0 = (start_pages - 1) * P + 14  # tokens before the first step
    q_all = np.stack([gen_qkv(7000 + i, H, 1, D, "normal")[0] for i in range(T)])
    _, K, V = gen_qkv(start_pages + budget, H, S0 + T, D, "outlier")
    cap = (S0 + T + P - 1) // P + 1
    lay = GpuLayer(cap, H, D, P, seed=start_pages)
    lay.fill(K[:S0], V[:S0])
    torch.cuda.synchronize()
    ref = lay.snapshot()
    cols = max(3, budget) if sink else budget
    ws_n = _lib.size_query("aoakv_step_workspace_size", H, D, cap, cols)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(q_all).cuda()
    kd = torch.from_numpy(np.ascontiguousarray(K[S0:])).cuda()
    vd = torch.from_numpy(np.ascontiguousarray(V[S0:])).cuda()
    o = torch.empty(T, H, D, dtype=torch.float16, device="cuda")
    sel = torch.full((T, H, cols), -9, dtype=torch.int32, device="cuda")
    mode_id = _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST
    torch.cuda.synchronize()
    for t in range(T):  # issued back to back; the host never waits
        S = S0 + t + 1
        n, last = (S + P - 1) // P, (S - 1) % P + 1
        _lib.call("aoakv_decode_step", ptr(qd[t]), ptr(kd[t]), ptr(vd[t]), ptr(o[t]),
                  ptr(lay.kv), ptr(lay.kv_idx), n, last, cap, ptr(lay.meta), ptr(lay.meta_idx),
                  lay.mcap, ptr(lay.vlog), H, D, P, budget, mode_id, int(sink), ptr(sel[t]),
                  ptr(ws), ws_n, stream())
    torch.cuda.synchronize()
    got_o, got_sel = o.float().cpu().numpy(), sel.cpu().numpy()
    fills = 0
    for t in range(T):
        S = S0 + t + 1
        n, last = (S + P - 1) // P, (S - 1) % P + 1
        fills += last == P
        want_o, want_sel = kt.step(q_all[t], K[S0 + t], V[S0 + t], ref, lay.kv_idx_np,
                                   lay.meta_idx_np, n, last, budget, mode, sink)
        kp = max(3, budget) if sink else budget
        k = min(kp, n)
        g_log = np.array(logical(got_sel[t], lay.kv_idx_np, n))
        w_log = np.array(logical(want_sel, lay.kv_idx_np, n))
        scores = kt.estimate(q_all[t], ref, lay.meta_idx_np, lay.kv_idx_np, n, mode)
        scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
        if sink:
            scores[:, 0] = np.inf
        assert not selection_mismatch(g_log, w_log, scores), t
        assert np.all(got_sel[t][:, k - 1] == lay.kv_idx_np[n - 1]), t
        phys = np.array([[int(p) for p in row[: k - 1]] for row in got_sel[t]], dtype=np.int64)
        o_ref = kt.sparse_decode(q_all[t], ref, phys.reshape(H, k - 1),
                                 int(lay.kv_idx_np[n - 1]), last)
        assert np.abs(got_o[t] - o_ref).max() < 2e-3, t
        if np.array_equal(g_log, w_log):
            assert np.abs(got_o[t] - want_o).max() < 2e-3, t
    assert fills == 2
    after = lay.snapshot()
    assert np.array_equal(after.meta, ref.meta)
    assert np.abs(after.vlog.astype(np.float32) - ref.vlog.astype(np.float32)).max() <= 2e-3
    assert _lib.device_error() == 0


@pytest.mark.parametrize("impl", ["cluster", "chain"])
@pytest.mark.parametrize("S,budget,D", [(8192 + 7, 64, 128), (2000, 16, 64), (16 * 40, 64, 128)])
def test_step_with_fused_rope_equals_rope_then_step(cuda, impl, S, budget, D):
    """RoPE fused into the step (aoakv_step_plan_set_rope) gives the same bits
    as aoakv_apply_rope_in_place followed by the step: output, selection,
    the cache afterwards, and q and k left rotated in place; and it matches
    the oracle's RoPE (kernel_tree.apply_rope) followed by kernel_tree.step."""
    H, P = 32, 16
    q, K, V = gen_qkv(S + D, H, S, D, "outlier")
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lays = []
    for fused in (False, True):
        lay = GpuLayer(n + 3, H, D, P, seed=9)
        lay.fill(K[:-1], V[:-1])
        plan = StepPlan(lay.kv, lay.cap, lay.meta, lay.mcap, lay.vlog, H, D, P, budget,
                        _lib.SCORE_AOAKV, chain=impl == "chain")
        qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, K[-1], V[-1]))
        if fused:
            plan.set_rope(1.0, 1e4)
        else:
            _lib.call("aoakv_apply_rope_in_place", ptr(qd), ptr(kd), 1, S - 1, H, D, 1.0, 1e4,
                      stream())
        ws_n = _lib.size_query("aoakv_step_workspace_size", H, D, lay.cap, budget)
        ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
        o = torch.empty(H, D, dtype=torch.float16, device="cuda")
        sel = torch.full((H, budget), -9, dtype=torch.int32, device="cuda")
        plan.run(qd, kd, vd, o, lay.kv_idx, n, last, lay.meta_idx, sel, ws, ws_n, stream())
        torch.cuda.synchronize()
        lays.append((o.cpu(), sel.cpu(), qd.cpu(), kd.cpu(), lay.kv.cpu(), lay.meta.cpu(),
                     lay.vlog.cpu(), lay))
    (o0, s0, q0, k0, kv0, m0, v0, lay0), (o1, s1, q1, k1, kv1, m1, v1, _) = lays
    assert torch.equal(q0, q1) and torch.equal(k0, k1)
    assert torch.equal(kv0, kv1) and torch.equal(m0, m1) and torch.equal(v0, v1)
    assert torch.equal(s0, s1) and torch.equal(o0, o1)
    # against the oracle: rotate, then the kernel-tree step
    qr = kt.apply_rope(q[None], S - 1)[0]
    kr = kt.apply_rope(K[-1][None], S - 1)[0]
    np.testing.assert_allclose(q1.float().numpy(), qr.astype(np.float32), rtol=2e-3, atol=3e-3)
    ref = kt.LayerCache(lay0.cap, H, D, P)
    lay_ref = GpuLayer(n + 3, H, D, P, seed=9)
    lay_ref.fill(K[:-1], V[:-1])
    ref = lay_ref.snapshot()
    want_o, want_sel = kt.step(q1.numpy(), k1.numpy(), V[-1], ref, lay_ref.kv_idx_np,
                               lay_ref.meta_idx_np, n, last, budget, "aoakv", False)
    got = logical(s1.numpy(), lay_ref.kv_idx_np, n)
    want = logical(want_sel, lay_ref.kv_idx_np, n)
    if got == want:
        assert np.abs(o1.float().numpy() - want_o).max() < 2e-3
    assert _lib.device_error() == 0
