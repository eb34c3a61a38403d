"""GPU parity of the grouped-query-attention step (aoakv_decode_step_gqa):
query heads sharing a KV head select the same pages from group-combined
scores (filter_util.py: Quest sums the group's page bounds, :219-221;
AOA-KV takes the logsumexp of 2*bound/sqrt(D) over the group and adds
2*log||mean V||, :352-361 and :367) and each attends its KV head's pages.

  * sink_first_page=0 against oracle.kernel_tree.step_gqa (the kernel tree's
    arithmetic with the simulation's group rule);
  * sink_first_page=1 against oracle.sim.decode_step with groups, which is
    pinned to the reference's own filter_util.py by the GQA golden vectors.
Selections must match except near-ties; outputs within 2e-3."""
import numpy as np
import pytest
import torch

from aoa_kv_b200 import _lib
from gen import gen_gqa
from gpu_util import GpuLayer, ptr, stream
from helpers import selection_mismatch
from oracle import kernel_tree as kt
from oracle import sim

pytestmark = pytest.mark.gpu


def run_gqa(lay, q, k, v, n, last, budget, mode, sink):
    Hk, D, P = lay.H, lay.D, lay.P
    Hq = q.shape[0]
    cols = max(3, budget) if sink else budget
    ws_n = _lib.size_query("aoakv_step_workspace_size", Hq, D, lay.cap, cols)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    sel = torch.full((Hk, cols), -9, dtype=torch.int32, device="cuda")
    o = torch.empty(Hq, D, dtype=torch.float16, device="cuda")
    qd, kd, vd = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, k, v))
    score = _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST
    _lib.call("aoakv_decode_step_gqa", ptr(qd), ptr(kd), ptr(vd), ptr(o), ptr(lay.kv),
              ptr(lay.kv_idx), n, last, lay.cap, ptr(lay.meta), ptr(lay.meta_idx), lay.mcap,
              ptr(lay.vlog), Hq, Hk, D, P, budget, score, int(sink), ptr(sel), ptr(ws), ws_n,
              stream())
    torch.cuda.synchronize()
    return o.float().cpu().numpy(), sel.cpu().numpy()


def logical(sel_phys, kv_idx, n):
    inv = {int(p): i for i, p in enumerate(kv_idx[:n])}
    return [sorted(inv[int(p)] for p in row if p >= 0) for row in sel_phys]


@pytest.mark.parametrize("mode", ["aoakv", "quest"])
@pytest.mark.parametrize("Hq,Hk,D,S,budget", [(32, 8, 128, 8192 + 5, 64), (32, 4, 128, 3000, 16),
                                              (16, 8, 64, 2000, 32), (8, 8, 128, 1500, 16),
                                              (32, 8, 128, 500, 64)])
def test_gqa_step_matches_kernel_tree_oracle(cuda, mode, Hq, Hk, D, S, budget):
    P = 16
    q, K, V = gen_gqa(S + Hq + D, Hq, Hk, S, D, "outlier")
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 2, Hk, D, P, seed=S + 3)
    lay.fill(K[:-1], V[:-1])
    torch.cuda.synchronize()
    ref = lay.snapshot()
    got_o, got_sel = run_gqa(lay, q, K[-1], V[-1], n, last, budget, mode, False)
    want_o, want_sel = kt.step_gqa(q, K[-1], V[-1], ref, lay.kv_idx_np, lay.meta_idx_np, n,
                                   last, budget, mode, False)
    k = min(budget, n)
    assert np.all(got_sel[:, k - 1] == lay.kv_idx_np[n - 1])  # the last page, last
    g_log = np.array(logical(got_sel, lay.kv_idx_np, n))
    w_log = np.array(logical(want_sel, lay.kv_idx_np, n))
    if n > k:
        scores = kt.estimate_gqa(q, ref, lay.meta_idx_np, lay.kv_idx_np, n, mode)
        scores = np.concatenate([scores, np.full((Hk, 1), np.inf, np.float32)], axis=1)
        assert not selection_mismatch(g_log, w_log, scores)
    else:
        assert np.array_equal(g_log, w_log)
    if np.array_equal(g_log, w_log):
        assert np.abs(got_o - want_o).max() < 2e-3
    # after the step, the cache holds the appended token exactly as the oracle's
    assert np.array_equal(lay.kv.cpu().numpy(), ref.kv)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("method", ["aoakv", "quest"])
@pytest.mark.parametrize("Hq,Hk,D,S,B", [(32, 8, 128, 4096 + 7, 1024), (8, 2, 128, 333, 96)])
def test_gqa_step_sink_matches_reference_simulation(cuda, method, Hq, Hk, D, S, B):
    P = 16
    q, K, V = gen_gqa(5 * S + B, Hq, Hk, S, D, "outlier")
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay = GpuLayer(n + 2, Hk, D, P, seed=S + 1)
    lay.fill(K[:-1], V[:-1])
    Kh, Vh = K.astype(np.float32).transpose(1, 0, 2), V.astype(np.float32).transpose(1, 0, 2)
    st = sim.SimLayerState(Kh[:, :-1], Vh[:, :-1], P)
    out_s, sel_s, sc_s = sim.decode_step(st, q.astype(np.float32), Kh[:, -1], Vh[:, -1], B,
                                         method, True, expand=False)
    got_o, got_sel = run_gqa(lay, q, K[-1], V[-1], n, last, min(S, B) // P, method, True)
    g_log = np.array(logical(got_sel, lay.kv_idx_np, n))
    assert g_log.shape == sel_s.shape
    assert not selection_mismatch(g_log, sel_s, sc_s)
    g = Hq // Hk
    mask = np.repeat(sim.token_mask(g_log, S, P), g, axis=0)
    o_ref = sim.masked_decode(q.astype(np.float32), np.repeat(st.K, g, axis=0),
                              np.repeat(st.V, g, axis=0), mask)
    assert np.abs(got_o - o_ref).max() < 2e-3
    if np.array_equal(g_log, sel_s):
        assert np.abs(got_o - out_s).max() < 2e-3
    assert _lib.device_error() == 0
