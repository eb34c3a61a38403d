"""Pins the CPU oracle against golden vectors made by the reference's own code
(tests/golden/make_golden.py): the simulation (filter_util.py) for semantics A
and the kernel tree's CPU test references for semantics B."""
import math
from pathlib import Path

import numpy as np
import pytest

from gen import digest, gen_gqa, gen_qkv
from helpers import golden_names, load_golden, selection_mismatch
from oracle import kernel_tree as kt
from oracle import sim


def _sim_inputs(meta):
    if "Hq" in meta:  # GQA case: Hq query heads over Hkv KV heads
        return gen_gqa(meta["seed"], meta["Hq"], meta["Hkv"], meta["S"], meta["D"], meta["dist"])
    return gen_qkv(meta["seed"], meta["H"], meta["S"], meta["D"], meta["dist"])


@pytest.mark.parametrize("name", golden_names("sim_"))
def test_sim_oracle_matches_reference_simulation(name):
    """MHA and GQA cases (the GQA ones pin the group sum / logsumexp of
    filter_util.py:219-221 and :352-361 and the replicated mask)."""
    meta, g = load_golden(name)
    q, K, V = _sim_inputs(meta)
    assert digest(q, K, V) == meta["digest"], "input regeneration diverged"
    Kh, Vh = K.astype(np.float32).transpose(1, 0, 2), V.astype(np.float32).transpose(1, 0, 2)
    st = sim.SimLayerState(Kh[:, :-1], Vh[:, :-1], meta["P"])
    out, sel, scores = sim.decode_step(st, q.astype(np.float32), Kh[:, -1], Vh[:, -1],
                                       meta["token_budget"], meta["method"], meta["fixed"])
    np.testing.assert_allclose(scores, g["scores"], rtol=2e-5, atol=2e-5)
    assert sel.shape == g["sel"].shape
    assert not selection_mismatch(sel, g["sel"], g["scores"]), (sel, g["sel"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("name", golden_names("sim_"))
def test_sim_expand_equals_per_page(name):
    """The reference's token-expanded bound (fu:1004-1016) equals the
    per-page bound the kernels compute."""
    meta, _ = load_golden(name)
    q, K, _ = _sim_inputs(meta)
    Kh = K.astype(np.float32).transpose(1, 0, 2)
    f = sim.get_max_min_filters(Kh, meta["P"])
    grp = q.shape[0] // Kh.shape[0]
    a = sim.attn_weights_for_selection(q.astype(np.float32), f, meta["P"], meta["S"], expand=True,
                                       groups=grp)
    b = sim.attn_weights_for_selection(q.astype(np.float32), f, meta["P"], meta["S"],
                                       expand=False, groups=grp)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-4)


def _prefill_then_decode(q, K, V, P, cap):
    """The reference tests' flow (test_estimate.py:108-134): prefill S-1 tokens,
    then append one decode token, on a fresh pool (physical == logical)."""
    S, H, D = K.shape
    c = kt.LayerCache(cap, H, D, P)
    idx = np.arange(cap, dtype=np.int32)
    n0 = (S - 1 + P - 1) // P
    kt.append_prefill(c, idx, idx, n0, (S - 2) % P + 1, K[:-1], V[:-1])
    n1 = (S + P - 1) // P
    kt.append_decode(c, idx, idx, n1, (S - 1) % P + 1, K[-1], V[-1])
    return c, idx, n1


@pytest.mark.parametrize("name", golden_names("kt_est_"))
def test_kernel_tree_estimate_matches_reference_test(name):
    meta, g = load_golden(name)
    q, K, V = gen_qkv(meta["seed"], meta["H"], meta["S"], meta["D"])
    assert digest(q, K, V) == meta["digest"]
    c, idx, n = _prefill_then_decode(q, K, V, meta["P"], 256)
    est = kt.estimate(q, c, idx, idx, n, "quest")
    # test_estimate.py:9-15 tolerance for fp16
    np.testing.assert_allclose(est, g["est"].astype(np.float32), rtol=5e-3, atol=5e-3)


@pytest.mark.parametrize("name", golden_names("kt_approx_"))
def test_kernel_tree_decode_matches_reference_test(name):
    meta, g = load_golden(name)
    q, K, V = gen_qkv(meta["seed"], meta["H"], meta["S"], meta["D"])
    assert digest(q, K, V) == meta["digest"]
    P, budget = meta["P"], meta["page_budget"]
    c, idx, n = _prefill_then_decode(q, K, V, P, 256)
    last_len = (meta["S"] - 1) % P + 1
    if "topk" in g:
        sel = g["topk"]
        # the oracle's own selection agrees with the reference's up to ties
        sc = kt.estimate(q, c, idx, idx, n, "quest")
        mine = kt.topk_positions(sc, budget - 1)
        assert not selection_mismatch(mine, sel, sc)
    else:
        sel = np.tile(np.arange(n - 1), (meta["H"], 1))
    out = kt.sparse_decode(q, c, sel, n - 1, last_len)
    np.testing.assert_allclose(out, g["out"].astype(np.float32), rtol=5e-3, atol=5e-3)


@pytest.mark.parametrize("name", golden_names("kt_vlog_"))
def test_kernel_tree_vlog_matches_reference_test(name):
    meta, g = load_golden(name)
    q, K, V = gen_qkv(meta["seed"], meta["H"], meta["S"], meta["D"])
    P, S = meta["P"], meta["S"]
    c = kt.LayerCache(64, meta["H"], meta["D"], P)
    idx = np.arange(64, dtype=np.int32)
    n = (S + P - 1) // P
    kt.append_prefill(c, idx, idx, n, (S - 1) % P + 1, K, V)
    nf = S // P
    # fp16 storage: within one fp16 ulp at |x| < 2 plus rounding of the sum
    np.testing.assert_allclose(c.vlog[:nf].astype(np.float32), g["vlog"], rtol=0, atol=2e-3)
    assert np.all(c.vlog[nf:] == 0)


def test_sink_mode_kernel_tree_agrees_with_simulation():
    """Semantics B with the sink (what the CUDA step computes with
    sink_first_page=1) selects the simulation's pages (fixed=True) up to
    near-ties and attends to the same output within 2e-3."""
    H, S, D, P, B = 8, 900, 128, 16, 256
    for method in ("aoakv", "quest"):
        q, K, V = gen_qkv(5, H, S, D, "outlier")
        Kh, Vh = K.astype(np.float32).transpose(1, 0, 2), V.astype(np.float32).transpose(1, 0, 2)
        st = sim.SimLayerState(Kh[:, :-1], Vh[:, :-1], P)
        out_s, sel_s, sc_s = sim.decode_step(st, q.astype(np.float32), Kh[:, -1], Vh[:, -1], B,
                                             method, True)
        c = kt.LayerCache(64, H, D, P)
        idx = np.arange(64, dtype=np.int32)
        n0 = (S - 1 + P - 1) // P
        kt.append_prefill(c, idx, idx, n0, (S - 2) % P + 1, K[:-1], V[:-1])
        n = (S + P - 1) // P
        budget_pages = min(S, B) // P
        out_k, sel_k = kt.step(q, K[-1], V[-1], c, idx, idx, n, (S - 1) % P + 1, budget_pages,
                               method, sink=True)
        assert not selection_mismatch(np.sort(sel_k, axis=1), sel_s, sc_s)
        assert np.abs(out_k - out_s).max() < 2e-3


def test_topk_positions_rules():
    s = np.array([[1.0, 5.0, 5.0, 3.0, np.nan, 5.0]], np.float32)
    # descending score, ties -> lower position first, NaN last
    assert kt.topk_positions(s, 2).tolist() == [[1, 2]]
    assert kt.topk_positions(s, 5).tolist() == [[1, 2, 5, 3, 0]]
    assert kt.topk_positions(s, 2, sink=True).tolist() == [[0, 1]]
    assert kt.topk_positions(s, 6).tolist() == [[1, 2, 5, 3, 0, 4]]
    z = np.array([[-0.0, 0.0, 1.0]], np.float32)  # -0 == +0: the lower position wins
    assert kt.topk_positions(z, 2).tolist() == [[2, 0]]
    big = np.arange(300, dtype=np.float32)[None]  # k > 256: ascending positions
    assert kt.topk_positions(big, 257).tolist() == [list(range(43, 300))]


def test_sim_budget_rule():
    assert sim.page_budget_k(1024, 16, 256) == 64
    assert sim.page_budget_k(32, 16, 100) == 3
    assert sim.page_budget_k(40, 16, 3) == 3
    assert math.isclose(float(sim.LOG_EPS), 1e-8)


def test_topk_positions_against_brute_force_sort():
    """The oracle's selection rule equals a plain sort by (-score, position)
    with NaN last and -0 == +0, for random rows full of ties."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=60, deadline=None)
    @given(st.integers(1, 60), st.integers(0, 10_000), st.booleans())
    def check(n, seed, sink):
        g = np.random.default_rng(seed)
        row = np.round(g.standard_normal(n) * 2).astype(np.float32)  # many ties
        if n > 3:
            row[g.integers(0, n)] = np.nan
            row[g.integers(0, n)] = -0.0
        k = int(g.integers(1, n + 1))
        got = kt.topk_positions(row[None], k, sink)[0]

        def key(i):
            v = row[i]
            if sink and i == 0:
                return (0, 0.0, i)
            if np.isnan(v):
                return (2, 0.0, i)
            return (1, -float(v) + 0.0, i)

        want = sorted(range(n), key=key)[:k]
        if k > kt.BITONIC_MAX_K:
            want = sorted(want)
        assert list(got) == want

    check()


PF_GOLDEN = sorted(p.stem for p in (Path(__file__).resolve().parent / "golden").glob("pf_*.npz"))


@pytest.mark.parametrize("name", PF_GOLDEN)
def test_prefill_oracle_matches_reference_test_attention(name):
    """oracle.kernel_tree.prefill_attention against the reference test's own
    CPU attention (test_prefill_attention.py:17-40), which rounds its
    softmax to fp16 before P.V: equal within that rounding."""
    g = np.load(Path(__file__).resolve().parent / "golden" / f"{name}.npz")
    o, _ = kt.prefill_attention(g["q"], g["k"], g["v"], True)
    ref = g["out"].astype(np.float32)
    assert np.abs(o - ref).max() <= 2e-3 + 5e-3 * np.abs(ref).max()
    assert np.abs(o - ref).mean() < 2e-4
