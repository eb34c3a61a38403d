"""GPU parity of each kernel against the CPU oracle (semantics B), through the
C ABI. Bit-exact where the work is exact (KV copies, key max/min, top-k
selection on identical scores); fp tolerances stated per test."""
import numpy as np
import pytest
import torch

from aoa_kv_b200 import _lib
from gen import gen_qkv
from gpu_util import GpuLayer, ptr, stream
from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


# ----------------------------------------------------------------- a1 / a2
@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("S0", [0, 5, 15, 16, 37, 300])
def test_append_prefill_matches_oracle(cuda, D, S0):
    """Prefill of 45 tokens after S0 existing ones (ragged starts and ends)."""
    H, P, cap = 8, 16, 64
    lay = GpuLayer(cap, H, D, P, seed=S0 + D)
    q, K, V = gen_qkv(100 + S0, H, S0 + 45, D, "outlier")
    if S0:
        lay.fill(K[:S0], V[:S0])
    ref = lay.snapshot()
    S = S0 + 45
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay.append_prefill(_dev(K[S0:]), _dev(V[S0:]), n, last)
    kt.append_prefill(ref, lay.kv_idx_np, lay.meta_idx_np, n, last, K[S0:], V[S0:])
    torch.cuda.synchronize()
    got = lay.snapshot()
    assert np.array_equal(got.kv, ref.kv)
    assert np.array_equal(got.meta, ref.meta)
    np.testing.assert_allclose(got.vlog.astype(np.float32), ref.vlog.astype(np.float32),
                               rtol=0, atol=2e-3)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("entry", [0, 1, 7, 14, 15])
def test_append_decode_matches_oracle(cuda, entry):
    """One decode token landing at page entry `entry` (0 opens a page, 15 fills it)."""
    H, D, P, cap = 32, 128, 16, 64
    lay = GpuLayer(cap, H, D, P, seed=entry)
    S = 5 * P + entry + 1
    q, K, V = gen_qkv(200 + entry, H, S, D)
    lay.fill(K[:-1], V[:-1])
    ref = lay.snapshot()
    n, last = (S + P - 1) // P, (S - 1) % P + 1
    lay.append_decode(_dev(K[-1]), _dev(V[-1]), n, last)
    kt.append_decode(ref, lay.kv_idx_np, lay.meta_idx_np, n, last, K[-1], V[-1])
    torch.cuda.synchronize()
    got = lay.snapshot()
    assert np.array_equal(got.kv, ref.kv)
    assert np.array_equal(got.meta, ref.meta)
    np.testing.assert_allclose(got.vlog.astype(np.float32), ref.vlog.astype(np.float32),
                               rtol=0, atol=2e-3)


# ----------------------------------------------------------------------- a3
@pytest.mark.parametrize("mode", ["quest", "aoakv"])
@pytest.mark.parametrize("S", [17, 33, 300, 8192 + 5])
@pytest.mark.parametrize("out_f32", [True, False])
def test_estimate_matches_oracle(cuda, mode, S, out_f32):
    H, D, P = 32, 128, 16
    n = (S + P - 1) // P
    lay = GpuLayer(n + 3, H, D, P, seed=S)
    q, K, V = gen_qkv(300 + S, H, S, D, "outlier")
    lay.fill(K, V)
    torch.cuda.synchronize()
    ref = lay.snapshot()
    qd = _dev(q)
    out = torch.full((H, n - 1), float("nan"), device="cuda",
                     dtype=torch.float32 if out_f32 else torch.float16)
    _lib.call("aoakv_estimate_attn_score", ptr(qd), ptr(out), 1 if out_f32 else 0, n - 1,
              ptr(lay.meta), ptr(lay.meta_idx), (n + P - 1) // P, (n - 1) % P + 1, lay.mcap,
              ptr(lay.kv_idx), lay.cap, ptr(lay.vlog), H, D, P, 0,
              _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST, stream())
    want = kt.estimate(q, ref, lay.meta_idx_np, lay.kv_idx_np, n, mode)
    got = out.float().cpu().numpy()
    if out_f32:
        np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-4)
    else:  # one fp16 rounding of the fp32 score
        np.testing.assert_allclose(got, want.astype(np.float16).astype(np.float32),
                                   rtol=2e-3, atol=2e-3)


# ----------------------------------------------------------------------- a4
@pytest.mark.parametrize("n,k", [(1, 1), (7, 3), (63, 63), (511, 63), (2047, 63), (2047, 1),
                                 (8191, 255), (49152, 1000), (100, 99)])
@pytest.mark.parametrize("f32", [True, False])
@pytest.mark.parametrize("sink", [False, True])
def test_topk_exact(cuda, n, k, f32, sink):
    rows = 32
    g = np.random.default_rng(n * 7 + k)
    s = g.standard_normal((rows, n), dtype=np.float32) * 10
    s[:, ::5] = np.round(s[:, ::5])           # ties
    if n > 10:
        s[3, 4] = np.nan
        s[5, :] = 1.0                          # an all-tie row
    if n > 20:
        s[7, :] = 1.0 + g.random(n, dtype=np.float32) * 1e-3   # one histogram bin, distinct
        s[9, :] = np.round(g.standard_normal(n) * 3)          # integer ties across bins
        s[11, :] = 100 + g.standard_normal(n) * 0.5           # a few crowded bins
    if not f32:
        s = s.astype(np.float16).astype(np.float32)
    idx = np.stack([g.permutation(10 * n)[:n] for _ in range(rows)]).astype(np.int32)
    sd = torch.from_numpy(s).cuda().to(torch.float32 if f32 else torch.float16)
    idd = torch.from_numpy(idx).cuda()
    out_i = torch.full((rows, k), -7, dtype=torch.int32, device="cuda")
    out_v = torch.empty((rows, k), dtype=sd.dtype, device="cuda")
    _lib.call("aoakv_topk_filtering", ptr(sd), 1 if f32 else 0, n, ptr(idd), n, rows, n, k,
              ptr(out_v), k, ptr(out_i), k, int(sink), stream())
    pos = kt.topk_positions(s, k, sink)
    want_i = np.take_along_axis(idx, pos, axis=1)
    assert np.array_equal(out_i.cpu().numpy(), want_i)
    got_v = out_v.float().cpu().numpy()
    want_v = np.take_along_axis(s, pos, axis=1)
    assert np.array_equal(np.isnan(got_v), np.isnan(want_v))
    assert np.array_equal(np.nan_to_num(got_v), np.nan_to_num(want_v))


def test_topk_shared_index_row_and_positions(cuda):
    rows, n, k = 4, 300, 20
    s = torch.randn(rows, n, device="cuda")
    shared = torch.arange(1000, 1000 + n, dtype=torch.int32, device="cuda")
    o1 = torch.empty(rows, k, dtype=torch.int32, device="cuda")
    o2 = torch.empty(rows, k, dtype=torch.int32, device="cuda")
    _lib.call("aoakv_topk_filtering", ptr(s), 1, n, ptr(shared), 0, rows, n, k, None, 0, ptr(o1),
              k, 0, stream())
    _lib.call("aoakv_topk_filtering", ptr(s), 1, n, None, 0, rows, n, k, None, 0, ptr(o2), k, 0,
              stream())
    assert torch.equal(o1 - 1000, o2)
    pos = kt.topk_positions(s.cpu().numpy(), k)
    assert np.array_equal(o2.cpu().numpy(), pos)


# ----------------------------------------------------------------------- a5
@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("n_sel", [0, 1, 3, 8, 63, 255])
@pytest.mark.parametrize("last_len", [1, 7, 16])
def test_sparse_decode_matches_oracle(cuda, D, n_sel, last_len):
    H, P, cap = 32, 16, 600
    lay = GpuLayer(cap, H, D, P, seed=n_sel + last_len)
    g = np.random.default_rng(n_sel * 31 + last_len)
    sel = np.stack([g.permutation(cap - 1)[:n_sel] for _ in range(H)]).astype(np.int32)
    last = cap - 1
    q = g.standard_normal((H, D), dtype=np.float32).astype(np.float16) * np.float16(3)
    ref = lay.snapshot()
    qd, o = _dev(q), torch.empty(H, D, dtype=torch.float16, device="cuda")
    seld = torch.from_numpy(sel).cuda() if n_sel else None
    ws_n = _lib.size_query("aoakv_decode_workspace_size", H, D, n_sel)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    for _ in range(2):  # second call reuses the workspace (tickets re-armed)
        _lib.call("aoakv_sparse_decode", ptr(qd), ptr(o), ptr(lay.kv), cap, ptr(seld), n_sel, n_sel,
                  last, last_len, H, D, P, 0, 0.0, ptr(ws), ws_n, stream())
        want = kt.sparse_decode(q, ref, sel, last, last_len)
        got = o.float().cpu().numpy()
        assert np.abs(got - want).max() < 2e-3
    assert _lib.device_error() == 0


@pytest.mark.parametrize("n_parts", [1, 2, 3])
@pytest.mark.parametrize("n_sel", [0, 5, 63])
def test_partial_decode_and_merge_equal_full_decode(cuda, n_parts, n_sel):
    """aoakv_sparse_decode_partial over disjoint page subsets (-1 = page not
    here; the last page on one part only) merged by aoakv_merge_states gives
    the full decode; a part with no pages has lse = -inf."""
    H, D, P, cap = 32, 128, 16, 200
    lay = GpuLayer(cap, H, D, P, seed=7 + n_sel)
    ref = lay.snapshot()
    g = np.random.default_rng(n_sel + 10 * n_parts)
    sel = np.stack([g.permutation(cap - 1)[:n_sel] for _ in range(H)]).astype(np.int32)
    last, last_len = cap - 1, 11
    q = g.standard_normal((H, D), dtype=np.float32).astype(np.float16)
    qd = _dev(q)
    owner = g.integers(0, n_parts, size=sel.shape)  # which part holds each selected page
    o_parts = torch.empty(n_parts, H, D, dtype=torch.float32, device="cuda")
    lse_parts = torch.empty(n_parts, H, dtype=torch.float32, device="cuda")
    ws_n = _lib.size_query("aoakv_decode_workspace_size", H, D, max(n_sel, 1))
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    for p in range(n_parts):
        mine = np.where(owner == p, sel, -1).astype(np.int32)
        md = _dev(mine) if n_sel else None
        _lib.call("aoakv_sparse_decode_partial", ptr(qd), ptr(o_parts[p]), ptr(lse_parts[p]),
                  ptr(lay.kv), cap, ptr(md), n_sel, n_sel, last if p == n_parts - 1 else -1,
                  last_len, H, D, P, 0, 0.0, ptr(ws), ws_n, stream())
    o = torch.empty(H, D, dtype=torch.float16, device="cuda")
    lse = torch.empty(H, dtype=torch.float32, device="cuda")
    _lib.call("aoakv_merge_states", ptr(o_parts), ptr(lse_parts), n_parts, H, D, ptr(o), ptr(lse),
              stream())
    want = kt.sparse_decode(q, ref, sel, last, last_len)
    assert np.abs(o.float().cpu().numpy() - want).max() < 2e-3
    # lse of the whole set, from the oracle's pages
    Kf = [np.concatenate([ref.kv[pg, 0, :, h] for pg in sel[h]] + [ref.kv[last, 0, :last_len, h]])
          .astype(np.float32) for h in range(H)]
    want_lse = np.array([np.log(np.exp(k @ q[h].astype(np.float32) / np.sqrt(D)).sum())
                         for h, k in enumerate(Kf)])
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=1e-3, atol=1e-3)
    if n_sel == 0 and n_parts > 1:
        assert np.all(np.isneginf(lse_parts[0].cpu().numpy()))
        assert np.all(o_parts[0].cpu().numpy() == 0)
    assert _lib.device_error() == 0


def test_sparse_decode_shared_row_and_bad_page(cuda):
    """Stride-0 index row (dense decode over a shared page list), then a page
    id beyond capacity: skipped and reported, no fault."""
    H, D, P, cap = 8, 128, 16, 64
    lay = GpuLayer(cap, H, D, P, seed=3)
    ref = lay.snapshot()
    rows = np.arange(40, dtype=np.int32)
    q = np.random.default_rng(1).standard_normal((H, D), dtype=np.float32).astype(np.float16)
    qd, o = _dev(q), torch.empty(H, D, dtype=torch.float16, device="cuda")
    ws_n = _lib.size_query("aoakv_decode_workspace_size", H, D, 40)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    rows_d = _dev(rows)
    _lib.call("aoakv_sparse_decode", ptr(qd), ptr(o), ptr(lay.kv), cap, ptr(rows_d), 0, 40, 50,
              9, H, D, P, 0, 0.0, ptr(ws), ws_n, stream())
    want = kt.sparse_decode(q, ref, rows, 50, 9)
    assert np.abs(o.float().cpu().numpy() - want).max() < 2e-3
    assert _lib.device_error() == 0
    bad = rows.copy()
    bad[3] = cap + 5
    bad_d = _dev(bad)
    _lib.call("aoakv_sparse_decode", ptr(qd), ptr(o), ptr(lay.kv), cap, ptr(bad_d), 0, 40, 50,
              9, H, D, P, 0, 0.0, ptr(ws), ws_n, stream())
    keep = np.delete(rows, 3)
    want = kt.sparse_decode(q, ref, keep, 50, 9)
    assert np.abs(o.float().cpu().numpy() - want).max() < 2e-3
    assert _lib.device_error() == 1  # AOAKV_DEV_ERR_BAD_PAGE, then cleared
    assert _lib.device_error() == 0


# -------------------------------------------------------------------- RoPE
@pytest.mark.parametrize("N,past,D", [(1, 0, 128), (1, 8191, 128), (37, 100, 128), (5, 3000, 64)])
def test_apply_rope_in_place_matches_oracle(cuda, N, past, D):
    """utils/__init__.py:25-52 semantics: q and k rotated in place. Positions
    stay below ~8K here: the angle is an fp32 product (as in the reference),
    so at 100K+ one ulp of the frequency moves the angle by ~1e-2 rad."""
    H = 8
    g = np.random.default_rng(N * 31 + past)
    q = g.standard_normal((N, H, D)).astype(np.float16)
    k = g.standard_normal((N, H, D)).astype(np.float16)
    qd, kd = _dev(q), _dev(k)
    _lib.call("aoakv_apply_rope_in_place", ptr(qd), ptr(kd), N, past, H, D, 1.0, 1e4, stream())
    torch.cuda.synchronize()
    for got, x in ((qd, q), (kd, k)):
        want = kt.apply_rope(x, past).astype(np.float32)
        np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=2e-3, atol=3e-3)


def test_apply_rope_zero_position_is_identity(cuda):
    q = torch.randn(3, 4, 128, device="cuda").half()
    k = torch.randn(3, 4, 128, device="cuda").half()
    q0, k0 = q[:1].clone(), k[:1].clone()
    _lib.call("aoakv_apply_rope_in_place", ptr(q), ptr(k), 3, 0, 4, 128, 1.0, 1e4, stream())
    torch.cuda.synchronize()
    assert torch.equal(q[:1], q0) and torch.equal(k[:1], k0)  # position 0: angle 0


# ----------------------------------------------------------------- RMSNorm
@pytest.mark.parametrize("rows,cols", [(1, 4096), (7, 128), (3, 8)])
def test_rms_norm_matches_numpy(cuda, rows, cols):
    """rms_norm.cu semantics: fp32 mean of squares, out = x * rsqrt(. + eps) * w."""
    g = np.random.default_rng(rows + cols)
    x = (g.standard_normal((rows, cols)) * 3).astype(np.float16)
    w = g.standard_normal(cols).astype(np.float16)
    o = torch.empty(rows, cols, dtype=torch.float16, device="cuda")
    xd, wd = _dev(x), _dev(w)  # keep both alive: a freed temporary's block is reused
    _lib.call("aoakv_rms_norm", ptr(xd), ptr(wd), ptr(o), rows, cols, 1e-5, stream())
    xf = x.astype(np.float32)
    r = 1.0 / np.sqrt((xf * xf).mean(axis=1, keepdims=True) + 1e-5)
    want = (xf * r * w.astype(np.float32)).astype(np.float16).astype(np.float32)
    np.testing.assert_allclose(o.float().cpu().numpy(), want, rtol=2e-3, atol=2e-3)
