"""GPU parity of the batched step (aoakv_decode_step_batched: config 4's one
launch over (request, head)) against the kernel-tree oracle, request by
request: several requests of different lengths in ONE layer pool with CSR
page tables, including a request short enough to be attended densely and one
whose new token fills its last page."""
import numpy as np
import pytest
import torch

from aoa_kv_b200 import _lib
from gen import gen_qkv
from gpu_util import ptr, stream
from helpers import selection_mismatch
from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,sink,budget", [("aoakv", False, 16), ("quest", False, 8),
                                              ("aoakv", True, 16)])
def test_batched_step_matches_oracle(cuda, mode, sink, budget):
    H, D, P = 32, 128, 16
    lengths = [2000, 16 * 40, 300, 16 * 25 + 7, 120, 16 * 63]  # tokens incl. the new one
    R = len(lengths)
    pages = [(S + P - 1) // P for S in lengths]
    cap = sum(pages) + 3
    mcap = sum((n + P - 1) // P for n in pages) + 1
    g = np.random.default_rng(budget + 7 * sink)
    perm = g.permutation(cap).astype(np.int32)
    mperm = g.permutation(mcap).astype(np.int32)
    kv = torch.from_numpy(g.standard_normal((cap, 2, P, H, D), dtype=np.float32)
                          .astype(np.float16)).cuda()
    meta = torch.from_numpy(g.standard_normal((mcap, 2, P, H, D), dtype=np.float32)
                            .astype(np.float16)).cuda()
    vlog = torch.zeros(cap, H, dtype=torch.float16, device="cuda")
    kv_indptr, meta_indptr, kv_tab, meta_tab = [0], [0], [], []
    news = []
    o_kv, o_m = 0, 0
    for r, S in enumerate(lengths):
        n, nm = pages[r], (pages[r] + P - 1) // P
        kv_tab.append(perm[o_kv:o_kv + n])
        meta_tab.append(mperm[o_m:o_m + nm])
        o_kv += n
        o_m += nm
        kv_indptr.append(o_kv)
        meta_indptr.append(o_m)
        q, K, V = gen_qkv(100 + r, H, S, D, "outlier")
        news.append((q, K[-1], V[-1]))
        # prefill the first S-1 tokens of request r through its own page table
        n_pref = (S - 1 + P - 1) // P
        kt_d = torch.from_numpy(kv_tab[r]).cuda()
        mt_d = torch.from_numpy(meta_tab[r]).cuda()
        Kd, Vd = torch.from_numpy(K[:-1]).cuda(), torch.from_numpy(V[:-1]).cuda()
        _lib.call("aoakv_append_kv_cache_prefill", ptr(Kd), ptr(Vd), S - 1, ptr(kv), ptr(kt_d), n_pref,
                  (S - 2) % P + 1, cap, ptr(meta), ptr(mt_d), (n_pref + P - 1) // P,
                  (n_pref - 1) % P + 1, mcap, ptr(vlog), H, D, P, 0, stream())
        torch.cuda.synchronize()  # Kd, Vd, kt_d, mt_d are freed at the next iteration
    torch.cuda.synchronize()
    ref = kt.LayerCache(cap, H, D, P)
    ref.kv, ref.meta, ref.vlog = (t.cpu().numpy().copy() for t in (kv, meta, vlog))
    cols = max(3, budget) if sink else budget
    last_lens = np.array([(S - 1) % P + 1 for S in lengths], np.int32)
    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()
    # every device array stays referenced until the kernel has run: a freed
    # temporary's block would be handed to the next one
    q_all = dev(np.stack([x[0] for x in news]))
    k_all = dev(np.stack([x[1] for x in news]))
    v_all = dev(np.stack([x[2] for x in news]))
    kv_indptr_d = dev(np.array(kv_indptr, np.int32))
    kv_tab_d = dev(np.concatenate(kv_tab))
    last_d = dev(last_lens)
    meta_indptr_d = dev(np.array(meta_indptr, np.int32))
    meta_tab_d = dev(np.concatenate(meta_tab))
    o = torch.empty(R, H, D, dtype=torch.float16, device="cuda")
    sel = torch.full((R, H, cols), -9, dtype=torch.int32, device="cuda")
    score = _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST
    _lib.call("aoakv_decode_step_batched", ptr(q_all), ptr(k_all), ptr(v_all), ptr(o), ptr(kv),
              cap, ptr(kv_indptr_d), ptr(kv_tab_d), ptr(last_d), ptr(meta), mcap,
              ptr(meta_indptr_d), ptr(meta_tab_d), ptr(vlog), R, max(pages), H, D, P, budget,
              score, int(sink), ptr(sel), stream())
    torch.cuda.synchronize()
    got_o, got_sel = o.float().cpu().numpy(), sel.cpu().numpy()
    for r in range(R):
        n, last = pages[r], int(last_lens[r])
        q, kn, vn = news[r]
        want_o, want_sel = kt.step(q, kn, vn, ref, kv_tab[r], meta_tab[r], n, last, budget, mode,
                                   sink)
        k = min(cols, n)
        inv = {int(p): i for i, p in enumerate(kv_tab[r])}
        g_log = np.array([sorted(inv[int(p)] for p in row if p >= 0) for row in got_sel[r]])
        w_log = np.array([sorted(inv[int(p)] for p in row if p >= 0) for row in want_sel])
        assert g_log.shape == (H, k), r
        assert np.all(got_sel[r][:, k - 1] == kv_tab[r][n - 1]), r
        if n > k:
            scores = kt.estimate(q, ref, meta_tab[r], kv_tab[r], n, mode)
            scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
            if sink:
                scores[:, 0] = np.inf
            assert not selection_mismatch(g_log, w_log, scores), r
        else:
            assert np.array_equal(g_log, w_log), r
        phys = np.array([[int(p) for p in row[: k - 1]] for row in got_sel[r]], np.int64)
        o_ref = kt.sparse_decode(q, ref, phys.reshape(H, k - 1), int(kv_tab[r][n - 1]), last)
        assert np.abs(got_o[r] - o_ref).max() < 2e-3, r
        if np.array_equal(g_log, w_log):
            assert np.abs(got_o[r] - want_o).max() < 2e-3, r
    after_meta = meta.cpu().numpy()
    assert np.array_equal(after_meta, ref.meta)  # every request's append, as the oracle's
    assert _lib.device_error() == 0
