"""GPU checks of the device-resident page table (aoakv_page_table_*,
aoakv_decode_step_table):

  * the device allocator against oracle/page_table.py (which reproduces the
    reference's KvCache page ids, tests/test_page_table_cpu.py) over appends,
    releases and a refused append, every page id and count compared;
  * a whole decode token (page-table append + the layer's step for every
    sequence) captured once as a CUDA graph and replayed for 30 tokens across
    page fills, outputs and selections checked token by token against
    oracle.kernel_tree.step on the same page ids."""
import numpy as np
import pytest
import torch

import aoa_kv_b200 as ak
from aoa_kv_b200 import _lib
from gen import gen_qkv
from gpu_util import ptr, stream
from helpers import selection_mismatch
from oracle import kernel_tree as kt
from oracle.page_table import PageTableOracle

pytestmark = pytest.mark.gpu


def check_same(pt: ak.DevicePageTable, orc: PageTableOracle):
    c = pt.counts()
    assert c["seq_len"] == orc.seq_len
    assert c["num_pages"] == [len(x) for x in orc.kv]
    assert c["meta_count"] == [len(x) for x in orc.meta]
    assert c["last_len"] == [orc.last_len(r) for r in range(orc.R)]
    assert c["kv_free"] == len(orc.kv_free) and c["meta_free"] == len(orc.meta_free)
    for r in range(orc.R):
        assert pt.kv_indices(r)[:len(orc.kv[r])].cpu().tolist() == orc.kv[r], r
        assert pt.metadata_indices(r)[:len(orc.meta[r])].cpu().tolist() == orc.meta[r], r


def test_device_allocator_matches_oracle(cuda):
    R, M, cap, mcap, P = 3, 40, 100, 8, 16
    pt = ak.DevicePageTable(R, M, cap, mcap, P)
    orc = PageTableOracle(R, M, cap, mcap, P)
    ops = [("a", 100, 0), ("a", 1, -1), ("a", 33, 2), ("a", 16, 1), ("a", 1, -1),
           ("r", 0, 1), ("a", 50, 1), ("a", 600, 0), ("a", 15, -1), ("r", 0, -1),
           ("a", 17, -1), ("a", 256, 2)]
    for kind, n, seq in ops:
        errors = orc.errors
        if kind == "a":
            pt.append(n, seq)
            orc.append(n, seq)
        else:
            pt.release(seq)
            orc.release(seq)
        torch.cuda.synchronize()
        dev = _lib.device_error()
        assert dev == (3 if orc.errors > errors else 0), (kind, n, seq)
        if orc.errors > errors:  # the host mirror assumed success: re-read it
            pt.sync_mirror()
            assert pt.seq_len == orc.seq_len
        check_same(pt, orc)
    pt.close()


@pytest.mark.parametrize("mode,sink", [("aoakv", False), ("quest", True)])
def test_table_decode_token_graph_matches_oracle(cuda, mode, sink):
    R, H, D, P, budget, T = 2, 8, 128, 16, 6, 30
    S0 = [100, 171]
    cap, mcap, M = 64, 8, 30
    g = np.random.default_rng(3)
    kv = torch.from_numpy(g.standard_normal((cap, 2, P, H, D), dtype=np.float32)
                          .astype(np.float16)).cuda()
    meta = torch.from_numpy(g.standard_normal((mcap, 2, P, H, D), dtype=np.float32)
                            .astype(np.float16)).cuda()
    vlog = torch.zeros(cap, H, dtype=torch.float16, device="cuda")
    pt = ak.DevicePageTable(R, M, cap, mcap, P)
    orc = PageTableOracle(R, M, cap, mcap, P)
    seqs = [gen_qkv(50 + r, H, S0[r] + T, D, "outlier") for r in range(R)]
    q_all = np.stack([np.stack([gen_qkv(900 + 31 * t + r, H, 1, D)[0] for r in range(R)])
                      for t in range(T)])                           # [T, R, H, D]
    for r in range(R):  # the prompts: page-table append, then the prefill append kernel
        pt.append(S0[r], r)
        orc.append(S0[r], r)
        n = pt.num_pages(r)
        nm = -(-n // P)
        K = torch.from_numpy(np.ascontiguousarray(seqs[r][1][:S0[r]])).cuda()
        V = torch.from_numpy(np.ascontiguousarray(seqs[r][2][:S0[r]])).cuda()
        _lib.call("aoakv_append_kv_cache_prefill", ptr(K), ptr(V), S0[r], ptr(kv),
                  ptr(pt.kv_indices(r)), n, pt.last_page_len(r), cap, ptr(meta),
                  ptr(pt.metadata_indices(r)), nm, (n - 1) % P + 1, mcap, ptr(vlog), H, D, P, 0,
                  stream())
    torch.cuda.synchronize()
    ref = kt.LayerCache(cap, H, D, P)
    ref.kv, ref.meta, ref.vlog = (x.cpu().numpy().copy() for x in (kv, meta, vlog))

    cols = max(3, budget) if sink else budget
    mode_id = _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST
    q_s = torch.empty(R, H, D, dtype=torch.float16, device="cuda")
    k_s, v_s, o_s = torch.empty_like(q_s), torch.empty_like(q_s), torch.empty_like(q_s)
    sel_s = torch.full((R, H, cols), -9, dtype=torch.int32, device="cuda")

    def token():
        pt.append(1)  # every sequence, on the device
        pt.decode_step(q_s, k_s, v_s, o_s, kv, meta, vlog, budget, mode_id, sink, sel_s)

    def load(t):
        q_s.copy_(torch.from_numpy(q_all[t]))
        k_s.copy_(torch.from_numpy(np.stack([seqs[r][1][S0[r] + t] for r in range(R)])))
        v_s.copy_(torch.from_numpy(np.stack([seqs[r][2][S0[r] + t] for r in range(R)])))

    outs, sels = [], []
    load(0)
    token()  # token 0 eagerly (first launch sets kernel attributes outside capture)
    outs.append(o_s.clone())
    sels.append(sel_s.clone())
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        graph.capture_begin()
        token()
        graph.capture_end()
    torch.cuda.current_stream().wait_stream(side)
    for t in range(1, T):
        load(t)
        graph.replay()
        pt.note_replayed(1)
        outs.append(o_s.clone())
        sels.append(sel_s.clone())
    torch.cuda.synchronize()
    pt.seq_len = [S0[r] + T for r in range(R)]  # capture advanced the mirror once more
    fills = 0
    for t in range(T):
        orc.append(1)
        for r in range(R):
            idx = np.array(orc.kv[r], np.int32)
            midx = np.array(orc.meta[r], np.int32)
            n, last = len(idx), orc.last_len(r)
            fills += last == 1
            q, kn, vn = q_all[t, r], seqs[r][1][S0[r] + t], seqs[r][2][S0[r] + t]
            want_o, want_sel = kt.step(q, kn, vn, ref, idx, midx, n, last, budget, mode, sink)
            got_o = outs[t][r].float().cpu().numpy()
            got_sel = sels[t][r].cpu().numpy()
            k = min(cols, n)
            assert np.all(got_sel[:, k - 1] == idx[n - 1]), (t, r)
            inv = {int(p): i for i, p in enumerate(idx)}
            g_log = np.array([sorted(inv[int(p)] for p in row[:k - 1]) for row in got_sel])
            w_log = np.array([sorted(inv[int(p)] for p in row[:k - 1]) for row in want_sel])
            if n > k:
                scores = kt.estimate(q, ref, midx, idx, n, mode)
                if sink:
                    scores[:, 0] = np.inf
                assert not selection_mismatch(g_log, w_log, scores), (t, r)
            o_ref = kt.sparse_decode(q, ref, got_sel[:, :k - 1].astype(np.int64), int(idx[n - 1]),
                                     last)
            assert np.abs(got_o - o_ref).max() < 2e-3, (t, r)
            if np.array_equal(g_log, w_log):
                assert np.abs(got_o - want_o).max() < 2e-3, (t, r)
    assert fills >= 3  # new pages allocated on the device inside the replayed graph
    check_same(pt, orc)
    assert _lib.device_error() == 0
    del graph
    pt.close()


def test_table_step_with_fused_rope_equals_rope_then_step(cuda):
    """RoPE fused into the page-table step (rope_scale > 0) gives the same bits
    as aoakv_apply_rope_in_place at each sequence's new-token position
    followed by the step without RoPE: outputs, selections, the caches after,
    and q and k left rotated in place."""
    R, H, D, P, budget = 2, 8, 128, 16, 6
    S0 = [100, 171]
    cap, mcap, M = 64, 8, 30
    runs = []
    for fused in (False, True):
        g = np.random.default_rng(5)
        kv = torch.from_numpy(g.standard_normal((cap, 2, P, H, D), dtype=np.float32)
                              .astype(np.float16)).cuda()
        meta = torch.from_numpy(g.standard_normal((mcap, 2, P, H, D), dtype=np.float32)
                                .astype(np.float16)).cuda()
        vlog = torch.zeros(cap, H, dtype=torch.float16, device="cuda")
        pt = ak.DevicePageTable(R, M, cap, mcap, P)
        for r in range(R):
            _, K, V = gen_qkv(70 + r, H, S0[r], D, "outlier")
            pt.append(S0[r], r)
            n = pt.num_pages(r)
            Kd, Vd = torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda()
            _lib.call("aoakv_append_kv_cache_prefill", ptr(Kd), ptr(Vd), S0[r], ptr(kv),
                      ptr(pt.kv_indices(r)), n, pt.last_page_len(r), cap, ptr(meta),
                      ptr(pt.metadata_indices(r)), -(-n // P), (n - 1) % P + 1, mcap, ptr(vlog),
                      H, D, P, 0, stream())
        q = torch.from_numpy(np.stack([gen_qkv(80 + r, H, 1, D)[0] for r in range(R)])).cuda()
        kn = torch.from_numpy(np.stack([gen_qkv(90 + r, H, 2, D)[1][0] for r in range(R)])).cuda()
        vn = torch.from_numpy(np.stack([gen_qkv(90 + r, H, 2, D)[2][0] for r in range(R)])).cuda()
        o = torch.empty_like(q)
        sel = torch.full((R, H, budget), -9, dtype=torch.int32, device="cuda")
        pt.append(1)
        if not fused:
            for r in range(R):  # the new token of sequence r sits at position S0[r]
                _lib.call("aoakv_apply_rope_in_place", ptr(q[r]), ptr(kn[r]), 1, S0[r], H, D,
                          1.0, 1e4, stream())
            pt.decode_step(q, kn, vn, o, kv, meta, vlog, budget, selected_out=sel)
        else:
            pt.decode_step(q, kn, vn, o, kv, meta, vlog, budget, selected_out=sel,
                           rope_scale=1.0, rope_theta=1e4)
        torch.cuda.synchronize()
        runs.append([x.cpu() for x in (o, sel, q, kn, kv, meta, vlog)])
        pt.close()
    for a, b in zip(*runs):
        assert torch.equal(a, b)
    assert _lib.device_error() == 0
