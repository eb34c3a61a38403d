"""The reference's own test flows (kernels/aoa_kv/quest/tests/*.py) run
through the drop-in surface (InferenceController + append_kv /
decode_estimate / decode_topk / decode_sparse_attn), checked against the
golden vectors the reference's CPU references produced, with the reference's
fp16 tolerance (rtol = atol = 5e-3, test_estimate.py:9-15) and against the
oracle at 2e-3."""
import numpy as np
import pytest
import torch

import aoa_kv_b200 as ak
from gen import digest, gen_qkv
from helpers import golden_names, load_golden, selection_mismatch
from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu


def assert_close(a, b):
    torch.testing.assert_close(a, b, rtol=5e-3, atol=5e-3)


def prefill_then_decode(meta, page_budget, max_seq_len=8192, method="quest", sink=False):
    """test_estimate.py:108-134 / test_approx_attention.py:150-176."""
    H, S, D, P = meta["H"], meta["S"], meta["D"], meta["P"]
    q, K, V = gen_qkv(meta["seed"], H, S, D, meta.get("dist", "normal"))
    assert digest(q, K, V) == meta["digest"]
    dev = torch.device("cuda:0")
    ctl = ak.InferenceController(32, H, D, P, page_budget, max_seq_len, torch.float16, dev,
                                 method=method, sink_first_page=sink)
    kp, vp = torch.from_numpy(K[:-1]).to(dev), torch.from_numpy(V[:-1]).to(dev)
    ctl.prepare_metadata(S - 1)
    ctl.begin_forward(S - 1)
    ak.append_kv(kp, vp, ctl, 0)
    ctl.end_forward()
    ctl.prepare_metadata(1)
    ctl.begin_forward(1)
    ak.append_kv(torch.from_numpy(K[-1:]).to(dev), torch.from_numpy(V[-1:]).to(dev), ctl, 0)
    return ctl, torch.from_numpy(q)[None].to(dev), (q, K, V)


@pytest.mark.parametrize("name", golden_names("kt_est_"))
def test_reference_estimate_flow(cuda, name):
    meta, g = load_golden(name)
    ctl, q, _ = prefill_then_decode(meta, 1024)
    est = ak.decode_estimate(q, ctl, 0)
    ctl.end_forward()
    assert est.dtype == torch.float16 and tuple(est.shape) == g["est"].shape
    assert_close(est.cpu(), torch.from_numpy(g["est"]))


@pytest.mark.parametrize("name", golden_names("kt_approx_"))
def test_reference_approx_attention_flow(cuda, name):
    meta, g = load_golden(name)
    ctl, q, (qn, K, V) = prefill_then_decode(meta, meta["page_budget"], max_seq_len=2048)
    if not ctl.need_estimate():
        o = ak.decode_sparse_attn(q, ctl, 0, ctl.kv_indices_without_last)
    else:
        idx = torch.from_numpy(g["topk"]).cuda()
        o = ak.decode_sparse_attn(q, ctl, 0, idx)
    ctl.end_forward()
    assert_close(o[0].cpu(), torch.from_numpy(g["out"]))


@pytest.mark.parametrize("name", golden_names("kt_approx_"))
def test_estimate_topk_decode_chain_selects_reference_pages(cuda, name):
    """decode_estimate -> decode_topk picks the reference's pages (up to
    near-ties of the fp16 scores) and the chained output matches."""
    meta, g = load_golden(name)
    if "topk" not in g:
        pytest.skip("dense case")
    ctl, q, _ = prefill_then_decode(meta, meta["page_budget"], max_seq_len=2048)
    est = ak.decode_estimate(q, ctl, 0)
    ak.decode_topk(est, ctl)
    got = ctl.topk_dindices_buffer.cpu().numpy()
    assert not selection_mismatch(got, g["topk"], est.float().cpu().numpy(), rtol=2e-3)
    vals = ctl.topk_dout_buffer.float().cpu().numpy()
    ref_vals = np.take_along_axis(est.float().cpu().numpy(), got, axis=1)
    assert np.array_equal(vals, ref_vals)
    o = ak.decode_sparse_attn(q, ctl, 0, ctl.topk_dindices_buffer)
    ctl.end_forward()
    if np.array_equal(np.sort(got, 1), np.sort(g["topk"], 1)):
        assert_close(o[0].cpu(), torch.from_numpy(g["out"]))


@pytest.mark.parametrize("name", golden_names("kt_vlog_"))
def test_reference_vlog_prefill_flow(cuda, name):
    """test_v_log_norm_prefill_claude.py:175-257 with a strict tolerance."""
    meta, g = load_golden(name)
    H, S, D, P = meta["H"], meta["S"], meta["D"], meta["P"]
    q, K, V = gen_qkv(meta["seed"], H, S, D)
    ctl = ak.InferenceController(2, H, D, P, 1024, 8192, torch.float16, torch.device("cuda:0"))
    ctl.prepare_metadata(S)
    ctl.begin_forward(S)
    ak.append_kv(torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(), ctl, 0)
    ctl.end_forward()
    nf = S // P
    got = ctl.v_log_norm_layer(0)[:nf].float().cpu().numpy()
    np.testing.assert_allclose(got, g["vlog"], rtol=0, atol=2e-3)


@pytest.mark.parametrize("kv_len", [13, 24, 51, 77, 244, 311, 502, 1110])
@pytest.mark.parametrize("k_budget", [2, 5, 7, 19, 31, 69, 111, 251])
def test_reference_topk_flow(cuda, kv_len, k_budget):
    """test_topk.py:22-64: the selected values sum like torch.topk's."""
    if k_budget > kv_len:
        pytest.skip("k should be less than kv_len")
    g = torch.Generator(device="cuda").manual_seed(kv_len * 1000 + k_budget)
    H, D = 32, 128
    q = torch.randn(H, 1, D, dtype=torch.float16, device="cuda", generator=g)
    k = torch.randn(H, kv_len, D, dtype=torch.float16, device="cuda", generator=g)
    w = torch.matmul(q, k.transpose(1, 2)) / np.sqrt(D)
    want = torch.topk(w, k=k_budget, dim=-1).values.sum(dim=-1).squeeze()
    idx = torch.arange(0, kv_len, dtype=torch.int32, device="cuda").repeat(H, 1)
    out_d = torch.randn(H, k_budget, dtype=torch.float16, device="cuda")
    out_i = torch.arange(0, k_budget, dtype=torch.int32, device="cuda").repeat(H, 1)
    ak.topk_filtering(w.squeeze().contiguous(), idx, out_d, out_i, k_budget)
    assert_close(out_d.sum(dim=-1).squeeze(), want)


@pytest.mark.parametrize("method", ["aoakv", "quest"])
@pytest.mark.parametrize("sink", [False, True])
def test_controller_decode_step_matches_oracle(cuda, method, sink):
    """InferenceController.decode_step (one library call per layer) over
    several layers and tokens vs the kernel-tree oracle."""
    H, D, P, L, B = 32, 128, 16, 3, 8
    S0 = 700
    q, K, V = gen_qkv(5, H, S0 + 3, D, "outlier")
    dev = torch.device("cuda:0")
    ctl = ak.InferenceController(L, H, D, P, B, 1024, torch.float16, dev, method=method,
                                 sink_first_page=sink)
    ctl.prepare_metadata(S0)
    ctl.begin_forward(S0)
    for layer in range(L):
        ak.append_kv(torch.from_numpy(K[:S0]).to(dev), torch.from_numpy(V[:S0]).to(dev), ctl, layer)
    ctl.end_forward()
    torch.cuda.synchronize()
    refs = []
    for layer in range(L):
        c = kt.LayerCache(ctl.kv_cache.pool.capacity, H, D, P)
        c.kv = ctl.kv_cache.buf_layer(layer).cpu().numpy().copy()
        c.meta = ctl.metadata_cache.buf_layer(layer).cpu().numpy().copy()
        c.vlog = ctl.v_log_norm_layer(layer).cpu().numpy().copy()
        refs.append(c)
    for t in range(S0, S0 + 3):
        ctl.prepare_metadata(1)
        ctl.begin_forward(1)
        idx = np.array(ctl.kv_cache.indicies, dtype=np.int32)
        midx = np.array(ctl.metadata_cache.indicies, dtype=np.int32)
        n, last = len(idx), ctl.kv_cache.last_page_len
        qd = torch.from_numpy(q).to(dev)[None]
        kd, vd = torch.from_numpy(K[t:t + 1]).to(dev), torch.from_numpy(V[t:t + 1]).to(dev)
        for layer in range(L):
            o = ctl.decode_step(qd, kd, vd, layer)
            want, _ = kt.step(q, K[t], V[t], refs[layer], idx, midx, n, last,
                              ctl.step_page_budget(), method, sink)
            assert np.abs(o[0].float().cpu().numpy() - want).max() < 2e-3
        ctl.end_forward()
    assert ak.device_error() == 0
