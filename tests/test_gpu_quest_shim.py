"""The drop-in ``quest`` tree (aoa_kv_b200/quest_tree) used exactly the way
the reference's tests use quest.utils / quest.utils._kernels
(kernels/aoa_kv/quest/tests/test_approx_attention.py:112-199,
test_topk.py:22-64, test_decode_attention.py:46-99), in the quest_orig
scoring mode, checked against the kernel-tree oracle."""
import importlib
import math
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu
TREE = Path(__file__).resolve().parents[1] / "aoa_kv_b200" / "quest_tree"


@pytest.fixture(scope="module")
def quest():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    os.environ["AOAKV_SCORE_MODE"] = "quest"
    sys.path.insert(0, str(TREE))
    for m in [m for m in sys.modules if m == "quest" or m.startswith("quest.")]:
        del sys.modules[m]
    mod = importlib.import_module("quest")
    importlib.import_module("quest.utils")
    assert Path(mod.__file__).resolve().parents[1] == TREE
    yield mod
    sys.path.remove(str(TREE))
    os.environ.pop("AOAKV_SCORE_MODE", None)


def assert_close(a, b):
    torch.testing.assert_close(a, b, rtol=5e-3, atol=5e-3)


@pytest.mark.parametrize("kv_len,page_budget", [(27, 4), (482, 15), (1541, 31), (577, 71)])
def test_shim_estimate_topk_decode(quest, kv_len, page_budget):
    dtype, device = torch.float16, torch.device("cuda:0")
    H, D, L, P = 32, 128, 32, 16
    g = torch.Generator(device=device).manual_seed(kv_len)
    q = torch.randn(1, H, D, dtype=dtype, device=device, generator=g)
    k_pre = torch.randn(kv_len - 1, H, D, dtype=dtype, device=device, generator=g)
    v_pre = torch.randn(kv_len - 1, H, D, dtype=dtype, device=device, generator=g)
    ctl = quest.utils.InferenceController(L, H, D, P, page_budget, 2048, dtype, device)
    assert ctl.method == "quest"
    ctl.prepare_metadata(kv_len - 1)
    ctl.begin_forward(kv_len - 1)
    quest.utils.append_kv(k_pre, v_pre, ctl, 0)
    ctl.end_forward()
    k_dec = torch.randn(1, H, D, dtype=dtype, device=device, generator=g)
    v_dec = torch.randn(1, H, D, dtype=dtype, device=device, generator=g)
    ctl.prepare_metadata(1)
    ctl.begin_forward(1)
    quest.utils.append_kv(k_dec, v_dec, ctl, 0)
    torch.cuda.synchronize()
    n = len(ctl.kv_cache.indicies)
    ref = kt.LayerCache(ctl.kv_cache.pool.capacity, H, D, P)
    ref.kv = ctl.kv_cache.buf_layer(0).cpu().numpy()
    ref.meta = ctl.metadata_cache.buf_layer(0).cpu().numpy()
    idx = np.arange(n, dtype=np.int32)
    if ctl.need_estimate():
        est = quest.utils.decode_estimate(q, ctl, 0)
        want = kt.estimate(q[0].cpu().numpy(), ref, idx, idx, n, "quest")
        assert_close(est.float().cpu(), torch.from_numpy(want))
        quest.utils.decode_topk(est, ctl)
        sel = ctl.topk_dindices_buffer
        o = quest.utils.decode_sparse_attn(q, ctl, 0, sel)
        want_o = kt.sparse_decode(q[0].cpu().numpy(), ref, sel.cpu().numpy(), n - 1,
                                  ctl.kv_cache.last_page_len)
    else:
        o = quest.utils.decode_sparse_attn(q, ctl, 0, ctl.kv_indices_without_last)
        want_o = kt.sparse_decode(q[0].cpu().numpy(), ref, idx[:-1], n - 1,
                                  ctl.kv_cache.last_page_len)
    ctl.end_forward()
    assert np.abs(o[0].float().cpu().numpy() - want_o).max() < 2e-3


def test_shim_kernels_topk(quest):
    dtype, device = torch.float16, torch.device("cuda:0")
    H, D, kv_len, kb = 32, 128, 502, 31
    q = torch.randn(H, 1, D, dtype=dtype, device=device)
    k = torch.randn(H, kv_len, D, dtype=dtype, device=device)
    w = torch.matmul(q, k.transpose(1, 2)) / math.sqrt(D)
    want = torch.topk(w, k=kb, dim=-1).values.sum(dim=-1).squeeze()
    out_d = torch.randn(H, kb, dtype=dtype, device=device)
    out_i = torch.arange(0, kb, dtype=torch.int32, device=device).repeat(H, 1)
    buf = torch.zeros((H, 8192 * 2 * (2 + 4) // 2 // 48), dtype=dtype, device=device)
    idx = torch.arange(0, kv_len, dtype=torch.int32, device=device).repeat(H, 1)
    quest.utils._kernels.topk_filtering(w.squeeze(), idx, out_d, out_i, buf, kb)
    assert_close(out_d.sum(dim=-1).squeeze(), want)


def test_shim_model_is_not_built(quest):
    with pytest.raises(NotImplementedError):
        quest.LlamaForCausalLM  # noqa: B018
