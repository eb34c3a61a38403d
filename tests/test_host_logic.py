"""Host-side page-table logic of the controller (no GPU): it must allocate,
count and budget pages exactly like quest.utils (kv_cache.py, controller.py)."""
import pytest
import torch

from aoa_kv_b200 import InferenceController, KvCache


def test_kvcache_append_and_last_page_len():
    c = KvCache(1, 2, 64, max_seq_len=100, page_size=16, dtype=torch.float16, device="cpu")
    assert c.append_seq(1) == 1 and c.seqlen == 1 and c.last_page_len == 1
    assert c.append_seq(15) == 0 and c.last_page_len == 16
    assert c.append_seq(1) == 1 and c.last_page_len == 1
    assert c.indicies == [0, 1]  # fresh pool: physical == logical
    c.release()
    assert c.seqlen == 0 and c.indicies == [] and c.pool.num_free_blocks == 7


def test_controller_budget_and_need_estimate():
    ic = InferenceController(2, 4, 64, 16, page_budget=4, max_seq_len=1024,
                             dtype=torch.float16, device="cpu")
    ic.prepare_metadata(100)          # 7 pages, last_page_len 4
    ic.begin_forward(100)
    ic.end_forward()
    ic.prepare_metadata(1)
    ic.begin_forward(1)
    assert len(ic.kv_cache.indicies) == 7 and ic.kv_cache.last_page_len == 5
    assert len(ic.metadata_cache.indicies) == 1 and ic.metadata_cache.last_page_len == 7
    assert ic.inference_page_budget == 4 and ic.need_estimate()
    assert ic.kv_indices_without_last.shape == (4, 6)
    assert ic.kv_indptr_for_approx_decode.tolist() == [0, 3]
    assert tuple(ic.topk_dindices_buffer.shape) == (4, 3)
    ic.set_page_budget(64)
    ic.begin_forward(1, updateTensor=False)
    assert ic.inference_page_budget == 7 and not ic.need_estimate()


def test_controller_sink_budget_follows_simulation():
    ic = InferenceController(1, 4, 64, 16, page_budget=64, max_seq_len=4096,
                             dtype=torch.float16, device="cpu", sink_first_page=True)
    ic.prepare_metadata(40)
    # simulation: token_budget = min(seq_len, budget) (quest_attention.py:326)
    assert ic.step_page_budget() == 40 // 16
    ic2 = InferenceController(1, 4, 64, 16, page_budget=64, max_seq_len=4096,
                              dtype=torch.float16, device="cpu")
    ic2.prepare_metadata(40)
    assert ic2.step_page_budget() == 64


def test_controller_rejects_non_fp16():
    with pytest.raises(RuntimeError, match="float16"):
        InferenceController(1, 4, 64, 16, 4, 128, torch.float32, "cpu")


def test_begin_forward_decode_needs_two_pages():
    ic = InferenceController(1, 4, 64, 16, 4, 128, torch.float16, "cpu")
    ic.prepare_metadata(1)
    with pytest.raises(AssertionError):
        ic.begin_forward(1)


def test_balance_requests_is_a_partition_and_balanced():
    from aoa_kv_b200 import batching
    import numpy as np
    g = np.random.default_rng(3)
    ctxs = [int(c) * 16 for c in g.integers(256, 1025, size=32)]
    w = [batching.step_bytes(c, 1024, 32, 128, 16) for c in ctxs]
    for n in (1, 2, 3, 4, 8):
        parts = batching.balance_requests(w, n)
        assert sorted(r for p in parts for r in p) == list(range(32))
        loads = [sum(w[r] for r in p) for p in parts]
        # LPT bound: no GPU above the mean by more than the largest request
        assert max(loads) <= sum(w) / n + max(w)
    assert batching.balance_requests([5, 5], 2) == [[0], [1]]


def test_step_bytes_matches_headline_figure():
    from aoa_kv_b200 import batching
    assert batching.step_bytes(32768, 1024, 32, 128, 16, "aoakv") == 50_462_656
    # dense when the context fits the budget: every page, no metadata
    assert batching.step_bytes(1024, 1024, 32, 128, 16) == 64 * 16 * 8192 * 2 + 16384
