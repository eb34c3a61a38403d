"""The drop-in ``quest`` package (aoa_kv_b200/quest_tree) imports without a
GPU and exposes the names the reference's code uses from quest.utils
(kernels/aoa_kv/quest/utils/__init__.py:11-23) and quest._kernels
(bsk_ops.cu:4-19), the way latency/bench_latency.py loads a kernel tree."""
import importlib
import sys
from pathlib import Path

import pytest

TREE = Path(__file__).resolve().parents[1] / "aoa_kv_b200" / "quest_tree"

UTILS_NAMES = ["InferenceController", "KvCache", "append_kv", "decode_estimate", "decode_topk",
               "decode_sparse_attn", "BatchDecodeWithPagedKVCacheWrapper", "TensorLayout",
               "prefill_forward", "apply_rope_in_place", "rms_norm_forward"]
KERNEL_NAMES = ["append_kv_cache_decode", "append_kv_cache_prefill", "estimate_attn_score",
                "topk_filtering", "BatchDecodeWithPagedKVCachePyTorchWrapper"]


@pytest.fixture()
def quest_tree():
    sys.path.insert(0, str(TREE))
    saved = {m: sys.modules.pop(m) for m in list(sys.modules)
             if m == "quest" or m.startswith("quest.")}
    try:
        yield importlib.import_module("quest")
    finally:
        for m in [m for m in sys.modules if m == "quest" or m.startswith("quest.")]:
            del sys.modules[m]
        sys.modules.update(saved)
        sys.path.remove(str(TREE))


def test_tree_resolves_inside_itself_and_exports_reference_names(quest_tree):
    assert Path(quest_tree.__file__).resolve().parents[1] == TREE
    utils = importlib.import_module("quest.utils")
    kernels = importlib.import_module("quest._kernels")
    for name in UTILS_NAMES:
        assert hasattr(utils, name), name
    for name in KERNEL_NAMES:
        assert hasattr(kernels, name), name


def test_prefill_is_the_library_op_and_the_model_is_not_provided(quest_tree):
    import aoa_kv_b200
    utils = importlib.import_module("quest.utils")
    kernels = importlib.import_module("quest._kernels")
    assert utils.prefill_forward is aoa_kv_b200.prefill_forward
    assert callable(kernels.prefill_with_paged_kv_cache)
    with pytest.raises(NotImplementedError):
        quest_tree.LlamaForCausalLM
