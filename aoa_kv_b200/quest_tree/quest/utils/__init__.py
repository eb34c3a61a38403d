"""quest.utils names (kernels/aoa_kv/quest/utils/__init__.py:11-23) backed by
aoa_kv_b200. InferenceController defaults its scoring mode to the tree's
AOAKV_SCORE_MODE."""
import functools

import quest._kernels as _kernels  # noqa: F401  (quest/tests/test_topk.py uses it)

from aoa_kv_b200 import (BatchDecodeWithPagedKVCacheWrapper, KvCache, TensorLayout, append_kv,
                         apply_rope_in_place, decode_estimate, decode_sparse_attn, decode_topk,
                         prefill_forward, rms_norm_forward)
from aoa_kv_b200 import InferenceController as _IC

__all__ = [
    "TensorLayout", "KvCache", "InferenceController", "BatchDecodeWithPagedKVCacheWrapper",
    "append_kv", "prefill_forward", "decode_estimate", "decode_topk", "decode_sparse_attn",
    "rms_norm_forward", "apply_rope_in_place",
]


class InferenceController(_IC):
    """controller.py:7-163 with the tree's scoring mode as default."""

    @functools.wraps(_IC.__init__)
    def __init__(self, *args, method=None, **kwargs):
        super().__init__(*args, method=method or _kernels.SCORE_MODE, **kwargs)
