"""aoa_kv_b200 — B200 (sm_100a) sparse-decode path of AOA-KV / Quest.

Public surface, named after the reference's quest.utils
(kernels/aoa_kv/quest/utils/__init__.py:11-23):

    TensorLayout, KvCache, InferenceController, BatchDecodeWithPagedKVCacheWrapper,
    append_kv, decode_estimate, decode_topk, decode_sparse_attn,
    apply_rope_in_place, rms_norm_forward, prefill_forward

plus ``topk_filtering`` (the raw top-k op),
``InferenceController.decode_step`` (append + estimate + top-k + decode in one
library call) and ``StepPlan`` (that step planned once per layer). The kernels live in libaoakv.so (C ABI: include/aoakv.h).
"""
from . import _lib
from ._lib import AoaKvError, check_device, device_error
from .controller import InferenceController, KvCache, KvPool, TensorLayout
from .decode_wrapper import BatchDecodeWithPagedKVCacheWrapper
from .ops import (append_kv, apply_rope_in_place, decode_estimate, decode_sparse_attn,
                  decode_topk, prefill_forward, prefill_with_paged_kv_cache, rms_norm_forward,
                  topk_filtering)
from .page_table import DevicePageTable
from .step_plan import StepPlan

__all__ = [
    "TensorLayout", "KvCache", "KvPool", "InferenceController",
    "BatchDecodeWithPagedKVCacheWrapper", "append_kv", "prefill_forward",
    "prefill_with_paged_kv_cache", "decode_estimate",
    "decode_topk", "decode_sparse_attn", "rms_norm_forward", "apply_rope_in_place",
    "topk_filtering", "StepPlan", "DevicePageTable", "AoaKvError", "check_device",
    "device_error",
]


def library_path() -> str:
    return str(_lib.LIB_PATH)
