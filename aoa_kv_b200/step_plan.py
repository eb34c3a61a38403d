"""StepPlan: the per-layer decode step planned once (aoakv_step_plan_*).

Replaces the reference's BatchDecodeWithPagedKVCacheWrapper begin_forward /
forward / end_forward cycle (kernels/aoa_kv/quest/utils/decode_wrapper.py:11-82,
decode_handler.cuh:73-136), which re-plans with a device synchronisation and
an allocation on every step: the plan binds one layer's buffers and the
step's parameters once; run() only launches.
"""
from __future__ import annotations

import ctypes

from . import _lib


class StepPlan:
    """One layer's step plan. Buffers are raw device pointers (ints) or
    tensors; ``chain=True`` forces the four-kernel chain instead of the one
    cluster launch; ``shard=True`` plans a page-range shard of a longer
    sequence (aoakv_shard_propose / aoakv_shard_finish)."""

    def __init__(self, kv, kv_cap, meta, meta_cap, vlog, num_heads, head_dim, page_size,
                 page_budget, score_mode, sink_first_page=False, max_pages=0, max_ctas=0,
                 chain=False, shard=False):
        self._h = ctypes.c_void_p()
        self._lib = _lib.load()
        _lib.call("aoakv_step_plan_create", ctypes.byref(self._h), _addr(kv), int(kv_cap),
                  _addr(meta), int(meta_cap), _addr(vlog), int(num_heads), int(head_dim),
                  int(page_size), int(page_budget), int(score_mode), int(bool(sink_first_page)),
                  int(max_pages), int(max_ctas),
                  (_lib.PLAN_CHAIN if chain else 0) | (_lib.PLAN_SHARD if shard else 0))
        self.page_budget = int(page_budget)
        self.max_ctas = int(max_ctas)
        self.rope = None

    def run(self, q, k_new, v_new, o, kv_indices, num_kv_pages, kv_last_page_len,
            metadata_indices, selected=None, workspace=None, workspace_bytes=0, stream=None):
        _lib.call("aoakv_step_plan_run", self._h, _addr(q), _addr(k_new), _addr(v_new), _addr(o),
                  _addr(kv_indices), int(num_kv_pages), int(kv_last_page_len),
                  _addr(metadata_indices), _addr(selected), _addr(workspace),
                  int(workspace_bytes), stream)

    def set_rope(self, rope_scale: float = 1.0, rope_theta: float = 1e4):
        """Fuse RoPE into run(): q and k_new arrive unrotated and are left
        rotated in place (rope_scale <= 0 turns it off)."""
        _lib.call("aoakv_step_plan_set_rope", self._h, float(rope_scale), float(rope_theta))
        self.rope = (float(rope_scale), float(rope_theta)) if rope_scale > 0 else None

    def info(self, num_kv_pages, want_selected=False):
        """(kernels per step, CTAs per head of the cluster launch or 0)."""
        kern, clus = ctypes.c_int32(0), ctypes.c_int32(0)
        _lib.call("aoakv_step_plan_info", self._h, int(num_kv_pages), int(bool(want_selected)),
                  ctypes.byref(kern), ctypes.byref(clus))
        return int(kern.value), int(clus.value)

    def close(self):
        if self._h:
            self._lib.aoakv_step_plan_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def _addr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()
