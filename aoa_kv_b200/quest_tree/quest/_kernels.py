"""Module-level functions with the names and arguments of the reference's
pybind extension ``quest._kernels`` (kernels/aoa_kv/quest/ops/csrc/bsk_ops.cu:4-19,
signatures bsk_ops.h:23-125), each forwarding to libaoakv.so's C ABI.

Differences, all documented in include/aoakv.h:
  * estimate_attn_score takes an optional ``kv_indices`` keyword so the
    value term reads the page's own v_log_norm; without it, physical page id
    == logical page id is assumed (a fresh KvPool hands out pages in order).
  * topk_filtering ignores ``buf`` (no scratch is needed) and any head count
    is accepted (the reference asserts 32, topk.cu:28).
  * prefill_with_paged_kv_cache runs the tcgen05 prefill kernel; like the
    reference (RotaryMode::kNone) it applies no RoPE.
"""
from __future__ import annotations

import os

import torch

from aoa_kv_b200 import _lib
from aoa_kv_b200 import ops as _ops
from aoa_kv_b200.decode_wrapper import BatchDecodeWithPagedKVCacheWrapper as _Wrapper

SCORE_MODE = os.environ.get("AOAKV_SCORE_MODE", "aoakv")
if SCORE_MODE not in ("aoakv", "quest"):
    raise ValueError(f"AOAKV_SCORE_MODE must be 'aoakv' or 'quest', got {SCORE_MODE!r}")


def _mode() -> int:
    return _lib.SCORE_AOAKV if SCORE_MODE == "aoakv" else _lib.SCORE_QUEST


def topk_filtering(estimated_value, estimated_indices, d_out, indices_out, buf, page_budget):
    _ops.topk_filtering(estimated_value, estimated_indices, d_out, indices_out, int(page_budget))


def estimate_attn_score(q, o, metadata_data, metadata_indices, metadata_indptr,
                        metadata_last_page_len, metadata_last_page_idx, v_log_norm, layout,
                        kv_indices=None):
    _ops._check_half_cuda(q, "q")
    _ops._check_cuda_contig(o, "o")
    _ops._check_i32_cuda(metadata_indices, "metadata_indices")
    H, D = q.size(1), q.size(2)
    P = metadata_data.size(2)
    n_meta = metadata_indices.numel()
    n_out = (n_meta - 1) * P + int(metadata_last_page_len) - 1
    if o.dim() != 2 or o.size(0) != H or o.size(1) < n_out:
        raise RuntimeError(f"o must be [num_heads, >= {n_out}]")
    dt = _lib.DTYPE_F32 if o.dtype == torch.float32 else _lib.DTYPE_F16
    if n_out == 0:
        return
    _lib.call("aoakv_estimate_attn_score", q.data_ptr(), o.data_ptr(), dt, o.stride(0),
              metadata_data.data_ptr(), metadata_indices.data_ptr(), n_meta,
              int(metadata_last_page_len), metadata_data.size(0),
              None if kv_indices is None else kv_indices.data_ptr(), v_log_norm.size(0),
              v_log_norm.data_ptr(), H, D, P, int(layout), _mode(), _ops._stream(q))


def _append(name, k, v, kv_data, kv_indices, kv_last_page_len, metadata_data, metadata_indices,
            metadata_last_page_len, v_log_norm, layout, *extra):
    for t, nm in ((k, "k"), (v, "v"), (kv_data, "kv_data"), (metadata_data, "metadata_data"),
                  (v_log_norm, "v_log_norm")):
        _ops._check_half_cuda(t, nm)
    _ops._check_i32_cuda(kv_indices, "kv_indices")
    _ops._check_i32_cuda(metadata_indices, "metadata_indices")
    H, D, P = k.size(1), k.size(2), kv_data.size(2)
    _lib.call(name, k.data_ptr(), v.data_ptr(), *extra, kv_data.data_ptr(), kv_indices.data_ptr(),
              kv_indices.numel(), int(kv_last_page_len), kv_data.size(0), metadata_data.data_ptr(),
              metadata_indices.data_ptr(), metadata_indices.numel(), int(metadata_last_page_len),
              metadata_data.size(0), v_log_norm.data_ptr(), H, D, P, int(layout), _ops._stream(k))


def append_kv_cache_decode(k, v, kv_data, kv_indices, kv_indptr, kv_last_page_len,
                           kv_last_page_idx, metadata_data, metadata_indices, metadata_indptr,
                           metadata_last_page_len, metadata_last_page_idx, v_log_norm, layout):
    if k.size(0) != 1:
        raise RuntimeError(f"CHECK_EQ(k.size(0), 1) failed. {k.size(0)} vs 1")
    _append("aoakv_append_kv_cache_decode", k, v, kv_data, kv_indices, kv_last_page_len,
            metadata_data, metadata_indices, metadata_last_page_len, v_log_norm, layout)


def append_kv_cache_prefill(k, v, kv_data, kv_indices, kv_indptr, kv_last_page_len,
                            kv_last_page_idx, metadata_data, metadata_indices, metadata_indptr,
                            metadata_last_page_len, metadata_last_page_idx, v_log_norm, layout):
    _append("aoakv_append_kv_cache_prefill", k, v, kv_data, kv_indices, kv_last_page_len,
            metadata_data, metadata_indices, metadata_last_page_len, v_log_norm, layout,
            k.size(0))


class BatchDecodeWithPagedKVCachePyTorchWrapper:
    """approx_attn.cu:27-151 (begin_forward / end_forward / forward)."""

    def __init__(self, layout: int):
        self._w = _Wrapper(["NHD", "HND"][int(layout)])

    def begin_forward(self, indptr, num_qo_heads, num_kv_heads, head_dim, page_size, empty_data):
        self._w.begin_forward(indptr, num_qo_heads, num_kv_heads, head_dim, page_size,
                              empty_data.dtype)

    def end_forward(self):
        self._w.end_forward()

    def forward(self, q, o, paged_kv_data, paged_kv_indices, paged_kv_indptr,
                paged_kv_last_page_len, paged_kv_last_page_idx, rope_scale, rope_theta):
        self._w.forward(q, o, paged_kv_data, paged_kv_indices, paged_kv_indptr,
                        paged_kv_last_page_len, paged_kv_last_page_idx, rope_scale, rope_theta)


def prefill_with_paged_kv_cache(q, kv_data, kv_indices, kv_last_page_len, causal, layout,
                                allow_fp16_qk_reduction, rope_scale, rope_theta):
    """batch_prefill.cu:27-116 (pybind prefill_with_paged_kv_cache)."""
    return _ops.prefill_with_paged_kv_cache(q, kv_data, kv_indices, kv_last_page_len, causal,
                                            int(layout), allow_fp16_qk_reduction, rope_scale,
                                            rope_theta)


def apply_rope_in_place(q, k, past_kv_len, rope_scale, rope_theta):
    """page.cu:224-264 (pybind apply_rope_in_place)."""
    _ops.apply_rope_in_place(q, k, past_kv_len, rope_scale, rope_theta)


def rms_norm_forward(input, weight, output, epsilon):
    """ops/csrc/rms_norm.cu (pybind rms_norm_forward): writes output."""
    output.copy_(_ops.rms_norm_forward(input, weight, epsilon))
