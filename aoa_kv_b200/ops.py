"""Operator surface mirroring kernels/aoa_kv/quest/utils/__init__.py:69-285.

append_kv / decode_estimate / decode_topk / decode_sparse_attn keep the
reference's names, arguments and return values and call the C ABI of
libaoakv.so on the current torch stream (the reference launches on the
legacy default stream). Shape/dtype violations raise RuntimeError like the
reference's TORCH_CHECKs (pytorch_extension_utils.h:52-66).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .controller import InferenceController


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda_contig(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_half_cuda(t: torch.Tensor, name: str):
    _check_cuda_contig(t, name)
    if t.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16, got {t.dtype}")


def _check_i32_cuda(t: torch.Tensor, name: str):
    _check_cuda_contig(t, name)
    if t.dtype != torch.int32:
        raise RuntimeError(f"{name} must be int32, got {t.dtype}")


def append_kv(k: torch.Tensor, v: torch.Tensor, iController: InferenceController, layer_idx: int):
    """utils/__init__.py:69-131: append k, v [S, H, D] into the layer's paged
    cache, metadata cache and v_log_norm; prefill kernel when S > 1."""
    _check_half_cuda(k, "k")
    _check_half_cuda(v, "v")
    if k.dim() != 3 or k.shape != v.shape:
        raise RuntimeError("k and v must be [seq_len, num_heads, head_dim] of equal shape")
    c = iController
    kv = c.kv_cache.buf_layer(layer_idx)
    meta = c.metadata_cache.buf_layer(layer_idx)
    if kv.size(3) != k.size(1) or kv.size(4) != k.size(2):
        raise RuntimeError("k/v heads or head_dim do not match the KV cache")
    common = (_ptr(kv), _ptr(c.kv_indices_with_last), len(c.kv_cache.indicies),
              c.kv_cache.last_page_len, kv.size(0), _ptr(meta), _ptr(c.metadata_indices),
              len(c.metadata_cache.indicies), c.metadata_cache.last_page_len, meta.size(0),
              _ptr(c.v_log_norm_layer(layer_idx)), k.size(1), k.size(2), kv.size(2), c.layout,
              _stream(k))
    seq_len = k.size(0)
    if seq_len > 1:
        _lib.call("aoakv_append_kv_cache_prefill", _ptr(k), _ptr(v), seq_len, *common)
    else:
        _lib.call("aoakv_append_kv_cache_decode", _ptr(k), _ptr(v), *common)


def decode_estimate(q: torch.Tensor, iController: InferenceController, layer_idx: int) -> torch.Tensor:
    """utils/__init__.py:177-214: page scores [H, N-1] (fp16) for every page
    except the last; value-aware when iController.method == "aoakv"."""
    _check_half_cuda(q, "q")
    c = iController
    n_out = c.metadata_cache.seqlen - 1
    o = torch.empty((c.num_heads, n_out), dtype=q.dtype, device=q.device)
    if n_out == 0:
        return o
    meta = c.metadata_cache.buf_layer(layer_idx)
    _lib.call("aoakv_estimate_attn_score", _ptr(q), _ptr(o), _lib.DTYPE_F16, n_out, _ptr(meta),
              _ptr(c.metadata_indices), len(c.metadata_cache.indicies),
              c.metadata_cache.last_page_len, meta.size(0), _ptr(c.kv_indices_with_last),
              c.kv_cache.pool.capacity, _ptr(c.v_log_norm_layer(layer_idx)), c.num_heads,
              c.head_dim, c.page_size, c.layout, c.score_mode, _stream(q))
    return o


def topk_filtering(estimated_value: torch.Tensor, estimated_indices: torch.Tensor,
                   d_out: Optional[torch.Tensor], indices_out: torch.Tensor, page_budget: int,
                   sink_first_page: bool = False):
    """topk.cu:7-46: per row, the page_budget largest of estimated_value and
    their estimated_indices entries, written in ascending position order."""
    _check_cuda_contig(estimated_value, "estimated_value")
    if estimated_value.dim() != 2:
        raise RuntimeError("estimated_value must be a 2D tensor")
    rows, n = estimated_value.shape
    if estimated_value.dtype == torch.float16:
        dt = _lib.DTYPE_F16
    elif estimated_value.dtype == torch.float32:
        dt = _lib.DTYPE_F32
    else:
        raise RuntimeError(f"estimated_value must be float16 or float32, got {estimated_value.dtype}")
    if estimated_indices is not None:
        _check_i32_cuda(estimated_indices, "estimated_indices")
        if estimated_indices.dim() != 2 or estimated_indices.size(1) != n or \
                estimated_indices.size(0) not in (1, rows):
            raise RuntimeError("estimated_indices must be [rows or 1, num_pages]")
        in_stride = 0 if estimated_indices.size(0) == 1 and rows > 1 else n
    else:
        in_stride = 0
    if not (1 <= page_budget <= n):
        raise RuntimeError(f"CHECK_GE(num_pages, page_budget) failed. {n} vs {page_budget}")
    _check_i32_cuda(indices_out, "indices_out")
    if indices_out.shape != (rows, page_budget):
        raise RuntimeError("indices_out must be [rows, page_budget]")
    if d_out is not None:
        _check_cuda_contig(d_out, "d_out")
        if d_out.shape != (rows, page_budget) or d_out.dtype != estimated_value.dtype:
            raise RuntimeError("d_out must be [rows, page_budget] with the scores' dtype")
    _lib.call("aoakv_topk_filtering", _ptr(estimated_value), dt, n, _ptr(estimated_indices),
              in_stride, rows, n, page_budget, _ptr(d_out), page_budget, _ptr(indices_out),
              page_budget, int(bool(sink_first_page)), _stream(estimated_value))


def decode_topk(estimated_attn_score: torch.Tensor, iController: InferenceController):
    """utils/__init__.py:216-246: top-(budget-1) pages per head into
    iController.topk_dout_buffer / topk_dindices_buffer (physical page ids)."""
    c = iController
    page_budget = c.inference_page_budget - 1
    topk_filtering(estimated_attn_score, c.kv_indices_without_last, c.topk_dout_buffer,
                   c.topk_dindices_buffer, page_budget, c.sink_first_page)


def decode_sparse_attn(q: torch.Tensor, iController: InferenceController, layer_idx: int,
                       topk_indices: torch.Tensor, rope_scale: Optional[float] = None,
                       rope_theta: Optional[float] = None) -> torch.Tensor:
    """utils/__init__.py:248-285: attention of q over topk_indices [H, k-1]
    plus the last page; returns o like q."""
    o = torch.empty_like(q)
    c = iController
    c._decode_handler.forward(q, o, c.kv_cache.buf_layer(layer_idx), topk_indices,
                              c.kv_indptr_for_approx_decode, c.kv_cache.last_page_len,
                              c.kv_last_page_idx, rope_scale, rope_theta)
    return o


def prefill_with_paged_kv_cache(q: torch.Tensor, kv_data: torch.Tensor, kv_indices: torch.Tensor,
                                kv_last_page_len: int, causal: bool = True, layout: int = 0,
                                allow_fp16_qk_reduction: bool = False, rope_scale: float = 1.0,
                                rope_theta: float = 1e4, lse: Optional[torch.Tensor] = None,
                                sm_scale: Optional[float] = None) -> torch.Tensor:
    """ops/csrc/batch_prefill.cu:27-116: attention of q [qo_len, Hq, D] over
    one sequence's paged KV, kv_data [cap, 2, P, Hk, D] (NHD), pages
    kv_indices (int32, last page last, holding kv_last_page_len tokens).
    Causal: query i attends KV tokens <= i + kv_len - qo_len. Returns o like
    q. The reference runs with RoPE off and fp32 score accumulation, so
    rope_scale, rope_theta and allow_fp16_qk_reduction change nothing here
    either. lse (optional, [qo_len, Hq] fp32) receives the natural-log
    log-sum-exp of every row."""
    _check_half_cuda(q, "q")
    _check_half_cuda(kv_data, "kv_data")
    _check_i32_cuda(kv_indices, "kv_indices")
    if q.dim() != 3 or kv_data.dim() != 5 or kv_data.size(1) != 2:
        raise RuntimeError("q must be [qo_len, H, D] and kv_data [pages, 2, P, H, D]")
    if int(layout) != _lib.LAYOUT_NHD:
        raise RuntimeError("prefill_with_paged_kv_cache: only the NHD layout is built")
    if q.size(2) != kv_data.size(4):
        raise RuntimeError("q and kv_data head_dim differ")
    if lse is not None:
        _check_cuda_contig(lse, "lse")
        if lse.dtype != torch.float32 or lse.shape != q.shape[:2]:
            raise RuntimeError("lse must be float32 [qo_len, num_qo_heads]")
    o = torch.empty_like(q)
    _lib.call("aoakv_prefill_paged", _ptr(q), _ptr(o), _ptr(lse), _ptr(kv_data), kv_data.size(0),
              _ptr(kv_indices), kv_indices.numel(), int(kv_last_page_len), q.size(0), q.size(1),
              kv_data.size(3), q.size(2), kv_data.size(2), int(layout), int(bool(causal)),
              0.0 if sm_scale is None else float(sm_scale), _stream(q))
    return o


def prefill_forward(q: torch.Tensor, iController: InferenceController, layer_idx: int,
                    rope_scale: Optional[float] = None,
                    rope_theta: Optional[float] = None) -> torch.Tensor:
    """utils/__init__.py:127-172: causal self-attention of the prompt's q
    [S, H, D] over the layer's paged cache, whose K/V (and metadata) the
    caller has already appended for these tokens."""
    c = iController
    return prefill_with_paged_kv_cache(q, c.kv_cache.buf_layer(layer_idx),
                                       c.kv_indices_with_last, c.kv_cache.last_page_len, True,
                                       c.layout, False,
                                       1.0 if rope_scale is None else rope_scale,
                                       1e4 if rope_theta is None else rope_theta)


def apply_rope_in_place(q: torch.Tensor, k: torch.Tensor, past_kv_len: int,
                        rope_scale: Optional[float] = None, rope_theta: Optional[float] = None):
    """utils/__init__.py:25-52: RoPE in place on q, k [N, H, D] fp16 (NHD),
    token t at position past_kv_len + t; scale 1 and theta 1e4 by default."""
    _check_half_cuda(q, "q")
    _check_half_cuda(k, "k")
    if q.dim() != 3 or q.shape != k.shape:
        raise RuntimeError("q and k must be [seq_len, num_heads, head_dim] of equal shape")
    _lib.call("aoakv_apply_rope_in_place", _ptr(q), _ptr(k), q.size(0), int(past_kv_len),
              q.size(1), q.size(2), 1.0 if rope_scale is None else float(rope_scale),
              1e4 if rope_theta is None else float(rope_theta), _stream(q))


def rms_norm_forward(input: torch.Tensor, weight: torch.Tensor, epsilon: float) -> torch.Tensor:
    """utils/__init__.py:54-67: RMSNorm over the last dimension of an fp16
    tensor (a multiple of 8), scaled by weight; returns a new tensor."""
    _check_half_cuda(input, "input")
    _check_half_cuda(weight, "weight")
    cols = input.size(-1)
    if weight.numel() != cols:
        raise RuntimeError("weight must have input.size(-1) elements")
    o = torch.empty_like(input)
    _lib.call("aoakv_rms_norm", _ptr(input), _ptr(weight), _ptr(o), input.numel() // cols, cols,
              float(epsilon), _stream(input))
    return o
