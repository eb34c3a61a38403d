"""BatchDecodeWithPagedKVCacheWrapper over the library's split-KV decode.

Mirrors kernels/aoa_kv/quest/utils/decode_wrapper.py:11-82 (begin_forward /
forward / end_forward). The reference's begin_forward copies indptr to the
host with a synchronising cudaMemcpy and allocates temporaries with
cudaMallocAsync on every step (decode_attn.cuh:909-912,
decode_handler.cuh:73-121); here the split-KV workspace is a zero-filled
torch buffer that grows only when a larger budget is first seen and is kept
across steps, and no call synchronises.
"""
from __future__ import annotations

import torch

from . import _lib
from .controller import TensorLayout


def _check_kv_layout(kv_layout: str):
    if not hasattr(TensorLayout, kv_layout):
        raise KeyError("Invalide kv_layout {}".format(kv_layout))


class BatchDecodeWithPagedKVCacheWrapper:

    def __init__(self, kv_layout: str = "NHD"):
        _check_kv_layout(kv_layout)
        self.kv_layout = kv_layout
        self._layout = getattr(TensorLayout, kv_layout)
        self._ws = None
        self._dims = None

    def begin_forward(self, indptr: torch.Tensor, num_qo_heads: int, num_kv_heads: int,
                      head_dim: int, page_size: int, data_type):
        if num_qo_heads != num_kv_heads:
            raise RuntimeError("aoa_kv_b200 decode supports MHA only (num_qo_heads == num_kv_heads)")
        if data_type != torch.float16:
            raise RuntimeError("aoa_kv_b200 decode supports float16 only")
        self._dims = (num_qo_heads, head_dim, page_size)

    def end_forward(self):
        """Nothing to free per step; the workspace is reused."""

    def _workspace(self, num_heads: int, head_dim: int, n_sel: int, device) -> torch.Tensor:
        need = _lib.size_query("aoakv_decode_workspace_size", num_heads, head_dim, n_sel)
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=device)
        return self._ws

    def forward(self, q: torch.Tensor, o: torch.Tensor, paged_kv_data: torch.Tensor,
                paged_kv_indices: torch.Tensor, paged_kv_indptr: torch.Tensor,
                paged_kv_last_page_len: int, paged_kv_last_page_idx: int,
                rope_scale=None, rope_theta=None):
        """approx_attn.cu:69-151: q [1, H, D]; paged_kv_indices [H, n_sel]
        (the row stride, like the reference's page_budget); the last page is
        added per head."""
        from .ops import _check_half_cuda, _check_i32_cuda, _ptr, _stream
        _check_half_cuda(q, "q")
        _check_half_cuda(o, "o")
        _check_half_cuda(paged_kv_data, "paged_kv_data")
        if paged_kv_data.dim() != 5 or paged_kv_data.size(1) != 2:
            raise RuntimeError("paged_kv_data must be [pages, 2, page_size, heads, head_dim]")
        H, D = q.size(-2), q.size(-1)
        if self._layout != TensorLayout.NHD:
            raise RuntimeError("aoa_kv_b200 builds the NHD layout only")
        if paged_kv_indices.dim() == 2:
            _check_i32_cuda(paged_kv_indices, "paged_kv_indices")
            if paged_kv_indices.size(0) != H:
                raise RuntimeError("paged_kv_indices must have one row per head")
            n_sel, stride = paged_kv_indices.size(1), paged_kv_indices.stride(0)
        else:
            _check_i32_cuda(paged_kv_indices, "paged_kv_indices")
            n_sel, stride = paged_kv_indices.numel(), 0
        ws = self._workspace(H, D, n_sel, q.device)
        _lib.call("aoakv_sparse_decode", _ptr(q), _ptr(o), _ptr(paged_kv_data),
                  paged_kv_data.size(0), _ptr(paged_kv_indices) if n_sel else None, stride, n_sel,
                  int(paged_kv_last_page_idx), int(paged_kv_last_page_len), H, D,
                  paged_kv_data.size(2), _lib.LAYOUT_NHD, 0.0, _ptr(ws), ws.numel(), _stream(q))
