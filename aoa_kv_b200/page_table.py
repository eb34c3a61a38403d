"""Device-resident page table (libaoakv's aoakv_page_table_*): the page
lists, counts and free stacks of several sequences in one device buffer, with
pages allocated on the GPU. It replaces the host-side KvCache / KvPool lists
of the reference (kernels/aoa_kv/quest/utils/kv_cache.py:7-133) and the index
tensors controller.py:82-141 rebuilds and copies every step, so a decode token
(append + every layer's step) can be captured once as a CUDA graph.

The host keeps only the token counts (deterministic from the appends), never
the page ids.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


class DevicePageTable:
    """num_seqs sequences of up to max_pages_per_seq pages each, drawing KV
    pages from a pool of kv_capacity_pages and metadata pages from one of
    metadata_capacity_pages (page size page_size)."""

    def __init__(self, num_seqs: int, max_pages_per_seq: int, kv_capacity_pages: int,
                 metadata_capacity_pages: int, page_size: int, device="cuda"):
        self.num_seqs, self.max_pages, self.page_size = num_seqs, max_pages_per_seq, page_size
        self.kv_capacity, self.metadata_capacity = kv_capacity_pages, metadata_capacity_pages
        n = _lib.size_query("aoakv_page_table_bytes", num_seqs, max_pages_per_seq,
                            kv_capacity_pages, metadata_capacity_pages, page_size)
        self.buffer = torch.empty(n // 4, dtype=torch.int32, device=device)
        self._h = ctypes.c_void_p()
        _lib.call("aoakv_page_table_create", ctypes.byref(self._h), num_seqs, max_pages_per_seq,
                  kv_capacity_pages, metadata_capacity_pages, page_size, self.buffer.data_ptr(),
                  n, self._stream())
        w = (ctypes.c_int64 * 16)()
        _lib.call("aoakv_page_table_layout", self._h, w)
        self._w = list(w)
        self.seq_len = [0] * num_seqs  # host mirror of the token counts

    @staticmethod
    def _stream():
        return torch.cuda.current_stream().cuda_stream

    @property
    def handle(self):
        return self._h

    def _region(self, i: int, n: int) -> torch.Tensor:
        return self.buffer[self._w[i]:self._w[i] + n]

    def append(self, num_tokens: int, seq: int = -1) -> None:
        """KvCache.append_seq + the metadata append (controller.py:82-87), on
        the device, for sequence `seq` (-1: all, in order)."""
        _lib.call("aoakv_page_table_append", self._h, seq, int(num_tokens), self._stream())
        for r in (range(self.num_seqs) if seq < 0 else [seq]):
            self.seq_len[r] += int(num_tokens)

    def sync_mirror(self) -> None:
        """Re-reads the token counts from the device (synchronises): after an
        append the device refused (AOAKV_DEV_ERR_NO_PAGES) the host mirror,
        which assumes every append succeeds, is corrected here."""
        self.seq_len = self.counts()["seq_len"]

    def note_replayed(self, num_tokens: int, seq: int = -1) -> None:
        """Advances the host mirror for appends replayed from a CUDA graph
        (capturing append() advances it once, at capture)."""
        for r in (range(self.num_seqs) if seq < 0 else [seq]):
            self.seq_len[r] += int(num_tokens)

    def release(self, seq: int = -1) -> None:
        """KvCache.release (kv_cache.py:128-133) for `seq` (-1: all)."""
        _lib.call("aoakv_page_table_release", self._h, seq, self._stream())
        for r in (range(self.num_seqs) if seq < 0 else [seq]):
            self.seq_len[r] = 0

    def num_pages(self, seq: int) -> int:
        return -(-self.seq_len[seq] // self.page_size)

    def last_page_len(self, seq: int) -> int:
        return (self.seq_len[seq] - 1) % self.page_size + 1

    def kv_indices(self, seq: int) -> torch.Tensor:
        """Device view of sequence `seq`'s KV page ids (its num_pages first)."""
        return self._region(8, self.num_seqs * self.max_pages)[
            seq * self.max_pages:(seq + 1) * self.max_pages]

    def metadata_indices(self, seq: int) -> torch.Tensor:
        mm = self._w[15]
        return self._region(9, self.num_seqs * mm)[seq * mm:(seq + 1) * mm]

    def counts(self) -> dict:
        """Device counters (copied to the host; synchronises)."""
        R = self.num_seqs
        g = lambda i: self._region(i, R).cpu().tolist()
        start, end = g(2), g(3)
        return {"num_pages": [e - s for s, e in zip(start, end)], "last_len": g(4),
                "seq_len": g(5), "meta_count": g(7),
                "kv_free": int(self.buffer[self._w[0]]), "meta_free": int(self.buffer[self._w[1]])}

    def decode_step(self, q, k_new, v_new, o, kv_data, metadata_data, v_log_norm, page_budget,
                    score_mode=_lib.SCORE_AOAKV, sink_first_page=False,
                    selected_out: Optional[torch.Tensor] = None,
                    rope_scale: Optional[float] = None, rope_theta: float = 1e4) -> None:
        """One layer's decode step for every sequence (aoakv_decode_step_table):
        q, k_new, v_new, o [num_seqs, H, D]; counts read on the device. With
        rope_scale, q and k_new arrive unrotated and are rotated at each
        sequence's new-token position (left rotated in place)."""
        H, D = q.shape[-2], q.shape[-1]
        _lib.call("aoakv_decode_step_table", self._h, q.data_ptr(), k_new.data_ptr(),
                  v_new.data_ptr(), o.data_ptr(), kv_data.data_ptr(), kv_data.shape[0],
                  metadata_data.data_ptr(), metadata_data.shape[0], v_log_norm.data_ptr(), H, D,
                  int(page_budget), int(score_mode), int(bool(sink_first_page)),
                  None if selected_out is None else selected_out.data_ptr(),
                  0.0 if rope_scale is None else float(rope_scale), float(rope_theta),
                  self._stream())

    def close(self) -> None:
        if self._h:
            _lib.call("aoakv_page_table_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
