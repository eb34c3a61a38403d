"""CPU restatement of the device page table (aoakv_page_table_*).

TEST INFRASTRUCTURE ONLY: the checker for libaoakv's page-table kernels.

Counting follows the reference's host allocator:
  KvCache.append_seq   kernels/aoa_kv/quest/utils/kv_cache.py:115-126 — per
                       token, a new page when last_page_len == page_size
                       (an empty sequence's last_page_len is page_size, :104-105)
  prepare_metadata     kernels/aoa_kv/quest/utils/controller.py:82-87 — the
                       metadata cache appends one entry per new KV page
  KvCache.release      kv_cache.py:128-133
Page ids come from one free stack per pool shared by all sequences (the
reference gives each sequence its own KvPool): a fresh pool hands out 0, 1,
2, ... as the reference's fresh set does (set.pop on range(capacity)); pages
released are pushed last page first, so they come back in their old order.
A sequence whose append would exceed max_pages or a pool is left unchanged
(the device records AOAKV_DEV_ERR_NO_PAGES).
"""
from __future__ import annotations


def _ceil(a: int, b: int) -> int:
    return -(-a // b)


class PageTableOracle:
    def __init__(self, num_seqs: int, max_pages: int, kv_capacity: int, meta_capacity: int,
                 page_size: int):
        self.R, self.M, self.P = num_seqs, max_pages, page_size
        self.kv_free = list(range(kv_capacity - 1, -1, -1))   # top = end
        self.meta_free = list(range(meta_capacity - 1, -1, -1))
        self.kv = [[] for _ in range(num_seqs)]
        self.meta = [[] for _ in range(num_seqs)]
        self.seq_len = [0] * num_seqs
        self.errors = 0

    def last_len(self, r: int) -> int:
        return (self.seq_len[r] - 1) % self.P + 1 if self.seq_len[r] else self.P

    def append(self, n_tokens: int, seq: int = -1) -> None:
        for r in (range(self.R) if seq < 0 else [seq]):
            new_len = self.seq_len[r] + n_tokens
            n_new = _ceil(new_len, self.P)
            need = n_new - len(self.kv[r])
            need_m = _ceil(n_new, self.P) - len(self.meta[r])
            if n_new > self.M or need > len(self.kv_free) or need_m > len(self.meta_free):
                self.errors += 1
                continue
            self.kv[r] += [self.kv_free.pop() for _ in range(need)]
            self.meta[r] += [self.meta_free.pop() for _ in range(need_m)]
            self.seq_len[r] = new_len

    def release(self, seq: int = -1) -> None:
        for r in (range(self.R - 1, -1, -1) if seq < 0 else [seq]):
            self.kv_free += self.kv[r][::-1]
            self.meta_free += self.meta[r][::-1]
            self.kv[r], self.meta[r], self.seq_len[r] = [], [], 0
