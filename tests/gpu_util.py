"""Helpers for the GPU parity tests: one layer's buffers on the device plus a
numpy snapshot in the oracle's format."""
from __future__ import annotations

import numpy as np
import torch

from aoa_kv_b200 import _lib
from oracle import kernel_tree as kt


def stream():
    return torch.cuda.current_stream().cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


class GpuLayer:
    """kv [cap,2,P,H,D], meta [mcap,2,P,H,D], vlog [cap,H] on cuda, with a
    page table (kv_idx, meta_idx). Contents start as seeded garbage so stale
    data in unused slots is exercised."""

    def __init__(self, cap, H, D, P, seed=0, permute=True, device="cuda"):
        self.cap, self.H, self.D, self.P = cap, H, D, P
        self.mcap = (cap + P - 1) // P
        g = np.random.default_rng(seed)
        self.kv = torch.from_numpy(
            g.standard_normal((cap, 2, P, H, D), dtype=np.float32).astype(np.float16)).to(device)
        self.meta = torch.from_numpy(
            g.standard_normal((self.mcap, 2, P, H, D), dtype=np.float32).astype(np.float16)).to(device)
        self.vlog = torch.zeros((cap, H), dtype=torch.float16, device=device)
        kvp = g.permutation(cap) if permute else np.arange(cap)
        mp = g.permutation(self.mcap) if permute else np.arange(self.mcap)
        self.kv_idx_np = kvp.astype(np.int32)
        self.meta_idx_np = mp.astype(np.int32)
        self.kv_idx = torch.from_numpy(self.kv_idx_np).to(device)
        self.meta_idx = torch.from_numpy(self.meta_idx_np).to(device)

    def snapshot(self) -> kt.LayerCache:
        c = kt.LayerCache(self.cap, self.H, self.D, self.P)
        c.kv = self.kv.cpu().numpy().copy()
        c.meta = self.meta.cpu().numpy().copy()
        c.vlog = self.vlog.cpu().numpy().copy()
        return c

    def append_prefill(self, k, v, n_pages, last_len):
        S = k.shape[0]
        _lib.call("aoakv_append_kv_cache_prefill", ptr(k), ptr(v), S, ptr(self.kv), ptr(self.kv_idx),
                  n_pages, last_len, self.cap, ptr(self.meta), ptr(self.meta_idx),
                  (n_pages + self.P - 1) // self.P, (n_pages - 1) % self.P + 1, self.mcap,
                  ptr(self.vlog), self.H, self.D, self.P, 0, stream())

    def append_decode(self, k, v, n_pages, last_len):
        _lib.call("aoakv_append_kv_cache_decode", ptr(k), ptr(v), ptr(self.kv), ptr(self.kv_idx),
                  n_pages, last_len, self.cap, ptr(self.meta), ptr(self.meta_idx),
                  (n_pages + self.P - 1) // self.P, (n_pages - 1) % self.P + 1, self.mcap,
                  ptr(self.vlog), self.H, self.D, self.P, 0, stream())

    def fill(self, K, V):
        """Prefill S tokens (numpy fp16 [S,H,D]) from an empty sequence."""
        S = K.shape[0]
        n = (S + self.P - 1) // self.P
        self.append_prefill(torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(), n,
                            (S - 1) % self.P + 1)
        return n
