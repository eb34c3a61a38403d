"""Semantics B: numpy restatement of the reference's CUDA kernel tree.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker for the
drop-in entry points (append, estimate, top-k, sparse decode) and for the
per-layer step with ``sink_first_page=0``.

Buffers mirror quest.utils.InferenceController for one layer
(kernels/aoa_kv/quest/utils/controller.py:20-47, kv_cache.py:20-23):
    kv    float16 [cap, 2, P, H, D]   (NHD pages; slot 0 = K, slot 1 = V)
    meta  float16 [mcap, 2, P, H, D]  (entry j of meta page m = KV page m*P+j;
                                       slot 0 = key max, slot 1 = key min)
    vlog  float16 [cap, H]            log(||mean V_page||_2 + 1e-6)
Citations are paths under kernels/aoa_kv/ of the reference.
"""
from __future__ import annotations

import math

import numpy as np

F16, F32 = np.float16, np.float32
HALF_MAX = F16(65504.0)
VLOG_EPS = 1e-6  # kernels/include/decode/decode_page.cuh:501, :686


class LayerCache:
    """One layer's paged KV, metadata and v_log_norm buffers."""

    def __init__(self, cap_pages: int, H: int, D: int, P: int, seed_garbage: int | None = None):
        self.H, self.D, self.P = H, D, P
        self.cap = cap_pages
        self.mcap = (cap_pages + P - 1) // P
        if seed_garbage is None:
            self.kv = np.zeros((cap_pages, 2, P, H, D), F16)
            self.meta = np.zeros((self.mcap, 2, P, H, D), F16)
        else:  # torch.empty-like contents: arbitrary finite values
            g = np.random.default_rng(seed_garbage)
            self.kv = g.standard_normal((cap_pages, 2, P, H, D), dtype=F32).astype(F16)
            self.meta = g.standard_normal((self.mcap, 2, P, H, D), dtype=F32).astype(F16)
        self.vlog = np.zeros((cap_pages, H), F16)  # controller.py:43-47 (zeros)


def _vlog_of_page(vpage: np.ndarray, P: int) -> np.ndarray:
    """decode_page.cuh:459-504: fp32 sum over entries, times 1/P, squared L2
    over channels, log(sqrt + 1e-6), stored fp16. vpage [P, H, D] fp16."""
    mean = vpage.astype(F32).sum(axis=0, dtype=F32) * F32(1.0 / P)
    l2 = (mean * mean).sum(axis=-1, dtype=F32)
    return np.log(np.sqrt(l2) + F32(VLOG_EPS)).astype(F32).astype(F16)


def append_decode(c: LayerCache, kv_indices: np.ndarray, meta_indices: np.ndarray,
                  n_pages: int, last_len: int, k: np.ndarray, v: np.ndarray) -> None:
    """decode_page.cuh:392-506. k, v [H, D] fp16 for the token at position
    (n_pages-1)*P + last_len - 1 (already reserved by the caller)."""
    P = c.P
    entry = last_len - 1
    pid = int(kv_indices[n_pages - 1])
    mp = int(meta_indices[(n_pages - 1) // P])
    me = (n_pages - 1) % P
    if entry > 0:
        mx, mn = c.meta[mp, 0, me].copy(), c.meta[mp, 1, me].copy()
    else:  # :431-434
        mx = np.full((c.H, c.D), -HALF_MAX, F16)
        mn = np.full((c.H, c.D), HALF_MAX, F16)
    k = k.astype(F16)
    c.kv[pid, 0, entry] = k
    c.kv[pid, 1, entry] = v.astype(F16)
    c.meta[mp, 0, me] = np.maximum(mx, k)
    c.meta[mp, 1, me] = np.minimum(mn, k)
    if entry + 1 == P:
        c.vlog[pid] = _vlog_of_page(c.kv[pid, 1], P)


def append_prefill(c: LayerCache, kv_indices: np.ndarray, meta_indices: np.ndarray,
                   n_pages: int, last_len: int, k: np.ndarray, v: np.ndarray) -> None:
    """decode_page.cuh:522-692. k, v [S, H, D]: the last S positions of the
    sequence. Partial pages get max/min only; full pages also v_log_norm,
    computed from the whole page as the reference re-reads it (:648-660)."""
    P = c.P
    S = k.shape[0]
    seq_total = (n_pages - 1) * P + last_len
    start = seq_total - S
    for p in range(start // P, n_pages):
        e0 = max(0, start - p * P)
        e1 = min(P, seq_total - p * P)
        pid = int(kv_indices[p])
        mp, me = int(meta_indices[p // P]), p % P
        src = slice(p * P + e0 - start, p * P + e1 - start)
        kk = k[src].astype(F16)
        c.kv[pid, 0, e0:e1] = kk
        c.kv[pid, 1, e0:e1] = v[src].astype(F16)
        if e0 > 0:
            mx, mn = c.meta[mp, 0, me], c.meta[mp, 1, me]
        else:
            mx = np.full((c.H, c.D), -HALF_MAX, F16)
            mn = np.full((c.H, c.D), HALF_MAX, F16)
        c.meta[mp, 0, me] = np.maximum(mx, kk.max(axis=0))
        c.meta[mp, 1, me] = np.minimum(mn, kk.min(axis=0))
        if e1 == P:
            c.vlog[pid] = _vlog_of_page(c.kv[pid, 1], P)


def estimate(q: np.ndarray, c: LayerCache, meta_indices: np.ndarray, kv_indices: np.ndarray,
             n_pages: int, mode: str) -> np.ndarray:
    """decode_attn.cuh:143-199 and :263-443 with the documented page indexing
    (docs/KERNEL_DIFF.md:33-41): for pages p in [0, N-1),
        s = sum_i max(q_i*kmax_i, q_i*kmin_i)          (quest)
        2*s/sqrt(D) + 2*vlog[kv_indices[p], h]         (aoakv)
    Returns float32 [H, N-1]."""
    P, H, D = c.P, c.H, c.D
    n = n_pages - 1
    p = np.arange(n)
    mx = c.meta[meta_indices[p // P], 0, p % P].astype(F32)  # [n, H, D]
    mn = c.meta[meta_indices[p // P], 1, p % P].astype(F32)
    qf = q.astype(F32)[None]
    s = np.maximum(qf * mx, qf * mn).sum(axis=-1, dtype=F32).T  # [H, n]
    if mode == "quest":
        return s.astype(F32)
    vl = c.vlog[kv_indices[p]].astype(F32).T  # [H, n]
    return (F32(2.0 / math.sqrt(D)) * s + F32(2) * vl).astype(F32)


def apply_rope(x: np.ndarray, past_kv_len: int, rope_scale: float = 1.0,
               rope_theta: float = 1e4) -> np.ndarray:
    """page.cu:224-264 / decode_page.cuh:786-869 (FlashInfer's llama rotate-
    half RoPE): token t at position past_kv_len + t, channel i with
    j = i mod D/2 rotated by angle pos * (1/scale) * (1/theta)^(2j/D) against
    its partner i +- D/2. The frequency and the angle are fp32 products as in
    the kernel; sine and cosine are exact. x [N, H, D] fp16 -> fp16."""
    N, H, D = x.shape
    half = D // 2
    j = np.arange(half, dtype=np.float32)
    f = (np.float32(1.0 / rope_scale) *
         np.exp2(np.float32(np.log2(np.float32(1.0 / rope_theta))) * (np.float32(2) * j / D)))
    pos = (past_kv_len + np.arange(N)).astype(np.float32)
    ang = (pos[:, None] * f[None, :]).astype(np.float32).astype(np.float64)  # [N, half]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    xf = x.astype(np.float64)
    x0, x1 = xf[..., :half], xf[..., half:]
    out = np.concatenate([x0 * c - x1 * s, x1 * c + x0 * s], axis=-1)
    return out.astype(np.float32).astype(F16)


BITONIC_MAX_K = 256


def score_keys(scores: np.ndarray) -> np.ndarray:
    """The selection's order-preserving uint32 key of each fp32 score (as
    uint64): larger score, larger key; -0 == +0; NaN 0, below -inf."""
    f = np.ascontiguousarray(scores, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = np.where(u == 0x80000000, 0, u)  # -0 == +0
    key = np.where(u & 0x80000000, ~u & 0xFFFFFFFF, u | 0x80000000)  # order-preserving
    return np.where(np.isnan(f), 0, key)  # NaN below -inf


def topk_positions(scores: np.ndarray, k: int, sink: bool = False) -> np.ndarray:
    """The library's exact selection rule (the reference's RAFT radix select,
    decode_select_k.cuh:25-61, leaves ties and order unspecified): the k
    largest per row, ties toward the lower position, NaN lowest, -0 == +0;
    with sink, position 0 always plus the k-1 largest of the rest. Output
    order as the library writes it: descending score (ties: lower position
    first) for k <= 256, ascending position above. [H, k]."""
    f = np.ascontiguousarray(scores, dtype=np.float32)
    key = score_keys(f)
    if sink:
        key[:, 0] = 0xFFFFFFFF
    n = f.shape[-1]
    comp = (key << np.uint64(32)) | (~np.arange(n, dtype=np.uint64) & np.uint64(0xFFFFFFFF))
    order = np.argsort(comp, axis=-1)[:, ::-1][:, :k]  # composite keys are distinct
    if k > BITONIC_MAX_K:
        order = np.sort(order, axis=-1)
    return np.ascontiguousarray(order)


def sparse_decode(q: np.ndarray, c: LayerCache, indices: np.ndarray, last_page: int,
                  last_len: int, sm_scale: float | None = None) -> np.ndarray:
    """decode_attn.cuh:469-688 + merge: per head softmax(q.K^T*sm_scale).V over
    the pages indices[h] (P tokens each) plus last_page (last_len tokens).
    Returns float32 [H, D]."""
    H, D, P = c.H, c.D, c.P
    scale = sm_scale if sm_scale else 1.0 / math.sqrt(D)
    out = np.zeros((H, D), F32)
    for h in range(H):
        pages = list(indices[h]) if indices.ndim == 2 else list(indices)
        ks = [c.kv[pg, 0, :, h] for pg in pages] + [c.kv[last_page, 0, :last_len, h]]
        vs = [c.kv[pg, 1, :, h] for pg in pages] + [c.kv[last_page, 1, :last_len, h]]
        K = np.concatenate(ks).astype(F32)
        V = np.concatenate(vs).astype(F32)
        w = (K @ q[h].astype(F32)) * F32(scale)
        w = np.exp(w - w.max(), dtype=F32)
        out[h] = (w / w.sum(dtype=F32)) @ V
    return out


def step(q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, c: LayerCache,
         kv_indices: np.ndarray, meta_indices: np.ndarray, n_pages: int, last_len: int,
         page_budget: int, mode: str, sink: bool):
    """One per-layer decode step (QuestAttention.py:99-157): append, then, if
    the sequence has more pages than the budget, estimate + top-k + sparse
    decode, else decode over every page. Returns (out [H, D] float32,
    attended page ids [H, k] with the last page last)."""
    append_decode(c, kv_indices, meta_indices, n_pages, last_len, k_new, v_new)
    kp = max(3, page_budget) if sink else page_budget
    k = min(kp, n_pages)
    last = int(kv_indices[n_pages - 1])
    if n_pages > k and k > 1:
        sc = estimate(q, c, meta_indices, kv_indices, n_pages, mode)
        pos = topk_positions(sc, k - 1, sink)
        sel = kv_indices[pos]
    elif n_pages > k:  # k == 1: last page only
        sel = np.zeros((c.H, 0), np.int64)
    else:
        sel = np.tile(kv_indices[: n_pages - 1], (c.H, 1))
    out = sparse_decode(q, c, sel, last, last_len)
    return out, np.concatenate([sel, np.full((c.H, 1), last)], axis=1)


def estimate_gqa(q: np.ndarray, c: LayerCache, meta_indices: np.ndarray,
                 kv_indices: np.ndarray, n_pages: int, mode: str) -> np.ndarray:
    """Group-consistent page scores for q [Hq, D] over a cache of Hkv heads
    (query head h reads KV head h // g, g = Hq / Hkv): the kernel tree's page
    bound per query head, combined per KV head as the simulation does —
    quest: the group's bounds summed (filter_util.py:219-221); aoakv:
    logsumexp over the group of 2*s/sqrt(D) (:352-361), plus 2*vlog of the
    KV head's page (:367). Returns float32 [Hkv, N-1]."""
    g = q.shape[0] // c.H
    s = np.stack([estimate(q[i::g], c, meta_indices, kv_indices, n_pages, "quest")
                  for i in range(g)])  # [g, Hkv, n]
    if mode == "quest":
        return s.sum(axis=0, dtype=F32).astype(F32)
    x = F32(2.0 / math.sqrt(c.D)) * s
    m = x.max(axis=0)
    lse = m + np.log(np.exp(x - m[None]).sum(axis=0, dtype=F32))
    p = np.arange(n_pages - 1)
    vl = c.vlog[kv_indices[p]].astype(F32).T  # [Hkv, n]
    return (lse + F32(2) * vl).astype(F32)


def step_gqa(q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, c: LayerCache,
             kv_indices: np.ndarray, meta_indices: np.ndarray, n_pages: int, last_len: int,
             page_budget: int, mode: str, sink: bool):
    """step() for GQA: q [Hq, D], k_new / v_new and the cache with Hkv heads;
    the selection per KV head from estimate_gqa, every query head of a group
    attending its KV head's pages. Returns (out [Hq, D], attended page ids
    [Hkv, k] with the last page last)."""
    g = q.shape[0] // c.H
    append_decode(c, kv_indices, meta_indices, n_pages, last_len, k_new, v_new)
    kp = max(3, page_budget) if sink else page_budget
    k = min(kp, n_pages)
    last = int(kv_indices[n_pages - 1])
    if n_pages > k and k > 1:
        sc = estimate_gqa(q, c, meta_indices, kv_indices, n_pages, mode)
        sel = kv_indices[topk_positions(sc, k - 1, sink)]
    elif n_pages > k:
        sel = np.zeros((c.H, 0), np.int64)
    else:
        sel = np.tile(kv_indices[: n_pages - 1], (c.H, 1))
    out = np.zeros((q.shape[0], c.D), F32)
    for i in range(g):
        out[i::g] = sparse_decode(q[i::g], c, sel, last, last_len)
    return out, np.concatenate([sel, np.full((c.H, 1), last)], axis=1)


def prefill_attention(q: np.ndarray, K: np.ndarray, V: np.ndarray, causal: bool = True,
                      sm_scale: float | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Prefill attention of one sequence (ops/csrc/batch_prefill.cu:27-116;
    the reference test's CPU form quest/tests/test_prefill_attention.py:17-40):
    q [Sq, Hq, D], K and V [Skv, Hk, D] (the whole sequence, new tokens
    last). Query i attends KV tokens j <= i + Skv - Sq when causal; scores
    q.k * sm_scale (1/sqrt(D) by default), softmax in fp32; query head h uses
    KV head h // (Hq / Hk). Returns o [Sq, Hq, D] fp32 and the natural-log
    log-sum-exp [Sq, Hq] of the scaled scores."""
    Sq, Hq, D = q.shape
    Skv, Hk = K.shape[0], K.shape[1]
    g = Hq // Hk
    scale = 1.0 / math.sqrt(D) if sm_scale is None else sm_scale
    qf = q.astype(F32).transpose(1, 0, 2)                       # [Hq, Sq, D]
    kf = np.repeat(K.astype(F32).transpose(1, 0, 2), g, axis=0)  # [Hq, Skv, D]
    vf = np.repeat(V.astype(F32).transpose(1, 0, 2), g, axis=0)
    s = np.matmul(qf, kf.transpose(0, 2, 1)) * F32(scale)      # [Hq, Sq, Skv]
    if causal:
        allowed = np.arange(Skv)[None, :] <= (np.arange(Sq)[:, None] + (Skv - Sq))
        s = np.where(allowed[None], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    o = np.matmul(p / l, vf)                                    # [Hq, Sq, D]
    lse = (m + np.log(l))[..., 0]                               # [Hq, Sq]
    return o.transpose(1, 0, 2).astype(F32), lse.T.astype(F32)
