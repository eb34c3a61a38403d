"""Semantics A: numpy restatement of the reference's PyTorch simulation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker for the CUDA
path's ``sink_first_page=1`` mode and the timed CPU baseline.

Shapes follow the reference with the batch dimension squeezed (b = 1):
    q [Hq, D];  K, V [Hkv, S, D];  page filters [Hkv, N, 2, D] (max at 0,
    min at 1); groups = Hq / Hkv query heads per KV head (1 for MHA, where
    the group sum / logsumexp of filter_util.py:219-221 and :352-361 is the
    identity). Query head h reads KV head h // groups (repeat_kv).
All arithmetic is float32, as the simulation runs on the CPU (fp16 inputs are
upcast). Page ids are logical (0 .. N-1).

Each function cites the file:line of the reference checkout it restates
(filtering/filter_util.py = "fu", evaluation/quest_attention.py = "qa").
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
FMIN = np.finfo(np.float32).min
FMAX = np.finfo(np.float32).max
LOG_EPS = 1e-8  # fu:325


def num_pages(seq_len: int, page_size: int) -> int:
    return (seq_len + page_size - 1) // page_size


def _pad_len(seq_len: int, page_size: int) -> int:
    return page_size - ((seq_len - 1) % page_size + 1)  # fu:561


def get_max_min_filters(K: np.ndarray, page_size: int) -> np.ndarray:
    """fu:555-638. Per-page per-channel key max/min; the partial last page is
    padded with finfo.min (for the max) and finfo.max (for the min)."""
    H, S, D = K.shape
    N, pad = num_pages(S, page_size), _pad_len(S, page_size)
    kmax = np.concatenate([K, np.full((H, pad, D), FMIN, F32)], axis=1)
    kmin = np.concatenate([K, np.full((H, pad, D), FMAX, F32)], axis=1)
    kmax = kmax.reshape(H, N, page_size, D).max(axis=2)
    kmin = kmin.reshape(H, N, page_size, D).min(axis=2)
    return np.stack([kmax, kmin], axis=2).astype(F32)


def update_page_filters(filters: np.ndarray, k_new: np.ndarray, past_len: int,
                        page_size: int) -> np.ndarray:
    """fu:758-795 with update_filter fu:524-553. k_new [H, D]."""
    if past_len % page_size != 0:
        last = filters[:, -1]
        upd = np.stack([np.maximum(last[:, 0], k_new), np.minimum(last[:, 1], k_new)], axis=1)
        return np.concatenate([filters[:, :-1], upd[:, None]], axis=1)
    new = np.stack([k_new, k_new], axis=1)[:, None]
    return np.concatenate([filters, new], axis=1)


def compute_page_v_mean(seq_len: int, page_size: int, V: np.ndarray) -> np.ndarray:
    """fu:797-834. Mean of V per page, the partial last page included."""
    H, _, D = V.shape
    nf = seq_len // page_size
    full = V[:, : nf * page_size].reshape(H, nf, page_size, D).mean(axis=2, dtype=F32)
    if seq_len % page_size:
        left = V[:, nf * page_size: seq_len].mean(axis=1, dtype=F32, keepdims=True)
        full = np.concatenate([full, left], axis=1)
    return full.astype(F32)


def update_mean_page_filters(means: np.ndarray, v_new: np.ndarray, past_len: int,
                             page_size: int) -> np.ndarray:
    """fu:681-716 with update_mean_filter fu:669-679: running mean of the last
    page, or a new page started by v_new. means [H, N, D], v_new [H, D]."""
    if past_len % page_size != 0:
        n_prev = past_len % page_size
        last = (means[:, -1] * F32(n_prev) + v_new) / F32(n_prev + 1)
        return np.concatenate([means[:, :-1], last[:, None]], axis=1)
    return np.concatenate([means, v_new[:, None]], axis=1)


def attn_weights_for_selection(q: np.ndarray, filters: np.ndarray, page_size: int,
                               seq_len: int, expand: bool = True, groups: int = 1) -> np.ndarray:
    """fu:968-1018. Quest upper bound per token, [H, S].

    sign = +1 where q > 0 else -1 (fu:990); bound = |q| . max(sign*kmax,
    sign*kmin) per page (fu:993-1002). The reference repeats every page's bound
    to its page_size tokens and runs one matmul (fu:1004-1016); expand=False
    computes the same numbers per page and repeats the result instead.
    """
    if groups > 1:  # repeat_filter: every query head reads its KV head's filters
        filters = np.repeat(filters, groups, axis=0)
    sign = np.where(q > 0, F32(1), F32(-1))
    pos_q = q * sign
    max_key = (filters * sign[:, None, None, :]).max(axis=2)  # [H, N, D]
    if expand:
        tok = np.repeat(max_key, page_size, axis=1)[:, :seq_len]  # [H, S, D]
        return np.matmul(pos_q[:, None, :], tok.transpose(0, 2, 1))[:, 0]
    per_page = np.matmul(pos_q[:, None, :], max_key.transpose(0, 2, 1))[:, 0]
    return np.repeat(per_page, page_size, axis=1)[:, :seq_len]


def chunk_scores(w: np.ndarray, page_size: int) -> np.ndarray:
    """fu:187-217 / fu:291-321: pad the token weights with finfo.min and take
    the max of each page, [H, N]."""
    H, S = w.shape
    N, pad = num_pages(S, page_size), _pad_len(S, page_size)
    wp = np.concatenate([w, np.full((H, pad), FMIN, F32)], axis=1)
    return wp.reshape(H, N, page_size).max(axis=2)


def page_budget_k(token_budget: int, page_size: int, n: int) -> int:
    """fu:231 / fu:373: k = min(max(3, token_budget // page_size), N)."""
    return min(max(3, token_budget // page_size), n)


def topk_pages(scores: np.ndarray, k: int) -> np.ndarray:
    """torch.topk stand-in over the last axis: the k largest, ties toward the
    lower page id; returned sorted ascending, [H, k]."""
    order = np.argsort(-scores, axis=-1, kind="stable")[:, :k]
    return np.sort(order, axis=-1)


def quest_scores(w: np.ndarray, page_size: int, fixed: bool, groups: int = 1) -> np.ndarray:
    """fu:165-228 (local_heavy_hitter_mask_group_consistent_sum): page score
    = amax of the token bound, summed over the query heads of a KV head's
    group (fu:219-221); fixed forces pages 0 and N-1 (fu:226-228). [Hkv, N]."""
    cs = chunk_scores(w, page_size).astype(F32)
    if groups > 1:
        cs = cs.reshape(-1, groups, cs.shape[-1]).sum(axis=1, dtype=F32)
    if fixed:
        cs[:, 0] = FMAX
        cs[:, -1] = FMAX
    return cs


def aoakv_scores(w: np.ndarray, page_size: int, v_page_mean: np.ndarray,
                 fixed: bool, groups: int = 1) -> np.ndarray:
    """fu:269-377 (local_heavy_hitter_mask_value_aware_group_consistent_sum):
    2 * amax / sqrt(d) (fu:329), logsumexp over the query heads of a KV
    head's group (fu:352-361), + 2 * log(||mean V_page|| + 1e-8) of the KV
    head (fu:325, fu:367); fixed forces pages 0 and N-1 (fu:375-377). [Hkv, N]."""
    D = v_page_mean.shape[-1]
    log_v = np.log(np.linalg.norm(v_page_mean, axis=-1).astype(F32) + F32(LOG_EPS)).astype(F32)
    cs = chunk_scores(w, page_size).astype(F32)
    cs = F32(2) * (cs / F32(math.sqrt(D)))
    if groups > 1:
        g = cs.reshape(-1, groups, cs.shape[-1])
        m = g.max(axis=1)
        cs = (m + np.log(np.exp(g - m[:, None]).sum(axis=1, dtype=F32))).astype(F32)
    cs = cs + F32(2) * log_v
    if fixed:
        cs[:, 0] = FMAX
        cs[:, -1] = FMAX
    return cs.astype(F32)


def token_mask(pages: np.ndarray, seq_len: int, page_size: int) -> np.ndarray:
    """fu:233-262 / fu:379-405: expand selected pages to their tokens, [H, S]."""
    H = pages.shape[0]
    mask = np.zeros((H, num_pages(seq_len, page_size) * page_size), bool)
    tok = (pages[:, :, None] * page_size + np.arange(page_size)[None, None]).reshape(H, -1)
    np.put_along_axis(mask, tok, True, axis=1)
    return mask[:, :seq_len]


def masked_decode(q: np.ndarray, K: np.ndarray, V: np.ndarray, mask: np.ndarray) -> np.ndarray:
    """qa:262-268 and qa:347-356: q.K^T / sqrt(d), unselected tokens set to
    finfo.min, fp32 softmax, times V. Returns [H, D]."""
    D = q.shape[-1]
    w = np.matmul(q[:, None, :], K.transpose(0, 2, 1))[:, 0] / F32(math.sqrt(D))
    w = np.where(mask, w, FMIN).astype(F32)
    w = w - w.max(axis=-1, keepdims=True)
    e = np.exp(w, dtype=F32)
    p = (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
    return np.matmul(p[:, None, :], V)[:, 0].astype(F32)


class SimLayerState:
    """Per-layer simulation cache after a prefill of K, V [H, S0, D]
    (qa:227-243 for layer_id >= 2): page filters and, for aoakv, page V means."""

    def __init__(self, K: np.ndarray, V: np.ndarray, page_size: int):
        self.page_size = page_size
        self.K = np.ascontiguousarray(K, dtype=F32)
        self.V = np.ascontiguousarray(V, dtype=F32)
        self.seq_len = K.shape[1]
        self.filters = get_max_min_filters(self.K, page_size)
        self.v_mean = compute_page_v_mean(self.seq_len, page_size, self.V)


def decode_step(state: SimLayerState, q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray,
                token_budget: int, method: str = "aoakv", fixed: bool = True,
                expand: bool = True):
    """One decode token of a layer with layer_id >= 2 (qa:249-356 for aoakv,
    qa:90-167 for quest). Mutates `state` (appends the token) and returns
    (out [Hq, D], selected page ids [Hkv, k] ascending, page scores
    [Hkv, N]); Hq / Hkv query heads share a KV head (GQA) when q has more
    heads than the state."""
    groups = q.shape[0] // state.K.shape[0]
    P = state.page_size
    past = state.seq_len
    if method == "aoakv":
        state.v_mean = update_mean_page_filters(state.v_mean, v_new.astype(F32), past, P)
    state.K = np.concatenate([state.K, k_new.astype(F32)[:, None]], axis=1)
    state.V = np.concatenate([state.V, v_new.astype(F32)[:, None]], axis=1)
    state.filters = update_page_filters(state.filters, k_new.astype(F32), past, P)
    S = past + 1
    state.seq_len = S
    w = attn_weights_for_selection(q.astype(F32), state.filters, P, S, expand=expand,
                                   groups=groups)
    tb = min(S, token_budget)  # qa:137 / qa:326
    if method == "aoakv":
        scores = aoakv_scores(w, P, state.v_mean, fixed, groups)
    elif method == "quest":
        scores = quest_scores(w, P, fixed, groups)
    else:
        raise ValueError(f"unknown method {method!r}")
    k = page_budget_k(tb, P, scores.shape[1])
    sel = topk_pages(scores, k)
    mask = np.repeat(token_mask(sel, S, P), groups, axis=0)  # repeat_kv of the mask
    K, V = (state.K, state.V) if groups == 1 else (np.repeat(state.K, groups, axis=0),
                                                   np.repeat(state.V, groups, axis=0))
    out = masked_decode(q.astype(F32), K, V, mask)
    return out, sel, scores
