"""Request sharding for batched decode (several independent requests).

Requests and heads are independent in the sparse-decode step, so a batch
spreads over GPUs with no collective on the data path: each GPU holds its
requests' KV, metadata and page tables and runs their steps. The split
balances the bytes each GPU streams per layer-step (the step is HBM-bound,
so bytes stand in for time): longest-processing-time-first greedy, i.e.
requests in decreasing byte order, each to the GPU with the fewest bytes so
far (ties to the lower GPU index), which is within 4/3 of the best split.
"""
from __future__ import annotations


def step_bytes(ctx_tokens: int, budget_tokens: int, num_heads: int, head_dim: int,
               page_size: int, method: str = "aoakv") -> int:
    """Algorithmic HBM bytes of one request's layer-step (fp16): the scored
    pages' key max/min metadata (+ v_log_norm for aoakv), the attended
    pages' K and V, and q and o. Every page is attended (no scoring) when
    the context fits the budget."""
    n = -(-ctx_tokens // page_size)
    k = min(budget_tokens // page_size, n)
    row = num_heads * head_dim * 2
    q_o = 2 * row
    if n <= k:  # dense: every page, no metadata read
        return n * page_size * row * 2 + q_o
    b = (n - 1) * 2 * row + k * page_size * row * 2 + q_o
    if method == "aoakv":
        b += (n - 1) * num_heads * 2
    return b


def balance_requests(weights: list[int], n_gpus: int) -> list[list[int]]:
    """Request indices per GPU, greedy by decreasing weight onto the least
    loaded GPU. Deterministic; every request appears exactly once."""
    if n_gpus < 1:
        raise ValueError("n_gpus must be >= 1")
    loads = [0] * n_gpus
    out: list[list[int]] = [[] for _ in range(n_gpus)]
    for r in sorted(range(len(weights)), key=lambda i: (-weights[i], i)):
        g = min(range(n_gpus), key=lambda j: (loads[j], j))
        out[g].append(r)
        loads[g] += weights[r]
    for lst in out:
        lst.sort()
    return out


def decode_step_batched(q, k_new, v_new, o, kv, kv_indptr, kv_indices, kv_last_page_len, meta,
                        meta_indptr, meta_indices, v_log_norm, max_pages: int, page_budget: int,
                        score_mode: str = "aoakv", sink_first_page: bool = False,
                        selected=None, stream=None):
    """One decode step of every request whose pages live in one layer pool,
    as ONE launch over (request, head) (aoakv_decode_step_batched).

    kv [cap, 2, P, H, D] and meta [mcap, 2, P, H, D] fp16 and v_log_norm
    [cap, H] are the layer's pools; request r's KV pages are
    kv_indices[kv_indptr[r]:kv_indptr[r+1]] (new token's page included, its
    fill kv_last_page_len[r]) and its metadata pages start at
    meta_indices[meta_indptr[r]] (all int32 on the device). q, k_new, v_new,
    o: [R, H, D] fp16; selected (optional): [R, H, B] int32 with B =
    page_budget (max(3, page_budget) with the sink)."""
    import torch

    from . import _lib
    R, H, D = q.shape
    cap, _, P = kv.shape[0], kv.shape[1], kv.shape[2]
    for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new), ("o", o), ("kv", kv),
                    ("meta", meta), ("v_log_norm", v_log_norm)):
        if not t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous fp16 CUDA tensor")
    for name, t in (("kv_indptr", kv_indptr), ("kv_indices", kv_indices),
                    ("kv_last_page_len", kv_last_page_len), ("meta_indptr", meta_indptr),
                    ("meta_indices", meta_indices)):
        if not t.is_cuda or t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 CUDA tensor")
    if kv_indptr.numel() != R + 1 or meta_indptr.numel() != R + 1 or \
            kv_last_page_len.numel() != R:
        raise ValueError("indptr arrays need num_requests + 1 entries, kv_last_page_len one "
                         "per request")
    mode = _lib.SCORE_AOAKV if score_mode == "aoakv" else _lib.SCORE_QUEST
    s = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
    _lib.call("aoakv_decode_step_batched", q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
              o.data_ptr(), kv.data_ptr(), cap, kv_indptr.data_ptr(), kv_indices.data_ptr(),
              kv_last_page_len.data_ptr(), meta.data_ptr(), meta.shape[0],
              meta_indptr.data_ptr(), meta_indices.data_ptr(), v_log_norm.data_ptr(), R,
              int(max_pages), H, D, P, int(page_budget), mode, int(bool(sink_first_page)),
              None if selected is None else selected.data_ptr(), s)
    return o
