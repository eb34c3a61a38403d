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
