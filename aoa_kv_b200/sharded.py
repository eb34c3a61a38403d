"""One long sequence split across GPUs by page range (one process per GPU).

The single-GPU step (append -> estimate -> top-k -> sparse decode,
QuestAttention.py:99-157) needs every page's score before it can choose the
k-1 pages a head attends. With the pages of one sequence spread over G GPUs
(GPU g holds logical pages [lo_g, hi_g), the last GPU also the last page),
the same result comes from two kernel passes around two exchanges:

1. propose (one launch of the cluster step kernel, aoakv_shard_propose):
   every GPU scores its own pages and writes its best k-1 per head as
   {order key, global page id}, best first (ties to the lower page) —
   k-1 from each GPU is enough for the global top-(k-1) to be among them;
2. one all_gather of the proposals, G * H * (k-1) * 8 bytes;
3. finish (one launch, aoakv_shard_finish): every GPU ranks its own
   proposals against the others' by binary search (the lists are sorted),
   so it knows which of its pages won without any further exchange, decodes
   them (the owner of the last page appends the new token to it first, a1,
   and attends it) and writes its partial softmax state {o, lse};
4. one all_gather of the partial states, G * H * (D + 1) * 4 bytes;
5. the log-sum-exp merge (FlashInfer VariableLengthMergeStates' math,
   decode_attn.cuh:1035-1043) gives every GPU the same output.

The two exchanges run one of two ways:
  exchange="nccl"  two all_gathers per layer through the process group
                   (NCCL over NVLink on GPUs, gloo in the CPU tests);
  exchange="p2p"   no collective: every GPU owns a mailbox in its memory,
                   mapped into the other GPUs' address space (CUDA IPC), and
                   the propose and finish kernels store their lists and
                   partial states straight into every mailbox over NVLink
                   and raise a per-rank flag there; the next pass on each GPU
                   waits for all flags (bounded) — the exchange is fused into
                   the kernels before it.
Both are capturable in a CUDA graph with the three launches. The kernels
are reached through an operations object: ``CudaShardOps`` calls
libaoakv.so; tests pass another implementation of the same operations to
exercise this host logic on CPU ranks.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib

SENTINEL_ID = -1  # 0xffffffff: an unused proposal entry (its key is 0)


def partition_pages(n_pages: int, world: int, page_size: int) -> list[tuple[int, int]]:
    """Contiguous page ranges, one per rank. Every range but the last starts
    and ends on a multiple of page_size pages, so a metadata page (page_size
    KV pages) never straddles two GPUs; the last range ends at n_pages."""
    if world < 1 or n_pages < 1:
        raise ValueError("world and n_pages must be >= 1")
    per = -(-n_pages // world)
    per = -(-per // page_size) * page_size
    out = []
    for g in range(world):
        lo = min(n_pages, g * per)
        hi = n_pages if g == world - 1 else min(n_pages, lo + per)
        out.append((lo, hi))
    if any(hi <= lo for lo, hi in out):
        raise ValueError(f"{n_pages} pages do not give each of {world} ranks a page range "
                         f"of whole metadata pages ({page_size} pages)")
    return out


@dataclass
class ShardLayer:
    """One layer's share of the sequence on this rank.

    kv [cap, 2, P, H, D], meta [mcap, 2, P, H, D], vlog [cap, H]: this rank's
    pools (cap >= n_local + 1). kv_idx / meta_idx: int32 physical ids of the
    local pages / local metadata pages in logical order (local page i is
    global page page_lo + i). n_local: pages held here (the last rank's
    count includes the last page). n_total / last_len: the whole sequence's
    page count and last-page fill, the new token included.
    """
    kv: torch.Tensor
    meta: torch.Tensor
    vlog: torch.Tensor
    kv_idx: torch.Tensor
    meta_idx: torch.Tensor
    page_lo: int
    n_local: int
    n_total: int
    last_len: int
    owns_last: bool
    last_phys: int = -1  # physical id of the last page on its owner


def _gather(t: torch.Tensor, group) -> torch.Tensor:
    """[world, *t.shape]: every rank's t, rank order (dim-0 concatenation,
    which both NCCL and gloo accept). A group object with its own
    ``all_gather_stack(t)`` (e.g. ranks emulated as threads) is used as is."""
    if hasattr(group, "all_gather_stack"):
        return group.all_gather_stack(t)
    world = dist.get_world_size(group)
    t = t.contiguous()
    out = torch.empty((world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t, group=group)
    return out.view(world, *t.shape)


def _group_rank(group) -> int:
    if hasattr(group, "all_gather_stack"):
        r = getattr(group, "rank", 0)
        return int(r() if callable(r) else r)
    return dist.get_rank(group)


class ShardedDecoder:
    """Per-layer decode step of a sequence split by page range; every rank
    of ``group`` calls ``step`` with its ShardLayer and the same q, k_new,
    v_new, and gets the same output."""

    def __init__(self, group, num_heads: int, head_dim: int, page_size: int, page_budget: int,
                 score_mode: str = "aoakv", sink_first_page: bool = False, ops=None,
                 rank: int | None = None, exchange: str = "nccl", device=None):
        if score_mode not in ("aoakv", "quest"):
            raise ValueError("score_mode must be 'aoakv' or 'quest'")
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.group = group
        self.H, self.D, self.P = num_heads, head_dim, page_size
        self.page_budget = page_budget
        self.score_mode = score_mode
        self.sink = bool(sink_first_page)
        self.rank = _group_rank(group) if rank is None else rank
        self.ops = ops if ops is not None else CudaShardOps(num_heads, head_dim, page_size,
                                                            page_budget, score_mode, self.sink)
        self.exchange = exchange
        self.mailbox = None
        if exchange == "p2p":  # collective: every rank constructs its decoder together
            kp = max(3, page_budget) if self.sink else page_budget
            self.mailbox = ShardMailbox(group, self.rank, num_heads, head_dim, max(1, kp - 1),
                                        device if device is not None else
                                        torch.device("cuda", torch.cuda.current_device()))

    def budget(self, n_total: int) -> int:
        """Pages attended per head, the last page included
        (controller.py:124 / filter_util.py:231)."""
        kp = max(3, self.page_budget) if self.sink else self.page_budget
        return min(kp, n_total)

    def step(self, layer: ShardLayer, q: torch.Tensor, k_new: torch.Tensor,
             v_new: torch.Tensor, want_selected: bool = True):
        """Returns (o [H, D] fp16, selected global page ids [H, k-1] int32,
        best first, or None when no selection runs)."""
        ops = self.ops
        k = self.budget(layer.n_total)
        sel = None
        if self.mailbox is not None:
            sparse = layer.n_total > k and k > 1
            if sparse:
                ops.propose_p2p(q, layer, self.mailbox)
            sel = ops.finish_p2p(q, k_new, v_new, layer, self.mailbox, k - 1 if sparse else 0,
                                 want_selected)
            return ops.merge_p2p(self.mailbox, sparse, q.device), sel
        if layer.n_total > k and k > 1:
            ks = k - 1
            cand = ops.propose(q, layer, ks, self.sink and layer.page_lo == 0)  # [H, ks, 2]
            cand_all = _gather(cand, self.group)  # [G, H, ks, 2]
            state, sel = ops.finish(q, k_new, v_new, layer, cand_all, ks, self.rank,
                                    want_selected)
        else:  # every page attended, or (k == 1) only the last
            state, _ = ops.finish(q, k_new, v_new, layer, None, 0, self.rank, False)
        states = _gather(state, self.group)  # [G, H, D + 1]
        return ops.merge(states), sel


class ShardMailbox:
    """This rank's mailbox of the peer-store exchange (aoakv_shard_mailbox_*):
    created on every rank of ``group`` together; the 64-byte IPC handles are
    all-gathered through the group and every rank maps the others'."""

    def __init__(self, group, rank: int, num_heads: int, head_dim: int, max_proposals: int,
                 device):
        world = int(getattr(group, "world", 1)) if hasattr(group, "all_gather_stack") \
            else dist.get_world_size(group)
        self._lib = _lib.load()
        self._h = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _lib.call("aoakv_shard_mailbox_create", ctypes.byref(self._h), world, rank, num_heads,
                  head_dim, max_proposals, handle)
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        every = _gather(mine, group).cpu().numpy().tobytes()  # [world, 64], rank order
        _lib.call("aoakv_shard_mailbox_connect", self._h,
                  (ctypes.c_uint8 * len(every)).from_buffer_copy(every))
        self.world = world

    def close(self):
        """Only after every rank finished its last pass (a barrier)."""
        if self._h:
            self._lib.aoakv_shard_mailbox_destroy(self._h)
            self._h = ctypes.c_void_p()


class CudaShardOps:
    """The shard operations on libaoakv.so (current torch stream); one step
    plan per layer pool, made on first use."""

    def __init__(self, num_heads: int, head_dim: int, page_size: int, page_budget: int,
                 score_mode: str, sink: bool):
        self.H, self.D, self.P = num_heads, head_dim, page_size
        self.page_budget, self.sink = page_budget, sink
        self.mode = _lib.SCORE_AOAKV if score_mode == "aoakv" else _lib.SCORE_QUEST
        self._plans: dict = {}

    @staticmethod
    def _stream(t: torch.Tensor):
        return torch.cuda.current_stream(t.device).cuda_stream

    def _plan(self, layer: ShardLayer):
        from .step_plan import StepPlan
        key = (layer.kv.data_ptr(), layer.meta.data_ptr(), layer.vlog.data_ptr(), layer.n_local)
        plan = self._plans.get(key)
        if plan is None:
            cap = layer.kv.shape[0]
            if layer.n_local + 1 > cap:
                raise ValueError("the layer pool needs one page more than the local pages")
            plan = StepPlan(layer.kv, cap, layer.meta, layer.meta.shape[0], layer.vlog, self.H,
                            self.D, self.P, self.page_budget, self.mode, self.sink,
                            max_pages=layer.n_local + 1, shard=True)
            self._plans[key] = plan
        return plan

    def propose(self, q, layer: ShardLayer, ks: int, sink_here: bool):
        cand = torch.empty(self.H, ks, 2, dtype=torch.int32, device=q.device)
        _lib.call("aoakv_shard_propose", self._plan(layer)._h, q.data_ptr(),
                  layer.kv_idx.data_ptr(), layer.n_local, layer.n_total, layer.page_lo,
                  layer.meta_idx.data_ptr(), cand.data_ptr(), self._stream(q))
        return cand

    def finish(self, q, k_new, v_new, layer: ShardLayer, cand_all, ks: int, rank: int,
               want_selected: bool):
        dev = q.device
        state = torch.empty(self.H, self.D + 1, dtype=torch.float32, device=dev)
        sel = torch.empty(self.H, ks, dtype=torch.int32, device=dev) \
            if (want_selected and ks) else None
        world = 1 if cand_all is None else cand_all.shape[0]
        _lib.call("aoakv_shard_finish", self._plan(layer)._h, q.data_ptr(), k_new.data_ptr(),
                  v_new.data_ptr(), layer.kv_idx.data_ptr(), layer.n_local, layer.n_total,
                  layer.page_lo, layer.last_len, layer.meta_idx.data_ptr(),
                  None if cand_all is None else cand_all.contiguous().data_ptr(), world, rank,
                  state.data_ptr(), None if sel is None else sel.data_ptr(), self._stream(q))
        return state, sel

    def propose_p2p(self, q, layer: ShardLayer, mailbox: ShardMailbox):
        _lib.call("aoakv_shard_propose_p2p", self._plan(layer)._h, mailbox._h, q.data_ptr(),
                  layer.kv_idx.data_ptr(), layer.n_local, layer.n_total, layer.page_lo,
                  layer.meta_idx.data_ptr(), self._stream(q))

    def finish_p2p(self, q, k_new, v_new, layer: ShardLayer, mailbox: ShardMailbox, ks: int,
                   want_selected: bool):
        sel = torch.empty(self.H, ks, dtype=torch.int32, device=q.device) \
            if (want_selected and ks) else None
        _lib.call("aoakv_shard_finish_p2p", self._plan(layer)._h, mailbox._h, q.data_ptr(),
                  k_new.data_ptr(), v_new.data_ptr(), layer.kv_idx.data_ptr(), layer.n_local,
                  layer.n_total, layer.page_lo, layer.last_len, layer.meta_idx.data_ptr(),
                  None if sel is None else sel.data_ptr(), self._stream(q))
        return sel

    def merge_p2p(self, mailbox: ShardMailbox, with_proposals: bool, device):
        o = torch.empty(self.H, self.D, dtype=torch.float16, device=device)
        _lib.call("aoakv_shard_merge_p2p", mailbox._h, int(bool(with_proposals)), o.data_ptr(),
                  torch.cuda.current_stream(device).cuda_stream)
        return o

    def merge(self, states):
        G, H, Dp1 = states.shape
        o = torch.empty(H, Dp1 - 1, dtype=torch.float16, device=states.device)
        _lib.call("aoakv_merge_packed_states", states.contiguous().data_ptr(), G, H, Dp1 - 1,
                  o.data_ptr(), self._stream(states))
        return o
