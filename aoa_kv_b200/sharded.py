"""One long sequence split across GPUs by page range (one process per GPU).

The single-GPU step (append -> estimate -> top-k -> sparse decode,
QuestAttention.py:99-157) needs every page's score before it can choose the
k-1 pages a head attends. With the pages of one sequence spread over G GPUs
(GPU g holds logical pages [lo_g, hi_g), the last GPU also the last page),
the same result comes from one exchange of candidates and one of partial
softmax states:

1. the owner of the last page appends the new token (a1);
2. every GPU scores its own pages (a3) and keeps its local top-(k-1) per
   head (a4) as (score, global page id) — k-1 from each GPU is enough for
   the global top-(k-1) to be among them;
3. one all_gather of the candidates, G * H * (k-1) * 8 bytes (score and
   page id packed in one fp32 tensor); every GPU selects
   the same global top-(k-1) from them (a4 again). Candidates are laid out
   GPU by GPU, each list in the library's selection order, so equal scores
   still resolve to the lower page id, as on one GPU;
4. every GPU decodes the selected pages it holds, plus the last page on its
   owner, into a partial (o, lse) per head (a5 without its merge);
5. one all_gather of the partial states, G * H * (D + 1) * 4 bytes, and the
   log-sum-exp merge (FlashInfer VariableLengthMergeStates' math,
   decode_attn.cuh:1035-1043) gives every GPU the same output.

The data path crosses no GPU boundary except through these two all_gathers
(NCCL over NVLink on GPUs, gloo in the CPU tests). The kernels are reached
through an operations object: ``CudaShardOps`` calls libaoakv.so; tests
pass another implementation of the same operations to exercise this host
logic on CPU ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib


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
    pools. kv_idx / meta_idx: int32 physical ids of the local pages / local
    metadata pages in logical order (local page i is global page_lo + i).
    n_local: pages held here (the last rank's count includes the last page).
    n_total / last_len: the whole sequence's page count and last-page fill.
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


class ShardedDecoder:
    """Per-layer decode step of a sequence split by page range; every rank
    of ``group`` calls ``step`` with its ShardLayer and the same q, k_new,
    v_new, and gets the same output."""

    def __init__(self, group, num_heads: int, head_dim: int, page_size: int, page_budget: int,
                 score_mode: str = "aoakv", sink_first_page: bool = False, ops=None):
        if score_mode not in ("aoakv", "quest"):
            raise ValueError("score_mode must be 'aoakv' or 'quest'")
        self.group = group
        self.H, self.D, self.P = num_heads, head_dim, page_size
        self.page_budget = page_budget
        self.score_mode = score_mode
        self.sink = bool(sink_first_page)
        self.ops = ops if ops is not None else CudaShardOps(num_heads, head_dim, page_size)

    def budget(self, n_total: int) -> int:
        """Pages attended per head, the last page included
        (controller.py:124 / filter_util.py:231)."""
        kp = max(3, self.page_budget) if self.sink else self.page_budget
        return min(kp, n_total)

    def step(self, layer: ShardLayer, q: torch.Tensor, k_new: torch.Tensor,
             v_new: torch.Tensor):
        """Returns (o [H, D] fp16, selected global page ids [H, k-1] int32 or
        None when every page is attended)."""
        ops = self.ops
        if layer.owns_last:
            ops.append_decode(layer, k_new, v_new)
        n_score = layer.n_local - (1 if layer.owns_last else 0)
        k = self.budget(layer.n_total)
        sel = None
        if layer.n_total > k and k > 1:
            ks = k - 1
            if n_score < ks:
                raise ValueError(f"rank holding pages [{layer.page_lo}, "
                                 f"{layer.page_lo + layer.n_local}) scores {n_score} pages, "
                                 f"fewer than the {ks} each rank must propose")
            sink_here = self.sink and layer.page_lo == 0
            vals, ids = ops.local_topk(q, layer, n_score, ks, self.score_mode, sink_here)
            # one collective for both: the ids travel as the bits of fp32 words
            packed = torch.stack([vals, ids.view(torch.float32)])  # [2, H, ks]
            allp = _gather(packed, self.group)  # [G, 2, H, ks]
            G = allp.shape[0]
            cand = allp.permute(1, 2, 0, 3).reshape(2, self.H, G * ks)
            cand_v = cand[0].contiguous()
            cand_i = cand[1].contiguous().view(torch.int32)
            # page 0, when forced, is GPU 0's first candidate: position 0
            sel = ops.select(cand_v, cand_i, ks, self.sink)
            local = ops.to_local(sel, layer)
        elif layer.n_total > k:  # k == 1: the last page only
            local = None
        else:  # every page is attended
            local = ops.all_local_pages(layer, n_score)
        o_part, lse = ops.decode_partial(q, layer, local)
        state = torch.cat([o_part, lse.unsqueeze(1)], dim=1)  # [H, D + 1], one collective
        alls = _gather(state, self.group)  # [G, H, D + 1]
        o = ops.merge(alls[:, :, :self.D].contiguous(), alls[:, :, self.D].contiguous())
        return o, sel


class CudaShardOps:
    """The shard operations on libaoakv.so (current torch stream)."""

    def __init__(self, num_heads: int, head_dim: int, page_size: int):
        self.H, self.D, self.P = num_heads, head_dim, page_size
        self._ws: Optional[torch.Tensor] = None
        self._rows: dict = {}

    @staticmethod
    def _stream(t: torch.Tensor):
        return torch.cuda.current_stream(t.device).cuda_stream

    def _workspace(self, n_slots: int, device) -> tuple[int, int]:
        need = _lib.size_query("aoakv_decode_workspace_size", self.H, self.D, n_slots)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
        return self._ws.data_ptr(), self._ws.numel()

    def append_decode(self, layer: ShardLayer, k_new, v_new):
        n_meta = -(-layer.n_local // self.P)
        meta_last = (layer.n_local - 1) % self.P + 1
        _lib.call("aoakv_append_kv_cache_decode", k_new.data_ptr(), v_new.data_ptr(),
                  layer.kv.data_ptr(), layer.kv_idx.data_ptr(), layer.n_local, layer.last_len,
                  layer.kv.size(0), layer.meta.data_ptr(), layer.meta_idx.data_ptr(), n_meta,
                  meta_last, layer.meta.size(0), layer.vlog.data_ptr(), self.H, self.D, self.P,
                  _lib.LAYOUT_NHD, self._stream(k_new))

    def local_topk(self, q, layer: ShardLayer, n_score: int, ks: int, mode: str, sink: bool):
        dev = q.device
        scores = torch.empty(self.H, n_score, dtype=torch.float32, device=dev)
        # describe n_score + 1 pages: the estimate scores all but the last
        # one it is told about, and never reads that extra page
        n_desc = n_score + 1
        _lib.call("aoakv_estimate_attn_score", q.data_ptr(), scores.data_ptr(), _lib.DTYPE_F32,
                  n_score, layer.meta.data_ptr(), layer.meta_idx.data_ptr(),
                  -(-n_desc // self.P), (n_desc - 1) % self.P + 1, layer.meta.size(0),
                  layer.kv_idx.data_ptr(), layer.kv.size(0), layer.vlog.data_ptr(), self.H,
                  self.D, self.P, _lib.LAYOUT_NHD,
                  _lib.SCORE_AOAKV if mode == "aoakv" else _lib.SCORE_QUEST, self._stream(q))
        key = (layer.page_lo, n_score, dev)
        ids_row = self._rows.get(key)
        if ids_row is None:  # global page ids of the scored pages, made once
            ids_row = torch.arange(layer.page_lo, layer.page_lo + n_score, dtype=torch.int32,
                                   device=dev)
            self._rows[key] = ids_row
        vals = torch.empty(self.H, ks, dtype=torch.float32, device=dev)
        ids = torch.empty(self.H, ks, dtype=torch.int32, device=dev)
        _lib.call("aoakv_topk_filtering", scores.data_ptr(), _lib.DTYPE_F32, n_score,
                  ids_row.data_ptr(), 0, self.H, n_score, ks, vals.data_ptr(), ks,
                  ids.data_ptr(), ks, int(sink), self._stream(q))
        return vals, ids

    def select(self, cand_v, cand_i, ks: int, sink: bool):
        n = cand_v.size(1)
        out = torch.empty(self.H, ks, dtype=torch.int32, device=cand_v.device)
        _lib.call("aoakv_topk_filtering", cand_v.data_ptr(), _lib.DTYPE_F32, n,
                  cand_i.data_ptr(), n, self.H, n, ks, None, 0, out.data_ptr(), ks, int(sink),
                  self._stream(cand_v))
        return out

    def to_local(self, sel, layer: ShardLayer):
        out = torch.empty_like(sel)
        _lib.call("aoakv_map_pages", sel.data_ptr(), sel.numel(), layer.page_lo, layer.n_local,
                  layer.kv_idx.data_ptr(), out.data_ptr(), self._stream(sel))
        return out

    def all_local_pages(self, layer: ShardLayer, n_score: int):
        return layer.kv_idx[:n_score].to(torch.int32).unsqueeze(0).expand(self.H, n_score) \
            .contiguous()

    def decode_partial(self, q, layer: ShardLayer, local):
        dev = q.device
        o_part = torch.empty(self.H, self.D, dtype=torch.float32, device=dev)
        lse = torch.empty(self.H, dtype=torch.float32, device=dev)
        n_sel = 0 if local is None else local.size(1)
        last = layer.last_phys if layer.owns_last else -1
        ws, ws_n = self._workspace(n_sel, dev)
        _lib.call("aoakv_sparse_decode_partial", q.data_ptr(), o_part.data_ptr(), lse.data_ptr(),
                  layer.kv.data_ptr(), layer.kv.size(0),
                  None if local is None else local.data_ptr(), n_sel, n_sel, last,
                  layer.last_len, self.H, self.D, self.P, _lib.LAYOUT_NHD, 0.0, ws, ws_n,
                  self._stream(q))
        return o_part, lse

    def merge(self, o_parts, lse_parts):
        o = torch.empty(self.H, self.D, dtype=torch.float16, device=o_parts.device)
        _lib.call("aoakv_merge_states", o_parts.data_ptr(), lse_parts.data_ptr(),
                  o_parts.size(0), self.H, self.D, o.data_ptr(), None,
                  self._stream(o_parts))
        return o
