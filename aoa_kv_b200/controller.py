"""Host-side page table and buffer owner, mirroring quest.utils.

Mirrors kernels/aoa_kv/quest/utils/kv_cache.py:7-133 (KvPool, KvCache) and
controller.py:7-163 (InferenceController) name for name, with the same
allocation order (a fresh pool hands out page 0, 1, 2, ...), the same
per-step index tensors and the same budget rules, so reference callers and
tests drive it unchanged. Additions, all keyword-only with the reference's
behaviour as default:
  * ``method``            "aoakv" (value-aware score, the aoa_kv tree) or "quest"
  * ``sink_first_page``   force page 0 like the simulation's ``fixed`` mode
  * ``decode_step()``     the whole per-layer decode step in one library call
"""
from __future__ import annotations

import torch

from . import _lib


class TensorLayout:
    """utils.py:1-4."""
    NHD = 0
    HND = 1
    FORMAT2STR = {0: "NHD", 1: "HND"}


class KvPool:
    """kv_cache.py:7-68: [num_layers, capacity, 2, block_len, num_heads, head_dim]."""

    def __init__(self, num_layers, num_heads, head_dim, capacity, block_len, dtype, device):
        self._layout = TensorLayout.NHD
        self._buf = torch.empty((num_layers, capacity, 2, block_len, num_heads, head_dim),
                                dtype=dtype, device=device)
        self._free = set(range(capacity))

    @property
    def layout(self):
        return self._layout

    @property
    def buf(self):
        return self._buf

    @property
    def num_layers(self):
        return self._buf.shape[0]

    @property
    def block_len(self):
        return self._buf.shape[3]

    @property
    def num_free_blocks(self):
        return len(self._free)

    @property
    def capacity(self):
        return self._buf.shape[1]

    def alloc_block(self) -> int:
        return self._free.pop()

    def free_block(self, idx: int):
        assert 0 <= idx < self.capacity
        assert idx not in self._free
        self._free.add(idx)


class KvCache:
    """kv_cache.py:71-133: one sequence's page list over a KvPool."""

    def __init__(self, num_layers, num_heads, head_dim, max_seq_len, page_size, dtype, device):
        if max_seq_len <= 0:
            raise ValueError("init_len must be non-negative")
        self._pool = KvPool(num_layers, num_heads, head_dim,
                            (max_seq_len + page_size - 1) // page_size, page_size, dtype, device)
        self._indicies = []
        self._seqlen = 0

    @property
    def pool(self) -> KvPool:
        return self._pool

    @property
    def seqlen(self) -> int:
        return self._seqlen

    @property
    def last_page_len(self) -> int:
        return (self.seqlen - 1) % self._pool.block_len + 1

    @property
    def indicies(self) -> list:
        return self._indicies

    def buf_layer(self, layer_idx: int):
        assert layer_idx < self.pool.num_layers
        return self._pool.buf[layer_idx]

    def append_seq(self, seq_len: int) -> int:
        """Reserves seq_len tokens; returns the number of pages opened."""
        if seq_len <= 0:
            return 0
        appended = 0
        for _ in range(seq_len):
            if self.last_page_len == self._pool.block_len:
                self._indicies.append(self._pool.alloc_block())
                appended += 1
            self._seqlen += 1
        return appended

    def release(self):
        self._seqlen = 0
        for idx in self._indicies:
            self._pool.free_block(idx)
        self._indicies.clear()


class InferenceController:
    """controller.py:7-163."""

    def __init__(self, num_layers, num_heads, head_dim, page_size, page_budget, max_seq_len,
                 dtype, device, *, method: str = "aoakv", sink_first_page: bool = False):
        if dtype != torch.float16:
            raise RuntimeError("aoa_kv_b200 kernels are built for float16 KV caches only")
        if method not in ("aoakv", "quest"):
            raise ValueError(f"method must be 'aoakv' or 'quest', got {method!r}")
        max_kv_pages_num = (max_seq_len + page_size - 1) // page_size
        self.kv_cache = KvCache(num_layers, num_heads, head_dim, max_seq_len, page_size, dtype, device)
        self.metadata_cache = KvCache(num_layers, num_heads, head_dim, max_kv_pages_num, page_size,
                                      dtype, device)
        # controller.py:43-47: [num_layers, max_pages, num_heads], zero-initialised
        self.v_log_norm = torch.zeros((num_layers, max_kv_pages_num, num_heads), dtype=dtype,
                                      device=device)
        self.layout = TensorLayout.NHD
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.page_size = page_size
        self.method = method
        self.sink_first_page = bool(sink_first_page)
        self._page_budget = page_budget
        from .decode_wrapper import BatchDecodeWithPagedKVCacheWrapper
        self._decode_handler = BatchDecodeWithPagedKVCacheWrapper(kv_layout="NHD")

        self.kv_indices_with_last = None
        self.kv_indices_without_last = None
        self.metadata_indices = None
        self.kv_last_page_idx = None
        self.metadata_last_page_idx = None
        self.kv_indptr_for_append = None
        self.metadata_indptr_for_append = None
        self.kv_indptr_for_approx_decode = None
        self.inference_page_budget = None
        self.topk_dout_buffer = None
        self.topk_dindices_buffer = None
        self.topk_buf = None
        self._step_ws = None
        self._step_ws_key = None
        self._layer_ptrs: dict = {}
        self._plans: dict = {}  # layer -> StepPlan (aoakv_step_plan_*)
        self._rope = None  # (rope_scale, rope_theta) when RoPE is fused into decode_step

    @property
    def score_mode(self) -> int:
        return _lib.SCORE_AOAKV if self.method == "aoakv" else _lib.SCORE_QUEST

    def set_page_budget(self, page_budget: int):
        self._page_budget = page_budget

    def prepare_metadata(self, seq_len: int):
        """controller.py:79-84: reserve token slots and metadata entries."""
        appended_new_pages = self.kv_cache.append_seq(seq_len)
        self.metadata_cache.append_seq(appended_new_pages)

    def begin_forward(self, seq_len: int, updateTensor: bool = True):
        """controller.py:88-141: per-step index tensors and top-k buffers."""
        dev = self.device
        if updateTensor:
            self.kv_indptr_for_append = torch.tensor([0, len(self.kv_cache.indicies)],
                                                     dtype=torch.int32, device=dev)
            self.metadata_indptr_for_append = torch.tensor(
                [0, len(self.metadata_cache.indicies)], dtype=torch.int32, device=dev)
            self.kv_last_page_idx = self.kv_cache.indicies[-1]
            self.metadata_last_page_idx = self.metadata_cache.indicies[-1]
        if seq_len > 1:
            if updateTensor:
                self.kv_indices_with_last = torch.tensor(self.kv_cache.indicies, dtype=torch.int32,
                                                         device=dev)
                self.metadata_indices = torch.tensor(self.metadata_cache.indicies,
                                                     dtype=torch.int32, device=dev)
        else:
            cur_page_nums = len(self.kv_cache.indicies)
            assert cur_page_nums > 1  # controller.py:111
            if updateTensor:
                self.kv_indices_with_last = torch.tensor(self.kv_cache.indicies, dtype=torch.int32,
                                                         device=dev)
                self.kv_indices_without_last = torch.tensor(
                    self.kv_cache.indicies[:-1], dtype=torch.int32,
                    device=dev).repeat(self.num_heads, 1)
                self.metadata_indices = torch.tensor(self.metadata_cache.indicies,
                                                     dtype=torch.int32, device=dev)
            self.inference_page_budget = min(self._page_budget, cur_page_nums)
            self.kv_indptr_for_approx_decode = torch.tensor(
                [0, self.inference_page_budget - 1], dtype=torch.int32, device=dev)
            self.topk_dout_buffer = torch.zeros((self.num_heads, self.inference_page_budget - 1),
                                                dtype=self.dtype, device=dev)
            self.topk_dindices_buffer = torch.zeros(
                (self.num_heads, self.inference_page_budget - 1), dtype=torch.int32, device=dev)
            # The reference sizes a RAFT scratch buffer here (controller.py:132); the
            # shared-memory top-k needs none, the attribute stays for callers.
            self.topk_buf = None
            self._decode_handler.begin_forward(self.kv_indptr_for_approx_decode, self.num_heads,
                                               self.num_heads, self.head_dim, self.page_size,
                                               self.dtype)

    def end_forward(self):
        self._decode_handler.end_forward()

    def need_estimate(self) -> bool:
        """controller.py:149-154."""
        if self.inference_page_budget is None:
            return False
        return len(self.kv_cache.indicies) > self.inference_page_budget

    def clean_states(self):
        self.kv_cache.release()
        self.metadata_cache.release()

    def v_log_norm_layer(self, layer_idx: int):
        return self.v_log_norm[layer_idx]

    # ------------------------------------------------------------ additions
    def step_page_budget(self) -> int:
        """Budget handed to the fused step. With the sink the simulation caps
        the token budget at the sequence length first (quest_attention.py:326,
        filter_util.py:373): pages = min(seq_len, budget_tokens) // page_size."""
        if self.sink_first_page:
            return min(self.kv_cache.seqlen, self._page_budget * self.page_size) // self.page_size
        return self._page_budget

    def _ensure_step_workspace(self) -> torch.Tensor:
        key = (self.kv_cache.pool.capacity, max(3, self._page_budget))
        if self._step_ws is None or self._step_ws_key != key:
            need = _lib.size_query("aoakv_step_workspace_size", self.num_heads, self.head_dim,
                                   *key)
            if self._step_ws is None or self._step_ws.numel() < need:
                self._step_ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
            self._step_ws_key = key
        return self._step_ws

    def _layer_buffers(self, layer_idx: int):
        """(kv ptr, kv pages, metadata ptr, metadata pages, v_log_norm ptr) of
        a layer; the pools never move, so this is computed once per layer."""
        t = self._layer_ptrs.get(layer_idx)
        if t is None:
            kv = self.kv_cache.buf_layer(layer_idx)
            meta = self.metadata_cache.buf_layer(layer_idx)
            t = (kv.data_ptr(), kv.shape[0], meta.data_ptr(), meta.shape[0],
                 self.v_log_norm_layer(layer_idx).data_ptr())
            self._layer_ptrs[layer_idx] = t
        return t

    def fuse_rope(self, rope_scale: float = 1.0, rope_theta: float = 1e4):
        """From now on decode_step takes q and k unrotated and applies RoPE
        at the new token's position inside the step (the reference's
        apply_rope_in_place before append_kv, fused); q and k are left
        rotated in place. rope_scale <= 0 turns it off."""
        self._rope = (float(rope_scale), float(rope_theta)) if rope_scale > 0 else None
        for plan in self._plans.values():
            plan.set_rope(*(self._rope or (0.0, 1.0)))

    def step_plan(self, layer_idx: int, max_ctas: int = 0):
        """The layer's StepPlan for the current budget (created on first use,
        re-created only when the budget or the CTA cap changes)."""
        from .step_plan import StepPlan
        budget = self.step_page_budget()
        plan = self._plans.get(layer_idx)
        if plan is None or plan.page_budget != budget or plan.max_ctas != max_ctas:
            kv_p, kv_cap, meta_p, meta_cap, vlog_p = self._layer_buffers(layer_idx)
            if plan is not None:
                plan.close()
            plan = StepPlan(kv_p, kv_cap, meta_p, meta_cap, vlog_p, self.num_heads,
                            self.head_dim, self.page_size, budget, self.score_mode,
                            self.sink_first_page, max_ctas=max_ctas)
            if self._rope:
                plan.set_rope(*self._rope)
            self._plans[layer_idx] = plan
        return plan

    def decode_step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_idx: int,
                    out: torch.Tensor | None = None, selected: torch.Tensor | None = None,
                    max_ctas: int = 0):
        """Append k, v and attend q in one library call (append, estimate,
        top-k, sparse decode) through the layer's StepPlan. Call after
        prepare_metadata(1) and begin_forward(1). q, k, v: [1, H, D] or [H, D]
        fp16. Returns o like q. max_ctas > 0 caps the step's CTAs (several
        requests' steps on separate streams then run side by side)."""
        from .ops import _check_half_cuda, _stream
        for name, t in (("q", q), ("k", k), ("v", v)):
            _check_half_cuda(t, name)
        o = torch.empty_like(q) if out is None else out
        plan = self.step_plan(layer_idx, max_ctas)
        ws = self._ensure_step_workspace()
        plan.run(q, k, v, o, self.kv_indices_with_last, len(self.kv_cache.indicies),
                 self.kv_cache.last_page_len, self.metadata_indices, selected, ws, ws.numel(),
                 _stream(q))
        return o
