"""GPU parity of the page-range sharded step (aoa_kv_b200.sharded with
CudaShardOps: the propose and finish passes of the cluster step kernel and
the packed-state merge) against the unsharded kernel-tree oracle. The ranks
are emulated as threads on one GPU that exchange tensors through an
in-process all_gather (the host waits for each pass, so no kernel waits on
another), so the test needs a single GPU; bench.py runs the same code over
NCCL."""
import threading

import numpy as np
import pytest
import torch

from aoa_kv_b200 import _lib, sharded
from gen import gen_qkv
from gpu_util import GpuLayer
from helpers import selection_mismatch
from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu


class ThreadGroup:
    """all_gather among `world` threads that share one GPU."""

    def __init__(self, world):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=60)
        self.slots = [None] * world
        self.local = threading.local()

    def all_gather_stack(self, t):
        torch.cuda.synchronize()
        self.slots[self.local.rank] = t
        self.barrier.wait()
        out = torch.stack(self.slots)
        torch.cuda.synchronize()
        self.barrier.wait()
        return out


def run_sharded(world, q, K, V, S, H, D, P, budget, mode, sink):
    n_total, last_len = S // P + 1, S % P + 1
    ranges = sharded.partition_pages(n_total, world, P)
    group = ThreadGroup(world)
    results, errors = [None] * world, []

    def rank_main(r):
        try:
            torch.cuda.set_device(0)
            group.local.rank = r
            lo, hi = ranges[r]
            n_local = hi - lo
            lay = GpuLayer(n_local + 2, H, D, P, seed=100 + r)
            t0, t1 = lo * P, min(hi * P, S)
            if t1 > t0:
                lay.fill(K[t0:t1], V[t0:t1])
            owns = r == world - 1
            layer = sharded.ShardLayer(
                kv=lay.kv, meta=lay.meta, vlog=lay.vlog, kv_idx=lay.kv_idx[:n_local].contiguous(),
                meta_idx=lay.meta_idx, page_lo=lo, n_local=n_local, n_total=n_total,
                last_len=last_len, owns_last=owns,
                last_phys=int(lay.kv_idx_np[n_local - 1]) if owns else -1)
            dec = sharded.ShardedDecoder(group, H, D, P, budget, mode, sink, rank=r)
            o, sel = dec.step(layer, torch.from_numpy(q).cuda(), torch.from_numpy(K[S]).cuda(),
                              torch.from_numpy(V[S]).cuda())
            torch.cuda.synchronize()
            results[r] = (o.float().cpu().numpy(), None if sel is None else sel.cpu().numpy())
        except BaseException as e:  # surfaced by the main thread
            errors.append(e)
            group.barrier.abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    return results


@pytest.mark.parametrize("world,S,budget,mode,sink,ties", [
    (2, 8192 + 5, 64, "aoakv", False, False),
    (4, 8192 + 5, 64, "quest", True, False),
    (3, 32768, 300, "aoakv", False, False),   # k-1 = 299 proposals per rank
    (8, 32768, 256, "quest", False, False),   # 8 x 255 candidates per head
    (4, 1000, 40, "aoakv", False, False),     # shards shorter than k-1: padded lists
    (2, 8192 + 5, 64, "quest", False, True),  # equal scores: the lowest pages win
    (2, 700, 100, "aoakv", False, False),     # every page attended
    (2, 700, 1, "aoakv", False, False),       # only the last page
])
def test_sharded_step_matches_oracle(cuda, world, S, budget, mode, sink, ties):
    H, D, P = 32, 128, 16
    q, K, V = gen_qkv(S + world, H, S + 1, D, "outlier")
    if ties:  # every page gets the same quest score
        K[:] = np.float16(0.5)
    results = run_sharded(world, q, K, V, S, H, D, P, budget, mode, sink)
    n_total, last_len = S // P + 1, S % P + 1
    c = kt.LayerCache(n_total + 1, H, D, P)
    idx = np.arange(n_total + 1, dtype=np.int32)
    midx = np.arange(c.mcap, dtype=np.int32)
    kt.append_prefill(c, idx, midx, -(-S // P), (S - 1) % P + 1, K[:S], V[:S])
    want_o, want_sel = kt.step(q, K[S], V[S], c, idx, midx, n_total, last_len, budget, mode, sink)
    kp = max(3, budget) if sink else budget
    k = min(kp, n_total)
    for r, (o, sel) in enumerate(results):
        if n_total > k and k > 1:
            scores = kt.estimate(q, c, midx, idx, n_total, mode)
            scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
            if sink:
                scores[:, 0] = np.inf
            g = [sorted(row.tolist()) for row in sel]
            w = [sorted(row.tolist()) for row in want_sel[:, :-1]]
            if ties:
                assert g == [list(range(k - 1))] * H, f"rank {r}"
            assert not selection_mismatch(np.array(g), np.array(w), scores), f"rank {r}"
            if g == w:
                assert np.abs(o - want_o).max() < 2e-3, f"rank {r}"
            else:  # near-tie swap: compare with the oracle on the pages chosen
                o_ref = kt.sparse_decode(q, c, np.array(g), int(idx[n_total - 1]), last_len)
                assert np.abs(o - o_ref).max() < 2e-3, f"rank {r}"
        else:
            assert np.abs(o - want_o).max() < 2e-3, f"rank {r}"


class SoloGroup:
    """The all_gather of a one-rank job."""
    world = 1

    @staticmethod
    def all_gather_stack(t):
        return t.unsqueeze(0)


def test_sharded_p2p_one_rank_matches_oracle(cuda):
    """The peer-store exchange with one rank (its own mailbox): two layers of
    different lengths, one attended densely and one with a selection,
    interleaved for three tokens, so the per-exchange counters advance
    unevenly; every output and selection matches the oracle."""
    H, D, P = 32, 128, 16
    cases = []
    for S, budget in ((700, 64), (8192 + 5, 64)):
        q, K, V = gen_qkv(S + 11, H, S + 1, D, "outlier")
        n_total, last_len = S // P + 1, S % P + 1
        lay = GpuLayer(n_total + 2, H, D, P, seed=5)
        lay.fill(K[:S], V[:S])
        layer = sharded.ShardLayer(
            kv=lay.kv, meta=lay.meta, vlog=lay.vlog, kv_idx=lay.kv_idx[:n_total].contiguous(),
            meta_idx=lay.meta_idx, page_lo=0, n_local=n_total, n_total=n_total,
            last_len=last_len, owns_last=True, last_phys=int(lay.kv_idx_np[n_total - 1]))
        c = kt.LayerCache(n_total + 1, H, D, P)
        idx = np.arange(n_total + 1, dtype=np.int32)
        midx = np.arange(c.mcap, dtype=np.int32)
        kt.append_prefill(c, idx, midx, -(-S // P), (S - 1) % P + 1, K[:S], V[:S])
        want_o, want_sel = kt.step(q, K[S], V[S], c, idx, midx, n_total, last_len, budget,
                                   "aoakv", False)
        cases.append((layer, q, K[S], V[S], want_o, want_sel, n_total > budget))
    dec = sharded.ShardedDecoder(SoloGroup(), H, D, P, 64, "aoakv", exchange="p2p")
    for _ in range(3):
        for layer, q, kn, vn, want_o, want_sel, sparse in cases:
            o, sel = dec.step(layer, torch.from_numpy(q).cuda(), torch.from_numpy(kn).cuda(),
                              torch.from_numpy(vn).cuda())
            torch.cuda.synchronize()
            assert np.abs(o.float().cpu().numpy() - want_o).max() < 2e-3
            if sparse:
                assert [sorted(r) for r in sel.cpu().numpy().tolist()] == \
                    [sorted(r) for r in want_sel[:, :-1].tolist()]
    assert _lib.device_error() == 0
    dec.mailbox.close()
