"""Host logic of the page-range sharded step (aoa_kv_b200.sharded) on CPU
ranks over gloo: partition, candidate exchange, the cross-rank tie rule,
page-id mapping and the log-sum-exp merge, against the unsharded kernel-tree
oracle on the same sequence.

The kernels are replaced by NumpyShardOps: the oracle's append / estimate /
top-k plus a numpy partial-state decode and merge, so no GPU is needed; the
GPU versions of the same operations are covered by test_gpu_sharded.py."""
import math
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aoa_kv_b200 import sharded
from oracle import kernel_tree as kt


class NumpyShardOps:
    """The shard operations on CPU tensors, computed with the oracle: the
    proposals as the propose kernel writes them ({order key, global id},
    best first, unused entries {0, -1}), the finish pass's ranking, append
    and partial decode, and the log-sum-exp merge."""

    def __init__(self, H, D, P):
        self.H, self.D, self.P = H, D, P

    def _cache(self, layer):
        c = kt.LayerCache(layer.kv.shape[0], self.H, self.D, self.P)
        c.kv, c.meta, c.vlog = layer.kv.numpy(), layer.meta.numpy(), layer.vlog.numpy()
        return c

    def propose(self, q, layer, ks, sink_here):
        n_score = layer.n_local - (1 if layer.owns_last else 0)
        out = np.zeros((self.H, ks, 2), np.int64)
        out[:, :, 1] = sharded.SENTINEL_ID
        if n_score > 0:
            sc = kt.estimate(q.numpy(), self._cache(layer), layer.meta_idx.numpy(),
                             layer.kv_idx.numpy(), n_score + 1, mode=self.mode)
            key = kt.score_keys(sc)
            if sink_here:
                key[:, 0] = 0xFFFFFFFF
            m = min(ks, n_score)
            pos = kt.topk_positions(sc, m, sink_here)
            if m > 256:  # the oracle lists large k by position: best first here
                kk = np.take_along_axis(key, pos, axis=1)
                order = np.lexsort((pos, -kk.astype(np.int64)), axis=1)
                pos = np.take_along_axis(pos, order, axis=1)
            out[:, :m, 0] = np.take_along_axis(key, pos, axis=1)
            out[:, :m, 1] = pos + layer.page_lo
        return torch.from_numpy(out.astype(np.uint32).view(np.int32))

    def finish(self, q, k_new, v_new, layer, cand_all, ks, rank, want_selected):
        c = self._cache(layer)
        if layer.owns_last:
            kt.append_decode(c, layer.kv_idx.numpy(), layer.meta_idx.numpy(), layer.n_local,
                             layer.last_len, k_new.numpy(), v_new.numpy())
        n_mine = layer.n_local - (1 if layer.owns_last else 0)
        sel = None
        if cand_all is not None:
            ca = cand_all.numpy().view(np.uint32).astype(np.int64)  # [G, H, ks, 2]
            G = ca.shape[0]
            sel = np.zeros((self.H, ks), np.int32)
            local = []
            for h in range(self.H):
                ent = ca[:, h].reshape(G * ks, 2)
                ent = ent[ent[:, 1] != 0xFFFFFFFF]
                order = np.lexsort((ent[:, 1], -ent[:, 0]))[:ks]
                win = ent[order, 1]
                sel[h] = win
                rel = win - layer.page_lo
                local.append([int(layer.kv_idx[r]) for r in rel if 0 <= r < n_mine])
            sel = torch.from_numpy(sel)
        else:
            k_all = ks == 0 and layer.n_total <= self._k(layer.n_total)
            local = [[int(p) for p in layer.kv_idx[:n_mine]] if k_all else []] * self.H
        return torch.from_numpy(self._partial(q, layer, local)), sel if want_selected else None

    def _k(self, n_total):
        kp = max(3, self.budget) if self.sink else self.budget
        return min(kp, n_total)

    def _partial(self, q, layer, local):
        kv = layer.kv.numpy()
        qf = q.numpy().astype(np.float32)
        st = np.zeros((self.H, self.D + 1), np.float32)
        st[:, self.D] = -np.inf
        for h in range(self.H):
            ks = [kv[p, 0, :, h] for p in local[h]]
            vs = [kv[p, 1, :, h] for p in local[h]]
            if layer.owns_last:
                ks.append(kv[layer.last_phys, 0, :layer.last_len, h])
                vs.append(kv[layer.last_phys, 1, :layer.last_len, h])
            if not ks:
                continue
            K = np.concatenate(ks).astype(np.float32)
            V = np.concatenate(vs).astype(np.float32)
            w = (K @ qf[h]) / math.sqrt(self.D)
            m = w.max()
            e = np.exp(w - m)
            st[h, :self.D] = (e / e.sum()) @ V
            st[h, self.D] = m + math.log(e.sum())
        return st

    def merge(self, states):
        s = states.numpy()
        op, lp = s[..., :self.D], s[..., self.D]
        m = lp.max(axis=0)
        w = np.where(np.isfinite(lp), np.exp(lp - m[None]), 0.0)
        o = (w[..., None] * op).sum(axis=0) / w.sum(axis=0)[:, None]
        return torch.from_numpy(o.astype(np.float16))


def make_sequence(seed, H, D, S, ties):
    g = np.random.default_rng(seed)
    q = g.standard_normal((H, D)).astype(np.float16)
    K = (g.standard_normal((S + 1, H, D)) * np.exp(g.standard_normal((H, D)))).astype(np.float16)
    V = g.standard_normal((S + 1, H, D)).astype(np.float16)
    if ties:  # every page gets the same score: the lowest page ids must win
        K[:] = np.float16(0.5)
        V[: S // 2] = np.float16(1.0)
    return q, K, V


def build_shard(rank, world, q, K, V, H, D, P, S, permute_seed):
    """Prefills this rank's page range of the S-token sequence (the new
    token's page already reserved on the last rank) in a local pool with
    permuted physical pages."""
    n_total = S // P + 1
    last_len = S % P + 1
    lo, hi = sharded.partition_pages(n_total, world, P)[rank]
    n_local = hi - lo
    cap = n_local + 3
    g = np.random.default_rng(permute_seed + rank)
    c = kt.LayerCache(cap, H, D, P, seed_garbage=permute_seed)
    kv_idx = g.permutation(cap)[:n_local].astype(np.int32)
    meta_idx = g.permutation(c.mcap)[: -(-n_local // P)].astype(np.int32)
    t0, t1 = lo * P, min(hi * P, S)  # tokens already in the sequence
    owns_last = rank == world - 1
    if t1 > t0:
        n_pref = -(-(t1 - t0) // P)
        kt.append_prefill(c, kv_idx, meta_idx, n_pref, (t1 - t0 - 1) % P + 1, K[t0:t1], V[t0:t1])
    layer = sharded.ShardLayer(
        kv=torch.from_numpy(c.kv), meta=torch.from_numpy(c.meta), vlog=torch.from_numpy(c.vlog),
        kv_idx=torch.from_numpy(kv_idx), meta_idx=torch.from_numpy(meta_idx), page_lo=lo,
        n_local=n_local, n_total=n_total, last_len=last_len, owns_last=owns_last,
        last_phys=int(kv_idx[n_local - 1]) if owns_last else -1)
    return layer


def _worker(rank, world, port, out_dir, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, D, P, S = case["H"], case["D"], case["P"], case["S"]
        q, K, V = make_sequence(case["seed"], H, D, S, case["ties"])
        layer = build_shard(rank, world, q, K, V, H, D, P, S, case["seed"] + 100)
        ops = NumpyShardOps(H, D, P)
        ops.mode, ops.budget, ops.sink = case["mode"], case["budget"], case["sink"]
        dec = sharded.ShardedDecoder(dist.group.WORLD, H, D, P, case["budget"], case["mode"],
                                     case["sink"], ops=ops)
        o, sel = dec.step(layer, torch.from_numpy(q), torch.from_numpy(K[S]),
                          torch.from_numpy(V[S]))
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), o=o.float().numpy(),
                 sel=np.zeros((0,)) if sel is None else sel.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CASES = [
    dict(H=4, D=16, P=4, S=300, budget=8, mode="aoakv", sink=False, ties=False, seed=1, world=2),
    dict(H=4, D=16, P=4, S=300, budget=8, mode="quest", sink=True, ties=False, seed=2, world=3),
    dict(H=3, D=16, P=4, S=257, budget=6, mode="aoakv", sink=True, ties=False, seed=3, world=2),
    dict(H=4, D=16, P=4, S=300, budget=8, mode="quest", sink=False, ties=True, seed=4, world=2),
    dict(H=2, D=16, P=4, S=60, budget=40, mode="aoakv", sink=False, ties=False, seed=5, world=2),
    dict(H=2, D=16, P=4, S=61, budget=1, mode="quest", sink=False, ties=False, seed=6, world=2),
    dict(H=3, D=16, P=2, S=203, budget=9, mode="aoakv", sink=True, ties=False, seed=7, world=4),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['mode']}-w{c['world']}-B{c['budget']}"
                         f"{'-sink' if c['sink'] else ''}{'-ties' if c['ties'] else ''}")
def test_sharded_step_matches_unsharded_oracle(case):
    H, D, P, S, world = case["H"], case["D"], case["P"], case["S"], case["world"]
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_worker, args=(world, _free_port(), tmp, case), nprocs=world,
                           join=True, start_method="spawn")
        outs = [np.load(os.path.join(tmp, f"r{r}.npz")) for r in range(world)]
    # unsharded oracle: identity physical ids, the same sequence
    q, K, V = make_sequence(case["seed"], H, D, S, case["ties"])
    n_total, last_len = S // P + 1, S % P + 1
    c = kt.LayerCache(n_total + 1, H, D, P)
    idx = np.arange(n_total + 1, dtype=np.int32)
    midx = np.arange(-(-(n_total + 1) // P), dtype=np.int32)
    kt.append_prefill(c, idx, midx, -(-S // P), (S - 1) % P + 1, K[:S], V[:S])
    want_o, want_sel = kt.step(q, K[S], V[S], c, idx, midx, n_total, last_len, case["budget"],
                               case["mode"], case["sink"])
    kp = max(3, case["budget"]) if case["sink"] else case["budget"]
    k = min(kp, n_total)
    for r, out in enumerate(outs):
        assert np.abs(out["o"] - want_o).max() < 2e-3, f"rank {r}"
        if n_total > k and k > 1:
            assert np.array_equal(np.sort(out["sel"], axis=1), np.sort(want_sel[:, :-1], axis=1))
    if case["ties"]:
        ks = k - 1
        assert np.array_equal(np.sort(outs[0]["sel"], axis=1),
                              np.tile(np.arange(ks), (H, 1)))


def test_partition_pages_whole_metadata_pages():
    assert sharded.partition_pages(8192, 8, 16) == [(g * 1024, (g + 1) * 1024) for g in range(8)]
    assert sharded.partition_pages(76, 3, 4) == [(0, 28), (28, 56), (56, 76)]
    for n, w, p in [(1000, 3, 16), (77, 2, 4), (33, 4, 2)]:
        r = sharded.partition_pages(n, w, p)
        assert r[0][0] == 0 and r[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert all(lo % p == 0 for lo, _ in r)
    with pytest.raises(ValueError):
        sharded.partition_pages(20, 8, 16)


def test_short_shard_pads_its_proposals():
    """A rank with fewer pages than k-1 proposes them all and pads the rest
    with {0, -1}, which never win."""
    H, D, P = 2, 16, 4
    g = np.random.default_rng(0)
    c = kt.LayerCache(8, H, D, P)
    idx = np.arange(5, dtype=np.int32)
    midx = np.arange(2, dtype=np.int32)
    kt.append_prefill(c, idx, midx, 4, P, g.standard_normal((16, H, D)).astype(np.float16),
                      g.standard_normal((16, H, D)).astype(np.float16))
    layer = sharded.ShardLayer(kv=torch.from_numpy(c.kv), meta=torch.from_numpy(c.meta),
                               vlog=torch.from_numpy(c.vlog), kv_idx=torch.from_numpy(idx[:4]),
                               meta_idx=torch.from_numpy(midx), page_lo=0, n_local=4,
                               n_total=100, last_len=1, owns_last=False)
    ops = NumpyShardOps(H, D, P)
    ops.mode = "aoakv"
    cand = ops.propose(torch.from_numpy(g.standard_normal((H, D)).astype(np.float16)), layer, 9,
                       False).numpy()
    assert cand.shape == (H, 9, 2)
    assert sorted(cand[0, :4, 1].tolist()) == [0, 1, 2, 3]
    assert (cand[:, 4:, 1] == -1).all() and (cand[:, 4:, 0] == 0).all()
    keys = cand[:, :4, 0].view(np.uint32)
    assert (np.diff(keys.astype(np.int64), axis=1) <= 0).all()  # best first
