"""The page-range sharded step on real GPUs, one process per GPU (needs 2):
both exchanges — NCCL all_gathers and the kernels' own peer stores into
each other's mailboxes over NVLink — against the unsharded kernel-tree
oracle, for several tokens in a row (one mailbox reused across layers and
tokens). Skipped with fewer than 2 GPUs."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
H, D, P = 32, 128, 16


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cases():
    # (S cached tokens, budget pages, mode, sink)
    return [(8192 + 5, 64, "aoakv", False), (12000, 40, "quest", True), (600, 64, "aoakv", False)]


def _worker(rank, port, out_dir):
    import datetime

    import torch.distributed as dist

    from aoa_kv_b200 import _lib, sharded
    from gen import gen_qkv
    from gpu_util import GpuLayer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        out = {}
        for ci, (S, budget, mode, sink) in enumerate(_cases()):
            q, K, V = gen_qkv(S + 3, H, S + 1, D, "outlier")
            n_total, last_len = S // P + 1, S % P + 1
            lo, hi = sharded.partition_pages(n_total, WORLD, P)[rank]
            n_local = hi - lo
            lay = GpuLayer(n_local + 2, H, D, P, seed=100 + rank)
            t0, t1 = lo * P, min(hi * P, S)
            if t1 > t0:
                lay.fill(K[t0:t1], V[t0:t1])
            owns = rank == WORLD - 1
            layer = sharded.ShardLayer(
                kv=lay.kv, meta=lay.meta, vlog=lay.vlog, kv_idx=lay.kv_idx[:n_local].contiguous(),
                meta_idx=lay.meta_idx, page_lo=lo, n_local=n_local, n_total=n_total,
                last_len=last_len, owns_last=owns,
                last_phys=int(lay.kv_idx_np[n_local - 1]) if owns else -1)
            args = (torch.from_numpy(q).to(dev), torch.from_numpy(K[S]).to(dev),
                    torch.from_numpy(V[S]).to(dev))
            for exchange in ("nccl", "p2p"):
                dec = sharded.ShardedDecoder(dist.group.WORLD, H, D, P, budget, mode, sink,
                                             exchange=exchange, device=dev)
                for t in range(3):
                    o, sel = dec.step(layer, *args)
                    torch.cuda.synchronize()
                    out[f"o_{ci}_{exchange}_{t}"] = o.float().cpu().numpy()
                    if sel is not None:
                        out[f"sel_{ci}_{exchange}_{t}"] = sel.cpu().numpy()
                if dec.mailbox is not None:
                    dist.barrier()
                    dec.mailbox.close()
        out["dev_err"] = np.array([_lib.device_error()])
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), **out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_step_two_gpus_both_exchanges(cuda):
    from gen import gen_qkv
    from helpers import selection_mismatch
    from oracle import kernel_tree as kt
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_worker, args=(_free_port(), tmp), nprocs=WORLD, join=True,
                           start_method="spawn")
        outs = [dict(np.load(os.path.join(tmp, f"r{r}.npz"))) for r in range(WORLD)]
    for r in range(WORLD):
        assert int(outs[r]["dev_err"][0]) == 0, f"rank {r}"
    for ci, (S, budget, mode, sink) in enumerate(_cases()):
        q, K, V = gen_qkv(S + 3, H, S + 1, D, "outlier")
        n_total, last_len = S // P + 1, S % P + 1
        c = kt.LayerCache(n_total + 1, H, D, P)
        idx = np.arange(n_total + 1, dtype=np.int32)
        midx = np.arange(c.mcap, dtype=np.int32)
        kt.append_prefill(c, idx, midx, -(-S // P), (S - 1) % P + 1, K[:S], V[:S])
        want_o, want_sel = kt.step(q, K[S], V[S], c, idx, midx, n_total, last_len, budget, mode,
                                   sink)
        kp = max(3, budget) if sink else budget
        k = min(kp, n_total)
        scores = None
        if n_total > k:
            scores = kt.estimate(q, c, midx, idx, n_total, mode)
            scores = np.concatenate([scores, np.full((H, 1), np.inf, np.float32)], axis=1)
            if sink:
                scores[:, 0] = np.inf
        for r in range(WORLD):
            for exchange in ("nccl", "p2p"):
                for t in range(3):
                    o = outs[r][f"o_{ci}_{exchange}_{t}"]
                    tag = f"case {ci} rank {r} {exchange} token {t}"
                    # every rank, both exchanges: the same output
                    assert np.array_equal(o, outs[0][f"o_{ci}_nccl_0"]), tag
                    if scores is None:
                        assert np.abs(o - want_o).max() < 2e-3, tag
                        continue
                    sel = outs[r][f"sel_{ci}_{exchange}_{t}"]
                    g = np.array([sorted(row.tolist()) for row in sel])
                    w = np.array([sorted(row.tolist()) for row in want_sel[:, :-1]])
                    assert not selection_mismatch(g, w, scores), tag
                    if np.array_equal(g, w):
                        assert np.abs(o - want_o).max() < 2e-3, tag
