"""GPU parity of the tcgen05 paged prefill attention (aoakv_prefill_paged;
reference ops/csrc/batch_prefill.cu:27-116) against the CPU oracle
oracle.kernel_tree.prefill_attention, which restates the reference test's
own CPU attention (quest/tests/test_prefill_attention.py:17-40).

  * the reference test's grid (qo_len x kv_len, 32 heads, head_dim 128, page
    size 16) through InferenceController + append_kv + prefill_forward, at
    its tolerance (rtol = atol = 5e-3);
  * GQA, head_dim 64, page sizes 8..128, non-causal, an explicit sm_scale, a
    chunked prefill (qo_len < kv_len), keys growing along the sequence (the
    running-max rescale of O in tensor memory), the log-sum-exp output;
  * unused cache slots hold NaN: the last page's tail must not reach O."""
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import aoa_kv_b200 as ak
from aoa_kv_b200 import _lib
from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu

RTOL = ATOL = 5e-3  # quest/tests/test_prefill_attention.py:11-13 (float16)


def close(got, want, rtol=RTOL, atol=ATOL):
    err = np.abs(got - want) - (atol + rtol * np.abs(want))
    return float(err.max()) <= 0, float(np.abs(got - want).max())


REF_GRID = [(q, k) for q in (13, 24, 51, 77, 244, 311, 502)
            for k in (33, 66, 129, 400, 700, 1110) if q <= k]


@pytest.mark.parametrize("qo_len,kv_len", REF_GRID)
def test_prefill_forward_matches_reference_test_grid(cuda, qo_len, kv_len):
    H, D, P = 32, 128, 16
    g = torch.Generator().manual_seed(qo_len * 10007 + kv_len)
    q = torch.randn(qo_len, H, D, generator=g).half()
    k = torch.randn(kv_len, H, D, generator=g).half()
    v = torch.randn(kv_len, H, D, generator=g).half()
    ctl = ak.InferenceController(1, H, D, P, 1024, 2048, torch.float16, torch.device("cuda"))
    ctl.kv_cache.buf_layer(0).fill_(float("nan"))  # stale slots must not leak into O
    ctl.prepare_metadata(kv_len)
    ctl.begin_forward(kv_len)
    ak.append_kv(k.cuda(), v.cuda(), ctl, 0)
    o = ak.prefill_forward(q.cuda(), ctl, 0)
    ctl.end_forward()
    torch.cuda.synchronize()
    want, _ = kt.prefill_attention(q.numpy(), k.numpy(), v.numpy(), True)
    ok, err = close(o.float().cpu().numpy(), want)
    assert ok, f"max |gpu - oracle| = {err}"
    assert ak.device_error() == 0


def paged(K, V, P, cap, seed):
    """Scatters K, V [S, Hk, D] into NaN-filled pages of a random page table."""
    S, Hk, D = K.shape
    n = (S + P - 1) // P
    rng = np.random.default_rng(seed)
    ids = rng.permutation(cap)[:n].astype(np.int32)
    kv = np.full((cap, 2, P, Hk, D), np.nan, np.float16)
    for i, pid in enumerate(ids):
        t0, t1 = i * P, min(S, i * P + P)
        kv[pid, 0, :t1 - t0] = K[t0:t1]
        kv[pid, 1, :t1 - t0] = V[t0:t1]
    return torch.from_numpy(kv).cuda(), torch.from_numpy(ids).cuda(), (S - 1) % P + 1


CASES = [
    # Sq, Skv, Hq, Hk, D, P, causal, grow
    (1, 1000, 8, 8, 128, 16, True, 0.0),
    (128, 128, 4, 4, 128, 16, True, 0.0),
    (129, 300, 4, 2, 128, 16, True, 0.0),
    (700, 700, 8, 2, 64, 32, True, 0.0),
    (256, 1000, 4, 4, 128, 8, False, 0.0),
    (333, 2000, 4, 1, 128, 128, True, 0.0),
    (300, 5000, 4, 4, 128, 16, True, 0.0),
    (4173, 4173, 2, 2, 128, 16, True, 0.0),
    (1024, 1500, 4, 4, 128, 16, True, 3.0),
    (600, 600, 4, 4, 64, 64, False, 3.0),
]


@pytest.mark.parametrize("Sq,Skv,Hq,Hk,D,P,causal,grow", CASES)
def test_prefill_paged_matches_oracle(cuda, Sq, Skv, Hq, Hk, D, P, causal, grow):
    rng = np.random.default_rng(Sq * 31 + Skv + D)
    q = rng.standard_normal((Sq, Hq, D), dtype=np.float32).astype(np.float16)
    K = rng.standard_normal((Skv, Hk, D), dtype=np.float32)
    if grow:  # scores rise along the sequence: later tiles raise the running max
        K *= (1.0 + grow * np.arange(Skv, dtype=np.float32) / Skv)[:, None, None]
    K = K.astype(np.float16)
    V = rng.standard_normal((Skv, Hk, D), dtype=np.float32).astype(np.float16)
    cap = (Skv + P - 1) // P + 5
    kv, ids, last = paged(K, V, P, cap, Sq + Skv)
    lse = torch.empty(Sq, Hq, dtype=torch.float32, device="cuda")
    o = ak.prefill_with_paged_kv_cache(torch.from_numpy(q).cuda(), kv, ids, last, causal, 0,
                                       lse=lse)
    torch.cuda.synchronize()
    want, want_lse = kt.prefill_attention(q, K, V, causal)
    ok, err = close(o.float().cpu().numpy(), want)
    assert ok, f"max |gpu - oracle| = {err}"
    assert np.abs(lse.cpu().numpy() - want_lse).max() < 2e-3
    assert ak.device_error() == 0


def test_prefill_sm_scale_and_repeat_are_deterministic(cuda):
    Sq = Skv = 500
    H, D, P = 4, 128, 16
    rng = np.random.default_rng(5)
    q = rng.standard_normal((Sq, H, D), dtype=np.float32).astype(np.float16)
    K = rng.standard_normal((Skv, H, D), dtype=np.float32).astype(np.float16)
    V = rng.standard_normal((Skv, H, D), dtype=np.float32).astype(np.float16)
    kv, ids, last = paged(K, V, P, 40, 9)
    qd = torch.from_numpy(q).cuda()
    o1 = ak.prefill_with_paged_kv_cache(qd, kv, ids, last, True, 0, sm_scale=0.3)
    o2 = ak.prefill_with_paged_kv_cache(qd, kv, ids, last, True, 0, sm_scale=0.3)
    torch.cuda.synchronize()
    want, _ = kt.prefill_attention(q, K, V, True, sm_scale=0.3)
    ok, err = close(o1.float().cpu().numpy(), want)
    assert ok, err
    assert torch.equal(o1, o2)


def test_prefill_rejects_qo_longer_than_kv(cuda):
    q = torch.zeros(40, 4, 128, dtype=torch.float16, device="cuda")
    kv = torch.zeros(4, 2, 16, 4, 128, dtype=torch.float16, device="cuda")
    ids = torch.arange(2, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.AoaKvError, match="qo_len <= kv_len"):
        ak.prefill_with_paged_kv_cache(q, kv, ids, 16, True, 0)


PF_GOLDEN = sorted(p.stem for p in (Path(__file__).resolve().parent / "golden").glob("pf_*.npz"))


@pytest.mark.parametrize("name", PF_GOLDEN)
def test_prefill_matches_reference_test_outputs(cuda, name):
    """The kernel against outputs of the reference test's own CPU attention
    (tests/golden/pf_*.npz, test_prefill_attention.py:17-40), at that test's
    tolerance, with the KV scattered over NaN-filled pages."""
    g = np.load(Path(__file__).resolve().parent / "golden" / f"{name}.npz")
    q, K, V = g["q"], g["k"], g["v"]
    P = 16
    kv, ids, last = paged(K, V, P, (K.shape[0] + P - 1) // P + 3, len(name))
    o = ak.prefill_with_paged_kv_cache(torch.from_numpy(q).cuda(), kv, ids, last, True, 0)
    torch.cuda.synchronize()
    ok, err = close(o.float().cpu().numpy(), g["out"].astype(np.float32))
    assert ok, f"max |gpu - reference| = {err}"
