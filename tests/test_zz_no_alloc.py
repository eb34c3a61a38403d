"""aoakv_sparse_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (a runtime that pre-reserves all device memory for its
own pool, a host that gives its plugins no allocator, or a caller that cannot
accept the device synchronisation an allocation may cause). It keeps its
partial states in a fixed 1 MiB array inside the library instead of a caller
workspace.

Checked through the C ABI on two calls in a row (the second reuses the array
the first left behind): bit-identical to aoakv_sparse_decode with a workspace
(same kernel, same page chunks) and within the decode tests' 2e-3 of the CPU
oracle. Also checked: the documented size limit on both sides. This file
sorts last so a run that stops at the first failure has already run every
other test; it also passes alone in a fresh process (the first call does the
per-device set-up)."""
import numpy as np
import pytest
import torch

from aoa_kv_b200 import _lib
from oracle import kernel_tree as kt

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _problem(H, D, n_sel, cap=800, P=16):
    g = torch.Generator(device="cuda").manual_seed(H * 1000 + n_sel)
    kv = torch.randn(cap, 2, P, H, D, device="cuda", generator=g).half()
    q = (torch.randn(H, D, device="cuda", generator=g) * 2).half()
    sel = torch.stack([torch.randperm(cap - 1, device="cuda", generator=g)[:n_sel]
                       for _ in range(H)]).int().contiguous()
    return kv, q, sel


def _noalloc(q, o, kv, cap, sel, n_sel, last, last_len, H, D, P):
    lib = _lib.load()
    return lib.aoakv_sparse_decode_noalloc(q.data_ptr(), o.data_ptr(), kv.data_ptr(), cap,
                                           sel.data_ptr() if n_sel else None, n_sel, n_sel, last,
                                           last_len, H, D, P, 0, 0.0, _stream())


@pytest.mark.parametrize("H,D,n_sel,last_len", [(32, 128, 63, 16), (32, 128, 255, 5),
                                                  (8, 64, 3, 1), (32, 128, 0, 9),
                                                  (32, 128, 503, 7)])
def test_noalloc_decode_matches_workspace_decode(cuda, H, D, n_sel, last_len):
    P, cap = 16, 800
    kv, q, sel = _problem(H, D, n_sel, cap, P)
    last = cap - 1
    sel_ptr = sel.data_ptr() if n_sel else None

    ws_n = _lib.size_query("aoakv_decode_workspace_size", H, D, n_sel)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    o_ws = torch.empty(H, D, dtype=torch.float16, device="cuda")
    _lib.call("aoakv_sparse_decode", q.data_ptr(), o_ws.data_ptr(), kv.data_ptr(), cap, sel_ptr,
              n_sel, n_sel, last, last_len, H, D, P, 0, 0.0, ws.data_ptr(), ws_n, _stream())
    torch.cuda.synchronize()
    cache = kt.LayerCache(cap, H, D, P)
    cache.kv = kv.cpu().numpy()
    oracle = kt.sparse_decode(q.cpu().numpy(), cache, sel.cpu().numpy().astype(np.int64), last,
                              last_len)

    for call in range(2):
        o = torch.full((H, D), float("nan"), dtype=torch.float16, device="cuda")
        assert _noalloc(q, o, kv, cap, sel, n_sel, last, last_len, H, D, P) == _lib.OK, call
        torch.cuda.synchronize()
        assert torch.equal(o, o_ws), call  # same kernel, same chunks: identical bits
        assert np.abs(o.float().cpu().numpy() - oracle).max() < 2e-3, call
    assert _lib.device_error() == 0


def test_noalloc_decode_limit_in_pages(cuda):
    """The documented limit for 32 heads of head_dim 128: 503 selected pages
    run, 504 are refused with AOAKV_ERR_UNSUPPORTED and nothing is launched."""
    H, D, P, cap = 32, 128, 16, 800
    kv, q, sel = _problem(H, D, 504, cap, P)
    o = torch.zeros(H, D, dtype=torch.float16, device="cuda")
    assert _noalloc(q, o, kv, cap, sel, 503, cap - 1, 3, H, D, P) == _lib.OK
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    o.zero_()
    rc = _noalloc(q, o, kv, cap, sel, 504, cap - 1, 3, H, D, P)
    assert rc == 2, _lib.load().aoakv_last_error()
    assert b"1 MiB" in _lib.load().aoakv_last_error()
    torch.cuda.synchronize()
    assert int(o.abs().sum()) == 0  # refused before any launch
    assert _lib.device_error() == 0


def test_noalloc_decode_rejects_oversized_problem(cuda):
    """A problem whose partial states exceed the fixed array is refused with a
    clear error instead of overrunning it."""
    H, D, P, cap, n_sel = 512, 128, 16, 4, 2000
    lib = _lib.load()
    rc = lib.aoakv_sparse_decode_noalloc(1, 1, 1, cap, 1, n_sel, n_sel, 0, 1, H, D, P, 0, 0.0,
                                         None)
    assert rc == 2, lib.aoakv_last_error()
    assert b"1 MiB" in lib.aoakv_last_error()
