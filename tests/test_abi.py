"""C-ABI checks that need no GPU: the library loads, exports exactly what
include/aoakv.h declares, and rejects bad arguments with status codes
before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

import aoa_kv_b200
from aoa_kv_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "aoakv.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"AOAKV_API\s+[\w\s\*]+?\b(aoakv_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "aoakv_decode_step" in names and "aoakv_topk_filtering" in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes table out of sync with the header"


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_version_and_empty_error():
    lib = _lib.load()
    assert lib.aoakv_version() == 10000
    assert isinstance(lib.aoakv_last_error(), bytes)


def _expect(rc_name, *args, code=1, match=""):
    lib = _lib.load()
    rc = getattr(lib, rc_name)(*args)
    assert rc == code, (rc_name, rc, lib.aoakv_last_error())
    assert match in lib.aoakv_last_error().decode()


def test_topk_rejects_k_above_n():
    _expect("aoakv_topk_filtering", 1, 0, 10, None, 0, 1, 10, 11, None, 0, 1, 11, 0, None,
            match="k must be in")


def test_topk_rejects_huge_rows():
    _expect("aoakv_topk_filtering", 1, 0, 60000, None, 0, 1, 60000, 5, None, 0, 1, 5, 0, None,
            match="num_pages")


def test_estimate_rejects_hnd_layout():
    _expect("aoakv_estimate_attn_score", 1, 1, 0, 100, 1, 1, 2, 1, 4, None, 4, None, 32, 128, 16,
            1, 0, None, code=2, match="NHD")


def test_append_rejects_inconsistent_metadata():
    # metadata_last_page_len must equal ((num_kv_pages-1) % P) + 1
    _expect("aoakv_append_kv_cache_decode", 1, 1, 1, 1, 5, 3, 8, 1, 1, 1, 3, 1, 1, 32, 128, 16,
            0, None, match="metadata_last_page_len")


def test_decode_rejects_bad_head_dim():
    _expect("aoakv_sparse_decode", 1, 1, 1, 8, 1, 4, 4, 0, 1, 32, 96, 16, 0, ctypes.c_float(0.0),
            None, 0, None, match="head_dim")


def test_decode_workspace_size_monotone():
    a = _lib.size_query("aoakv_decode_workspace_size", 32, 128, 63)
    b = _lib.size_query("aoakv_decode_workspace_size", 32, 128, 255)
    assert 0 < a < b


def test_step_workspace_size():
    n = _lib.size_query("aoakv_step_workspace_size", 32, 128, 2048, 64)
    assert n >= 32 * 2048 * 4


def test_call_raises_with_message():
    with pytest.raises(aoa_kv_b200.AoaKvError, match="INVALID_ARG"):
        _lib.call("aoakv_topk_filtering", 1, 0, 10, None, 0, 1, 10, 0, None, 0, 1, 0, 0, None)


def test_partial_decode_argument_checks():
    f0 = ctypes.c_float(0.0)
    _expect("aoakv_sparse_decode_partial", 1, 1, None, 1, 8, 1, 4, 4, 0, 1, 32, 128, 16, 0, f0,
            None, 0, None, match="NULL")
    _expect("aoakv_sparse_decode_partial", 1, 1, 1, 1, 8, 1, 4, 4, -2, 1, 32, 128, 16, 0, f0,
            None, 0, None, match="last_page_idx")
    # -1 ("the last page is on another GPU") is only for the partial decode
    _expect("aoakv_sparse_decode", 1, 1, 1, 8, 1, 4, 4, -1, 1, 32, 128, 16, 0, f0, None, 0, None,
            match="last_page_idx")


def test_merge_and_map_argument_checks():
    _expect("aoakv_merge_states", 1, 1, 0, 32, 128, 1, None, None, match="bad sizes")
    _expect("aoakv_merge_states", None, 1, 2, 32, 128, 1, None, None, match="NULL")
    _expect("aoakv_map_pages", 1, -1, 0, 4, 1, 1, None, match="bad sizes")
    _expect("aoakv_map_pages", 1, 0, 0, 4, 1, 1, None, code=0)  # nothing to map: no launch


def _prefill_args(qo_len=10, n_pages=2, last=16, hq=32, hk=32, d=128, p=16, causal=1):
    # q, o, lse, kv_data, cap, kv_indices, n_pages, last_len, qo_len, hq, hk, d, p, layout,
    # causal, sm_scale, stream (pointers are dummies: every case fails or returns before use)
    return (16, 16, None, 16, 8, 16, n_pages, last, qo_len, hq, hk, d, p, 0, causal,
            ctypes.c_float(0.0), None)


def test_prefill_rejects_bad_shapes():
    _expect("aoakv_prefill_paged", *_prefill_args(d=96), match="head_dim")
    _expect("aoakv_prefill_paged", *_prefill_args(p=24), match="page_size")
    _expect("aoakv_prefill_paged", *_prefill_args(hq=12, hk=8), match="multiple")
    _expect("aoakv_prefill_paged", *_prefill_args(last=17), match="kv_last_page_len")
    # causal needs qo_len <= kv_len = (2 - 1) * 16 + 3 = 19
    _expect("aoakv_prefill_paged", *_prefill_args(qo_len=20, last=3), match="qo_len <= kv_len")


def test_prefill_empty_query_is_a_no_op():
    _expect("aoakv_prefill_paged", *_prefill_args(qo_len=0), code=0)
