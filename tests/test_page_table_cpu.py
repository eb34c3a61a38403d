"""The page-table oracle (oracle/page_table.py) against the reference's own
host allocator: golden vectors written by tests/golden/make_golden.py from
kernels/aoa_kv/quest/utils/kv_cache.py's KvCache, driven as
controller.py:82-87 prepare_metadata drives it. A single sequence on a fresh
pool gets exactly the reference's page ids, metadata page ids and last-page
lengths after every append."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle.page_table import PageTableOracle

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("pt_*.npz"))


def test_page_table_goldens_present():
    assert len(CASES) >= 4


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_kv_cache(name):
    g = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(g["meta"]))
    P, max_len, appends = meta["page_size"], meta["max_seq_len"], meta["appends"]
    cap = (max_len + P - 1) // P
    o = PageTableOracle(1, cap, cap, (cap + P - 1) // P, P)
    for i, n in enumerate(appends):
        o.append(n, 0)
        kv = g["kv_ids"][i]
        mids = g["meta_ids"][i]
        assert o.kv[0] == kv[kv >= 0].tolist(), (name, i)
        assert o.meta[0] == mids[mids >= 0].tolist(), (name, i)
        assert o.last_len(0) == int(g["last_page_len"][i]), (name, i)
    assert o.errors == 0


def test_oracle_shared_pool_counts_and_release():
    P = 16
    o = PageTableOracle(3, 10, 20, 4, P)
    o.append(100, 0)            # 7 pages
    o.append(1, -1)             # seq 0: 101 tokens; seqs 1, 2: first page each
    assert [len(x) for x in o.kv] == [7, 1, 1]
    assert o.kv[0] == list(range(7)) and o.kv[1] == [7] and o.kv[2] == [8]
    assert [o.last_len(r) for r in range(3)] == [5, 1, 1]
    o.append(200, 1)            # 201 tokens = 13 pages > 10: refused, unchanged
    assert o.errors == 1 and o.seq_len[1] == 1
    o.release(0)
    o.append(40, 2)             # 41 tokens: 2 more pages, the released ones first
    assert o.kv[2] == [8, 0, 1]
    assert len(o.meta[2]) == 1
