"""Shared test utilities: golden-file loading and selection comparison."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


def golden_names(prefix: str) -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz"))


def selection_mismatch(sel_a: np.ndarray, sel_b: np.ndarray, scores: np.ndarray,
                       rtol: float = 1e-3) -> list[tuple[int, int, float, float]]:
    """Pages selected by one side only whose score is NOT within rtol of the
    selection threshold (the k-th largest score of the row), relative to
    that threshold (plus 1e-5 absolute, the fp32 summation-order noise of a
    score near zero). An empty list means the selections agree up to
    near-ties.

    sel_a, sel_b: [H, k] page ids; scores: [H, N] indexed by page id.
    Returns (head, page, score, threshold) for each genuine mismatch."""
    bad = []
    for h in range(sel_a.shape[0]):
        a, b = set(map(int, sel_a[h])), set(map(int, sel_b[h]))
        if a == b:
            continue
        k = len(a)
        row = scores[h].astype(np.float64)
        thr = np.sort(row)[::-1][k - 1] if k <= len(row) else row.min()
        tol = rtol * abs(thr) + 1e-5
        for p in a ^ b:
            if abs(row[p] - thr) > tol:
                bad.append((h, p, float(row[p]), float(thr)))
    return bad
