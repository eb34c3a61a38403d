"""Seeded synthetic inputs shared by the golden-vector script and the tests.

Inputs are regenerated from (seed, shape, distribution) with numpy's PCG64
generator and rounded to fp16, so fixtures store only outputs plus a SHA-256
of the inputs (a test fails loudly if regeneration ever diverges).

Distributions (the benchmark configurations):
  "normal"  : q, K, V ~ N(0, 1)                                  (config 1)
  "outlier" : K = N(0, 1) * s[h, d], s ~ LogNormal(0, 1) per channel; q, V
              ~ N(0, 1)                                          (config 2)
Layouts are the reference's NHD: q [H, D], K and V [S, H, D].
"""
from __future__ import annotations

import hashlib

import numpy as np


def gen_qkv(seed: int, H: int, S: int, D: int, dist: str = "normal"):
    g = np.random.default_rng(seed)
    q = g.standard_normal((H, D), dtype=np.float32)
    K = g.standard_normal((S, H, D), dtype=np.float32)
    V = g.standard_normal((S, H, D), dtype=np.float32)
    if dist == "outlier":
        scale = np.exp(g.standard_normal((H, D), dtype=np.float32))
        K = K * scale[None]
    elif dist != "normal":
        raise ValueError(dist)
    return q.astype(np.float16), K.astype(np.float16), V.astype(np.float16)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def gen_gqa(seed: int, Hq: int, Hkv: int, S: int, D: int, dist: str = "normal"):
    """GQA inputs: K, V [S, Hkv, D] as gen_qkv draws them for Hkv heads, and
    q [Hq, D] from a second generator (seed + 7777)."""
    _, K, V = gen_qkv(seed, Hkv, S, D, dist)
    q = np.random.default_rng(seed + 7777).standard_normal((Hq, D), dtype=np.float32)
    return q.astype(np.float16), K, V
