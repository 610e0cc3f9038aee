"""Seeded input generation shared by the golden-fixture generator and the tests.

A spec is a dict {"kind": "normal"|"uniform"|"stored", "seed": int, "std": float}.
normal:  np.random.default_rng(seed).standard_normal(shape, dtype=float32) * std
uniform: np.random.default_rng(seed).uniform(-1, 1, numel).astype(float32)
(numpy's PCG64 generator is stable across releases, so the same arrays are
produced on any host.)
"""
from __future__ import annotations

import numpy as np


def generate(spec: dict, shape, dtype: str = "float32", fortran: bool = False) -> np.ndarray:
    kind = spec["kind"]
    rng = np.random.default_rng(int(spec["seed"]))
    if kind == "normal":
        a = rng.standard_normal(tuple(shape), dtype=np.float32)
        std = np.float32(spec.get("std", 1.0))
        if std != 1:
            a *= std
    elif kind == "uniform":
        a = rng.uniform(-1.0, 1.0, int(np.prod(shape))).astype(np.float32).reshape(shape)
    elif kind == "randint":
        a = rng.integers(spec.get("lo", -100), spec.get("hi", 100), tuple(shape), dtype=np.int64)
    else:
        raise ValueError(kind)
    a = a.astype(np.dtype(dtype), copy=False)
    return np.asfortranarray(a) if fortran else a


def special_values(n: int, seed: int) -> np.ndarray:
    """Float32 vector mixing edge values (NaN, +-0, +-inf, subnormals, huge)
    with uniform draws, for relu/add/mul edge-case parity."""
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1.0, 1.0, n).astype(np.float32)
    specials = np.array([np.nan, -np.nan, 0.0, -0.0, np.inf, -np.inf, 1e-45, -1e-45, 1.1754942e-38,
                         -1.1754942e-38, 3.4028235e38, -3.4028235e38, 1.0, -1.0], dtype=np.float32)
    idx = rng.choice(n, size=min(n, 4 * specials.size), replace=False)
    a[idx] = np.resize(specials, idx.size)
    return a
