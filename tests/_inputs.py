"""Seeded inputs shared by the tests (CPU numpy + device copies)."""

from __future__ import annotations

import numpy as np

from stockfish_trainer_b200 import positions


def feature_batch(n: int, feature_set: str, seed: int = 0):
    """White / black [n, K] int32 indices of n synthetic positions, and T."""
    white, black, _ = positions.synthetic_batch(n, feature_set, seed=seed)
    T = positions.feature_set_info(feature_set)[1]
    return white, black, T


def random_table(T: int, C: int, seed: int = 0, std: float = 0.01) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((T, C), dtype=np.float32) * np.float32(std)).astype(np.float32)


def random_indices(B: int, K: int, T: int, seed: int = 0, holes: bool = True) -> np.ndarray:
    """Unique indices per row; -1 anywhere in the row when ``holes``."""
    rng = np.random.default_rng(seed)
    idx = np.full((B, K), -1, np.int32)
    for b in range(B):
        n = int(rng.integers(0, min(K, T) + 1))
        vals = rng.choice(T, size=n, replace=False).astype(np.int32)
        if holes:
            pos = rng.choice(K, size=n, replace=False)
            idx[b, pos] = vals
        else:
            idx[b, :n] = vals
    return idx
