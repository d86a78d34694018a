"""Arguments for the exp checks: every value the oracle's softmax passes to exp on the five benchmark
configurations (unique), plus seeded random arguments over the whole range the sampler can produce (x <= 0, down
to the underflow of exp) and a few edge values.  Test infrastructure."""

from __future__ import annotations

import numpy as np

from oracle import oracle
from voxwerk_b200 import workloads


def config_args() -> np.ndarray:
    parts = []
    for c in range(5):
        w = workloads.make(c)
        parts += [oracle.exp_args(s, w.options).astype(np.float64) for s in w.segments]
    return np.unique(np.concatenate(parts))


def edge_args(seed: int = 3) -> np.ndarray:
    rng = np.random.default_rng(seed)
    edges = np.array([0.0, -0.0, -1e-300, -2.0 ** -54, -2.0 ** -55, -2.0 ** -53, -1.0, -512.0, -511.9999999,
                      -708.3964185322641, -709.0, -744.44, -745.1332191019411, -745.2, -1023.9, -1024.0, -1e9,
                      -np.inf, 1.0, 700.0, 709.78, 800.0, np.inf, np.nan])
    return np.concatenate([edges, -rng.random(300000) * 745.5, -rng.random(300000) * 50, -rng.random(100000) * 1e-3,
                           -745.2 + rng.random(50000) * 3, -700 + rng.random(50000) * 200])
