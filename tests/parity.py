"""Id parity with flip accounting: GPU ids against the CPU oracle over every row of a workload.

A "flip" is a row whose GPU id differs from the oracle's.  For every flip the oracle's own final distribution
(the probabilities its draw scans, Sampler.cs:77-87) gives the CDF boundaries in index order; the row's distance
|r - nearest boundary| says whether the flip is attributable to the uniform lying at a boundary (the benchmark
specification accepts a flip only within 1e-6 of one).  Test and benchmark infrastructure: it calls the oracle.
"""

from __future__ import annotations

import os
from typing import List, Sequence

import numpy as np

from oracle import oracle

BOUNDARY_TOL = 1e-6


def boundary_distance(probs: np.ndarray, r: float) -> float:
    """|r - nearest boundary| of the index-order CDF over the positive probabilities (the draw's scan)."""
    p = probs[probs > 0]
    if p.size == 0:
        return float("inf")
    acc = np.cumsum(p)   # the boundary positions; the sequential rounding is irrelevant at 1e-6
    return float(np.min(np.abs(acc - r)))


def compare(w, got: Sequence[np.ndarray], threads: int = 0) -> dict:
    """{"rows", "flips", "attributable", "max_boundary_dist", "first_flips"} of `got` (ids per segment) vs the
    oracle on workload `w`."""
    threads = threads or os.cpu_count() or 1
    rows = flips = attributable = 0
    worst = None
    first: List[tuple] = []
    for k, (seg, ids) in enumerate(zip(w.segments, got)):
        ref = oracle.sample_segment(seg, w.options, threads=threads)
        rows += int(ref.size)
        bad = np.flatnonzero(np.asarray(ids) != ref)
        if bad.size == 0:
            continue
        flips += int(bad.size)
        sub_p = oracle.sample_segment(seg.take(bad), w.options, threads=threads, want_probs=True)[1]
        for j, r in enumerate(bad):
            d = boundary_distance(sub_p[j], float(seg.uniforms[r]))
            worst = d if worst is None else max(worst, d)
            attributable += int(d <= BOUNDARY_TOL)
            if len(first) < 8:
                first.append((k, int(r), int(ids[r]), int(ref[r]), d))
    return {"rows": rows, "flips": flips, "attributable": attributable, "max_boundary_dist": worst,
            "first_flips": first}
