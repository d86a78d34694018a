"""Benchmark and parity-accounting host logic, without a GPU.

* The reference arm (`bench.py --impl reference`) maps no shared library of this repository other than the
  oracle, and prints the same `config` as the GPU arm.
* tests/parity.py counts a planted flip and measures its distance to the oracle's nearest CDF boundary.
"""

import json
import os
import subprocess
import sys

import numpy as np

from oracle import oracle
from tests.parity import boundary_distance, compare
from voxwerk_b200 import workloads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import io, json, sys, contextlib
sys.path.insert(0, sys.argv[1])
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--config", "1"]
import bench
buf = io.StringIO()
with contextlib.redirect_stdout(buf):
    bench.main()
maps = [ln.split()[-1] for ln in open("/proc/self/maps") if ln.rstrip().endswith(".so")]
mine = sorted({m for m in maps if m.startswith(bench.ROOT)})
print(json.dumps({"line": json.loads(buf.getvalue().strip().splitlines()[-1]), "repo_so": mine}))
"""


def test_reference_arm_maps_only_the_oracle():
    res = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out["repo_so"] == [os.path.join(ROOT, "oracle", "liboracle.so")], out["repo_so"]
    line = out["line"]
    assert line["impl"] == "reference" and line["e2e"]["h2d_bytes_per_step"] == 0
    sys.path.insert(0, ROOT)
    import bench
    assert line["config"] == bench.bench_config(workloads.make(1), 1)


def test_boundary_distance():
    p = np.array([0.0, 0.25, 0.0, 0.5, 0.25])
    assert boundary_distance(p, 0.25) == 0.0
    assert abs(boundary_distance(p, 0.7) - 0.05) < 1e-15
    assert boundary_distance(np.zeros(4), 0.5) == float("inf")


def test_compare_counts_and_attributes_a_planted_flip():
    w = workloads.make(2, 64)
    seg = w.segments[0]
    ref = oracle.sample_segment(seg, w.options, threads=4)
    assert compare(w, [ref])["flips"] == 0
    bad = ref.copy()
    bad[7] = (bad[7] + 1) % seg.vocab
    c = compare(w, [bad])
    assert c["rows"] == 64 and c["flips"] == 1
    assert c["first_flips"][0][:4] == (0, 7, int(bad[7]), int(ref[7]))
    _, probs = oracle.sample_segment(seg.take([7]), w.options, want_probs=True)
    assert c["max_boundary_dist"] == boundary_distance(probs[0], float(seg.uniforms[7]))


def test_take_matches_slice():
    w = workloads.make(2, 16)
    s = w.segments[0]
    a, b = s.take(np.arange(3, 9)), s.slice(3, 9)
    for f in ("logits", "uniforms", "opt_index", "hist_offsets", "hist_ids", "steps"):
        np.testing.assert_array_equal(getattr(a, f), getattr(b, f))
