"""The sequential replay paths (taken when a parallel decision lies inside the error band) against the oracle.

VW_FORCE_EXACT=1 at handle creation routes every sampled row through the replay, so these tests pin code that
ordinary inputs reach only rarely.  They run in a child process so the setting cannot leak into other tests.
"""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, os, sys
sys.path.insert(0, sys.argv[1])
import numpy as np
from oracle import oracle
from tests.gpu_util import run_workload
from voxwerk_b200 import Device, workloads
out = {}
with Device(0) as dev:
    for cfg, rows in ((0, None), (1, None), (2, 256), (3, 16), (4, 256)):
        w = workloads.make(cfg, rows)
        got = run_workload(dev, w)
        ok = all(np.array_equal(g, oracle.sample_segment(s, w.options, threads=os.cpu_count()))
                 for g, s in zip(got, w.segments))
        out[str(cfg)] = ok
    dev.synchronize()
    out["stats"] = dev.stats()
print(json.dumps(out))
"""


def test_forced_replay_matches_oracle():
    env = dict(os.environ, VW_FORCE_EXACT="1")
    res = subprocess.run([sys.executable, "-c", CHILD, ROOT], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    st = out.pop("stats")
    assert all(out.values()), out
    assert st["rows_fast"] == 0 and st["rows_general"] == 0, st
    assert st["rows_fast_replayed"] > 0 and st["rows_general_replayed"] > 0, st


STALL_CHILD = r"""
import json, os, sys
sys.path.insert(0, sys.argv[1])
import numpy as np
from oracle import oracle
from tests.gpu_util import run_workload
from voxwerk_b200 import Device, VwError, workloads
out = {}
with Device(0) as dev:
    w = workloads.make(4, 512)   # top-k off: every sampling row goes through the whole-row kernel
    try:
        run_workload(dev, w)
        out["first"] = "ok"
    except VwError as e:
        out["first"] = e.status
    got = run_workload(dev, w)
    out["second_exact"] = bool(np.array_equal(got[0], oracle.sample_segment(w.segments[0], w.options, threads=8)))
print(json.dumps(out))
"""


def test_timeout_is_reported_and_the_handle_recovers():
    """VW_TEST_STALL_ROW: the whole-row kernel's producer withholds one row's stage, so an element warp's bounded mbarrier
    wait (cut to 1 ms by the hook) runs out.  The call returns VW_ERR_TIMEOUT; the next call on the same handle is
    bit-exact against the oracle.  No wait is unbounded, so nothing hangs."""
    env = dict(os.environ, VW_TEST_STALL_ROW="101")   # a sampling row (every 10th row is greedy)
    res = subprocess.run([sys.executable, "-c", STALL_CHILD, ROOT], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out == {"first": 4, "second_exact": True}, out


def test_parallel_paths_are_taken(device):
    from tests.gpu_util import run_workload
    from voxwerk_b200 import workloads
    device.stats(reset=True)
    run_workload(device, workloads.make(2, 512))
    run_workload(device, workloads.make(4, 256))
    device.synchronize()
    st = device.stats(reset=True)
    assert st["rows_fast"] > 400, st
    assert st["rows_general"] > 150, st
    assert st["rows_greedy"] > 0, st
