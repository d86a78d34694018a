"""The sampler's exp (voxwerk_b200/csrc/vw_libm_exp.h) compiled for the host, against the C library's exp.

voxwerk's softmax calls Math.Exp (Sampler.cs:57), i.e. the C runtime's exp; the oracle calls the same function.
The device must reproduce its values bit for bit for the sequential replays to equal the reference, so the
restatement is checked here, on the CPU, on every softmax argument of the five benchmark configurations and on
seeded arguments over the whole range (the GPU test then checks the device build against the same values).
"""

import os
import subprocess
import sys

import numpy as np
import pytest

from tests.exp_args import config_args, edge_args

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    d = tmp_path_factory.mktemp("exp")
    exe = str(d / "exp_host_check")
    subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math",
                    "-I", os.path.join(ROOT, "voxwerk_b200", "csrc"), os.path.join(ROOT, "tests", "exp_host_check.cpp"),
                    "-o", exe, "-lm"], check=True)
    return exe, d


def _run(checker, args):
    exe, d = checker
    path = str(d / "args.bin")
    np.ascontiguousarray(args, dtype=np.float64).tofile(path)
    out = subprocess.run([exe, path], capture_output=True, text=True, check=True).stdout.strip().splitlines()
    n, bad = (int(v) for v in out[-1].split())
    return n, bad, out[:-1]


def test_libm_exp_matches_c_library_on_config_arguments(checker, record_property):
    args = config_args()
    n, bad, first = _run(checker, args)
    record_property("exp_args", n)
    sys.stderr.write(f"\nlibm_exp vs C library exp: {bad} of {n} softmax arguments of configs 0-4 differ\n")
    assert n == args.size and bad == 0, first


def test_libm_exp_matches_c_library_over_the_range(checker):
    args = edge_args()
    n, bad, first = _run(checker, args)
    assert n == args.size and bad == 0, first
