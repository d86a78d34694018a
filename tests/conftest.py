import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# measured figures the tests report (exp mismatch counts, parity and flip counts), printed after the run
REPORT = []


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if REPORT:
        terminalreporter.section("measured")
        for line in REPORT:
            terminalreporter.write_line(line)


@pytest.fixture(scope="session")
def device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from voxwerk_b200 import Device
    d = Device(0)
    yield d
    d.close()
