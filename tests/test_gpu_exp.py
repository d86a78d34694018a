"""The device exp against the host C library's exp (what the oracle and the reference's Math.Exp call).

Every softmax argument of the five benchmark configurations, plus seeded arguments over the whole range, goes
through vw_exp_diagnostic.  The sampler's exp (the restatement in vw_libm_exp.h) must equal the C library's bit for
bit; CUDA's own exp is measured beside it and its mismatch count reported (it is not used by the sampler).
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import REPORT
from tests.exp_args import config_args, edge_args

pytestmark = pytest.mark.gpu


def _device_exps(device, x):
    import torch
    from voxwerk_b200._lib import check, lib
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    a = torch.empty_like(xd)
    b = torch.empty_like(xd)
    check(lib.vw_exp_diagnostic(device.handle, ctypes.c_void_p(xd.data_ptr()), xd.numel(),
                                ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr())), device.handle)
    return a.cpu().numpy(), b.cpu().numpy()


def _same(a, b):
    return (a == b) | (np.isnan(a) & np.isnan(b))


@pytest.mark.parametrize("which", ["configs", "range"])
def test_device_exp_equals_c_library(device, which):
    x = config_args() if which == "configs" else edge_args()
    ours, cuda = _device_exps(device, x)
    ref = oracle.glibc_exp(x)
    bad = np.flatnonzero(~_same(ours, ref))
    cuda_bad = int((~_same(cuda, ref)).sum())
    REPORT.append(f"exp ({which}): {x.size} arguments; sampler exp != C library exp: {bad.size}; "
                  f"CUDA exp != C library exp: {cuda_bad} ({100.0 * cuda_bad / x.size:.3f} %)")
    assert bad.size == 0, [(float(x[i]).hex(), float(ours[i]).hex(), float(ref[i]).hex()) for i in bad[:5]]
