"""vw_head_sample: the tcgen05 vocabulary-head GEMM, then the sampler on its logits.

The GEMM (bf16 in, fp32 accumulate and out) is checked against a float64 product of the same bf16 inputs: each logit
within 1e-4 x sum_k |hidden_k * weight_k| (fp32 accumulation over K <= 2048 terms stays orders of magnitude inside
it; a wrong descriptor, swizzle or tile offset misses it by O(1)).  The ids must equal the CPU oracle's on the GEMM's
own logits, bit for bit, and those of vw_sample run separately on the same logits.
"""

import os

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import REPORT
from tests.gpu_util import make_segment, options_table, to_device
from voxwerk_b200 import workloads
from voxwerk_b200.workloads import F32, SegData

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1
GEMM_RTOL = 1e-4


def _operands(torch, n, V, H, seed, w_scale=0.125):
    g = torch.Generator(device="cpu").manual_seed(seed)
    hidden = torch.randn((n, H), generator=g).to(torch.bfloat16).cuda()
    weight = (torch.randn((V, H), generator=g) * w_scale).to(torch.bfloat16).cuda()
    return hidden, weight


def _check_gemm(torch, hidden, weight, got):
    h, w = hidden.double(), weight.double()
    ref = h @ w.T
    bound = h.abs() @ w.abs().T
    err = (got.double() - ref).abs()
    worst = float((err / bound.clamp_min(1e-30)).max())
    assert bool((err <= GEMM_RTOL * bound + 1e-30).all()), f"GEMM error {worst:.3e} of sum|a*b| exceeds {GEMM_RTOL}"
    return worst


# tile widths the host picks for these shapes (148 SMs): 32 (rows 1 .. 257, 6 x 3072 x 256, 1 x 1024, 1 x 2048),
# 64 (300, 273 x 3072 x 512, 137), 96 (386, 392 x 3072 x 2048), 128 (519, 8192 x 2048), 192 (771), 256 (1156, 4096);
# 4096 x 3072 and 8192 x 2048 give each persistent CTA several tiles (both accumulators reused); 257 x 1000 x 1000 is
# ragged in N and K
@pytest.mark.parametrize("n,V,H", [(1, 3072, 1024), (64, 3072, 1024), (130, 2048, 1024), (257, 1000, 1000),
                                   (16, 3072, 2048), (300, 3072, 1024), (386, 3072, 1024), (519, 3072, 1024),
                                   (771, 3072, 1024), (1156, 3072, 1024), (4096, 3072, 1024), (8192, 2048, 1024),
                                   (6, 3072, 256), (1, 1024, 1024), (273, 3072, 512), (1, 2048, 1024),
                                   (137, 3072, 1024), (392, 3072, 2048)])
def test_head_gemm_matches_float64(device, n, V, H):
    import torch
    from voxwerk_b200 import SamplingOptions, Segment, head_logits, head_sample, vw_options
    hidden, weight = _operands(torch, n, V, H, seed=n * 7 + V)
    logits = torch.full((n, V), float("nan"), dtype=torch.float32, device="cuda")
    seg = Segment(None, kind=workloads.SUB, vocab=V, out_ids=torch.full((n,), -1, dtype=torch.int32, device="cuda"),
                  uniforms=torch.zeros(n, dtype=torch.float64, device="cuda"),
                  opt_index=torch.zeros(n, dtype=torch.int32, device="cuda"))
    head_sample(device, hidden, weight, seg, [vw_options(SamplingOptions.greedy())], out_logits=logits)
    assert not bool(torch.isnan(logits).any()), "the GEMM left logits unwritten"
    worst = _check_gemm(torch, hidden, weight, logits)
    alone = torch.full((n, V), float("nan"), dtype=torch.float32, device="cuda")
    head_logits(device, hidden, weight, alone)          # the GEMM-only entry writes the same logits
    assert torch.equal(alone.view(torch.int32), logits.view(torch.int32))
    REPORT.append(f"head GEMM {n}x{V}x{H}: max error {worst:.2e} of sum|a*b|")
    # greedy ids are the argmax of the GEMM's logits (Sampler.ArgMax: first maximum)
    np.testing.assert_array_equal(seg.out_ids.cpu().numpy(), logits.cpu().numpy().argmax(axis=1))


@pytest.mark.parametrize("cfg,rows,H", [(2, 512, 1024), (1, None, 1024), (3, 16, 1024), (2, 37, 2048)])
def test_head_sample_ids_match_oracle(device, cfg, rows, H):
    """Talker rows (histories, penalty, mask, top-k/top-p) and sub-talker rows: the ids of one vw_head_sample call
    equal the oracle's on the logits that call's GEMM produced."""
    import torch
    from voxwerk_b200 import head_sample, sample_rows
    w = workloads.make(cfg, rows)
    opts = options_table(w)
    for k, sd in enumerate(w.segments):
        hidden, weight = _operands(torch, sd.n_rows, sd.vocab, H, seed=100 + 10 * cfg + k)
        arr = to_device(sd, torch)
        arr["logits"] = None
        seg = make_segment(sd, arr)
        logits = torch.empty((sd.n_rows, sd.vocab), dtype=torch.float32, device="cuda")
        head_sample(device, hidden, weight, seg, opts, out_logits=logits)
        got = arr["out_ids"].cpu().numpy()
        host_logits = logits.cpu().numpy()
        ref_seg = SegData(host_logits, F32, sd.kind, sd.vocab, sd.uniforms, sd.opt_index, sd.hist_offsets,
                          sd.hist_ids, sd.steps, sd.suppress_lo, sd.suppress_hi, sd.eos_id, sd.min_new_tokens)
        ref = oracle.sample_segment(ref_seg, w.options, threads=THREADS)
        bad = np.flatnonzero(got != ref)
        assert bad.size == 0, f"{w.name} segment {k}: {bad.size} of {got.size} ids differ, rows {bad[:10]}"
        # the handle's own logits buffer (no out_logits) gives the same ids
        arr2 = to_device(sd, torch)
        arr2["logits"] = None
        head_sample(device, hidden, weight, make_segment(sd, arr2), opts)
        np.testing.assert_array_equal(arr2["out_ids"].cpu().numpy(), got)
        # and vw_sample over the same logits gives the same ids
        arr3 = to_device(sd, torch)
        arr3["logits"] = logits
        sample_rows(device, [make_segment(sd, arr3)], opts)
        np.testing.assert_array_equal(arr3["out_ids"].cpu().numpy(), got)
        REPORT.append(f"head+sample {w.name} segment {k}: {got.size} rows (H {H}), ids equal to the oracle's")


def test_head_sample_rejects_bad_operands(device):
    import torch
    from voxwerk_b200 import Segment, SamplingOptions, VwInvalidArgument, head_sample, vw_options
    hidden, weight = _operands(torch, 8, 2048, 1024, seed=5)
    opts = [vw_options(SamplingOptions.greedy())]
    mk = lambda n, V: Segment(None, kind=workloads.SUB, vocab=V,
                              out_ids=torch.full((n,), -1, dtype=torch.int32, device="cuda"),
                              uniforms=torch.zeros(n, dtype=torch.float64, device="cuda"),
                              opt_index=torch.zeros(n, dtype=torch.int32, device="cuda"))
    flat = torch.empty(8 * 1024 + 8, dtype=torch.bfloat16, device="cuda")
    misaligned = flat[1:1 + 8 * 1024].view(8, 1024)          # 2-byte offset: not 16-byte aligned
    misaligned.copy_(hidden)
    with pytest.raises(VwInvalidArgument):
        head_sample(device, misaligned, weight, mk(8, 2048), opts)
    with pytest.raises(VwInvalidArgument):                    # H not a multiple of 8
        head_sample(device, hidden[:, :1020], weight[:, :1020], mk(8, 2048), opts)
    with pytest.raises(VwInvalidArgument):                    # vocab not a multiple of 4
        head_sample(device, hidden, weight[:2046], mk(8, 2046), opts)
    seg = mk(8, 2048)                                         # the handle still works
    head_sample(device, hidden, weight, seg, opts)
    logits = torch.empty((8, 2048), dtype=torch.float32, device="cuda")
    seg2 = mk(8, 2048)
    head_sample(device, hidden, weight, seg2, opts, out_logits=logits)
    np.testing.assert_array_equal(seg2.out_ids.cpu().numpy(), logits.argmax(dim=1).cpu().numpy())
    np.testing.assert_array_equal(seg.out_ids.cpu().numpy(), seg2.out_ids.cpu().numpy())
