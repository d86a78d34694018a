"""vw_sample_static, the entry point that allocates no device memory, against vw_sample on the same inputs.

Kept in its own file, collected last, so that it runs both after every other test (the library's shared static
scratch has then seen other calls) and alone.  Ids must be identical; probabilities within the 1e-6 relative
tolerance of the parity tests.  Each workload runs through vw_sample_static twice in a row.
"""

import numpy as np
import pytest

from oracle import oracle
from tests.gpu_util import make_segment, options_table, to_device
from voxwerk_b200 import Segment, VwInvalidArgument, sample_rows, sample_rows_static, workloads
from voxwerk_b200._lib import VW_ROWS_SUB, VwOptions

PROB_RTOL = 1e-6


def _run(w, call, want_probs):
    import torch
    segs, outs, probs = [], [], []
    for seg in w.segments:
        arr = to_device(seg, torch)
        pr = torch.zeros((seg.n_rows, seg.vocab), dtype=torch.float64, device="cuda") if want_probs else None
        segs.append(make_segment(seg, arr, pr))
        outs.append(arr["out_ids"])
        probs.append(pr)
    call(segs, options_table(w))
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs], [p.cpu().numpy() if p is not None else None for p in probs]


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,rows,want_probs", [(0, None, True), (1, None, True), (2, 1024, False), (2, 96, True),
                                                 (3, None, False), (4, 1024, False), (4, 96, True)])
def test_static_matches_vw_sample_twice(device, cfg, rows, want_probs):
    w = workloads.make(cfg, rows)
    ref_ids, ref_probs = _run(w, lambda s, o: sample_rows(device, s, o), want_probs)
    for call in range(2):
        ids, probs = _run(w, lambda s, o: sample_rows_static(0, s, o), want_probs)
        for k, (g, r) in enumerate(zip(ids, ref_ids)):
            bad = np.flatnonzero(g != r)
            assert bad.size == 0, f"{w.name} call {call} segment {k}: {bad.size} ids differ, rows {bad[:10]}"
        if want_probs:
            for g, r in zip(probs, ref_probs):
                np.testing.assert_allclose(g, r, rtol=PROB_RTOL, atol=0.0)
    # and against the CPU oracle directly, so a regression shared by both entry points shows too
    for seg, got in zip(w.segments, ids):
        np.testing.assert_array_equal(got, oracle.sample_segment(seg, w.options, threads=8))


@pytest.mark.gpu
def test_static_allocates_nothing_and_recovers_after_an_error(device):
    """Repeated calls leave the device's free memory unchanged; a call that ends in an error (a history id out of
    range, which the kernel checks and reports) leaves the shared array usable for the next call."""
    import torch
    from voxwerk_b200 import VwOutOfRange
    w = workloads.make(2, 512)
    run = lambda: _run(w, lambda s, o: sample_rows_static(0, s, o), False)[0]
    run()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        ids = run()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    bad = workloads.make(2, 512)
    bad.segments[0].hist_ids[100] = 5000
    with pytest.raises(VwOutOfRange):
        _run(bad, lambda s, o: sample_rows_static(0, s, o), False)
    again = run()
    for g, r in zip(again, ids):
        np.testing.assert_array_equal(g, r)
    np.testing.assert_array_equal(again[0], oracle.sample_segment(w.segments[0], w.options, threads=8))


@pytest.mark.gpu
def test_static_rejects_host_pointers(device):
    """Every array of a segment must be device memory: a host array fails with a status, not a fault."""
    import ctypes
    import torch
    from voxwerk_b200._lib import VW_ERR_INVALID_ARG, VwSegment, lib
    w = workloads.make(1)
    seg = w.segments[0]
    c = make_segment(seg, to_device(seg, torch)).to_c(0)
    host_uniforms = torch.from_numpy(seg.uniforms).pin_memory()
    c.uniforms = host_uniforms.data_ptr()
    msg = ctypes.create_string_buffer(256)
    opts = (VwOptions * 1)(*options_table(w))
    st = lib.vw_sample_static(0, (VwSegment * 1)(c), 1, opts, 1, None, msg, len(msg))
    assert st == VW_ERR_INVALID_ARG and b"uniforms must be device memory" in msg.value, (st, msg.value)


@pytest.mark.gpu
def test_static_rejects_sizes_beyond_its_limits(device):
    import torch
    opts = [VwOptions(1, 50, 0.8, 0.9, 1.0)]
    logits = torch.zeros((4, 8192), dtype=torch.float32, device="cuda")
    out = torch.zeros(4, dtype=torch.int32, device="cuda")
    uni = torch.zeros(4, dtype=torch.float64, device="cuda")
    big_vocab = Segment(logits, kind=VW_ROWS_SUB, vocab=8192, out_ids=out, uniforms=uni)
    with pytest.raises(VwInvalidArgument, match="vocab 8192 exceeds"):
        sample_rows_static(0, [big_vocab], opts)
    many = torch.zeros((65537, 16), dtype=torch.float32, device="cuda")
    seg = Segment(many, kind=VW_ROWS_SUB, vocab=16, out_ids=torch.zeros(65537, dtype=torch.int32, device="cuda"),
                  uniforms=torch.zeros(65537, dtype=torch.float64, device="cuda"))
    with pytest.raises(VwInvalidArgument, match="65537 rows exceed"):
        sample_rows_static(0, [seg], opts)
    small = torch.zeros((4, 2048), dtype=torch.float32, device="cuda")
    with pytest.raises(VwInvalidArgument, match="at most 32 options"):
        sample_rows_static(0, [Segment(small, kind=VW_ROWS_SUB, vocab=2048, out_ids=out, uniforms=uni)], opts * 33)


def test_static_limits_checked_before_any_device_work():
    """The row limit is enforced on the host, before the device is touched (runs without a GPU)."""
    import ctypes
    from voxwerk_b200._lib import VwSegment, lib, VW_ERR_INVALID_ARG, VW_F32
    seg = VwSegment()
    seg.logits = 1 << 20
    seg.row_stride = 16
    seg.n_rows = 70000
    seg.vocab = 16
    seg.dtype = VW_F32
    seg.kind = VW_ROWS_SUB
    seg.out_ids = 1 << 21
    seg.uniforms = 1 << 22
    opts = (VwOptions * 1)(VwOptions(1, 5, 0.8, 0.9, 1.0))
    msg = ctypes.create_string_buffer(256)
    st = lib.vw_sample_static(0, (VwSegment * 1)(seg), 1, opts, 1, None, msg, len(msg))
    assert st == VW_ERR_INVALID_ARG
    assert b"70000 rows exceed" in msg.value
