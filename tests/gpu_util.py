"""Helpers that run a workloads.Workload through the C ABI (test and benchmark infrastructure)."""

from __future__ import annotations

from typing import List

import numpy as np

from voxwerk_b200 import Segment, sample_rows, vw_options
from voxwerk_b200._lib import VwOptions


def options_table(w) -> List[VwOptions]:
    return [VwOptions(int(o[0]), int(o[1]), float(o[2]), float(o[3]), float(o[4])) for o in w.options]


def _logits_view(seg):
    return seg.logits.view(np.int16) if seg.logits.dtype == np.uint16 else seg.logits


def to_device(seg, torch, device="cuda"):
    """Device copies of a SegData's arrays (dict of tensors)."""
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return dict(logits=t(_logits_view(seg)), uniforms=t(seg.uniforms), opt_index=t(seg.opt_index),
                hist_offsets=t(seg.hist_offsets), hist_ids=t(seg.hist_ids), steps=t(seg.steps),
                out_ids=torch.full((seg.n_rows,), -1, dtype=torch.int32, device=device))


def make_segment(seg, arrays, out_probs=None, max_hist_len=0) -> Segment:
    return Segment(arrays["logits"], kind=seg.kind, vocab=seg.vocab, out_ids=arrays["out_ids"],
                   uniforms=arrays["uniforms"], opt_index=arrays["opt_index"], hist_offsets=arrays["hist_offsets"],
                   hist_ids=arrays["hist_ids"], steps=arrays["steps"], suppress_lo=seg.suppress_lo,
                   suppress_hi=seg.suppress_hi, eos_id=seg.eos_id, min_new_tokens=seg.min_new_tokens,
                   max_hist_len=max_hist_len, out_probs=out_probs)


def run_workload(dev, w, mem: str = "device", want_probs: bool = False, stream=None):
    """Ids per segment (numpy), and probabilities if asked."""
    import torch
    segs, outs, probs = [], [], []
    for seg in w.segments:
        if mem == "device":
            arr = to_device(seg, torch)
            pr = torch.zeros((seg.n_rows, seg.vocab), dtype=torch.float64, device="cuda") if want_probs else None
        else:
            arr = dict(logits=_logits_view(seg), uniforms=seg.uniforms, opt_index=seg.opt_index,
                       hist_offsets=seg.hist_offsets, hist_ids=seg.hist_ids, steps=seg.steps,
                       out_ids=np.full(seg.n_rows, -1, dtype=np.int32))
            pr = np.zeros((seg.n_rows, seg.vocab), dtype=np.float64) if want_probs else None
        segs.append(make_segment(seg, arr, pr))
        outs.append(arr["out_ids"])
        probs.append(pr)
    sample_rows(dev, segs, options_table(w), stream=stream)
    if stream is not None:
        dev.synchronize(stream)
    conv = lambda a: a.cpu().numpy() if hasattr(a, "cpu") else a
    ids = [conv(o) for o in outs]
    if want_probs:
        return ids, [conv(p) for p in probs]
    return ids
