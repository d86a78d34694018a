"""Device-resident batch state (vw_batch_*) against the reference's GenerateBatch loop run on the host.

TalkerGenerator.GenerateBatch (TalkerGenerator.cs:322-455) per frame: every active job samples codebook 0 with its
history penalised and EOS suppressed while Step < 2 (:366-372), appends it to its history (:374), retires on EOS or
at Step == MaxNewTokens - 1 (:375-380); the survivors sample codebooks 1..15 from their Seed + 1 sampler (:416-420)
and advance their step (:440).  A freed slot is refilled with a new job (:336-358).  The host side of this test
runs exactly that loop with the CPU oracle and DotNetRandom; the device side keeps all of it in a vw_batch.
"""

import numpy as np
import pytest

from oracle import oracle
from voxwerk_b200.dotnet_random import DotNetRandom
from voxwerk_b200.workloads import SegData

pytestmark = pytest.mark.gpu


class HostJob:
    def __init__(self, opts, history=()):
        self.opts = opts
        self.rng = DotNetRandom(opts.seed)
        self.sub_rng = DotNetRandom(opts.seed + 1)
        self.history = list(history)
        self.step = 0
        self.done = False


def _talker_ref(job, row):
    o = job.opts
    u = job.rng.next_double() if o.talker.do_sample else 0.0
    seg = SegData(row[None, :], 0, 0, 3072, np.array([u]), None, np.array([0, len(job.history)], np.int64),
                  np.array(job.history or [0], np.int32), np.array([job.step], np.int32), 2048, 3072, 2150, 2)
    return int(oracle.sample_segment(seg, [(int(o.talker.do_sample), o.talker.top_k, o.talker.top_p,
                                            o.talker.temperature, o.repetition_penalty)])[0])


def _sub_ref(job, row):
    o = job.opts.sub_talker
    u = job.sub_rng.next_double() if o.do_sample else 0.0
    return int(oracle.select(row, (int(o.do_sample), o.top_k, o.top_p, o.temperature, 1.0), u))


def test_device_batch_matches_generate_batch_loop(device):
    import torch
    from voxwerk_b200 import DeviceBatchState, GenerationOptions, SamplingOptions
    rng = np.random.default_rng(2024)
    jobs = [GenerationOptions(seed=100 + j, max_new_tokens=5 if j == 1 else 64,
                              repetition_penalty=1.3 if j % 2 else 1.05,
                              talker=SamplingOptions(top_p=0.8 if j % 3 else 1.0),
                              sub_talker=SamplingOptions(top_k=20 if j == 2 else 50)) for j in range(5)]
    jobs.append(GenerationOptions(seed=7, talker=SamplingOptions.greedy(), sub_talker=SamplingOptions.greedy()))
    spare = GenerationOptions(seed=999, repetition_penalty=1.1, max_new_tokens=64)
    n = len(jobs)
    state = DeviceBatchState(device, n, max_history=2048 + 64)
    host = []
    for s, job in enumerate(jobs):
        hist = rng.integers(0, 2048, 40 if s == 3 else 0).tolist()
        state.start(s, job, hist)
        host.append(HostJob(job, hist))
    refilled = False
    for frame in range(10):
        lg = (rng.normal(0, 4, (n, 3072))).astype(np.float32)
        lg[0, 2150] = 60.0                      # EOS boosted for slot 0: suppressed at steps 0 and 1, then taken
        ids, done = state.talker_step(torch.from_numpy(lg).cuda())
        ids, done = ids.cpu().numpy(), done.cpu().numpy()
        for s, job in enumerate(host):
            if job.done:
                assert ids[s] == -1 and done[s] == 0, (frame, s)
                continue
            want = _talker_ref(job, lg[s])
            assert ids[s] == want, (frame, s, int(ids[s]), want)
            job.history.append(want)
            finished = want == 2150 or job.step == job.opts.max_new_tokens - 1
            assert bool(done[s]) == finished, (frame, s)
            job.done = finished
        for g in range(1, 16):
            cl = rng.normal(0, 3, (n, 2048)).astype(np.float32)
            sub = state.sub_step(torch.from_numpy(cl).cuda()).cpu().numpy()
            for s, job in enumerate(host):
                assert sub[s] == (-1 if job.done else _sub_ref(job, cl[s])), (frame, g, s)
        for s, job in enumerate(host):
            if not job.done:
                job.step += 1
            st, hl, act = state.query(s)
            assert (st, hl, act) == (job.step, len(job.history), not job.done), (frame, s)
        if not refilled and host[0].done:        # continuous batching: a finished slot takes the next job
            state.start(0, spare)
            host[0] = HostJob(spare)
            refilled = True
    assert refilled and host[1].done and len(host[1].history) == 5
    state.close()
