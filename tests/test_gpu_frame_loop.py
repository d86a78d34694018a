"""The device frame loop (vw_batch_*_head_step, vw_batch_code_embedding, vw_batch_frame_embedding) against the
reference's GenerateBatch frame (TalkerGenerator.cs:362-439) run on the host with the CPU oracle.

Even frames gather the next code-predictor inputs inside the head steps (vw_embed_out), odd frames with separate
vw_batch_code_embedding calls.  The caller's transformer steps are replaced by a fixed stand-in (next hidden rows = bf16 of the previous step's
input rows), applied identically on both sides.  Per frame the host side: samples codebook 0 of every running job
(oracle, the job's Random(Seed) draws) from CodecHead's logits, appends it, retires on EOS / MaxNewTokens; for the
survivors gathers CodecEmbedding(code0), then for g = 1..15 samples from CodePredictorHead(g)'s logits (Random(Seed + 1)
draws) and gathers CodePredictorEmbedding(g, code); finally FrameEmbedding(frame) + text.  The logits on both sides
are the tcgen05 GEMM's (vw_head_logits on the same rows; the GEMM itself is checked against float64 elsewhere), so
ids, codes, done flags and every gathered row must match exactly.
"""

import numpy as np
import pytest

from oracle import oracle
from oracle.embedding import frame_embedding as ref_frame_embedding
from tests.test_gpu_batch import HostJob
from voxwerk_b200.workloads import SegData

pytestmark = pytest.mark.gpu

H, V, CV, G = 256, 3072, 2048, 16


def _bf16_bits(rng, shape, scale):
    return (rng.normal(0, scale, shape).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _widen(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _talker_ref(job, row):
    o = job.opts
    u = job.rng.next_double() if o.talker.do_sample else 0.0
    seg = SegData(row[None, :], 0, 0, V, np.array([u]), None, np.array([0, len(job.history)], np.int64),
                  np.array(job.history or [0], np.int32), np.array([job.step], np.int32), V - 1024, V, 2150, 2)
    return int(oracle.sample_segment(seg, [(int(o.talker.do_sample), o.talker.top_k, o.talker.top_p,
                                            o.talker.temperature, o.repetition_penalty)])[0])


def _sub_ref(job, row):
    o = job.opts.sub_talker
    u = job.sub_rng.next_double() if o.do_sample else 0.0
    return int(oracle.select(row, (int(o.do_sample), o.top_k, o.top_p, o.temperature, 1.0), u))


def test_device_frame_loop_matches_generate_batch(device):
    import torch
    from voxwerk_b200 import DeviceBatchState, GenerationOptions, SamplingOptions, head_logits
    rng = np.random.default_rng(77)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    codec_head = t(_bf16_bits(rng, (V, H), 0.125).view(np.int16))
    cp_heads = [t(_bf16_bits(rng, (CV, H), 0.125).view(np.int16)) for _ in range(G - 1)]
    codec_emb_bits = _bf16_bits(rng, (V, H), 1.0)
    cp_emb_bits = [_bf16_bits(rng, (CV, H), 1.0) for _ in range(G - 1)]
    codec_emb = t(codec_emb_bits.view(np.int16))
    cp_emb = [t(b.view(np.int16)) for b in cp_emb_bits]

    jobs = [GenerationOptions(seed=300 + j, max_new_tokens=4 if j == 1 else 64,
                              repetition_penalty=1.3 if j % 2 else 1.05,
                              talker=SamplingOptions(top_p=0.8 if j % 3 else 1.0),
                              sub_talker=SamplingOptions(top_k=20 if j == 2 else 50)) for j in range(5)]
    jobs.append(GenerationOptions(seed=9, talker=SamplingOptions.greedy(), sub_talker=SamplingOptions.greedy()))
    spare = GenerationOptions(seed=4242, repetition_penalty=1.1, max_new_tokens=64)
    n = len(jobs)
    state = DeviceBatchState(device, n, max_history=2048 + 64)
    host = []
    for s, job in enumerate(jobs):
        hist = rng.integers(0, 2048, 30 if s == 3 else 0).tolist()
        state.start(s, job, hist)
        host.append(HostJob(job, hist))

    last = torch.from_numpy(rng.normal(0, 1, (n, H)).astype(np.float32)).cuda()   # the talker's hidden rows
    cp_in = torch.zeros((n, H), dtype=torch.float32, device="cuda")                 # code-predictor input rows
    step_in = torch.zeros((n, H), dtype=torch.float32, device="cuda")               # next talker input rows
    ref_cp_in = np.zeros((n, H), np.float32)
    ref_step_in = np.zeros((n, H), np.float32)
    refilled = False
    for frame in range(7):
        hidden = last.to(torch.bfloat16)
        logits = torch.empty((n, V), dtype=torch.float32, device="cuda")
        head_logits(device, hidden, codec_head, logits)
        lg = logits.cpu().numpy()
        fused = frame % 2 == 0   # even frames: the gathers ride along with the head steps
        ids, done = state.talker_head_step(hidden, codec_head, *((codec_emb, cp_in) if fused else ()))
        ids, done = ids.cpu().numpy(), done.cpu().numpy()
        going = []
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
            if not finished:
                going.append(s)
        frame_codes = np.full((n, G), -1, np.int32)
        for s in going:
            frame_codes[s, 0] = ids[s]
        np.testing.assert_array_equal(state.codes()[:, 0], frame_codes[:, 0])

        if not fused:
            state.code_embedding(0, codec_emb, cp_in)                 # CodecEmbedding(code0), :411
        for s in going:
            ref_cp_in[s] = _widen(codec_emb_bits[frame_codes[s, 0]])
        for g in range(1, G):
            got_in = cp_in.cpu().numpy()
            np.testing.assert_array_equal(got_in[going].view(np.uint32), ref_cp_in[going].view(np.uint32))
            cp_hidden = cp_in.to(torch.bfloat16)                      # the code predictor's step (stand-in)
            cl = torch.empty((n, CV), dtype=torch.float32, device="cuda")
            head_logits(device, cp_hidden, cp_heads[g - 1], cl)
            cl = cl.cpu().numpy()
            sub = state.sub_head_step(g, cp_hidden, cp_heads[g - 1],
                                      *((cp_emb[g - 1], cp_in) if fused else ())).cpu().numpy()
            for s, job in enumerate(host):
                want = _sub_ref(job, cl[s]) if s in going else -1
                assert sub[s] == want, (frame, g, s, int(sub[s]), want)
                if s in going:
                    frame_codes[s, g] = want
            if not fused:
                state.code_embedding(g, cp_emb[g - 1], cp_in)         # CodePredictorEmbedding(g, code), :422
            for s in going:
                ref_cp_in[s] = _widen(cp_emb_bits[g - 1][frame_codes[s, g]])
        codes = state.codes()
        np.testing.assert_array_equal(codes[going], frame_codes[going])
        assert (codes[[s for s in range(n) if s not in going], 0] == -1).all()

        text = rng.normal(0, 1, (n, H)).astype(np.float32)
        state.frame_embedding(codec_emb, cp_emb, t(text), step_in)    # FrameEmbedding + text, :428-439
        if going:
            ref_step_in[going] = ref_frame_embedding(frame_codes[going], codec_emb_bits, cp_emb_bits, text[going])
        got_step = step_in.cpu().numpy()
        np.testing.assert_array_equal(got_step[going].view(np.uint32), ref_step_in[going].view(np.uint32))
        for s in going:
            host[s].step += 1
        for s, job in enumerate(host):
            st, hl, act = state.query(s)
            assert (st, hl, act) == (job.step, len(job.history), not job.done), (frame, s)
        last = step_in.clone()                                        # the talker's step (stand-in)
        if not refilled and host[1].done:                             # a finished slot takes the next job
            state.start(1, spare)
            host[1] = HostJob(spare)
            refilled = True
    assert refilled
    state.close()


def test_code_embedding_rejects_out_of_range(device):
    import torch
    from voxwerk_b200 import DeviceBatchState, GenerationOptions, SamplingOptions, VwInvalidArgument, VwOutOfRange
    rng = np.random.default_rng(5)
    state = DeviceBatchState(device, 2, max_history=256)
    state.start(0, GenerationOptions(seed=1, max_new_tokens=8, talker=SamplingOptions.greedy()))
    hidden = torch.from_numpy(rng.normal(0, 1, (2, H)).astype(np.float32)).cuda().to(torch.bfloat16)
    head = torch.from_numpy(_bf16_bits(rng, (V, H), 0.125).view(np.int16)).cuda()
    state.talker_head_step(hidden, head)
    small = torch.from_numpy(_bf16_bits(rng, (4, H), 1.0).view(np.int16)).cuda()   # 4 rows: code0 is out of range
    out = torch.zeros((2, H), dtype=torch.float32, device="cuda")
    code0 = int(state.codes()[0, 0])
    assert code0 >= 4
    with pytest.raises(VwOutOfRange):
        state.code_embedding(0, small, out)
    with pytest.raises(VwInvalidArgument):
        state.sub_head_step(16, hidden, head[:CV])                   # groups are 1..15
    full = torch.from_numpy(_bf16_bits(rng, (V, H), 1.0).view(np.int16)).cuda()
    state.code_embedding(0, full, out)                               # the batch is usable afterwards
    want = _widen(full.cpu().numpy().view(np.uint16)[code0])
    np.testing.assert_array_equal(out.cpu().numpy()[0].view(np.uint32), want.view(np.uint32))
    state.close()


def test_batch_outlives_its_handle():
    """vw_destroy releases the device memory of the batches still alive on the handle; the batch object can then
    only be destroyed (every other call is refused), and destroying it is safe."""
    import torch
    from voxwerk_b200 import Device, DeviceBatchState, GenerationOptions, VwInvalidArgument
    d = Device(0)
    state = DeviceBatchState(d, 2, max_history=64)
    state.start(0, GenerationOptions(seed=1, max_new_tokens=8))
    logits = torch.zeros((2, V), dtype=torch.float32, device="cuda")
    state.talker_step(logits)
    d.close()
    with pytest.raises((RuntimeError, VwInvalidArgument)):
        state.talker_step(logits)
    state.close()
