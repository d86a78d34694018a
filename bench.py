"""Benchmark of the fused sampler on the headline configuration (config 2: a batched talker step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

One step = one vw_sample call over one batch of 4096 talker rows (V = 3072 fp32 logits, 1024-id histories,
T 0.9, top-k 50, top-p 0.8, repetition penalty 1.05, suppress mask).  Under torchrun each rank samples its own
4096-row batch (rows are independent; weak scaling; no collective on the data path -- NCCL only carries the
barrier and the max-over-ranks of the timings).  At N > 1 the line also carries `strong` (the one 4096-row batch
of config 2 split into N row shards) and `cfg3_sharded` (config 3's heterogeneous frame split by cost).

value: rows/s of the whole job with inputs resident in HBM (3 rotating input copies, larger than the 126 MB L2, so
no step reads another step's data from L2); K steps captured in one CUDA graph and timed with CUDA events on the
launching stream.  e2e: the same metric through the public C-ABI call with host buffers (pinned host -> device
copies of logits, histories and uniforms, and the ids back) inside the timed region.  cpu_baseline: the CPU
restatement of voxwerk's Sampler (oracle/, "port": the C# reference cannot run here) on a bounded sample.
`e2e_resident`: the same step through the device-resident batch API (vw_batch_*), where histories and samplers
stay on the GPU and a step copies in only the logit columns the sampler reads.
`parity`: every row of the timed batch against that restatement, with flips counted and attributed.
At N = 1 `configs` holds the other four configurations (µs per call, rows/s, roofline fraction, parity), and
`frame_embedding` the next-input gather (vw_frame_embedding) for 1024 sequences, and `head` the vocabulary head
(vw_head_logits, the tcgen05 GEMM; vw_head_sample, GEMM + sampler) against cuBLAS (+ vw_sample), with
`head.frame_loop` one whole device frame of the batch loop (every sampling step of a frame for 1024 sequences).
`--impl reference` times only the CPU implementation, with every host thread, and prints its own line; that
process loads no GPU library of this repository.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/s & HBM GB/s (B=4096,V=3072 talker step) at 1/2/4/8 B200"
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "traffic.json")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
N_COPIES = 3
LAUNCHES_PER_CALL = 2   # the warp-per-row kernel and the whole-row kernel


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def hbm_peak():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def workload_keys(w) -> dict:
    """The workload's shape and decoding settings for the JSON line's `config`."""
    seg = w.segments[0]
    hist = int(np.max(np.diff(seg.hist_offsets))) if seg.hist_offsets is not None else 0
    opts = [dict(zip(("do_sample", "top_k", "top_p", "temperature", "repetition_penalty"), o)) for o in w.options]
    return {"vocab": [s.vocab for s in w.segments], "history": hist, "options": opts}


def bench_config(w, world: int) -> dict:
    """`config` of the JSON line; both arms print the same dict for the same workload and N."""
    alg = w.algorithmic_bytes()
    return {"workload": w.name, "rows_per_gpu": w.n_rows, "global_rows": w.n_rows * world, **workload_keys(w),
            "parallelism": f"row shards x{world}, no collective",
            "l2": f"{N_COPIES} rotating input copies ({N_COPIES * alg / 1e6:.0f} MB > 126 MB L2)",
            "timing": "K steps in one CUDA graph, CUDA events on the launching stream, max over ranks"}


def cpu_reference(workload, seconds: float, threads: int):
    """Times the CPU restatement (oracle port) on repeated passes over the workload's rows."""
    from oracle import oracle
    t0 = time.perf_counter()
    rows = 0
    while True:
        for seg in workload.segments:
            oracle.sample_segment(seg, workload.options, threads=threads)
            rows += seg.n_rows
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return rows / el, rows, el


def run_reference_arm(args):
    """The reference's own CPU implementation of the path: voxwerk is C# and cannot run here, so the CPU
    restatement (oracle/) stands in for it.  Rank 0 alone works under torchrun; the other ranks exit at once."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    from voxwerk_b200 import workloads   # pure Python: maps no library of this repository
    w = workloads.make(args.config)
    threads = host_threads()
    per_step = []
    for i in range(args.warmup + args.steps):
        _, _, el = cpu_reference(w, 0.0, threads)
        if i >= args.warmup:
            per_step.append(el)
    t = float(np.sum(per_step))
    value = args.steps * w.n_rows / t
    sample = f"{w.n_rows} rows of {w.name} per step (one rank's batch), {threads} threads (std::thread over rows)"
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(w, world),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port", "sample": sample,
                         "what": "C++ restatement of voxwerk Sampler.cs (oracle/vw_oracle.cpp); the C# reference "
                                 "cannot be built or run in this environment"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------- GPU arm helpers
def device_copies(w, torch, n_copies=N_COPIES):
    """n_copies distinct device copies of the workload: (segments, arrays) per copy."""
    from tests.gpu_util import make_segment, to_device
    copies = []
    for c in range(n_copies):
        segs, keep = [], []
        for s in w.segments:
            arr = to_device(s, torch)
            keep.append(arr)
            hist_max = int(np.max(np.diff(s.hist_offsets))) if s.hist_offsets is not None else 0
            segs.append(make_segment(s, arr, max_hist_len=hist_max))
        copies.append((segs, keep))
    return copies


def timed_graph(dev, copies, opts, steps, warmup, stream, torch, barrier=None, clocks_gpu=None):
    """Warm-up, then `steps` calls (rotating copies) captured in one CUDA graph and timed with CUDA events on the
    launching stream.  Returns (ms, clocks summary or None, path counters)."""
    from voxwerk_b200 import sample_rows
    sp = stream.cuda_stream
    with torch.cuda.stream(stream):
        for i in range(max(warmup, 3)):
            sample_rows(dev, copies[i % len(copies)][0], opts, stream=sp)
    dev.synchronize(sp)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            sample_rows(dev, copies[i % len(copies)][0], opts, stream=torch.cuda.current_stream().cuda_stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cs = ClockSampler(clocks_gpu) if clocks_gpu is not None else None
    if cs is not None:
        cs.__enter__()   # nvidia-smi samples from here on (its start-up pause comes before the warm replays)
    try:
        # untimed replays for at least 50 ms (two at least), right before the timed one, so the SM clock has left
        # its idle level
        t_end = time.perf_counter() + 0.05
        n_warm = 0
        while n_warm < 2 or time.perf_counter() < t_end:
            graph.replay()
            torch.cuda.synchronize()
            n_warm += 1
        dev.stats(reset=True)
        if barrier:
            barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    finally:
        if cs is not None:
            cs.__exit__(None, None, None)
    clocks = cs.summary() if cs is not None else None
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    dev.synchronize(sp)   # raises if the kernel latched an error
    paths = dev.stats(reset=True)
    del graph
    return ms, clocks, paths


def gpu_ids(dev, w, torch, stream):
    """One device call over the whole workload; ids per segment (numpy)."""
    from tests.gpu_util import make_segment, options_table, to_device
    from voxwerk_b200 import sample_rows
    arrs = [to_device(s, torch) for s in w.segments]
    sample_rows(dev, [make_segment(s, a) for s, a in zip(w.segments, arrs)], options_table(w),
                stream=stream.cuda_stream)
    dev.synchronize(stream.cuda_stream)
    return [a["out_ids"].cpu().numpy() for a in arrs]


def parity_summary(w, ids) -> dict:
    from tests.parity import compare
    c = compare(w, ids, threads=host_threads())
    c.pop("first_flips", None)
    return c


def roofline(w, ms_per_step, peak, peak_kind):
    alg = w.algorithmic_bytes()
    achieved = alg / (ms_per_step * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_kind": peak_kind, "algorithmic_bytes_per_launch": alg}


def e2e_resident(dev, w, steps, torch, barrier, rank):
    """The talker step through the device-resident batch API (vw_batch_*): each slot keeps its history and its
    sampler on the device, so a step copies in only the logit columns the sampler reads (pinned host -> device, one
    2D copy) and copies the ids back.  Rows/s counts the slots sampled (every slot runs for the whole test)."""
    from cuda.bindings import runtime as cudart
    from voxwerk_b200 import DeviceBatchState, GenerationOptions, SamplingOptions
    seg = w.segments[0]
    n, V = seg.n_rows, seg.vocab
    o = w.options[0]
    hist = seg.hist_offsets
    state = DeviceBatchState(dev, n, max_history=int(np.max(np.diff(hist))) + steps + 16, vocab=V)
    for r in range(n):
        job = GenerationOptions(seed=1000 * rank + r, max_new_tokens=steps + 8, repetition_penalty=o[4],
                                talker=SamplingOptions(bool(o[0]), int(o[1]), float(o[2]), float(o[3])))
        state.start(r, job, seg.hist_ids[hist[r]:hist[r + 1]].tolist())
    lg = np.ascontiguousarray(seg.logits).copy()
    lg[:, seg.eos_id] = -np.inf                  # keep every slot running for the whole measurement
    cols = (seg.eos_id // 4 + 1) * 4             # the sampler reads [0, 2048) and the EOS vector: columns [0, 2152)
    host = torch.from_numpy(np.ascontiguousarray(lg[:, :cols])).pin_memory()
    dlog = torch.empty((n, V), dtype=torch.float32, device="cuda")
    ids_host = torch.empty(n, dtype=torch.int32).pin_memory()
    st = torch.cuda.Stream()

    def step():
        cudart.cudaMemcpy2DAsync(dlog.data_ptr(), V * 4, host.data_ptr(), cols * 4, cols * 4, n,
                                 cudart.cudaMemcpyKind.cudaMemcpyHostToDevice, st.cuda_stream)
        ids, _ = state.talker_step(dlog, stream=st.cuda_stream)
        with torch.cuda.stream(st):
            ids_host.copy_(ids, non_blocking=True)
        st.synchronize()

    for _ in range(2):
        step()
    if barrier:
        barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    el = time.perf_counter() - t0
    sampled = int((ids_host.numpy() >= 0).sum())
    state.close()
    return el, sampled, n * cols * 4, n * 4


def graph_us(torch, st, fn, reps):
    """µs per call of fn(stream handle): `reps` calls captured in one CUDA graph (no host overhead in the timed
    region), replayed untimed for at least 50 ms (so the SM clock has left its idle level), then the median of three
    timed replays (CUDA events on the launching stream)."""
    with torch.cuda.stream(st):
        for _ in range(3):
            fn(st.cuda_stream)
    st.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for _ in range(reps):
            fn(torch.cuda.current_stream().cuda_stream)
    t_end = time.perf_counter() + 0.05
    while time.perf_counter() < t_end:
        graph.replay()
        st.synchronize()
    times = []
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record(st)
            graph.replay()
            e1.record(st)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    del graph
    return 1e3 * float(np.median(times)) / reps


def frame_embedding_timing(dev, torch, peak, peak_kind, rows=1024, reps=50):
    """vw_frame_embedding on `rows` sequences (config 3's stream count): Qwen3-TTS sizes (hidden 1024, 3072 + 15 x
    2048 embedding rows), random codes and tables, `reps` calls in a CUDA graph (graph_us)."""
    from voxwerk_b200 import frame_embedding
    H, G = 1024, 16
    g = torch.Generator(device="cuda").manual_seed(5)
    codec = torch.randint(-20000, 20000, (3072, H), dtype=torch.int16, device="cuda", generator=g)
    cps = [torch.randint(-20000, 20000, (2048, H), dtype=torch.int16, device="cuda", generator=g) for _ in range(G - 1)]
    codes = torch.cat([torch.randint(0, 3072, (rows, 1), device="cuda", generator=g),
                       torch.randint(0, 2048, (rows, G - 1), device="cuda", generator=g)], 1).to(torch.int32)
    text = torch.randn((rows, H), device="cuda", generator=g)
    out = torch.empty((rows, H), device="cuda")
    st = torch.cuda.Stream()
    us = graph_us(torch, st, lambda sp: frame_embedding(dev, codes, codec, cps, text, out, stream=sp), reps)
    dev.synchronize(st.cuda_stream)
    alg = rows * (G * H * 2 + 2 * H * 4)   # the gathered bf16 rows, the text row in, the fp32 row out
    achieved = alg / (us * 1e-6) / 1e9
    return {"rows": rows, "hidden": H, "groups": G, "us_per_call": us,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "algorithmic_bytes_per_launch": alg}}


def tensor_peak():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def head_timing(dev, torch, hbm, hbm_kind, reps=50, cases=((64, 3072), (1024, 3072), (4096, 3072), (1024, 2048))):
    """The vocabulary head (hidden 1024) ahead of the sampler: vw_head_logits (tcgen05 GEMM) against cuBLAS
    (torch.mm, bf16 in, fp32 out), and vw_head_sample (GEMM + sampler in one call) against cuBLAS followed by
    vw_sample on its logits.  Talker rows (V 3072) carry config 2's histories and options; sub rows (V 2048) config
    1's options.  CUDA events over `reps` calls on one stream; the weight (6 MB) stays in L2 between calls, as it
    does between a model's steps."""
    from tests.gpu_util import make_segment, options_table, to_device
    from voxwerk_b200 import head_logits, head_sample, sample_rows
    from voxwerk_b200 import workloads
    tflops, t_kind = tensor_peak()
    H = 1024
    st = torch.cuda.Stream()
    out = {}
    for rows, V in cases:
        w = workloads.make(2, rows) if V == 3072 else workloads.make(1)
        sd = w.segments[0]
        if sd.n_rows != rows:   # sub rows: config 1's options over `rows` rows with fresh draws
            sd = workloads.SegData(np.zeros((rows, V), np.float32), workloads.F32, workloads.SUB, V,
                                   np.random.default_rng(7).random(rows), np.zeros(rows, np.int32))
        opts = options_table(w)
        g = torch.Generator(device="cuda").manual_seed(rows + V)
        hidden = torch.randn((rows, H), device="cuda", generator=g).to(torch.bfloat16)
        weight = (torch.randn((V, H), device="cuda", generator=g) * 0.125).to(torch.bfloat16)
        logits = torch.empty((rows, V), dtype=torch.float32, device="cuda")
        arr = to_device(sd, torch)
        arr["logits"] = None
        seg_head = make_segment(sd, arr)
        arr2 = dict(arr)
        arr2["logits"] = logits
        seg_lib = make_segment(sd, arr2)

        def cublas(sp):
            torch.mm(hidden, weight.t(), out_dtype=torch.float32, out=logits)

        def lib_then_sample(sp):
            cublas(sp)
            sample_rows(dev, [seg_lib], opts, stream=sp)

        def timed(fn):
            return graph_us(torch, st, fn, reps)

        def try_timed(fn):
            try:
                return timed(fn)
            except Exception as e:   # torch without mm(out_dtype=...): no cuBLAS fp32-output baseline
                return f"unavailable: {type(e).__name__}: {str(e)[:120]}"

        t_ours = timed(lambda sp: head_logits(dev, hidden, weight, logits, stream=sp))
        t_fused = timed(lambda sp: head_sample(dev, hidden, weight, seg_head, opts, stream=sp))
        t_lib = try_timed(cublas)
        t_lib_sample = try_timed(lib_then_sample)
        head_logits(dev, hidden, weight, logits, stream=st.cuda_stream)
        dev.synchronize(st.cuda_stream)
        dev.stats(reset=True)
        t_sample = timed(lambda sp: sample_rows(dev, [seg_lib], opts, stream=sp))
        dev.synchronize(st.cuda_stream)
        paths = dev.stats(reset=True)
        s = st.cuda_stream
        dev.synchronize(s)
        flops = 2.0 * rows * V * H
        alg = V * H * 2 + rows * H * 2 + rows * V * 4
        t_flop, t_byte = flops / (tflops * 1e12), alg / (hbm * 1e9)
        bound = "tensor" if t_flop >= t_byte else "hbm"
        floor_us = 1e6 * max(t_flop, t_byte)
        out[f"{rows}x{V}x{H}"] = {
            "us_head_logits": t_ours, "us_cublas_mm": t_lib, "us_head_sample": t_fused,
            "us_cublas_then_vw_sample": t_lib_sample, "us_vw_sample_on_head_logits": t_sample,
            "sampler_rows_by_path": paths,
            "roofline": {"bound": bound, "floor_us": floor_us, "frac": floor_us / t_ours,
                         "achieved_tflops": flops / (t_ours * 1e-6) / 1e12, "tflops_peak": tflops,
                         "tflops_peak_kind": t_kind, "achieved_gbs": alg / (t_ours * 1e-6) / 1e9, "hbm_peak": hbm,
                         "hbm_peak_kind": hbm_kind, "algorithmic_bytes": alg, "flops": flops}}
    return out


def frame_loop_timing(dev, torch, streams=1024, reps=10):
    """One frame of the device loop for `streams` sequences (config 3's stream count; hidden 1024, Qwen3-TTS
    vocabularies): vw_batch_talker_head_step, 15 x vw_batch_sub_head_step (each with its next-input gather),
    vw_batch_frame_embedding -- everything of TalkerGenerator.cs:362-439 except the transformer steps, whose hidden
    rows are fixed random inputs here.  Talker options as config 3 (top-k 50, top-p 0.8, rp 1.05, 1024-id
    histories), sub-talker top-k 50; `reps` frames in one CUDA graph (graph_us)."""
    from voxwerk_b200 import DeviceBatchState, GenerationOptions, SamplingOptions
    H, V, CV, G = 1024, 3072, 2048, 16
    g = torch.Generator(device="cuda").manual_seed(11)
    bf = lambda *shape, s=1.0: (torch.randn(shape, device="cuda", generator=g) * s).to(torch.bfloat16)
    codec_head, cp_heads = bf(V, H, s=0.125), [bf(CV, H, s=0.125) for _ in range(G - 1)]
    codec_head[2150].zero_()   # EOS logit 0, far below the top-50 cut: no sequence retires while timing
    codec_emb, cp_emb = bf(V, H), [bf(CV, H) for _ in range(G - 1)]
    last, cp_hidden = bf(streams, H), bf(streams, H)
    text = torch.randn((streams, H), device="cuda", generator=g)
    cp_in = torch.empty((streams, H), device="cuda")
    step_in = torch.empty((streams, H), device="cuda")
    # 1024-id starting histories (config 3); jobs long enough that no slot reaches MaxNewTokens while timing
    state = DeviceBatchState(dev, streams, max_history=1024 + 50000)
    job = GenerationOptions(seed=42, max_new_tokens=50000, repetition_penalty=1.05,
                            talker=SamplingOptions(top_k=50, top_p=0.8), sub_talker=SamplingOptions(top_k=50))
    hist = np.random.default_rng(3).integers(0, 2048, (streams, 1024))
    for s in range(streams):
        state.start(s, job, hist[s].tolist())

    def frame(sp):   # the next-input gathers ride along with the head steps
        state.talker_head_step(last, codec_head, codec_emb, cp_in, stream=sp)
        for grp in range(1, G):
            state.sub_head_step(grp, cp_hidden, cp_heads[grp - 1], cp_emb[grp - 1], cp_in, stream=sp)
        state.frame_embedding(codec_emb, cp_emb, text, step_in, stream=sp)

    st = torch.cuda.Stream()
    us = graph_us(torch, st, frame, reps)
    dev.synchronize(st.cuda_stream)
    steps = state.query(0)[0]
    state.close()
    # kernels per frame: talker (GEMM, draw, 2 sampler, commit + gather) + 15 x (GEMM, draw, 2 sampler,
    # record + gather) + frame embedding
    return {"streams": streams, "hidden": H, "us_per_frame": us, "frames_per_s": 1e6 / us,
            "sampled_rows_per_s": streams * G / (us * 1e-6), "kernels_per_frame": 5 + 15 * 5 + 1,
            "slot0_steps_after_timing": steps, "note": "talker EOS logit held at 0 (no slot retires while timing)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the other configurations and the shard keys")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    barrier = dist.barrier if world > 1 else None

    from tests.gpu_util import make_segment, options_table
    from voxwerk_b200 import Device, sample_rows, workloads
    from voxwerk_b200.shard import max_over_ranks, sum_over_ranks

    dev = Device(local)
    stream = torch.cuda.Stream()
    peak, peak_kind = hbm_peak()
    w = workloads.make(args.config)
    if rank > 0:   # weak scaling: each rank its own batch of the same shape
        import copy
        rng = np.random.default_rng(7919 * rank)
        w = copy.deepcopy(w)
        for s in w.segments:
            perm = rng.permutation(s.n_rows)
            s.logits = np.ascontiguousarray(s.logits[perm])
    opts = options_table(w)

    # ---- parity: every row of this rank's batch against the CPU restatement, flips counted and attributed
    par = parity_summary(w, gpu_ids(dev, w, torch, stream))
    flips_all = int(sum_over_ranks(par["flips"], device="cuda"))
    rows_all = int(sum_over_ranks(par["rows"], device="cuda"))

    # ---- headline: K steps of this rank's batch in one CUDA graph
    copies = device_copies(w, torch)
    elapsed_ms, clocks, paths = timed_graph(dev, copies, opts, args.steps, args.warmup, stream, torch, barrier,
                                            clocks_gpu=local)
    elapsed_max = max_over_ranks(elapsed_ms, device="cuda")
    value = w.n_rows * world * args.steps / (elapsed_max * 1e-3)
    ms_per_step = elapsed_max / args.steps
    del copies

    # ---- e2e through the public API with host buffers (pinned), copies inside the timed region
    host_arrays = []
    for s in w.segments:
        pin = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        lg = s.logits.view(np.int16) if s.logits.dtype == np.uint16 else s.logits
        arr = dict(logits=pin(lg), uniforms=pin(s.uniforms), opt_index=pin(s.opt_index),
                   hist_offsets=pin(s.hist_offsets), hist_ids=pin(s.hist_ids), steps=pin(s.steps),
                   out_ids=torch.full((s.n_rows,), -1, dtype=torch.int32).pin_memory())
        host_arrays.append((s, arr))
    hsegs = [make_segment(s, arr) for s, arr in host_arrays]
    d2h = sum(int(arr["out_ids"].numel() * 4) for _, arr in host_arrays)
    for _ in range(2):
        sample_rows(dev, hsegs, opts)
    dev.stats(reset=True)
    if barrier:
        barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        sample_rows(dev, hsegs, opts)
    e2e_s = time.perf_counter() - t0
    # bytes the library copied host -> device per step (it skips the logit columns no kernel reads)
    h2d = dev.stats(reset=True)["h2d_bytes"] // max(args.e2e_steps, 1)
    e2e_value = w.n_rows * world * args.e2e_steps / max_over_ranks(e2e_s, device="cuda")
    del host_arrays, hsegs

    # ---- e2e through the device-resident batch API (histories and samplers stay on the GPU)
    resident = None
    if len(w.segments) == 1 and w.segments[0].kind == 0:
        el, sampled, h2d_r, d2h_r = e2e_resident(dev, w, args.e2e_steps, torch, barrier, rank)
        el_max = max_over_ranks(el, device="cuda")
        sampled_all = int(sum_over_ranks(sampled, device="cuda"))
        resident = {"value": sampled_all * args.e2e_steps / el_max, "unit": "rows/s", "h2d_bytes_per_step": h2d_r,
                    "d2h_bytes_per_step": d2h_r, "steps": args.e2e_steps,
                    "path": "vw_batch_talker_step: logits columns [0, 2152) copied from pinned host memory each step "
                            "(one 2D copy), ids copied back; histories, steps and samplers stay on the device"}

    # ---- N > 1: config 2's one batch split over the ranks (strong scaling), and config 3 sharded by cost
    strong = cfg3 = None
    if world > 1 and not args.no_extra:
        for name in ("strong", "cfg3_sharded"):
            full = workloads.make(args.config if name == "strong" else 3)
            part = full.shard(rank, world)
            pp = parity_summary(part, gpu_ids(dev, part, torch, stream))
            cps = device_copies(part, torch)
            ms, _, _ = timed_graph(dev, cps, options_table(part), args.steps, args.warmup, stream, torch, barrier)
            del cps
            t_max = max_over_ranks(ms, device="cuda") / args.steps
            t_min = -max_over_ranks(-ms, device="cuda") / args.steps
            entry = {"workload": full.name, "global_rows": full.n_rows, "rows_per_gpu_max":
                     int(max_over_ranks(part.n_rows, device="cuda")),
                     "value": full.n_rows / (t_max * 1e-3), "unit": "rows/s", "ms_per_step": t_max,
                     "ms_per_step_fastest_rank": t_min, "scaling": "strong",
                     "roofline": roofline(full, t_max, peak, peak_kind),
                     "parity": {"rows": int(sum_over_ranks(pp["rows"], device="cuda")),
                                "flips": int(sum_over_ranks(pp["flips"], device="cuda"))}}
            if name == "strong":
                strong = entry
            else:
                cfg3 = entry

    # ---- N = 1: the other four configurations
    configs = None
    if world == 1 and not args.no_extra:
        configs = {}
        for cfg in (0, 1, 3, 4):
            if cfg == args.config:
                continue
            wc = workloads.make(cfg)
            pc = parity_summary(wc, gpu_ids(dev, wc, torch, stream))
            cps = device_copies(wc, torch)
            k = max(20, min(args.steps, 100))
            ms, ck, pth = timed_graph(dev, cps, options_table(wc), k, args.warmup, stream, torch, clocks_gpu=local)
            del cps
            per = ms / k
            configs[wc.name] = {"us_per_call": 1e3 * per, "rows_per_s": wc.n_rows / (per * 1e-3), "steps": k,
                                "roofline": roofline(wc, per, peak, peak_kind), "parity": pc, "clocks": ck,
                                "rows_by_path": pth}

    gather = frame_embedding_timing(dev, torch, peak, peak_kind) if world == 1 and not args.no_extra else None
    head = None
    if world == 1 and not args.no_extra:
        with ClockSampler(local) as cs:
            head = head_timing(dev, torch, peak, peak_kind)
        head["clocks"] = cs.summary()
        head["frame_loop"] = frame_loop_timing(dev, torch)

    line = None
    if rank == 0:
        need = w.needed_bytes()
        traffic = None
        if os.path.exists(TRAFFIC_PATH):
            try:
                traffic = json.load(open(TRAFFIC_PATH)).get(w.name)
            except Exception:
                traffic = None
        cpu = None
        if world == 1 and not args.no_cpu:
            thr = host_threads()
            v_all, rows_all_cpu, el_all = cpu_reference(w, args.cpu_seconds, thr)
            v_one, _, _ = cpu_reference(w.shard(0, 16), min(3.0, args.cpu_seconds), 1)
            cpu = {"value": v_all, "unit": "rows/s", "cores": thr, "kind": "port",
                   "sample": f"{rows_all_cpu} rows ({rows_all_cpu // w.n_rows} passes over {w.name}) in "
                             f"{el_all:.1f} s on {thr} threads; 1 thread: {v_one:.0f} rows/s",
                   "what": "C++ restatement of voxwerk Sampler.cs (oracle/), the C# reference cannot run here"}
        rl = roofline(w, ms_per_step, peak, peak_kind)
        rl.update({"traffic": traffic,
                   "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one full-size "
                                     "warp-per-row kernel launch, read from profiles/traffic.json (not measured in "
                                     "this run)",
                   "needed_bytes_per_launch": need,
                   "frac_of_needed_bytes": need / (ms_per_step * 1e-3) / 1e9 / peak,
                   "kernel": "row_warp_kernel (the step: warp-per-row kernel + whole-row kernel launch, CUDA events)"})
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": bench_config(w, world),
            "roofline": rl,
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": args.e2e_steps,
                    "path": "vw_sample(VW_MEM_HOST) from pinned host buffers: logits (without the suppressed "
                            "span's columns), histories, steps, options, uniforms in; ids out"},
            "e2e_resident": resident,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": LAUNCHES_PER_CALL * args.steps,
            "parity": {"rows": rows_all, "flips": flips_all, "rank0": par},
            "rows_by_path": paths,
        }
        if strong is not None:
            line["strong"] = strong
        if cfg3 is not None:
            line["cfg3_sharded"] = cfg3
        if configs is not None:
            line["configs"] = configs
        if gather is not None:
            line["frame_embedding"] = gather
        if head is not None:
            line["head"] = head
        print(json.dumps(line), flush=True)
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
