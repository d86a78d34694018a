"""Benchmark of the fused sampler on the headline configuration (config 2: a batched talker step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

One step = one vw_sample call over one batch of 4096 talker rows (V = 3072 fp32 logits, 1024-id histories,
T 0.9, top-k 50, top-p 0.8, repetition penalty 1.05, suppress mask).  Under torchrun each rank samples its own
4096-row batch (rows are independent; weak scaling; no collective on the data path -- NCCL only carries the
barrier and the max-over-ranks of the timings).

value: rows/s of the whole job with inputs resident in HBM (3 rotating input copies, 201 MB > the 126 MB L2, so
no step reads another step's data from L2); K steps captured in one CUDA graph and timed with CUDA events on the
launching stream.  e2e: the same metric through the public C-ABI call with host buffers (pinned host -> device
copies of logits, histories and uniforms, and the ids back) inside the timed region.  cpu_baseline: the CPU
restatement of voxwerk's Sampler (oracle/, "port": the C# reference cannot run here) on a bounded sample.
`--impl reference` times only that CPU implementation, with every host thread, and prints its own line.
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
FALLBACK_HBM_GBS = 6650.0


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


def cpu_reference(workload, seconds: float, threads: int):
    """Times the CPU restatement (oracle port) on repeated passes over the workload's rows."""
    from oracle import oracle
    seg = workload.segments[0]
    t0 = time.perf_counter()
    rows = 0
    while True:
        oracle.sample_segment(seg, workload.options, threads=threads)
        rows += seg.n_rows
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return rows / el, rows, el


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from voxwerk_b200 import workloads
    w = workloads.make(args.config)
    threads = host_threads()
    per_step = []
    for i in range(args.warmup + args.steps):
        v, rows, el = cpu_reference(w, 0.0, threads)
        if i >= args.warmup:
            per_step.append(el)
    t = float(np.sum(per_step))
    value = args.steps * w.n_rows / t
    sample = f"{w.n_rows} rows of {w.name} per step, {threads} threads (std::thread over rows)"
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "rows_per_step": w.n_rows, **workload_keys(w)},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port", "sample": sample,
                         "what": "C++ restatement of voxwerk Sampler.cs (oracle/vw_oracle.cpp); the C# reference "
                                 "cannot be built or run in this environment"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


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

    from tests.gpu_util import make_segment, options_table, to_device
    from voxwerk_b200 import Device, sample_rows, workloads
    from voxwerk_b200.shard import max_over_ranks

    dev = Device(local)
    w = workloads.make(args.config)
    if rank > 0:   # weak scaling: each rank its own batch of the same shape
        import copy
        rng = np.random.default_rng(7919 * rank)
        w = copy.deepcopy(w)
        for s in w.segments:
            perm = rng.permutation(s.n_rows)
            s.logits = np.ascontiguousarray(s.logits[perm])
    opts = options_table(w)
    n_copies = 3
    copies = []
    for c in range(n_copies):
        segs, keep = [], []
        for s in w.segments:
            arr = to_device(s, torch)
            if c > 0:   # distinct buffers with the same contents
                arr = {k: (v.clone() if v is not None else None) for k, v in arr.items()}
            keep.append(arr)
            hist_max = 0
            if s.hist_offsets is not None:
                hist_max = int(np.max(np.diff(s.hist_offsets)))
            segs.append(make_segment(s, arr, max_hist_len=hist_max))
        copies.append((segs, keep))
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    # ---- warm-up (also sizes the library's scratch before capture)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            sample_rows(dev, copies[i % n_copies][0], opts, stream=sp)
    dev.synchronize(sp)

    # ---- parity spot check on this rank's first copy (rank 0, first 256 rows)
    parity = None
    if rank == 0:
        from oracle import oracle
        ids = copies[0][1][0]["out_ids"].cpu().numpy()
        sub = w.segments[0].slice(0, min(256, w.segments[0].n_rows))
        sample_rows(dev, copies[0][0], opts, stream=sp)
        dev.synchronize(sp)
        ids = copies[0][1][0]["out_ids"].cpu().numpy()[:sub.n_rows]
        ref = oracle.sample_segment(sub, w.options, threads=host_threads())
        parity = f"{int((ids == ref).sum())}/{sub.n_rows} rows bit-exact vs oracle"

    # ---- capture K steps in one graph (rotating input copies)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            sample_rows(dev, copies[i % n_copies][0], opts, stream=torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    dev.stats(reset=True)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    elapsed_ms = ev0.elapsed_time(ev1)
    dev.synchronize(sp)   # raises if the kernel latched an error
    paths = dev.stats(reset=True)
    elapsed_max = max_over_ranks(elapsed_ms, device="cuda")
    rows_per_rank = w.n_rows
    total_rows = rows_per_rank * world * args.steps
    value = total_rows / (elapsed_max * 1e-3)
    ms_per_step = elapsed_max / args.steps

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
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        sample_rows(dev, hsegs, opts)
    e2e_s = time.perf_counter() - t0
    # bytes the library copied host -> device per step (it skips the logit columns no kernel reads)
    h2d = dev.stats(reset=True)["h2d_bytes"] // max(args.e2e_steps, 1)
    e2e_value = rows_per_rank * world * args.e2e_steps / max_over_ranks(e2e_s, device="cuda")

    line = None
    if rank == 0:
        alg = w.algorithmic_bytes()
        need = w.needed_bytes()
        peak, peak_kind = hbm_peak()
        achieved = alg / (ms_per_step * 1e-3) / 1e9
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tpath):
            try:
                traffic = json.load(open(tpath)).get(w.name)
            except Exception:
                traffic = None
        cpu = None
        if world == 1 and not args.no_cpu:
            thr = host_threads()
            v_all, rows_all, el_all = cpu_reference(w, args.cpu_seconds, thr)
            v_one, rows_one, el_one = cpu_reference(w.shard(0, 16), min(3.0, args.cpu_seconds), 1)
            cpu = {"value": v_all, "unit": "rows/s", "cores": thr, "kind": "port",
                   "sample": f"{rows_all} rows ({rows_all // w.n_rows} passes over {w.name}) in {el_all:.1f} s "
                             f"on {thr} threads; 1 thread: {v_one:.0f} rows/s",
                   "what": "C++ restatement of voxwerk Sampler.cs (oracle/), the C# reference cannot run here"}
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w.name, "rows_per_gpu": rows_per_rank, "global_rows": rows_per_rank * world,
                       **workload_keys(w), "parallelism": f"row shards x{world}, no collective",
                       "l2": f"{n_copies} rotating input copies ({n_copies * alg / 1e6:.0f} MB > 126 MB L2)",
                       "timing": "K steps in one CUDA graph, CUDA events on the launching stream, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": alg, "needed_bytes_per_launch": need,
                         "frac_of_needed_bytes": need / (ms_per_step * 1e-3) / 1e9 / peak,
                         "kernel": "cand_kernel (the step: cand_kernel + whole-row kernel launch, CUDA events)"},
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": args.e2e_steps,
                    "path": "vw_sample(VW_MEM_HOST) from pinned host buffers: logits (without the suppressed "
                            "span's columns), histories, steps, options, uniforms in; ids out"},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "gpu_launches": 2 * args.steps,   # per step: the candidate kernel + the whole-row kernel
            "parity": parity,
            "rows_by_path": paths,
        }
        print(json.dumps(line), flush=True)
    del graph
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
