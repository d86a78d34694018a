"""ctypes wrapper of oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arms may import this module.
The restatement follows src/Voxwerk/Talker/Sampler.cs:25-95 and TalkerGenerator.cs:246-251 of voxwerk; parity is
UNPINNED (no golden vectors exist for the sampled path and the C# reference cannot run here) and rests on the
hand-derived known-answer tests in tests/test_oracle_kat.py.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "liboracle.so")


class OracleOptions(ctypes.Structure):
    _fields_ = [("do_sample", ctypes.c_int32), ("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("temperature", ctypes.c_float), ("repetition_penalty", ctypes.c_float)]


def _load():
    if not os.path.exists(_PATH):
        raise ImportError(f"{_PATH} missing: run `make -C oracle`")
    lib = ctypes.CDLL(_PATH)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.oracle_sample_rows.restype = ctypes.c_int
    lib.oracle_sample_rows.argtypes = [vp, i32, i64, i32, i32, i32, vp, vp, vp, vp, ctypes.POINTER(OracleOptions),
                                       vp, i32, i32, i32, i32, vp, vp, i32]
    lib.oracle_apply_repetition_penalty.restype = ctypes.c_int
    lib.oracle_apply_repetition_penalty.argtypes = [vp, i32, vp, i64, ctypes.c_float]
    lib.oracle_select.restype = ctypes.c_int
    lib.oracle_select.argtypes = [vp, i32, ctypes.POINTER(OracleOptions), ctypes.c_double, vp]
    lib.oracle_argmax.restype = ctypes.c_int
    lib.oracle_argmax.argtypes = [vp, i32]
    lib.oracle_dotnet_random.restype = None
    lib.oracle_dotnet_random.argtypes = [i32, vp, i32]
    lib.oracle_dotnet_random_next.restype = None
    lib.oracle_dotnet_random_next.argtypes = [i32, vp, i32]
    lib.oracle_exp_args.restype = i64
    lib.oracle_exp_args.argtypes = [vp, i32, i64, i32, i32, i32, vp, vp, vp, vp, ctypes.POINTER(OracleOptions),
                                    i32, i32, i32, i32, vp, i64]
    lib.oracle_exp.restype = None
    lib.oracle_exp.argtypes = [vp, vp, i64]
    return lib


lib = _load()


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def options(t: Sequence) -> OracleOptions:
    do_sample, top_k, top_p, temperature, rep = t
    return OracleOptions(int(do_sample), int(top_k), float(top_p), float(temperature), float(rep))


def sample_segment(seg, opts: Sequence, threads: int = 1, want_probs: bool = False):
    """Reference ids (and optionally final probabilities) for one workloads.SegData."""
    n = seg.n_rows
    out = np.full(n, -1, dtype=np.int32)
    probs = np.zeros((n, seg.vocab), dtype=np.float64) if want_probs else None
    table = (OracleOptions * len(opts))(*[options(o) for o in opts])
    logits = np.ascontiguousarray(seg.logits)
    st = lib.oracle_sample_rows(
        logits.ctypes.data, int(seg.dtype), int(logits.shape[1]), n, int(seg.vocab), int(seg.kind),
        _p(seg.hist_offsets), _p(seg.hist_ids), _p(seg.steps), _p(seg.opt_index), table, _p(seg.uniforms),
        int(seg.suppress_lo), int(seg.suppress_hi), int(seg.eos_id), int(seg.min_new_tokens), out.ctypes.data,
        _p(probs), int(threads))
    if st != 0:
        raise IndexError("history id out of range")
    return (out, probs) if want_probs else out


def exp_args(seg, opts: Sequence) -> np.ndarray:
    """Every argument the oracle's softmax passes to exp (the fp32 x - max of each survivor), row by row."""
    table = (OracleOptions * len(opts))(*[options(o) for o in opts])
    logits = np.ascontiguousarray(seg.logits)
    call = lambda out, cap: lib.oracle_exp_args(
        logits.ctypes.data, int(seg.dtype), int(logits.shape[1]), seg.n_rows, int(seg.vocab), int(seg.kind),
        _p(seg.hist_offsets), _p(seg.hist_ids), _p(seg.steps), _p(seg.opt_index), table, int(seg.suppress_lo),
        int(seg.suppress_hi), int(seg.eos_id), int(seg.min_new_tokens), out, cap)
    n = call(None, 0)
    if n < 0:
        raise IndexError("history id out of range")
    out = np.empty(n, dtype=np.float32)
    call(out.ctypes.data, n)
    return out


def select(logits: np.ndarray, opt: Sequence, r: float, want_probs: bool = False):
    """Sampler.Select on a copy of one fp32 row."""
    row = np.array(logits, dtype=np.float32, copy=True)
    probs = np.zeros(row.size, dtype=np.float64) if want_probs else None
    o = options(opt)
    res = lib.oracle_select(row.ctypes.data, row.size, ctypes.byref(o), float(r), _p(probs))
    return (res, probs) if want_probs else res


def apply_repetition_penalty(logits: np.ndarray, history: Sequence[int], penalty: float) -> np.ndarray:
    row = np.array(logits, dtype=np.float32, copy=True)
    h = np.ascontiguousarray(np.asarray(history, dtype=np.int32))
    if lib.oracle_apply_repetition_penalty(row.ctypes.data, row.size, h.ctypes.data, h.size, float(penalty)) != 0:
        raise IndexError("history id out of range")
    return row


def argmax(logits: np.ndarray) -> int:
    row = np.ascontiguousarray(logits, dtype=np.float32)
    return lib.oracle_argmax(row.ctypes.data, row.size)


def dotnet_random(seed: int, count: int) -> np.ndarray:
    out = np.zeros(count, dtype=np.float64)
    lib.oracle_dotnet_random(int(seed), out.ctypes.data, int(count))
    return out


def dotnet_random_next(seed: int, count: int) -> np.ndarray:
    out = np.zeros(count, dtype=np.int32)
    lib.oracle_dotnet_random_next(int(seed), out.ctypes.data, int(count))
    return out


def glibc_exp(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty_like(x)
    lib.oracle_exp(x.ctypes.data, y.ctypes.data, x.size)
    return y
