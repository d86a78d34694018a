"""A second, independent restatement of voxwerk's Sampler in pure Python (small rows only).

Test infrastructure: used to cross-check the C++ oracle (oracle/vw_oracle.cpp) rule by rule.  Follows
src/Voxwerk/Talker/Sampler.cs:25-95 and TalkerGenerator.cs:247-248; fp32 steps use numpy float32 scalars, fp64
steps Python floats, Math.Exp -> math.exp (libm), OrderBy -> sorted (stable).
"""

import math

import numpy as np

f32 = np.float32
NEG_INF = f32(-np.inf)


def apply_repetition_penalty(x, history, penalty):
    x = [f32(v) for v in x]
    if f32(penalty) == f32(1.0):
        return x
    seen = set()
    for i in history:
        if i < 0 or i >= len(x):
            raise IndexError(i)
        if i in seen:
            continue
        seen.add(i)
        s = x[i]
        x[i] = f32(s * f32(penalty)) if s < 0 else f32(s / f32(penalty))
    return x


def suppress(x, lo, hi, eos, step, min_new=2):
    x = list(x)
    for i in range(max(lo, 0), min(hi, len(x))):
        if i != eos:
            x[i] = NEG_INF
    if step < min_new and 0 <= eos < len(x):
        x[eos] = NEG_INF
    return x


def argmax(x):
    best = 0
    for i in range(1, len(x)):
        if x[i] > x[best]:
            best = i
    return best


def select(x, do_sample, top_k, top_p, temperature, r):
    """Returns (id, probs)."""
    x = [f32(v) for v in x]
    n = len(x)
    if not do_sample:
        return argmax(x), [0.0] * n
    inv_t = f32(f32(1.0) / f32(temperature))
    x = [f32(v * inv_t) for v in x]
    if 0 < top_k < n:
        kth = sorted(x)[n - top_k]
        x = [NEG_INF if v < kth else v for v in x]
    mx = NEG_INF
    for v in x:
        mx = max(mx, v)
    probs = [0.0] * n
    s = 0.0
    for i in range(n):
        probs[i] = 0.0 if (np.isinf(x[i]) and x[i] < 0) else math.exp(float(f32(x[i] - mx)))
        s += probs[i]
    probs = [p / s for p in probs]
    if f32(top_p) < f32(1.0):
        idx = sorted(range(n), key=lambda i: probs[i])
        thr = float(f32(f32(1.0) - f32(top_p)))
        cum = 0.0
        for j in range(n - 1):
            cum += probs[idx[j]]
            if cum <= thr:
                probs[idx[j]] = 0.0
            else:
                break
        s = 0.0
        for p in probs:
            s += p
        probs = [p / s for p in probs]
    acc, last = 0.0, 0
    for i in range(n):
        if probs[i] <= 0:
            continue
        acc += probs[i]
        last = i
        if r < acc:
            return i, probs
    return last, probs
