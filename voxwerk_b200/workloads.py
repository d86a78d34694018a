"""Seeded synthetic inputs with the shapes of the five benchmark configurations.

No dataset is involved: the reference benchmarks nothing on this path, and the configurations are synthetic by
definition.  Logits, boosts and histories come from ``numpy.random.default_rng(1000 + config)``; uniforms come
from ``DotNetRandom`` exactly as the reference draws them: talker rows from ``Random(42)`` (the job seed) in row
order, sub-talker rows from ``Random(43)`` (``Seed + 1``, TalkerGenerator.cs:218) in (stream, codebook 1..15) order,
greedy rows taking no draw.

Configurations (talker V = 3072, code-predictor V = 2048):
  0  1 talker row fp32, N(0, 4^2), 8 ids +12, mask, T 0.9 K 50 P 1.0 rp 1.05, 256-id history
  1  15 sub rows fp32, N(0, 3^2), one id +10 per row, T 0.9 K 50 P 1.0
  2  4096 talker rows fp32, N(0, 4^2), 1-16 ids +12, mask, T 0.9 K 50 P 0.8 rp 1.05, 1024-id histories
  3  1024 talker rows + 15360 sub rows, bf16 N(0, 3^2) (RNE), talker as 2, sub T 0.9 K 50 P 1.0
  4  8192 talker rows fp32: rows < 4096 on a 16-level grid (l - 7.5), the rest N(0, 0.01^2); top-k off (K = V),
     P 0.5, rp 1.3 over 4096-id histories in [0, 3072) with duplicates, no mask, greedy on every 10th row
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from .dotnet_random import DotNetRandom
from .qwen3_tts import CODEC_EOS_ID, CP_VOCAB_SIZE, MIN_NEW_TOKENS, VOCAB_SIZE

F32, BF16 = 0, 1
TALKER, SUB = 0, 1


@dataclass
class SegData:
    """One segment's host arrays (mirrors vw_segment)."""

    logits: np.ndarray                 # [n, V] float32, or uint16 bf16 bit patterns
    dtype: int
    kind: int
    vocab: int
    uniforms: np.ndarray               # [n] float64
    opt_index: Optional[np.ndarray] = None
    hist_offsets: Optional[np.ndarray] = None
    hist_ids: Optional[np.ndarray] = None
    steps: Optional[np.ndarray] = None
    suppress_lo: int = 0
    suppress_hi: int = 0
    eos_id: int = CODEC_EOS_ID
    min_new_tokens: int = MIN_NEW_TOKENS

    @property
    def n_rows(self) -> int:
        return int(self.logits.shape[0])

    def algorithmic_bytes(self) -> int:
        """Logits + int32 history bytes (the benchmark's roofline numerator)."""
        b = self.logits.nbytes
        if self.hist_ids is not None and self.hist_offsets is not None:
            b += int(self.hist_offsets[-1] - self.hist_offsets[0]) * 4
        return b

    def needed_bytes(self) -> int:
        """Bytes the sampler must read: logits outside the suppressed span (plus the EOS vector) + history."""
        esize = 4 if self.dtype == F32 else 2
        row = self.vocab
        if self.kind == TALKER and self.suppress_lo < self.suppress_hi:
            vw = 16 // esize
            la = -(-self.suppress_lo // vw) * vw
            ha = self.suppress_hi // vw * vw
            if la < ha:
                row = la + (self.vocab - ha) + vw
        b = self.n_rows * row * esize
        if self.hist_ids is not None and self.hist_offsets is not None:
            b += int(self.hist_offsets[-1] - self.hist_offsets[0]) * 4
        return b

    def take(self, rows) -> "SegData":
        """The listed rows (any order) with their histories gathered into a fresh CSR."""
        rows = np.asarray(rows, dtype=np.int64)
        ho = hid = None
        if self.hist_offsets is not None:
            lens = self.hist_offsets[rows + 1] - self.hist_offsets[rows]
            ho = np.zeros(rows.size + 1, dtype=np.int64)
            ho[1:] = np.cumsum(lens)
            parts = [self.hist_ids[self.hist_offsets[r]:self.hist_offsets[r + 1]] for r in rows]
            hid = np.concatenate(parts).astype(np.int32) if parts and ho[-1] > 0 else np.zeros(4, np.int32)
        pick = lambda a: None if a is None else np.ascontiguousarray(a[rows])
        return SegData(np.ascontiguousarray(self.logits[rows]), self.dtype, self.kind, self.vocab,
                       pick(self.uniforms), pick(self.opt_index), ho, hid, pick(self.steps), self.suppress_lo,
                       self.suppress_hi, self.eos_id, self.min_new_tokens)

    def slice(self, lo: int, hi: int) -> "SegData":
        """Rows [lo, hi) with histories re-based (a contiguous row shard)."""
        ho = hid = None
        if self.hist_offsets is not None:
            a, b = int(self.hist_offsets[lo]), int(self.hist_offsets[hi])
            ho = (self.hist_offsets[lo:hi + 1] - a).astype(np.int64)
            hid = np.ascontiguousarray(self.hist_ids[a:b])
            if hid.size == 0:
                hid = np.zeros(4, dtype=np.int32)
        return SegData(np.ascontiguousarray(self.logits[lo:hi]), self.dtype, self.kind, self.vocab,
                       np.ascontiguousarray(self.uniforms[lo:hi]),
                       None if self.opt_index is None else np.ascontiguousarray(self.opt_index[lo:hi]),
                       ho, hid, None if self.steps is None else np.ascontiguousarray(self.steps[lo:hi]),
                       self.suppress_lo, self.suppress_hi, self.eos_id, self.min_new_tokens)


@dataclass
class Workload:
    name: str
    config: int
    segments: List[SegData]
    options: List[tuple]               # (do_sample, top_k, top_p, temperature, repetition_penalty)
    notes: dict = field(default_factory=dict)

    @property
    def n_rows(self) -> int:
        return sum(s.n_rows for s in self.segments)

    def algorithmic_bytes(self) -> int:
        return sum(s.algorithmic_bytes() for s in self.segments)

    def needed_bytes(self) -> int:
        return sum(s.needed_bytes() for s in self.segments)

    def shard(self, rank: int, world: int) -> "Workload":
        """Contiguous row shard for `rank` of `world`, cost-weighted across segments by bytes per row."""
        from .shard import shard_bounds
        costs = [(s.n_rows, s.algorithmic_bytes() / max(s.n_rows, 1)) for s in self.segments]
        out = [self.segments[k].slice(a, b) for k, a, b in shard_bounds(costs, rank, world)]
        return Workload(f"{self.name}[{rank}/{world}]", self.config, out, self.options, dict(self.notes))


def _bf16_rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (Bf16.FromFloat, Bf16.cs:16-22; no NaNs here)."""
    b = x.astype(np.float32).view(np.uint32)
    return ((b + (np.uint32(0x7FFF) + ((b >> 16) & 1))) >> 16).astype(np.uint16)


def _histories(rng, n: int, length: int, hi: int):
    ids = rng.integers(0, hi, size=(n, length), dtype=np.int32).reshape(-1)
    offs = np.arange(n + 1, dtype=np.int64) * length
    return offs, ids


def _uniforms(seed: int, count: int, greedy: Optional[np.ndarray] = None) -> np.ndarray:
    g = DotNetRandom(seed)
    u = np.zeros(count, dtype=np.float64)
    for i in range(count):
        if greedy is None or not greedy[i]:
            u[i] = g.next_double()
    return u


def make(config: int, rows: Optional[int] = None) -> Workload:
    """The synthetic workload of `config` (0-4); `rows` truncates config 2 / 4 (or scales config 3's streams)."""
    rng = np.random.default_rng(1000 + config)
    V, CV = VOCAB_SIZE, CP_VOCAB_SIZE
    talker_mask = dict(suppress_lo=V - 1024, suppress_hi=V)
    if config == 0:
        x = rng.normal(0.0, 4.0, size=(1, V)).astype(np.float32)
        ids = rng.choice(2048, size=8, replace=False)
        x[0, ids] += np.float32(12.0)
        ho, hi = _histories(rng, 1, 256, 2048)
        seg = SegData(x, F32, TALKER, V, _uniforms(42, 1), np.zeros(1, np.int32), ho, hi,
                      np.full(1, 2, np.int32), **talker_mask)
        return Workload("cfg0_talker_1x3072_f32", 0, [seg], [(1, 50, 1.0, 0.9, 1.05)])
    if config == 1:
        x = rng.normal(0.0, 3.0, size=(15, CV)).astype(np.float32)
        x[np.arange(15), rng.integers(0, CV, size=15)] += np.float32(10.0)
        seg = SegData(x, F32, SUB, CV, _uniforms(43, 15), np.zeros(15, np.int32))
        return Workload("cfg1_sub_15x2048_f32", 1, [seg], [(1, 50, 1.0, 0.9, 1.0)])
    if config == 2:
        n = rows or 4096
        x = rng.normal(0.0, 4.0, size=(n, V)).astype(np.float32)
        nb = rng.integers(1, 17, size=n)
        for r in range(n):
            x[r, rng.choice(2048, size=nb[r], replace=False)] += np.float32(12.0)
        ho, hi = _histories(rng, n, 1024, 2048)
        seg = SegData(x, F32, TALKER, V, _uniforms(42, n), np.zeros(n, np.int32), ho, hi,
                      np.full(n, 2, np.int32), **talker_mask)
        return Workload(f"cfg2_talker_{n}x3072_f32_topk50_topp0.8", 2, [seg], [(1, 50, 0.8, 0.9, 1.05)])
    if config == 3:
        streams = rows or 1024
        xt = rng.normal(0.0, 3.0, size=(streams, V)).astype(np.float32)
        nb = rng.integers(1, 17, size=streams)
        for r in range(streams):
            xt[r, rng.choice(2048, size=nb[r], replace=False)] += np.float32(12.0)
        ho, hi = _histories(rng, streams, 1024, 2048)
        talker = SegData(_bf16_rne(xt), BF16, TALKER, V, _uniforms(42, streams), np.zeros(streams, np.int32), ho,
                         hi, np.full(streams, 2, np.int32), **talker_mask)
        xs = rng.normal(0.0, 3.0, size=(streams * 15, CV)).astype(np.float32)
        sub = SegData(_bf16_rne(xs), BF16, SUB, CV, _uniforms(43, streams * 15), np.ones(streams * 15, np.int32))
        return Workload(f"cfg3_frame_{streams}x3072+{streams * 15}x2048_bf16", 3, [talker, sub],
                        [(1, 50, 0.8, 0.9, 1.05), (1, 50, 1.0, 0.9, 1.0)])
    if config == 4:
        n = rows or 8192
        half = n // 2
        x = np.empty((n, V), dtype=np.float32)
        x[:half] = (rng.integers(0, 16, size=(half, V)).astype(np.float32) - np.float32(7.5))
        x[half:] = rng.normal(0.0, 0.01, size=(n - half, V)).astype(np.float32)
        ho, hi = _histories(rng, n, 4096, V)
        greedy = (np.arange(n) % 10) == 0
        opt_index = greedy.astype(np.int32)   # 0: sample, 1: greedy
        seg = SegData(x, F32, TALKER, V, _uniforms(42, n, greedy), opt_index, ho, hi, np.full(n, 2, np.int32),
                      suppress_lo=0, suppress_hi=0)
        return Workload(f"cfg4_adversarial_{n}x3072_f32", 4, [seg], [(1, V, 0.5, 0.9, 1.3), (0, V, 0.5, 0.9, 1.3)],
                        notes={"temperature": "0.9 (not stated by the configuration)"})
    raise ValueError(f"unknown config {config}")
