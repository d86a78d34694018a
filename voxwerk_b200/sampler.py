"""Host-side mirror of voxwerk's sampling interface over the B200 kernel.

Reference types and methods mirrored here (paths inside the voxwerk repository):

* ``SamplingOptions``   -- src/Voxwerk/Talker/Sampler.cs:4-13
* ``GenerationOptions`` -- src/Voxwerk/Talker/TalkerGenerator.cs:7-22
* ``Sampler``           -- src/Voxwerk/Talker/Sampler.cs:17-96 (``apply_repetition_penalty``, ``select``, ``arg_max``)
* ``TalkerBatchSampler``-- the per-step sampling of ``TalkerGenerator.GenerateBatch``
  (TalkerGenerator.cs:366-385 talker rows, :416-420 sub-talker rows) as one GPU call per stage.
* ``DotNetRandom``      -- ``System.Random(int)`` used by ``Sampler`` (Sampler.cs:21), restated from the published
  subtractive-generator method (Knuth, TAOCP Vol. 2 3.2.2; Numerical Recipes ``ran3``) with .NET's modulus
  2^31-1 and second tap 21.

Everything numeric runs in libvwsampler.so on the GPU; this module only builds the C structs, draws the
uniforms the reference would draw, and converts status codes to exceptions.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import (VW_BF16, VW_F32, VW_MEM_DEVICE, VW_MEM_HOST, VW_ROWS_SUB, VW_ROWS_TALKER, VwOptions,
                   VwSegment, check, lib)
from .dotnet_random import DotNetRandom
from .qwen3_tts import (CODEC_EOS_ID, CP_VOCAB_SIZE, MIN_NEW_TOKENS, NUM_CODE_GROUPS, SUPPRESS_SPAN,  # noqa: F401
                        VOCAB_SIZE)

@dataclass(frozen=True)
class SamplingOptions:
    """SamplingOptions (Sampler.cs:4-13): one stage's decoding settings."""

    do_sample: bool = True
    top_k: int = 50
    top_p: float = 1.0
    temperature: float = 0.9

    @staticmethod
    def greedy() -> "SamplingOptions":
        """SamplingOptions.Greedy (Sampler.cs:12)."""
        return SamplingOptions(do_sample=False)


@dataclass(frozen=True)
class GenerationOptions:
    """GenerationOptions (TalkerGenerator.cs:7-22)."""

    max_new_tokens: int = 2048
    repetition_penalty: float = 1.05
    talker: SamplingOptions = field(default_factory=SamplingOptions)
    sub_talker: SamplingOptions = field(default_factory=SamplingOptions)
    non_streaming_mode: Optional[bool] = None
    seed: Optional[int] = None

    @staticmethod
    def greedy() -> "GenerationOptions":
        """GenerationOptions.Greedy (TalkerGenerator.cs:21)."""
        return GenerationOptions(talker=SamplingOptions.greedy(), sub_talker=SamplingOptions.greedy())


def vw_options(opts: SamplingOptions, repetition_penalty: float = 1.0) -> VwOptions:
    """The C struct for one stage (talker rows carry the job's RepetitionPenalty, sub rows 1.0)."""
    return VwOptions(int(bool(opts.do_sample)), int(opts.top_k), float(opts.top_p), float(opts.temperature),
                     float(repetition_penalty))


class Device:
    """One vw_handle: the sampler bound to one CUDA device (not shared between host threads)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        st = lib.vw_create(int(device), ctypes.byref(h))
        if st != _lib.VW_OK:
            raise _lib.VwError(st, f"vw_create({device}) failed: {lib.vw_status_string(st).decode()}")
        self._h = h
        self.device = int(device)

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise RuntimeError("device handle is closed")
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None) is not None:
            lib.vw_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def stats(self, reset: bool = False) -> dict:
        """vw_get_stats: rows sampled per path (call after synchronizing the work of interest)."""
        st = _lib.VwStats()
        check(lib.vw_get_stats(self.handle, ctypes.byref(st), 1 if reset else 0), self.handle)
        return st.as_dict()

    def synchronize(self, stream: Optional[int] = None) -> None:
        """vw_synchronize: waits for `stream` and raises any device-side error latched by earlier calls."""
        check(lib.vw_synchronize(self.handle, ctypes.c_void_p(stream) if stream else None), self.handle)


# ----------------------------------------------------------------------------- batched rows
def _is_torch_cuda(x) -> bool:
    return hasattr(x, "data_ptr") and hasattr(x, "is_cuda") and bool(x.is_cuda)


def _ptr(x, mem: int) -> Optional[int]:
    if x is None:
        return None
    if mem == VW_MEM_DEVICE:
        if not _is_torch_cuda(x):
            raise TypeError("device calls take CUDA tensors for every array")
        return int(x.data_ptr())
    if _is_torch_cuda(x):
        raise TypeError("host calls take host arrays for every array")
    if hasattr(x, "data_ptr"):   # CPU torch tensor (pinned or not)
        return int(x.data_ptr())
    if not isinstance(x, np.ndarray) or not x.flags["C_CONTIGUOUS"]:
        raise TypeError("host arrays must be C-contiguous numpy arrays or CPU tensors")
    return int(x.ctypes.data)


def _dtype_code(x) -> int:
    name = str(getattr(x, "dtype", ""))
    if "bfloat16" in name:
        return VW_BF16
    if name in ("float32", "torch.float32"):
        return VW_F32
    if name in ("uint16", "torch.uint16", "torch.int16", "int16"):   # raw bf16 bit patterns
        return VW_BF16
    raise TypeError(f"logits must be float32 or bfloat16, got {name}")


@dataclass
class Segment:
    """A block of rows for one ``sample_rows`` call (mirrors vw_segment).

    ``logits`` is [n_rows, row_stride] (float32, or bfloat16 / raw uint16 bf16 bits).  Talker segments also take
    CSR histories (``hist_offsets`` [n_rows + 1] int64, ``hist_ids`` int32), per-row ``steps`` (int32) and the
    suppress mask.  ``opt_index`` (int32) picks each row's entry of the options table; ``uniforms`` (float64)
    holds each row's NextDouble() draw; ``out_ids`` (int32) receives the ids and the optional ``out_probs``
    (float64 [n_rows, vocab]) the final probabilities.
    """

    logits: object
    kind: int = VW_ROWS_SUB
    vocab: Optional[int] = None
    out_ids: object = None
    uniforms: object = None
    opt_index: object = None
    hist_offsets: object = None
    hist_ids: object = None
    steps: object = None
    suppress_lo: Optional[int] = None
    suppress_hi: Optional[int] = None
    eos_id: int = CODEC_EOS_ID
    min_new_tokens: int = MIN_NEW_TOKENS
    max_hist_len: int = 0
    out_probs: object = None

    def to_c(self, mem: int, shape: Optional[tuple] = None) -> VwSegment:
        """The C struct; `shape` stands in for logits.shape when the logits come from vw_head_sample's GEMM."""
        shape = tuple(self.logits.shape) if shape is None else tuple(shape)
        if len(shape) != 2:
            raise ValueError("logits must be 2-D [n_rows, row_stride]")
        n_rows, stride = int(shape[0]), int(shape[1])
        vocab = int(self.vocab if self.vocab is not None else stride)
        if self.kind == VW_ROWS_TALKER:
            lo = vocab - SUPPRESS_SPAN if self.suppress_lo is None else int(self.suppress_lo)
            hi = vocab if self.suppress_hi is None else int(self.suppress_hi)
        else:
            lo = hi = 0
        dtype = VW_F32 if self.logits is None else _dtype_code(self.logits)
        return VwSegment(
            _ptr(self.logits, mem), stride, n_rows, vocab, dtype, int(self.kind),
            _ptr(self.hist_offsets, mem), _ptr(self.hist_ids, mem), _ptr(self.steps, mem), lo, hi,
            int(self.eos_id), int(self.min_new_tokens), int(self.max_hist_len), _ptr(self.opt_index, mem),
            _ptr(self.uniforms, mem), _ptr(self.out_ids, mem), _ptr(self.out_probs, mem))


def _mem_of(segments: Sequence[Segment]) -> int:
    kinds = {_is_torch_cuda(s.logits) for s in segments}
    if len(kinds) != 1:
        raise TypeError("all segments of one call must live on the same side (host or device)")
    return VW_MEM_DEVICE if kinds.pop() else VW_MEM_HOST


def sample_rows(device: Device, segments: Sequence[Segment], options: Sequence[VwOptions],
                stream: Optional[int] = None) -> None:
    """One vw_sample call over `segments` (<= 8).  Ids land in each segment's ``out_ids``.

    CUDA tensors -> VW_MEM_DEVICE (stream-ordered on `stream` when given, else synchronous); host arrays ->
    VW_MEM_HOST (synchronous).
    """
    if not 1 <= len(segments) <= _lib.VW_MAX_SEGMENTS:
        raise ValueError("1..8 segments per call")
    mem = _mem_of(segments)
    segs = (VwSegment * len(segments))(*[s.to_c(mem) for s in segments])
    opts = (VwOptions * len(options))(*options)
    st = ctypes.c_void_p(stream) if stream else None
    check(lib.vw_sample(device.handle, segs, len(segments), opts, len(options), mem, st), device.handle)


def sample_rows_static(device: int, segments: Sequence[Segment], options: Sequence[VwOptions],
                       stream: Optional[int] = None) -> None:
    """One vw_sample_static call: ``sample_rows`` on CUDA tensors of GPU `device`, without a handle and without any
    device allocation (for processes whose device memory is all held elsewhere, e.g. by a serving engine's pool).

    The library's fixed per-device scratch bounds a call to 65536 rows, vocab <= 4096 and 32 options.  The call
    returns after `stream` (None: the default stream) has finished it.  Two calls on one device must not overlap
    in time: they share that scratch.
    """
    if not 1 <= len(segments) <= _lib.VW_MAX_SEGMENTS:
        raise ValueError("1..8 segments per call")
    if _mem_of(segments) != VW_MEM_DEVICE:
        raise ValueError("vw_sample_static takes device tensors only")
    segs = (VwSegment * len(segments))(*[s.to_c(VW_MEM_DEVICE) for s in segments])
    opts = (VwOptions * len(options))(*options)
    msg = ctypes.create_string_buffer(512)
    st = lib.vw_sample_static(device, segs, len(segments), opts, len(options),
                              ctypes.c_void_p(stream) if stream else None, msg, len(msg))
    if st != _lib.VW_OK:
        text = msg.value.decode() or lib.vw_status_string(st).decode()
        if st == _lib.VW_ERR_INVALID_ARG:
            raise _lib.VwInvalidArgument(st, text)
        if st == _lib.VW_ERR_OUT_OF_RANGE:
            raise _lib.VwOutOfRange(st, text)
        raise _lib.VwError(st, text)


# ----------------------------------------------------------------------------- Sampler mirror
_default_device: Optional[Device] = None


def default_device() -> Device:
    global _default_device
    if _default_device is None:
        _default_device = Device(0)
    return _default_device


def _host_f32(logits) -> np.ndarray:
    a = np.ascontiguousarray(logits, dtype=np.float32)
    if a.ndim != 1:
        raise ValueError("one logits row expected")
    return a


class Sampler:
    """Sampler (Sampler.cs:17-96) over the GPU kernel.

    ``Sampler(seed)`` owns a ``DotNetRandom(seed)`` exactly like the reference (``seed=None`` -> unseeded) and takes one
    NextDouble() per sampled ``select``; greedy selects draw nothing.  Logits are host float32 rows.
    """

    def __init__(self, seed: Optional[int], device: Optional[Device] = None):
        self.rng = DotNetRandom(seed)
        self.device = device or default_device()

    @staticmethod
    def apply_repetition_penalty(logits: np.ndarray, history: Sequence[int], penalty: float,
                                 device: Optional[Device] = None) -> None:
        """Sampler.ApplyRepetitionPenalty (Sampler.cs:25-33), in place on a host float32 row."""
        if not isinstance(logits, np.ndarray) or logits.dtype != np.float32 or not logits.flags["C_CONTIGUOUS"]:
            raise TypeError("logits must be a C-contiguous float32 numpy array (modified in place)")
        dev = device or default_device()
        h = np.ascontiguousarray(np.asarray(history, dtype=np.int32))
        check(lib.vw_apply_repetition_penalty(dev.handle, logits.ctypes.data, logits.size, h.ctypes.data,
                                              h.size, ctypes.c_float(penalty), VW_MEM_HOST), dev.handle)

    def select(self, logits, opts: SamplingOptions) -> int:
        """Sampler.Select (Sampler.cs:35-88).  Unlike the reference the row is not modified."""
        row = _host_f32(logits)
        r = self.rng.next_double() if opts.do_sample else 0.0
        out = ctypes.c_int32(-1)
        o = vw_options(opts)
        check(lib.vw_select(self.device.handle, row.ctypes.data, row.size, ctypes.byref(o), ctypes.c_double(r),
                            VW_MEM_HOST, ctypes.byref(out)), self.device.handle)
        return int(out.value)

    @staticmethod
    def arg_max(logits, device: Optional[Device] = None) -> int:
        """Sampler.ArgMax (Sampler.cs:90-95)."""
        row = _host_f32(logits)
        dev = device or default_device()
        out = ctypes.c_int32(-1)
        check(lib.vw_argmax(dev.handle, row.ctypes.data, row.size, VW_MEM_HOST, ctypes.byref(out)), dev.handle)
        return int(out.value)


class TalkerBatchSampler:
    """Per-step sampling of ``TalkerGenerator.GenerateBatch`` as one GPU call per stage.

    Holds, per job, the reference's ``Sampler(Seed)`` / ``Sampler(Seed + 1)`` RNGs (TalkerGenerator.cs:345-346),
    the talker history (``Active.History``) and step counter (``Active.Step``).  ``talker_step`` replaces the loop
    at :366-385 (penalty, mask, Select) and ``sub_step`` the loop at :419-420.  Logits are host float32 arrays.
    """

    def __init__(self, jobs: Sequence[GenerationOptions], device: Optional[Device] = None,
                 vocab: int = VOCAB_SIZE, cp_vocab: int = CP_VOCAB_SIZE, eos_id: int = CODEC_EOS_ID):
        self.device = device or default_device()
        self.jobs = list(jobs)
        self.vocab, self.cp_vocab, self.eos_id = vocab, cp_vocab, eos_id
        self.rng = [DotNetRandom(j.seed) for j in self.jobs]
        self.sub_rng = [DotNetRandom(None if j.seed is None else int(np.int32(np.int64(j.seed) + 1)))
                        for j in self.jobs]
        self.history: List[List[int]] = [[] for _ in self.jobs]
        self.step: List[int] = [0 for _ in self.jobs]

    def _tables(self, active: Sequence[int], stage: str):
        opts, index = [], {}
        for j in active:
            job = self.jobs[j]
            key = (job.talker, job.repetition_penalty) if stage == "talker" else (job.sub_talker, 1.0)
            if key not in index:
                index[key] = len(opts)
                opts.append(vw_options(*key))
        return opts, np.array([index[(self.jobs[j].talker, self.jobs[j].repetition_penalty) if stage == "talker"
                                      else (self.jobs[j].sub_talker, 1.0)] for j in active], dtype=np.int32)

    def talker_step(self, active: Sequence[int], logits: np.ndarray) -> np.ndarray:
        """Codebook-0 ids for the active jobs (rows of `logits` [A, V] in `active` order); appends to histories."""
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        opts, oi = self._tables(active, "talker")
        u = np.array([self.rng[j].next_double() if self.jobs[j].talker.do_sample else 0.0 for j in active])
        lens = [len(self.history[j]) for j in active]
        offs = np.zeros(len(active) + 1, dtype=np.int64)
        offs[1:] = np.cumsum(lens)
        hist = np.array([t for j in active for t in self.history[j]], dtype=np.int32)
        if hist.size == 0:
            hist = np.zeros(4, dtype=np.int32)
        steps = np.array([self.step[j] for j in active], dtype=np.int32)
        out = np.full(len(active), -1, dtype=np.int32)
        seg = Segment(logits, kind=VW_ROWS_TALKER, vocab=self.vocab, out_ids=out, uniforms=u, opt_index=oi,
                      hist_offsets=offs, hist_ids=hist, steps=steps, eos_id=self.eos_id)
        sample_rows(self.device, [seg], opts)
        for j, c in zip(active, out):
            self.history[j].append(int(c))
        return out

    def sub_step(self, active: Sequence[int], cp_logits: np.ndarray) -> np.ndarray:
        """One codebook's ids for the active jobs (rows of `cp_logits` [A, CV])."""
        cp_logits = np.ascontiguousarray(cp_logits, dtype=np.float32)
        opts, oi = self._tables(active, "sub")
        u = np.array([self.sub_rng[j].next_double() if self.jobs[j].sub_talker.do_sample else 0.0 for j in active])
        out = np.full(len(active), -1, dtype=np.int32)
        sample_rows(self.device, [Segment(cp_logits, kind=VW_ROWS_SUB, vocab=self.cp_vocab, out_ids=out,
                                          uniforms=u, opt_index=oi)], opts)
        return out

    def advance(self, active: Sequence[int]) -> None:
        """Active.Step++ for the jobs that produced a frame (TalkerGenerator.cs:440)."""
        for j in active:
            self.step[j] += 1


def frame_embedding(device: Device, codes, codec_embedding, cp_embeddings: Sequence, text, out,
                    stream: Optional[int] = None) -> None:
    """vw_frame_embedding: out = FrameEmbedding(codes) + text (TalkerModel.cs:114-118, TalkerGenerator.cs:437-438).

    CUDA tensors: codes [n, G] int32, codec_embedding [V, H] and each of cp_embeddings [CV, H] as bf16 (or int16 /
    uint16 bits), text [n, H] float32 or None, out [n, H] float32.  Rows whose codes[r, 0] is -1 are left alone.
    """
    for t in [codes, codec_embedding, out, *cp_embeddings] + ([text] if text is not None else []):
        if not _is_torch_cuda(t):
            raise TypeError("frame_embedding takes CUDA tensors")
    n, groups = int(codes.shape[0]), int(codes.shape[1])
    ptrs = (ctypes.c_void_p * max(len(cp_embeddings), 1))(*[t.data_ptr() for t in cp_embeddings])
    check(lib.vw_frame_embedding(device.handle, ctypes.c_void_p(codes.data_ptr()), n, groups,
                                 int(codec_embedding.shape[1]), ctypes.c_void_p(codec_embedding.data_ptr()),
                                 int(codec_embedding.shape[0]), ptrs,
                                 int(cp_embeddings[0].shape[0]) if cp_embeddings else 0,
                                 ctypes.c_void_p(text.data_ptr()) if text is not None else None,
                                 ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream) if stream else None),
          device.handle)


def _head_operands(hidden, weight, *more) -> None:
    for t in [hidden, weight, *[m for m in more if m is not None]]:
        if not _is_torch_cuda(t):
            raise TypeError("the head takes CUDA tensors")
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise ValueError("hidden [n, H] and weight [V, H] must share H")
    if hidden.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("hidden and weight rows must be contiguous")


def head_logits(device: Device, hidden, weight, out_logits, stream: Optional[int] = None) -> None:
    """vw_head_logits: out_logits = hidden x weight^T (TalkerModel.CodecHead / CodePredictorHead, TalkerModel.cs:133-137)
    on the tensor cores.  CUDA tensors: hidden [n, H], weight [V, H] bf16 (or int16 / uint16 bits), out_logits a
    contiguous float32 [n, V]."""
    _head_operands(hidden, weight, out_logits)
    n, v = int(hidden.shape[0]), int(weight.shape[0])
    if tuple(out_logits.shape) != (n, v) or not out_logits.is_contiguous() or str(out_logits.dtype) != "torch.float32":
        raise ValueError("out_logits must be a contiguous float32 [n, V] tensor")
    check(lib.vw_head_logits(device.handle, ctypes.c_void_p(hidden.data_ptr()), int(hidden.stride(0)),
                             int(hidden.shape[1]), ctypes.c_void_p(weight.data_ptr()), int(weight.stride(0)), n, v,
                             ctypes.c_void_p(out_logits.data_ptr()), ctypes.c_void_p(stream) if stream else None),
          device.handle)


def head_sample(device: Device, hidden, weight, segment: Segment, options: Sequence[VwOptions], out_logits=None,
                stream: Optional[int] = None) -> None:
    """vw_head_sample: logits = hidden x weight^T on the tensor cores (TalkerModel.CodecHead / CodePredictorHead,
    TalkerModel.cs:133-137), then the sampler over them; ids land in ``segment.out_ids``.

    CUDA tensors: hidden [n, H] and weight [V, H] bf16 (or raw int16 / uint16 bf16 bits), H a multiple of 8, V a
    multiple of 4; ``segment`` carries the rows' histories, steps, options, uniforms and outputs (its ``logits`` is
    ignored and may be None); ``out_logits`` [n, V] float32 optionally receives the GEMM's logits.
    """
    _head_operands(hidden, weight, out_logits)
    n, v = int(hidden.shape[0]), int(weight.shape[0])
    if out_logits is not None and (tuple(out_logits.shape) != (n, v) or not out_logits.is_contiguous()
                                   or str(out_logits.dtype) != "torch.float32"):
        raise ValueError("out_logits must be a contiguous float32 [n, V] tensor")
    seg = segment.to_c(VW_MEM_DEVICE, shape=(n, v))
    opts = (VwOptions * len(options))(*options)
    check(lib.vw_head_sample(device.handle, ctypes.c_void_p(hidden.data_ptr()), int(hidden.stride(0)),
                             int(hidden.shape[1]), ctypes.c_void_p(weight.data_ptr()), int(weight.stride(0)),
                             ctypes.byref(seg), opts, len(options),
                             ctypes.c_void_p(out_logits.data_ptr()) if out_logits is not None else None,
                             ctypes.c_void_p(stream) if stream else None), device.handle)
