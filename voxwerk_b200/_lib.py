"""ctypes binding of libvwsampler.so (the C ABI declared in include/vwsampler.h).

The library is built in-tree (``voxwerk_b200/libvwsampler.so``, see ``voxwerk_b200/build.py``).  There is no
fallback: if the shared library is missing or fails to load, importing this module raises.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvwsampler.so")

VW_OK = 0
VW_ERR_INVALID_ARG = 1
VW_ERR_OUT_OF_RANGE = 2
VW_ERR_CUDA = 3
VW_ERR_TIMEOUT = 4
VW_ERR_NO_DEVICE = 5

VW_F32 = 0
VW_BF16 = 1
VW_ROWS_TALKER = 0
VW_ROWS_SUB = 1
VW_MEM_DEVICE = 0
VW_MEM_HOST = 1
VW_MAX_SEGMENTS = 8

# Every symbol include/vwsampler.h declares.
EXPORTED = (
    "vw_version",
    "vw_status_string",
    "vw_create",
    "vw_destroy",
    "vw_last_error",
    "vw_sample",
    "vw_synchronize",
    "vw_get_stats",
    "vw_apply_repetition_penalty",
    "vw_select",
    "vw_argmax",
    "vw_sample_static",
    "vw_exp_diagnostic",
    "vw_batch_create",
    "vw_batch_destroy",
    "vw_batch_start",
    "vw_batch_stop",
    "vw_batch_talker_step",
    "vw_batch_sub_step",
    "vw_batch_query",
    "vw_frame_embedding",
    "vw_head_logits",
    "vw_head_sample",
    "vw_batch_talker_head_step",
    "vw_batch_sub_head_step",
    "vw_batch_code_embedding",
    "vw_batch_frame_embedding",
    "vw_batch_get_codes",
)


class VwOptions(ctypes.Structure):
    """vw_options: SamplingOptions (Sampler.cs:4-13) + GenerationOptions.RepetitionPenalty."""

    _fields_ = [
        ("do_sample", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("top_p", ctypes.c_float),
        ("temperature", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
    ]


class VwSegment(ctypes.Structure):
    """vw_segment: a block of rows sharing vocabulary size, dtype and kind."""

    _fields_ = [
        ("logits", ctypes.c_void_p),
        ("row_stride", ctypes.c_int64),
        ("n_rows", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("kind", ctypes.c_int32),
        ("hist_offsets", ctypes.c_void_p),
        ("hist_ids", ctypes.c_void_p),
        ("steps", ctypes.c_void_p),
        ("suppress_lo", ctypes.c_int32),
        ("suppress_hi", ctypes.c_int32),
        ("eos_id", ctypes.c_int32),
        ("min_new_tokens", ctypes.c_int32),
        ("max_hist_len", ctypes.c_int32),
        ("opt_index", ctypes.c_void_p),
        ("uniforms", ctypes.c_void_p),
        ("out_ids", ctypes.c_void_p),
        ("out_probs", ctypes.c_void_p),
    ]


class VwSlotConfig(ctypes.Structure):
    """vw_slot_config: one job of a device-resident batch."""

    _fields_ = [
        ("talker_option", ctypes.c_int32),
        ("sub_option", ctypes.c_int32),
        ("max_new_tokens", ctypes.c_int32),
        ("seed", ctypes.c_int32),
        ("seeded", ctypes.c_int32),
    ]


class VwEmbedOut(ctypes.Structure):
    """vw_embed_out: the next input row a head step also gathers for each continuing slot."""

    _fields_ = [
        ("table", ctypes.c_void_p),
        ("table_rows", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("out_stride", ctypes.c_int64),
    ]


class VwStats(ctypes.Structure):
    """vw_stats: rows sampled per path."""

    _fields_ = [
        ("rows_greedy", ctypes.c_uint64),
        ("rows_fast", ctypes.c_uint64),
        ("rows_fast_replayed", ctypes.c_uint64),
        ("rows_general", ctypes.c_uint64),
        ("rows_general_replayed", ctypes.c_uint64),
        ("rows_large", ctypes.c_uint64),
        ("rows_overflow", ctypes.c_uint64),
        ("rows_threshold_miss", ctypes.c_uint64),
        ("h2d_bytes", ctypes.c_uint64),
    ]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class VwError(RuntimeError):
    """A non-zero vw_status.  `status` holds the code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


class VwInvalidArgument(VwError, ValueError):
    pass


class VwOutOfRange(VwError, IndexError):
    """A history id outside [0, V): the reference throws IndexOutOfRangeException at Sampler.cs:30."""


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(there is no CPU fallback)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    lib.vw_version.restype = ctypes.c_char_p
    lib.vw_version.argtypes = []
    lib.vw_status_string.restype = ctypes.c_char_p
    lib.vw_status_string.argtypes = [ctypes.c_int]
    lib.vw_create.restype = ctypes.c_int
    lib.vw_create.argtypes = [i32, ctypes.POINTER(vp)]
    lib.vw_destroy.restype = ctypes.c_int
    lib.vw_destroy.argtypes = [vp]
    lib.vw_last_error.restype = ctypes.c_char_p
    lib.vw_last_error.argtypes = [vp]
    lib.vw_sample.restype = ctypes.c_int
    lib.vw_sample.argtypes = [vp, ctypes.POINTER(VwSegment), i32, ctypes.POINTER(VwOptions), i32, i32, vp]
    lib.vw_synchronize.restype = ctypes.c_int
    lib.vw_synchronize.argtypes = [vp, vp]
    lib.vw_get_stats.restype = ctypes.c_int
    lib.vw_get_stats.argtypes = [vp, ctypes.POINTER(VwStats), i32]
    lib.vw_apply_repetition_penalty.restype = ctypes.c_int
    lib.vw_apply_repetition_penalty.argtypes = [vp, vp, i32, vp, i64, ctypes.c_float, i32]
    lib.vw_select.restype = ctypes.c_int
    lib.vw_select.argtypes = [vp, vp, i32, ctypes.POINTER(VwOptions), ctypes.c_double, i32,
                              ctypes.POINTER(i32)]
    lib.vw_argmax.restype = ctypes.c_int
    lib.vw_argmax.argtypes = [vp, vp, i32, i32, ctypes.POINTER(i32)]
    lib.vw_sample_static.restype = ctypes.c_int
    lib.vw_sample_static.argtypes = [i32, ctypes.POINTER(VwSegment), i32, ctypes.POINTER(VwOptions), i32, vp,
                                     ctypes.c_char_p, i32]
    lib.vw_exp_diagnostic.restype = ctypes.c_int
    lib.vw_exp_diagnostic.argtypes = [vp, vp, i64, vp, vp]
    for name, args in (("vw_batch_create", [vp, i32, i32, i32, i32, i32, i32, i32, ctypes.POINTER(vp)]),
                       ("vw_batch_destroy", [vp]),
                       ("vw_batch_start", [vp, i32, ctypes.POINTER(VwSlotConfig), vp, i32]),
                       ("vw_batch_stop", [vp, i32]),
                       ("vw_batch_talker_step", [vp, vp, i64, i32, ctypes.POINTER(VwOptions), i32, vp, vp, vp]),
                       ("vw_batch_sub_step", [vp, vp, i64, i32, i32, ctypes.POINTER(VwOptions), i32, vp, vp]),
                       ("vw_batch_query", [vp, i32, vp, vp, vp]),
                       ("vw_frame_embedding", [vp, vp, i32, i32, i32, vp, i32, vp, i32, vp, vp, vp]),
                       ("vw_head_logits", [vp, vp, i64, i32, vp, i64, i32, i32, vp, vp]),
                       ("vw_batch_talker_head_step", [vp, vp, i64, i32, vp, i64, ctypes.POINTER(VwOptions), i32, vp,
                                                      vp, ctypes.POINTER(VwEmbedOut), vp]),
                       ("vw_batch_sub_head_step", [vp, i32, vp, i64, i32, vp, i64, i32, ctypes.POINTER(VwOptions), i32,
                                                   vp, ctypes.POINTER(VwEmbedOut), vp]),
                       ("vw_batch_code_embedding", [vp, i32, vp, i32, i32, vp, i64, vp]),
                       ("vw_batch_frame_embedding", [vp, i32, vp, vp, i32, vp, vp, vp]),
                       ("vw_batch_get_codes", [vp, vp]),
                       ("vw_head_sample", [vp, vp, i64, i32, vp, i64, ctypes.POINTER(VwSegment),
                                           ctypes.POINTER(VwOptions), i32, vp, vp])):
        getattr(lib, name).restype = ctypes.c_int
        getattr(lib, name).argtypes = args
    return lib


lib = _load()


def check(status: int, handle=None) -> None:
    """Raises the exception matching a non-zero vw_status."""
    if status == VW_OK:
        return
    msg = ""
    if handle is not None:
        msg = (lib.vw_last_error(handle) or b"").decode()
    if not msg:
        msg = (lib.vw_status_string(status) or b"").decode()
    if status == VW_ERR_INVALID_ARG:
        raise VwInvalidArgument(status, msg)
    if status == VW_ERR_OUT_OF_RANGE:
        raise VwOutOfRange(status, msg)
    raise VwError(status, msg)
