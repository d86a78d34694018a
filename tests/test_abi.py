"""The C ABI (include/vwsampler.h) without a GPU: the library loads, exports every declared symbol, its
struct layouts match the header as compiled by the host C compiler, and argument errors come back as status
codes (no compute call)."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from voxwerk_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vwsampler.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vw_[a-z_]+)\s*\(", text)))


def test_header_declares_exactly_the_bound_symbols():
    assert declared_functions() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_library_exports_nothing_else_named_vw():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    names = {ln.split()[-1] for ln in out.stdout.splitlines() if ln.split() and ln.split()[-1].startswith("vw_")}
    assert names == set(declared_functions())


def _c_layout():
    src = r'''
#include <stddef.h>
#include <stdio.h>
#include "vwsampler.h"
#define F(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("vw_options %zu\n", sizeof(vw_options));
  printf("vw_segment %zu\n", sizeof(vw_segment));
  printf("vw_stats %zu\n", sizeof(vw_stats));
  F(vw_options, do_sample) F(vw_options, top_k) F(vw_options, top_p) F(vw_options, temperature)
  F(vw_options, repetition_penalty)
  F(vw_segment, logits) F(vw_segment, row_stride) F(vw_segment, n_rows) F(vw_segment, vocab) F(vw_segment, dtype)
  F(vw_segment, kind) F(vw_segment, hist_offsets) F(vw_segment, hist_ids) F(vw_segment, steps)
  F(vw_segment, suppress_lo) F(vw_segment, suppress_hi) F(vw_segment, eos_id) F(vw_segment, min_new_tokens)
  F(vw_segment, max_hist_len) F(vw_segment, opt_index) F(vw_segment, uniforms) F(vw_segment, out_ids)
  F(vw_segment, out_probs)
  printf("vw_slot_config %zu\n", sizeof(vw_slot_config));
  F(vw_slot_config, talker_option) F(vw_slot_config, sub_option) F(vw_slot_config, max_new_tokens)
  F(vw_slot_config, seed) F(vw_slot_config, seeded)
  printf("vw_embed_out %zu\n", sizeof(vw_embed_out));
  F(vw_embed_out, table) F(vw_embed_out, table_rows) F(vw_embed_out, hidden) F(vw_embed_out, out)
  F(vw_embed_out, out_stride)
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    return dict((k, int(v)) for k, v in (ln.split() for ln in out.splitlines()))


def test_ctypes_structs_match_c_layout():
    lay = _c_layout()
    assert lay["vw_options"] == ctypes.sizeof(_lib.VwOptions)
    assert lay["vw_segment"] == ctypes.sizeof(_lib.VwSegment)
    assert lay["vw_stats"] == ctypes.sizeof(_lib.VwStats)
    assert lay["vw_slot_config"] == ctypes.sizeof(_lib.VwSlotConfig)
    assert lay["vw_embed_out"] == ctypes.sizeof(_lib.VwEmbedOut)
    for cls, cname in ((_lib.VwOptions, "vw_options"), (_lib.VwSegment, "vw_segment"),
                       (_lib.VwSlotConfig, "vw_slot_config"), (_lib.VwEmbedOut, "vw_embed_out")):
        for fname, _ in cls._fields_:
            key = "eos_id" if fname == "eos_id" else fname
            assert getattr(cls, fname).offset == lay[f"{cname}.{key}"], (cname, fname)


def test_status_strings_and_version():
    assert _lib.lib.vw_version().startswith(b"vwsampler")
    assert _lib.lib.vw_status_string(0) == b"ok"
    assert _lib.lib.vw_status_string(2) == b"history id out of range"


def test_null_handle_is_invalid_argument():
    L = _lib.lib
    assert L.vw_sample(None, None, 0, None, 0, 0, None) == _lib.VW_ERR_INVALID_ARG
    assert L.vw_synchronize(None, None) == _lib.VW_ERR_INVALID_ARG
    assert L.vw_destroy(None) == _lib.VW_OK
    assert L.vw_last_error(None) == b""
    assert L.vw_batch_destroy(None) == _lib.VW_OK
    assert L.vw_batch_start(None, 0, None, None, 0) == _lib.VW_ERR_INVALID_ARG
    assert L.vw_batch_talker_step(None, None, 0, 0, None, 0, None, None, None) == _lib.VW_ERR_INVALID_ARG
    out = ctypes.c_int32()
    assert L.vw_argmax(None, None, 1, 0, ctypes.byref(out)) == _lib.VW_ERR_INVALID_ARG


def test_create_without_device_reports_no_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    h = ctypes.c_void_p()
    assert _lib.lib.vw_create(0, ctypes.byref(h)) == _lib.VW_ERR_NO_DEVICE
    assert _lib.lib.vw_create(-1, ctypes.byref(h)) == _lib.VW_ERR_NO_DEVICE
    assert _lib.lib.vw_create(0, None) == _lib.VW_ERR_INVALID_ARG


def test_check_maps_status_to_exceptions():
    with pytest.raises(_lib.VwInvalidArgument):
        _lib.check(_lib.VW_ERR_INVALID_ARG)
    with pytest.raises(_lib.VwOutOfRange):
        _lib.check(_lib.VW_ERR_OUT_OF_RANGE)
    with pytest.raises(_lib.VwError):
        _lib.check(_lib.VW_ERR_TIMEOUT)
