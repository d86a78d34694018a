"""Device-resident generation state for TalkerGenerator.GenerateBatch (src/Voxwerk/Talker/TalkerGenerator.cs:322-455).

``DeviceBatchState`` keeps every job's talker history, step counter, MaxNewTokens and its two samplers
(``Sampler(Seed)`` / ``Sampler(Seed + 1)``, :345-346) on the GPU, one slot per job, through the ``vw_batch_*`` C ABI.
A step then moves only logits in and ids out:

    state.start(slot, GenerationOptions(seed=...))           # slot refill, :336-358
    ids, done = state.talker_step(talker_logits)             # :366-385, history append and retirement :374-380
    for g in range(1, 16): state.sub_step(cp_logits[g])      # :416-420

or, with the vocabulary heads on the tensor cores and the frame kept on the device (hidden rows from the caller's
transformer steps):

    ids, done = state.talker_head_step(last_hidden, codec_head, codec_embedding, cp_input)   # :366-385, :411, :443
    for g in range(1, 16):
        state.sub_head_step(g, cp_hidden, cp_heads[g - 1], cp_embeddings[g - 1], cp_input)     # :418-422
    state.frame_embedding(codec_embedding, cp_embeddings, text, step_input)                # :428-439

Logits are CUDA tensors [n_slots, V] (row r belongs to slot r); ids and done flags come back as CUDA int32 tensors.
Finished slots are not sampled (id -1).  Each step's options table is built from the jobs' options, so slots with
different options share one call.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

from . import _lib
from ._lib import VW_BF16, VW_F32, VwEmbedOut, VwOptions, VwSlotConfig, check, lib
from .qwen3_tts import CODEC_EOS_ID, CP_VOCAB_SIZE, MIN_NEW_TOKENS, SUPPRESS_SPAN, VOCAB_SIZE
from .sampler import Device, GenerationOptions, vw_options


def _dtype(t) -> int:
    name = str(t.dtype)
    if "bfloat16" in name:
        return VW_BF16
    if name == "torch.float32":
        return VW_F32
    raise TypeError(f"logits must be float32 or bfloat16, got {name}")


class DeviceBatchState:
    """One vw_batch: up to `n_slots` concurrent jobs on `device`."""

    def __init__(self, device: Device, n_slots: int, max_history: int = 4096, vocab: int = VOCAB_SIZE,
                 cp_vocab: int = CP_VOCAB_SIZE, eos_id: int = CODEC_EOS_ID, min_new_tokens: int = MIN_NEW_TOKENS):
        import torch
        self.device, self.n_slots, self.vocab, self.cp_vocab = device, int(n_slots), int(vocab), int(cp_vocab)
        h = ctypes.c_void_p()
        check(lib.vw_batch_create(device.handle, self.n_slots, self.vocab, int(max_history), int(eos_id),
                                  int(min_new_tokens), self.vocab - SUPPRESS_SPAN, self.vocab, ctypes.byref(h)),
              device.handle)
        self._b = h
        self.jobs: List[Optional[GenerationOptions]] = [None] * self.n_slots
        self._talker_opts: List[VwOptions] = []
        self._sub_opts: List[VwOptions] = []
        self._talker_index, self._sub_index = {}, {}
        dev = torch.device("cuda", device.device)
        self.ids = torch.full((self.n_slots,), -1, dtype=torch.int32, device=dev)
        self.done = torch.zeros(self.n_slots, dtype=torch.int32, device=dev)
        self.sub_ids = torch.full((self.n_slots,), -1, dtype=torch.int32, device=dev)

    def close(self) -> None:
        if getattr(self, "_b", None) is not None:
            lib.vw_batch_destroy(self._b)
            self._b = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _option_index(self, table, index, key, opts, penalty) -> int:
        if key not in index:
            if len(table) >= 32:
                raise ValueError("at most 32 distinct option sets per batch")
            index[key] = len(table)
            table.append(vw_options(opts, penalty))
        return index[key]

    def start(self, slot: int, job: GenerationOptions, history: Sequence[int] = ()) -> None:
        """Starts `job` in `slot`: step 0, its samplers seeded from job.seed (Seed + 1 for the sub-talker)."""
        ti = self._option_index(self._talker_opts, self._talker_index, (job.talker, job.repetition_penalty),
                                job.talker, job.repetition_penalty)
        si = self._option_index(self._sub_opts, self._sub_index, (job.sub_talker,), job.sub_talker, 1.0)
        cfg = VwSlotConfig(ti, si, int(job.max_new_tokens), int(job.seed or 0), 0 if job.seed is None else 1)
        h = (ctypes.c_int32 * max(len(history), 1))(*history)
        check(lib.vw_batch_start(self._b, int(slot), ctypes.byref(cfg), h, len(history)), self.device.handle)
        self.jobs[slot] = job

    def stop(self, slot: int) -> None:
        check(lib.vw_batch_stop(self._b, int(slot)), self.device.handle)

    def talker_step(self, logits, stream: Optional[int] = None):
        """Codebook-0 ids of every running slot; (ids, done) as CUDA int32 tensors (id -1 for idle slots)."""
        if tuple(logits.shape[:1]) != (self.n_slots,) or not logits.is_cuda:
            raise ValueError("logits must be a CUDA tensor [n_slots, V]")
        opts = (VwOptions * len(self._talker_opts))(*self._talker_opts)
        check(lib.vw_batch_talker_step(self._b, ctypes.c_void_p(logits.data_ptr()), int(logits.stride(0)),
                                       _dtype(logits), opts, len(self._talker_opts),
                                       ctypes.c_void_p(self.ids.data_ptr()), ctypes.c_void_p(self.done.data_ptr()),
                                       ctypes.c_void_p(stream) if stream else None), self.device.handle)
        return self.ids, self.done

    def sub_step(self, cp_logits, stream: Optional[int] = None):
        """One code-predictor group's ids for every running slot (CUDA int32 tensor, -1 for idle slots)."""
        if tuple(cp_logits.shape[:1]) != (self.n_slots,) or not cp_logits.is_cuda:
            raise ValueError("cp_logits must be a CUDA tensor [n_slots, CV]")
        opts = (VwOptions * len(self._sub_opts))(*self._sub_opts)
        check(lib.vw_batch_sub_step(self._b, ctypes.c_void_p(cp_logits.data_ptr()), int(cp_logits.stride(0)),
                                    int(cp_logits.shape[1]), _dtype(cp_logits), opts, len(self._sub_opts),
                                    ctypes.c_void_p(self.sub_ids.data_ptr()),
                                    ctypes.c_void_p(stream) if stream else None), self.device.handle)
        return self.sub_ids

    # ---- the frame loop around the caller's transformer steps (vw_batch_*_head_step, include/vwsampler.h)
    def _head(self, hidden, weight):
        for t in (hidden, weight):
            if not t.is_cuda or t.dim() != 2 or t.stride(1) != 1:
                raise ValueError("hidden and weight must be 2-D CUDA tensors with contiguous rows")
        if hidden.shape[0] != self.n_slots or hidden.shape[1] != weight.shape[1]:
            raise ValueError("hidden must be [n_slots, H] and weight [V, H]")
        return (ctypes.c_void_p(hidden.data_ptr()), int(hidden.stride(0)), int(hidden.shape[1]),
                ctypes.c_void_p(weight.data_ptr()), int(weight.stride(0)))

    @staticmethod
    def _embed(table, out):
        if table is None:
            return None
        return ctypes.byref(VwEmbedOut(table.data_ptr(), int(table.shape[0]), int(table.shape[1]), out.data_ptr(),
                                       int(out.stride(0))))

    def talker_head_step(self, hidden, weight, embed_table=None, embed_out=None, stream: Optional[int] = None):
        """Codebook 0 from the talker's last hidden rows: logits = hidden x weight^T (CodecHead,
        TalkerGenerator.cs:443) on the tensor cores, then talker_step over them; (ids, done).  With embed_table (the
        codec embedding) each continuing slot's CodecEmbedding(code0) row also goes to embed_out (:411)."""
        opts = (VwOptions * len(self._talker_opts))(*self._talker_opts)
        check(lib.vw_batch_talker_head_step(self._b, *self._head(hidden, weight), opts, len(self._talker_opts),
                                            ctypes.c_void_p(self.ids.data_ptr()),
                                            ctypes.c_void_p(self.done.data_ptr()), self._embed(embed_table, embed_out),
                                            ctypes.c_void_p(stream) if stream else None), self.device.handle)
        return self.ids, self.done

    def sub_head_step(self, group: int, hidden, weight, embed_table=None, embed_out=None,
                      stream: Optional[int] = None):
        """Codebook `group` (1..15): CodePredictorHead(group) then SubSampler.Select (TalkerGenerator.cs:418-420);
        the ids are also recorded in the batch's frame (codes()).  With embed_table (code-predictor embedding
        group - 1) each continuing slot's CodePredictorEmbedding(group, code) row also goes to embed_out (:422)."""
        opts = (VwOptions * len(self._sub_opts))(*self._sub_opts)
        check(lib.vw_batch_sub_head_step(self._b, int(group), *self._head(hidden, weight), int(weight.shape[0]),
                                         opts, len(self._sub_opts), ctypes.c_void_p(self.sub_ids.data_ptr()),
                                         self._embed(embed_table, embed_out),
                                         ctypes.c_void_p(stream) if stream else None), self.device.handle)
        return self.sub_ids

    def code_embedding(self, group: int, table, out, stream: Optional[int] = None) -> None:
        """out[s] = table[codes[s][group]] widened to fp32 for every slot whose frame goes on (CodecEmbedding for
        group 0, CodePredictorEmbedding for 1..15: TalkerGenerator.cs:411, :422).  table [rows, H] bf16 (or int16
        bits), out [n_slots, H'] float32 with H' >= H."""
        check(lib.vw_batch_code_embedding(self._b, int(group), ctypes.c_void_p(table.data_ptr()), int(table.shape[0]),
                                          int(table.shape[1]), ctypes.c_void_p(out.data_ptr()), int(out.stride(0)),
                                          ctypes.c_void_p(stream) if stream else None), self.device.handle)

    def frame_embedding(self, codec_embedding, cp_embeddings, text, out, stream: Optional[int] = None) -> None:
        """FrameEmbedding(frame) + text of every continuing slot (TalkerGenerator.cs:428-439) from the batch's frame."""
        ptrs = (ctypes.c_void_p * len(cp_embeddings))(*[t.data_ptr() for t in cp_embeddings])
        check(lib.vw_batch_frame_embedding(self._b, int(codec_embedding.shape[1]),
                                           ctypes.c_void_p(codec_embedding.data_ptr()), ptrs,
                                           int(cp_embeddings[0].shape[0]),
                                           ctypes.c_void_p(text.data_ptr()) if text is not None else None,
                                           ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream) if stream else None),
              self.device.handle)

    def codes(self):
        """The frame being built, [n_slots, 16] int32 on the host (-1: not sampled / slot not continuing)."""
        import numpy as np
        out = np.empty((self.n_slots, 16), dtype=np.int32)
        check(lib.vw_batch_get_codes(self._b, out.ctypes.data), self.device.handle)
        return out

    def query(self, slot: int):
        """(step, history length, running) of `slot`."""
        v = [ctypes.c_int32() for _ in range(3)]
        check(lib.vw_batch_query(self._b, int(slot), *[ctypes.byref(x) for x in v]), self.device.handle)
        return v[0].value, v[1].value, bool(v[2].value)
