"""voxwerk_b200: B200 (sm_100a) token sampler for voxwerk's Qwen3-TTS generation loop.

The compute path is libvwsampler.so (CUDA, C ABI in include/vwsampler.h); this package is its host-side mirror of
voxwerk's ``SamplingOptions`` / ``GenerationOptions`` / ``Sampler`` interface (src/Voxwerk/Talker/Sampler.cs,
TalkerGenerator.cs).

The shared library is loaded on first use of any name that needs it (``Device``, ``Sampler``, ``sample_rows`` ...):
that access raises ImportError when the library is missing, and there is no CPU fallback.  The pure-Python
submodules (``dotnet_random``, ``qwen3_tts``, ``workloads``, ``shard``) load no native code, so a process that only
generates inputs or shards a batch does not map the GPU library.
"""

from importlib import import_module

from .dotnet_random import DotNetRandom
from .qwen3_tts import CODEC_EOS_ID, CP_VOCAB_SIZE, MIN_NEW_TOKENS, NUM_CODE_GROUPS, VOCAB_SIZE

# name -> submodule that defines it; importing that submodule loads libvwsampler.so
_NATIVE = {
    **{n: "._lib" for n in ("VW_BF16", "VW_F32", "VW_MEM_DEVICE", "VW_MEM_HOST", "VW_ROWS_SUB", "VW_ROWS_TALKER",
                            "VwError", "VwInvalidArgument", "VwOutOfRange")},
    **{n: ".sampler" for n in ("Device", "GenerationOptions", "Sampler", "SamplingOptions", "Segment",
                               "TalkerBatchSampler", "frame_embedding", "head_logits", "head_sample", "sample_rows", "sample_rows_static",
                               "vw_options")},
    **{n: ".batch_state" for n in ("DeviceBatchState",)},
}


def __getattr__(name):
    mod = _NATIVE.get(name)
    if mod is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(import_module(mod, __name__), name)
    globals()[name] = value
    return value


__all__ = ["CODEC_EOS_ID", "CP_VOCAB_SIZE", "MIN_NEW_TOKENS", "NUM_CODE_GROUPS", "VOCAB_SIZE", "DotNetRandom",
           *_NATIVE]
