"""voxwerk_b200: B200 (sm_100a) token sampler for voxwerk's Qwen3-TTS generation loop.

The compute path is libvwsampler.so (CUDA, C ABI in include/vwsampler.h); this package is its host-side mirror of
voxwerk's ``SamplingOptions`` / ``GenerationOptions`` / ``Sampler`` interface (src/Voxwerk/Talker/Sampler.cs,
TalkerGenerator.cs).  Importing it loads the shared library and fails if it is missing.
"""

from ._lib import (VW_BF16, VW_F32, VW_MEM_DEVICE, VW_MEM_HOST, VW_ROWS_SUB, VW_ROWS_TALKER, VwError,
                   VwInvalidArgument, VwOutOfRange)
from .sampler import (CODEC_EOS_ID, CP_VOCAB_SIZE, MIN_NEW_TOKENS, NUM_CODE_GROUPS, VOCAB_SIZE, Device,
                      DotNetRandom, GenerationOptions, Sampler, SamplingOptions, Segment, TalkerBatchSampler,
                      sample_rows, sample_rows_static, vw_options)

__all__ = [
    "VW_BF16", "VW_F32", "VW_MEM_DEVICE", "VW_MEM_HOST", "VW_ROWS_SUB", "VW_ROWS_TALKER", "VwError",
    "VwInvalidArgument", "VwOutOfRange", "CODEC_EOS_ID", "CP_VOCAB_SIZE", "MIN_NEW_TOKENS", "NUM_CODE_GROUPS",
    "VOCAB_SIZE", "Device", "DotNetRandom", "GenerationOptions", "Sampler", "SamplingOptions", "Segment",
    "TalkerBatchSampler", "sample_rows", "sample_rows_static", "vw_options",
]
