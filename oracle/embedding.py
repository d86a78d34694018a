"""CPU restatement of voxwerk's next-talker-input gather -- TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module, as the checker of vw_frame_embedding.  Restated from
src/Voxwerk/Talker/TalkerModel.cs:114-118 (FrameEmbedding: CodecEmbedding of codes[0] written, then
CodePredictorEmbedding of codes[g] added for g = 1..15, each through AddRow :120-130 and Bf16.ToFloat, Bf16.cs:13)
and src/Voxwerk/Talker/TalkerGenerator.cs:437-438 (st[d] += text[off + d]).  Every addition is one float32 rounding,
in that order; NumPy float32 addition rounds the same way, element by element.
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Bf16.ToFloat (Bf16.cs:13): the 16 bits become the high half of an fp32."""
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def frame_embedding(codes: np.ndarray, codec_embedding: np.ndarray, cp_embeddings: Sequence[np.ndarray],
                    text: Optional[np.ndarray]) -> np.ndarray:
    """[n, hidden] fp32 next inputs for codes [n, G]; rows with codes[r, 0] == -1 come back as NaN (not written)."""
    n, groups = codes.shape
    hidden = codec_embedding.shape[1]
    out = np.full((n, hidden), np.nan, dtype=np.float32)
    for r in range(n):
        if codes[r, 0] == -1:
            continue
        acc = bf16_to_f32(codec_embedding[codes[r, 0]])                 # CodecEmbedding(code0, dst, add: false)
        for g in range(1, groups):                                      # CodePredictorEmbedding(g, codes[g], add)
            acc = (acc + bf16_to_f32(cp_embeddings[g - 1][codes[r, g]])).astype(np.float32)
        if text is not None:
            acc = (acc + text[r].astype(np.float32)).astype(np.float32)  # st[d] += text[off + d]
        out[r] = acc
    return out
