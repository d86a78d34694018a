"""vw_frame_embedding (the next talker input: FrameEmbedding + text row) against the CPU restatement, bit for bit."""

import numpy as np
import pytest

from oracle.embedding import frame_embedding as ref_frame_embedding

pytestmark = pytest.mark.gpu


def _tables(rng, V=3072, CV=2048, H=1024, groups=16):
    f = lambda shape: (rng.normal(0, 0.05, shape).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return f((V, H)), [f((CV, H)) for _ in range(groups - 1)]


def _run(device, codes, codec, cps, text):
    import torch
    from voxwerk_b200 import frame_embedding
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = torch.full((codes.shape[0], codec.shape[1]), float("nan"), dtype=torch.float32, device="cuda")
    frame_embedding(device, t(codes), t(codec.view(np.int16)), [t(c.view(np.int16)) for c in cps],
                    None if text is None else t(text), out)
    return out.cpu().numpy()


@pytest.mark.parametrize("with_text", [True, False])
def test_frame_embedding_bit_exact(device, with_text):
    rng = np.random.default_rng(11)
    codec, cps = _tables(rng)
    n = 257
    codes = np.concatenate([rng.integers(0, 3072, (n, 1)), rng.integers(0, 2048, (n, 15))], axis=1).astype(np.int32)
    codes[5, 0] = -1     # a finished sequence: its row is left alone
    text = rng.normal(0, 1, (n, 1024)).astype(np.float32) if with_text else None
    got = _run(device, codes, codec, cps, text)
    ref = ref_frame_embedding(codes, codec, cps, text)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_frame_embedding_rejects_out_of_range_codes(device):
    from voxwerk_b200 import VwOutOfRange
    rng = np.random.default_rng(12)
    codec, cps = _tables(rng, H=64)
    codes = np.zeros((4, 16), np.int32)
    codes[2, 7] = 2048
    with pytest.raises(VwOutOfRange):
        _run(device, codes, codec, cps, None)
    codes[2, 7] = 3
    got = _run(device, codes, codec, cps, None)   # the handle is usable afterwards
    np.testing.assert_array_equal(got.view(np.uint32), ref_frame_embedding(codes, codec, cps, None).view(np.uint32))
