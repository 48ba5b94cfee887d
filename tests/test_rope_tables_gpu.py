"""aex_rope_tables (the device rotary tables every DiT and sequence-parallel call
uses) against the oracle's restatement of Flux2PosEmbed / Flux2RoPE
(O.rope_freqs; Sources/ImarelloDiT/PosEmbed.swift:12-47,
Sources/ImarelloCore/Flux2RoPE.swift:16-95), itself pinned to the reference's
known answers (tests/test_oracle_golden.py), at the joint lengths the model runs:
1024^2 (512 text + 64x64 = 4608), the i2i sequence (512 text + 64x64 target +
64x64 reference ids with t = 10, LatentOps.swift:43-45 = 8704) and 2048^2
(512 text + 128x128 = 16896), with the reference's text ids [0,0,0,i] and with
all-zero text positions. Both sides compute the angle
pos * theta^(-2i/32) in f32; the libraries' powf/cosf/sinf may differ by an ulp
or two, and an angle of up to 511 rad carries that as ~1e-4 absolute, so the
bound is max-abs <= 3e-4 (and 1e-5 where every angle is below 2 rad)."""
import numpy as np
import pytest
import torch

from aestrix_b200 import attention
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _ids(kind, text_ids=True):
    txt = O.text_ids(512) if text_ids else np.zeros((512, 4), np.float32)
    if kind == "1024":
        img = O.grid_ids(64, 64)
    elif kind == "i2i":
        img = np.concatenate([O.grid_ids(64, 64), O.grid_ids(64, 64, 10.0)], 0)
    else:
        img = O.grid_ids(128, 128)
    return np.concatenate([txt, img], 0)


@pytest.mark.parametrize("kind,seq", [("1024", 4608), ("i2i", 8704), ("2048", 16896)])
@pytest.mark.parametrize("text_ids", [True, False])
def test_rope_tables_match_oracle(cuda_ctx, kind, seq, text_ids):
    ids = _ids(kind, text_ids)
    assert ids.shape == (seq, 4)
    cos_d, sin_d = attention.rope_tables(torch.from_numpy(ids).cuda(), 2000.0, ctx=cuda_ctx)
    torch.cuda.synchronize()
    cos_r, sin_r = O.rope_freqs(ids, 2000.0)
    cos_g, sin_g = cos_d.cpu().numpy(), sin_d.cpu().numpy()
    assert cos_g.shape == (seq, 64) and sin_g.shape == (seq, 64)
    err = max(np.abs(cos_g - cos_r).max(), np.abs(sin_g - sin_r).max())
    assert err <= 3e-4, f"max-abs {err:.3e}"
    # small angles (image rows of the 1024^2 grid: positions <= 63 times omega <= 1 on the h/w axes
    # only; the t axis is 0): the f32 functions agree to a few ulp
    small = np.abs(ids[:, None, :].repeat(16, 2).reshape(seq, 64)) <= 1.0
    if small.any():
        e2 = max(np.abs(cos_g - cos_r)[small].max(), np.abs(sin_g - sin_r)[small].max())
        assert e2 <= 1e-5, f"max-abs {e2:.3e} where |pos| <= 1"
    # the layout: axis a occupies columns [16a, 16a + 16); column 16a is omega = 1, angle = pos
    for a in range(4):
        np.testing.assert_allclose(cos_g[:, 16 * a], np.cos(ids[:, a].astype(np.float64)), atol=3e-4)
