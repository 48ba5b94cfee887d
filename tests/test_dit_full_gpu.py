"""The DiT step engine at the real FLUX.2-klein widths against the oracle's
composition of the reference wiring (oracle/dit_ref.py): hidden 3072, 24 heads,
5 double + 20 single blocks, mlp 9216, text_dim 7680, timestep_dim 256
(DirectDiTStep.swift:308-335, 546-618), on a short joint sequence (32 text +
16x16 image tokens) so the CPU oracle finishes in about a minute. Every GEMM
shape of the real model runs here: the K = 12288 single-block to_out, the
K = 9216 feed-forward down projections, the N = 27648 single-block projection
(gate/up interleaved), the fused per-stream Q|K|V with the 24-head norm + RoPE
epilogue and the text/image norm switch, the K = 7680 context embedder, the
128 -> 3072 x_embedder and the 3072 -> 128 proj_out, and the f32 conditioning
GEMVs (one grouped launch of the four modulation heads).
Random-init 4-bit weights (codes U{0..15}, scales |N(0, 0.02)|, biases N(0, 0.02)),
RoPE tables from the oracle. Tolerance: relative L2 <= 2e-2 on the velocity."""
import numpy as np
import pytest
import torch

from aestrix_b200 import dit
from oracle import oracle as O
from oracle.dit_ref import DitRef

pytestmark = pytest.mark.gpu

CFG = dit.DitConfig(l_txt=32, l_img=256)  # Klein widths, short sequence


def _np(t):
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


def test_full_width_forward_matches_oracle(cuda_ctx):
    lin, norms = dit.random_weights(CFG, seed=31)
    eng = dit.DitEngine(CFG, ctx=cuda_ctx)
    eng.load(lin, norms)
    cos, sin = O.rope_freqs(np.concatenate([O.text_ids(CFG.l_txt), O.grid_ids(16, 16)], 0), 2000.0)
    g = torch.Generator().manual_seed(8)
    embeds = torch.randn(CFG.l_txt, CFG.text_dim, generator=g).to(torch.bfloat16)
    lat = torch.randn(CFG.l_img, CFG.in_channels, generator=g)
    t = 1000.0 * float(O.schedule(4, CFG.l_img)[0][1])
    eng.set_rope(torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
    eng.project_context(embeds.cuda())
    eng.set_timestep(t)
    v = eng.forward(lat.cuda())
    torch.cuda.synchronize()
    got = _np(v)
    assert cuda_ctx.device_status() == 0
    eng.close()
    ref = DitRef(CFG, {k: tuple(_np(a) for a in w) for k, w in lin.items()}, {k: _np(w) for k, w in norms.items()})
    del lin
    torch.cuda.empty_cache()
    e0 = ref.project_context(O.bf16_to_f32(_np(embeds)))
    vr = ref.forward(lat.numpy(), e0, cos, sin, ref.conditioning(t))
    assert np.isfinite(got).all() and np.isfinite(vr).all()
    rel = float(np.linalg.norm(got - vr) / np.linalg.norm(vr))
    print(f"full-width forward: velocity rel-L2 {rel:.3e}, |v| {np.linalg.norm(vr):.3e}")
    assert rel <= 2e-2, f"velocity rel-L2 {rel:.3e}"
