"""The DiT step engine (aex_dit_* through the C ABI) against the oracle's
composition of the reference wiring (oracle/dit_ref.py) on a small config of the
same architecture (hidden 256 = 2 heads x 128, 1 double + 2 single blocks, mlp
768, l_txt 32, l_img 64): one transformer pass, the Euler step and a 4-step
denoise. The RoPE tables both sides use are the oracle's (O.rope_freqs of the
reference's text ids [0,0,0,i] and image ids [0,h,w,0]), so a table error in
the library cannot cancel out (aex_rope_tables has its own test). Tolerance:
relative L2 <= 2e-2 on the velocity / latents (bf16 activations through 3
blocks of random 4-bit weights). The drift of the 4-step latents from an
all-f32 composition (no bf16 storage point) is printed, not asserted."""
import numpy as np
import pytest
import torch

from aestrix_b200 import dit
from oracle import oracle as O
from oracle.dit_ref import DitRef

pytestmark = pytest.mark.gpu

CFG = dit.DitConfig(hidden=256, heads=2, n_double=1, n_single=2, mlp_hidden=768, in_channels=128, text_dim=384,
                    timestep_dim=256, l_txt=32, l_img=64)


def _np(t):
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def setup(cuda_ctx):
    lin, norms = dit.random_weights(CFG, seed=2024)
    eng = dit.DitEngine(CFG, ctx=cuda_ctx)
    eng.load(lin, norms)
    side = int(round(CFG.l_img ** 0.5))
    cos_np, sin_np = O.rope_freqs(np.concatenate([O.text_ids(CFG.l_txt), O.grid_ids(side, side)], 0), 2000.0)
    cos, sin = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()
    g = torch.Generator().manual_seed(7)
    embeds = torch.randn(CFG.l_txt, CFG.text_dim, generator=g).to(torch.bfloat16).cuda()
    lat = torch.randn(CFG.l_img, CFG.in_channels, generator=g).cuda()
    eng.set_rope(cos, sin)
    eng.project_context(embeds)
    ref = DitRef(CFG, {k: tuple(_np(t) for t in v) for k, v in lin.items()}, {k: _np(v) for k, v in norms.items()})
    e0 = ref.project_context(O.bf16_to_f32(_np(embeds)))
    return eng, ref, lat, e0, cos_np, sin_np, O.bf16_to_f32(_np(embeds))


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_forward_matches_oracle(setup):
    eng, ref, lat, e0, cos, sin, emb = setup
    t = 1000.0 * float(O.schedule(4, CFG.l_img)[0][0])
    eng.set_timestep(t)
    v = eng.forward(lat)
    torch.cuda.synchronize()
    vr = ref.forward(_np(lat), e0, cos, sin, ref.conditioning(t))
    got = _np(v)
    assert np.isfinite(got).all()
    rel = _rel(got, vr)
    assert rel <= 2e-2, f"velocity rel-L2 {rel:.3e}"


def test_denoise_step_and_full_denoise(setup):
    eng, ref, lat, e0, cos, sin, emb = setup
    sig, ts = O.schedule(4, CFG.l_img)
    # one Euler step through the engine == forward + Euler on the host
    eng.set_timestep(float(ts[0]))
    out = torch.empty_like(lat)
    eng.denoise_step(lat, out, float(sig[1] - sig[0]))
    v = eng.forward(lat)
    torch.cuda.synchronize()
    assert np.allclose(_np(out), _np(lat) + (sig[1] - sig[0]) * _np(v), rtol=1e-5, atol=1e-5)
    # the full 4-step denoise vs the oracle loop
    x = lat.clone()
    eng.denoise(x, steps=4)
    torch.cuda.synchronize()
    xr = _np(lat).copy()
    for i in range(4):
        vr = ref.forward(xr, e0, cos, sin, ref.conditioning(float(ts[i])))
        xr = xr + (sig[i + 1] - sig[i]) * vr
    rel = _rel(_np(x), xr)
    assert rel <= 2e-2, f"4-step latents rel-L2 {rel:.3e}"
    assert eng.ctx.device_status() == 0
    # drift from the all-f32 composition (same weights, no activation rounded to bf16)
    r32 = DitRef(CFG, ref.lin, ref.norms, storage="f32")
    e32 = r32.project_context(emb)
    x32 = _np(lat).copy()
    for i in range(4):
        x32 = x32 + (sig[i + 1] - sig[i]) * r32.forward(x32, e32, cos, sin, r32.conditioning(float(ts[i])))
    print(f"4-step latents rel-L2: engine vs bf16-storage oracle {rel:.3e}, engine vs all-f32 oracle "
          f"{_rel(_np(x), x32):.3e}, bf16-storage oracle vs all-f32 oracle {_rel(xr, x32):.3e}")


def test_missing_weight_is_reported(cuda_ctx):
    eng = dit.DitEngine(CFG, ctx=cuda_ctx)
    cos, sin = dit.rope_tables(CFG)
    eng.set_rope(cos, sin)
    with pytest.raises(Exception) as e:
        eng.project_context(torch.zeros(CFG.l_txt, CFG.text_dim, dtype=torch.bfloat16, device="cuda"))
    assert "context_embedder" in str(e.value)


def _eager_denoise(eng, lat, steps):
    """The denoise loop issued step by step (set_timestep + denoise_step), no graph."""
    sig, ts = O.schedule(steps, CFG.l_img)
    cur, alt = lat.clone(), torch.empty_like(lat)
    for i in range(steps):
        eng.set_timestep(float(ts[i]))
        eng.denoise_step(cur, alt, float(sig[i + 1] - sig[i]))
        cur, alt = alt, cur
    return cur


def test_graph_replay_matches_eager_and_tracks_weight_reloads(setup, cuda_ctx):
    """aex_dit_denoise replays one captured step per iteration: twice in a row and
    against the same loop launched kernel by kernel it must agree bit for bit; after
    a weight is re-loaded the captured step is rebuilt and still agrees."""
    eng, ref, lat, e0, cos, sin, emb = setup
    a = eng.denoise(lat.clone(), steps=3)
    b = eng.denoise(lat.clone(), steps=3)
    e = _eager_denoise(eng, lat, 3)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, e)
    lin, _ = dit.random_weights(CFG, seed=99)
    name = "single_transformer_blocks.1.attn.to_out"
    eng.load_linear(name, *lin[name])
    c = eng.denoise(lat.clone(), steps=3)
    e2 = _eager_denoise(eng, lat, 3)
    torch.cuda.synchronize()
    assert not torch.equal(c, a)
    assert torch.equal(c, e2)
    assert cuda_ctx.device_status() == 0
