"""aex_dit_load_safetensors on the GPU: the small DiT config's random 4-bit
weights written as MLX-style safetensors shards (U32 packed weights, bf16
scales/biases, f32 norm weights, index.json) and loaded back give a forward
pass identical bit for bit to the same weights loaded tensor by tensor; F16
scales/biases holding bf16-exact values load identically; unexpected or
incomplete tensors are reported by name."""
import json

import pytest
import torch
from safetensors.torch import save_file

from aestrix_b200 import _lib, dit

pytestmark = pytest.mark.gpu

CFG = dit.DitConfig(hidden=256, heads=2, n_double=1, n_single=2, mlp_hidden=768, in_channels=128, text_dim=384,
                    timestep_dim=256, l_txt=32, l_img=64)


def _cpu_tensors(lin, norms, scale_dtype=torch.bfloat16):
    out = {}
    for name, (p, s, b) in lin.items():
        out[name + ".weight"] = p.cpu().view(torch.uint32)
        out[name + ".scales"] = s.cpu().to(scale_dtype)
        out[name + ".biases"] = b.cpu().to(scale_dtype)
    for name, w in norms.items():
        out[name + ".weight"] = w.cpu().to(torch.bfloat16)  # bf16 on disk like the hub packs
    return out


def _write_shards(tmp_path, tensors):
    keys = sorted(tensors)
    half = len(keys) // 2
    shards = {"model-00001-of-00002.safetensors": keys[:half], "model-00002-of-00002.safetensors": keys[half:]}
    wm = {}
    for fname, ks in shards.items():
        save_file({k: tensors[k].contiguous() for k in ks}, str(tmp_path / fname))
        wm.update({k: fname for k in ks})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    return tmp_path


def _run(eng, lat, embeds):
    cos, sin = dit.rope_tables(CFG)
    eng.set_rope(cos, sin)
    eng.project_context(embeds)
    eng.set_timestep(900.0)
    v = eng.forward(lat)
    torch.cuda.synchronize()
    return v


@pytest.fixture(scope="module")
def weights():
    lin, norms = dit.random_weights(CFG, seed=31)
    norms = {k: v.to(torch.bfloat16).float() for k, v in norms.items()}  # bf16-exact, as written
    g = torch.Generator().manual_seed(3)
    lat = torch.randn(CFG.l_img, CFG.in_channels, generator=g).cuda()
    embeds = torch.randn(CFG.l_txt, CFG.text_dim, generator=g).to(torch.bfloat16).cuda()
    return lin, norms, lat, embeds


@pytest.mark.parametrize("scale_dtype", [torch.bfloat16, torch.float16])
def test_safetensors_load_matches_direct_load(tmp_path, cuda_ctx, weights, scale_dtype):
    lin, norms, lat, embeds = weights
    if scale_dtype == torch.float16:
        # Keep |scale|, |bias| inside f16's normal range, where bf16 -> f16 -> bf16 is exact.
        def normal(t):
            return (t.float().sign() * t.float().abs().clamp(min=2.0 ** -10)).to(torch.bfloat16)
        lin = {k: (p, normal(s), normal(b)) for k, (p, s, b) in lin.items()}
    ref = dit.DitEngine(CFG, ctx=cuda_ctx)
    ref.load(lin, norms)
    v_ref = _run(ref, lat, embeds)
    d = _write_shards(tmp_path, _cpu_tensors(lin, norms, scale_dtype))
    eng = dit.DitEngine(CFG, ctx=cuda_ctx)
    nl, nn = eng.load_safetensors(d)
    assert (nl, nn) == (len(lin), len(norms))
    v = _run(eng, lat, embeds)
    assert torch.equal(v, v_ref)
    assert cuda_ctx.device_status() == 0


def test_safetensors_reports_bad_tensors(tmp_path, cuda_ctx, weights):
    lin, norms, _, _ = weights
    t = _cpu_tensors(lin, norms)
    t["transformer_blocks.0.attn.extra_bias"] = torch.zeros(256)
    f = tmp_path / "a.safetensors"
    save_file(t, str(f))
    eng = dit.DitEngine(CFG, ctx=cuda_ctx)
    with pytest.raises(_lib.AexError) as e:
        eng.load_safetensors(f)
    assert "transformer_blocks.0.attn.extra_bias" in str(e.value)
    t.pop("transformer_blocks.0.attn.extra_bias")
    t.pop("proj_out.biases")
    f2 = tmp_path / "b.safetensors"
    save_file(t, str(f2))
    with pytest.raises(_lib.AexError) as e:
        eng.load_safetensors(f2)
    assert "proj_out" in str(e.value)
