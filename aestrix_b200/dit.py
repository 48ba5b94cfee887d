"""FLUX.2-klein DiT step engine over libaestrix_cuda (ctypes binding used by the
tests and the benchmark).

Mirrors the reference direct engine's surface: ``DirectDiTStep`` (loadBlocks /
loadHead / setStepConditioning / encodeDenoiseStep,
Sources/ImarelloDirect/DirectDiTStep.swift), ``DirectConditioner`` (projectContext,
stepConditioning, DirectConditioner.swift) and ``DirectDiTPackedDenoiser.denoise``
(DirectDiTAdapter.swift:25-81). Weights are keyed by their MLX names.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import torch

from . import _lib, qmm


aex_dit_config = _lib.aex_dit_config


@dataclass
class DitConfig:
    hidden: int = 3072
    heads: int = 24
    n_double: int = 5
    n_single: int = 20
    mlp_hidden: int = 9216
    in_channels: int = 128
    text_dim: int = 7680
    timestep_dim: int = 256
    l_txt: int = 512
    l_img: int = 4096
    rms_eps: float = 1e-5
    ln_eps: float = 1e-6

    def c(self):
        return aex_dit_config(*(getattr(self, f[0]) for f in aex_dit_config._fields_))

    @property
    def seq(self):
        return self.l_txt + self.l_img


def linear_shapes(cfg: DitConfig) -> dict[str, tuple[int, int]]:
    """Every 4-bit linear of the model: MLX key -> (n, k) (DirectDiTStep.swift:308-335, 844-884;
    DirectConditioner.swift:75-82)."""
    Cd, mlp = cfg.hidden, cfg.mlp_hidden
    out = {
        "x_embedder": (Cd, cfg.in_channels), "proj_out": (cfg.in_channels, Cd),
        "context_embedder": (Cd, cfg.text_dim),
        "time_guidance_embed.linear_1": (Cd, cfg.timestep_dim), "time_guidance_embed.linear_2": (Cd, Cd),
        "double_stream_modulation_img.linear": (6 * Cd, Cd), "double_stream_modulation_txt.linear": (6 * Cd, Cd),
        "single_stream_modulation.linear": (3 * Cd, Cd), "norm_out.linear": (2 * Cd, Cd),
    }
    for i in range(cfg.n_double):
        p = f"transformer_blocks.{i}."
        for leaf in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out", "to_add_out"):
            out[p + "attn." + leaf] = (Cd, Cd)
        for ff in ("ff", "ff_context"):
            out[p + ff + ".linear_in"] = (2 * mlp, Cd)
            out[p + ff + ".linear_out"] = (Cd, mlp)
    for i in range(cfg.n_single):
        p = f"single_transformer_blocks.{i}.attn."
        out[p + "to_qkv_mlp_proj"] = (3 * Cd + 2 * mlp, Cd)
        out[p + "to_out"] = (Cd, Cd + mlp)
    return out


def norm_names(cfg: DitConfig) -> list[str]:
    names = []
    for i in range(cfg.n_double):
        names += [f"transformer_blocks.{i}.attn.{n}" for n in ("norm_q", "norm_k", "norm_added_q", "norm_added_k")]
    for i in range(cfg.n_single):
        names += [f"single_transformer_blocks.{i}.attn.{n}" for n in ("norm_q", "norm_k")]
    return names


def random_weights(cfg: DitConfig, seed: int, device="cuda"):
    """Random-init weights of the architecture in the MLX layout, generated on the device:
    codes U{0..15}, scales |N(0, 0.02)|, biases N(0, 0.02) (BASELINE configs[2]/[3]); RMSNorm
    weights 1 + 0.1 N(0, 1). Returns ({name: (packed int32, scales bf16, biases bf16)}, {name: f32})."""
    g = torch.Generator(device=device).manual_seed(seed)
    lin = {}
    for name, (n, k) in linear_shapes(cfg).items():
        packed = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=g, device=device, dtype=torch.int32)
        scales = (torch.randn(n, k // 64, generator=g, device=device) * 0.02).abs().to(torch.bfloat16)
        biases = (torch.randn(n, k // 64, generator=g, device=device) * 0.02).to(torch.bfloat16)
        lin[name] = (packed, scales, biases)
    norms = {n: (1 + 0.1 * torch.randn(128, generator=g, device=device)).float() for n in norm_names(cfg)}
    return lin, norms


class DitEngine:
    """Owns an aex_dit (one image, one device)."""

    def __init__(self, cfg: DitConfig, ctx=None, device=0):
        self.cfg = cfg
        self.ctx = ctx or _lib.context(device)
        self.L = _lib.lib()
        h = C.c_void_p()
        c = cfg.c()
        self.ctx.check(self.L.aex_dit_create(self.ctx.handle, C.byref(c), C.byref(h)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            self.L.aex_dit_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _s(stream):
        return (stream or torch.cuda.current_stream()).cuda_stream

    def load_linear(self, name, packed, scales, biases, stream=None):
        n, k = packed.shape[0], packed.shape[1] * 8
        self.ctx.check(self.L.aex_dit_load_linear(self.handle, name.encode(), packed.data_ptr(), scales.data_ptr(),
                                                  biases.data_ptr(), n, k, self._s(stream)))

    def load_norm(self, name, weight, stream=None):
        self.ctx.check(self.L.aex_dit_load_norm(self.handle, name.encode(), weight.data_ptr(), self._s(stream)))

    def load(self, lin, norms, stream=None):
        for name, (p, s, b) in lin.items():
            self.load_linear(name, p, s, b, stream)
        for name, w in norms.items():
            self.load_norm(name, w, stream)

    def set_rope(self, cos, sin, stream=None):
        self.ctx.check(self.L.aex_dit_set_rope(self.handle, cos.data_ptr(), sin.data_ptr(), self._s(stream)))

    def project_context(self, embeds_bf16, stream=None):
        self.ctx.check(self.L.aex_dit_project_context(self.handle, embeds_bf16.data_ptr(), self._s(stream)))

    def set_timestep(self, t: float, stream=None):
        self.ctx.check(self.L.aex_dit_set_timestep(self.handle, C.c_float(t), self._s(stream)))

    def forward(self, latents, out=None, stream=None):
        out = torch.empty_like(latents) if out is None else out
        self.ctx.check(self.L.aex_dit_forward(self.handle, latents.data_ptr(), out.data_ptr(), self._s(stream)))
        return out

    def denoise_step(self, lat_in, lat_out, dt: float, stream=None):
        self.ctx.check(self.L.aex_dit_denoise_step(self.handle, lat_in.data_ptr(), lat_out.data_ptr(), C.c_float(dt),
                                                   self._s(stream)))

    def denoise(self, latents, steps=4, stream=None):
        """In place: noise in, denoised latents out."""
        self.ctx.check(self.L.aex_dit_denoise(self.handle, latents.data_ptr(), steps, self._s(stream)))
        return latents

    def set_sequence_parallel(self, comm, l_txt_total: int, l_img_total: int):
        """This engine holds one contiguous shard of the joint sequence; joint attention runs as a
        ring over `comm` (an aex_comm handle, or None to return to one GPU)."""
        self.ctx.check(self.L.aex_dit_set_sequence_parallel(self.handle, comm, l_txt_total, l_img_total))

    def load_safetensors(self, path, stream=None):
        """Every 4-bit linear and norm weight of a safetensors file or shard directory
        (aex_dit_load_safetensors). Returns (linears, norms) loaded."""
        nl, nn = C.c_int(0), C.c_int(0)
        self.ctx.check(self.L.aex_dit_load_safetensors(self.handle, os.fspath(path).encode(), C.byref(nl),
                                                       C.byref(nn), self._s(stream)))
        return nl.value, nn.value


def scan_safetensors(path, max_bytes=1 << 22):
    """Tensors of a safetensors file or shard directory without the GPU (aex_safetensors_scan):
    {name: (dtype, shape, file_offset, nbytes)}. Raises AexError for a malformed file."""
    L = _lib.lib()
    buf = C.create_string_buffer(max_bytes)
    rc = L.aex_safetensors_scan(os.fspath(path).encode(), buf, max_bytes)
    text = buf.value.decode()
    if rc != 0:
        raise _lib.AexError(rc, text)
    out = {}
    for line in text.splitlines():
        name, dtype, shape, off, nb = line.split(" ")
        out[name] = (dtype, tuple(int(v) for v in shape.split(",")) if shape else (), int(off), int(nb))
    return out


def rope_tables(cfg: DitConfig, device="cuda", text_positions="ids", theta=2000.0):
    """cos/sin [l_txt + l_img, 64] for text ids [0,0,0,i] (or all-zero text positions) and image ids
    (0, h, w, 0) on a square grid (Flux2RoPE.prepareTextIDs / prepareGridIDs), via aex_rope_tables."""
    side = int(round(cfg.l_img ** 0.5))
    assert side * side == cfg.l_img, "square image grid expected"
    ids = torch.zeros(cfg.seq, 4, dtype=torch.float32)
    if text_positions == "ids":
        ids[:cfg.l_txt, 3] = torch.arange(cfg.l_txt, dtype=torch.float32)
    hh, ww = torch.meshgrid(torch.arange(side), torch.arange(side), indexing="ij")
    ids[cfg.l_txt:, 1] = hh.reshape(-1).float()
    ids[cfg.l_txt:, 2] = ww.reshape(-1).float()
    ids = ids.to(device)
    cos = torch.empty(cfg.seq, 64, device=device)
    sin = torch.empty(cfg.seq, 64, device=device)
    ctx = _lib.context(ids.device.index or 0)
    axes = (C.c_int * 4)(32, 32, 32, 32)
    ctx.check(_lib.lib().aex_rope_tables(ctx.handle, ids.data_ptr(), cfg.seq, C.c_float(theta), axes, 4,
                                         cos.data_ptr(), sin.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return cos, sin


def dit_flops(cfg: DitConfig) -> dict:
    """Algorithmic FLOPs of one transformer pass (2*M*N*K per linear; 4*S^2*D*H per attention)."""
    lt, li, J = cfg.l_txt, cfg.l_img, cfg.seq
    lin = 0.0
    for name, (n, k) in linear_shapes(cfg).items():
        if name.startswith("transformer_blocks."):
            m = lt if (".add_" in name or "to_add_out" in name or "ff_context" in name) else li
        elif name.startswith("single_transformer_blocks."):
            m = J
        elif name == "x_embedder" or name == "proj_out":
            m = li
        else:
            continue  # conditioning / context: once per step or per generate, negligible
        lin += 2.0 * m * n * k
    att = (cfg.n_double + cfg.n_single) * 4.0 * J * J * 128 * cfg.heads
    return {"linear": lin, "attention": att, "total": lin + att}

