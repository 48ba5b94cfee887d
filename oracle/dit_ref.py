"""CPU reference of the FLUX.2-klein transformer step, composed from the oracle's
C functions (aex_oracle.cpp).

TEST INFRASTRUCTURE ONLY (imported by tests/). Follows the reference wiring:
Flux2Transformer / DirectDiTStep.encodeDenoiseStep (Sources/ImarelloDiT/Transformer.swift:183-333,
Sources/ImarelloDirect/DirectDiTStep.swift:546-971), the double block
(TransformerBlock.swift:25-74, JointAttention.swift:44-110), the single block
(ParallelSelfAttention.swift:30-132) and the conditioner (DirectConditioner.swift:160-213).
Activations are rounded to bf16 where the reference stores bf16 (GEMM inputs,
projection outputs, normalized Q/K, attention output; the conditioning chain
stays f32 like the reference's f32 qmm, DirectConditioner.swift:183-190), so a
comparison isolates kernel arithmetic from the storage dtype; everything else
is f32/f64. With storage="f32" no activation is rounded at all (the weights are
still the bf16 dequantized ones): the all-f32 composition that measures how far
the bf16 storage points move the result.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def bf(x):
    return O.bf16_to_f32(O.f32_to_bf16(np.asarray(x, np.float32)))


def _ident(x):
    return np.asarray(x, np.float32)


class DitRef:
    def __init__(self, cfg, lin, norms, storage="bf16"):
        """lin: {name: (packed uint32 [n, k/8], scales uint16, biases uint16)}; norms: {name: f32 [128]};
        storage "bf16" (the reference's storage points) or "f32" (no activation rounding)."""
        self.cfg = cfg
        self.lin = lin
        self.norms = norms
        self.bf = bf if storage == "bf16" else _ident

    def linear(self, name, x, f32_in=False):
        """x . deq(W)^T: the bf16 qmm (x rounded to bf16, bf16 dequantized weights), or with f32_in the
        f32 qmm of the conditioner (MLX qmv: f32 x, unrounded dequantized weights)."""
        p, s, b = self.lin[name]
        n, k = p.shape[0], p.shape[1] * 8
        if f32_in:
            return O.qmv(np.asarray(x, np.float32), p, s, b, n, k)
        return O.qmm(self.bf(x), p, s, b, n, k)

    # DirectConditioner.stepConditioning (:172-213): f32 activations through the f32 qmm.
    def conditioning(self, t):
        c = self.cfg
        temb_in = O.timestep_embedding(np.array([t], np.float32), c.timestep_dim)
        t1 = self.linear("time_guidance_embed.linear_1", temb_in, f32_in=True)
        temb = self.linear("time_guidance_embed.linear_2", t1 / (1 + np.exp(-t1)), f32_in=True)
        ts = temb / (1 + np.exp(-temb))
        return {k: self.linear(n, ts, f32_in=True)[0] for k, n in (("img", "double_stream_modulation_img.linear"),
                                                                   ("txt", "double_stream_modulation_txt.linear"),
                                                                   ("single", "single_stream_modulation.linear"),
                                                                   ("out", "norm_out.linear"))}

    # DirectConditioner.projectContext (:217-240): bf16 qmm, bf16 output widened to f32.
    def project_context(self, embeds):
        return self.bf(self.linear("context_embedder", embeds))

    def _prep(self, x, w, cos, sin, rows=None):
        """RMSNorm per head (weights w or a (w_txt, w_img, split) triple) + interleaved RoPE, bf16."""
        c = self.cfg
        J = x.shape[0]
        xh = x.reshape(J, c.heads, 128).astype(np.float32)
        if isinstance(w, tuple):
            wt, wi, split = w
            y = np.empty_like(xh)
            y[:split] = O.rmsnorm(xh[:split], wt, c.rms_eps)
            y[split:] = O.rmsnorm(xh[split:], wi, c.rms_eps)
        else:
            y = O.rmsnorm(xh, w, c.rms_eps)
        return self.bf(O.rope_apply(y, cos, sin))

    def _attend(self, q, k, v):
        c = self.cfg
        J = q.shape[0]
        o = O.sdpa(q.reshape(1, J, c.heads, 128), k.reshape(1, J, c.heads, 128),
                   self.bf(v).reshape(1, J, c.heads, 128), 1.0 / np.sqrt(128))
        return self.bf(o.reshape(J, c.hidden))

    def forward(self, latents, e0, cos, sin, mods):
        c = self.cfg
        C, lt, mlp = c.hidden, c.l_txt, c.mlp_hidden
        ln = lambda x, m, s0: self.bf(O.ln_mod_rows(x, m[s0 + C:s0 + 2 * C], m[s0:s0 + C], c.ln_eps))
        silu = lambda g: g / (1 + np.exp(-g))
        X = np.concatenate([e0.astype(np.float32), self.linear("x_embedder", latents)], 0)
        for i in range(c.n_double):
            p = f"transformer_blocks.{i}."
            mt, mi = mods["txt"], mods["img"]
            nt, ni = ln(X[:lt], mt, 0), ln(X[lt:], mi, 0)
            q = self.bf(np.concatenate([self.linear(p + "attn.add_q_proj", nt), self.linear(p + "attn.to_q", ni)]))
            k = self.bf(np.concatenate([self.linear(p + "attn.add_k_proj", nt), self.linear(p + "attn.to_k", ni)]))
            v = self.bf(np.concatenate([self.linear(p + "attn.add_v_proj", nt), self.linear(p + "attn.to_v", ni)]))
            n = self.norms
            qn = self._prep(q, (n[p + "attn.norm_added_q"], n[p + "attn.norm_q"], lt), cos, sin)
            kn = self._prep(k, (n[p + "attn.norm_added_k"], n[p + "attn.norm_k"], lt), cos, sin)
            o = self._attend(qn, kn, v)
            X[:lt] += mt[2 * C:3 * C] * self.linear(p + "attn.to_add_out", o[:lt])
            X[lt:] += mi[2 * C:3 * C] * self.linear(p + "attn.to_out", o[lt:])
            for rows, m, ff in ((slice(0, lt), mt, "ff_context"), (slice(lt, None), mi, "ff")):
                h = self.bf(self.linear(p + ff + ".linear_in", ln(X[rows], m, 3 * C)))
                sw = self.bf(silu(h[:, :mlp]) * h[:, mlp:])
                X[rows] += m[5 * C:6 * C] * self.linear(p + ff + ".linear_out", sw)
        for i in range(c.n_single):
            p = f"single_transformer_blocks.{i}.attn."
            ms = mods["single"]
            pr = self.bf(self.linear(p + "to_qkv_mlp_proj", ln(X, ms, 0)))
            qn = self._prep(pr[:, :C], self.norms[p + "norm_q"], cos, sin)
            kn = self._prep(pr[:, C:2 * C], self.norms[p + "norm_k"], cos, sin)
            o = self._attend(qn, kn, pr[:, 2 * C:3 * C])
            sw = self.bf(silu(pr[:, 3 * C:3 * C + mlp]) * pr[:, 3 * C + mlp:])
            X += ms[2 * C:3 * C] * self.linear(p + "to_out", np.concatenate([o, sw], 1))
        mo = mods["out"]
        nh = self.bf(O.ln_mod_rows(X[lt:], mo[:C], mo[C:2 * C], c.ln_eps))
        return self.linear("proj_out", nh)
