"""Joint attention operators over libaestrix_cuda (ctypes binding used by the
tests and the benchmark).

Mirrors the reference operator surface:

* :func:`scaled_dot_product_attention` — ``MetalFlashAttention.scaledDotProductAttention(
  query:key:value:scale:mask:)`` (Sources/ImarelloDiT/MetalFlashAttention.swift:44-78) on
  ``[B, H, S, D]`` tensors; ``mask`` must be ``None`` (the product path never passes one).
* :func:`joint_attention` — the fused QK-RMSNorm -> interleaved RoPE -> SDPA of
  ``Flux2Attention`` / ``Flux2ParallelSelfAttention`` (Sources/ImarelloDiT/JointAttention.swift:44-110,
  ParallelSelfAttention.swift:30-132) on ``[B, S, H, D]`` token-major tensors, the layout of the
  direct engine's ``jointQ/K/V`` buffers (Sources/ImarelloDirect/DirectDiTStep.swift:464-484).

Inputs are CUDA bf16 tensors whose last dimension is contiguous; everything runs in the CUDA
library (there is no Python or CPU fallback).
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib


def _bshd(t: torch.Tensor, b_dim: int, s_dim: int, h_dim: int) -> _lib.aex_bshd:
    if t.dtype != torch.bfloat16 or not t.is_cuda:
        raise TypeError("attention tensors must be CUDA bfloat16")
    if t.stride(-1) != 1:
        raise ValueError("the head_dim axis must be contiguous")
    st = t.stride()
    return _lib.aex_bshd(t.data_ptr(), st[b_dim], st[s_dim], st[h_dim])


def _f32_ptr(t):
    if t is None:
        return None
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise TypeError("norm weights / rope tables must be contiguous CUDA float32")
    return t.data_ptr()


def _stream_ptr(stream):
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def make_args(q, k, v, out, layout, norm_q_weight=None, norm_k_weight=None, eps=1e-6, cos=None, sin=None,
              scale=None) -> _lib.aex_attention_args:
    if layout == "bshd":
        dims = (0, 1, 2)
        b, s, h, d = q.shape
    elif layout == "bhsd":
        dims = (0, 2, 1)
        b, h, s, d = q.shape
    else:
        raise ValueError(layout)
    for t in (k, v, out):
        if t.shape != q.shape:
            raise ValueError("q, k, v and out must have the same shape")
    a = _lib.aex_attention_args()
    a.q, a.k, a.v, a.out = (_bshd(t, *dims) for t in (q, k, v, out))
    a.batch, a.seq, a.heads, a.head_dim = b, s, h, d
    a.norm_q_weight = _f32_ptr(norm_q_weight)
    a.norm_k_weight = _f32_ptr(norm_k_weight)
    a.eps = float(eps)
    a.rope_cos = _f32_ptr(cos)
    a.rope_sin = _f32_ptr(sin)
    a.scale = float(scale) if scale is not None else 1.0 / math.sqrt(d)
    return a


def joint_attention(q, k, v, norm_q_weight=None, norm_k_weight=None, eps=1e-6, cos=None, sin=None, scale=None,
                    out=None, ctx=None, stream=None):
    """softmax(scale * RoPE(RMSNorm(Q)) RoPE(RMSNorm(K))^T) V on [B, S, H, 128] bf16 tensors.

    ``cos``/``sin``: [S, 64] float32 tables (row r rotates token r), or None to skip RoPE.
    ``norm_*_weight``: [128] float32 RMSNorm weights, or None to skip that norm.
    Returns ``out`` ([B, S, H, 128] bf16, allocated if not given).
    """
    ctx = ctx or _lib.context(q.device.index or 0)
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    a = make_args(q, k, v, out, "bshd", norm_q_weight, norm_k_weight, eps, cos, sin, scale)
    ctx.check(_lib.lib().aex_joint_attention(ctx.handle, C.byref(a), _stream_ptr(stream)))
    return out


def scaled_dot_product_attention(query, key, value, scale=None, mask=None, out=None, ctx=None, stream=None):
    """softmax(scale * Q K^T) V on [B, H, S, 128] bf16 tensors (no mask)."""
    if mask is not None:
        raise NotImplementedError("attention masks are not supported (the DiT path never uses one)")
    ctx = ctx or _lib.context(query.device.index or 0)
    if out is None:
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
    a = make_args(query, key, value, out, "bhsd", scale=scale)
    ctx.check(_lib.lib().aex_joint_attention(ctx.handle, C.byref(a), _stream_ptr(stream)))
    return out


def rope_tables(ids: torch.Tensor, theta: float = 2000.0, axes_dim=(32, 32, 32, 32), ctx=None, stream=None):
    """cos/sin [n, sum(axes_dim)/2] f32 on the device of `ids` ([n, len(axes_dim)] f32 CUDA position ids,
    e.g. text (0,0,0,i), image (t,h,w,0)) through aex_rope_tables (Flux2PosEmbed, PosEmbed.swift:5-48)."""
    if not (ids.is_cuda and ids.dtype == torch.float32 and ids.is_contiguous() and ids.dim() == 2):
        raise TypeError("ids must be a contiguous CUDA float32 [n, n_axes] tensor")
    n = ids.shape[0]
    half = sum(a // 2 for a in axes_dim)
    cos = torch.empty(n, half, device=ids.device)
    sin = torch.empty(n, half, device=ids.device)
    ctx = ctx or _lib.context(ids.device.index or 0)
    axes = (C.c_int * len(axes_dim))(*axes_dim)
    ctx.check(_lib.lib().aex_rope_tables(ctx.handle, ids.data_ptr(), n, C.c_float(theta), axes, len(axes_dim),
                                         cos.data_ptr(), sin.data_ptr(), _stream_ptr(stream)))
    return cos, sin


def grid_ids(height: int, width: int, t: float = 0.0, device="cuda") -> torch.Tensor:
    """Image position ids (t, h, w, 0) row-major over the grid (Flux2RoPE.prepareGridIDs)."""
    hh, ww = torch.meshgrid(torch.arange(height), torch.arange(width), indexing="ij")
    ids = torch.zeros(height * width, 4, dtype=torch.float32)
    ids[:, 0] = t
    ids[:, 1] = hh.reshape(-1).float()
    ids[:, 2] = ww.reshape(-1).float()
    return ids.to(device)


def text_ids(length: int, device="cuda") -> torch.Tensor:
    """Text position ids (0, 0, 0, i) (Flux2RoPE.prepareTextIDs)."""
    ids = torch.zeros(length, 4, dtype=torch.float32)
    ids[:, 3] = torch.arange(length, dtype=torch.float32)
    return ids.to(device)


def attention_flops(batch: int, seq: int, heads: int, head_dim: int = 128) -> float:
    """Algorithmic FLOPs of one call: two GEMMs of 2*S*S*D per (batch, head)."""
    return 4.0 * batch * heads * seq * seq * head_dim
