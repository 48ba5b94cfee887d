"""4-bit affine quantized linears over libaestrix_cuda (ctypes binding used by the
tests and the benchmark).

Mirrors the reference surface:

* :class:`QuantizedWeight` — an MLX 4-bit affine weight (``.weight`` uint32 [n, k/8],
  ``.scales`` / ``.biases`` bf16 [n, k/64]) uploaded and unpacked on the device
  (TransformerWeights.loadQuantized, Sources/ImarelloDiT/TransformerWeights.swift:13-54;
  DirectDiTStep.quant, Sources/ImarelloDirect/DirectDiTStep.swift:278-335).
* :func:`quantized_mm` — ``quantizedMM(x, w, scales:, biases:, transpose: true, groupSize: 64,
  bits: 4)`` (Sources/ImarelloDiT/AttentionUtils.swift:212-221).
* :func:`dequantize` — MLX ``dequantized`` (Sources/ImarelloDirect/DirectTEEncoder.swift:129-134).

Packed words are passed as int32 CUDA tensors (same bits as MLX's uint32).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


def _stream_ptr(stream):
    return (stream or torch.cuda.current_stream()).cuda_stream


def _check_mlx(packed, scales, biases):
    for t, dt in ((packed, (torch.int32, torch.uint32)), (scales, (torch.bfloat16,)), (biases, (torch.bfloat16,))):
        if not t.is_cuda or t.dtype not in dt or not t.is_contiguous():
            raise TypeError("packed int32/uint32, scales/biases bfloat16: contiguous CUDA tensors")
    n, k8 = packed.shape
    if scales.shape != (n, k8 * 8 // 64) or biases.shape != scales.shape:
        raise ValueError("scales/biases must be [n, k/64]")
    return n, k8 * 8


def dequantize(packed, scales, biases, group_size=64, bits=4, ctx=None, stream=None):
    """bf16 [n, k] = bf16_rne(f32(scale * q + bias)), straight from the MLX layout."""
    n, k = _check_mlx(packed, scales, biases)
    ctx = ctx or _lib.context(packed.device.index or 0)
    out = torch.empty(n, k, dtype=torch.bfloat16, device=packed.device)
    ctx.check(_lib.lib().aex_dequantize_mlx(ctx.handle, packed.data_ptr(), scales.data_ptr(), biases.data_ptr(), n, k,
                                            group_size, bits, out.data_ptr(), _stream_ptr(stream)))
    return out


class QuantizedWeight:
    """Device-resident tile-layout 4-bit weight (owns an aex_qweight handle)."""

    def __init__(self, packed, scales, biases, group_size=64, bits=4, ctx=None, stream=None):
        self.n, self.k = _check_mlx(packed, scales, biases)
        self.ctx = ctx or _lib.context(packed.device.index or 0)
        self.device = packed.device
        h = C.c_void_p()
        self.ctx.check(_lib.lib().aex_qweight_create(self.ctx.handle, packed.data_ptr(), scales.data_ptr(),
                                                     biases.data_ptr(), self.n, self.k, group_size, bits, C.byref(h),
                                                     _stream_ptr(stream)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            _lib.lib().aex_qweight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def dequantize(self, stream=None):
        out = torch.empty(self.n, self.k, dtype=torch.bfloat16, device=self.device)
        self.ctx.check(_lib.lib().aex_qweight_dequantize(self.ctx.handle, self.handle, out.data_ptr(),
                                                         _stream_ptr(stream)))
        return out

    def __call__(self, x, out_dtype=torch.bfloat16, out=None, stream=None):
        return quantized_mm(x, self, out_dtype=out_dtype, out=out, stream=stream)


def quantized_mm(x, w: QuantizedWeight, out_dtype=torch.bfloat16, out=None, stream=None):
    """y[m, n] = x[m, k] . deq(W)[n, k]^T; x bf16 [m, k] (row stride ldx), or f32 for m <= 16 (the
    conditioner's f32 qmm, DirectConditioner.swift:48); y bf16 or f32."""
    if x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda or x.dim() != 2 or x.stride(1) != 1:
        raise TypeError("x must be a 2-D CUDA bfloat16 or float32 tensor with contiguous rows")
    m = x.shape[0]
    if out is None:
        out = torch.empty(m, w.n, dtype=out_dtype, device=x.device)
    dt = _lib.AEX_DTYPE_F32 if out.dtype == torch.float32 else _lib.AEX_DTYPE_BF16
    xdt = _lib.AEX_DTYPE_F32 if x.dtype == torch.float32 else _lib.AEX_DTYPE_BF16
    w.ctx.check(_lib.lib().aex_qmm_ex(w.ctx.handle, w.handle, x.data_ptr(), xdt, x.stride(0), m, out.data_ptr(),
                                      out.stride(0), dt, _stream_ptr(stream)))
    return out


def synthetic_weight(n, k, seed, device="cuda"):
    """BASELINE configs[2] weights: codes U{0..15} packed LSB-first 8 per uint32, bf16 scales
    |N(0, 0.02)|, bf16 biases N(0, 0.02), group 64. Returns (packed int32, scales, biases) on `device`."""
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int64)
    shifts = torch.arange(8, dtype=torch.int64) * 4
    words = (codes.view(n, k // 8, 8) << shifts).sum(-1)
    packed = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    scales = (torch.randn(n, k // 64, generator=g) * 0.02).abs().to(torch.bfloat16)
    biases = (torch.randn(n, k // 64, generator=g) * 0.02).to(torch.bfloat16)
    return packed.to(device), scales.to(device), biases.to(device)
