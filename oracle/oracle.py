"""ctypes/numpy binding of the CPU oracle (liboracle.so, built from aex_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py, never by the product package.
Every function mirrors the C function of the same name (see aex_oracle.h for
the reference file:line each follows).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build() -> None:
    subprocess.run(["make", "-C", _HERE, "-s", "liboracle.so"], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.aexo_f32_to_bf16.restype = C.c_uint16
        L.aexo_f32_to_bf16.argtypes = [C.c_float]
        L.aexo_bf16_to_f32.restype = C.c_float
        L.aexo_bf16_to_f32.argtypes = [C.c_uint16]
        L.aexo_f32_to_bf16_array.argtypes = [_f32p, C.c_size_t, _u16p]
        L.aexo_bf16_to_f32_array.argtypes = [_u16p, C.c_size_t, _f32p]
        L.aexo_dequant_q4.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int, C.c_int, _u16p]
        L.aexo_pack_q4.argtypes = [_u8p, C.c_int, C.c_int, _u32p]
        L.aexo_qmm.argtypes = [_f32p, C.c_int, _u32p, _u16p, _u16p, C.c_int, C.c_int, C.c_int, _f32p]
        L.aexo_qmv.argtypes = [_f32p, C.c_int, _u32p, _u16p, _u16p, C.c_int, C.c_int, C.c_int, _f32p]
        L.aexo_rope_freqs.argtypes = [_f32p, C.c_int, C.c_float, _i32p, C.c_int, _f32p, _f32p]
        L.aexo_grid_ids.argtypes = [C.c_int, C.c_int, C.c_float, C.c_float, _f32p]
        L.aexo_text_ids.argtypes = [C.c_int, _f32p]
        L.aexo_rmsnorm.argtypes = [_f32p, C.c_int, C.c_int, C.c_void_p, C.c_float, _f32p]
        L.aexo_rope_apply.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.aexo_sdpa.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_int64, C.c_int64, C.c_int64, C.c_float, C.c_int, C.c_int]
        L.aexo_joint_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p,
                                           C.c_float, C.c_int, C.c_int]
        L.aexo_linear_mu.restype = C.c_float
        L.aexo_linear_mu.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.c_float]
        L.aexo_time_shift.restype = C.c_float
        L.aexo_time_shift.argtypes = [C.c_float, C.c_float, C.c_float]
        L.aexo_schedule.argtypes = [C.c_int, C.c_int, _f32p, _f32p]
        L.aexo_timestep_embedding.argtypes = [_f32p, C.c_int, C.c_int, _f32p]
        L.aexo_ln_mod.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _f32p, C.c_float, _f32p]
        L.aexo_swiglu.argtypes = [_f32p, _f32p, C.c_size_t, _f32p]
        L.aexo_gate_add.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, _f32p]
        _lib = L
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr_or_none(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32_to_bf16(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().aexo_f32_to_bf16_array(x.reshape(-1), x.size, out.reshape(-1))
    return out


def bf16_to_f32(u) -> np.ndarray:
    u = _c(u, np.uint16)
    out = np.empty(u.shape, np.float32)
    lib().aexo_bf16_to_f32_array(u.reshape(-1), u.size, out.reshape(-1))
    return out


def dequant_q4(packed, scales, biases, n, k, group_size=64) -> np.ndarray:
    out = np.empty((n, k), np.uint16)
    lib().aexo_dequant_q4(_c(packed, np.uint32), _c(scales, np.uint16), _c(biases, np.uint16), n, k, group_size,
                          out)
    return out


def pack_q4(codes) -> np.ndarray:
    codes = _c(codes, np.uint8)
    n, k = codes.shape
    out = np.empty((n, k // 8), np.uint32)
    lib().aexo_pack_q4(codes, n, k, out)
    return out


def qmm(x, packed, scales, biases, n, k, group_size=64) -> np.ndarray:
    x = _c(x, np.float32)
    m = x.shape[0]
    y = np.empty((m, n), np.float32)
    lib().aexo_qmm(x, m, _c(packed, np.uint32), _c(scales, np.uint16), _c(biases, np.uint16), n, k, group_size,
                   y)
    return y


def qmv(x, packed, scales, biases, n, k, group_size=64) -> np.ndarray:
    """MLX qmv on f32 activations: scale * sum(x * q) + bias * sum(x) per group (unrounded weights)."""
    x = _c(x, np.float32)
    m = x.shape[0]
    y = np.empty((m, n), np.float32)
    lib().aexo_qmv(x, m, _c(packed, np.uint32), _c(scales, np.uint16), _c(biases, np.uint16), n, k, group_size,
                   y)
    return y


def rope_freqs(ids, theta=2000.0, axes_dim=(32, 32, 32, 32)):
    ids = _c(ids, np.float32)
    axes = _c(axes_dim, np.int32)
    n = ids.shape[0]
    half = int(sum(a // 2 for a in axes_dim))
    c = np.empty((n, half), np.float32)
    s = np.empty((n, half), np.float32)
    lib().aexo_rope_freqs(ids, n, theta, axes, len(axes_dim), c, s)
    return c, s


def grid_ids(height, width, t_coord=0.0, layer=0.0):
    out = np.empty((height * width, 4), np.float32)
    lib().aexo_grid_ids(height, width, t_coord, layer, out)
    return out


def text_ids(length):
    out = np.empty((length, 4), np.float32)
    lib().aexo_text_ids(length, out)
    return out


def rmsnorm(x, w, eps):
    x = _c(x, np.float32)
    d = x.shape[-1]
    y = np.empty_like(x)
    wc = None if w is None else _c(w, np.float32)
    lib().aexo_rmsnorm(x, x.size // d, d, _ptr_or_none(wc), eps, y)
    return y


def rope_apply(x, cos_t, sin_t):
    """x: [s, h, d] f32 (copied), cos/sin [s, d/2]."""
    x = np.array(x, dtype=np.float32, order="C", copy=True)
    s, h, d = x.shape
    lib().aexo_rope_apply(x, s, h, d, _c(cos_t, np.float32), _c(sin_t, np.float32))
    return x


def sdpa(q, k, v, scale, q_begin=0, q_end=None):
    """q, k, v: [b, s, h, d] f32; returns [b, s, h, d] (rows outside the range are NaN)."""
    q, k, v = (_c(a, np.float32) for a in (q, k, v))
    b, s, h, d = q.shape
    out = np.full(q.shape, np.nan, np.float32)
    lib().aexo_sdpa(q, k, v, out, b, s, h, d, s * h * d, h * d, d, scale, q_begin, s if q_end is None else q_end)
    return out


def joint_attention(q, k, v, norm_q_w=None, norm_k_w=None, eps=1e-6, cos_t=None, sin_t=None, scale=None,
                    q_begin=0, q_end=None):
    """[b, s, h, d] f32 in/out; the composition norm -> RoPE -> SDPA."""
    q, k, v = (_c(a, np.float32) for a in (q, k, v))
    b, s, h, d = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    out = np.full(q.shape, np.nan, np.float32)
    arrs = [None if a is None else _c(a, np.float32) for a in (norm_q_w, norm_k_w, cos_t, sin_t)]
    lib().aexo_joint_attention(q, k, v, out, b, s, h, d, *(_ptr_or_none(a) for a in arrs[:2]), eps,
                               *(_ptr_or_none(a) for a in arrs[2:]), scale, q_begin,
                               s if q_end is None else q_end)
    return out


def linear_mu(image_seq_len, base_seq_len=256, max_seq_len=4096, base_shift=0.5, max_shift=1.15):
    return lib().aexo_linear_mu(image_seq_len, base_seq_len, max_seq_len, base_shift, max_shift)


def time_shift(mu, t, sigma_power=1.0):
    return lib().aexo_time_shift(mu, t, sigma_power)


def schedule(steps, image_seq_len):
    sig = np.empty(steps + 1, np.float32)
    ts = np.empty(steps, np.float32)
    lib().aexo_schedule(steps, image_seq_len, sig, ts)
    return sig, ts


def ln_mod_rows(x, scale, shift, eps):
    """LayerNorm (no affine) + (1 + scale) * n + shift over rows [r, d] (aexo_ln_mod)."""
    x = _c(x, np.float32)
    rows, d = x.shape
    y = np.empty_like(x)
    lib().aexo_ln_mod(x, rows, d, _c(scale, np.float32), _c(shift, np.float32), eps, y)
    return y


def timestep_embedding(t, dim=256):
    t = _c(t, np.float32)
    out = np.empty((t.size, dim), np.float32)
    lib().aexo_timestep_embedding(t, t.size, dim, out)
    return out
