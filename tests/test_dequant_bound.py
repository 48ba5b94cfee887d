"""CPU check of the bound that lets the GEMM's in-register dequant use one
bf16 rounding (qmm_sm100.cu: one_rounding_exact): whenever the bound holds,
f32(scale * q + bias) is exact for every code q, so rounding the exact value
once to bf16 equals the reference's f32-then-bf16 rounding
(DirectTEEncoder.swift:104-123). Sweeps every pair of bf16 exponents with
random mantissas and signs, all 16 codes."""
import numpy as np


def one_rounding_exact(s16, b16):
    """Mirror of the device function (bf16 bit patterns in, bool out)."""
    s16 = np.asarray(s16, np.int64)
    b16 = np.asarray(b16, np.int64)
    zero = ((s16 & 0x7FFF) == 0) | ((b16 & 0x7FFF) == 0)
    es = (s16 >> 7) & 0xFF
    eb = (b16 >> 7) & 0xFF
    special = (es == 0) | (eb == 0) | (es == 0xFF) | (eb == 0xFF)
    ok = (np.maximum(es + 5, eb + 1) - np.minimum(es, eb)) <= 16
    return zero | (~special & ok)


def bf16_to_f64(u):
    return (np.asarray(u, np.uint32) << 16).view(np.float32).astype(np.float64)


def test_bound_implies_exact_f32():
    rng = np.random.default_rng(0)
    e = np.arange(1, 255)
    es, eb = np.meshgrid(e, e, indexing="ij")
    es, eb = es.ravel(), eb.ravel()
    n = es.size
    checked = 0
    for _ in range(4):
        s16 = (rng.integers(0, 2, n) << 15) | (es << 7) | rng.integers(0, 128, n)
        b16 = (rng.integers(0, 2, n) << 15) | (eb << 7) | rng.integers(0, 128, n)
        keep = one_rounding_exact(s16, b16)
        s = bf16_to_f64(s16[keep])
        b = bf16_to_f64(b16[keep])
        q = np.arange(16, dtype=np.float64)[:, None]
        exact = s[None, :] * q + b[None, :]  # float64 is exact here (at most 24 significant bits)
        with np.errstate(over="ignore"):
            f32 = exact.astype(np.float32).astype(np.float64)
        fin = np.isfinite(f32)
        assert np.array_equal(f32[fin], exact[fin])
        # Beyond the f32 range both roundings give +-inf: such values also lie past
        # the bf16 overflow threshold (2 - 2^-8) * 2^127.
        assert (np.abs(exact[~fin]) >= (2 - 2.0 ** -8) * 2.0 ** 127).all()
        checked += int(keep.sum())
    assert checked > 20000  # about 6,700 accepted exponent pairs per sweep


def test_bound_rejects_wide_gaps_and_subnormals():
    one = 0x3F80  # 1.0
    tiny = 0x3F80 - (20 << 7)  # 2^-20
    assert not one_rounding_exact(one, tiny)  # 1.0 * q + 2^-20 needs 25+ bits for odd q
    assert not one_rounding_exact(tiny, one)
    assert not one_rounding_exact(0x0001, one)  # subnormal scale
    assert one_rounding_exact(0x0000, tiny)  # zero scale: bias alone
    assert one_rounding_exact(one, 0x8000)  # -0 bias
    assert one_rounding_exact(0x3C23, 0xBD8F)  # ~0.01 and ~-0.07: typical affine-quant pair
