"""Parity of the 4-bit affine linears (through the C ABI) with the CPU oracle.

* Dequantization (aex_dequantize_mlx, aex_qweight_create + aex_qweight_dequantize):
  bit-exact against the oracle's restatement of the reference CPU dequant and the
  golden fixtures (incl. the double-rounding cases).
* aex_qmm: against the oracle (small shapes) and, at BASELINE configs[2] sizes, against
  an fp32 matmul of the bit-exact dequantized weights. Tolerances: relative L2 <= 1e-2
  (bf16 output) and max-abs <= 2e-2 relative to the output's max magnitude; f32 output
  of the tensor-core path (m > 16) within 1e-4, of the GEMV path (m <= 16, which like
  MLX's qmv uses the unrounded dequantized weights) within 1e-4 of the oracle's qmv
  and 5e-3 of the bf16-weight product.
"""
import json
import os

import numpy as np
import pytest
import torch

from aestrix_b200 import _lib, qmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _np_u32(t):
    return t.cpu().numpy().view(np.uint32)


def _np_u16(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _assert_close(got, ref, rel=1e-2, absr=2e-2):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert np.isfinite(got).all()
    rl2 = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    mx = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert rl2 <= rel and mx <= absr, f"rel-L2 {rl2:.3e} max-abs/max {mx:.3e}"


@pytest.mark.parametrize("n,k", [(300, 640), (256, 64), (1, 3072), (3072, 128)])
def test_dequant_bit_exact(cuda_ctx, n, k):
    packed, scales, biases = qmm.synthetic_weight(n, k, seed=n + k)
    ref = O.dequant_q4(_np_u32(packed), _np_u16(scales), _np_u16(biases), n, k)
    got = _np_u16(qmm.dequantize(packed, scales, biases))
    assert np.array_equal(got, ref)
    w = qmm.QuantizedWeight(packed, scales, biases)
    assert np.array_equal(_np_u16(w.dequantize()), ref)


def test_dequant_golden_and_double_rounding(cuda_ctx):
    with open(os.path.join(GOLD, "bf16_dequant.json")) as f:
        g = json.load(f)
    cases = g["dequant_words"] + [
        {"packed": c["q"] * 0x11111111, "scale": c["scale"], "bias": c["bias"], "out": [c["out"]] * 8}
        for c in g["double_rounding"]]
    n = len(cases)
    packed = np.zeros((n, 8), np.uint32)
    scales = np.zeros((n, 1), np.uint16)
    biases = np.zeros((n, 1), np.uint16)
    for i, c in enumerate(cases):
        packed[i, :] = c["packed"]
        scales[i, 0], biases[i, 0] = c["scale"], c["bias"]
    tp = torch.from_numpy(packed.view(np.int32)).cuda()
    ts = torch.from_numpy(scales.view(np.int16)).view(torch.bfloat16).cuda()
    tb = torch.from_numpy(biases.view(np.int16)).view(torch.bfloat16).cuda()
    got = _np_u16(qmm.dequantize(tp, ts, tb))
    for i, c in enumerate(cases):
        assert got[i, :8].tolist() == c["out"], c
    assert np.array_equal(_np_u16(qmm.QuantizedWeight(tp, ts, tb).dequantize()), got)


@pytest.mark.parametrize("m,n,k", [(1, 300, 640), (2, 512, 256), (5, 1000, 192), (16, 768, 3072),
                                   (17, 300, 640), (130, 520, 256), (300, 256, 1024), (1, 256, 9216),
                                   (3, 1300, 1536), (8, 640, 12288), (1, 128, 24576)])
def test_qmm_vs_oracle(cuda_ctx, m, n, k):
    packed, scales, biases = qmm.synthetic_weight(n, k, seed=7 * m + n)
    g = torch.Generator().manual_seed(m * 1000 + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = qmm.QuantizedWeight(packed, scales, biases)
    ref = O.qmm(x.float().numpy(), _np_u32(packed), _np_u16(scales), _np_u16(biases), n, k)
    y32 = w(x.cuda(), out_dtype=torch.float32)
    y16 = w(x.cuda())
    torch.cuda.synchronize()
    if m > 16 or k > 24576:
        # tensor-core path: the bit-exact bf16 weights, f32 accumulation (order differs only)
        _assert_close(y32.cpu().numpy(), ref, rel=1e-4, absr=1e-4)
    else:
        # GEMV path: scale*sum(x*q) + bias*sum(x) with unrounded weights (MLX qmv's formulation): against the
        # oracle's qmv (f64) tightly, against the bf16-weight product within the weight rounding
        qv = O.qmv(x.float().numpy(), _np_u32(packed), _np_u16(scales), _np_u16(biases), n, k)
        _assert_close(y32.cpu().numpy(), qv, rel=1e-4, absr=2e-4)
        _assert_close(y32.cpu().numpy(), ref, rel=5e-3, absr=1e-2)
    _assert_close(y16.float().cpu().numpy(), ref)


@pytest.mark.parametrize("m,n", [(4608, 9216), (512, 9216), (4608, 18432), (1, 9216), (1, 18432), (512, 18432)])
def test_qmm_baseline_config3(cuda_ctx, m, n):
    """QKV 3072->9216 and SwiGLU 3072->18432 at M in {4608, 512, 1}."""
    k = 3072
    packed, scales, biases = qmm.synthetic_weight(n, k, seed=n + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16).cuda()
    w = qmm.QuantizedWeight(packed, scales, biases)
    y = w(x)
    wd = qmm.dequantize(packed, scales, biases)  # bit-exact (tested above)
    ref = x.float() @ wd.float().t()
    torch.cuda.synchronize()
    rl2 = ((y.float() - ref).norm() / ref.norm()).item()
    mx = ((y.float() - ref).abs().max() / ref.abs().max()).item()
    assert rl2 <= 1e-2 and mx <= 2e-2, f"rel-L2 {rl2:.3e} max-abs/max {mx:.3e}"


def test_qmm_strided_io_and_errors(cuda_ctx):
    n, k, m = 512, 256, 200
    packed, scales, biases = qmm.synthetic_weight(n, k, seed=3)
    w = qmm.QuantizedWeight(packed, scales, biases)
    xb = torch.randn(m, k + 64).to(torch.bfloat16).cuda()
    x = xb[:, 32:32 + k]  # row pitch k+64, 64-byte offset
    yb = torch.zeros(m, n + 128, dtype=torch.bfloat16, device="cuda")
    y = yb[:, 64:64 + n]
    w(x, out=y)
    ref = x.float() @ w.dequantize().float().t()
    torch.cuda.synchronize()
    assert ((y.float() - ref).norm() / ref.norm()).item() < 1e-2
    assert bool((yb[:, :64] == 0).all()) and bool((yb[:, 64 + n:] == 0).all())
    with pytest.raises(_lib.AexError) as e:
        qmm.QuantizedWeight(packed, scales, biases, group_size=32)
    assert e.value.code == _lib.AEX_ERR_UNSUPPORTED
    with pytest.raises(_lib.AexError):
        w(torch.zeros(4, k + 8, dtype=torch.bfloat16, device="cuda")[:, 4:4 + k])  # 8-byte misaligned rows
    assert cuda_ctx.device_status() == 0


def test_f32_activations_outside_the_gemv_path_are_rejected(cuda_ctx):
    """f32 activations run on the GEMV path only: m > 16 or K > 24576 returns AEX_ERR_UNSUPPORTED, launching
    nothing."""
    w = qmm.QuantizedWeight(*qmm.synthetic_weight(128, 256, seed=4))
    with pytest.raises(_lib.AexError) as e:
        w(torch.zeros(17, 256, device="cuda"), out_dtype=torch.float32)
    assert e.value.code == _lib.AEX_ERR_UNSUPPORTED
    wk = qmm.QuantizedWeight(*qmm.synthetic_weight(128, 24576 + 64, seed=5))
    with pytest.raises(_lib.AexError) as e:
        wk(torch.zeros(1, 24576 + 64, device="cuda"), out_dtype=torch.float32)
    assert e.value.code == _lib.AEX_ERR_UNSUPPORTED
    assert cuda_ctx.device_status() == 0


def test_gemm_weights_bit_exact_identity(cuda_ctx):
    """x = identity: the GEMM's f32 output is then exactly the bf16 weights it
    dequantized in registers, which must equal the reference dequant bit for bit
    on both of its paths (one bf16 rounding where the bound allows it, the f32
    path elsewhere): random groups, the golden double-rounding cases, wide
    scale/bias exponent gaps, zeros and subnormal scales."""
    n, k = 256, 256
    rng = np.random.default_rng(11)
    tp, ts, tb = qmm.synthetic_weight(n, k, seed=5)
    packed, scales, biases = _np_u32(tp).copy(), _np_u16(ts).copy(), _np_u16(tb).copy()
    with open(os.path.join(GOLD, "bf16_dequant.json")) as f:
        g = json.load(f)
    cases = [(c["q"] * 0x11111111, c["scale"], c["bias"]) for c in g["double_rounding"]]
    cases += [(w["packed"], w["scale"], w["bias"]) for w in g["dequant_words"]]
    r = 0
    for word, sc, bi in cases:  # rows 0.. : one golden case per (row, group 0)
        packed[r, :8] = word
        scales[r, 0], biases[r, 0] = sc, bi
        r += 1
    gaps = [(0x3F80, 0x3F80 - (20 << 7)), (0x3F80 - (20 << 7), 0x3F80), (0x0003, 0x3C00), (0x0000, 0x3D00),
            (0x3D00, 0x0000), (0x4700, 0xB900), (0xB900, 0x4700)]
    for sc, bi in gaps:  # further rows: wide gaps / zeros / subnormals in group 1
        packed[r, 8:16] = rng.integers(0, 2**32, 8, dtype=np.uint64).astype(np.uint32)
        scales[r, 1], biases[r, 1] = sc, bi
        r += 1
    assert r < n
    ref = O.dequant_q4(packed, scales, biases, n, k)  # [n, k] bf16 bits
    tp = torch.from_numpy(packed.view(np.int32)).cuda()
    ts = torch.from_numpy(scales.view(np.int16)).view(torch.bfloat16).cuda()
    tb = torch.from_numpy(biases.view(np.int16)).view(torch.bfloat16).cuda()
    w = qmm.QuantizedWeight(tp, ts, tb)
    eye = torch.eye(k, dtype=torch.bfloat16, device="cuda")
    y = w(eye, out_dtype=torch.float32)  # y[m, n] = W[n, m]
    torch.cuda.synchronize()
    got = O.f32_to_bf16(y.cpu().numpy().T.copy())
    # A zero weight sums to +0 in the accumulator whatever its sign.
    ref = np.where(ref == 0x8000, np.uint16(0), ref)
    assert np.array_equal(got, ref), np.argwhere(got != ref)[:8]
