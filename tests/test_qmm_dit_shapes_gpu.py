"""aex_qmm at every (K, N) the FLUX.2-klein denoise runs (DirectDiTStep.swift:308-335,
844-884; DirectConditioner.swift:75-82), at M in {1, 512, 4608}:

  K=3072  -> N=3072 (to_q/k/v, to_out, time linear_2), 9216 (fused Q|K|V, single
             modulation), 18432 (feed-forward in, double modulation), 27648 (single
             block projection), 128 (proj_out)
  K=9216  -> N=3072 (feed-forward out)
  K=12288 -> N=3072 (single block to_out)
  K=7680  -> N=3072 (context embedder)
  K=128   -> N=3072 (x_embedder)
  K=256   -> N=3072 (time linear_1)

Each output is checked twice: every row against an fp32 matmul of the bit-exact
dequantized weights (aex_dequantize_mlx, itself bit-exact with the oracle), and a
sample of rows against the oracle: the tensor-core path (M > 16) against O.qmm
(quantizedMM on bf16 dequantized weights, f64 accumulation) within 1e-4 relative
(same weights, only the summation order differs); the GEMV path (M <= 16) against
O.qmv (MLX qmv: scale * sum(x q) + bias * sum(x), the unrounded weights, f64)
within 1e-4, and against the bf16-weight matmul within 5e-3 (the weight rounding);
bf16 output within rel-L2 1e-2 / max-abs 2e-2 of the output's magnitude.
The M = 1 rows also run with f32 activations, the reference's f32 qmm (the conditioner's
K = 256 and 3072, DirectConditioner.swift:48, 183-190); f32 activations take the GEMV
path only (m <= 16, K <= 24576)."""
import numpy as np
import pytest
import torch

from aestrix_b200 import _lib, qmm
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(3072, 3072), (3072, 9216), (3072, 18432), (3072, 27648), (3072, 128), (9216, 3072), (12288, 3072),
          (7680, 3072), (128, 3072), (256, 3072)]


def _np_u32(t):
    return t.cpu().numpy().view(np.uint32)


def _np_u16(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _rel(got, ref):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    return (np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30),
            np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


_W = {}


def _weight(k, n):
    if (k, n) not in _W:
        _W.clear()
        packed, scales, biases = qmm.synthetic_weight(n, k, seed=k * 7 + n)
        w = qmm.QuantizedWeight(packed, scales, biases)
        wd = qmm.dequantize(packed, scales, biases).float()
        _W[(k, n)] = (w, wd, _np_u32(packed), _np_u16(scales), _np_u16(biases))
    return _W[(k, n)]


@pytest.mark.parametrize("m", [1, 512, 4608])
@pytest.mark.parametrize("k,n", SHAPES)
def test_qmm_every_dit_shape(cuda_ctx, k, n, m):
    w, wd, p, s, b = _weight(k, n)
    g = torch.Generator().manual_seed(m + 3 * k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    y32 = w(x, out_dtype=torch.float32)
    y16 = w(x)
    full = x.float() @ wd.t()
    torch.cuda.synchronize()
    tol = 1e-4 if m > 16 else 5e-3
    rl2, mx = _rel(y32.cpu().numpy(), full.cpu().numpy())
    assert rl2 <= tol and mx <= 2 * tol, f"f32 out vs fp32 matmul: rel-L2 {rl2:.3e} max {mx:.3e}"
    rl2, mx = _rel(y16.float().cpu().numpy(), full.cpu().numpy())
    assert rl2 <= 1e-2 and mx <= 2e-2, f"bf16 out vs fp32 matmul: rel-L2 {rl2:.3e} max {mx:.3e}"
    rows = np.unique(np.linspace(0, m - 1, min(m, 12)).astype(int))
    gemv = m <= 16  # the GEMV path (K <= 24576: at most 8 K splits x 48 K blocks)
    ref = (O.qmv if gemv else O.qmm)(x[rows].float().cpu().numpy(), p, s, b, n, k)
    rl2, mx = _rel(y32.cpu().numpy()[rows], ref)
    assert rl2 <= 1e-4 and mx <= 2e-4, f"f32 out vs oracle rows: rel-L2 {rl2:.3e} max {mx:.3e}"
    if m == 1:
        xf = torch.randn(1, k, generator=g).cuda()  # f32 activations, not bf16-representable
        yf = w(xf, out_dtype=torch.float32)
        torch.cuda.synchronize()
        ref = O.qmv(xf.cpu().numpy(), p, s, b, n, k)
        rl2, mx = _rel(yf.cpu().numpy(), ref)
        assert rl2 <= 1e-4 and mx <= 2e-4, f"f32 x vs oracle qmv: rel-L2 {rl2:.3e} max {mx:.3e}"
    assert cuda_ctx.device_status() == 0
