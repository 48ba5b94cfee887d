"""aestrix_b200 — B200-native (sm_100a) FLUX.2-klein DiT joint attention and
MLX-layout 4-bit affine linears, behind the C ABI of libaestrix_cuda
(include/aestrix_cuda.h). The Python modules here are the ctypes binding used
by the tests and the benchmark; the product path is the CUDA library."""

__all__ = ["_lib"]
