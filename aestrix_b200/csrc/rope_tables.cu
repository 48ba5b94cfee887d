// rope_tables.cu — 4-axis rotary tables on the device.
//
// Restates Flux2PosEmbed / Flux2RoPE.frequencies (Sources/ImarelloDiT/PosEmbed.swift:12-47,
// Sources/ImarelloCore/Flux2RoPE.swift:16-76): for axis a of dimension dim_a and
// i < dim_a / 2, omega = 1 / theta^(2i / dim_a), angle = pos_a * omega; the cos
// and sin columns of the axes are concatenated in axis order. f32 throughout,
// with the accurate powf / cosf / sinf of the CUDA math library.
#include "internal.h"

namespace aex {
namespace {

constexpr int kMaxAxes = 8;

struct RopeParams {
  const float* ids;  // [n, n_axes]
  int n, n_axes, half_total;
  float theta;
  int dim[kMaxAxes];
  int col0[kMaxAxes];  // first output column of each axis
  float* cos_out;
  float* sin_out;
};

__global__ void rope_tables_kernel(RopeParams p) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.n) * p.half_total) return;
  const int r = static_cast<int>(idx / p.half_total);
  const int col = static_cast<int>(idx % p.half_total);
  int a = 0;
  while (a + 1 < p.n_axes && col >= p.col0[a + 1]) ++a;
  const int i = col - p.col0[a];
  const float sc = static_cast<float>(2 * i) / static_cast<float>(p.dim[a]);
  const float omega = 1.0f / powf(p.theta, sc);
  const float angle = p.ids[static_cast<int64_t>(r) * p.n_axes + a] * omega;
  p.cos_out[idx] = cosf(angle);
  p.sin_out[idx] = sinf(angle);
}

}  // namespace
}  // namespace aex

extern "C" int aex_rope_tables(aex_ctx* ctx, const float* ids, int n, float theta, const int* axes_dim, int n_axes,
                               float* cos_out, float* sin_out, aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (!ids || !axes_dim || !cos_out || !sin_out) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL pointer");
  if (n <= 0 || n_axes <= 0 || n_axes > kMaxAxes)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "n must be positive and n_axes in [1, %d]", kMaxAxes);
  if (!(theta > 0.f)) return set_error(ctx, AEX_ERR_INVALID_ARG, "theta must be positive");
  RopeParams p{};
  p.ids = ids;
  p.n = n;
  p.n_axes = n_axes;
  p.theta = theta;
  p.cos_out = cos_out;
  p.sin_out = sin_out;
  int total = 0;
  for (int a = 0; a < n_axes; ++a) {
    if (axes_dim[a] <= 0 || axes_dim[a] % 2)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "axes_dim[%d] = %d must be positive and even", a, axes_dim[a]);
    p.dim[a] = axes_dim[a];
    p.col0[a] = total;
    total += axes_dim[a] / 2;
  }
  p.half_total = total;
  if (int r = bind_device(ctx)) return r;
  const int64_t elems = static_cast<int64_t>(n) * total;
  const int threads = 256;
  rope_tables_kernel<<<static_cast<unsigned>((elems + threads - 1) / threads), threads, 0,
                       static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch(ctx, "rope_tables_kernel");
}
