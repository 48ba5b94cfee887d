// dit_internal.h — launchers of the DiT glue kernels (dit_glue.cu) used by the
// DiT step engine (dit_engine.cpp). All asynchronous on `s`; pointers device.
#pragma once
#include "internal.h"

namespace aex {
namespace glue {

// y_bf16[r, :] = (1 + scale) * LayerNorm(x[r, :]) + shift, rows r < rows, width C.
int ln_mod(aex_ctx* ctx, const float* x, int64_t ldx, int rows, int C, const float* scale, const float* shift,
           float eps, void* y, int64_t ldy, cudaStream_t s);
// x_f32[r, c] += gate[c] * scale * v_bf16[r, c] (gate NULL: 1).
int gate_add(aex_ctx* ctx, float* x, int64_t ldx, int rows, int C, const float* gate, const void* v, int64_t ldv,
             float scale, cudaStream_t s);
// lat_out = lat_in + *dt * v (n elements; lat_out may equal lat_in).
int euler(aex_ctx* ctx, const float* lat_in, const float* v, const float* dt, int64_t n, float* lat_out,
          cudaStream_t s);
// out[0:dim] = [cos(t*f_i) | sin(t*f_i)], t = *t_dev, f_i = exp(-ln(10000) i / (dim/2)).
int timestep_embedding(aex_ctx* ctx, const float* t_dev, int dim, float* out, cudaStream_t s);
// *dst = v (device scalar written in stream order).
int set_scalar(aex_ctx* ctx, float* dst, float v, cudaStream_t s);
// cur[0..1] = steps[2i .. 2i+1], i = (*counter)++.
int step_select(aex_ctx* ctx, const float* steps, int* counter, float* cur, cudaStream_t s);
// y = silu(x) = x / (1 + exp(-x)), f32 (y may equal x).
int silu_f32(aex_ctx* ctx, const float* x, int n, float* y, cudaStream_t s);
int f32_to_bf16(aex_ctx* ctx, const float* x, int64_t n, void* y, cudaStream_t s);
int bf16_to_f32_rows(aex_ctx* ctx, const void* x, int64_t ldx, int rows, int cols, float* y, int64_t ldy,
                     cudaStream_t s);

}  // namespace glue
}  // namespace aex
