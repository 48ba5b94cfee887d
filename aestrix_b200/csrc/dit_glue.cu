// dit_glue.cu — the elementwise / row-reduction kernels between the DiT's
// linears and attention calls (all HBM-bound). Restates the arithmetic of the
// direct engine's glue kernels (Sources/ImarelloDirect/DirectDiTKernels.swift)
// for a bf16 activation path (the reference's f16 /16 x16 scaling sandwich is
// not needed with bf16's range):
//   ln_mod      LayerNorm (no affine, eps) + AdaLN modulate (1+scale)*n + shift -> bf16
//               (dd_ln_mod_prescale :15-57; Flux2TransformerBlock norm1/modApply,
//               Sources/ImarelloDiT/TransformerBlock.swift:42-44, ModulationOps.swift)
//   (SwiGLU, dd_swiglu_pitched :138-159, is fused into the feed-forward GEMM's
//   epilogue: qmm_sm100.cu, swiglu1)
//   gate_add    x += gate * v, x f32 (dd_gate_add :208-221) — used where the
//               producing GEMM did not already fuse it
//   euler       lat_out = lat_in + dt * v (Flux2Scheduler.step, Flux2Scheduler.swift:101-109)
//   timestep    cos/sin sinusoid, flip_sin_to_cos (DirectConditioner.sinusoid,
//               Sources/ImarelloDirect/DirectConditioner.swift:160-170)
//   silu (f32), f32 -> bf16, bf16 -> f32 row copies.
#include "dit_internal.h"
#include "sm100.cuh"

namespace aex {
namespace glue {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (w == 0) {
    t = l < (blockDim.x >> 5) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (w == 0) {
    t = l < (blockDim.x >> 5) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// One CTA per row; C a multiple of 4. Two-pass (mean, then centered variance)
// in f32 from registers/L1. A row whose magnitude exceeds 2^48 (where the sum
// of C squares could pass the f32 range; the residual stream of a deep stack
// can grow that large) takes its variance on x scaled by an exact power of two
// 2^-e, so the result is the one an unbounded-range f32 computation would
// give; other rows compute exactly as without the scaling.
__global__ void __launch_bounds__(kRowThreads) ln_mod_kernel(const float* __restrict__ x, int64_t ldx, int C,
                                                             const float* __restrict__ scale,
                                                             const float* __restrict__ shift, float eps,
                                                             __nv_bfloat16* __restrict__ y, int64_t ldy) {
  __shared__ float red[32];
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * ldx;
  float s = 0.f, amax = 0.f;
  for (int i = threadIdx.x * 4; i < C; i += kRowThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    s += (v.x + v.y) + (v.z + v.w);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  const float mean = block_sum(s, red) / C;
  amax = block_max(amax, red);
  // 2^-e with 2^e the power of two at or below amax, when amax > 2^48 (else 1)
  const float sc = (amax > 281474976710656.0f && amax <= 3.4028235e38f) ? __uint_as_float((254u - ((__float_as_uint(amax) >> 23) & 0xFFu)) << 23)
                                             : 1.0f;
  float q = 0.f;
  for (int i = threadIdx.x * 4; i < C; i += kRowThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float a = (v.x - mean) * sc, b = (v.y - mean) * sc, c = (v.z - mean) * sc, d = (v.w - mean) * sc;
    q += (a * a + b * b) + (c * c + d * d);
  }
  const float inv = rsqrtf(block_sum(q, red) / C + eps * sc * sc) * sc;
  __nv_bfloat16* yr = y + static_cast<int64_t>(blockIdx.x) * ldy;
  for (int i = threadIdx.x * 4; i < C; i += kRowThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 sc = __ldg(reinterpret_cast<const float4*>(scale + i));
    const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + i));
    const float o0 = fmaf(1.f + sc.x, (v.x - mean) * inv, sh.x);
    const float o1 = fmaf(1.f + sc.y, (v.y - mean) * inv, sh.y);
    const float o2 = fmaf(1.f + sc.z, (v.z - mean) * inv, sh.z);
    const float o3 = fmaf(1.f + sc.w, (v.w - mean) * inv, sh.w);
    *reinterpret_cast<uint2*>(yr + i) = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
  }
}


// The same LayerNorm + modulation with the row held in registers (C <= NV * 4 * kRowThreads): one read of
// the row from memory, the sum and the magnitude reduced together, then the centered variance from registers.
// Sums are taken in a different order than ln_mod_kernel's (each thread's four-element groups first).
__device__ __forceinline__ float2 block_sum_max(float2 v, float2* red2) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y = fmaxf(v.y, __shfl_xor_sync(0xffffffffu, v.y, o));
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red2[w] = v;
  __syncthreads();
  float2 t = l < (blockDim.x >> 5) ? red2[l] : make_float2(0.f, 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    t.x += __shfl_xor_sync(0xffffffffu, t.x, o);
    t.y = fmaxf(t.y, __shfl_xor_sync(0xffffffffu, t.y, o));
  }
  return t;  // every warp reduces the partials itself: no second barrier
}

template <int NV>
__global__ void __launch_bounds__(kRowThreads) ln_mod_reg_kernel(const float* __restrict__ x, int64_t ldx, int C,
                                                                 const float* __restrict__ scale,
                                                                 const float* __restrict__ shift, float eps,
                                                                 __nv_bfloat16* __restrict__ y, int64_t ldy) {
  __shared__ float2 red2[2][32];
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * ldx;
  float4 v[NV];
  float s = 0.f, amax = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = (threadIdx.x + k * kRowThreads) * 4;
    v[k] = i < C ? *reinterpret_cast<const float4*>(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
  }
  const float2 sm = block_sum_max(make_float2(s, amax), red2[0]);
  const float mean = sm.x / C;
  // 2^-e with 2^e the power of two at or below amax, when amax > 2^48 (else 1)
  const float sc = (sm.y > 281474976710656.0f && sm.y <= 3.4028235e38f)
                       ? __uint_as_float((254u - ((__float_as_uint(sm.y) >> 23) & 0xFFu)) << 23)
                       : 1.0f;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = (threadIdx.x + k * kRowThreads) * 4;
    if (i < C) {
      const float a = (v[k].x - mean) * sc, b = (v[k].y - mean) * sc, c = (v[k].z - mean) * sc,
                  d = (v[k].w - mean) * sc;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float inv = rsqrtf(block_sum_max(make_float2(q, 0.f), red2[1]).x / C + eps * sc * sc) * sc;
  __nv_bfloat16* yr = y + static_cast<int64_t>(blockIdx.x) * ldy;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = (threadIdx.x + k * kRowThreads) * 4;
    if (i < C) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(scale + i));
      const float4 h = __ldg(reinterpret_cast<const float4*>(shift + i));
      const float o0 = fmaf(1.f + g.x, (v[k].x - mean) * inv, h.x);
      const float o1 = fmaf(1.f + g.y, (v[k].y - mean) * inv, h.y);
      const float o2 = fmaf(1.f + g.z, (v[k].z - mean) * inv, h.z);
      const float o3 = fmaf(1.f + g.w, (v[k].w - mean) * inv, h.w);
      *reinterpret_cast<uint2*>(yr + i) = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
    }
  }
}

__global__ void gate_add_kernel(float* __restrict__ x, int64_t ldx, int rows, int C, const float* __restrict__ gate,
                                const uint16_t* __restrict__ v, int64_t ldv, float scale) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * C) return;
  const int64_t r = idx / C;
  const int c = static_cast<int>(idx % C);
  float* xp = x + r * ldx + c;
  *xp = fmaf(gate ? gate[c] : 1.f, __uint_as_float(static_cast<uint32_t>(v[r * ldv + c]) << 16) * scale, *xp);
}

// In place when lat_out == lat_in (each element reads then writes itself).
__global__ void euler_kernel(const float* lat_in, const float* __restrict__ v, const float* __restrict__ dt_p,
                             int64_t n, float* lat_out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const float dt = *dt_p;
  if (i < n) lat_out[i] = fmaf(dt, v[i], lat_in[i]);
}

__global__ void timestep_kernel(const float* __restrict__ t_p, int dim, float* __restrict__ out) {
  const float t = *t_p;
  const int half = dim / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float freq = expf(-logf(10000.0f) * static_cast<float>(i) / static_cast<float>(half));
    const float arg = t * freq;
    out[i] = cosf(arg);
    out[half + i] = sinf(arg);
  }
  if (dim % 2 && threadIdx.x == 0) out[dim - 1] = 0.f;
}

__global__ void set_scalar_kernel(float* dst, float v) { *dst = v; }

// cur[0..1] = steps[2i .. 2i+1] for i = (*counter)++ (the per-step scalars of a replayed step).
__global__ void step_select_kernel(const float* __restrict__ steps, int* counter, float* __restrict__ cur) {
  const int i = *counter;
  cur[0] = steps[2 * i];
  cur[1] = steps[2 * i + 1];
  *counter = i + 1;
}

// silu in f32 (dd_silu_f32, DirectDiTKernels.swift:175-184; DirectConditioner.silu :135-149).
__global__ void silu_f32_kernel(const float* __restrict__ x, int n, float* __restrict__ y) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = x[i];
    y[i] = v / (1.f + expf(-v));
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, int64_t n, uint16_t* __restrict__ y) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = static_cast<uint16_t>(pack_bf16x2(x[i], 0.f) & 0xFFFFu);
}

__global__ void bf16_to_f32_rows_kernel(const uint16_t* __restrict__ x, int64_t ldx, int rows, int cols,
                                        float* __restrict__ y, int64_t ldy) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * cols) return;
  const int64_t r = idx / cols;
  const int c = static_cast<int>(idx % cols);
  y[r * ldy + c] = __uint_as_float(static_cast<uint32_t>(x[r * ldx + c]) << 16);
}

unsigned blocks_for(int64_t n, int threads) { return static_cast<unsigned>((n + threads - 1) / threads); }

}  // namespace

int ln_mod(aex_ctx* ctx, const float* x, int64_t ldx, int rows, int C, const float* scale, const float* shift,
           float eps, void* y, int64_t ldy, cudaStream_t s) {
  if (rows <= 0) return AEX_OK;
  if (C % 4 || ldx % 4 || ldy % 4) return set_error(ctx, AEX_ERR_INVALID_ARG, "ln_mod: C and pitches must be multiples of 4");
  __nv_bfloat16* yb = static_cast<__nv_bfloat16*>(y);
  const int nv = (C + 4 * kRowThreads - 1) / (4 * kRowThreads);  // float4 per thread to hold the row
  if (nv <= 1)
    ln_mod_reg_kernel<1><<<rows, kRowThreads, 0, s>>>(x, ldx, C, scale, shift, eps, yb, ldy);
  else if (nv <= 2)
    ln_mod_reg_kernel<2><<<rows, kRowThreads, 0, s>>>(x, ldx, C, scale, shift, eps, yb, ldy);
  else if (nv <= 3)
    ln_mod_reg_kernel<3><<<rows, kRowThreads, 0, s>>>(x, ldx, C, scale, shift, eps, yb, ldy);
  else if (nv <= 4)
    ln_mod_reg_kernel<4><<<rows, kRowThreads, 0, s>>>(x, ldx, C, scale, shift, eps, yb, ldy);
  else
    ln_mod_kernel<<<rows, kRowThreads, 0, s>>>(x, ldx, C, scale, shift, eps, yb, ldy);
  return check_launch(ctx, "ln_mod_kernel");
}


int gate_add(aex_ctx* ctx, float* x, int64_t ldx, int rows, int C, const float* gate, const void* v, int64_t ldv,
             float scale, cudaStream_t s) {
  if (rows <= 0) return AEX_OK;
  const int64_t n = static_cast<int64_t>(rows) * C;
  gate_add_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, ldx, rows, C, gate, static_cast<const uint16_t*>(v), ldv,
                                                      scale);
  return check_launch(ctx, "gate_add_kernel");
}

int euler(aex_ctx* ctx, const float* lat_in, const float* v, const float* dt, int64_t n, float* lat_out,
          cudaStream_t s) {
  euler_kernel<<<blocks_for(n, 256), 256, 0, s>>>(lat_in, v, dt, n, lat_out);
  return check_launch(ctx, "euler_kernel");
}

int timestep_embedding(aex_ctx* ctx, const float* t, int dim, float* out, cudaStream_t s) {
  timestep_kernel<<<1, 128, 0, s>>>(t, dim, out);
  return check_launch(ctx, "timestep_kernel");
}

int set_scalar(aex_ctx* ctx, float* dst, float v, cudaStream_t s) {
  set_scalar_kernel<<<1, 1, 0, s>>>(dst, v);
  return check_launch(ctx, "set_scalar_kernel");
}

int step_select(aex_ctx* ctx, const float* steps, int* counter, float* cur, cudaStream_t s) {
  step_select_kernel<<<1, 1, 0, s>>>(steps, counter, cur);
  return check_launch(ctx, "step_select_kernel");
}

int silu_f32(aex_ctx* ctx, const float* x, int n, float* y, cudaStream_t s) {
  silu_f32_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, n, y);
  return check_launch(ctx, "silu_f32_kernel");
}

int f32_to_bf16(aex_ctx* ctx, const float* x, int64_t n, void* y, cudaStream_t s) {
  f32_to_bf16_kernel<<<blocks_for(n, 256), 256, 0, s>>>(x, n, static_cast<uint16_t*>(y));
  return check_launch(ctx, "f32_to_bf16_kernel");
}

int bf16_to_f32_rows(aex_ctx* ctx, const void* x, int64_t ldx, int rows, int cols, float* y, int64_t ldy,
                     cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(rows) * cols;
  bf16_to_f32_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(static_cast<const uint16_t*>(x), ldx, rows, cols, y,
                                                              ldy);
  return check_launch(ctx, "bf16_to_f32_rows_kernel");
}

}  // namespace glue
}  // namespace aex
