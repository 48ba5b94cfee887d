/*
 * aex_oracle.h — CPU restatement of the reference (PowerBeef/Aestrix,
 * "Imarello") arithmetic on the B200 hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for
 * libaestrix_cuda and the timed CPU baseline of bench.py. Nothing in the product
 * path (aestrix_b200/, include/) links, loads or calls it.
 *
 * Pinning: the reference (Swift + MLX + Metal) cannot run here. The functions
 * below are pinned against the reference's own known-answer tests
 * (Tests/ImarelloCoreTests/Flux2MathTests.swift) and against values derived by
 * hand from its CPU dequant (Sources/ImarelloDirect/DirectTEEncoder.swift:39-46,
 * 104-123); the golden fixtures live in tests/golden/. The attention reference
 * is the fp32 formula of Tests/ImarelloDiTTests/MetalFlashAttentionTests.swift:
 * 10-17, softmax(scale * Q K^T) V.
 *
 * All arrays are row-major host memory. bf16 values are uint16_t bit patterns.
 */
#ifndef AEX_ORACLE_H
#define AEX_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DirectTEEncoder.f32ToBF16 (DirectTEEncoder.swift:39-43): round-to-nearest-even
 * by adding 0x7FFF + lsb and truncating (no NaN special case, as in the
 * reference). */
uint16_t aexo_f32_to_bf16(float v);
/* DirectTEEncoder.bf16ToF32 (DirectTEEncoder.swift:44-46). */
float aexo_bf16_to_f32(uint16_t u);
void aexo_f32_to_bf16_array(const float* x, size_t n, uint16_t* out);
void aexo_bf16_to_f32_array(const uint16_t* x, size_t n, float* out);

/* MLX affine 4-bit dequant, restating DirectTEEncoder.embedRow
 * (DirectTEEncoder.swift:104-123) over a whole [n, k] matrix:
 * q = (packed[n, (c)/8] >> 4*(c%8)) & 0xF, out = f32ToBF16(scale*q + bias)
 * with f32 multiply then f32 add (two roundings, no FMA). */
void aexo_dequant_q4(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int n, int k,
                     int group_size, uint16_t* out_bf16);

/* MLX `quantize(bits: 4, groupSize: gs)` affine packing, used to build
 * synthetic weights: codes [n, k] in 0..15 packed LSB-first, 8 per uint32. */
void aexo_pack_q4(const uint8_t* codes, int n, int k, uint32_t* packed);

/* y[m, n] = x[m, k] . deq(W)[n, k]^T with deq(W) rounded to bf16 exactly as
 * aexo_dequant_q4 and f64 accumulation (quantizedMM(transpose: true),
 * Sources/ImarelloDiT/AttentionUtils.swift:212-221). x is f32 (pass bf16
 * values widened to f32 to model a bf16 activation). OpenMP over rows of W. */
void aexo_qmm(const float* x, int m, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
              int n, int k, int group_size, float* y);

/* The quantized matrix-vector product of MLX's qmv on f32 activations (the
 * conditioner's affine_qmm_t_float_gs_64_b_4, DirectConditioner.swift:48,
 * 183-190): per group, scale * sum(x * q) + bias * sum(x), i.e. the unrounded
 * dequantized weights, f64 accumulation. */
void aexo_qmv(const float* x, int m, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int n,
              int k, int group_size, float* y);

/* Flux2RoPE.rope1D / frequencies (Sources/ImarelloCore/Flux2RoPE.swift:16-76):
 * ids [n, n_axes] f32; for each axis of dimension dim_a and i < dim_a/2:
 * omega = 1/pow(theta, 2i/dim_a), angle = pos*omega; cos/sin [n, sum(dim_a/2)]. */
void aexo_rope_freqs(const float* ids, int n, float theta, const int* axes_dim, int n_axes, float* cos_out,
                     float* sin_out);

/* Flux2RoPE.prepareGridIDs (Flux2RoPE.swift:78-89): rows [t, h, w, layer]. */
void aexo_grid_ids(int height, int width, float t_coord, float layer, float* ids_out);
/* Flux2RoPE.prepareTextIDs (Flux2RoPE.swift:91-95): rows [0, 0, 0, i]. */
void aexo_text_ids(int length, float* ids_out);

/* MLXNN.RMSNorm over the last dim of rows [rows, d] (JointAttention.swift:31-36):
 * y = x * (1/sqrt(mean(x^2) + eps)) * w, f32 in/out, f64 sum of squares. */
void aexo_rmsnorm(const float* x, int rows, int d, const float* w, float eps, float* y);

/* Interleaved-pair rotation of rows [s, h, d] in place with cos/sin [s, d/2]
 * (AttentionUtils.compiledRopeMix, AttentionUtils.swift:283-297):
 * out0 = re*cos - im*sin, out1 = im*cos + re*sin. */
void aexo_rope_apply(float* x, int s, int h, int d, const float* cos_t, const float* sin_t);

/* softmax(scale * Q K^T) V over [b, s, h, d] tensors with element strides
 * (stride_b, stride_s, stride_h), dim stride 1. f32 math with f64 row sums.
 * Only query rows [q_begin, q_end) of every (batch, head) are computed (the
 * rest of `out` is untouched) so large shapes can be sampled. OpenMP. */
void aexo_sdpa(const float* q, const float* k, const float* v, float* out, int b, int s, int h, int d,
               int64_t stride_b, int64_t stride_s, int64_t stride_h, float scale, int q_begin, int q_end);

/* The joint attention composition of Flux2Attention / the direct engine
 * (JointAttention.swift:44-110, DirectDiTStep.swift:546-588) on [b, s, h, d]
 * contiguous f32 tensors: RMSNorm(q) and RMSNorm(k) per head (if the weight is
 * non-NULL), interleaved RoPE with cos/sin [s, d/2] (if non-NULL), then SDPA.
 * q/k are copied, not modified. Rows [q_begin, q_end) only. */
void aexo_joint_attention(const float* q, const float* k, const float* v, float* out, int b, int s, int h, int d,
                          const float* norm_q_w, const float* norm_k_w, float eps, const float* cos_t,
                          const float* sin_t, float scale, int q_begin, int q_end);

/* Flux2Scheduler (Sources/ImarelloCore/Flux2Scheduler.swift:56-109). */
float aexo_linear_mu(int image_seq_len, int base_seq_len, int max_seq_len, float base_shift, float max_shift);
float aexo_time_shift(float mu, float t, float sigma_power);
/* sigmas [steps+1] (terminal 0), timesteps [steps]. */
void aexo_schedule(int steps, int image_seq_len, float* sigmas, float* timesteps);
/* Flux2TimestepEmbedding.embed (Flux2TimestepEmbedding.swift:16-52), flip_sin_to_cos. */
void aexo_timestep_embedding(const float* t, int n, int dim, float* out);

/* Glue of the direct engine (Sources/ImarelloDirect/DirectDiTKernels.swift):
 * LayerNorm (no affine, eps) + AdaLN modulate: y = (1+scale)*n + shift (:15-57, without the /16). */
void aexo_ln_mod(const float* x, int rows, int d, const float* scale, const float* shift, float eps, float* y);
/* silu(g) * u (:138-159, FeedForward.swift:11-24). */
void aexo_swiglu(const float* g, const float* u, size_t n, float* y);
/* y = x + gate (.) v per row (:208-221). */
void aexo_gate_add(const float* x, const float* gate, const float* v, int rows, int d, float* y);

#ifdef __cplusplus
}
#endif
#endif
