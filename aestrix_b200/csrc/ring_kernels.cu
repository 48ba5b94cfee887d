// ring_kernels.cu — merging partial attention results of different K/V shards
// (the ring-attention accumulation step). Each hop's attention kernel writes a
// normalized partial output O_h (bf16) and its per-row log2-sum-exp lse_h; the
// running result is
//   lse = log2(2^lse_acc + 2^lse_h),
//   O   = (2^(lse_acc - lse) O_acc + 2^(lse_h - lse) O_h),
// i.e. the online-softmax rescaling of FlashAttention applied across shards.
#include "internal.h"
#include "sm100.cuh"

namespace aex {
namespace ring {
namespace {

// One thread per (token s, head h, 8 columns).
__global__ void merge_kernel(const uint16_t* __restrict__ o_h, int64_t oh_ss, int64_t oh_sh,
                             const float* __restrict__ lse_h, const float* __restrict__ lse_in,
                             float* __restrict__ lse_out, float* __restrict__ o_acc, int S, int H, int first, int final,
                             uint16_t* __restrict__ out, int64_t out_ss, int64_t out_sh) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(S) * H * 16) return;
  const int c = static_cast<int>(idx & 15);
  const int64_t sh = idx >> 4;
  const int h = static_cast<int>(sh % H);
  const int s = static_cast<int>(sh / H);
  const float lh = lse_h[static_cast<int64_t>(h) * S + s];
  const uint4 raw = *reinterpret_cast<const uint4*>(o_h + s * oh_ss + h * oh_sh + c * 8);
  const uint32_t rv[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16lo_to_f32(rv[i]);
    v[2 * i + 1] = bf16hi_to_f32(rv[i]);
  }
  float* acc = o_acc + (static_cast<int64_t>(s) * H + h) * 128 + c * 8;
  float lse_new = lh;
  if (!first) {
    const float la = lse_in[static_cast<int64_t>(h) * S + s];
    const float mx = fmaxf(la, lh);
    const float wa = exp2f(la - mx), wh = exp2f(lh - mx);
    const float inv = 1.f / (wa + wh);
    lse_new = mx + log2f(wa + wh);
    const float4 a0 = *reinterpret_cast<const float4*>(acc);
    const float4 a1 = *reinterpret_cast<const float4*>(acc + 4);
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (av[i] * wa + v[i] * wh) * inv;
  }
  if (final) {
    *reinterpret_cast<uint4*>(out + s * out_ss + h * out_sh + c * 8) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  } else {
    *reinterpret_cast<float4*>(acc) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(acc + 4) = make_float4(v[4], v[5], v[6], v[7]);
    if (c == 0) lse_out[static_cast<int64_t>(h) * S + s] = lse_new;
  }
}

// One thread per (token s, head h, 8 columns): all k ranges at once. Range r's
// partial output sits at o + r * o_rs (token stride o_ss, head stride o_sh) and
// its log2-sum-exp at lse[r * lse_rs + h * S + s].
constexpr int kMaxSplits = 16;
__global__ void merge_splits_kernel(const uint16_t* __restrict__ o, int64_t o_rs, int64_t o_ss, int64_t o_sh,
                                    const float* __restrict__ lse, int64_t lse_rs, int k, int S, int H,
                                    uint16_t* __restrict__ out, int64_t out_ss, int64_t out_sh) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(S) * H * 16) return;
  const int c = static_cast<int>(idx & 15);
  const int64_t sh = idx >> 4;
  const int h = static_cast<int>(sh % H);
  const int s = static_cast<int>(sh / H);
  float mx = -INFINITY;
  for (int r = 0; r < k; ++r) mx = fmaxf(mx, lse[r * lse_rs + static_cast<int64_t>(h) * S + s]);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  for (int r = 0; r < k; ++r) {
    const float w = exp2f(lse[r * lse_rs + static_cast<int64_t>(h) * S + s] - mx);
    wsum += w;
    const uint4 raw = *reinterpret_cast<const uint4*>(o + r * o_rs + s * o_ss + h * o_sh + c * 8);
    const uint32_t rv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] += w * bf16lo_to_f32(rv[i]);
      acc[2 * i + 1] += w * bf16hi_to_f32(rv[i]);
    }
  }
  const float inv = 1.f / wsum;
  *reinterpret_cast<uint4*>(out + s * out_ss + h * out_sh + c * 8) =
      make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                 pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
}

}  // namespace

int merge_splits(aex_ctx* ctx, const void* o, int64_t o_rs, int64_t o_ss, int64_t o_sh, const float* lse,
                 int64_t lse_rs, int k, int S, int H, void* out, int64_t out_ss, int64_t out_sh, cudaStream_t s) {
  if (k < 1 || k > kMaxSplits) return set_error(ctx, AEX_ERR_INVALID_ARG, "merge_splits: %d ranges (1..%d)", k, kMaxSplits);
  const int64_t n = static_cast<int64_t>(S) * H * 16;
  merge_splits_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
      static_cast<const uint16_t*>(o), o_rs, o_ss, o_sh, lse, lse_rs, k, S, H, static_cast<uint16_t*>(out), out_ss,
      out_sh);
  return check_launch(ctx, "merge_splits_kernel");
}

int merge(aex_ctx* ctx, const void* o_h, int64_t oh_ss, int64_t oh_sh, const float* lse_h, const float* lse_in,
          float* lse_out, float* o_acc, int S, int H, bool first, bool final, void* out, int64_t out_ss, int64_t out_sh,
          cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(S) * H * 16;
  merge_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
      static_cast<const uint16_t*>(o_h), oh_ss, oh_sh, lse_h, lse_in, lse_out, o_acc, S, H, first ? 1 : 0,
      final ? 1 : 0, static_cast<uint16_t*>(out), out_ss, out_sh);
  return check_launch(ctx, "ring merge_kernel");
}

}  // namespace ring
}  // namespace aex
