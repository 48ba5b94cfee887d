// attention_sm100.cu — K1: fused QK-RMSNorm + 2-D axial RoPE + non-causal
// flash attention for head_dim 128 on sm_100a.
//
// Replaces the reference composition AttentionUtils.processQKV (norm step,
// Sources/ImarelloDiT/AttentionUtils.swift:37-50) -> applyRopeBSHD
// (AttentionUtils.swift:263-298) -> MetalFlashAttention.scaledDotProductAttention
// (Sources/ImarelloDiT/MetalFlashAttention.swift:44-78), and the direct engine's
// rms / rope / attention dispatches (Sources/ImarelloDirect/DirectDiTStep.swift:
// 408-488).
//
// Two kernels:
//  * qk_prep_kernel — one warp per (operand, batch, token, head) row: f32
//    RMSNorm over the 128-wide head with the learned weight, then the
//    interleaved-pair rotation with the row's cos/sin, rounded once to bf16
//    into head-major scratch [B][H][S][128] (TMA-friendly: a 128-row tile is
//    one contiguous 32 KB block). HBM-bound.
//  * attn_fwd_kernel — one CTA per (256 query rows, head, batch), 10 warps:
//      warps 0-3  softmax warpgroup of query tile 0 (one query row per thread)
//      warps 4-7  softmax warpgroup of query tile 1
//      warp 8     TMA producer (Q tiles once, K/V blocks through a 4-slot ring)
//      warp 9     UMMA issuer (one thread)
//    Tensor memory (512 columns): S0 [0,128), S1 [128,256), O0 [256,384),
//    O1 [384,512). P_t is written as packed bf16 over the first 64 columns of
//    S_t and consumed from tensor memory by the P.V UMMA. While one warpgroup
//    runs its softmax the tensor core works on the other tile (ping-pong).
//    Rescaling of O is lazy: the running max only moves when a block's max
//    exceeds it by more than 2^8, so most blocks skip the O round trip.
//    The epilogue divides by the row sum, stages the tile in the (now free) Q
//    buffer with the 128-byte swizzle and writes it with TMA stores, so any
//    output row pitch that is a multiple of 16 bytes works (e.g. the 12288-wide
//    concat buffer of the single-stream block).
#include <cmath>

#include "internal.h"
#include "sm100.cuh"

namespace aex {
namespace attn {

constexpr int kD = 128;
constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // keys per block
constexpr int kTiles = 2;
constexpr int kStages = 4;
constexpr int kTileBytes = kBM * kD * 2;  // 32 KB, two 16 KB swizzle regions of 64 columns
constexpr int kRegionBytes = kTileBytes / 2;
constexpr int kThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;

constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kTiles * kTileBytes;
constexpr int kOffBar = kOffKV + kStages * kTileBytes;
// barrier indices
constexpr int kBarQFull = 0;                      // [2]
constexpr int kBarKVFull = 2;                     // [kStages]
constexpr int kBarKVEmpty = kBarKVFull + kStages; // [kStages]
constexpr int kBarSFull = kBarKVEmpty + kStages;  // [2]
constexpr int kBarPFull = kBarSFull + 2;          // [2]
constexpr int kBarOFull = kBarPFull + 2;          // [2]
constexpr int kBarDrain = kBarOFull + 2;          // [1]
constexpr int kNumBars = kBarDrain + 1;
constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, false, false);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, false, true);

struct Params {
  int seq;
  int n_kv;
  float scale_log2;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, Params p,
                    int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  __shared__ int abort_flag;

  const int warp = static_cast<int>(warp_id_uniform());
  const int lane = static_cast<int>(lane_id());
  const int q0 = blockIdx.x * (kTiles * kBM);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int n_kv = p.n_kv;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bars[kBarQFull + 0], 1);
    mbar_init(&bars[kBarQFull + 1], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kBarKVFull + s], 1);
      mbar_init(&bars[kBarKVEmpty + s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars[kBarSFull + t], 1);
      mbar_init(&bars[kBarPFull + t], 4);  // one arrive per softmax warp
      mbar_init(&bars[kBarOFull + t], 1);
    }
    mbar_init(&bars[kBarDrain], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0; t < kTiles; ++t) {
        uint8_t* dst = smem + kOffQ + t * kTileBytes;
        mbar_arrive_expect_tx(&bars[kBarQFull + t], kTileBytes);
        tma_load_4d(dst, &tm_q, &bars[kBarQFull + t], 0, q0 + t * kBM, h, b);
        tma_load_4d(dst + kRegionBytes, &tm_q, &bars[kBarQFull + t], 64, q0 + t * kBM, h, b);
      }
      const int n_loads = 2 * n_kv;  // K_0, V_0, K_1, V_1, ...
      int issued = 0;
      for (int idx = 0; idx < n_loads; ++idx) {
        const int slot = idx % kStages;
        const int use = idx / kStages;
        if (use > 0 && !mbar_wait(&bars[kBarKVEmpty + slot], (use - 1) & 1, &abort_flag, status, kDevTimeoutTma))
          break;
        const CUtensorMap* m = (idx & 1) ? &tm_v : &tm_k;
        const int kv0 = (idx >> 1) * kBN;
        uint8_t* dst = smem + kOffKV + slot * kTileBytes;
        mbar_arrive_expect_tx(&bars[kBarKVFull + slot], kTileBytes);
        tma_load_4d(dst, m, &bars[kBarKVFull + slot], 0, kv0, h, b);
        tma_load_4d(dst + kRegionBytes, m, &bars[kBarKVFull + slot], 64, kv0, h, b);
        issued = idx + 1;
      }
      if (abort_flag) {
        // Let every copy already issued land before the CTA releases its
        // shared memory (bounded: the waits themselves time out).
        for (int idx = (issued > kStages ? issued - kStages : 0); idx < issued; ++idx) {
          const uint32_t a = smem_u32(&bars[kBarKVFull + idx % kStages]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, (idx / kStages) & 1) && globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ UMMA issue
    if (lane == 0) {
      bool ok = mbar_wait(&bars[kBarQFull + 0], 0, &abort_flag, status, kDevTimeoutMma) &&
                mbar_wait(&bars[kBarQFull + 1], 0, &abort_flag, status, kDevTimeoutMma);
      const uint32_t sQ = smem_u32(smem + kOffQ);
      const uint32_t sKV = smem_u32(smem + kOffKV);
      auto issue_s = [&](int t, int slot) {
        const uint32_t qa = sQ + t * kTileBytes;
        const uint32_t ka = sKV + slot * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kRegionBytes + (kk & 3) * 32;
          umma_ss(tmem + t * 128, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), kIdescS,
                  kk > 0);
        }
      };
      auto issue_pv = [&](int t, int slot, bool accumulate) {
        const uint32_t va = sKV + slot * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, sdesc_sw128(va + kk * 2048, kRegionBytes, 1024),
                  kIdescPV, (accumulate || kk > 0) ? 1u : 0u);
      };
      if (ok) ok = mbar_wait(&bars[kBarKVFull + 0], 0, &abort_flag, status, kDevTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        umma_commit(&bars[kBarSFull + 0]);
        issue_s(1, 0);
        umma_commit(&bars[kBarSFull + 1]);
        umma_commit(&bars[kBarKVEmpty + 0]);
      }
      for (int j = 1; j < n_kv && ok; ++j) {
        const int kidx = 2 * j, vidx = 2 * j - 1;
        const int kslot = kidx % kStages, vslot = vidx % kStages;
        ok = mbar_wait(&bars[kBarKVFull + kslot], (kidx / kStages) & 1, &abort_flag, status, kDevTimeoutMma) &&
             mbar_wait(&bars[kBarKVFull + vslot], (vidx / kStages) & 1, &abort_flag, status, kDevTimeoutMma);
        for (int t = 0; t < kTiles && ok; ++t) {
          ok = mbar_wait(&bars[kBarPFull + t], (j - 1) & 1, &abort_flag, status, kDevTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, vslot, j - 1 > 0);
          issue_s(t, kslot);
          umma_commit(&bars[kBarSFull + t]);
        }
        if (ok) {
          umma_commit(&bars[kBarKVEmpty + vslot]);
          umma_commit(&bars[kBarKVEmpty + kslot]);
        }
      }
      if (ok) {
        const int vidx = 2 * n_kv - 1;
        const int vslot = vidx % kStages;
        ok = mbar_wait(&bars[kBarKVFull + vslot], (vidx / kStages) & 1, &abort_flag, status, kDevTimeoutMma);
        for (int t = 0; t < kTiles && ok; ++t) {
          ok = mbar_wait(&bars[kBarPFull + t], (n_kv - 1) & 1, &abort_flag, status, kDevTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, vslot, n_kv - 1 > 0);
          umma_commit(&bars[kBarOFull + t]);
        }
      }
      // Drain: whatever was issued completes before tensor memory is freed.
      umma_commit(&bars[kBarDrain]);
      mbar_wait(&bars[kBarDrain], 0, &abort_flag, status, kDevTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;
    const int quad = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + t * 128;
    const uint32_t tO = tmem + lane_base + 256 + t * 128;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait(&bars[kBarSFull + t], j & 1, &abort_flag, status, kDevTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t r[128];
      tmem_ld32(tS + 0, r + 0);
      tmem_ld32(tS + 32, r + 32);
      tmem_ld32(tS + 64, r + 64);
      tmem_ld32(tS + 96, r + 96);
      tmem_wait_ld();
      const int valid = p.seq - j * kBN;
      if (valid < kBN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= valid) r[i] = __float_as_uint(-INFINITY);
      }
      float mx0 = __uint_as_float(r[0]), mx1 = __uint_as_float(r[1]);
#pragma unroll
      for (int i = 2; i < 128; i += 2) {
        mx0 = fmaxf(mx0, __uint_as_float(r[i]));
        mx1 = fmaxf(mx1, __uint_as_float(r[i + 1]));
      }
      const float m_blk = fmaxf(mx0, mx1) * sl2;
      float alpha = 1.f;
      bool rescale = false;
      if (m_blk > m_run + 8.f) {
        alpha = ex2_approx(m_run - m_blk);
        m_run = m_blk;
        rescale = (j > 0);
      }
      l_run *= alpha;
      const float neg_m = -m_run;
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(r[c * 32 + 2 * i]), sl2, neg_m));
          const float p1 = ex2_approx(fmaf(__uint_as_float(r[c * 32 + 2 * i + 1]), sl2, neg_m));
          sum0 += p0;
          sum1 += p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tS + c * 16, pk);
      }
      l_run += sum0 + sum1;
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t o[32];
          tmem_ld32(tO + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarPFull + t]);
    }
    // ------------------------------------------------------------ epilogue
    if (ok) ok = mbar_wait(&bars[kBarOFull + t], 0, &abort_flag, status, kDevTimeoutEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    uint8_t* stage = smem + kOffQ + t * kTileBytes;  // Q_t is dead once O_t is final
    const int row = quad * 32 + lane;
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t o[32];
        tmem_ld32(tO + c, o);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
        uint8_t* rowp = stage + (c >> 6) * kRegionBytes + row * 128;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int chunk = (((c & 63) >> 3) + qd) ^ (row & 7);
          *reinterpret_cast<uint4*>(rowp + chunk * 16) =
              make_uint4(pk[4 * qd], pk[4 * qd + 1], pk[4 * qd + 2], pk[4 * qd + 3]);
        }
      }
      fence_async_shared();
    }
    named_bar_sync(1 + t, 128);
    if (ok && quad == 0 && lane == 0 && q0 + t * kBM < p.seq) {
      tma_store_4d(&tm_o, stage, 0, q0 + t * kBM, h, b);
      tma_store_4d(&tm_o, stage + kRegionBytes, 64, q0 + t * kBM, h, b);
      bulk_commit_group();
      bulk_wait_group_read0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ prep
struct PrepParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  const float* wq;
  const float* wk;
  const float* cos_t;
  const float* sin_t;
  float eps;
  int batch, seq, heads;
  __nv_bfloat16* out;  // [2][B][H][S][128]
};

__global__ void __launch_bounds__(256) qk_prep_kernel(PrepParams p) {
  const int64_t rows_per_op = static_cast<int64_t>(p.batch) * p.seq * p.heads;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= 2 * rows_per_op) return;
  const int lane = threadIdx.x & 31;
  const int which = row >= rows_per_op ? 1 : 0;
  const int64_t r = row - which * rows_per_op;
  const int hh = static_cast<int>(r % p.heads);
  const int s = static_cast<int>((r / p.heads) % p.seq);
  const int bb = static_cast<int>(r / (static_cast<int64_t>(p.heads) * p.seq));
  const __nv_bfloat16* src = which ? p.k + bb * p.k_sb + s * p.k_ss + hh * p.k_sh
                                   : p.q + bb * p.q_sb + s * p.q_ss + hh * p.q_sh;
  const float* w = which ? p.wk : p.wq;
  const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
  float x0 = bf16lo_to_f32(raw.x), x1 = bf16hi_to_f32(raw.x);
  float x2 = bf16lo_to_f32(raw.y), x3 = bf16hi_to_f32(raw.y);
  if (w) {
    float ss = x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss * (1.0f / kD) + p.eps);
    const float4 wv = *reinterpret_cast<const float4*>(w + lane * 4);
    x0 = x0 * inv * wv.x;
    x1 = x1 * inv * wv.y;
    x2 = x2 * inv * wv.z;
    x3 = x3 * inv * wv.w;
  }
  if (p.cos_t) {
    const float2 c = *reinterpret_cast<const float2*>(p.cos_t + static_cast<int64_t>(s) * (kD / 2) + lane * 2);
    const float2 sn = *reinterpret_cast<const float2*>(p.sin_t + static_cast<int64_t>(s) * (kD / 2) + lane * 2);
    const float y0 = x0 * c.x - x1 * sn.x, y1 = x1 * c.x + x0 * sn.x;
    const float y2 = x2 * c.y - x3 * sn.y, y3 = x3 * c.y + x2 * sn.y;
    x0 = y0;
    x1 = y1;
    x2 = y2;
    x3 = y3;
  }
  __nv_bfloat16* dst = p.out + which * rows_per_op * kD +
                       ((static_cast<int64_t>(bb) * p.heads + hh) * p.seq + s) * kD + lane * 4;
  *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(x0, x1), pack_bf16x2(x2, x3));
}

}  // namespace attn

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate(aex_ctx* ctx, const aex_attention_args* a) {
  if (!a) return set_error(ctx, AEX_ERR_INVALID_ARG, "args is NULL");
  if (a->head_dim != 128)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "head_dim %d unsupported (only 128)", a->head_dim);
  if (a->batch <= 0 || a->seq <= 0 || a->heads <= 0)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "batch/seq/heads must be positive (%d, %d, %d)", a->batch, a->seq,
                     a->heads);
  if (a->batch > 65535 || a->heads > 65535)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "batch/heads above 65535");
  const aex_bshd* ts[4] = {&a->q, &a->k, &a->v, &a->out};
  const char* names[4] = {"q", "k", "v", "out"};
  for (int i = 0; i < 4; ++i) {
    if (!ts[i]->data) return set_error(ctx, AEX_ERR_INVALID_ARG, "%s.data is NULL", names[i]);
    if (!aligned16(ts[i]->data))
      return set_error(ctx, AEX_ERR_INVALID_ARG, "%s.data is not 16-byte aligned", names[i]);
    if (ts[i]->stride_s % 8 || ts[i]->stride_h % 8 || ts[i]->stride_b % 8 || ts[i]->stride_s <= 0 ||
        ts[i]->stride_h <= 0 || ts[i]->stride_b <= 0)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "%s strides must be positive multiples of 8 elements", names[i]);
  }
  if ((a->rope_cos == nullptr) != (a->rope_sin == nullptr))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "rope_cos and rope_sin must both be set or both be NULL");
  const void* ws[4] = {a->norm_q_weight, a->norm_k_weight, a->rope_cos, a->rope_sin};
  for (const void* w : ws)
    if (w && !aligned16(w)) return set_error(ctx, AEX_ERR_INVALID_ARG, "norm/rope tables must be 16-byte aligned");
  if ((a->norm_q_weight || a->norm_k_weight) && !(a->eps >= 0.f))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "eps must be >= 0");
  return AEX_OK;
}

bool needs_prep(const aex_attention_args* a) {
  return a->norm_q_weight || a->norm_k_weight || a->rope_cos;
}

int bshd_tmap(aex_ctx* ctx, CUtensorMap* m, const void* base, int64_t sb, int64_t ss, int64_t sh, int batch,
              int seq, int heads) {
  uint64_t dims[4] = {128, static_cast<uint64_t>(seq), static_cast<uint64_t>(heads), static_cast<uint64_t>(batch)};
  uint64_t strides[3] = {static_cast<uint64_t>(ss) * 2, static_cast<uint64_t>(sh) * 2,
                         static_cast<uint64_t>(sb) * 2};
  uint32_t box[4] = {64, 128, 1, 1};
  return make_tmap(ctx, m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, 4, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

int joint_attention_impl(aex_ctx* ctx, const aex_attention_args* a, void* scratch, size_t scratch_bytes,
                         cudaStream_t stream) {
  const int B = a->batch, S = a->seq, H = a->heads;
  const void* qsrc = a->q.data;
  const void* ksrc = a->k.data;
  int64_t qs[3] = {a->q.stride_b, a->q.stride_s, a->q.stride_h};
  int64_t ks[3] = {a->k.stride_b, a->k.stride_s, a->k.stride_h};
  if (needs_prep(a)) {
    const size_t need = aex_joint_attention_scratch_bytes(a);
    if (!scratch || scratch_bytes < need)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "scratch of %zu bytes is smaller than the %zu needed", scratch_bytes,
                       need);
    if (reinterpret_cast<uintptr_t>(scratch) % 256)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "scratch must be 256-byte aligned");
    attn::PrepParams pp{};
    pp.q = static_cast<const __nv_bfloat16*>(a->q.data);
    pp.k = static_cast<const __nv_bfloat16*>(a->k.data);
    pp.q_sb = a->q.stride_b;
    pp.q_ss = a->q.stride_s;
    pp.q_sh = a->q.stride_h;
    pp.k_sb = a->k.stride_b;
    pp.k_ss = a->k.stride_s;
    pp.k_sh = a->k.stride_h;
    pp.wq = a->norm_q_weight;
    pp.wk = a->norm_k_weight;
    pp.cos_t = a->rope_cos;
    pp.sin_t = a->rope_sin;
    pp.eps = a->eps;
    pp.batch = B;
    pp.seq = S;
    pp.heads = H;
    pp.out = static_cast<__nv_bfloat16*>(scratch);
    const int64_t rows = 2ll * B * S * H;
    const int64_t blocks = (rows + 7) / 8;
    if (blocks > 0x7FFFFFFFll) return set_error(ctx, AEX_ERR_INVALID_ARG, "problem too large");
    attn::qk_prep_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(pp);
    if (int r = check_launch(ctx, "qk_prep_kernel")) return r;
    const int64_t plane = static_cast<int64_t>(B) * H * S * 128;
    qsrc = scratch;
    ksrc = static_cast<const __nv_bfloat16*>(scratch) + plane;
    qs[0] = static_cast<int64_t>(H) * S * 128;
    qs[1] = 128;
    qs[2] = static_cast<int64_t>(S) * 128;
    ks[0] = qs[0];
    ks[1] = qs[1];
    ks[2] = qs[2];
  }
  CUtensorMap tq, tk, tv, to;
  if (int r = bshd_tmap(ctx, &tq, qsrc, qs[0], qs[1], qs[2], B, S, H)) return r;
  if (int r = bshd_tmap(ctx, &tk, ksrc, ks[0], ks[1], ks[2], B, S, H)) return r;
  if (int r = bshd_tmap(ctx, &tv, a->v.data, a->v.stride_b, a->v.stride_s, a->v.stride_h, B, S, H)) return r;
  if (int r = bshd_tmap(ctx, &to, a->out.data, a->out.stride_b, a->out.stride_s, a->out.stride_h, B, S, H)) return r;
  attn::Params prm{};
  prm.seq = S;
  prm.n_kv = (S + attn::kBN - 1) / attn::kBN;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / std::sqrt(128.0f);
  prm.scale_log2 = scale * 1.4426950408889634f;
  static bool attr_set = false;
  if (!attr_set) {
    AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(attn::attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           attn::kSmemBytes));
    attr_set = true;
  }
  dim3 grid((S + attn::kTiles * attn::kBM - 1) / (attn::kTiles * attn::kBM), H, B);
  attn::attn_fwd_kernel<<<grid, attn::kThreads, attn::kSmemBytes, stream>>>(tq, tk, tv, to, prm, ctx->d_status);
  return check_launch(ctx, "attn_fwd_kernel");
}

}  // namespace aex

extern "C" {

size_t aex_joint_attention_scratch_bytes(const aex_attention_args* a) {
  if (!a || !(a->norm_q_weight || a->norm_k_weight || a->rope_cos)) return 0;
  if (a->batch <= 0 || a->seq <= 0 || a->heads <= 0) return 0;
  return 2ull * static_cast<size_t>(a->batch) * a->heads * a->seq * 128 * 2;
}

int aex_joint_attention_ws(aex_ctx* ctx, const aex_attention_args* args, void* scratch, size_t scratch_bytes,
                           aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (int r = validate(ctx, args)) return r;
  if (int r = bind_device(ctx)) return r;
  return joint_attention_impl(ctx, args, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

int aex_joint_attention(aex_ctx* ctx, const aex_attention_args* args, aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (int r = validate(ctx, args)) return r;
  if (int r = bind_device(ctx)) return r;
  const size_t need = aex_joint_attention_scratch_bytes(args);
  void* ws = nullptr;
  if (int r = ensure_scratch(ctx, need, &ws)) return r;
  return joint_attention_impl(ctx, args, ws, need, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
