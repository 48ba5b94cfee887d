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
//  * qk_prep_kernel — one half-warp per (operand, batch, token, head) row: f32
//    RMSNorm over the 128-wide head with the learned weight, then the
//    interleaved-pair rotation with the row's cos/sin, rounded once to bf16
//    into scratch: token-major [B][S][H][128] for the fused call (the input's
//    row order, so its writes are sequential), head-major [B][H][S][128] for
//    the sequence-parallel slots. HBM-bound.
//  * attn_fwd_kernel — one CTA per (256 query rows, head, batch), 12 warps:
//      warps 0-3   softmax warpgroup of query tile 0 (one query row per thread)
//      warps 4-7   softmax warpgroup of query tile 1
//      warp 8      TMA producer (Q tiles once, K/V blocks through a 5-slot ring)
//      warp 9      UMMA issuer (one thread)
//      warps 10-11 idle (complete the control warpgroup for setmaxnreg)
//    Tensor memory (512 columns): S0 [0,128), S1 [128,256), O0 [256,384),
//    O1 [384,512). P_t is written as packed bf16 over the first 64 columns of
//    S_t and consumed from tensor memory by the P.V UMMA. While one warpgroup
//    runs its softmax the tensor core works on the other tile (ping-pong).
//    Rescaling of O is lazy: the running max only moves when a block's max
//    exceeds it by more than 2^8, so most blocks skip the O round trip. P is
//    handed to the UMMA warp in two halves so P.V starts on keys 0-63 while
//    the exponentials of keys 64-127 are still being computed.
//    The epilogue divides by the row sum, stages the tile in the (now free) Q
//    buffer with the 128-byte swizzle and writes it with TMA stores, so any
//    output row pitch that is a multiple of 16 bytes works (e.g. the 12288-wide
//    concat buffer of the single-stream block).
#include <cmath>
#include <mutex>

#include "internal.h"
#include "sm100.cuh"

namespace aex {
namespace attn {

constexpr int kD = 128;
constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // keys per block
constexpr int kTiles = 2;
constexpr int kStages = 5;  // K/V ring slots: 2 x 32 KB Q + 5 x 32 KB = 224 KB of the 227 KB a CTA may use
constexpr int kTileBytes = kBM * kD * 2;  // 32 KB, two 16 KB swizzle regions of 64 columns
constexpr int kRegionBytes = kTileBytes / 2;
// 12 warps = 3 warpgroups: two softmax warpgroups (one query row per thread)
// and one control warpgroup (TMA producer warp, UMMA warp, two idle warps).
// Launched at 168 registers per thread (the per-sub-partition limit with 3
// warps each); the control warpgroup then gives registers to the softmax
// warpgroups: 64 + 2 * 216 = 496 <= 3 * 168 = 504.
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = (kSoftmaxWarps + 4) * 32;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kCtrlRegs = 64;
constexpr int kSoftmaxRegs = 216;
static_assert(kCtrlRegs + 2 * kSoftmaxRegs <= 3 * 168, "register split exceeds the launch allocation");

// Tuning knobs (compile-time).
// Of every 16 exponential pairs, how many use the FMA-pipe polynomial
// (exp2_poly2) instead of MUFU ex2. Measured on B200 at 1024^2: 0 is fastest
// (0.202 ms vs 0.208 ms at 4 and 0.223 ms at 8): the softmax is bound by
// instruction issue of its single warp per sub-partition, not by MUFU.
#ifndef AEX_ATTN_POLY_PAIRS
#define AEX_ATTN_POLY_PAIRS 0
#endif
#ifndef AEX_ATTN_SPLIT_P
#define AEX_ATTN_SPLIT_P 1  // hand P to the UMMA warp in two halves (keys 0-63, 64-127)
#endif
#ifndef AEX_ATTN_PIPE_LD
#define AEX_ATTN_PIPE_LD 1  // overlap the S loads from tensor memory with the row-max computation
#endif
constexpr int kPolyPairs = AEX_ATTN_POLY_PAIRS;
constexpr bool kSplitP = AEX_ATTN_SPLIT_P != 0;

constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kTiles * kTileBytes;
constexpr int kOffBar = kOffKV + kStages * kTileBytes;
// barrier indices
constexpr int kBarQFull = 0;                       // [2]
constexpr int kBarKVFull = 2;                      // [kStages]
constexpr int kBarKVEmpty = kBarKVFull + kStages;  // [kStages]
constexpr int kBarSFull = kBarKVEmpty + kStages;   // [2]  S_t ready (UMMA commit)
constexpr int kBarPFull = kBarSFull + 2;           // [2 tile][2 half] P_t half written (4 warps)
constexpr int kBarOFull = kBarPFull + 4;           // [2]  O_t final (UMMA commit)
constexpr int kBarDrain = kBarOFull + 2;           // [1]
constexpr int kNumBars = kBarDrain + 1;
constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, false, false);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, false, true);

struct Params {
  int seq;       // query rows
  int seq_kv;    // key/value rows (== seq except for sequence-parallel calls)
  // Keys may be split into kv_splits contiguous ranges of n_kv blocks (the
  // last one shorter, n_kv_total in all), one CTA per (query rows, head,
  // batch, range); range r of batch b writes its normalized partial output
  // and log-sum-exp at batch index b * kv_splits + r of O and lse.
  int n_kv;
  int n_kv_total;
  int kv_splits;
  float scale_log2;
  // Optional per-row log-sum-exp of the scaled scores in log2 units,
  // lse2 = m + log2(l), stored at lse[b * lse_sb + h * lse_sh + row]; lets
  // partial results over different K/V sets be merged exactly.
  float* lse;
  int64_t lse_sb, lse_sh;
};

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
  const int ob = blockIdx.z;  // batch index of O and lse
  const int b = ob / p.kv_splits;
  const int split = ob - b * p.kv_splits;
  const int kv_base = split * p.n_kv * kBN;  // first key of this CTA's range
  const int n_kv = min(p.n_kv, p.n_kv_total - split * p.n_kv);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars[kBarQFull + t], 1);
      mbar_init(&bars[kBarSFull + t], 1);
      mbar_init(&bars[kBarPFull + 2 * t], 4);
      mbar_init(&bars[kBarPFull + 2 * t + 1], 4);
      mbar_init(&bars[kBarOFull + t], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kBarKVFull + s], 1);
      mbar_init(&bars[kBarKVEmpty + s], 1);
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
  // Each role's code sits inside the branch that set its register budget, so
  // ptxas compiles the softmax and the control warps with their own limits.
  if (warp >= kSoftmaxWarps) {
    regs_dealloc<kCtrlRegs>();
    if (warp == kProducerWarp && lane == 0) {
      // ---------------------------------------------------------- producer
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
        const int kv0 = kv_base + (idx >> 1) * kBN;
        uint8_t* dst = smem + kOffKV + slot * kTileBytes;
        mbar_arrive_expect_tx(&bars[kBarKVFull + slot], kTileBytes);
        tma_load_4d(dst, m, &bars[kBarKVFull + slot], 0, kv0, h, b);
        tma_load_4d(dst + kRegionBytes, m, &bars[kBarKVFull + slot], 64, kv0, h, b);
        issued = idx + 1;
      }
      if (abort_flag) {
        // Let every copy already issued land before the CTA releases its
        // shared memory (bounded: each wait gives up after the timeout).
        for (int idx = (issued > kStages ? issued - kStages : 0); idx < issued; ++idx) {
          const uint32_t a = smem_u32(&bars[kBarKVFull + idx % kStages]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, (idx / kStages) & 1) && globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    } else if (warp == kMmaWarp && lane == 0) {
      // ---------------------------------------------------------- UMMA issue
      bool ok = mbar_wait(&bars[kBarQFull + 0], 0, &abort_flag, status, kDevTimeoutMma) &&
                mbar_wait(&bars[kBarQFull + 1], 0, &abort_flag, status, kDevTimeoutMma);
      const uint32_t sQ = smem_u32(smem + kOffQ);
      const uint32_t sKV = smem_u32(smem + kOffKV);
      // Descriptors are built once; advancing along K adds the byte offset / 16
      // to the start-address field (all offsets stay inside the 14-bit field).
      const uint64_t dq = sdesc_sw128(sQ, 16, 1024);
      const uint64_t dkv_k = sdesc_sw128(sKV, 16, 1024);
      const uint64_t dkv_v = sdesc_sw128(sKV, kRegionBytes, 1024);
      auto issue_s = [&](int t, int slot) {
        const uint64_t qa = dq + ((t * kTileBytes) >> 4);
        const uint64_t ka = dkv_k + ((slot * kTileBytes) >> 4);
#pragma unroll 1
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kRegionBytes + (kk & 3) * 32) >> 4;
          umma_ss(tmem + t * 128, qa + off, ka + off, kIdescS, kk > 0);
        }
      };
      // P_t[j].V for key steps [kk0, kk1) (16 keys each).
      auto issue_pv = [&](int t, int slot, bool accumulate, int kk0, int kk1) {
        const uint64_t va = dkv_v + ((slot * kTileBytes) >> 4);
#pragma unroll 1
        for (int kk = kk0; kk < kk1; ++kk)
          umma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, va + ((kk * 2048) >> 4), kIdescPV,
                  (accumulate || kk > 0) ? 1u : 0u);
      };
      // Waits for P_t of block `jj` (one or two halves) and issues its P.V.
      auto wait_p_issue_pv = [&](int t, int slot, int jj) -> bool {
        if (kSplitP) {
          if (!mbar_wait(&bars[kBarPFull + 2 * t], jj & 1, &abort_flag, status, kDevTimeoutMma)) return false;
          tc_fence_after();
          issue_pv(t, slot, jj > 0, 0, 4);
          if (!mbar_wait(&bars[kBarPFull + 2 * t + 1], jj & 1, &abort_flag, status, kDevTimeoutMma)) return false;
          tc_fence_after();
          issue_pv(t, slot, true, 4, 8);
        } else {
          if (!mbar_wait(&bars[kBarPFull + 2 * t + 1], jj & 1, &abort_flag, status, kDevTimeoutMma)) return false;
          tc_fence_after();
          issue_pv(t, slot, jj > 0, 0, 8);
        }
        return true;
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
          // P_t[j-1].V (reads P from tensor memory), then S_t[j] overwrites
          // the same columns: UMMAs issued by one thread execute in order.
          ok = wait_p_issue_pv(t, vslot, j - 1);
          if (!ok) break;
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
          ok = wait_p_issue_pv(t, vslot, n_kv - 1);
          if (!ok) break;
          umma_commit(&bars[kBarOFull + t]);
        }
      }
      // Drain: whatever was issued completes before tensor memory is freed.
      umma_commit(&bars[kBarDrain]);
      mbar_wait(&bars[kBarDrain], 0, &abort_flag, status, kDevTimeoutMma);
    }
  } else {
    regs_alloc<kSoftmaxRegs>();
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + t * 128;
    const uint32_t tO = tmem + lane_base + 256 + t * 128;
    const uint32_t bar_s = smem_u32(&bars[kBarSFull + t]);
    const uint32_t bar_p = smem_u32(&bars[kBarPFull + 2 * t]);
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait_warp_addr(bar_s, j & 1, &abort_flag, status, kDevTimeoutSoftmax);
      if (!ok) break;
      tc_fence_after();
      uint32_t r[128];
      const int valid = p.seq_kv - kv_base - j * kBN;
      float mx0, mx1, mx2, mx3;
      auto mask_chunk = [&](int c0) {
        if (valid < kBN) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c0 + i >= valid) r[c0 + i] = __float_as_uint(-INFINITY);
        }
      };
      auto max_chunk = [&](int c0) {  // 32 columns into the four chains
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          mx0 = fmax3(mx0, __uint_as_float(r[c0 + i]), __uint_as_float(r[c0 + i + 1]));
          mx1 = fmax3(mx1, __uint_as_float(r[c0 + i + 2]), __uint_as_float(r[c0 + i + 3]));
          mx2 = fmax3(mx2, __uint_as_float(r[c0 + i + 4]), __uint_as_float(r[c0 + i + 5]));
          mx3 = fmax3(mx3, __uint_as_float(r[c0 + i + 6]), __uint_as_float(r[c0 + i + 7]));
        }
      };
      mx0 = mx1 = mx2 = mx3 = -INFINITY;
      if (AEX_ATTN_PIPE_LD) {
        // Each wait covers the chunk just issued; the max of the previous
        // chunk is computed while the next one is in flight.
        tmem_ld32(tS + 0, r + 0);
        tmem_wait_ld();
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          if (c0 + 32 < 128) tmem_ld32(tS + c0 + 32, r + c0 + 32);
          mask_chunk(c0);
          max_chunk(c0);
          if (c0 + 32 < 128) tmem_wait_ld();
        }
      } else {
        tmem_ld32(tS + 0, r + 0);
        tmem_ld32(tS + 32, r + 32);
        tmem_ld32(tS + 64, r + 64);
        tmem_ld32(tS + 96, r + 96);
        tmem_wait_ld();
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          mask_chunk(c0);
          max_chunk(c0);
        }
      }
      const float m_blk = fmax3(mx0, mx1, fmaxf(mx2, mx3)) * sl2;
      // Lazy rescale: the reference max only moves when the block max exceeds
      // it by more than 8 (a factor 2^8), so P stays <= 256.
      float alpha = 1.f;
      bool rescale = false;
      if (m_blk > m_run + 8.f) {
        alpha = ex2_approx(m_run - m_blk);
        m_run = m_blk;
        rescale = (j > 0);
      }
      l_run *= alpha;
      if (__any_sync(0xffffffffu, rescale)) {
        // O_t holds P.V of blocks < j (its UMMAs completed before S_t[j]).
#pragma unroll 1
        for (int cc = 0; cc < 128; cc += 32) {
          uint32_t o[32];
          tmem_ld32(tO + cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + cc, o);
        }
      }
      const float2 sl2x2 = make_float2(sl2, sl2);
      const float2 negm2 = make_float2(-m_run, -m_run);
      float2 sum_a = make_float2(0.f, 0.f), sum_b = make_float2(0.f, 0.f);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = ffma2(make_float2(__uint_as_float(r[ch * 32 + 2 * i]),
                                             __uint_as_float(r[ch * 32 + 2 * i + 1])),
                                 sl2x2, negm2);
          // kPolyPairs of every 16 pairs on the FMA pipe, the rest on MUFU.
          const float2 pe = (i < kPolyPairs) ? exp2_poly2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
          if (i & 1)
            sum_b = fadd2(sum_b, pe);
          else
            sum_a = fadd2(sum_a, pe);
          pk[i] = pack_bf16x2(pe.x, pe.y);
        }
        tmem_st16(tS + ch * 16, pk);
        if (ch == 1 && kSplitP) {
          // keys 0-63 of P are in tensor memory: the UMMA warp may start P.V
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_addr(bar_p);
        }
      }
      l_run += (sum_a.x + sum_a.y) + (sum_b.x + sum_b.y);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_addr(bar_p + 8);
    }
    // ------------------------------------------------------------ epilogue
    if (ok) ok = mbar_wait_warp(&bars[kBarOFull + t], 0, &abort_flag, status, kDevTimeoutEpilogue);
    uint8_t* stage = smem + kOffQ + t * kTileBytes;  // Q_t is dead once O_t is final
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      if (p.lse && q0 + t * kBM + row < p.seq)
        p.lse[ob * p.lse_sb + h * p.lse_sh + q0 + t * kBM + row] = m_run + __log2f(l_run);
#pragma unroll 1
      for (int cc = 0; cc < 128; cc += 32) {
        uint32_t o[32];
        tmem_ld32(tO + cc, o);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
        // columns [cc, cc+32) live in swizzle region cc/64, 16-byte chunks (cc%64)/8 .. +4
        uint8_t* rowp = stage + (cc >> 6) * kRegionBytes + row * 128;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int chunk = (((cc & 63) >> 3) + qd) ^ (row & 7);
          *reinterpret_cast<uint4*>(rowp + chunk * 16) =
              make_uint4(pk[4 * qd], pk[4 * qd + 1], pk[4 * qd + 2], pk[4 * qd + 3]);
        }
      }
      fence_async_shared();
    }
    // The four warps of this tile have staged their rows (bounded: the
    // warps of a tile reach this point together or all abort).
    asm volatile("bar.sync %0, %1;" ::"r"(1 + t), "r"(128) : "memory");
    if (ok && quad == 0 && lane == 0 && q0 + t * kBM < p.seq) {
      tma_store_4d(&tm_o, stage, 0, q0 + t * kBM, h, ob);
      tma_store_4d(&tm_o, stage + kRegionBytes, 64, q0 + t * kBM, h, ob);
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
  // Norm weights per row segment: tokens s < split use (wq_a, wk_a), the rest
  // (wq, wk). The double-stream block norms its text rows with norm_added_q/k
  // and its image rows with norm_q/k (JointAttention.swift:61-83).
  const float* wq;
  const float* wk;
  const float* wq_a;
  const float* wk_a;
  int split;
  const float* cos_t;
  const float* sin_t;
  float eps;
  int batch, seq, heads;
  __nv_bfloat16* out;    // Q (and K when k_out is NULL): [2][B][H][S][128], or [2][B][S][H][128] when out_token_major
  __nv_bfloat16* k_out;  // K elsewhere: [B][H][S][128], or [B][S][H][128] when k_token_major
  int k_token_major;
  int out_token_major;
};

// Each half-warp owns one 128-wide row (16 lanes x 8 elements = one 16-byte
// load per lane); a warp keeps kPrepRowsPerWarp rows in flight so every lane
// has several independent 16-byte loads outstanding (HBM-bound kernel).
#ifndef AEX_PREP_ROWS
#define AEX_PREP_ROWS 16
#endif
constexpr int kPrepRowsPerWarp = AEX_PREP_ROWS;
constexpr int kPrepWarps = 8;

// Row coordinates (operand, batch, token, head) of a flat row index, advanced
// incrementally: rows are ordered operand-major, then batch, token, head.
struct PrepRow {
  uint32_t which, b, s, h;
  __device__ __forceinline__ void init(uint32_t row, uint32_t rows_per_op, uint32_t heads, uint32_t seq) {
    which = row >= rows_per_op ? 1 : 0;
    const uint32_t r = row - which * rows_per_op;
    h = r % heads;
    const uint32_t t = r / heads;
    s = t % seq;
    b = t / seq;
  }
  __device__ __forceinline__ void advance(uint32_t by, uint32_t heads, uint32_t seq, uint32_t batch) {
    h += by;
    while (h >= heads) {  // at most by / heads + 1 rounds
      h -= heads;
      if (++s == seq) {
        s = 0;
        if (++b == batch) {
          b = 0;
          which = 1;
        }
      }
    }
  }
};

__global__ void __launch_bounds__(256) qk_prep_kernel(PrepParams p) {
  // 32-bit index math: the host guarantees 2*B*S*H < 2^31.
  const uint32_t rows_per_op = static_cast<uint32_t>(p.batch) * p.seq * p.heads;
  const uint32_t total = 2 * rows_per_op;
  const uint32_t heads = p.heads, seq = p.seq, batch = p.batch;
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;  // which row of the pair
  const int l16 = lane & 15;   // 8-element slice of the row
  const uint32_t row0 = (blockIdx.x * kPrepWarps + (threadIdx.x >> 5)) * kPrepRowsPerWarp + half;
  constexpr int kIt = kPrepRowsPerWarp / 2;
  // Issue every row-slice load of this thread first (kIt x 16 bytes in flight
  // per lane); rotary tables and norm weights are read at compute time (the
  // same token's tables serve all its heads, so they hit in L1).
  uint4 raw[kIt];
  PrepRow c;
  c.init(row0 < total ? row0 : 0, rows_per_op, heads, seq);
  const PrepRow c0 = c;
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    raw[it] = make_uint4(0, 0, 0, 0);
    if (row0 + 2 * it < total) {
      const __nv_bfloat16* src = c.which ? p.k + c.b * p.k_sb + c.s * p.k_ss + c.h * p.k_sh
                                         : p.q + c.b * p.q_sb + c.s * p.q_ss + c.h * p.q_sh;
      raw[it] = __ldg(reinterpret_cast<const uint4*>(src) + l16);
    }
    c.advance(2, heads, seq, batch);
  }
  c = c0;
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    const bool valid = row0 + 2 * it < total;
    float x[8];
    const uint32_t wv4[4] = {raw[it].x, raw[it].y, raw[it].z, raw[it].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = bf16lo_to_f32(wv4[i]);
      x[2 * i + 1] = bf16hi_to_f32(wv4[i]);
    }
    // The two half-warps may hold rows of different operands (Q and K), so the
    // reduction runs for every lane and only its use depends on the operand.
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const bool seg_a = static_cast<int>(c.s) < p.split;
    const float* w = c.which ? (seg_a ? p.wk_a : p.wk) : (seg_a ? p.wq_a : p.wq);
    if (w) {
      const float4 wa = __ldg(reinterpret_cast<const float4*>(w + l16 * 8));
      const float4 wb = __ldg(reinterpret_cast<const float4*>(w + l16 * 8 + 4));
      const float wl[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const float inv = rsqrtf(ss * (1.0f / kD) + p.eps);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = x[i] * inv * wl[i];
    }
    if (p.cos_t) {
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.cos_t + c.s * (kD / 2) + l16 * 4));
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.sin_t + c.s * (kD / 2) + l16 * 4));
      const float ca[4] = {c4.x, c4.y, c4.z, c4.w};
      const float sa[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float re = x[2 * i], im = x[2 * i + 1];
        x[2 * i] = re * ca[i] - im * sa[i];
        x[2 * i + 1] = im * ca[i] + re * sa[i];
      }
    }
    if (valid) {
      __nv_bfloat16* base = p.out;
      const int64_t in_op = p.out_token_major ? static_cast<int64_t>(c.b * seq + c.s) * heads + c.h
                                              : static_cast<int64_t>(c.b * heads + c.h) * seq + c.s;
      int64_t dst = static_cast<int64_t>(c.which) * rows_per_op * kD + in_op * kD;
      if (c.which && p.k_out) {
        base = p.k_out;
        dst = p.k_token_major ? (static_cast<int64_t>(c.b * seq + c.s) * heads + c.h) * kD
                              : (static_cast<int64_t>(c.b * heads + c.h) * seq + c.s) * kD;
      }
      *reinterpret_cast<uint4*>(base + dst + l16 * 8) = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]),
                                                                  pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
    }
    c.advance(2, heads, seq, batch);
  }
}

}  // namespace attn

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

int validate_attention_args(aex_ctx* ctx, const aex_attention_args* a) {
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

namespace {

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

int launch_qk_prep(aex_ctx* ctx, const void* q, const int64_t qs[3], const void* k, const int64_t ks[3], int B, int S,
                   int H, const float* wq, const float* wk, const float* wq_a, const float* wk_a, int split,
                   float eps, const float* cos_t, const float* sin_t, void* out, cudaStream_t stream, void* k_out,
                   bool k_token_major, bool out_token_major) {
  if (B <= 0 || S <= 0 || H <= 0) return set_error(ctx, AEX_ERR_INVALID_ARG, "qk prep: empty batch, seq or heads");
  attn::PrepParams pp{};
  pp.q = static_cast<const __nv_bfloat16*>(q);
  pp.k = static_cast<const __nv_bfloat16*>(k);
  pp.q_sb = qs[0];
  pp.q_ss = qs[1];
  pp.q_sh = qs[2];
  pp.k_sb = ks[0];
  pp.k_ss = ks[1];
  pp.k_sh = ks[2];
  pp.wq = wq;
  pp.wk = wk;
  pp.wq_a = wq_a;
  pp.wk_a = wk_a;
  pp.split = split;
  pp.cos_t = cos_t;
  pp.sin_t = sin_t;
  pp.eps = eps;
  pp.batch = B;
  pp.seq = S;
  pp.heads = H;
  pp.out = static_cast<__nv_bfloat16*>(out);
  pp.k_out = static_cast<__nv_bfloat16*>(k_out);
  pp.k_token_major = k_token_major ? 1 : 0;
  pp.out_token_major = out_token_major ? 1 : 0;
  const int64_t rows = 2ll * B * S * H;
  const int64_t per_block = attn::kPrepWarps * attn::kPrepRowsPerWarp;
  const int64_t blocks = (rows + per_block - 1) / per_block;
  if (rows >= (1ll << 31)) return set_error(ctx, AEX_ERR_INVALID_ARG, "batch*seq*heads too large");
  attn::qk_prep_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(pp);
  return check_launch(ctx, "qk_prep_kernel");
}

namespace {
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// Scratch of a key-split call: k partial outputs per batch [B][k][S][H][128] bf16, then their
// log2-sum-exp [B][k][H][S] f32.
size_t split_scratch_bytes(int B, int S, int H, int k) {
  if (k <= 1) return 0;
  const size_t rows = static_cast<size_t>(B) * k * S * H;
  return align256(rows * 256) + align256(rows * 4);
}
}  // namespace

int joint_attention_impl(aex_ctx* ctx, const aex_attention_args* a, void* scratch, size_t scratch_bytes,
                         cudaStream_t stream, int kv_splits) {
  const int B = a->batch, S = a->seq, H = a->heads;
  const void* qsrc = a->q.data;
  const void* ksrc = a->k.data;
  int64_t qs[3] = {a->q.stride_b, a->q.stride_s, a->q.stride_h};
  int64_t ks[3] = {a->k.stride_b, a->k.stride_s, a->k.stride_h};
  const size_t qk_need = aex_joint_attention_scratch_bytes(a);
  const size_t need = align256(qk_need) + split_scratch_bytes(B, S, H, kv_splits);
  if (need > 0) {
    if (!scratch || scratch_bytes < need)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "scratch of %zu bytes is smaller than the %zu needed", scratch_bytes,
                       need);
    if (reinterpret_cast<uintptr_t>(scratch) % 256)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "scratch must be 256-byte aligned");
  }
  if (needs_prep(a)) {
    // Token-major scratch: the same row order as the inputs, so the prep writes sequentially (measured about
    // 1 % faster per fused call at 1024^2 than head-major, the values identical); the attention kernel's TMA
    // reads 128-token boxes of one head with an H*256-byte row pitch either way.
    if (int r = launch_qk_prep(ctx, a->q.data, qs, a->k.data, ks, B, S, H, a->norm_q_weight, a->norm_k_weight,
                               nullptr, nullptr, 0, a->eps, a->rope_cos, a->rope_sin, scratch, stream, nullptr, false,
                               true))
      return r;
    const int64_t plane = static_cast<int64_t>(B) * H * S * 128;
    qsrc = scratch;
    ksrc = static_cast<const __nv_bfloat16*>(scratch) + plane;
    qs[0] = static_cast<int64_t>(H) * S * 128;
    qs[1] = static_cast<int64_t>(H) * 128;
    qs[2] = 128;
    ks[0] = qs[0];
    ks[1] = qs[1];
    ks[2] = qs[2];
  }
  if (kv_splits <= 1)
    return launch_attention_core(ctx, qsrc, qs, ksrc, ks, a->v.data, &a->v.stride_b, a->out.data, &a->out.stride_b, B,
                                 S, S, H, a->scale, nullptr, 0, 0, stream);
  // Keys in kv_splits contiguous ranges run by separate CTAs of one launch (each range's normalized partial
  // output and log-sum-exp), then one merge pass per batch into the caller's output.
  const int k = kv_splits;
  uint8_t* base = static_cast<uint8_t*>(scratch) + align256(qk_need);
  uint16_t* parts = reinterpret_cast<uint16_t*>(base);
  float* lse = reinterpret_cast<float*>(base + align256(static_cast<size_t>(B) * k * S * H * 256));
  const int64_t plane1 = static_cast<int64_t>(S) * H * 128;  // one range of one batch
  const int64_t p_st[3] = {plane1, static_cast<int64_t>(H) * 128, 128};
  if (int r = launch_attention_core(ctx, qsrc, qs, ksrc, ks, a->v.data, &a->v.stride_b, parts, p_st, B, S, S, H,
                                    a->scale, lse, static_cast<int64_t>(H) * S, S, stream, k))
    return r;
  for (int b = 0; b < B; ++b) {
    if (int r = ring::merge_splits(ctx, parts + static_cast<int64_t>(b) * k * plane1, plane1, p_st[1], p_st[2],
                                   lse + static_cast<int64_t>(b) * k * H * S, static_cast<int64_t>(H) * S, k, S, H,
                                   static_cast<uint16_t*>(a->out.data) + static_cast<int64_t>(b) * a->out.stride_b,
                                   a->out.stride_s, a->out.stride_h, stream))
      return r;
  }
  return AEX_OK;
}

int fused_kv_splits(const aex_ctx* ctx, int B, int S, int H) {
  const int ctas = (S + 2 * 128 - 1) / (2 * 128) * H * B;
  return attention_kv_splits(ctas, (S + 127) / 128, ctx->sm_count);
}

int attention_kv_splits(int ctas, int n_kv, int sms) {
  if (ctas <= 0 || n_kv <= 0 || sms <= 0) return 1;
  auto fill = [&](int k) {  // share of the SM slots of the last wave's rounds that hold work
    const int64_t units = static_cast<int64_t>(ctas) * k;
    const int64_t waves = (units + sms - 1) / sms;
    return static_cast<double>(units) / static_cast<double>(waves * sms);
  };
  int best = 1;
  double best_fill = fill(1);
  for (int k = 2; k <= 4; ++k) {
    const int per = (n_kv + k - 1) / k;
    if (per < 8 || (k - 1) * per >= n_kv) break;  // ranges of at least 8 blocks, none empty
    if (fill(k) > best_fill + 0.05) {  // pays for the merge pass
      best = k;
      best_fill = fill(k);
    }
  }
  return best;
}

int launch_attention_core(aex_ctx* ctx, const void* q, const int64_t qs[3], const void* k, const int64_t ks[3],
                          const void* v, const int64_t* vs, void* o, const int64_t* os, int B, int S, int S_kv, int H,
                          float scale, float* lse, int64_t lse_sb, int64_t lse_sh, cudaStream_t stream,
                          int kv_splits) {
  const int n_kv_total = (S_kv + attn::kBN - 1) / attn::kBN;
  if (kv_splits < 1 || B * kv_splits > 65535)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "attention: bad key split count %d", kv_splits);
  const int per_split = (n_kv_total + kv_splits - 1) / kv_splits;
  if ((kv_splits - 1) * per_split >= n_kv_total)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "attention: %d key blocks do not fill %d splits", n_kv_total,
                     kv_splits);
  CUtensorMap tq, tk, tv, to;
  if (int r = bshd_tmap(ctx, &tq, q, qs[0], qs[1], qs[2], B, S, H)) return r;
  if (int r = bshd_tmap(ctx, &tk, k, ks[0], ks[1], ks[2], B, S_kv, H)) return r;
  if (int r = bshd_tmap(ctx, &tv, v, vs[0], vs[1], vs[2], B, S_kv, H)) return r;
  if (int r = bshd_tmap(ctx, &to, o, os[0], os[1], os[2], B * kv_splits, S, H)) return r;
  attn::Params prm{};
  prm.seq = S;
  prm.seq_kv = S_kv;
  prm.n_kv = per_split;
  prm.n_kv_total = n_kv_total;
  prm.kv_splits = kv_splits;
  const float sc = scale > 0.f ? scale : 1.0f / std::sqrt(128.0f);
  prm.scale_log2 = sc * 1.4426950408889634f;
  prm.lse = lse;
  prm.lse_sb = lse_sb;
  prm.lse_sh = lse_sh;
  // Per call (cheap): the attribute is per device, and a process may drive several.
  AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(attn::attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn::kSmemBytes));
  dim3 grid((S + attn::kTiles * attn::kBM - 1) / (attn::kTiles * attn::kBM), H, B * kv_splits);
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
  if (int r = validate_attention_args(ctx, args)) return r;
  if (int r = bind_device(ctx)) return r;
  return joint_attention_impl(ctx, args, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

int aex_joint_attention(aex_ctx* ctx, const aex_attention_args* args, aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (int r = validate_attention_args(ctx, args)) return r;
  if (int r = bind_device(ctx)) return r;
  // A call whose CTAs (256 query rows x head x batch) would underfill the SMs' waves (a few heads, e.g. a
  // head-sharded call, or a short sequence) splits its keys into ranges merged by log-sum-exp.
  const int k = fused_kv_splits(ctx, args->batch, args->seq, args->heads);
  const size_t need = align256(aex_joint_attention_scratch_bytes(args)) +
                      split_scratch_bytes(args->batch, args->seq, args->heads, k);
  void* ws = nullptr;
  if (int r = ensure_scratch(ctx, need, &ws)) return r;
  return joint_attention_impl(ctx, args, ws, need, static_cast<cudaStream_t>(stream), k);
}

}  // extern "C"

// ------------------------------------------------------------------ no-alloc
// aex_joint_attention_noalloc: the same fused attention for callers that must
// not allocate device memory. Some callers cannot call cudaMalloc: a host
// framework that owns the whole device memory pool (the reference's engines
// size one static placement heap up front, DirectDiTStep.swift:155-274, and an
// embedding of this library may be held to the same rule), or a latency-bound
// caller for whom cudaMalloc's implicit device-wide synchronisation would stall
// every other stream. This entry point therefore uses a fixed scratch array
// compiled into the library instead of context scratch.
namespace aex {
namespace {

// 64 MiB of device memory, held by every GPU that loads the library until the
// process exits. It covers the normalized Q and K of batch*heads*seq <= 131072
// rows (2 * rows * 128 * 2 bytes), e.g. the 1024^2 call (1 * 24 * 4608 rows).
constexpr size_t kNoAllocScratchBytes = 64ull << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device ordinal, resolved with that
// device current (host code must not pass the host-side symbol itself) at the
// first call on the device, together with the CUDA context it was resolved
// in. A later call in another context of the device (after cudaDeviceReset
// tore the primary context down and a new one was created) resolves it again,
// so a stale address is never launched on.
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};
CUcontext g_noalloc_cu_ctx[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

int noalloc_scratch(aex_ctx* ctx, void** out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "device ordinal %d beyond %d", ctx->device, kMaxDevices);
  // Since CUDA 12 cudaSetDevice makes the device's primary context current (initializing it if needed).
  AEX_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  CUcontext cur = nullptr;
  auto get_ctx = ctx_get_current_fn();
  if (!get_ctx || get_ctx(&cur) != CUDA_SUCCESS || !cur)
    return set_error(ctx, AEX_ERR_CUDA, "cuCtxGetCurrent failed: no current CUDA context for device %d", ctx->device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[ctx->device] || g_noalloc_cu_ctx[ctx->device] != cur) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(ctx, e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_addr[ctx->device] = p;
    g_noalloc_cu_ctx[ctx->device] = cur;
  }
  *out = g_noalloc_addr[ctx->device];
  return AEX_OK;
}

}  // namespace
}  // namespace aex

extern "C" int aex_joint_attention_noalloc(aex_ctx* ctx, const aex_attention_args* args, aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (int r = validate_attention_args(ctx, args)) return r;
  const size_t need = aex_joint_attention_scratch_bytes(args);
  if (need > kNoAllocScratchBytes)
    return set_error(ctx, AEX_ERR_INVALID_ARG,
                     "aex_joint_attention_noalloc: these args need %zu bytes of scratch (2*batch*heads*seq*256), "
                     "above its fixed %zu-byte array (batch*heads*seq <= %zu); use aex_joint_attention or "
                     "aex_joint_attention_ws",
                     need, kNoAllocScratchBytes, kNoAllocScratchBytes / 512);
  if (int r = bind_device(ctx)) return r;
  void* ws = nullptr;
  if (need > 0)
    if (int r = noalloc_scratch(ctx, &ws)) return r;
  return joint_attention_impl(ctx, args, ws, need, static_cast<cudaStream_t>(stream));
}
