// qmm_sm100.cu — MLX-layout 4-bit affine linears on sm_100a.
//
// Replaces AttentionUtils.applyLinearCore -> quantizedMM(transpose: true,
// groupSize: 64, bits: 4) (Sources/ImarelloDiT/AttentionUtils.swift:198-230)
// and the direct engine's qmm dispatch (Sources/ImarelloDirect/DirectDiTStep.swift:
// 374-406). y[m, n] = sum_k x[m, k] * deq(W)[n, k] with
// deq(W)[n, k] = bf16_rne(f32(scale[n, k/64] * q[n, k] + bias[n, k/64])), the CPU
// dequant of DirectTEEncoder.embedRow (Sources/ImarelloDirect/DirectTEEncoder.swift:
// 104-123): the product of a bf16 scale and a 4-bit code is exact in f32, so one
// fused multiply-add rounds exactly like the reference's multiply-then-add.
//
// K0  unpack_kernel — MLX layout (packed uint32 [n, k/8], LSB-first nibbles;
//     bf16 scales/biases [n, k/64]) -> tile layout: for every 256-row tile `nt`
//     and 64-wide K block `kb` one contiguous 9216-byte chunk
//        [0, 8192)     row r's 32 packed bytes at r*32 (the MLX words, unchanged)
//        [8192, 8704)  bf16 scale of row r at 8192 + 2r
//        [8704, 9216)  bf16 bias  of row r at 8704 + 2r
//     chunk (nt, kb) at byte (nt * k_blocks + kb) * 9216; rows past n are zero.
//     One bulk copy moves one chunk into shared memory.
// K2  gemm_kernel<MT> — tcgen05 GEMM, CTA tile (128*MT) x 256 x 64-wide K steps:
//     warp 0 TMA producer (x tile) + bulk copy (packed chunk), warp 1 UMMA
//     issuer, warps 4..19 dequantize the chunk in registers into the 128-byte
//     swizzled K-major bf16 B tile and, after the main loop, drain the f32
//     accumulators from tensor memory (epilogue).
//     gemv_kernel<R> — R <= 16 activation rows, HBM-bound: one thread per
//     weight row, split-K over a thread-block cluster, partial sums reduced
//     through distributed shared memory (no scratch, no atomics). The dot uses
//     y = sum_g scale_g * (sum_{k in g} x_k q_k) + bias_g * (sum_{k in g} x_k)
//     (f32), i.e. the unrounded dequantized weights.
#include <algorithm>

#include "internal.h"
#include "sm100.cuh"

namespace aex {
namespace qmm {

constexpr int kTileN = 256;
constexpr int kKB = 64;
constexpr int kChunkPacked = kTileN * 32;
constexpr int kChunkBytes = kChunkPacked + kTileN * 4;  // + bf16 scales + bf16 biases
constexpr int kOffScale = kChunkPacked;
constexpr int kOffBias = kChunkPacked + kTileN * 2;

__host__ __device__ inline size_t chunk_offset(int nt, int kb, int k_blocks) {
  return (static_cast<size_t>(nt) * k_blocks + kb) * kChunkBytes;
}

// ------------------------------------------------------------------ K0 unpack
__global__ void __launch_bounds__(256) unpack_kernel(const uint32_t* __restrict__ packed,
                                                     const uint16_t* __restrict__ scales,
                                                     const uint16_t* __restrict__ biases, int n, int k_blocks,
                                                     uint8_t* __restrict__ tiles) {
  const int kb = blockIdx.x, nt = blockIdx.y, r = threadIdx.x;
  const int row = nt * kTileN + r;
  uint8_t* chunk = tiles + chunk_offset(nt, kb, k_blocks);
  uint4 a = make_uint4(0, 0, 0, 0), b = make_uint4(0, 0, 0, 0);
  uint16_t s = 0, bi = 0;
  if (row < n) {
    const uint4* src = reinterpret_cast<const uint4*>(packed + (static_cast<size_t>(row) * k_blocks + kb) * 8);
    a = src[0];
    b = src[1];
    s = scales[static_cast<size_t>(row) * k_blocks + kb];
    bi = biases[static_cast<size_t>(row) * k_blocks + kb];
  }
  uint4* dst = reinterpret_cast<uint4*>(chunk + r * 32);
  dst[0] = a;
  dst[1] = b;
  reinterpret_cast<uint16_t*>(chunk + kOffScale)[r] = s;
  reinterpret_cast<uint16_t*>(chunk + kOffBias)[r] = bi;
}

// Dequantize one packed word (8 codes of one row) to 8 bf16 values, bit-exact
// with the reference: code -> f32 via a byte permute into the mantissa of
// 2^23 (0x4B00000q) minus 2^23, then fma(q, scale, bias), then RNE to bf16.
__device__ __forceinline__ uint4 dequant_word(uint32_t w, float s, float b) {
  const uint32_t lo = w & 0x0F0F0F0Fu;         // codes 0, 2, 4, 6 in the byte lanes
  const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;  // codes 1, 3, 5, 7
  uint32_t out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float ql = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + i));
    const float qh = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + i));
    const float2 q = fadd2(make_float2(ql, qh), make_float2(-8388608.0f, -8388608.0f));
    const float2 v = ffma2(q, make_float2(s, s), make_float2(b, b));
    out[i] = pack_bf16x2(v.x, v.y);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t u) { return __uint_as_float(static_cast<uint32_t>(u) << 16); }

// Tile layout (or MLX layout) -> row-major bf16 [n, k]; one thread per word.
__global__ void __launch_bounds__(256) dequant_tiles_kernel(const uint8_t* __restrict__ tiles, int n, int k_blocks,
                                                            uint16_t* __restrict__ out) {
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;  // word index over [n][k/8]
  const int64_t total = static_cast<int64_t>(n) * k_blocks * 8;
  if (wi >= total) return;
  const int row = static_cast<int>(wi / (k_blocks * 8));
  const int rem = static_cast<int>(wi % (k_blocks * 8));
  const int kb = rem >> 3, c = rem & 7;
  const uint8_t* chunk = tiles + chunk_offset(row / kTileN, kb, k_blocks);
  const int r = row % kTileN;
  const uint32_t w = *reinterpret_cast<const uint32_t*>(chunk + r * 32 + c * 4);
  const float s = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(chunk + kOffScale)[r]);
  const float b = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(chunk + kOffBias)[r]);
  *reinterpret_cast<uint4*>(out + wi * 8) = dequant_word(w, s, b);
}

__global__ void __launch_bounds__(256) dequant_mlx_kernel(const uint32_t* __restrict__ packed,
                                                          const uint16_t* __restrict__ scales,
                                                          const uint16_t* __restrict__ biases, int n, int k_blocks,
                                                          uint16_t* __restrict__ out) {
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  const int64_t total = static_cast<int64_t>(n) * k_blocks * 8;
  if (wi >= total) return;
  const int64_t g = wi >> 3;  // (row, kb) group index = row * k_blocks + kb
  const float s = bf16_bits_to_f32(scales[g]);
  const float b = bf16_bits_to_f32(biases[g]);
  *reinterpret_cast<uint4*>(out + wi * 8) = dequant_word(packed[wi], s, b);
}

// ------------------------------------------------------------------ K2 GEMM
enum OutMode : int { kOutBf16 = 0, kOutF32 = 1, kOutResidualGate = 2 };

constexpr int kGemmThreads = 640;  // warps 0 producer, 1 UMMA, 2-3 idle, 4-19 dequant + epilogue
constexpr int kDequantWarp0 = 4;
constexpr int kDequantThreads = 512;  // one half-row (4 packed words, 32 codes) per thread per K block
constexpr int kGemmStages = 3;
constexpr uint32_t kIdescGemm = idesc_bf16_f32(128, 256, false, false);

template <int MT>
struct GemmLayout {
  static constexpr int kABytes = MT * 128 * kKB * 2;  // MT boxes of 128 rows x 64 (16 KB each)
  static constexpr int kBBytes = kTileN * kKB * 2;    // 32 KB dequantized B tile
  static constexpr int kStageBytes = kABytes + kBBytes + kChunkBytes;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kABytes;
  static constexpr int kOffPk = kABytes + kBBytes;
  static constexpr int kOffBar = kGemmStages * kStageBytes;
  // bars: full[S], bready[S], empty[S], acc
  static constexpr int kNumBars = 3 * kGemmStages + 1;
  static constexpr int kSmem = kOffBar + kNumBars * 8 + 16 + 1024;
  static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment");
};

struct GemmParams {
  const uint8_t* tiles;
  int m, n, k_blocks;
  void* y;
  int64_t ldy;
  int mode;           // kOutBf16, kOutF32, kOutResidualGate
  const float* gate;  // kOutResidualGate: y_f32[row, col] += gate[col] * acc
  int vec;  // y base and row pitch are 16-byte aligned: full 32-column runs use 16-byte stores
};

template <int MT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_x, GemmParams p, int* status) {
  using L = GemmLayout<MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full = bars;
  uint64_t* bready = bars + kGemmStages;
  uint64_t* empty = bars + 2 * kGemmStages;
  uint64_t* acc = bars + 3 * kGemmStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  __shared__ int abort_flag;

  const int warp = static_cast<int>(warp_id_uniform());
  const int lane = static_cast<int>(lane_id());
  const int nt = blockIdx.x;
  const int m0 = blockIdx.y * 128 * MT;
  const int KB = p.k_blocks;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], kDequantThreads / 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, MT * 256);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tm_x);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int issued = 0;
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kGemmStages, use = kb / kGemmStages;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, &abort_flag, status, kDevTimeoutTma)) break;
        uint8_t* st = smem + s * L::kStageBytes;
        mbar_arrive_expect_tx(&full[s], L::kABytes + kChunkBytes);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          tma_load_2d(st + L::kOffA + mt * 16384, &tm_x, &full[s], kb * kKB, m0 + mt * 128);
        bulk_load(st + L::kOffPk, p.tiles + chunk_offset(nt, kb, KB), kChunkBytes, &full[s]);
        issued = kb + 1;
      }
      if (abort_flag) {
        for (int kb = (issued > kGemmStages ? issued - kGemmStages : 0); kb < issued; ++kb) {
          const uint32_t a = smem_u32(&full[kb % kGemmStages]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, (kb / kGemmStages) & 1) && globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- UMMA
      bool ok = true;
      const uint32_t s0 = smem_u32(smem);
      for (int kb = 0; kb < KB && ok; ++kb) {
        const int s = kb % kGemmStages, use = kb / kGemmStages;
        ok = mbar_wait(&full[s], use & 1, &abort_flag, status, kDevTimeoutMma) &&
             mbar_wait(&bready[s], use & 1, &abort_flag, status, kDevTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t st = s0 + s * L::kStageBytes;
        const uint64_t db = sdesc_sw128(st + L::kOffB, 16, 1024);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint64_t da = sdesc_sw128(st + L::kOffA + mt * 16384, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kKB / 16; ++kk)
            umma_ss(tmem + mt * 256, da + (kk * 2), db + (kk * 2), kIdescGemm, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(acc);  // arrives once every UMMA above has completed (also on abort)
      mbar_wait(acc, 0, &abort_flag, status, kDevTimeoutMma);
    }
  } else if (warp >= kDequantWarp0) {
    // ------------------------------------------------------------ dequant
    const int dt = threadIdx.x - kDequantWarp0 * 32;  // 0..255
    bool ok = true;
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % kGemmStages, use = kb / kGemmStages;
      ok = mbar_wait_warp(&full[s], use & 1, &abort_flag, status, kDevTimeoutProducer);
      if (!ok) break;
      const uint8_t* pk = smem + s * L::kStageBytes + L::kOffPk;
      uint8_t* bt = smem + s * L::kStageBytes + L::kOffB;
      {
        const int row = dt >> 1, hw = dt & 1;  // row of the B tile, half (words 4*hw .. 4*hw+3)
        const uint4 w4 = *reinterpret_cast<const uint4*>(pk + row * 32 + hw * 16);
        const float sc = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(pk + kOffScale)[row]);
        const float bi = bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(pk + kOffBias)[row]);
        uint8_t* brow = bt + (row >> 3) * 1024 + (row & 7) * 128;
        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = hw * 4 + i;
          *reinterpret_cast<uint4*>(brow + ((c ^ (row & 7)) << 4)) = dequant_word(ws[i], sc, bi);
        }
      }
      fence_async_shared();  // generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[s]);
    }
    // ------------------------------------------------------------ epilogue
    if (ok) ok = mbar_wait_warp(acc, 0, &abort_flag, status, kDevTimeoutEpilogue);
    if (ok) {
      tc_fence_after();
      const int quad = warp & 3;
      const int quarter = (warp - kDequantWarp0) >> 2;  // columns [64*quarter, +64)
      const int n0 = nt * kTileN + quarter * 64;
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const int row = m0 + mt * 128 + quad * 32 + lane;
        const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + mt * 256 + quarter * 64;
#pragma unroll 1
        for (int c0 = 0; c0 < 64; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c0, r);
          tmem_wait_ld();
          const int col = n0 + c0;
          if (row < p.m && col < p.n) {
            if (p.mode == kOutResidualGate) {
              // Gated residual (dd_gate_add, DirectDiTKernels.swift:208-221): y += gate * acc, f32.
              float* yr = static_cast<float*>(p.y) + static_cast<int64_t>(row) * p.ldy + col;
              if (p.vec && col + 32 <= p.n) {
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                  const float4 g = __ldg(reinterpret_cast<const float4*>(p.gate + col + i));
                  float4 v = *reinterpret_cast<float4*>(yr + i);
                  v.x = fmaf(g.x, __uint_as_float(r[i]), v.x);
                  v.y = fmaf(g.y, __uint_as_float(r[i + 1]), v.y);
                  v.z = fmaf(g.z, __uint_as_float(r[i + 2]), v.z);
                  v.w = fmaf(g.w, __uint_as_float(r[i + 3]), v.w);
                  *reinterpret_cast<float4*>(yr + i) = v;
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (col + i < p.n) yr[i] = fmaf(p.gate[col + i], __uint_as_float(r[i]), yr[i]);
              }
            } else if (p.mode == kOutF32) {
              float* yr = static_cast<float*>(p.y) + static_cast<int64_t>(row) * p.ldy + col;
              if (p.vec && col + 32 <= p.n) {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                  *reinterpret_cast<float4*>(yr + i) = make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                                                                   __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (col + i < p.n) yr[i] = __uint_as_float(r[i]);
              }
            } else {
              uint16_t* yr = static_cast<uint16_t*>(p.y) + static_cast<int64_t>(row) * p.ldy + col;
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
              if (p.vec && col + 32 <= p.n) {
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                  *reinterpret_cast<uint4*>(yr + 2 * i) = make_uint4(pk[i], pk[i + 1], pk[i + 2], pk[i + 3]);
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (col + i < p.n) yr[i] = static_cast<uint16_t>((i & 1) ? (pk[i >> 1] >> 16) : (pk[i >> 1] & 0xFFFFu));
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, MT * 256);
  }
}

// ------------------------------------------------------------------ GEMV
constexpr int kGemvRows = 128;     // weight rows (outputs) per CTA, one per thread
constexpr int kGemvMaxSplit = 8;   // cluster size along K (portable limit)
constexpr int kGemvMaxKbps = 8;    // K blocks per CTA (weights prefetched into registers)

struct GemvParams {
  const uint16_t* x;  // bf16 [m, ldx]
  int64_t ldx;
  const uint8_t* tiles;
  int m, n, k_blocks, kb_per_split;
  void* y;
  int64_t ldy;
  int mode;
  const float* gate;
};

template <int R>
__global__ void __launch_bounds__(kGemvRows) gemv_kernel(GemvParams p) {
  extern __shared__ float gsm[];  // x slice [R][kbps*64] f32, group sums [R][kbps], partials [R][128]
  const int kbps = p.kb_per_split;
  float* xs = gsm;
  float* gsum = xs + R * kbps * kKB;
  float* part = gsum + R * kbps;
  const int t = threadIdx.x;
  const int split = blockIdx.y;
  const int kb0 = split * kbps;
  const int kb1 = min(p.k_blocks, kb0 + kbps);
  const int nkb = max(0, kb1 - kb0);
  const int row = blockIdx.x * kGemvRows + t;  // weight row (output column)
  const int nt = row / kTileN, r = row % kTileN;
  const bool active = row < p.n;
  // 1. Issue every weight load of this thread's K range (kGemvMaxKbps blocks
  //    of 32 packed bytes + scale + bias) before anything else, so the HBM
  //    fetch overlaps the x staging below.
  uint4 wv[2 * kGemvMaxKbps];
  uint16_t sv[kGemvMaxKbps], bv[kGemvMaxKbps];
#pragma unroll
  for (int g = 0; g < kGemvMaxKbps; ++g) {
    if (active && g < nkb) {
      const uint8_t* chunk = p.tiles + chunk_offset(nt, kb0 + g, p.k_blocks);
      wv[2 * g] = __ldg(reinterpret_cast<const uint4*>(chunk + r * 32));
      wv[2 * g + 1] = __ldg(reinterpret_cast<const uint4*>(chunk + r * 32) + 1);
      sv[g] = __ldg(reinterpret_cast<const uint16_t*>(chunk + kOffScale) + r);
      bv[g] = __ldg(reinterpret_cast<const uint16_t*>(chunk + kOffBias) + r);
    }
  }
  // 2. Stage this split's x slice as f32, then per-group sums (one warp per
  //    (row, group) pair, shuffle-reduced).
  for (int i = t; i < R * nkb * kKB; i += kGemvRows) {
    const int mr = i / (nkb * kKB), kk = i % (nkb * kKB);
    xs[mr * kbps * kKB + kk] =
        mr < p.m ? bf16_bits_to_f32(p.x[static_cast<int64_t>(mr) * p.ldx + kb0 * kKB + kk]) : 0.f;
  }
  __syncthreads();
  {
    const int warp = t >> 5, lane = t & 31;
    for (int i = warp; i < R * nkb; i += kGemvRows / 32) {
      const int mr = i / nkb, g = i % nkb;
      const float* xg = xs + mr * kbps * kKB + g * kKB;
      float s = xg[lane] + xg[lane + 32];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) gsum[mr * kbps + g] = s;
    }
  }
  __syncthreads();
  // 3. Dot products: y_m += scale * sum_k(x_mk * q_k) + bias * sum_k(x_mk) per group.
  float acc[R];
#pragma unroll
  for (int mr = 0; mr < R; ++mr) acc[mr] = 0.f;
  if (active) {
#pragma unroll
    for (int g = 0; g < kGemvMaxKbps; ++g) {
      if (g >= nkb) break;
      const float sc = bf16_bits_to_f32(sv[g]);
      const float bi = bf16_bits_to_f32(bv[g]);
      const uint32_t ws[8] = {wv[2 * g].x, wv[2 * g].y, wv[2 * g].z, wv[2 * g].w,
                              wv[2 * g + 1].x, wv[2 * g + 1].y, wv[2 * g + 1].z, wv[2 * g + 1].w};
      float2 tq[R];
#pragma unroll
      for (int mr = 0; mr < R; ++mr) tq[mr] = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t lo = ws[c] & 0x0F0F0F0Fu, hi = (ws[c] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float ql = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + i));
          const float qh = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + i));
          const float2 q = fadd2(make_float2(ql, qh), make_float2(-8388608.0f, -8388608.0f));
          const int kk = g * kKB + c * 8 + 2 * i;  // codes kk, kk+1
#pragma unroll
          for (int mr = 0; mr < R; ++mr)
            tq[mr] = ffma2(q, *reinterpret_cast<const float2*>(xs + mr * kbps * kKB + kk), tq[mr]);
        }
      }
#pragma unroll
      for (int mr = 0; mr < R; ++mr)
        acc[mr] = fmaf(sc, tq[mr].x + tq[mr].y, fmaf(bi, gsum[mr * kbps + g], acc[mr]));
    }
  }
#pragma unroll
  for (int mr = 0; mr < R; ++mr) part[mr * kGemvRows + t] = acc[mr];
  // 4. Reduce the K splits of this cluster in CTA rank 0 through distributed shared memory.
  cluster_sync_all();
  if (cluster_ctarank() == 0 && active) {
    const uint32_t my_part = smem_u32(part);
    for (int mr = 0; mr < R && mr < p.m; ++mr) {
      float v = 0.f;
      for (int c = 0; c < static_cast<int>(gridDim.y); ++c)
        v += ld_shared_cluster_f32(mapa_shared(my_part + (mr * kGemvRows + t) * 4, c));
      if (p.mode == kOutResidualGate)
        static_cast<float*>(p.y)[static_cast<int64_t>(mr) * p.ldy + row] += p.gate[row] * v;
      else if (p.mode == kOutF32)
        static_cast<float*>(p.y)[static_cast<int64_t>(mr) * p.ldy + row] = v;
      else
        static_cast<uint16_t*>(p.y)[static_cast<int64_t>(mr) * p.ldy + row] =
            static_cast<uint16_t>(pack_bf16x2(v, 0.f) & 0xFFFFu);
    }
  }
  cluster_sync_all();  // keep every CTA's shared memory alive until rank 0 has read it
}

}  // namespace qmm

namespace {

int validate_q(aex_ctx* ctx, const void* packed, const void* scales, const void* biases, int n, int k, int gs,
               int bits) {
  if (!packed || !scales || !biases) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL weight pointer");
  if (gs != 64 || bits != 4)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "group_size %d / bits %d unsupported (64 / 4 only)", gs, bits);
  if (n <= 0 || k <= 0 || k % 64)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "n must be positive and k a positive multiple of 64 (n=%d k=%d)", n, k);
  if ((reinterpret_cast<uintptr_t>(packed) & 15) || (reinterpret_cast<uintptr_t>(scales) & 1) ||
      (reinterpret_cast<uintptr_t>(biases) & 1))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "packed must be 16-byte aligned, scales/biases 2-byte aligned");
  return AEX_OK;
}

template <int MT>
int launch_gemm(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy,
                int mode, const float* gate, cudaStream_t s) {
  using L = qmm::GemmLayout<MT>;
  CUtensorMap tx;
  uint64_t dims[2] = {static_cast<uint64_t>(w->k), static_cast<uint64_t>(m)};
  uint64_t strides[1] = {static_cast<uint64_t>(ldx) * 2};
  uint32_t box[2] = {64, 128};
  if (int r = make_tmap(ctx, &tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, 2, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  const int esz = mode == qmm::kOutBf16 ? 2 : 4;
  const int vec = ((reinterpret_cast<uintptr_t>(y) & 15) == 0 && (ldy * esz) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(gate) & 15) == 0)
                      ? 1
                      : 0;
  qmm::GemmParams p{w->tiles, m, w->n, w->k_blocks, y, ldy, mode, gate, vec};
  auto kern = qmm::gemm_kernel<MT>;
  AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem));
  dim3 grid(w->n_tiles, (m + 128 * MT - 1) / (128 * MT));
  kern<<<grid, qmm::kGemmThreads, L::kSmem, s>>>(tx, p, ctx->d_status);
  return check_launch(ctx, "qmm gemm_kernel");
}

template <int R>
int launch_gemv(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy,
                int mode, const float* gate, cudaStream_t s) {
  const int n_ctas = (w->n + qmm::kGemvRows - 1) / qmm::kGemvRows;
  // Enough CTAs to cover every SM several times, and at most kGemvMaxKbps K blocks per CTA.
  int split = std::max(1, std::min(qmm::kGemvMaxSplit, (4 * ctx->sm_count + n_ctas - 1) / n_ctas));
  split = std::max(split, (w->k_blocks + qmm::kGemvMaxKbps - 1) / qmm::kGemvMaxKbps);
  if (split > qmm::kGemvMaxSplit)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "qmm gemv: k=%d needs more than %d K splits", w->k,
                     qmm::kGemvMaxSplit);
  split = std::min(split, w->k_blocks);
  int kbps = (w->k_blocks + split - 1) / split;
  // x slice + group sums + partials in dynamic shared memory (<= 200 KB).
  auto smem_for = [&](int kb) { return static_cast<size_t>(R) * (kb * 64 + kb + qmm::kGemvRows) * 4; };
  constexpr size_t kMaxSmem = 200 * 1024;
  if (smem_for(kbps) > kMaxSmem)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "qmm gemv: k=%d too large for %d rows", w->k, R);
  split = (w->k_blocks + kbps - 1) / kbps;
  AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(qmm::gemv_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kMaxSmem)));
  qmm::GemvParams p{static_cast<const uint16_t*>(x), ldx, w->tiles, m, w->n, w->k_blocks, kbps, y, ldy, mode, gate};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(n_ctas, split, 1);
  cfg.blockDim = dim3(qmm::kGemvRows, 1, 1);
  cfg.dynamicSmemBytes = smem_for(kbps);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = split;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AEX_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, qmm::gemv_kernel<R>, p));
  return check_launch(ctx, "qmm gemv_kernel");
}

}  // namespace

int qmm_run(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy, int mode,
            const float* gate, cudaStream_t s) {
  if (m <= 0) return set_error(ctx, AEX_ERR_INVALID_ARG, "m must be positive");
  if (mode == qmm::kOutResidualGate && !gate) return set_error(ctx, AEX_ERR_INVALID_ARG, "gate is NULL");
  if (m <= 16 && w->k_blocks <= qmm::kGemvMaxSplit * qmm::kGemvMaxKbps) {
    if (m <= 1) return launch_gemv<1>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
    if (m <= 2) return launch_gemv<2>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
    if (m <= 4) return launch_gemv<4>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
    if (m <= 8) return launch_gemv<8>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
    return launch_gemv<16>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
  }
#ifndef AEX_QMM_MT2_MIN_M
#define AEX_QMM_MT2_MIN_M 2048
#endif
  if (m >= AEX_QMM_MT2_MIN_M) return launch_gemm<2>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
  return launch_gemm<1>(ctx, w, x, ldx, m, y, ldy, mode, gate, s);
}

}  // namespace aex

extern "C" {

int aex_dequantize_mlx(aex_ctx* ctx, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int n,
                       int k, int group_size, int bits, uint16_t* out, aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (int r = validate_q(ctx, packed, scales, biases, n, k, group_size, bits)) return r;
  if (!out || (reinterpret_cast<uintptr_t>(out) & 15)) return set_error(ctx, AEX_ERR_INVALID_ARG, "out must be 16-byte aligned");
  if (int r = bind_device(ctx)) return r;
  const int64_t words = static_cast<int64_t>(n) * (k / 8);
  qmm::dequant_mlx_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, scales, biases, n, k / 64, out);
  return check_launch(ctx, "dequant_mlx_kernel");
}

int aex_qweight_create(aex_ctx* ctx, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int n,
                       int k, int group_size, int bits, aex_qweight** out, aex_stream stream) {
  using namespace aex;
  if (!ctx || !out) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx/out");
  *out = nullptr;
  if (int r = validate_q(ctx, packed, scales, biases, n, k, group_size, bits)) return r;
  if (int r = bind_device(ctx)) return r;
  auto* w = new aex_qweight();
  w->device = ctx->device;
  w->n = n;
  w->k = k;
  w->n_tiles = (n + qmm::kTileN - 1) / qmm::kTileN;
  w->k_blocks = k / 64;
  w->bytes = static_cast<size_t>(w->n_tiles) * w->k_blocks * qmm::kChunkBytes;
  cudaError_t e = cudaMalloc(&w->tiles, w->bytes);
  if (e != cudaSuccess) {
    delete w;
    return cuda_error(ctx, e, "cudaMalloc(qweight tiles)");
  }
  qmm::unpack_kernel<<<dim3(w->k_blocks, w->n_tiles), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, scales, biases, n, w->k_blocks, w->tiles);
  if (int r = check_launch(ctx, "unpack_kernel")) {
    cudaFree(w->tiles);
    delete w;
    return r;
  }
  *out = w;
  return AEX_OK;
}

void aex_qweight_destroy(aex_qweight* w) {
  if (!w) return;
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(w->device);
  cudaDeviceSynchronize();
  cudaFree(w->tiles);
  if (cur >= 0) cudaSetDevice(cur);
  delete w;
}

int aex_qweight_shape(const aex_qweight* w, int* n, int* k) {
  if (!w || !n || !k) return AEX_ERR_INVALID_ARG;
  *n = w->n;
  *k = w->k;
  return AEX_OK;
}

int aex_qweight_dequantize(aex_ctx* ctx, const aex_qweight* w, uint16_t* out, aex_stream stream) {
  using namespace aex;
  if (!ctx || !w || !out) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  if (reinterpret_cast<uintptr_t>(out) & 15) return set_error(ctx, AEX_ERR_INVALID_ARG, "out must be 16-byte aligned");
  if (int r = bind_device(ctx)) return r;
  const int64_t words = static_cast<int64_t>(w->n) * (w->k / 8);
  qmm::dequant_tiles_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0,
                              static_cast<cudaStream_t>(stream)>>>(w->tiles, w->n, w->k_blocks, out);
  return check_launch(ctx, "dequant_tiles_kernel");
}

int aex_qmm(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy,
            int y_dtype, aex_stream stream) {
  using namespace aex;
  if (!ctx || !w || !x || !y) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  if (m <= 0) return set_error(ctx, AEX_ERR_INVALID_ARG, "m must be positive");
  if (y_dtype != AEX_DTYPE_BF16 && y_dtype != AEX_DTYPE_F32)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "y_dtype must be AEX_DTYPE_BF16 or AEX_DTYPE_F32");
  if (ldx < w->k || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "x must be 16-byte aligned with ldx >= k and ldx %% 8 == 0");
  if (ldy < w->n || (reinterpret_cast<uintptr_t>(y) & (y_dtype == AEX_DTYPE_F32 ? 3 : 1)))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "y must be aligned to its element size with ldy >= n");
  if (ctx->device != w->device) return set_error(ctx, AEX_ERR_INVALID_ARG, "weight lives on another device");
  if (int r = bind_device(ctx)) return r;
  return qmm_run(ctx, w, x, ldx, m, y, ldy, y_dtype == AEX_DTYPE_F32 ? qmm::kOutF32 : qmm::kOutBf16, nullptr,
                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
