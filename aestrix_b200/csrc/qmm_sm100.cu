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
//     and 64-wide K block `kb` one contiguous 9216-byte chunk made of two
//     4608-byte halves (rows 0-127, rows 128-255); in half h, for row r = 128h + i
//        [0, 4096)     row r's 32 packed bytes at 32i (the MLX words, unchanged)
//        [4096, 4352)  bf16 scale of row r at 4096 + 2i
//        [4352, 4608)  bf16 bias  of row r at 4352 + 2i
//     chunk (nt, kb) at byte (nt * k_blocks + kb) * 9216; rows past n are zero.
//     One bulk copy moves one chunk (or, in the CTA-pair GEMM, one half) into
//     shared memory.
// K2  gemm_pair_kernel — tcgen05 GEMM on CTA pairs (cta_group::2), 256 x 256
//     output tiles, persistent over up to two problems per launch; the
//     weights are dequantized in registers into the 128-byte swizzled K-major
//     bf16 B tile (see the kernel's comment for the roles and the pipeline).
//     gemv_kernel<R> — R <= 16 activation rows, HBM-bound: per CTA 128 weight
//     rows (one chunk half) and one K split of a thread-block cluster; the
//     half-chunks are bulk-copied into shared memory, one thread per weight row
//     computes, partial sums are reduced through distributed shared memory (no
//     scratch, no atomics). The dot uses
//     y = sum_g scale_g * (sum_{k in g} x_k q_k) + bias_g * (sum_{k in g} x_k)
//     (f32), i.e. the unrounded dequantized weights.
#include <algorithm>

#include "internal.h"
#include "sm100.cuh"

namespace aex {
namespace qmm {

constexpr int kTileN = 256;
constexpr int kKB = 64;
constexpr int kHalfBytes = 128 * 36;  // 128 rows x (32 packed bytes + bf16 scale + bf16 bias)
constexpr int kChunkBytes = 2 * kHalfBytes;

// Byte offsets of row r (0..255) inside a chunk.
__host__ __device__ constexpr int pk_off(int r) { return (r >> 7) * kHalfBytes + (r & 127) * 32; }
__host__ __device__ constexpr int sc_off(int r) { return (r >> 7) * kHalfBytes + 4096 + (r & 127) * 2; }
__host__ __device__ constexpr int bi_off(int r) { return (r >> 7) * kHalfBytes + 4352 + (r & 127) * 2; }

__host__ __device__ inline size_t chunk_offset(int nt, int kb, int k_blocks) {
  return (static_cast<size_t>(nt) * k_blocks + kb) * kChunkBytes;
}

// The tile layout stores each packed word with its nibbles permuted: nibble i
// (bits 4i..4i+3) holds code 2i for i < 4 and code 2(i-4)+1 for i >= 4, so
// that (w >> 4j) & 0x000F000F puts codes (2j, 2j+1) in the two 16-bit halves.
__host__ __device__ __forceinline__ uint32_t nibble_compress(uint32_t x) {  // 4 bytes < 16 -> 4 nibbles
  x = (x | (x >> 4)) & 0x00FF00FFu;
  return (x | (x >> 8)) & 0x0000FFFFu;
}
__host__ __device__ __forceinline__ uint32_t permute_word(uint32_t w) {
  return nibble_compress(w & 0x0F0F0F0Fu) | (nibble_compress((w >> 4) & 0x0F0F0F0Fu) << 16);
}

// Codes (2j, 2j+1) of a permuted word as a bf16 pair (128 + q): 0x4300 is
// bf16 128.0 and the code lands in the low mantissa bits.
__device__ __forceinline__ uint32_t code_pair_128(uint32_t wp, int j) {
  return ((wp >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
}

// Byte `b` (0..3) of a word whose bytes each hold a code in their low nibble,
// as the exact f32 128 + q: 0x43 is the top byte of f32 128.0 and the code
// lands in mantissa bits 16..19 (one byte permute).
__device__ __forceinline__ float code_f32_128(uint32_t v, int b) {
  return __uint_as_float(__byte_perm(v, 0x43u, 0x4055u | (static_cast<uint32_t>(b) << 8)));
}

// Exact dequant of a permuted word (the reference's f32 scale*q + bias, then
// RNE to bf16), 8 bf16 in K order.
__device__ __forceinline__ uint4 dequant_word_exact(uint32_t wp, float s, float b) {
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t = code_pair_128(wp, j);
    const float2 q = fadd2(make_float2(__uint_as_float(t << 16), __uint_as_float(t & 0xFFFF0000u)),
                           make_float2(-128.0f, -128.0f));
    const float2 v = ffma2(q, make_float2(s, s), make_float2(b, b));
    out[j] = pack_bf16x2(v.x, v.y);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// True when f32(scale * q + bias) is exact for every code q in 0..15, so that
// one bf16 rounding of the exact value (a bf16 fma) equals the reference's
// f32-then-bf16 rounding. scale * q is a multiple of 2^(Es-7) below 2^(Es+5),
// bias a multiple of 2^(Eb-7) below 2^(Eb+1); their sum fits a 24-bit
// significand when max(Es+5, Eb+1) - min(Es, Eb) <= 16. Zeros are exact;
// subnormals, infinities and NaN take the f32 path.
__device__ __forceinline__ bool one_rounding_exact(uint32_t s16, uint32_t b16) {
  if ((s16 & 0x7FFFu) == 0 || (b16 & 0x7FFFu) == 0) return true;
  const int es = static_cast<int>((s16 >> 7) & 0xFFu), eb = static_cast<int>((b16 >> 7) & 0xFFu);
  if (es == 0 || eb == 0 || es == 0xFF || eb == 0xFF) return false;
  return max(es + 5, eb + 1) - min(es, eb) <= 16;
}

// Fast dequant of a permuted word: exact codes (128 + q) - 128 in bf16, then
// one fma.rn.bf16x2 (q * scale + bias, rounded once). Bit-exact with the
// reference when one_rounding_exact(scale, bias).
__device__ __forceinline__ uint4 dequant_word_fast(uint32_t wp, uint32_t s2, uint32_t b2) {
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t q;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(code_pair_128(wp, j)), "r"(0x43004300u));
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(out[j]) : "r"(q), "r"(s2), "r"(b2));
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
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
    a = make_uint4(permute_word(a.x), permute_word(a.y), permute_word(a.z), permute_word(a.w));
    b = make_uint4(permute_word(b.x), permute_word(b.y), permute_word(b.z), permute_word(b.w));
    s = scales[static_cast<size_t>(row) * k_blocks + kb];
    bi = biases[static_cast<size_t>(row) * k_blocks + kb];
  }
  uint4* dst = reinterpret_cast<uint4*>(chunk + pk_off(r));
  dst[0] = a;
  dst[1] = b;
  *reinterpret_cast<uint16_t*>(chunk + sc_off(r)) = s;
  *reinterpret_cast<uint16_t*>(chunk + bi_off(r)) = bi;
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
  const uint32_t w = *reinterpret_cast<const uint32_t*>(chunk + pk_off(r) + c * 4);
  const float s = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(chunk + sc_off(r)));
  const float b = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(chunk + bi_off(r)));
  *reinterpret_cast<uint4*>(out + wi * 8) = dequant_word_exact(w, s, b);
}

// Copies 128-row chunk halves: dst half (t, kb, h) <- src half given by the
// row maps below (qmm_glu_interleave); one CTA per destination half.
__global__ void __launch_bounds__(256) glu_interleave_kernel(const uint8_t* __restrict__ src, int k_blocks,
                                                             int plain_tiles, int mlp, uint8_t* __restrict__ dst) {
  const int kb = blockIdx.x, h = blockIdx.y & 1, t = blockIdx.y >> 1;
  int src_row;  // first of the 128 source rows of this destination half
  if (t < plain_tiles) {
    src_row = t * kTileN + h * 128;
  } else {
    const int j = t - plain_tiles;  // gate rows [128j, +128) then up rows, after the plain rows
    src_row = plain_tiles * kTileN + h * mlp + j * 128;
  }
  const uint4* sp = reinterpret_cast<const uint4*>(src + chunk_offset(src_row / kTileN, kb, k_blocks) +
                                                   ((src_row / 128) & 1) * kHalfBytes);
  uint4* dp = reinterpret_cast<uint4*>(dst + chunk_offset(t, kb, k_blocks) + h * kHalfBytes);
  for (int i = threadIdx.x; i < kHalfBytes / 16; i += blockDim.x) dp[i] = sp[i];
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

// Epilogue modes of the GEMM and GEMV kernels.
enum OutMode : int { kOutBf16 = 0, kOutF32 = 1, kOutResidualGate = 2 };

// SwiGLU of one pair of bf16-rounded linear outputs (the storage points of
// the reference's linear_in -> silu(g) * u, FeedForward.swift:11-24 and
// dd_swiglu_pitched, DirectDiTKernels.swift:138-159).
__device__ __forceinline__ float swiglu1(float g, float u) {
  g = __uint_as_float(pack_bf16x2(g, 0.f) << 16);
  u = __uint_as_float(pack_bf16x2(u, 0.f) << 16);
  return g / (1.f + __expf(-g)) * u;
}

// ------------------------------------------------------------------ K2 CTA-pair GEMM
// Two CTAs of a cluster compute one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): CTA r holds x rows [128r, 128r + 128) of
// the tile (A, by TMA) and dequantizes weight rows [128r, 128r + 128) of the
// N-tile (its half of B, from its half of the chunk), and receives the f32
// accumulators of its 128 x rows for all 256 columns in its tensor memory. Per
// SM the tensor core reads 8 KB of shared memory per 128-cycle MMA instead of
// 12 KB for a one-CTA 128 x 256 MMA.
// Persistent: cluster c walks tiles c, c + clusters, ...; a tile index covers
// up to two problems (same kernel, different x / weights / outputs) so that a
// short problem (text rows) shares the launch with a long one. Two 256-column
// accumulator buffers let the epilogue of one tile overlap the main loop of
// the next.
//   warp 0      producer: TMA of the A box + bulk copy of the chunk half
//   warp 1      UMMA issuer (even CTA only)
//   warp 2      tensor-memory allocation
//   warps 4-7   epilogue (tensor-memory lane quadrant = warp % 4)
//   warps 8-    dequantize: kPairGroups groups of warps take turns over the K
//               blocks; within a group each thread converts 8 / kPairSplit
//               packed words of one row per K block.
// Synchronisation per K block (stage s): the producers' TMA + bulk copy land on
// each CTA's full[s]; each dequant warp of either CTA arrives on the even CTA's
// bready[s] (count: both CTAs' warps of one group); the UMMA thread waits on
// bready[s], issues 4 MMAs and commits once to the even CTA's empty[s], whose
// producer forwards the completion to the odd CTA's empty[s]. Measured on B200:
// remote arrives use the default CTA-scope release (a cluster-scope release
// cost ~1000 cycles per arrive), and the UMMA loop is kept short (one commit,
// stage and phase advanced incrementally) because the tensor core's queue of
// pending MMAs is short: cycles the issuing thread spends between MMAs idle it.
#ifndef AEX_PAIR_GROUPS
#define AEX_PAIR_GROUPS 2
#endif
#ifndef AEX_PAIR_SPLIT
#define AEX_PAIR_SPLIT 1
#endif
constexpr int kPairGroups = AEX_PAIR_GROUPS;
constexpr int kPairSplit = AEX_PAIR_SPLIT;                // threads per row (1, 2 or 4)
static_assert(kPairSplit == 1 || kPairSplit == 2 || kPairSplit == 4, "AEX_PAIR_SPLIT must be 1, 2 or 4");
constexpr int kPairWords = 8 / kPairSplit;                // packed words per thread per K block
constexpr int kPairDeqWarps = 4 * kPairSplit;             // dequant warps per group
constexpr int kPairThreads = 32 * (8 + kPairGroups * kPairDeqWarps);
constexpr int kPairEpi0 = 4;
constexpr int kPairDeq0 = 8;
constexpr int kPairStages = 6;
constexpr int kPairABytes = 128 * kKB * 2;
constexpr int kPairBBytes = 128 * kKB * 2;
constexpr int kPairOffB = kPairABytes;
constexpr int kPairOffPk = kPairABytes + kPairBBytes;
constexpr int kPairStage = (kPairOffPk + kHalfBytes + 1023) & ~1023;
constexpr int kPairOffBar = kPairStages * kPairStage;
// bars: full[S], bready[S], empty[S], accf[2], acce[2], drain
constexpr int kPairNumBars = 3 * kPairStages + 5;
constexpr int kPairSmem = kPairOffBar + kPairNumBars * 8 + 16 + 1024;
static_assert(kPairSmem <= 232448, "pair GEMM exceeds the shared-memory limit");
constexpr uint32_t kIdescPair = idesc_bf16_f32(256, 256, false, false);
constexpr int kPairMaxProblems = 2;

struct PairProblem {
  const uint8_t* tiles;
  int m, n, k_blocks;
  int m_tiles;  // 256-row tiles of x
  int tile0;    // first global tile index of this problem
  void* y;
  int64_t ldy;
  int mode;
  const float* gate;
  int vec;
  // Weight tiles nt >= glu_tile0 hold 128 gate rows then 128 up rows (see
  // qmm_glu_interleave); their epilogue writes silu(g) * u, bf16, into
  // y2[row, (nt - glu_tile0) * 128 + c] (row pitch ldy2, 16-byte aligned).
  int glu_tile0;
  uint16_t* y2;
  int64_t ldy2;
  // Weight tiles nt < qk_tiles hold the Q then K projections (128 columns per
  // head, two heads per tile): their epilogue applies the joint attention's
  // QK-RMSNorm + RoPE and writes head-major prep[which][head][tok0 + row][128]
  // (which 0 = Q, 1 = K; heads h_total, tokens j_total), the layout the
  // attention kernel reads, instead of y. K goes to prep_k instead when it is
  // set: [h_total][j_total][128], or [j_total][h_total][128] when k_tok_major.
  int qk_tiles;
  uint16_t* prep;
  uint16_t* prep_k;
  int k_tok_major;
  int tok0, j_total, h_total;
  const float* norm_q;  // [128] f32 (NULL: no norm)
  const float* norm_k;
  float eps;
  const float* rope_cos;  // [j_total, 64] f32 (NULL: no rotation)
  const float* rope_sin;
};

struct PairParams {
  PairProblem prob[kPairMaxProblems];
  int n_prob;
  int tiles;
};

struct PairTile {
  int pi, mt, nt;
};

__device__ __forceinline__ PairTile pair_tile(const PairParams& p, int t) {
  const int pi = (p.n_prob > 1 && t >= p.prob[1].tile0) ? 1 : 0;
  const int lt = t - p.prob[pi].tile0;
  return PairTile{pi, lt % p.prob[pi].m_tiles, lt / p.prob[pi].m_tiles};
}

// Writes 32 accumulator columns [col, col + 32) of one output row.
__device__ __forceinline__ void store_run(const PairProblem& q, int row, int col, const uint32_t* r) {
  if (q.mode == kOutResidualGate) {
    // Gated residual (dd_gate_add, DirectDiTKernels.swift:208-221): y += gate * acc, f32.
    float* yr = static_cast<float*>(q.y) + static_cast<int64_t>(row) * q.ldy + col;
    if (q.vec && col + 32 <= q.n) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(q.gate + col + i));
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
        if (col + i < q.n) yr[i] = fmaf(q.gate[col + i], __uint_as_float(r[i]), yr[i]);
    }
  } else if (q.mode == kOutF32) {
    float* yr = static_cast<float*>(q.y) + static_cast<int64_t>(row) * q.ldy + col;
    if (q.vec && col + 32 <= q.n) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(yr + i) = make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                                                         __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < q.n) yr[i] = __uint_as_float(r[i]);
    }
  } else {
    uint16_t* yr = static_cast<uint16_t*>(q.y) + static_cast<int64_t>(row) * q.ldy + col;
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    if (q.vec && col + 32 <= q.n) {
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<uint4*>(yr + 2 * i) = make_uint4(pk[i], pk[i + 1], pk[i + 2], pk[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < q.n) yr[i] = static_cast<uint16_t>((i & 1) ? (pk[i >> 1] >> 16) : (pk[i >> 1] & 0xFFFFu));
    }
  }
}

__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x0, const __grid_constant__ CUtensorMap tm_x1,
                     const __grid_constant__ PairParams p, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairOffBar);
  uint64_t* full = bars;
  uint64_t* bready = bars + kPairStages;
  uint64_t* empty = bars + 2 * kPairStages;
  uint64_t* accf = bars + 3 * kPairStages;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPairNumBars);
  __shared__ int abort_flag;

  const int warp = static_cast<int>(warp_id_uniform());
  const int lane = static_cast<int>(lane_id());
  const uint32_t rank = cluster_ctarank();
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int clusters = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], 2 * kPairDeqWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 2 * 4);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x0);
    if (p.n_prob > 1) prefetch_tmap(&tm_x1);
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialized, tensor memory allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      // Stage s and its phase bit advance together; the even CTA's producer
      // also forwards each "stage free" completion (a tensor-core commit on
      // its own empty barrier) to the odd CTA's empty barrier.
      const uint32_t empty0 = smem_u32(&empty[0]);
      const uint32_t peer_empty0 = mapa_shared(empty0, 1);
      uint32_t s = 0, ph = 0;
      int g = 0;
      bool ok = true;
      for (int t = cluster; t < p.tiles && ok; t += clusters) {
        const PairTile tl = pair_tile(p, t);
        const PairProblem& q = p.prob[tl.pi];
        const CUtensorMap* tm = tl.pi ? &tm_x1 : &tm_x0;
        const int row0 = tl.mt * 256 + static_cast<int>(rank) * 128;
        const uint8_t* wsrc = q.tiles + chunk_offset(tl.nt, 0, q.k_blocks) + rank * kHalfBytes;
        const int kbs = q.k_blocks;
        for (int kb = 0; kb < kbs; ++kb, ++g) {
          if (g >= kPairStages) {
            if (!mbar_wait_cl(empty0 + 8 * s, ph ^ 1, &abort_flag, status, kDevTimeoutTma)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_cluster(peer_empty0 + 8 * s);
          }
          uint8_t* st = smem + s * kPairStage;
          mbar_arrive_expect_tx(&full[s], kPairABytes + kHalfBytes);
          tma_load_2d(st, tm, &full[s], kb * kKB, row0);
          bulk_load(st + kPairOffPk, wsrc + static_cast<size_t>(kb) * kChunkBytes, kHalfBytes, &full[s]);
          if (++s == kPairStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA can exit.
        for (int j = (g > kPairStages ? g - kPairStages : 0); j < g; ++j) {
          const uint32_t a = smem_u32(&full[j % kPairStages]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, (j / kPairStages) & 1) && globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------- UMMA (even CTA)
      // Lean loop: the tensor core's queue of pending MMAs is short, so every
      // cycle this thread spends outside the issue of MMAs can idle it.
      const uint32_t s0 = smem_u32(smem);
      const uint32_t bready0 = smem_u32(&bready[0]);
      const uint32_t empty0 = smem_u32(&empty[0]);
      const uint64_t da0 = sdesc_sw128(s0, 16, 1024);
      const uint64_t db0 = sdesc_sw128(s0 + kPairOffB, 16, 1024);
      uint32_t s = 0, ph = 0;
      int i = 0;
      bool ok = true;
      for (int t = cluster; t < p.tiles && ok; t += clusters, ++i) {
        const int kbs = p.prob[pair_tile(p, t).pi].k_blocks;
        const int b = i & 1;
        if (i >= 2 && !mbar_wait_cl(smem_u32(&acce[b]), ((i >> 1) + 1) & 1, &abort_flag, status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + b * 256;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!mbar_wait_cl(bready0 + 8 * s, ph, &abort_flag, status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t off = (s * kPairStage) >> 4;  // stage offset in the descriptors' 16-byte units
#pragma unroll
          for (int kk = 0; kk < kKB / 16; ++kk)
            umma_ss_pair(d, da0 + off + kk * 2, db0 + off + kk * 2, kIdescPair, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(empty0 + 8 * s);
          if (++s == kPairStages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&accf[b]));
        umma_commit_pair(mapa_shared(smem_u32(&accf[b]), 1));
      }
      // Arrives once every MMA above has completed; waited for also on abort
      // (hence a flag of its own), so no MMA is in flight at the teardown.
      umma_commit_pair(smem_u32(drain));
      int no_abort = 0;
      mbar_wait_cl(smem_u32(drain), 0, &no_abort, status, kDevTimeoutMma);
    }
  } else if (warp >= kPairEpi0 && warp < kPairEpi0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    int i = 0;
    for (int t = cluster; t < p.tiles; t += clusters, ++i) {
      const PairTile tl = pair_tile(p, t);
      const PairProblem& q = p.prob[tl.pi];
      const int b = i & 1;
      if (!mbar_wait_warp_cl(smem_u32(&accf[b]), (i >> 1) & 1, &abort_flag, status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int row = tl.mt * 256 + static_cast<int>(rank) * 128 + quad * 32 + lane;
      const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * 256;
      if (tl.nt < q.qk_tiles) {
        // QK-RMSNorm + RoPE of two heads (the reference's storage points: the linear's output rounded to bf16,
        // f32 norm and rotation, one rounding; as qk_prep_kernel and AttentionUtils.processQKV / applyRopeBSHD).
        const int heads_per_op = q.h_total;
        const int tok = q.tok0 + row;
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {
          const int gh = tl.nt * 2 + h2;  // head index over Q then K
          const int which = gh >= heads_per_op ? 1 : 0;
          const int head = gh - which * heads_per_op;
          const float* w = which ? q.norm_k : q.norm_q;
          const uint32_t tb = tbase + h2 * 128;
          // pass 1: sum of squares of the bf16-rounded outputs (pairs)
          float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll 1
          for (int c0 = 0; c0 < 128; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tb + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const uint32_t hb = pack_bf16x2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
              const float2 v = make_float2(bf16lo_to_f32(hb), bf16hi_to_f32(hb));
              ss2 = ffma2(v, v, ss2);
            }
          }
          const float inv = rsqrtf((ss2.x + ss2.y) * (1.0f / 128.0f) + q.eps);
          uint16_t* dst = q.prep + ((static_cast<int64_t>(which) * heads_per_op + head) * q.j_total + tok) * 128;
          if (which && q.prep_k)
            dst = q.prep_k + (q.k_tok_major ? static_cast<int64_t>(tok) * heads_per_op + head
                                            : static_cast<int64_t>(head) * q.j_total + tok) * 128;
          const float* crow = q.rope_cos ? q.rope_cos + static_cast<int64_t>(tok) * 64 : nullptr;
          const float* srow = q.rope_sin ? q.rope_sin + static_cast<int64_t>(tok) * 64 : nullptr;
          // pass 2: normalize, rotate, round once
#pragma unroll 1
          for (int c0 = 0; c0 < 128; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tb + c0, r);
            tmem_wait_ld();
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float4 w0 = make_float4(inv, inv, inv, inv), w1 = w0;
              if (w) {
                w0 = __ldg(reinterpret_cast<const float4*>(w + c0 + i));
                w1 = __ldg(reinterpret_cast<const float4*>(w + c0 + i + 4));
                w0 = make_float4(w0.x * inv, w0.y * inv, w0.z * inv, w0.w * inv);
                w1 = make_float4(w1.x * inv, w1.y * inv, w1.z * inv, w1.w * inv);
              }
              const float wl[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
              float4 c4 = make_float4(1.f, 1.f, 1.f, 1.f), s4 = make_float4(0.f, 0.f, 0.f, 0.f);
              if (crow) {
                c4 = __ldg(reinterpret_cast<const float4*>(crow + (c0 + i) / 2));
                s4 = __ldg(reinterpret_cast<const float4*>(srow + (c0 + i) / 2));
              }
              const float ca[4] = {c4.x, c4.y, c4.z, c4.w}, sa[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t hb = pack_bf16x2(__uint_as_float(r[i + 2 * e]), __uint_as_float(r[i + 2 * e + 1]));
                // x * (w * inv): the prep kernel's x * inv * w up to the order of the product
                const float2 x = fmul2(make_float2(bf16lo_to_f32(hb), bf16hi_to_f32(hb)),
                                       make_float2(wl[2 * e], wl[2 * e + 1]));
                const float re = x.x, im = x.y;
                pk[(i >> 1) + e] = pack_bf16x2(re * ca[e] - im * sa[e], im * ca[e] + re * sa[e]);
              }
            }
            if (row < q.m) {
#pragma unroll
              for (int i = 0; i < 16; i += 4)
                *reinterpret_cast<uint4*>(dst + c0 + 2 * i) = make_uint4(pk[i], pk[i + 1], pk[i + 2], pk[i + 3]);
            }
          }
        }
      } else if (tl.nt >= q.glu_tile0) {
        // Gate columns [0, 128), up columns [128, 256) of this tile.
        uint16_t* yr = q.y2 + static_cast<int64_t>(row) * q.ldy2 + (tl.nt - q.glu_tile0) * 128;
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t gr[32], ur[32];
          tmem_ld32(tbase + c0, gr);
          tmem_ld32(tbase + 128 + c0, ur);
          tmem_wait_ld();
          if (row < q.m) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = pack_bf16x2(swiglu1(__uint_as_float(gr[2 * i]), __uint_as_float(ur[2 * i])),
                                  swiglu1(__uint_as_float(gr[2 * i + 1]), __uint_as_float(ur[2 * i + 1])));
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<uint4*>(yr + c0 + 2 * i) = make_uint4(pk[i], pk[i + 1], pk[i + 2], pk[i + 3]);
          }
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < 256; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c0, r);
          tmem_wait_ld();
          const int col = tl.nt * kTileN + c0;
          if (row < q.m && col < q.n) store_run(q, row, col, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acce[b]), 0));
    }
  } else if (warp >= kPairDeq0) {
    // ------------------------------------------------------------ dequant
    const int dw = warp - kPairDeq0;
    const int group = dw / kPairDeqWarps;
    const int dt = (dw % kPairDeqWarps) * 32 + lane;  // 0 .. 128 * kPairSplit - 1
    const int row = dt / kPairSplit, part = dt % kPairSplit;  // row of this CTA's B half; words part*kPairWords ..
    uint8_t* bdst = smem + kPairOffB + row * 128;
    const uint32_t full0 = smem_u32(&full[0]);
    const uint32_t bready_lead0 = mapa_shared(smem_u32(&bready[0]), 0);
    uint32_t s = 0, ph = 0;
    int g = 0;
    bool ok = true;
    for (int t = cluster; t < p.tiles && ok; t += clusters) {
      const int kbs = p.prob[pair_tile(p, t).pi].k_blocks;
      for (int kb = 0; kb < kbs; ++kb, ++g) {
        const uint32_t cs = s, cph = ph;  // this K block's stage and phase
        if (++s == kPairStages) {
          s = 0;
          ph ^= 1;
        }
        if (kPairGroups > 1 && g % kPairGroups != group) continue;
        if (!mbar_wait_warp_cl(full0 + 8 * cs, cph, &abort_flag, status, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint8_t* pk = smem + cs * kPairStage + kPairOffPk;
        uint32_t ws[kPairWords];
        if (kPairWords >= 4) {
#pragma unroll
          for (int j = 0; j < kPairWords; j += 4) {
            const uint4 w4 = *reinterpret_cast<const uint4*>(pk + row * 32 + part * kPairWords * 4 + j * 4);
            ws[j] = w4.x;
            ws[j + 1] = w4.y;
            ws[j + 2] = w4.z;
            ws[j + 3] = w4.w;
          }
        } else {
          const uint2 w2 = *reinterpret_cast<const uint2*>(pk + row * 32 + part * 8);
          ws[0] = w2.x;
          ws[kPairWords - 1] = w2.y;
        }
        const uint32_t s16 = *reinterpret_cast<const uint16_t*>(pk + 4096 + row * 2);
        const uint32_t b16 = *reinterpret_cast<const uint16_t*>(pk + 4352 + row * 2);
        uint8_t* brow = bdst + cs * kPairStage;
        if (one_rounding_exact(s16, b16)) {
          const uint32_t s2 = s16 | (s16 << 16), b2 = b16 | (b16 << 16);
#pragma unroll
          for (int j = 0; j < kPairWords; ++j) {
            const int c = part * kPairWords + j;
            *reinterpret_cast<uint4*>(brow + ((c ^ (row & 7)) << 4)) = dequant_word_fast(ws[j], s2, b2);
          }
        } else {
          const float sc = __uint_as_float(s16 << 16), bi = __uint_as_float(b16 << 16);
#pragma unroll
          for (int j = 0; j < kPairWords; ++j) {
            const int c = part * kPairWords + j;
            *reinterpret_cast<uint4*>(brow + ((c ^ (row & 7)) << 4)) = dequant_word_exact(ws[j], sc, bi);
          }
        }
        fence_async_shared();  // generic-proxy stores -> visible to the pair's tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(bready_lead0 + 8 * cs);
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // no peer access to this CTA's shared or tensor memory after this point
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ------------------------------------------------------------------ GEMV
// A CTA owns 128 weight rows (outputs) — exactly one half of a 256-row tile, so
// its weights for a K block are one contiguous 4608-byte half-chunk — and one
// K split of the cluster. The split's half-chunks stream through a ring of
// kGemvRing shared-memory slots owned by a producer warp (lane 0 bulk-copies a
// K block into a slot, one "full" mbarrier per slot, and refills the slot once
// each of the four compute warps has arrived on its "empty" mbarrier), so no
// CTA-wide barrier sits in the K loop. The compute warps stage x meanwhile
// (group sums of x formed on the way, by shuffles) and then take the K blocks
// in order as they land, one weight row per thread. The ring keeps the shared
// memory of a CTA small, so even a 3072 x 18432 weight (215 KB per SM) runs in
// one wave. Partial sums of the cluster's splits are reduced in CTA rank 0
// through distributed shared memory (no scratch, no atomics, fixed order).
// One launch may cover up to kGemvMaxProblems weights that read the same x
// (the conditioning's modulation heads): the CTAs along x are numbered across
// the problems, so one launch and one fill/drain serve all of them.
// x is bf16 or f32 (the reference's f32 conditioning qmm,
// affine_qmm_t_float_gs_64_b_4, DirectConditioner.swift:48,183-190); it is
// staged as f32 either way, so the arithmetic is the same.
constexpr int kGemvRows = 128;
constexpr int kGemvThreads = kGemvRows + 32;  // four compute warps + the producer warp
constexpr int kGemvMaxSplit = 8;   // cluster size along K (portable limit)
constexpr int kGemvMaxKbps = 48;   // K blocks per CTA
constexpr int kGemvRing = 4;       // weight slots per CTA
constexpr int kGemvMaxProblems = 4;

struct GemvProblem {
  const uint8_t* tiles;
  int n;
  int cta0;  // first blockIdx.x of this problem
  void* y;
  int64_t ldy;
  int mode;
  const float* gate;
};

struct GemvParams {
  const void* x;  // bf16 or f32 [m, ldx]
  int64_t ldx;
  int m, k_blocks, kb_per_split;
  int n_prob;
  GemvProblem prob[kGemvMaxProblems];
  int* status;
};

// Shared memory of gemv_kernel<R> for `kbps` K blocks per CTA.
__host__ __device__ constexpr size_t gemv_smem_bytes(int R, int kbps) {
  return static_cast<size_t>(kGemvRing) * kHalfBytes                              // weight ring
         + static_cast<size_t>(R) * (kbps * kKB + kbps + kGemvRows) * 4          // x, group sums, partials
         + 8 + static_cast<size_t>(kGemvRing) * 16;                              // align + full/empty barriers
}

template <int R, bool XF32>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) uint8_t gsm_raw[];
  const int kbps = p.kb_per_split;
  uint8_t* wsm = gsm_raw;
  float* xs = reinterpret_cast<float*>(gsm_raw + static_cast<size_t>(kGemvRing) * kHalfBytes);
  float* gsum = xs + R * kbps * kKB;
  float* part = gsum + R * kbps;
  uint64_t* full = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(part + R * kGemvRows) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + kGemvRing;
  __shared__ int abort_flag;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  int pi = 0;
#pragma unroll
  for (int i = 1; i < kGemvMaxProblems; ++i)
    if (i < p.n_prob && static_cast<int>(blockIdx.x) >= p.prob[i].cta0) pi = i;
  const GemvProblem& q = p.prob[pi];
  const int cta = static_cast<int>(blockIdx.x) - q.cta0;
  const int split = blockIdx.y;
  const int kb0 = split * kbps;
  const int kb1 = min(p.k_blocks, kb0 + kbps);
  const int nkb = max(0, kb1 - kb0);
  const int row = cta * kGemvRows + t;  // weight row (output column) of a compute thread
  const int nt = cta >> 1, half = cta & 1;
  const bool active = t < kGemvRows && row < q.n;
  if (t == 0) {
    abort_flag = 0;
    for (int s = 0; s < kGemvRing; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvRows / 32);
    }
    fence_barrier_init();
  }
  __syncthreads();
  float acc[R];
#pragma unroll
  for (int mr = 0; mr < R; ++mr) acc[mr] = 0.f;
  if (warp == kGemvRows / 32) {
    // 1. Producer: K block g of the range into slot g % kGemvRing once the slot's previous block is used.
    if (lane == 0) {
      int issued = 0;
      for (int g = 0; g < nkb; ++g) {
        const int s = g % kGemvRing;
        if (g >= kGemvRing &&
            !mbar_wait(&empty[s], ((g / kGemvRing) - 1) & 1, &abort_flag, p.status, kDevTimeoutProducer))
          break;
        mbar_arrive_expect_tx(&full[s], kHalfBytes);
        bulk_load(wsm + s * kHalfBytes, q.tiles + chunk_offset(nt, kb0 + g, p.k_blocks) + half * kHalfBytes,
                  kHalfBytes, &full[s]);
        issued = g + 1;
      }
      if (issued < nkb) {
        // Aborting: the copies still in flight (at most the last kGemvRing issued) land before the CTA exits.
        for (int g = max(0, issued - kGemvRing); g < issued; ++g) {
          const uint32_t a = smem_u32(&full[g % kGemvRing]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, (g / kGemvRing) & 1) && globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
    __syncwarp();
  } else {
    // 2. Stage this split's x slice as f32 (16-byte loads: x 16-byte aligned and its row pitch a multiple of 16
    //    bytes, checked on the host; every load of a thread issued before its stores) and the per-group sums:
    //    the 16-byte vectors of one 64-element group sit in kVpg consecutive lanes, summed by shuffles.
    {
      constexpr int kPerVec = XF32 ? 4 : 8;  // elements per 16-byte load
      constexpr int kVpg = kKB / kPerVec;     // vectors per group
      constexpr int kBatch = 4;               // loads in flight per thread before their stores
      const int per_row = nkb * kKB / kPerVec, nvec = R * per_row;
#pragma unroll 1
      for (int j0 = 0; j0 * kGemvRows < nvec; j0 += kBatch) {
        uint4 xv[kBatch];
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj) {
          const int i = t + (j0 + jj) * kGemvRows;
          xv[jj] = make_uint4(0, 0, 0, 0);
          if (i < nvec) {
            const int mr = i / per_row, c = i % per_row;
            if (mr < p.m) {
              if (XF32)
                xv[jj] = __ldg(reinterpret_cast<const uint4*>(static_cast<const float*>(p.x) +
                                                              static_cast<int64_t>(mr) * p.ldx + kb0 * kKB) + c);
              else
                xv[jj] = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) +
                                                              static_cast<int64_t>(mr) * p.ldx + kb0 * kKB) + c);
            }
          }
        }
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj) {
          const int i = t + (j0 + jj) * kGemvRows;
          float vs = 0.f;
          if (i < nvec) {
            const int mr = i / per_row, c = i % per_row;
            float* d = xs + mr * kbps * kKB + c * kPerVec;
            const uint32_t u[4] = {xv[jj].x, xv[jj].y, xv[jj].z, xv[jj].w};
            if (XF32) {
              const float4 f = make_float4(__uint_as_float(u[0]), __uint_as_float(u[1]), __uint_as_float(u[2]),
                                           __uint_as_float(u[3]));
              *reinterpret_cast<float4*>(d) = f;
              vs = (f.x + f.y) + (f.z + f.w);
            } else {
              float f[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                f[2 * e] = bf16lo_to_f32(u[e]);
                f[2 * e + 1] = bf16hi_to_f32(u[e]);
              }
              *reinterpret_cast<float4*>(d) = make_float4(f[0], f[1], f[2], f[3]);
              *reinterpret_cast<float4*>(d + 4) = make_float4(f[4], f[5], f[6], f[7]);
              vs = ((f[0] + f[1]) + (f[2] + f[3])) + ((f[4] + f[5]) + (f[6] + f[7]));
            }
          }
#pragma unroll
          for (int o = 1; o < kVpg; o <<= 1) vs += __shfl_xor_sync(0xffffffffu, vs, o);
          if (i < nvec && i % kVpg == 0) {
            const int mr = i / per_row, c = i % per_row;
            gsum[mr * kbps + c / kVpg] = vs;
          }
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kGemvRows) : "memory");  // the four compute warps
    // 3. Dot products per group as its weights land: y_m += scale * sum_k(x_mk * q_k) +
    //    bias * sum_k(x_mk), the unrounded dequantized weights. The codes enter as exact f32 (128 + q)
    //    and the offset is removed once per group (sum x (128 + q) - 128 sum x; products exact, f32 sums).
    for (int g = 0; g < nkb; ++g) {
      const int s = g % kGemvRing;
      if (!mbar_wait_warp(&full[s], (g / kGemvRing) & 1, &abort_flag, p.status, kDevTimeoutTma)) break;
      uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0;
      float sc = 0.f, bi = 0.f;
      if (active) {
        const uint8_t* hb = wsm + s * kHalfBytes;
        w0 = *reinterpret_cast<const uint4*>(hb + t * 32);
        w1 = *reinterpret_cast<const uint4*>(hb + t * 32 + 16);
        sc = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(hb + 4096 + t * 2));
        bi = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(hb + 4352 + t * 2));
      }
      // The warp's reads of the slot are done: release it to the producer.
      __syncwarp();
      if (lane == 0) mbar_arrive_addr(smem_u32(&empty[s]));
      if (!active) continue;
      const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      // Two accumulator pairs per row (codes 0,1,4,5 and 2,3,6,7 of each word) at R = 1 for a shorter
      // dependency chain; one pair per row otherwise.
      constexpr int kAcc = R == 1 ? 2 : 1;
      float2 tq[R][kAcc];
#pragma unroll
      for (int mr = 0; mr < R; ++mr)
#pragma unroll
        for (int a = 0; a < kAcc; ++a) tq[mr][a] = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        // Codes 2j / 2j+1 of a permuted word sit at bits 4j / 16+4j, so the low nibbles of its bytes are codes
        // 0, 4, 1, 5 and the high nibbles codes 2, 6, 3, 7; one byte permute per code makes the f32 128 + q.
        const uint32_t lo = ws[c] & 0x0F0F0F0Fu, hi = (ws[c] >> 4) & 0x0F0F0F0Fu;
        const float2 q01 = make_float2(code_f32_128(lo, 0), code_f32_128(lo, 2));
        const float2 q23 = make_float2(code_f32_128(hi, 0), code_f32_128(hi, 2));
        const float2 q45 = make_float2(code_f32_128(lo, 1), code_f32_128(lo, 3));
        const float2 q67 = make_float2(code_f32_128(hi, 1), code_f32_128(hi, 3));
        const int kk = g * kKB + c * 8;  // codes kk .. kk+7
#pragma unroll
        for (int mr = 0; mr < R; ++mr) {
          const float4 xa = *reinterpret_cast<const float4*>(xs + mr * kbps * kKB + kk);
          const float4 xb = *reinterpret_cast<const float4*>(xs + mr * kbps * kKB + kk + 4);
          tq[mr][0] = ffma2(q01, make_float2(xa.x, xa.y), tq[mr][0]);
          tq[mr][kAcc - 1] = ffma2(q23, make_float2(xa.z, xa.w), tq[mr][kAcc - 1]);
          tq[mr][0] = ffma2(q45, make_float2(xb.x, xb.y), tq[mr][0]);
          tq[mr][kAcc - 1] = ffma2(q67, make_float2(xb.z, xb.w), tq[mr][kAcc - 1]);
        }
      }
#pragma unroll
      for (int mr = 0; mr < R; ++mr) {
        const float gs = gsum[mr * kbps + g];
        const float dot = kAcc == 2 ? (tq[mr][0].x + tq[mr][0].y) + (tq[mr][kAcc - 1].x + tq[mr][kAcc - 1].y)
                                    : tq[mr][0].x + tq[mr][0].y;
        acc[mr] = fmaf(sc, fmaf(-128.0f, gs, dot), fmaf(bi, gs, acc[mr]));
      }
    }
#pragma unroll
    for (int mr = 0; mr < R; ++mr) part[mr * kGemvRows + t] = acc[mr];
  }
  // 4. Reduce the K splits of this cluster in CTA rank 0 through distributed shared memory.
  cluster_sync_all();
  if (cluster_ctarank() == 0 && active) {
    const uint32_t my_part = smem_u32(part);
    const int nsplit = static_cast<int>(gridDim.y);
    for (int mr = 0; mr < R && mr < p.m; ++mr) {
      // every remote load first, then the sum in split order
      float pv[kGemvMaxSplit];
#pragma unroll
      for (int c = 0; c < kGemvMaxSplit; ++c)
        pv[c] = c < nsplit ? ld_shared_cluster_f32(mapa_shared(my_part + (mr * kGemvRows + t) * 4, c)) : 0.f;
      float v = 0.f;
#pragma unroll
      for (int c = 0; c < kGemvMaxSplit; ++c) v += pv[c];
      if (q.mode == kOutResidualGate)
        static_cast<float*>(q.y)[static_cast<int64_t>(mr) * q.ldy + row] += q.gate[row] * v;
      else if (q.mode == kOutF32)
        static_cast<float*>(q.y)[static_cast<int64_t>(mr) * q.ldy + row] = v;
      else
        static_cast<uint16_t*>(q.y)[static_cast<int64_t>(mr) * q.ldy + row] =
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

// One GEMV launch over jobs[0, n) (n <= kGemvMaxProblems), which share x, its
// pitch and dtype, m and k; every job's rows get their own CTAs along x.
template <int R, bool XF32>
int launch_gemv(aex_ctx* ctx, const QmmJob* jobs, int n, cudaStream_t s) {
  const aex_qweight* w0 = jobs[0].w;
  qmm::GemvParams p{};
  p.x = jobs[0].x;
  p.ldx = jobs[0].ldx;
  p.m = jobs[0].m;
  p.k_blocks = w0->k_blocks;
  p.n_prob = n;
  p.status = ctx->d_status;
  int n_ctas = 0;
  for (int i = 0; i < n; ++i) {
    const QmmJob& j = jobs[i];
    qmm::GemvProblem& q = p.prob[i];
    q.tiles = j.w->tiles;
    q.n = j.w->n;
    q.cta0 = n_ctas;
    q.y = j.y;
    q.ldy = j.ldy;
    q.mode = j.mode;
    q.gate = j.gate;
    n_ctas += (j.w->n + qmm::kGemvRows - 1) / qmm::kGemvRows;
  }
  // The K split (cluster size along K, at most kGemvMaxKbps K blocks per CTA): the one whose CTAs take the
  // fewest waves of the SMs at the residency their shared memory allows, then the largest (more copies in
  // flight per output row).
  auto smem_for = [&](int kb) { return qmm::gemv_smem_bytes(R, kb); };
  auto kern = qmm::gemv_kernel<R, XF32>;
  // CTAs per SM allowed by threads and registers (65536 per SM, allocated per warp in units of 256).
  static const int reg_limit = [&] {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs <= 0) return 1;
    const int per_warp = (fa.numRegs * 32 + 255) / 256 * 256;
    return std::max(1, 65536 / (per_warp * (qmm::kGemvThreads / 32)));
  }();
  constexpr size_t kMaxSmem = 200 * 1024;
  constexpr size_t kSmPerSm = 228 * 1024;  // shared memory of one SM
  const int min_split = (w0->k_blocks + qmm::kGemvMaxKbps - 1) / qmm::kGemvMaxKbps;
  if (min_split > qmm::kGemvMaxSplit)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "qmm gemv: k=%d needs more than %d K splits", w0->k,
                     qmm::kGemvMaxSplit);
  int split = 0;
  int64_t best_waves = 0;
  for (int sp = min_split; sp <= std::min(qmm::kGemvMaxSplit, w0->k_blocks); ++sp) {
    const int kb = (w0->k_blocks + sp - 1) / sp;
    if ((w0->k_blocks + kb - 1) / kb != sp || smem_for(kb) > kMaxSmem) continue;  // an empty split, or too big
    const int64_t per_sm = std::min<int64_t>(std::min({16, 2048 / qmm::kGemvThreads, reg_limit}),
                                             static_cast<int64_t>(kSmPerSm / (smem_for(kb) + 1024)));
    const int64_t slots = per_sm * ctx->sm_count;
    const int64_t waves = (static_cast<int64_t>(n_ctas) * sp + slots - 1) / slots;
    if (split == 0 || waves <= best_waves) {
      split = sp;
      best_waves = waves;
    }
  }
  if (split == 0) return set_error(ctx, AEX_ERR_UNSUPPORTED, "qmm gemv: k=%d too large for %d rows", w0->k, R);
  const int kbps = (w0->k_blocks + split - 1) / split;
  p.kb_per_split = kbps;
  AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kMaxSmem)));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(n_ctas, split, 1);
  cfg.blockDim = dim3(qmm::kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_for(kbps);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = split;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AEX_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, p));
  return check_launch(ctx, "qmm gemv_kernel");
}

template <bool XF32>
int run_gemv_t(aex_ctx* ctx, const QmmJob* jobs, int n, cudaStream_t s) {
  const int m = jobs[0].m;
  if (m <= 1) return launch_gemv<1, XF32>(ctx, jobs, n, s);
  if (m <= 2) return launch_gemv<2, XF32>(ctx, jobs, n, s);
  if (m <= 4) return launch_gemv<4, XF32>(ctx, jobs, n, s);
  if (m <= 8) return launch_gemv<8, XF32>(ctx, jobs, n, s);
  return launch_gemv<16, XF32>(ctx, jobs, n, s);
}

int run_gemv(aex_ctx* ctx, const QmmJob* jobs, int n, cudaStream_t s) {
  return jobs[0].x_f32 ? run_gemv_t<true>(ctx, jobs, n, s) : run_gemv_t<false>(ctx, jobs, n, s);
}

}  // namespace

namespace {

int pair_vec(const QmmJob& j) {
  const int esz = j.mode == qmm::kOutBf16 ? 2 : 4;
  return ((reinterpret_cast<uintptr_t>(j.y) & 15) == 0 && (j.ldy * esz) % 16 == 0 &&
          (reinterpret_cast<uintptr_t>(j.gate) & 15) == 0)
             ? 1
             : 0;
}

// The CTA-pair GEMM over one or two jobs (each m > 16).
int launch_gemm_pair(aex_ctx* ctx, const QmmJob* jobs, int n_jobs, cudaStream_t s) {
  CUtensorMap tm[qmm::kPairMaxProblems];
  qmm::PairParams p{};
  p.n_prob = n_jobs;
  int tiles = 0;
  for (int i = 0; i < n_jobs; ++i) {
    const QmmJob& j = jobs[i];
    uint64_t dims[2] = {static_cast<uint64_t>(j.w->k), static_cast<uint64_t>(j.m)};
    uint64_t strides[1] = {static_cast<uint64_t>(j.ldx) * 2};
    uint32_t box[2] = {64, 128};
    if (int r = make_tmap(ctx, &tm[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, j.x, 2, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
    qmm::PairProblem& q = p.prob[i];
    q.tiles = j.w->tiles;
    q.m = j.m;
    q.n = j.w->n;
    q.k_blocks = j.w->k_blocks;
    q.m_tiles = (j.m + 255) / 256;
    q.tile0 = tiles;
    q.y = j.y;
    q.ldy = j.ldy;
    q.mode = j.mode;
    q.gate = j.gate;
    q.vec = pair_vec(j);
    q.glu_tile0 = j.glu_tile0;
    q.y2 = j.y2;
    q.ldy2 = j.ldy2;
    q.qk_tiles = j.qk_tiles;
    q.prep = j.prep;
    q.prep_k = j.prep_k;
    q.k_tok_major = j.k_tok_major ? 1 : 0;
    q.tok0 = j.tok0;
    q.j_total = j.j_total;
    q.h_total = j.h_total;
    q.norm_q = j.norm_q;
    q.norm_k = j.norm_k;
    q.eps = j.eps;
    q.rope_cos = j.rope_cos;
    q.rope_sin = j.rope_sin;
    tiles += q.m_tiles * j.w->n_tiles;
  }
  if (n_jobs == 1) tm[1] = tm[0];
  p.tiles = tiles;
  auto kern = qmm::gemm_pair_kernel;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(qmm::kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = qmm::kPairSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, qmm::kPairSmem));
  if (ctx->pair_clusters <= 0) {
    // How many 2-CTA clusters of this kernel fit on the device at once (the
    // persistent grid); at most one per SM pair.
    cfg.gridDim = dim3(2 * (ctx->sm_count / 2), 1, 1);
    int n = 0;
    AEX_CUDA_TRY(ctx, cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    if (n <= 0) return set_error(ctx, AEX_ERR_UNSUPPORTED, "qmm: the CTA-pair GEMM cannot be resident on this device");
    ctx->pair_clusters = n;
  }
  const int clusters = std::min(tiles, ctx->pair_clusters);
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  AEX_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, tm[0], tm[1], p, ctx->d_status));
  return check_launch(ctx, "qmm gemm_pair_kernel");
}

bool gemv_path(const aex_qweight* w, int m) { return m <= 16 && w->k_blocks <= qmm::kGemvMaxSplit * qmm::kGemvMaxKbps; }
// The GEMV has no SwiGLU epilogue: jobs that need it take the GEMM at any m.
bool use_gemv(const QmmJob& j) { return gemv_path(j.w, j.m) && j.glu_tile0 >= j.w->n_tiles && j.qk_tiles == 0; }

int run_one(aex_ctx* ctx, const QmmJob& j, cudaStream_t s) {
  if (use_gemv(j)) return run_gemv(ctx, &j, 1, s);
  if (j.x_f32) return set_error(ctx, AEX_ERR_UNSUPPORTED, "qmm: f32 activations take the GEMV path only (m <= 16)");
  return launch_gemm_pair(ctx, &j, 1, s);
}

int check_job(aex_ctx* ctx, const QmmJob& j) {
  if (j.m <= 0) return set_error(ctx, AEX_ERR_INVALID_ARG, "m must be positive");
  if ((reinterpret_cast<uintptr_t>(j.x) & 15) || j.ldx % (j.x_f32 ? 4 : 8) || j.ldx < j.w->k)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "x must be 16-byte aligned with ldx >= k and a row pitch of a multiple "
                     "of 16 bytes");
  if (j.mode == qmm::kOutResidualGate && !j.gate) return set_error(ctx, AEX_ERR_INVALID_ARG, "gate is NULL");
  if (j.glu_tile0 < j.w->n_tiles && (!j.y2 || (reinterpret_cast<uintptr_t>(j.y2) & 15) || j.ldy2 % 8))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "glu output must be 16-byte aligned rows");
  if (j.qk_tiles > 0 && (!j.prep || (reinterpret_cast<uintptr_t>(j.prep) & 15) ||
                         (reinterpret_cast<uintptr_t>(j.prep_k) & 15) || j.qk_tiles != j.h_total ||
                         j.tok0 < 0 || j.tok0 + j.m > j.j_total))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "qk prep epilogue: bad destination, head or token range");
  return AEX_OK;
}

}  // namespace

int qmm_glu_interleave(aex_ctx* ctx, const aex_qweight* src, int plain_rows, int mlp, aex_qweight** out,
                       cudaStream_t s) {
  *out = nullptr;
  if (plain_rows % qmm::kTileN || mlp % 128 || mlp <= 0 || src->n != plain_rows + 2 * mlp)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "glu interleave: n=%d is not %d plain rows + 2 x %d (128-row multiples)",
                     src->n, plain_rows, mlp);
  auto* w = new aex_qweight(*src);
  w->tiles = nullptr;
  cudaError_t e = cudaMalloc(&w->tiles, w->bytes);
  if (e != cudaSuccess) {
    delete w;
    return cuda_error(ctx, e, "cudaMalloc(glu interleave)");
  }
  const int plain_tiles = plain_rows / qmm::kTileN;
  qmm::glu_interleave_kernel<<<dim3(src->k_blocks, 2 * src->n_tiles), 256, 0, s>>>(src->tiles, src->k_blocks,
                                                                                  plain_tiles, mlp, w->tiles);
  if (int r = check_launch(ctx, "glu_interleave_kernel")) {
    cudaFree(w->tiles);
    delete w;
    return r;
  }
  *out = w;
  return AEX_OK;
}

int qmm_run(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy, int mode,
            const float* gate, cudaStream_t s) {
  const QmmJob j{w, x, ldx, m, y, ldy, mode, gate};
  if (int r = check_job(ctx, j)) return r;
  return run_one(ctx, j, s);
}

int qmm_run_job(aex_ctx* ctx, const QmmJob& j, cudaStream_t s) {
  if (int r = check_job(ctx, j)) return r;
  return run_one(ctx, j, s);
}

int qmm_run_gemv_group(aex_ctx* ctx, const QmmJob* jobs, int n, cudaStream_t s) {
  if (n < 1 || n > qmm::kGemvMaxProblems)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "gemv group: %d jobs (1..%d)", n, qmm::kGemvMaxProblems);
  for (int i = 0; i < n; ++i) {
    const QmmJob& j = jobs[i];
    if (int r = check_job(ctx, j)) return r;
    if (!use_gemv(j) || j.x != jobs[0].x || j.ldx != jobs[0].ldx || j.m != jobs[0].m || j.w->k != jobs[0].w->k ||
        j.x_f32 != jobs[0].x_f32)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "gemv group: jobs must share x, ldx, m <= 16, k and the x dtype");
  }
  return run_gemv(ctx, jobs, n, s);
}

int qmm_run2(aex_ctx* ctx, const QmmJob& a, const QmmJob& b, cudaStream_t s) {
  if (int r = check_job(ctx, a)) return r;
  if (int r = check_job(ctx, b)) return r;
  if (!use_gemv(a) && !use_gemv(b)) {
    const QmmJob jobs[2] = {a, b};
    return launch_gemm_pair(ctx, jobs, 2, s);
  }
  if (int r = run_one(ctx, a, s)) return r;
  return run_one(ctx, b, s);
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

int aex_qmm_ex(aex_ctx* ctx, const aex_qweight* w, const void* x, int x_dtype, int64_t ldx, int m, void* y,
               int64_t ldy, int y_dtype, aex_stream stream) {
  using namespace aex;
  if (!ctx || !w || !x || !y) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  if (m <= 0) return set_error(ctx, AEX_ERR_INVALID_ARG, "m must be positive");
  if (x_dtype != AEX_DTYPE_BF16 && x_dtype != AEX_DTYPE_F32)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "x_dtype must be AEX_DTYPE_BF16 or AEX_DTYPE_F32");
  if (y_dtype != AEX_DTYPE_BF16 && y_dtype != AEX_DTYPE_F32)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "y_dtype must be AEX_DTYPE_BF16 or AEX_DTYPE_F32");
  const bool xf32 = x_dtype == AEX_DTYPE_F32;
  if (ldx < w->k || ldx % (xf32 ? 4 : 8) || (reinterpret_cast<uintptr_t>(x) & 15))
    return set_error(ctx, AEX_ERR_INVALID_ARG,
                     "x must be 16-byte aligned with ldx >= k and a row pitch of a multiple of 16 bytes");
  if (ldy < w->n || (reinterpret_cast<uintptr_t>(y) & (y_dtype == AEX_DTYPE_F32 ? 3 : 1)))
    return set_error(ctx, AEX_ERR_INVALID_ARG, "y must be aligned to its element size with ldy >= n");
  if (xf32 && m > 16)
    return set_error(ctx, AEX_ERR_UNSUPPORTED, "f32 activations are supported for m <= 16 (the conditioning GEMV)");
  if (ctx->device != w->device) return set_error(ctx, AEX_ERR_INVALID_ARG, "weight lives on another device");
  if (int r = bind_device(ctx)) return r;
  QmmJob j{w, x, ldx, m, y, ldy, y_dtype == AEX_DTYPE_F32 ? qmm::kOutF32 : qmm::kOutBf16, nullptr};
  j.x_f32 = xf32;
  return qmm_run_job(ctx, j, static_cast<cudaStream_t>(stream));
}

int aex_qmm(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy,
            int y_dtype, aex_stream stream) {
  return aex_qmm_ex(ctx, w, x, AEX_DTYPE_BF16, ldx, m, y, ldy, y_dtype, stream);
}

}  // extern "C"
