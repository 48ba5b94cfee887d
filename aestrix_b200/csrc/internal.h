// internal.h — host-side internals shared by the translation units of
// libaestrix_cuda: the context object, error reporting and TMA tensor-map
// construction.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/aestrix_cuda.h"

struct aex_ctx {
  int device = 0;
  int sm_count = 0;
  int* d_status = nullptr;  // device status word written by kernels on a bounded-wait expiry
  void* scratch = nullptr;  // grown on demand by entry points that need workspace
  size_t scratch_bytes = 0;
  int pair_clusters = 0;    // co-resident 2-CTA clusters of the pair GEMM (0 = not yet queried)
  std::string last_error;
};

struct aex_qweight {
  int device = 0;
  int n = 0, k = 0, group_size = 64;
  int n_tiles = 0;          // ceil(n / 256)
  int k_blocks = 0;         // k / 64
  uint8_t* tiles = nullptr; // tile layout (qmm_sm100.cu): one 9 KB chunk per (256-row tile, 64-wide K block)
  size_t bytes = 0;
};

namespace aex {

int set_error(aex_ctx* ctx, int code, const char* fmt, ...);
int cuda_error(aex_ctx* ctx, cudaError_t e, const char* what);

#define AEX_CUDA_TRY(ctx, expr)                                   \
  do {                                                            \
    cudaError_t _e = (expr);                                      \
    if (_e != cudaSuccess) return ::aex::cuda_error(ctx, _e, #expr); \
  } while (0)

// Ensure the context's device is current on this thread.
int bind_device(aex_ctx* ctx);

// Grow-only context scratch.
int ensure_scratch(aex_ctx* ctx, size_t bytes, void** out);

// Encode a tiled TMA descriptor for a bf16 (or other 2-byte) tensor.
// dims[0] is the contiguous dimension; strides_bytes has rank-1 entries
// (strides of dims 1..rank-1). Returns AEX_OK or AEX_ERR_INVALID_ARG/CUDA.
int make_tmap(aex_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dtype, const void* base, int rank,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swizzle);

// Check the last kernel launch.
int check_launch(aex_ctx* ctx, const char* what);

// ---- internal entry points shared by the DiT engine (dit_engine.cpp)
// qmm with an epilogue mode: 0 bf16 out, 1 f32 out, 2 gated residual
// (y_f32[row, col] += gate[col] * acc). No argument validation beyond m/gate.
int qmm_run(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy, int mode,
            const float* gate, cudaStream_t s);
// Up to two independent linears in one launch where both take the GEMM path
// (the text and image streams of a double block); otherwise one after the other.
struct QmmJob {
  const aex_qweight* w;
  const void* x;
  int64_t ldx;
  int m;
  void* y;
  int64_t ldy;
  int mode;
  const float* gate;
  // Weight tiles from glu_tile0 on are gate/up interleaved (qmm_glu_interleave):
  // their output is silu(g) * u, bf16, into y2 (row pitch ldy2) at column
  // (tile - glu_tile0) * 128.
  int glu_tile0 = 1 << 30;
  uint16_t* y2 = nullptr;
  int64_t ldy2 = 0;
  // Weight tiles before qk_tiles are the Q then K projections of h_total heads
  // (qk_tiles = h_total: two heads per 256-row tile): their output goes through
  // QK-RMSNorm (norm_q / norm_k, eps; NULL: none) + RoPE (rope_cos / rope_sin
  // [j_total, 64]; NULL: none) into prep [2][h_total][j_total][128], row r of
  // this job being token tok0 + r.
  int qk_tiles = 0;
  uint16_t* prep = nullptr;
  // K elsewhere (NULL: in prep after Q): [h_total][j_total][128], or
  // token-major [j_total][h_total][128] when k_tok_major.
  uint16_t* prep_k = nullptr;
  bool k_tok_major = false;
  int tok0 = 0, j_total = 0, h_total = 0;
  const float* norm_q = nullptr;
  const float* norm_k = nullptr;
  float eps = 0.f;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  // x is f32 instead of bf16 (GEMV path only: m <= 16).
  bool x_f32 = false;
};
int qmm_run_job(aex_ctx* ctx, const QmmJob& j, cudaStream_t s);
// One GEMV launch over up to 4 jobs that share x (pointer, pitch, dtype), m <= 16 and k
// (the conditioning's modulation heads).
int qmm_run_gemv_group(aex_ctx* ctx, const QmmJob* jobs, int n, cudaStream_t s);
int qmm_run2(aex_ctx* ctx, const QmmJob& a, const QmmJob& b, cudaStream_t s);
// A copy of `src` (n = plain_rows + 2 * mlp rows: plain rows, then gate rows,
// then up rows) whose tiles after the plain ones each hold 128 gate rows then
// the matching 128 up rows, for the SwiGLU epilogue.
int qmm_glu_interleave(aex_ctx* ctx, const aex_qweight* src, int plain_rows, int mlp, aex_qweight** out,
                       cudaStream_t s);
// QK-RMSNorm + RoPE pre-pass into scratch [2][B][H][S][128] (head-major), or
// [2][B][S][H][128] with out_token_major; K goes to k_out instead when given.
// Tokens s < split use (wq_a, wk_a), the others (wq, wk).
int launch_qk_prep(aex_ctx* ctx, const void* q, const int64_t qs[3], const void* k, const int64_t ks[3], int B, int S,
                   int H, const float* wq, const float* wk, const float* wq_a, const float* wk_a, int split,
                   float eps, const float* cos_t, const float* sin_t, void* out, cudaStream_t stream,
                   void* k_out = nullptr, bool k_token_major = false, bool out_token_major = false);
// The attention kernel on prepared operands: strided [B, S, H, 128] views
// (strides in elements: batch, seq, head) for Q/O with S rows and K/V with
// S_kv rows; optional per-row log2-sum-exp output lse[b*lse_sb + h*lse_sh + row].
// kv_splits > 1 splits the keys into that many contiguous ranges of whole
// 128-key blocks (every range non-empty), computed by separate CTAs: O and lse
// then hold B * kv_splits batches (range r of batch b at b * kv_splits + r),
// each normalized over its own keys, to be combined by merge_splits.
int launch_attention_core(aex_ctx* ctx, const void* q, const int64_t qs[3], const void* k, const int64_t ks[3],
                          const void* v, const int64_t* vs, void* o, const int64_t* os, int B, int S, int S_kv, int H,
                          float scale, float* lse, int64_t lse_sb, int64_t lse_sh, cudaStream_t stream,
                          int kv_splits = 1);
namespace ring {
// out = the k partial outputs ([S][H][128] bf16 each: range r at o + r * o_rs, token stride o_ss, head
// stride o_sh) weighted by 2^(lse_r - lse), lse = log2 sum_r 2^lse_r (range r's log2-sum-exp at
// lse[r * lse_rs + h * S + s]), rounded to bf16 at out[s * out_ss + h * out_sh]; k <= 16.
int merge_splits(aex_ctx* ctx, const void* o, int64_t o_rs, int64_t o_ss, int64_t o_sh, const float* lse,
                 int64_t lse_rs, int k, int S, int H, void* out, int64_t out_ss, int64_t out_sh, cudaStream_t s);
}  // namespace ring
// Key-range count for one attention call of `ctas` CTAs over n_kv key blocks
// on `sms` SMs: the smallest count that fills whole waves noticeably better
// than no split (at most 4, every range non-empty), else 1.
int attention_kv_splits(int ctas, int n_kv, int sms);
// Sequence-parallel attention internals (ring_attention.cpp) for callers that
// prepare Q/K themselves. sp_buffers grows this communicator's state for S
// local rows of H heads and returns where the local operands go: Q head-major
// [H][S][128]; K head-major (directly after Q) or token-major [S][H][128]
// (k_token_major); V token-major [S][H][128]. sp_run then computes the joint
// attention of the local queries against every rank's K/V into out (bf16,
// strides in elements: token, head), by the schedule sp_buffers chose (a ring
// of NCCL sends with log-sum-exp merges, or one all-gather and one call).
struct SpSlots {
  uint16_t* q;
  uint16_t* k;
  bool k_token_major;
  uint16_t* v;
};
int sp_buffers(aex_ctx* ctx, aex_comm* c, int S, int H, SpSlots* out);
int comm_world(const aex_comm* c);
int comm_rank(const aex_comm* c);
int sp_run(aex_ctx* ctx, aex_comm* c, int S, int H, float scale, void* out, int64_t out_ss, int64_t out_sh,
           cudaStream_t s);
// The context a DiT engine was created on.
aex_ctx* dit_context(aex_dit* d);
// The checks every attention entry point applies to its args (shapes, NULL
// and 16-byte-aligned pointers, strides, paired rope tables, eps); AEX_OK or
// AEX_ERR_INVALID_ARG / AEX_ERR_UNSUPPORTED with the message set.
int validate_attention_args(aex_ctx* ctx, const aex_attention_args* a);
// Attention (and prep if args ask for it) on validated args; kv_splits > 1 splits the keys into that many
// ranges (partial outputs in the scratch after the prepared Q/K, merged into args->out).
int joint_attention_impl(aex_ctx* ctx, const aex_attention_args* a, void* scratch, size_t scratch_bytes,
                         cudaStream_t stream, int kv_splits = 1);
// Key ranges the allocating fused call uses for B x S x H on this device (1: no split).
int fused_kv_splits(const aex_ctx* ctx, int B, int S, int H);

}  // namespace aex
