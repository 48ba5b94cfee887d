// dit_engine.cpp — the FLUX.2-klein transformer step on one B200: host-side
// engine over the library's kernels (qmm, attention, glue).
//
// Mirrors the reference direct engine (Sources/ImarelloDirect/DirectDiTStep.swift)
// and its conditioner (DirectConditioner.swift):
//  * one static buffer plan allocated at creation (allocateScratch :155-274);
//  * weights keyed by their MLX names (loadBlocks/loadHead :294-335, 844-884);
//  * one f32 residual X [J, hidden] whose rows [0, l_txt) are the text stream
//    and [l_txt, J) the image stream, so the double->single "concat" blit
//    (encodeBlocks :662-670) disappears;
//  * double block (encodeDouble :546-588, Flux2TransformerBlock
//    TransformerBlock.swift:25-74): per stream LN+mod -> fused Q|K|V linear;
//    joint QK-RMSNorm (norm_added_* on text rows, norm_* on image rows) + RoPE;
//    attention; out-projections with the gated residual fused into the GEMM
//    epilogue; LN+mod -> FFN in -> SwiGLU -> FFN out (gated residual fused);
//  * single block (encodeSingle :590-618, ParallelSelfAttention.swift:30-132):
//    LN+mod -> to_qkv_mlp_proj -> [Q|K|V|g|u]; SwiGLU into the right half of
//    the concat buffer; attention into its left half; to_out with the gated
//    residual fused;
//  * head (encodeDenoiseStep :908-971): norm_out LN+mod on image rows ->
//    proj_out -> velocity; Euler update.
// Modulation vectors are [shift | scale | gate] per set (two sets for each
// double stream, one for the single blocks); norm_out is [scale | shift]
// (DirectConditioner.stepConditioning :172-213, AdaLayerNormContinuous.swift).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "dit_internal.h"

struct aex_dit {
  aex_ctx* ctx = nullptr;
  aex_dit_config cfg{};
  int J = 0, C = 0, H = 0, mlp = 0, proj = 0, cat = 0;
  std::unordered_map<std::string, aex_qweight*> lin;
  std::unordered_map<std::string, float*> norms;
  std::vector<void*> allocs;
  // buffers
  float* X = nullptr;         // [J, C] f32 residual (text rows first)
  float* E0 = nullptr;        // [l_txt, C] f32 projected context
  uint16_t* NH = nullptr;     // [J, C] bf16 LN+mod output
  uint16_t* PROJ = nullptr;   // [J, max(3C + 2 mlp, 2 mlp)] bf16: Q|K|V(|g|u) or FFN-in output
  uint16_t* ATT = nullptr;    // [J, C + mlp] bf16: attention output | SwiGLU (single); SwiGLU [rows, mlp] (double FFN)
  uint16_t* PREP = nullptr;   // [2][H][J][128] bf16 normalized + rotated Q, K
  float* COS = nullptr;       // [J, 64]
  float* SIN = nullptr;
  uint16_t* LAT16 = nullptr;  // [l_img, in_ch] bf16
  float* PRED = nullptr;      // [l_img, in_ch] f32 velocity
  float* LATB = nullptr;      // [l_img, in_ch] f32 Euler ping-pong
  float* TSIN = nullptr;      // [timestep_dim]
  float* T1 = nullptr;        // [C] time MLP hidden, then silu of it in place
  float* TEMB = nullptr;      // [C]
  float* TEMBS = nullptr;     // [C] silu(temb), the modulation heads' input
  float* MOD_IMG = nullptr;   // [6C]
  float* MOD_TXT = nullptr;   // [6C]
  float* MOD_SINGLE = nullptr;  // [3C]
  float* MOD_OUT = nullptr;   // [2C]
  float* CUR = nullptr;       // [2] this step's timestep (sigma * 1000) and dt, read by the kernels
  float* STEPS = nullptr;     // [2 * kMaxGraphSteps] (timestep, dt) per step of a replayed denoise
  int* STEP_I = nullptr;      // index of the next STEPS entry
  bool rope_set = false, context_set = false, timestep_set = false;
  // One denoise step (step_select, conditioning, forward, in-place Euler on LATB) captured as a CUDA
  // graph by aex_dit_denoise and replayed once per step; dropped when weights change.
  cudaGraphExec_t step_graph = nullptr;
  cudaStream_t cap_stream = nullptr;  // engine-owned stream the step is captured on (never the legacy stream)
  // Sequence parallelism (aex_dit_set_sequence_parallel): this engine holds one contiguous shard of the
  // joint sequence; joint attention runs as a ring over `comm`. The scheduler's image length is the
  // whole image's (l_img_sched).
  aex_comm* comm = nullptr;
  int l_img_sched = 0;
};

namespace aex {

aex_ctx* dit_context(aex_dit* d) { return d->ctx; }

namespace {

constexpr int kMaxGraphSteps = 1024;

void drop_graph(aex_dit* d) {
  if (d->step_graph) {
    cudaGraphExecDestroy(d->step_graph);
    d->step_graph = nullptr;
  }
}

template <class T>
int dalloc(aex_dit* d, T** p, size_t count) {
  void* v = nullptr;
  const cudaError_t e = cudaMalloc(&v, count * sizeof(T));
  if (e != cudaSuccess) return cuda_error(d->ctx, e, "cudaMalloc(dit buffer)");
  d->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return AEX_OK;
}

std::string blk(const char* kind, int i, const char* leaf) {
  return std::string(kind) + "." + std::to_string(i) + "." + leaf;
}

// Concatenate three [n, k] tile-layout weights along n into one (their n must
// be multiples of the 256-row tile, so the chunks simply follow each other).
int fuse3(aex_dit* d, const std::string& a, const std::string& b, const std::string& c, const std::string& out,
          cudaStream_t s) {
  auto ia = d->lin.find(a), ib = d->lin.find(b), ic = d->lin.find(c);
  if (ia == d->lin.end() || ib == d->lin.end() || ic == d->lin.end())
    return set_error(d->ctx, AEX_ERR_INVALID_ARG, "missing linear among %s / %s / %s", a.c_str(), b.c_str(),
                     c.c_str());
  aex_qweight* w[3] = {ia->second, ib->second, ic->second};
  for (auto* x : w)
    if (x->k != w[0]->k || x->n % 256)
      return set_error(d->ctx, AEX_ERR_UNSUPPORTED, "cannot fuse %s: shapes differ or n %% 256 != 0", out.c_str());
  auto* f = new aex_qweight();
  f->device = d->ctx->device;
  f->n = w[0]->n + w[1]->n + w[2]->n;
  f->k = w[0]->k;
  f->n_tiles = w[0]->n_tiles + w[1]->n_tiles + w[2]->n_tiles;
  f->k_blocks = w[0]->k_blocks;
  f->bytes = w[0]->bytes + w[1]->bytes + w[2]->bytes;
  cudaError_t e = cudaMalloc(&f->tiles, f->bytes);
  if (e != cudaSuccess) {
    delete f;
    return cuda_error(d->ctx, e, "cudaMalloc(fused qkv)");
  }
  size_t off = 0;
  for (auto* x : w) {
    e = cudaMemcpyAsync(f->tiles + off, x->tiles, x->bytes, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_error(d->ctx, e, "cudaMemcpyAsync(fused qkv)");
    off += x->bytes;
  }
  d->lin[out] = f;
  return AEX_OK;
}

// "<name>#glu": the gate/up-interleaved copy of a linear whose last 2 * mlp
// rows are [gate | up] (qmm_glu_interleave), built once and dropped when
// <name> is re-loaded.
int glu_copy(aex_dit* d, const std::string& name, int plain_rows, cudaStream_t s) {
  const std::string out = name + "#glu";
  if (d->lin.count(out)) return AEX_OK;
  auto it = d->lin.find(name);
  if (it == d->lin.end()) return set_error(d->ctx, AEX_ERR_INVALID_ARG, "missing linear %s", name.c_str());
  aex_qweight* w = nullptr;
  if (int r = qmm_glu_interleave(d->ctx, it->second, plain_rows, d->mlp, &w, s)) return r;
  d->lin[out] = w;
  return AEX_OK;
}

const aex_qweight* need_lin(aex_dit* d, const std::string& name, int n, int k) {
  auto it = d->lin.find(name);
  if (it == d->lin.end()) {
    set_error(d->ctx, AEX_ERR_INVALID_ARG, "linear '%s' not loaded", name.c_str());
    return nullptr;
  }
  if (it->second->n != n || it->second->k != k) {
    set_error(d->ctx, AEX_ERR_INVALID_ARG, "linear '%s' is [%d, %d], expected [%d, %d]", name.c_str(), it->second->n,
              it->second->k, n, k);
    return nullptr;
  }
  return it->second;
}

const float* need_norm(aex_dit* d, const std::string& name) {
  auto it = d->norms.find(name);
  if (it == d->norms.end()) {
    set_error(d->ctx, AEX_ERR_INVALID_ARG, "norm '%s' not loaded", name.c_str());
    return nullptr;
  }
  return it->second;
}

#define AEX_TRY(expr)           \
  do {                          \
    if (int _r = (expr)) return _r; \
  } while (0)

#define AEX_NEED(var, expr)              \
  auto var = (expr);                     \
  if (!var) return AEX_ERR_INVALID_ARG;

// Joint attention on prepared operands: q/k in PREP (head-major), v and out
// strided views of the engine's buffers.
int attend(aex_dit* d, const uint16_t* v, int64_t v_ld, uint16_t* out, int64_t out_ld, cudaStream_t s) {
  const int J = d->J, H = d->H;
  const int64_t plane = static_cast<int64_t>(H) * J * 128;
  aex_attention_args a{};
  a.q = {d->PREP, plane, 128, static_cast<int64_t>(J) * 128};
  a.k = {d->PREP + plane, plane, 128, static_cast<int64_t>(J) * 128};
  a.v = {const_cast<uint16_t*>(v), static_cast<int64_t>(J) * v_ld, v_ld, 128};
  a.out = {out, static_cast<int64_t>(J) * out_ld, out_ld, 128};
  a.batch = 1;
  a.seq = J;
  a.heads = H;
  a.head_dim = 128;
  a.scale = 1.0f / std::sqrt(128.0f);
  return joint_attention_impl(d->ctx, &a, nullptr, 0, s);
}

// One or two GEMM-path jobs in one launch; a job without rows (the text stream
// of a sequence shard that holds none) is left out.
int run_jobs(aex_dit* d, const QmmJob& a, const QmmJob& b, cudaStream_t s) {
  if (a.m <= 0) return b.m > 0 ? qmm_run_job(d->ctx, b, s) : AEX_OK;
  if (b.m <= 0) return qmm_run_job(d->ctx, a, s);
  return qmm_run2(d->ctx, a, b, s);
}

int ln_mod_rows(aex_dit* d, const float* x, int rows, const float* scale, const float* shift, uint16_t* y,
                cudaStream_t s) {
  if (rows <= 0) return AEX_OK;
  return glue::ln_mod(d->ctx, x, d->C, rows, d->C, scale, shift, d->cfg.ln_eps, y, d->C, s);
}

// Where Q, K and V go for the joint attention: Q and K after QK-RMSNorm + RoPE
// (the QKV GEMM's epilogue writes them) head-major [2][H][J][128] in this GPU's
// PREP buffer or, sequence-parallel, this rank's slots of the exchange state
// (V then copied into its slot by joint_attend).
int qk_destination(aex_dit* d, SpSlots* sl) {
  if (d->comm) return sp_buffers(d->ctx, d->comm, d->J, d->H, sl);
  sl->q = d->PREP;
  sl->k = nullptr;
  sl->k_token_major = false;
  sl->v = nullptr;
  return AEX_OK;
}

// A QKV job with the QK-RMSNorm + RoPE epilogue for rows [tok0, tok0 + m) of the joint sequence.
void with_qk_prep(aex_dit* d, QmmJob& j, const SpSlots& sl, int tok0, const float* wq, const float* wk) {
  j.qk_tiles = d->H;
  j.prep = sl.q;
  j.prep_k = sl.k;
  j.k_tok_major = sl.k_token_major;
  j.tok0 = tok0;
  j.j_total = d->J;
  j.h_total = d->H;
  j.norm_q = wq;
  j.norm_k = wk;
  j.eps = d->cfg.rms_eps;
  j.rope_cos = d->COS;
  j.rope_sin = d->SIN;
}

// Joint attention on the prepared Q / K (qk_destination) and the V columns of PROJ (row pitch ld) into out:
// on this GPU, or over the sequence shards of all ranks.
int joint_attend(aex_dit* d, const SpSlots& sl, int64_t ld, uint16_t* out, int64_t out_ld, cudaStream_t s) {
  const int J = d->J, H = d->H, C = d->C;
  const uint16_t* v = d->PROJ + 2 * C;
  if (d->comm) {
    AEX_CUDA_TRY(d->ctx, cudaMemcpy2DAsync(sl.v, static_cast<size_t>(H) * 256, v, static_cast<size_t>(ld) * 2,
                                           static_cast<size_t>(H) * 256, J, cudaMemcpyDeviceToDevice, s));
    return sp_run(d->ctx, d->comm, J, H, 1.0f / std::sqrt(128.0f), out, out_ld, 128, s);
  }
  return attend(d, v, ld, out, out_ld, s);
}

int double_block(aex_dit* d, int i, cudaStream_t s) {
  const int C = d->C, J = d->J, lt = d->cfg.l_txt, li = d->cfg.l_img, mlp = d->mlp;
  const float eps_ln = d->cfg.ln_eps;
  float* Xt = d->X;
  float* Xi = d->X + static_cast<int64_t>(lt) * C;
  uint16_t* NHt = d->NH;
  uint16_t* NHi = d->NH + static_cast<int64_t>(lt) * C;
  const float* mi = d->MOD_IMG;  // set 0 (msa): shift, scale, gate at 0, C, 2C; set 1 (mlp) at 3C...
  const float* mt = d->MOD_TXT;
  AEX_NEED(qkv_i, need_lin(d, blk("transformer_blocks", i, "attn.qkv"), 3 * C, C));
  AEX_NEED(qkv_t, need_lin(d, blk("transformer_blocks", i, "attn.add_qkv"), 3 * C, C));
  AEX_NEED(out_i, need_lin(d, blk("transformer_blocks", i, "attn.to_out"), C, C));
  AEX_NEED(out_t, need_lin(d, blk("transformer_blocks", i, "attn.to_add_out"), C, C));
  AEX_NEED(ffi_i, need_lin(d, blk("transformer_blocks", i, "ff.linear_in#glu"), 2 * mlp, C));
  AEX_NEED(ffo_i, need_lin(d, blk("transformer_blocks", i, "ff.linear_out"), C, mlp));
  AEX_NEED(ffi_t, need_lin(d, blk("transformer_blocks", i, "ff_context.linear_in#glu"), 2 * mlp, C));
  AEX_NEED(ffo_t, need_lin(d, blk("transformer_blocks", i, "ff_context.linear_out"), C, mlp));
  AEX_NEED(nq, need_norm(d, blk("transformer_blocks", i, "attn.norm_q")));
  AEX_NEED(nk, need_norm(d, blk("transformer_blocks", i, "attn.norm_k")));
  AEX_NEED(naq, need_norm(d, blk("transformer_blocks", i, "attn.norm_added_q")));
  AEX_NEED(nak, need_norm(d, blk("transformer_blocks", i, "attn.norm_added_k")));
  // attention half
  AEX_TRY(ln_mod_rows(d, Xt, lt, mt + C, mt, NHt, s));
  AEX_TRY(ln_mod_rows(d, Xi, li, mi + C, mi, NHi, s));
  const int64_t pq = 3 * C;  // PROJ row pitch for Q|K|V
  // Each text-stream linear shares one launch with its image-stream twin. Q and K leave the GEMM normalized
  // and rotated (per-stream norm weights: norm_added_* on text rows, norm_* on image rows); V goes to PROJ.
  SpSlots sl{};
  AEX_TRY(qk_destination(d, &sl));
  QmmJob jt{qkv_t, NHt, C, lt, d->PROJ, pq, 0, nullptr};
  QmmJob ji{qkv_i, NHi, C, li, d->PROJ + static_cast<int64_t>(lt) * pq, pq, 0, nullptr};
  with_qk_prep(d, jt, sl, 0, naq, nak);
  with_qk_prep(d, ji, sl, lt, nq, nk);
  AEX_TRY(run_jobs(d, jt, ji, s));
  AEX_TRY(joint_attend(d, sl, pq, d->ATT, C, s));
  AEX_TRY(run_jobs(d, QmmJob{out_t, d->ATT, C, lt, Xt, C, 2, mt + 2 * C},
                   QmmJob{out_i, d->ATT + static_cast<int64_t>(lt) * C, C, li, Xi, C, 2, mi + 2 * C}, s));
  // MLP half (per stream)
  AEX_TRY(ln_mod_rows(d, Xt, lt, mt + 4 * C, mt + 3 * C, NHt, s));
  AEX_TRY(ln_mod_rows(d, Xi, li, mi + 4 * C, mi + 3 * C, NHi, s));
  uint16_t* SWt = d->ATT;                                   // [lt, mlp]
  uint16_t* SWi = d->ATT + static_cast<int64_t>(lt) * mlp;  // [li, mlp]
  // linear_in with the SwiGLU in its epilogue (gate/up interleaved weights): silu(g) * u straight into SW.
  QmmJob ff_t{ffi_t, NHt, C, lt, nullptr, 0, 0, nullptr};
  QmmJob ff_i{ffi_i, NHi, C, li, nullptr, 0, 0, nullptr};
  ff_t.glu_tile0 = ff_i.glu_tile0 = 0;
  ff_t.y2 = SWt;
  ff_i.y2 = SWi;
  ff_t.ldy2 = ff_i.ldy2 = mlp;
  AEX_TRY(run_jobs(d, ff_t, ff_i, s));
  AEX_TRY(run_jobs(d, QmmJob{ffo_t, SWt, mlp, lt, Xt, C, 2, mt + 5 * C},
                   QmmJob{ffo_i, SWi, mlp, li, Xi, C, 2, mi + 5 * C}, s));
  return AEX_OK;
}

int single_block(aex_dit* d, int i, cudaStream_t s) {
  const int C = d->C, J = d->J;
  AEX_NEED(proj, need_lin(d, blk("single_transformer_blocks", i, "attn.to_qkv_mlp_proj#glu"), d->proj, C));
  AEX_NEED(out, need_lin(d, blk("single_transformer_blocks", i, "attn.to_out"), C, d->cat));
  AEX_NEED(nq, need_norm(d, blk("single_transformer_blocks", i, "attn.norm_q")));
  AEX_NEED(nk, need_norm(d, blk("single_transformer_blocks", i, "attn.norm_k")));
  const float* ms = d->MOD_SINGLE;
  AEX_TRY(glue::ln_mod(d->ctx, d->X, C, J, C, ms + C, ms, d->cfg.ln_eps, d->NH, C, s));
  const int64_t pp = d->proj;
  // Q|K|V columns into PROJ; the gate/up tiles (interleaved) go through the SwiGLU epilogue into
  // columns [C, C + mlp) of the concat buffer (ParallelSelfAttention.swift:117-123).
  QmmJob pj{proj, d->NH, C, J, d->PROJ, pp, 0, nullptr};
  pj.glu_tile0 = 3 * C / 256;
  pj.y2 = d->ATT + C;
  pj.ldy2 = d->cat;
  SpSlots sl{};
  AEX_TRY(qk_destination(d, &sl));
  with_qk_prep(d, pj, sl, 0, nq, nk);  // Q, K normalized and rotated in the epilogue
  AEX_TRY(qmm_run_job(d->ctx, pj, s));
  AEX_TRY(joint_attend(d, sl, pp, d->ATT, d->cat, s));
  AEX_TRY(qmm_run(d->ctx, out, d->ATT, d->cat, J, d->X, C, 2, ms + 2 * C, s));
  return AEX_OK;
}

// An f32-activation GEMV job (the conditioner's f32 qmm, affine_qmm_t_float_gs_64_b_4).
QmmJob f32_job(const aex_qweight* w, const float* x, int k, float* y, int n) {
  QmmJob j{w, x, k, 1, y, n, 1, nullptr};
  j.x_f32 = true;
  return j;
}

// Step conditioning from the timestep in CUR[0] (DirectConditioner.stepConditioning,
// Sources/ImarelloDirect/DirectConditioner.swift:168-213), in f32 like the reference's f32 qmm
// chain: sinusoid -> linear_1 -> SiLU -> linear_2 -> temb -> SiLU -> the modulation vectors of the
// double (img, txt), single and output layers (the four heads read the same SiLU(temb): one launch).
int conditioning(aex_dit* d, cudaStream_t s) {
  const int C = d->C, td = d->cfg.timestep_dim;
  AEX_NEED(l1, need_lin(d, "time_guidance_embed.linear_1", C, td));
  AEX_NEED(l2, need_lin(d, "time_guidance_embed.linear_2", C, C));
  AEX_NEED(mimg, need_lin(d, "double_stream_modulation_img.linear", 6 * C, C));
  AEX_NEED(mtxt, need_lin(d, "double_stream_modulation_txt.linear", 6 * C, C));
  AEX_NEED(msin, need_lin(d, "single_stream_modulation.linear", 3 * C, C));
  AEX_NEED(mout, need_lin(d, "norm_out.linear", 2 * C, C));
  AEX_TRY(glue::timestep_embedding(d->ctx, d->CUR, td, d->TSIN, s));
  AEX_TRY(qmm_run_job(d->ctx, f32_job(l1, d->TSIN, td, d->T1, C), s));
  AEX_TRY(glue::silu_f32(d->ctx, d->T1, C, d->T1, s));
  AEX_TRY(qmm_run_job(d->ctx, f32_job(l2, d->T1, C, d->TEMB, C), s));
  AEX_TRY(glue::silu_f32(d->ctx, d->TEMB, C, d->TEMBS, s));
  const QmmJob heads[4] = {f32_job(mimg, d->TEMBS, C, d->MOD_IMG, 6 * C), f32_job(mtxt, d->TEMBS, C, d->MOD_TXT, 6 * C),
                           f32_job(msin, d->TEMBS, C, d->MOD_SINGLE, 3 * C), f32_job(mout, d->TEMBS, C, d->MOD_OUT, 2 * C)};
  AEX_TRY(qmm_run_gemv_group(d->ctx, heads, 4, s));
  d->timestep_set = true;
  return AEX_OK;
}

int forward(aex_dit* d, const float* latents, float* velocity, cudaStream_t s);

// One replayable denoise step on LATB in place: scalars of step (*STEP_I)++,
// conditioning, forward, Euler.
int graph_step(aex_dit* d, cudaStream_t s) {
  AEX_TRY(glue::step_select(d->ctx, d->STEPS, d->STEP_I, d->CUR, s));
  AEX_TRY(conditioning(d, s));
  AEX_TRY(forward(d, d->LATB, d->PRED, s));
  return glue::euler(d->ctx, d->LATB, d->PRED, d->CUR + 1,
                     static_cast<int64_t>(d->cfg.l_img) * d->cfg.in_channels, d->LATB, s);
}

// Records graph_step (nothing executes) on the engine's own stream; the graph
// is then launched on the caller's stream.
int capture_step(aex_dit* d) {
  if (!d->cap_stream) AEX_CUDA_TRY(d->ctx, cudaStreamCreateWithFlags(&d->cap_stream, cudaStreamNonBlocking));
  cudaStream_t s = d->cap_stream;
  AEX_CUDA_TRY(d->ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  const int r = graph_step(d, s);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(s, &g);
  if (r || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return r ? r : cuda_error(d->ctx, e, "cudaStreamEndCapture(denoise step)");
  }
  const cudaError_t ei = cudaGraphInstantiate(&d->step_graph, g, 0);
  cudaGraphDestroy(g);
  if (ei != cudaSuccess) {
    d->step_graph = nullptr;
    return cuda_error(d->ctx, ei, "cudaGraphInstantiate(denoise step)");
  }
  return AEX_OK;
}

// Derived weights, built once outside any captured step: fused Q|K|V of the
// double blocks and the gate/up-interleaved feed-forward inputs.
int prepare_weights(aex_dit* d, cudaStream_t s) {
  for (int i = 0; i < d->cfg.n_double; ++i) {
    AEX_TRY(glu_copy(d, blk("transformer_blocks", i, "ff.linear_in"), 0, s));
    AEX_TRY(glu_copy(d, blk("transformer_blocks", i, "ff_context.linear_in"), 0, s));
    if (!d->lin.count(blk("transformer_blocks", i, "attn.qkv")))
      AEX_TRY(fuse3(d, blk("transformer_blocks", i, "attn.to_q"), blk("transformer_blocks", i, "attn.to_k"),
                    blk("transformer_blocks", i, "attn.to_v"), blk("transformer_blocks", i, "attn.qkv"), s));
    if (!d->lin.count(blk("transformer_blocks", i, "attn.add_qkv")))
      AEX_TRY(fuse3(d, blk("transformer_blocks", i, "attn.add_q_proj"), blk("transformer_blocks", i, "attn.add_k_proj"),
                    blk("transformer_blocks", i, "attn.add_v_proj"), blk("transformer_blocks", i, "attn.add_qkv"), s));
  }
  for (int i = 0; i < d->cfg.n_single; ++i)
    AEX_TRY(glu_copy(d, blk("single_transformer_blocks", i, "attn.to_qkv_mlp_proj"), 3 * d->C, s));
  return AEX_OK;
}

int forward(aex_dit* d, const float* latents, float* velocity, cudaStream_t s) {
  if (!d->rope_set || !d->context_set || !d->timestep_set)
    return set_error(d->ctx, AEX_ERR_INVALID_ARG, "set rope, context and timestep before forward");
  const int C = d->C, lt = d->cfg.l_txt, li = d->cfg.l_img, ic = d->cfg.in_channels;
  AEX_NEED(xemb, need_lin(d, "x_embedder", C, ic));
  AEX_NEED(pout, need_lin(d, "proj_out", ic, C));
  AEX_TRY(prepare_weights(d, s));
  // Embedders: image rows from x_embedder (f32 out), text rows from the projected context.
  AEX_TRY(glue::f32_to_bf16(d->ctx, latents, static_cast<int64_t>(li) * ic, d->LAT16, s));
  AEX_TRY(qmm_run(d->ctx, xemb, d->LAT16, ic, li, d->X + static_cast<int64_t>(lt) * C, C, 1, nullptr, s));
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->X, d->E0, static_cast<size_t>(lt) * C * 4, cudaMemcpyDeviceToDevice, s));
  for (int i = 0; i < d->cfg.n_double; ++i) AEX_TRY(double_block(d, i, s));
  for (int i = 0; i < d->cfg.n_single; ++i) AEX_TRY(single_block(d, i, s));
  // Head: norm_out (scale | shift) on image rows, proj_out -> f32 velocity.
  uint16_t* NHi = d->NH + static_cast<int64_t>(lt) * C;
  AEX_TRY(glue::ln_mod(d->ctx, d->X + static_cast<int64_t>(lt) * C, C, li, C, d->MOD_OUT, d->MOD_OUT + C,
                       d->cfg.ln_eps, NHi, C, s));
  AEX_TRY(qmm_run(d->ctx, pout, NHi, C, li, velocity, ic, 1, nullptr, s));
  return AEX_OK;
}

// Flux2Scheduler (Sources/ImarelloCore/Flux2Scheduler.swift:20-109): linear mu
// from the image sequence length, exponential time shift of linspace(1, 1/N, N),
// terminal 0; timesteps = sigmas * 1000.
void schedule(int steps, int l_img, std::vector<float>& sigmas, std::vector<float>& timesteps) {
  const float m = (1.15f - 0.5f) / static_cast<float>(4096 - 256);
  const float mu = m * static_cast<float>(l_img) + (0.5f - m * 256.0f);
  sigmas.assign(steps + 1, 0.f);
  timesteps.assign(steps, 0.f);
  for (int i = 0; i < steps; ++i) {
    const float t = steps == 1 ? 1.0f
                               : 1.0f + (1.0f / static_cast<float>(steps) - 1.0f) * static_cast<float>(i) /
                                            static_cast<float>(steps - 1);
    const float e = std::exp(mu);
    sigmas[i] = e / (e + (1.0f / t - 1.0f));
    timesteps[i] = sigmas[i] * 1000.0f;
  }
}

}  // namespace
}  // namespace aex

extern "C" {

int aex_dit_create(aex_ctx* ctx, const aex_dit_config* cfg, aex_dit** out) {
  using namespace aex;
  if (!ctx || !cfg || !out) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  *out = nullptr;
  const aex_dit_config& c = *cfg;
  if (c.hidden <= 0 || c.heads <= 0 || c.hidden != c.heads * 128)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "hidden must be heads * 128 (head_dim 128)");
  if (c.n_double < 0 || c.n_single < 0 || c.mlp_hidden <= 0 || c.mlp_hidden % 128 || c.hidden % 256 ||
      c.in_channels % 64 || c.text_dim % 64 || c.timestep_dim % 64 || c.l_txt < 0 || c.l_img <= 0)
    return set_error(ctx, AEX_ERR_INVALID_ARG,
                     "dims must be positive; hidden a multiple of 256; mlp_hidden of 128; in_channels, "
                     "text_dim, timestep_dim of 64");
  if (int r = bind_device(ctx)) return r;
  auto* d = new aex_dit();
  d->ctx = ctx;
  d->cfg = c;
  d->C = c.hidden;
  d->H = c.heads;
  d->J = c.l_txt + c.l_img;
  d->l_img_sched = c.l_img;
  d->mlp = c.mlp_hidden;
  d->proj = 3 * c.hidden + 2 * c.mlp_hidden;
  d->cat = c.hidden + c.mlp_hidden;
  const size_t J = d->J, C = d->C;
  const size_t proj_w = std::max<size_t>(d->proj, 2 * static_cast<size_t>(d->mlp));
  int r = AEX_OK;
  if (!r) r = dalloc(d, &d->X, J * C);
  if (!r) r = dalloc(d, &d->E0, static_cast<size_t>(std::max(c.l_txt, 1)) * C);
  if (!r) r = dalloc(d, &d->NH, J * C);
  if (!r) r = dalloc(d, &d->PROJ, J * proj_w);
  if (!r) r = dalloc(d, &d->ATT, J * static_cast<size_t>(d->cat));
  if (!r) r = dalloc(d, &d->PREP, 2 * J * C);
  if (!r) r = dalloc(d, &d->COS, J * 64);
  if (!r) r = dalloc(d, &d->SIN, J * 64);
  if (!r) r = dalloc(d, &d->LAT16, static_cast<size_t>(c.l_img) * c.in_channels);
  if (!r) r = dalloc(d, &d->PRED, static_cast<size_t>(c.l_img) * c.in_channels);
  if (!r) r = dalloc(d, &d->LATB, static_cast<size_t>(c.l_img) * c.in_channels);
  if (!r) r = dalloc(d, &d->TSIN, static_cast<size_t>(c.timestep_dim));
  if (!r) r = dalloc(d, &d->T1, C);
  if (!r) r = dalloc(d, &d->TEMB, C);
  if (!r) r = dalloc(d, &d->TEMBS, C);
  if (!r) r = dalloc(d, &d->MOD_IMG, 6 * C);
  if (!r) r = dalloc(d, &d->MOD_TXT, 6 * C);
  if (!r) r = dalloc(d, &d->MOD_SINGLE, 3 * C);
  if (!r) r = dalloc(d, &d->MOD_OUT, 2 * C);
  if (!r) r = dalloc(d, &d->CUR, 2);
  if (!r) r = dalloc(d, &d->STEPS, 2 * static_cast<size_t>(kMaxGraphSteps));
  if (!r) r = dalloc(d, &d->STEP_I, 1);
  if (r) {
    aex_dit_destroy(d);
    return r;
  }
  *out = d;
  return AEX_OK;
}

void aex_dit_destroy(aex_dit* d) {
  if (!d) return;
  cudaSetDevice(d->ctx->device);
  cudaDeviceSynchronize();
  aex::drop_graph(d);
  if (d->cap_stream) cudaStreamDestroy(d->cap_stream);
  for (auto& kv : d->lin) aex_qweight_destroy(kv.second);
  for (auto& kv : d->norms) cudaFree(kv.second);
  for (void* p : d->allocs) cudaFree(p);
  delete d;
}

int aex_dit_load_linear(aex_dit* d, const char* name, const uint32_t* packed, const uint16_t* scales,
                        const uint16_t* biases, int n, int k, aex_stream stream) {
  using namespace aex;
  if (!d || !name) return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  aex_qweight* w = nullptr;
  if (int r = aex_qweight_create(d->ctx, packed, scales, biases, n, k, 64, 4, &w, stream)) return r;
  drop_graph(d);
  auto it = d->lin.find(name);
  if (it != d->lin.end()) aex_qweight_destroy(it->second);
  d->lin[name] = w;
  // A re-loaded part invalidates a fused Q|K|V or a gate/up-interleaved copy built from it.
  const std::string s(name);
  auto glu = d->lin.find(s + "#glu");
  if (glu != d->lin.end()) {
    aex_qweight_destroy(glu->second);
    d->lin.erase(glu);
  }
  for (const char* part : {"attn.to_q", "attn.to_k", "attn.to_v", "attn.add_q_proj", "attn.add_k_proj",
                           "attn.add_v_proj"}) {
    const std::string p(part);
    if (s.size() > p.size() && s.compare(s.size() - p.size(), p.size(), p) == 0) {
      const std::string prefix = s.substr(0, s.size() - p.size());
      for (const char* fused : {"attn.qkv", "attn.add_qkv"}) {
        auto f = d->lin.find(prefix + fused);
        if (f != d->lin.end()) {
          aex_qweight_destroy(f->second);
          d->lin.erase(f);
        }
      }
    }
  }
  return AEX_OK;
}

int aex_dit_load_norm(aex_dit* d, const char* name, const float* weight, aex_stream stream) {
  using namespace aex;
  if (!d || !name || !weight) return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  if (int r = bind_device(d->ctx)) return r;
  float* w = nullptr;
  auto it = d->norms.find(name);
  if (it != d->norms.end()) {
    w = it->second;
  } else {
    AEX_CUDA_TRY(d->ctx, cudaMalloc(&w, 128 * sizeof(float)));
    d->norms[name] = w;
    drop_graph(d);
  }
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(w, weight, 128 * sizeof(float), cudaMemcpyDeviceToDevice,
                                       static_cast<cudaStream_t>(stream)));
  return AEX_OK;
}

int aex_dit_set_rope(aex_dit* d, const float* cos_t, const float* sin_t, aex_stream stream) {
  using namespace aex;
  if (!d || !cos_t || !sin_t) return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  if (int r = bind_device(d->ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  const size_t bytes = static_cast<size_t>(d->J) * 64 * sizeof(float);
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->COS, cos_t, bytes, cudaMemcpyDeviceToDevice, s));
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->SIN, sin_t, bytes, cudaMemcpyDeviceToDevice, s));
  d->rope_set = true;
  return AEX_OK;
}

int aex_dit_project_context(aex_dit* d, const void* embeds, aex_stream stream) {
  using namespace aex;
  if (!d || !embeds) return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  if (int r = bind_device(d->ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  const int C = d->C, lt = d->cfg.l_txt;
  if (lt == 0) {  // a sequence shard without text rows
    d->context_set = true;
    return AEX_OK;
  }
  AEX_NEED(ctxemb, need_lin(d, "context_embedder", C, d->cfg.text_dim));
  // bf16 output (the reference's bf16 qmm), widened to the f32 text residual.
  AEX_TRY(qmm_run(d->ctx, ctxemb, embeds, d->cfg.text_dim, lt, d->NH, C, 0, nullptr, s));
  AEX_TRY(glue::bf16_to_f32_rows(d->ctx, d->NH, C, lt, C, d->E0, C, s));
  d->context_set = true;
  return AEX_OK;
}

int aex_dit_set_timestep(aex_dit* d, float timestep, aex_stream stream) {
  using namespace aex;
  if (!d) return set_error(nullptr, AEX_ERR_INVALID_ARG, "NULL dit");
  if (int r = bind_device(d->ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  AEX_TRY(glue::set_scalar(d->ctx, d->CUR, timestep, s));
  return conditioning(d, s);
}

int aex_dit_forward(aex_dit* d, const float* latents, float* velocity, aex_stream stream) {
  using namespace aex;
  if (!d || !latents || !velocity) return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  if ((reinterpret_cast<uintptr_t>(latents) | reinterpret_cast<uintptr_t>(velocity)) & 3)
    return set_error(d->ctx, AEX_ERR_INVALID_ARG, "latents and velocity must be 4-byte aligned f32 arrays");
  if (int r = bind_device(d->ctx)) return r;
  return forward(d, latents, velocity, static_cast<cudaStream_t>(stream));
}

int aex_dit_denoise_step(aex_dit* d, const float* lat_in, float* lat_out, float dt, aex_stream stream) {
  using namespace aex;
  if (!d || !lat_in || !lat_out) return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  if ((reinterpret_cast<uintptr_t>(lat_in) | reinterpret_cast<uintptr_t>(lat_out)) & 3)
    return set_error(d->ctx, AEX_ERR_INVALID_ARG, "latents must be 4-byte aligned f32 arrays");
  if (int r = bind_device(d->ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  AEX_TRY(glue::set_scalar(d->ctx, d->CUR + 1, dt, s));
  AEX_TRY(forward(d, lat_in, d->PRED, s));
  return glue::euler(d->ctx, lat_in, d->PRED, d->CUR + 1, static_cast<int64_t>(d->cfg.l_img) * d->cfg.in_channels,
                     lat_out, s);
}

int aex_dit_denoise(aex_dit* d, float* latents, int steps, aex_stream stream) {
  using namespace aex;
  if (!d || !latents || steps < 1 || steps > kMaxGraphSteps)
    return set_error(d ? d->ctx : nullptr, AEX_ERR_INVALID_ARG, "bad argument (steps in 1..%d)", kMaxGraphSteps);
  if (!d->rope_set || !d->context_set)
    return set_error(d->ctx, AEX_ERR_INVALID_ARG, "set rope and context before denoise");
  if (int r = bind_device(d->ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  std::vector<float> sig, ts;
  schedule(steps, d->l_img_sched, sig, ts);
  std::vector<float> sc(2 * static_cast<size_t>(steps));
  for (int i = 0; i < steps; ++i) {
    sc[2 * i] = ts[i];
    sc[2 * i + 1] = sig[i + 1] - sig[i];
  }
  const size_t lat_bytes = static_cast<size_t>(d->cfg.l_img) * d->cfg.in_channels * sizeof(float);
  // Pageable source: the copy is staged before cudaMemcpyAsync returns, so `sc` may go out of scope.
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->STEPS, sc.data(), sc.size() * sizeof(float), cudaMemcpyHostToDevice, s));
  AEX_CUDA_TRY(d->ctx, cudaMemsetAsync(d->STEP_I, 0, sizeof(int), s));
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->LATB, latents, lat_bytes, cudaMemcpyDeviceToDevice, s));
  AEX_TRY(prepare_weights(d, s));
  d->timestep_set = true;  // the replayed step sets it from STEPS
  if (d->comm) {
    // Sequence-parallel steps exchange K/V over NCCL on a side stream: launched step by step.
    for (int i = 0; i < steps; ++i) AEX_TRY(graph_step(d, s));
  } else {
    if (!d->step_graph) AEX_TRY(capture_step(d));
    for (int i = 0; i < steps; ++i) AEX_CUDA_TRY(d->ctx, cudaGraphLaunch(d->step_graph, s));
  }
  AEX_CUDA_TRY(d->ctx, cudaMemcpyAsync(latents, d->LATB, lat_bytes, cudaMemcpyDeviceToDevice, s));
  return AEX_OK;
}

int aex_dit_set_sequence_parallel(aex_dit* d, aex_comm* comm, int l_txt_total, int l_img_total) {
  using namespace aex;
  if (!d) return set_error(nullptr, AEX_ERR_INVALID_ARG, "NULL dit");
  drop_graph(d);
  if (!comm) {
    d->comm = nullptr;
    d->l_img_sched = d->cfg.l_img;
    return AEX_OK;
  }
  const int P = comm_world(comm), r = comm_rank(comm);
  const int64_t J_total = static_cast<int64_t>(l_txt_total) + l_img_total;
  if (l_txt_total < 0 || l_img_total <= 0 || J_total % P || J_total / P != d->J)
    return set_error(d->ctx, AEX_ERR_INVALID_ARG,
                     "sequence shards must be equal: %lld joint rows over %d ranks, this engine holds %d",
                     static_cast<long long>(J_total), P, d->J);
  if ((r == 0 && d->cfg.l_txt != l_txt_total) || (r > 0 && d->cfg.l_txt != 0))
    return set_error(d->ctx, AEX_ERR_INVALID_ARG,
                     "the text rows (%d) must all be on rank 0: this rank (%d) holds %d", l_txt_total, r,
                     d->cfg.l_txt);
  d->comm = comm;
  d->l_img_sched = l_img_total;
  return AEX_OK;
}

}  // extern "C"
