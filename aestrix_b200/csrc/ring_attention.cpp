// ring_attention.cpp — sequence-parallel joint attention over P GPUs (one
// process per GPU) for long sequences (2048^2: 512 text + 16384 image tokens).
//
// The reference keeps the full sequence on one device (ParallelSelfAttention
// runs one SDPA over full-length Q/K/V, Sources/ImarelloDiT/ParallelSelfAttention.swift:
// 134-136); this is the multi-GPU form of the same computation. The joint
// sequence is split into P equal contiguous shards (rank r holds tokens
// [r*S_r, (r+1)*S_r), text rows in shard 0). Each rank RMS-normalizes and
// rotates its own Q and K rows (RoPE uses absolute positions, so rotating
// before the exchange is exact). Three schedules, the same on every rank:
//  * overlap: P - 1 pairwise NCCL groups on a high-priority stream; each
//    shard's attention starts as soon as it has landed (the local one at
//    once), one partial per shard, merged by log-sum-exp at the end;
//  * ring: for hop h = 0..P-1 attend the local queries to the K/V shard of rank
//    (r - h) mod P while the next shard travels around the ring (ncclSend to
//    r+1 / ncclRecv from r-1 on a dedicated stream, double buffered); partial
//    outputs merged by their log-sum-exp (ring_kernels.cu);
//  * gather: one ncclAllGather of every rank's K and V (token-major, in place)
//    and one attention call of the local queries over all P*S keys (its keys
//    split into ranges merged by log-sum-exp when a short shard's CTAs would
//    underfill the SMs' waves).
//
// NCCL is resolved at run time (the copy already loaded in the process, else
// libnccl.so.2), so the library has no link-time NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "internal.h"

namespace aex {
namespace ring {
int merge(aex_ctx* ctx, const void* o_h, int64_t oh_ss, int64_t oh_sh, const float* lse_h, const float* lse_in,
          float* lse_out, float* o_acc, int S, int H, bool first, bool final, void* out, int64_t out_ss, int64_t out_sh,
          cudaStream_t s);
}

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) commInitRankConfig = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclCommGetAsyncError) commGetAsyncError = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  decltype(&ncclGroupStart) groupStart = nullptr;
  decltype(&ncclGroupEnd) groupEnd = nullptr;
  decltype(&ncclGetErrorString) errorString = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen(nullptr, RTLD_NOW);  // prefer a copy already in the process (e.g. torch's)
    if (!h || !dlsym(h, "ncclGetUniqueId")) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](auto& f, const char* name) { f = reinterpret_cast<std::remove_reference_t<decltype(f)>>(dlsym(h, name)); };
    sym(api.getUniqueId, "ncclGetUniqueId");
    sym(api.commInitRankConfig, "ncclCommInitRankConfig");
    sym(api.commDestroy, "ncclCommDestroy");
    sym(api.commAbort, "ncclCommAbort");
    sym(api.commGetAsyncError, "ncclCommGetAsyncError");
    sym(api.send, "ncclSend");
    sym(api.recv, "ncclRecv");
    sym(api.allGather, "ncclAllGather");
    sym(api.groupStart, "ncclGroupStart");
    sym(api.groupEnd, "ncclGroupEnd");
    sym(api.errorString, "ncclGetErrorString");
    api.ok = api.getUniqueId && api.commInitRankConfig && api.commDestroy && api.commAbort && api.commGetAsyncError &&
             api.send && api.recv && api.allGather && api.groupStart && api.groupEnd && api.errorString;
  });
  return api;
}

int nccl_error(aex_ctx* ctx, ncclResult_t r, const char* what) {
  return set_error(ctx, AEX_ERR_NCCL, "%s failed: %s", what, nccl().errorString ? nccl().errorString(r) : "?");
}

// ncclGroupEnd on a non-blocking communicator: wait (bounded) until the group
// is enqueued on its stream.
int group_end(aex_ctx* ctx, ncclComm_t comm, ncclResult_t issued, const char* what) {
  ncclResult_t ne = nccl().groupEnd();
  if (issued != ncclSuccess && issued != ncclInProgress) return nccl_error(ctx, issued, what);
  const auto t0 = std::chrono::steady_clock::now();
  while (ne == ncclInProgress) {
    ncclResult_t st = ncclInProgress;
    const ncclResult_t q = nccl().commGetAsyncError(comm, &st);
    if (q != ncclSuccess) return nccl_error(ctx, q, "ncclCommGetAsyncError");
    ne = st;
    if (ne == ncclInProgress && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(30))
      return set_error(ctx, AEX_ERR_TIMEOUT, "NCCL group not enqueued after 30 s");
  }
  if (ne != ncclSuccess) return nccl_error(ctx, ne, "ncclGroupEnd");
  return AEX_OK;
}

// Schedule of the sequence-parallel attention, the same on every rank (it
// depends only on the shapes, equal on all ranks):
//  * overlap (default for P > 1 while the gathered K and V fit in
//    kGatherMaxBytes): the K/V exchange as P - 1 pairwise NCCL groups on a
//    high-priority stream, the attention over each shard launched as soon as
//    that shard has landed (the local shard at once), partials merged by
//    log-sum-exp;
//  * gather (default at P = 1): one grouped all-gather of K/V, then one
//    attention call over all keys (measured faster than the ring at every P
//    tried: 2048^2, P = 2: 1.74 vs 1.81 ms per call; P = 8: 0.747 vs 2.78 ms);
//  * ring (when the gathered K/V would not fit): K/V passed to rank r + 1 per
//    hop, memory per rank O(S).
// AEX_SP_SCHEDULE=overlap|gather|ring overrides.
constexpr size_t kGatherMaxBytes = size_t{8} << 30;
constexpr int kMaxOverlapRanks = 16;  // partials merged in one pass (merge_splits)
enum Schedule : int { kRing = 0, kGather = 1, kOverlap = 2 };

int schedule_for(int P, size_t plane_bytes) {
  static const int forced = [] {
    const char* e = getenv("AEX_SP_SCHEDULE");
    if (!e) return -1;
    return !strcmp(e, "overlap") ? static_cast<int>(kOverlap)
           : !strcmp(e, "gather") ? static_cast<int>(kGather)
           : !strcmp(e, "ring")   ? static_cast<int>(kRing)
                                  : -1;
  }();
  if (forced == kRing || forced == kGather) return forced;
  if (forced == kOverlap && P <= kMaxOverlapRanks) return kOverlap;
  if (2 * static_cast<size_t>(P) * plane_bytes > kGatherMaxBytes) return kRing;
  // Overlap only at two ranks: there it hides the larger exchange (1.59 vs 1.72 ms per 2048^2 call on B200);
  // at four ranks one all-gather and one attention over all keys win (1.07 vs 1.58 ms: the per-shard launches
  // repeat the partial last wave and add a merge, while the smaller exchange has little left to hide).
  return P == 2 ? kOverlap : kGather;
}

}  // namespace
}  // namespace aex

struct aex_comm {
  aex_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;
  int world = 0, rank = 0;
  cudaStream_t stream = nullptr;  // exchange stream (highest priority: its copies take SMs as they free up)
  cudaStream_t side = nullptr;    // second compute stream of the overlap schedule
  cudaEvent_t ev_attn[2] = {nullptr, nullptr}, ev_recv = nullptr, ev_start = nullptr, ev_side = nullptr;
  cudaEvent_t ev_piece[aex::kMaxOverlapRanks] = {};  // overlap schedule: exchange group h has landed
  // exchange state (ring or gather layout), grown on demand
  void* buf = nullptr;
  size_t buf_bytes = 0;
};

namespace aex {
namespace {

int grow(aex_comm* c, size_t bytes) {
  if (c->buf_bytes >= bytes) return AEX_OK;
  if (c->buf) {
    AEX_CUDA_TRY(c->ctx, cudaDeviceSynchronize());
    cudaFree(c->buf);
    c->buf = nullptr;
    c->buf_bytes = 0;
  }
  AEX_CUDA_TRY(c->ctx, cudaMalloc(&c->buf, bytes));
  c->buf_bytes = bytes;
  return AEX_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace
}  // namespace aex

namespace aex {

int comm_world(const aex_comm* c) { return c->world; }
int comm_rank(const aex_comm* c) { return c->rank; }

// Ring layout: Q plane | K ring[2] (head-major) | V ring[2] (token-major) | O_h bf16 | O_acc f32 | lse_h |
// lse ping-pong[2]; this rank's Q and K are prepared into the Q plane and K ring[0].
// Gather layout: Q plane (head-major) | K all ranks [P*S][H][128] | V all ranks [P*S][H][128] (token-major;
// this rank's rows at r*S) | with k > 1 key ranges (gather_splits): partial outputs [k][S][H][128] bf16 and
// their log-sum-exp [k][H][S] f32.
// Key ranges of the gather schedule's attention call: the local queries (S rows, H heads) over all P*S keys
// make ceil(S/256)*H CTAs, too few to fill the SMs' waves at short shards (2048^2 at P = 8: 216 CTAs, 1.46
// waves); splitting the keys fills them (432 CTAs, 2.92 waves) at the cost of one merge pass.
int key_ranges(int P, int S, int H, int sms) {
  const int ctas = (S + 255) / 256 * H;
  const int n_kv = (P * S + 127) / 128;
  return attention_kv_splits(ctas, n_kv, sms);
}

int gather_splits(const aex_ctx* ctx, int P, int S, int H) { return key_ranges(P, S, H, ctx->sm_count); }

// The overlap schedule's plan for `rank` of `world` (host logic shared by the CUDA path and the
// CPU tests): the local shard's attention first (no exchange), then the P - 1 pairwise exchange
// groups (group h: this rank's K/V to rank r + h, rank r - h's K/V into its slot; a permutation,
// so the groups pair up on every rank in the same order), then per landed shard one attention
// into its own partial (alternating two compute streams), then one merge of the P partials.
int overlap_plan(int P, int r, aex_sp_op* ops, int max_ops) {
  if (P < 1 || r < 0 || r >= P || P > kMaxOverlapRanks) return -1;
  const int n = 1 + 2 * (P - 1) + 1;
  if (!ops) return n;
  if (max_ops < n) return -1;
  int i = 0;
  ops[i++] = aex_sp_op{AEX_SP_OP_ATTEND, -1, -1, r, 0, -1, 0};
  for (int h = 1; h < P; ++h) ops[i++] = aex_sp_op{AEX_SP_OP_EXCHANGE, (r + h) % P, (r - h + P) % P, -1, h, -1, -1};
  for (int h = 1; h < P; ++h) ops[i++] = aex_sp_op{AEX_SP_OP_ATTEND, -1, -1, (r - h + P) % P, h, h, h & 1};
  ops[i++] = aex_sp_op{AEX_SP_OP_MERGE, -1, -1, -1, P, -1, 0};
  return i;
}

int sp_buffers(aex_ctx* ctx, aex_comm* c, int S, int H, SpSlots* out) {
  if (!c->comm) return set_error(ctx, AEX_ERR_NCCL, "communicator aborted");
  const int P = c->world, r = c->rank;
  const size_t plane = static_cast<size_t>(H) * S * 128;
  if (align256(plane * 2) != plane * 2) return set_error(ctx, AEX_ERR_INVALID_ARG, "shard size must keep 256-byte alignment");
  uint8_t* base;
  const int sched = schedule_for(P, plane * 2);
  if (sched != kRing) {
    // gather / overlap layout; the overlap schedule keeps one partial per shard
    const size_t k = sched == kOverlap ? static_cast<size_t>(P) : static_cast<size_t>(gather_splits(ctx, P, S, H));
    const size_t parts = k > 1 ? k * plane * 2 + align256(k * H * static_cast<size_t>(S) * 4) : 0;
    if (int e = grow(c, plane * 2 * (1 + 2 * static_cast<size_t>(P)) + parts)) return e;
    base = static_cast<uint8_t*>(c->buf);
    out->q = reinterpret_cast<uint16_t*>(base);
    out->k = reinterpret_cast<uint16_t*>(base + plane * 2) + r * plane;
    out->k_token_major = true;
    out->v = reinterpret_cast<uint16_t*>(base + plane * 2 * (1 + static_cast<size_t>(P))) + r * plane;
    return AEX_OK;
  }
  const size_t bq = plane * 2, bkv = plane * 2, bo = plane * 2, bacc = plane * 4,
               blse = align256(static_cast<size_t>(H) * S * 4);
  const size_t off_k = bq, off_v = off_k + 2 * bkv, off_o = off_v + 2 * bkv, off_acc = off_o + bo,
               off_lh = off_acc + bacc, off_l0 = off_lh + blse, total = off_l0 + 2 * blse;
  if (int e = grow(c, total)) return e;
  base = static_cast<uint8_t*>(c->buf);
  out->q = reinterpret_cast<uint16_t*>(base);
  out->k = reinterpret_cast<uint16_t*>(base + off_k);
  out->k_token_major = false;
  out->v = reinterpret_cast<uint16_t*>(base + off_v);
  return AEX_OK;
}

namespace {

int ring_run(aex_ctx* ctx, aex_comm* c, int S, int H, float scale, void* out, int64_t out_ss, int64_t out_sh,
             cudaStream_t s) {
  const int P = c->world, r = c->rank;
  const size_t plane = static_cast<size_t>(H) * S * 128;  // elements of one [H][S][128] or [S][H][128] block
  const size_t bq = align256(plane * 2), bkv = align256(plane * 2), bo = align256(plane * 2),
               bacc = align256(plane * 4), blse = align256(static_cast<size_t>(H) * S * 4);
  const size_t off_q = 0, off_k = bq, off_v = off_k + 2 * bkv, off_o = off_v + 2 * bkv, off_acc = off_o + bo,
               off_lh = off_acc + bacc, off_l0 = off_lh + blse;
  uint8_t* base = static_cast<uint8_t*>(c->buf);
  uint16_t* Q = reinterpret_cast<uint16_t*>(base + off_q);
  uint16_t* Kr[2] = {reinterpret_cast<uint16_t*>(base + off_k), reinterpret_cast<uint16_t*>(base + off_k + bkv)};
  uint16_t* Vr[2] = {reinterpret_cast<uint16_t*>(base + off_v), reinterpret_cast<uint16_t*>(base + off_v + bkv)};
  uint16_t* Oh = reinterpret_cast<uint16_t*>(base + off_o);
  float* Oacc = reinterpret_cast<float*>(base + off_acc);
  float* lse_h = reinterpret_cast<float*>(base + off_lh);
  float* lse_acc[2] = {reinterpret_cast<float*>(base + off_l0), reinterpret_cast<float*>(base + off_l0 + blse)};
  AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_start, s));
  AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(c->stream, c->ev_start, 0));
  const int64_t q_st[3] = {static_cast<int64_t>(plane), 128, static_cast<int64_t>(S) * 128};   // head-major
  const int64_t v_st[3] = {static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128, 128};  // token-major
  const int64_t o_st[3] = {static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128, 128};
  const size_t kv_bytes = plane * 2;
  const int next = (r + 1) % P, prev = (r - 1 + P) % P;
  for (int hop = 0; hop < P; ++hop) {
    const int cur = hop & 1, nxt = cur ^ 1;
    if (hop + 1 < P) {
      // Exchange on the ring stream: send the shard in hand, receive the next one.
      if (hop > 0) AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(c->stream, c->ev_attn[nxt], 0));  // nxt no longer read
      ncclResult_t nr = nccl().groupStart();
      if (nr == ncclSuccess) nr = nccl().send(Kr[cur], kv_bytes, ncclChar, next, c->comm, c->stream);
      if (nr == ncclSuccess) nr = nccl().send(Vr[cur], kv_bytes, ncclChar, next, c->comm, c->stream);
      if (nr == ncclSuccess) nr = nccl().recv(Kr[nxt], kv_bytes, ncclChar, prev, c->comm, c->stream);
      if (nr == ncclSuccess) nr = nccl().recv(Vr[nxt], kv_bytes, ncclChar, prev, c->comm, c->stream);
      if (int e = group_end(ctx, c->comm, nr, "ncclSend/ncclRecv")) return e;
      AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_recv, c->stream));
    }
    // Attention of the local queries against the shard in hand, then merge.
    if (int e = launch_attention_core(ctx, Q, q_st, Kr[cur], q_st, Vr[cur], v_st, Oh, o_st, 1, S, S, H, scale,
                                      lse_h, 0, S, s))
      return e;
    AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_attn[cur], s));
    if (int e = ring::merge(ctx, Oh, static_cast<int64_t>(H) * 128, 128, lse_h, lse_acc[hop & 1],
                            lse_acc[(hop + 1) & 1], Oacc, S, H, hop == 0, hop == P - 1, out, out_ss, out_sh, s))
      return e;
    if (hop + 1 < P) AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(s, c->ev_recv, 0));
  }
  return AEX_OK;
}


// K/V of every rank gathered in place (one grouped ncclAllGather on the exchange stream), then one attention
// call of the local queries over all P*S keys.
int gather_run(aex_ctx* ctx, aex_comm* c, int S, int H, float scale, void* out, int64_t out_ss, int64_t out_sh,
               cudaStream_t s) {
  const int P = c->world;
  const size_t plane = static_cast<size_t>(H) * S * 128;
  uint8_t* base = static_cast<uint8_t*>(c->buf);
  uint16_t* Q = reinterpret_cast<uint16_t*>(base);
  uint16_t* Kall = reinterpret_cast<uint16_t*>(base + plane * 2);
  uint16_t* Vall = reinterpret_cast<uint16_t*>(base + plane * 2 * (1 + static_cast<size_t>(P)));
  AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_start, s));
  AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(c->stream, c->ev_start, 0));
  const size_t bytes = plane * 2;
  ncclResult_t nr = nccl().groupStart();
  if (nr == ncclSuccess)
    nr = nccl().allGather(reinterpret_cast<uint8_t*>(Kall) + c->rank * bytes, Kall, bytes, ncclChar, c->comm,
                          c->stream);
  if (nr == ncclSuccess)
    nr = nccl().allGather(reinterpret_cast<uint8_t*>(Vall) + c->rank * bytes, Vall, bytes, ncclChar, c->comm,
                          c->stream);
  if (int e = group_end(ctx, c->comm, nr, "ncclAllGather")) return e;
  AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_recv, c->stream));
  AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(s, c->ev_recv, 0));
  const int64_t q_st[3] = {static_cast<int64_t>(plane), 128, static_cast<int64_t>(S) * 128};  // head-major
  const int64_t kv_st[3] = {static_cast<int64_t>(P) * static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128,
                            128};  // token-major over all ranks
  const int k = gather_splits(ctx, P, S, H);
  if (k == 1) {
    const int64_t o_st[3] = {static_cast<int64_t>(S) * out_ss, out_ss, out_sh};
    return launch_attention_core(ctx, Q, q_st, Kall, kv_st, Vall, kv_st, out, o_st, 1, S, P * S, H, scale, nullptr,
                                 0, 0, s);
  }
  // k key ranges in parallel CTAs, each to its own normalized partial, then one merge.
  uint16_t* parts = reinterpret_cast<uint16_t*>(base + plane * 2 * (1 + 2 * static_cast<size_t>(P)));
  float* lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(parts) + static_cast<size_t>(k) * plane * 2);
  const int64_t p_st[3] = {static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128, 128};  // token-major
  if (int e = launch_attention_core(ctx, Q, q_st, Kall, kv_st, Vall, kv_st, parts, p_st, 1, S, P * S, H, scale, lse,
                                    static_cast<int64_t>(H) * S, S, s, k))
    return e;
  return ring::merge_splits(ctx, parts, static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128, 128, lse,
                            static_cast<int64_t>(H) * S, k, S, H, out, out_ss, out_sh, s);
}

// The overlap schedule (gather layout with P partials): runs overlap_plan. Exchange groups go to the
// high-priority exchange stream, each recording ev_piece[h] once its shard has landed; an attention over
// shard h waits for that event on its compute stream (the caller's stream or the side stream), so it starts
// while later shards are still in flight and the two streams' launches fill each other's tail waves.
int overlap_run(aex_ctx* ctx, aex_comm* c, int S, int H, float scale, void* out, int64_t out_ss, int64_t out_sh,
                cudaStream_t s) {
  const int P = c->world, r = c->rank;
  const size_t plane = static_cast<size_t>(H) * S * 128;
  uint8_t* base = static_cast<uint8_t*>(c->buf);
  uint16_t* Q = reinterpret_cast<uint16_t*>(base);
  uint16_t* Kall = reinterpret_cast<uint16_t*>(base + plane * 2);
  uint16_t* Vall = reinterpret_cast<uint16_t*>(base + plane * 2 * (1 + static_cast<size_t>(P)));
  uint16_t* parts = reinterpret_cast<uint16_t*>(base + plane * 2 * (1 + 2 * static_cast<size_t>(P)));
  float* lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(parts) + static_cast<size_t>(P) * plane * 2);
  aex_sp_op ops[2 * kMaxOverlapRanks + 2];
  const int n_ops = overlap_plan(P, r, ops, 2 * kMaxOverlapRanks + 2);
  if (n_ops < 0) return set_error(ctx, AEX_ERR_UNSUPPORTED, "overlap schedule: %d ranks", P);
  // Q, K, V of this rank were written on s: the exchange and the side stream start after them.
  AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_start, s));
  AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(c->stream, c->ev_start, 0));
  AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(c->side, c->ev_start, 0));
  const size_t bytes = plane * 2;
  const int64_t q_st[3] = {static_cast<int64_t>(plane), 128, static_cast<int64_t>(S) * 128};  // head-major
  const int64_t kv_st[3] = {static_cast<int64_t>(P) * static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128,
                            128};  // token-major slot of one rank
  const int64_t p_st[3] = {static_cast<int64_t>(plane), static_cast<int64_t>(H) * 128, 128};
  for (int i = 0; i < n_ops; ++i) {
    const aex_sp_op& op = ops[i];
    if (op.kind == AEX_SP_OP_EXCHANGE) {
      ncclResult_t nr = nccl().groupStart();
      if (nr == ncclSuccess)
        nr = nccl().send(reinterpret_cast<uint8_t*>(Kall) + r * bytes, bytes, ncclChar, op.send_to, c->comm, c->stream);
      if (nr == ncclSuccess)
        nr = nccl().send(reinterpret_cast<uint8_t*>(Vall) + r * bytes, bytes, ncclChar, op.send_to, c->comm, c->stream);
      if (nr == ncclSuccess)
        nr = nccl().recv(reinterpret_cast<uint8_t*>(Kall) + op.recv_from * bytes, bytes, ncclChar, op.recv_from,
                         c->comm, c->stream);
      if (nr == ncclSuccess)
        nr = nccl().recv(reinterpret_cast<uint8_t*>(Vall) + op.recv_from * bytes, bytes, ncclChar, op.recv_from,
                         c->comm, c->stream);
      if (int e = group_end(ctx, c->comm, nr, "ncclSend/ncclRecv (overlap)")) return e;
      AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_piece[op.part], c->stream));
    } else if (op.kind == AEX_SP_OP_ATTEND) {
      cudaStream_t t = op.stream ? c->side : s;
      if (op.wait_exchange >= 0) AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(t, c->ev_piece[op.wait_exchange], 0));
      if (int e = launch_attention_core(ctx, Q, q_st, Kall + op.slot * plane, kv_st, Vall + op.slot * plane, kv_st,
                                        parts + op.part * plane, p_st, 1, S, S, H, scale,
                                        lse + static_cast<size_t>(op.part) * H * S, 0, S, t))
        return e;
    } else {
      AEX_CUDA_TRY(ctx, cudaEventRecord(c->ev_side, c->side));
      AEX_CUDA_TRY(ctx, cudaStreamWaitEvent(s, c->ev_side, 0));
      if (int e = ring::merge_splits(ctx, parts, static_cast<int64_t>(plane), p_st[1], p_st[2], lse,
                                     static_cast<int64_t>(H) * S, op.part, S, H, out, out_ss, out_sh, s))
        return e;
    }
  }
  return AEX_OK;
}

}  // namespace

int sp_run(aex_ctx* ctx, aex_comm* c, int S, int H, float scale, void* out, int64_t out_ss, int64_t out_sh,
           cudaStream_t s) {
  if (!c->comm) return set_error(ctx, AEX_ERR_NCCL, "communicator aborted");
  switch (schedule_for(c->world, static_cast<size_t>(H) * S * 256)) {
    case kOverlap:
      return overlap_run(ctx, c, S, H, scale, out, out_ss, out_sh, s);
    case kGather:
      return gather_run(ctx, c, S, H, scale, out, out_ss, out_sh, s);
    default:
      return ring_run(ctx, c, S, H, scale, out, out_ss, out_sh, s);
  }
}


}  // namespace aex

extern "C" {

int aex_comm_unique_id(void* id_out) {
  using namespace aex;
  if (!id_out) return set_error(nullptr, AEX_ERR_INVALID_ARG, "NULL id");
  if (!nccl().ok) return set_error(nullptr, AEX_ERR_NCCL, "NCCL library not found (libnccl.so.2)");
  ncclUniqueId id;
  ncclResult_t r = nccl().getUniqueId(&id);
  if (r != ncclSuccess) return nccl_error(nullptr, r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == AEX_COMM_ID_BYTES, "unique id size");
  std::memcpy(id_out, &id, sizeof id);
  return AEX_OK;
}

int aex_comm_create(aex_ctx* ctx, int world, int rank, const void* id, int timeout_ms, aex_comm** out) {
  using namespace aex;
  if (!ctx || !id || !out) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return set_error(ctx, AEX_ERR_INVALID_ARG, "bad world/rank");
  if (!nccl().ok) return set_error(ctx, AEX_ERR_NCCL, "NCCL library not found (libnccl.so.2)");
  if (int r = bind_device(ctx)) return r;
  auto* c = new aex_comm();
  c->ctx = ctx;
  c->world = world;
  c->rank = rank;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof uid);
  // Non-blocking init, polled with a deadline, so a missing peer cannot hang the caller.
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = nccl().commInitRankConfig(&c->comm, world, uid, rank, &cfg);
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  while (r == ncclSuccess || r == ncclInProgress) {
    r = nccl().commGetAsyncError(c->comm, &st);
    if (r != ncclSuccess || st != ncclInProgress) break;
    if (timeout_ms > 0 && std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      nccl().commAbort(c->comm);
      delete c;
      return set_error(ctx, AEX_ERR_TIMEOUT, "NCCL communicator init did not complete in %d ms", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess || st != ncclSuccess) {
    if (c->comm) nccl().commAbort(c->comm);
    delete c;
    return nccl_error(ctx, r != ncclSuccess ? r : st, "ncclCommInitRankConfig");
  }
  // The exchange stream at the highest priority: its copy kernels take SMs as attention CTAs retire.
  int least = 0, greatest = 0;
  cudaError_t e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&c->stream, cudaStreamNonBlocking, greatest);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&c->ev_attn[i], cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_recv, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_side, cudaEventDisableTiming);
  for (int i = 0; i < std::min(world, static_cast<int>(kMaxOverlapRanks)) && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&c->ev_piece[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    aex_comm_destroy(c);
    return cuda_error(ctx, e, "stream/event creation");
  }
  *out = c;
  return AEX_OK;
}

void aex_comm_destroy(aex_comm* c) {
  using namespace aex;
  if (!c) return;
  cudaSetDevice(c->ctx->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->side) cudaStreamSynchronize(c->side);
  if (c->comm) nccl().commDestroy(c->comm);
  for (auto* ev : {c->ev_attn[0], c->ev_attn[1], c->ev_recv, c->ev_start, c->ev_side})
    if (ev) cudaEventDestroy(ev);
  for (auto* ev : c->ev_piece)
    if (ev) cudaEventDestroy(ev);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->side) cudaStreamDestroy(c->side);
  if (c->buf) cudaFree(c->buf);
  delete c;
}

int aex_comm_abort(aex_comm* c) {
  using namespace aex;
  if (!c || !c->comm) return AEX_ERR_INVALID_ARG;
  ncclResult_t r = nccl().commAbort(c->comm);
  c->comm = nullptr;
  return r == ncclSuccess ? AEX_OK : AEX_ERR_NCCL;
}

int aex_sp_key_ranges(int world, int seq, int heads, int sms) {
  if (world < 1 || seq <= 0 || heads <= 0 || sms <= 0) return -1;
  return aex::key_ranges(world, seq, heads, sms);
}

int aex_sp_schedule(int world, int seq, int heads) {
  if (world < 1 || seq <= 0 || heads <= 0) return -1;
  return aex::schedule_for(world, static_cast<size_t>(heads) * seq * 256);
}

int aex_sp_plan(int world, int rank, aex_sp_op* ops, int max_ops) { return aex::overlap_plan(world, rank, ops, max_ops); }

int aex_ring_attention(aex_ctx* ctx, aex_comm* c, const aex_attention_args* a, aex_stream stream) {
  using namespace aex;
  if (!ctx || !c || !a) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  if (!c->comm) return set_error(ctx, AEX_ERR_NCCL, "communicator aborted");
  if (int r = validate_attention_args(ctx, a)) return r;
  if (a->batch != 1) return set_error(ctx, AEX_ERR_UNSUPPORTED, "ring attention takes batch 1");
  if (a->v.stride_h != 128) return set_error(ctx, AEX_ERR_UNSUPPORTED, "ring attention needs V heads contiguous");
  if (int r = bind_device(ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  const int S = a->seq, H = a->heads;
  SpSlots sl{};
  if (int e = sp_buffers(ctx, c, S, H, &sl)) return e;
  // 1. This rank's Q and K: norm + RoPE (rows of the local shard, absolute positions) into their slots.
  const int64_t qs[3] = {a->q.stride_b, a->q.stride_s, a->q.stride_h};
  const int64_t ks[3] = {a->k.stride_b, a->k.stride_s, a->k.stride_h};
  if (int e = launch_qk_prep(ctx, a->q.data, qs, a->k.data, ks, 1, S, H, a->norm_q_weight, a->norm_k_weight, nullptr,
                             nullptr, 0, a->eps, a->rope_cos, a->rope_sin, sl.q, s, sl.k, sl.k_token_major))
    return e;
  // 2. This rank's V into its slot (token-major, contiguous rows of H*128).
  AEX_CUDA_TRY(ctx, cudaMemcpy2DAsync(sl.v, static_cast<size_t>(H) * 256, a->v.data,
                                      static_cast<size_t>(a->v.stride_s) * 2, static_cast<size_t>(H) * 256, S,
                                      cudaMemcpyDeviceToDevice, s));
  return sp_run(ctx, c, S, H, a->scale, a->out.data, a->out.stride_s, a->out.stride_h, s);
}

}  // extern "C"
