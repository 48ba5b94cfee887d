/*
 * aestrix_cuda.h — C ABI of libaestrix_cuda, the B200 (sm_100a) implementation of
 * the FLUX.2-klein DiT joint attention and the MLX-layout 4-bit affine linears
 * that feed it.
 *
 * Conventions
 *  - Every entry point returns an int status (AEX_OK == 0). On failure the
 *    context's message is available from aex_last_error_string(ctx). No entry
 *    point aborts, traps or exits the process.
 *  - Device pointers are plain `void*`/typed pointers into CUDA global memory of
 *    the context's device. `aex_stream` is a cudaStream_t (NULL = legacy
 *    default stream). All compute entry points are asynchronous on that stream.
 *  - bf16 data is passed as uint16_t bit patterns (or void*), f32 as float.
 *  - One aex_ctx per device per host thread; distinct contexts may be used
 *    concurrently, a single context may not.
 *  - Kernels never spin without bound: a device-side wait that expires records
 *    a code that aex_sync / aex_device_status report as AEX_ERR_DEVICE.
 *
 * Each declaration cites the reference (PowerBeef/Aestrix, "Imarello") interface
 * it replaces as path:line within that project.
 */
#ifndef AESTRIX_CUDA_H
#define AESTRIX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AEX_ABI_VERSION 1

/* Status codes. Reference: Swift `throws` of DirectQmmSpike.SpikeError
 * (Sources/ImarelloDirect/DirectQmmSpike.swift:17-27) and the command-buffer
 * error check (Sources/ImarelloDirect/DirectDiTStep.swift:968-970). */
#define AEX_OK 0
#define AEX_ERR_INVALID_ARG 1 /* bad shape, stride, alignment or NULL pointer; nothing launched */
#define AEX_ERR_UNSUPPORTED 2 /* valid but not implemented (e.g. head_dim != 128) */
#define AEX_ERR_CUDA 3        /* a CUDA runtime/driver call failed */
#define AEX_ERR_NCCL 4        /* an NCCL call failed */
#define AEX_ERR_TIMEOUT 5     /* aex_sync gave up waiting */
#define AEX_ERR_OOM 6         /* device allocation failed */
#define AEX_ERR_DEVICE 7      /* a kernel reported a device-side status (bounded wait expired) */

typedef struct aex_ctx aex_ctx;
typedef struct aex_qweight aex_qweight;
typedef void* aex_stream; /* cudaStream_t */

/* ------------------------------------------------------------------ context */

int aex_abi_version(void);

/* Create a context bound to CUDA device `device`. Reference: the engine
 * constructors that own a device and queue, DirectDiTStep.init
 * (Sources/ImarelloDirect/DirectDiTStep.swift:74-132). */
int aex_ctx_create(int device, aex_ctx** out);
void aex_ctx_destroy(aex_ctx* ctx);

/* Last error message of this context ("" if none). Valid until the next call
 * on the same context. NULL ctx returns the message of the last failed
 * aex_ctx_create on this thread. */
const char* aex_last_error_string(const aex_ctx* ctx);

/* Wait for `stream` with a bound. timeout_ms <= 0 waits without a bound on the
 * host side (kernels themselves still never spin forever). Returns
 * AEX_ERR_TIMEOUT if the stream is still busy at the deadline, AEX_ERR_DEVICE
 * if a kernel recorded a device-side status. Reference: the blocking
 * `waitUntilCompleted` + error check at DirectDiTStep.swift:968-970. */
int aex_sync(aex_ctx* ctx, aex_stream stream, int timeout_ms);

/* Read (and clear) the device status word the kernels write on a bounded-wait
 * expiry. *code receives 0 when no kernel reported anything. Synchronizes the
 * device. */
int aex_device_status(aex_ctx* ctx, int* code);

/* Number of SMs of the context's device. */
int aex_device_sm_count(const aex_ctx* ctx);

/* -------------------------------------------------------------- attention */

/* Strided 4-D view [batch, seq, head, dim] of a bf16 tensor; the dim stride is
 * 1. [B,H,S,D] tensors of the MLX path use (H*S*D, D, S*D); the direct
 * engine's [J, 24, 128] rows use (J*3072, 3072, 128). All strides in elements,
 * each a multiple of 8 (16 bytes), base pointer 16-byte aligned. */
typedef struct aex_bshd {
  void* data;
  int64_t stride_b;
  int64_t stride_s;
  int64_t stride_h;
} aex_bshd;

typedef struct aex_attention_args {
  aex_bshd q, k, v; /* bf16 inputs (pre-norm, pre-RoPE when the norm/rope fields are set) */
  aex_bshd out;     /* bf16 output; may alias nothing else */
  int batch;
  int seq;          /* joint length J = text rows then image rows */
  int heads;
  int head_dim;     /* must be 128 */
  /* QK-RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, f32 math, per head over
   * head_dim. NULL weights skip the norm for that operand. */
  const float* norm_q_weight; /* [head_dim] f32 or NULL */
  const float* norm_k_weight; /* [head_dim] f32 or NULL */
  float eps;
  /* Interleaved-pair rotary embedding with per-row tables [seq, head_dim/2]
   * f32 (row r of the tables rotates token r). NULL skips RoPE. */
  const float* rope_cos;
  const float* rope_sin;
  float scale; /* softmax scale; <= 0 selects 1/sqrt(head_dim) */
} aex_attention_args;

/* Fused QK-RMSNorm -> 2-D axial RoPE -> non-causal softmax(scale*QK^T)V.
 * Replaces the composition AttentionUtils.processQKV's norm step
 * (Sources/ImarelloDiT/AttentionUtils.swift:37-50), applyRopeBSHD
 * (AttentionUtils.swift:263-298) and computeAttention ->
 * MetalFlashAttention.scaledDotProductAttention (AttentionUtils.swift:65-135,
 * Sources/ImarelloDiT/MetalFlashAttention.swift:44-78); and in the direct
 * engine rms + rope + attention (Sources/ImarelloDirect/DirectDiTStep.swift:
 * 408-488, 568-571, 612-615). With both norm weights and the rope tables NULL
 * it is exactly scaledDotProductAttention(query:key:value:scale:mask: nil).
 * Uses context-owned scratch for the normalized Q/K (grown on demand). */
int aex_joint_attention(aex_ctx* ctx, const aex_attention_args* args, aex_stream stream);

/* Bytes of scratch aex_joint_attention needs for these args (0 when no norm
 * and no RoPE are requested). */
size_t aex_joint_attention_scratch_bytes(const aex_attention_args* args);

/* Same computation with caller-provided scratch of at least
 * aex_joint_attention_scratch_bytes(args) bytes (256-byte aligned). */
int aex_joint_attention_ws(aex_ctx* ctx, const aex_attention_args* args, void* scratch, size_t scratch_bytes,
                           aex_stream stream);

/* Fused attention that allocates nothing, for callers that cannot call
 * cudaMalloc (for example an embedding whose host framework owns the whole
 * device memory pool, or a latency-bound caller that cannot accept
 * cudaMalloc's implicit device-wide synchronisation). No counterpart in the
 * reference. Same computation and arguments as aex_joint_attention, but the
 * normalized Q/K go to a fixed scratch array compiled into the library:
 * 64 MiB, held on every GPU that loads the library until the process exits,
 * enough for
 * batch*heads*seq <= 131072 (the 1024^2 call uses 110592). Larger args are
 * rejected with AEX_ERR_INVALID_ARG. The first call on a device resolves the
 * array's device address (cudaGetSymbolAddress) with that device current; make
 * that first call before any stream capture. The address is cached per device
 * together with the CUDA context it was resolved in, and resolved again by the
 * first call in a new context (after cudaDeviceReset). Every call shares the one array:
 * calls whose executions overlap on the GPU (different streams or contexts of
 * the same device) race on it. Each call fully rewrites the part it reads, so
 * no state from an earlier call leaks into a result. */
int aex_joint_attention_noalloc(aex_ctx* ctx, const aex_attention_args* args, aex_stream stream);

/* Rotary tables. ids: [n, n_axes] f32 positions (FLUX.2: 4 axes t, h, w, l);
 * axes_dim: host array of n_axes even dimensions (FLUX.2: 32, 32, 32, 32);
 * out cos/sin: [n, sum(axes_dim)/2] f32. ids/cos/sin are device pointers.
 * Reference: Flux2PosEmbed
 * (Sources/ImarelloDiT/PosEmbed.swift:12-47), Flux2RoPE.frequencies
 * (Sources/ImarelloCore/Flux2RoPE.swift:16-63). */
int aex_rope_tables(aex_ctx* ctx, const float* ids, int n, float theta, const int* axes_dim, int n_axes,
                    float* cos_out, float* sin_out, aex_stream stream);

/* ------------------------------------------------------ 4-bit affine linear */

/* Dequantize an MLX affine-quantized matrix straight from its on-disk layout:
 * packed uint32 [n, k/8] (LSB-first nibbles), scales/biases bf16 [n, k/group],
 * out bf16 [n, k] = bf16_rne(f32(scale*q + bias)). Device pointers.
 * Reference: the CPU dequant DirectTEEncoder.embedRow
 * (Sources/ImarelloDirect/DirectTEEncoder.swift:104-123) and MLX `dequantized`
 * (DirectTEEncoder.swift:129-134). group_size must be 64, bits 4. */
int aex_dequantize_mlx(aex_ctx* ctx, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
                       int n, int k, int group_size, int bits, uint16_t* out, aex_stream stream);

/* Unpack an MLX affine 4-bit weight (device pointers in the MLX layout above)
 * into the device-resident tile layout the qmm kernels read (K0). The handle
 * owns its device memory until aex_qweight_destroy. Reference: weight upload
 * DirectDiTStep.quant / loadBlocks (Sources/ImarelloDirect/DirectDiTStep.swift:
 * 278-335) and TransformerWeights.loadQuantized
 * (Sources/ImarelloDiT/TransformerWeights.swift:13-54). */
int aex_qweight_create(aex_ctx* ctx, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
                       int n, int k, int group_size, int bits, aex_qweight** out, aex_stream stream);
void aex_qweight_destroy(aex_qweight* w);
int aex_qweight_shape(const aex_qweight* w, int* n, int* k);

/* Dequantize a tile-layout weight back to row-major bf16 [n, k] (bit-exact
 * with aex_dequantize_mlx on the source). */
int aex_qweight_dequantize(aex_ctx* ctx, const aex_qweight* w, uint16_t* out, aex_stream stream);

#define AEX_DTYPE_BF16 0
#define AEX_DTYPE_F32 1

/* y[m, n] = x[m, k] . deq(W)[n, k]^T, x bf16 (row pitch ldx elements), y bf16
 * or f32 (row pitch ldy), f32 accumulation. Reference: AttentionUtils.applyLinear
 * -> quantizedMM(transpose: true, groupSize: 64, bits: 4)
 * (Sources/ImarelloDiT/AttentionUtils.swift:140-230) and the direct engine's
 * qmm dispatch (Sources/ImarelloDirect/DirectDiTStep.swift:374-406). */
int aex_qmm(aex_ctx* ctx, const aex_qweight* w, const void* x, int64_t ldx, int m, void* y, int64_t ldy,
            int y_dtype, aex_stream stream);

/* aex_qmm with the activation dtype chosen: x_dtype AEX_DTYPE_BF16 (as
 * aex_qmm) or AEX_DTYPE_F32 (row pitch ldx a multiple of 4 elements; m <= 16
 * and k <= 24576, else AEX_ERR_UNSUPPORTED). Reference: the conditioner's f32 qmm
 * affine_qmm_t_float_gs_64_b_4 on f32 activations (timestep MLP, modulation
 * heads, norm_out; Sources/ImarelloDirect/DirectConditioner.swift:48,98-116,
 * 183-190). The dot keeps f32 throughout: y = sum_g scale_g * sum(x * q) +
 * bias_g * sum(x), the unrounded dequantized weights. */
int aex_qmm_ex(aex_ctx* ctx, const aex_qweight* w, const void* x, int x_dtype, int64_t ldx, int m, void* y,
               int64_t ldy, int y_dtype, aex_stream stream);

/* ------------------------------------------------------------ DiT engine */

/* The FLUX.2-klein transformer denoise step on one device: the direct
 * engine's static-plan step (DirectDiTStep, Sources/ImarelloDirect/
 * DirectDiTStep.swift:11-977) plus its conditioner (DirectConditioner,
 * Sources/ImarelloDirect/DirectConditioner.swift:14-255) and the packed-latent
 * denoiser (DirectDiTPackedDenoiser.denoise, DirectDiTAdapter.swift:25-81).
 * head_dim is 128. Klein 4B: hidden 3072, heads 24, 5 double + 20 single
 * blocks, mlp_hidden 9216, in_channels 128, text_dim 7680, timestep_dim 256,
 * l_txt 512, l_img = (W/16)*(H/16), rms_eps 1e-5, ln_eps 1e-6. */
typedef struct aex_dit aex_dit;

typedef struct aex_dit_config {
  int hidden;
  int heads;
  int n_double;
  int n_single;
  int mlp_hidden;
  int in_channels;
  int text_dim;
  int timestep_dim;
  int l_txt;
  int l_img;
  float rms_eps;
  float ln_eps;
} aex_dit_config;

/* Allocates the engine's static buffer plan (DirectDiTStep.allocateScratch,
 * DirectDiTStep.swift:155-274). */
int aex_dit_create(aex_ctx* ctx, const aex_dit_config* cfg, aex_dit** out);
void aex_dit_destroy(aex_dit* dit);

/* Upload one 4-bit linear from its MLX arrays (device pointers: packed uint32
 * [n, k/8], bf16 scales/biases [n, k/64]) under its MLX key, e.g.
 * "transformer_blocks.0.attn.to_q", "single_transformer_blocks.3.attn.to_out",
 * "x_embedder", "norm_out.linear" (DirectDiTStep.quant/loadBlocks/loadHead,
 * DirectDiTStep.swift:278-335, 844-884; DirectConditioner.init :30-83). */
int aex_dit_load_linear(aex_dit* dit, const char* name, const uint32_t* packed, const uint16_t* scales,
                        const uint16_t* biases, int n, int k, aex_stream stream);
/* Upload one RMSNorm weight ([128] f32 device), e.g.
 * "transformer_blocks.0.attn.norm_added_q" (DirectDiTStep.normW :285-293). */
int aex_dit_load_norm(aex_dit* dit, const char* name, const float* weight, aex_stream stream);
/* Rotary tables [l_txt + l_img, 64] f32 (device), text rows first
 * (DirectConditioner.rope; setConditioning cos/sin, DirectDiTStep.swift:337-355). */
int aex_dit_set_rope(aex_dit* dit, const float* cos_t, const float* sin_t, aex_stream stream);
/* Context embedding: bf16 [l_txt, text_dim] -> context_embedder (4-bit,
 * bf16 output) -> f32 text residual (DirectConditioner.projectContext :217-240). */
int aex_dit_project_context(aex_dit* dit, const void* embeds, aex_stream stream);
/* Per-step conditioning on the device for one timestep (sigma * 1000):
 * sinusoid -> time MLP -> SiLU -> modulation heads and norm_out
 * (DirectConditioner.stepConditioning :172-213, setStepConditioning
 * DirectDiTStep.swift:887-904). */
int aex_dit_set_timestep(aex_dit* dit, float timestep, aex_stream stream);
/* One transformer pass: latents f32 [l_img, in_channels] -> predicted velocity
 * f32 [l_img, in_channels] (x_embedder, 25 blocks, norm_out, proj_out;
 * DirectDiTStep.encodeDenoiseStep :908-950 without the Euler update). */
int aex_dit_forward(aex_dit* dit, const float* latents, float* velocity, aex_stream stream);
/* forward + Euler update lat_out = lat_in + dt * v (encodeDenoiseStep :908-971). */
int aex_dit_denoise_step(aex_dit* dit, const float* lat_in, float* lat_out, float dt, aex_stream stream);
/* The whole denoise: Flux2Scheduler(steps, l_img) (Flux2Scheduler.swift:20-109),
 * per step set_timestep + denoise_step; `latents` holds the noise on entry and
 * the result on return (DirectDiTPackedDenoiser.denoise :25-81). */
int aex_dit_denoise(aex_dit* dit, float* latents, int steps, aex_stream stream);

/* Weights from MLX safetensors (TransformerWeights.loadQuantized,
 * Sources/ImarelloDiT/TransformerWeights.swift:13-32; shard discovery as
 * SafetensorsLoader.shardFileNames, Sources/ImarelloWeights/SafetensorsLoader.swift:6-29;
 * keys as DirectDiTStep.loadBlocks / loadHead, Sources/ImarelloDirect/DirectDiTStep.swift:278-335,844-884).
 * `path`: one .safetensors file, or a directory of shards (those named by
 * model.safetensors.index.json when present, else every *.safetensors, sorted;
 * a later shard's tensor replaces an earlier one of the same name). Every
 * "<name>.weight" of dtype U32 [n, k/8] with "<name>.scales" and "<name>.biases"
 * [n, k/64] (BF16, or F16/F32 holding bf16-exact values) is loaded as the 4-bit
 * linear <name> (aex_dit_load_linear); every other "<name>.weight" of 128 floats
 * as the norm weight <name> (aex_dit_load_norm). Any other tensor: AEX_ERR_UNSUPPORTED
 * naming it. Blocks until the uploads are done. *n_linear / *n_norm (may be NULL)
 * receive the counts. */
int aex_dit_load_safetensors(aex_dit* dit, const char* path, int* n_linear, int* n_norm, aex_stream stream);

/* Lists the tensors of a safetensors file or shard directory without touching
 * the GPU, one line per tensor: "name dtype d0,d1,.. file_offset nbytes\n",
 * NUL-terminated in out (truncated to out_len). AEX_ERR_INVALID_ARG, with the
 * reason in out, for a missing, unreadable or malformed file. No reference
 * counterpart: the inspection side of aex_dit_load_safetensors. */
int aex_safetensors_scan(const char* path, char* out, size_t out_len);

/* ------------------------------------------------ multi-GPU (NCCL, NVLink) */

/* Sequence-parallel attention over P GPUs, one process per GPU: a ring of
 * NCCL point-to-point K/V hops merged by log-sum-exp, or (the default while
 * the gathered K/V fit in 8 GiB) one all-gather of K/V and one attention call
 * over all keys; AEX_SP_SCHEDULE=ring|gather overrides, the same on every rank. No
 * counterpart exists in the single-device reference, which keeps the full
 * sequence on one device (ParallelSelfAttention.swift:134-136); this computes
 * the same softmax(scale*QK^T)V for the 2048^2 joint sequence (512 text +
 * 16384 image tokens) split into P equal contiguous shards. NCCL is resolved
 * at run time (libnccl.so.2 or the copy already loaded in the process). */
typedef struct aex_comm aex_comm;
#define AEX_COMM_ID_BYTES 128

/* 128-byte NCCL unique id, created on one rank and shared with the others. */
int aex_comm_unique_id(void* id_out);
/* Collective over `world` ranks; gives up after timeout_ms (<= 0: no bound). */
int aex_comm_create(aex_ctx* ctx, int world, int rank, const void* id, int timeout_ms, aex_comm** out);
void aex_comm_destroy(aex_comm* comm);
/* Abort in-flight NCCL work of this communicator (after a failed/timed-out sync). */
int aex_comm_abort(aex_comm* comm);
/* args describe this rank's shard: batch 1, seq = shard length (equal on all
 * ranks), the norm weights and the RoPE rows of the shard's tokens; V heads
 * contiguous. Every rank calls it with the same shapes. */
int aex_ring_attention(aex_ctx* ctx, aex_comm* comm, const aex_attention_args* args, aex_stream stream);
/* The exchange schedule aex_ring_attention and the sequence-parallel engine take
 * for `world` shards of `seq` tokens x `heads` heads: 0 ring, 1 all-gather,
 * 2 overlap (pairwise exchange overlapped with per-shard attention). While
 * the gathered K/V fit in 8 GiB the default is overlap at world 2 and
 * all-gather otherwise, else ring; -1 bad arguments.
 * AEX_SP_SCHEDULE=overlap|gather|ring overrides. */
int aex_sp_schedule(int world, int seq, int heads);

/* One step of the overlap schedule's plan (host logic, no GPU needed). */
#define AEX_SP_OP_EXCHANGE 0 /* one NCCL group: this rank's K/V to send_to, recv_from's K/V into slot recv_from */
#define AEX_SP_OP_ATTEND 1   /* attention of the local queries over slot `slot` into partial `part` */
#define AEX_SP_OP_MERGE 2    /* log-sum-exp merge of partials [0, part) into the output */
typedef struct aex_sp_op {
  int kind;
  int send_to, recv_from; /* EXCHANGE */
  int slot;               /* ATTEND: the rank whose K/V shard it reads */
  int part;               /* EXCHANGE: its index h (1..world-1); ATTEND: partial index; MERGE: partial count */
  int wait_exchange;      /* ATTEND: the EXCHANGE index h whose shard it reads, -1 for the local shard */
  int stream;             /* ATTEND: 0 the caller's stream, 1 the communicator's second compute stream */
} aex_sp_op;
/* The overlap schedule's steps for `rank` of `world`, in issue order, into ops
 * (max_ops entries); returns the step count (ops NULL: just the count), -1 for
 * bad arguments or world > 16. The same plan drives aex_ring_attention's
 * overlap schedule. No reference counterpart (the reference is one device). */
int aex_sp_plan(int world, int rank, aex_sp_op* ops, int max_ops);
/* Key ranges the all-gather schedule's attention call splits into on a device
 * of `sms` SMs (1: no split; at most 4), chosen so the CTAs of a short shard
 * fill whole waves: 2048^2 at world 8 (2,112 rows, 24 heads) on 148 SMs gives
 * 2. -1 for bad arguments. */
int aex_sp_key_ranges(int world, int seq, int heads, int sms);

/* Sequence parallelism for one image over the ranks of `comm` (the long
 * sequence, 2048^2; ImarelloPipeline.swift:921-927 drives one GPU per image): this engine
 * was created for one contiguous shard of the joint sequence (cfg.l_txt +
 * cfg.l_img = (l_txt_total + l_img_total) / world rows; all text rows on rank 0,
 * cfg.l_txt = 0 elsewhere; RoPE tables and latents are the shard's rows). Linears
 * and glue stay on the shard; each block's joint attention runs over all ranks
 * (aex_ring_attention's schedule, NCCL point-to-point or all-gather); the scheduler
 * uses l_img_total. Every rank makes the same calls in the same order.
 * aex_dit_denoise then launches its steps one by one (no CUDA graph). comm NULL
 * returns the engine to one GPU. */
int aex_dit_set_sequence_parallel(aex_dit* dit, aex_comm* comm, int l_txt_total, int l_img_total);


/* -------------------------------------------------------------- self test */

/* Tensor-core path self test (no reference counterpart; a device bring-up
 * check like the reference's `direct-spike` ladder, ImarelloCLI.swift:1701-1805).
 * d[128, n] (f32) = a[128, 128] . op(b), a bf16 row-major;
 * mode 0: b is [n, 128] (K-major), op(b) = b^T, operands from shared memory;
 * mode 1: b is [128, n] (N-major), op(b) = b, A operand from tensor memory;
 * mode 2: b is [128, n] (N-major), op(b) = b, operands from shared memory.
 * n must be 128 or 256 (256 only for mode 0). Device pointers. */
int aex_selftest_umma(aex_ctx* ctx, int mode, const uint16_t* a, const uint16_t* b, int n, float* d,
                      aex_stream stream);

/* Failure-detection self test (no reference counterpart; the analogue of the
 * reference's command-buffer error check after waitUntilCompleted,
 * DirectDiTStep.swift:968-970): launches one kernel that waits on a barrier
 * nothing arrives on, bounded by timeout_us (1 .. 1e6) of device time instead
 * of the library's 2 s, after which it records a device status and returns
 * without faulting. The next aex_sync on `stream` then returns AEX_ERR_DEVICE
 * (and clears the status); the context stays usable. */
int aex_selftest_wait(aex_ctx* ctx, int timeout_us, aex_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* AESTRIX_CUDA_H */
