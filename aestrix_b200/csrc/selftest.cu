// selftest.cu — device self tests. aex_selftest_wait: a bounded wait that is
// made to run out (failure detection without a GPU fault). aex_selftest_umma:
// tensor-core bring-up check, one 128 x N x 128 bf16 UMMA with
// the three operand configurations the attention and qmm kernels rely on:
//   mode 0: A, B from shared memory, both K-major (S = Q K^T; qmm mainloop)
//   mode 1: A from tensor memory, B N-major in shared memory (O += P V)
//   mode 2: A K-major, B N-major, both from shared memory
// Operands arrive by TMA with 128-byte swizzle; the accumulator is read back
// through tcgen05.ld into a row-major f32 [128, N] result.
#include "internal.h"
#include "sm100.cuh"

namespace aex {
namespace {

constexpr int kSelftestSmem = 32768 + 65536 + 1024 + 1024;

template <int N, int MODE>
__global__ void __launch_bounds__(128, 1)
    umma_selftest_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                         const uint16_t* __restrict__ a_gmem, float* __restrict__ d, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 32768 + 65536);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  __shared__ int abort_flag;

  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[0], 32768u + N * 256u);
    tma_load_2d(sA, &tm_a, &bars[0], 0, 0);
    tma_load_2d(sA + 16384, &tm_a, &bars[0], 64, 0);
    if (MODE == 0) {
      tma_load_2d(sB, &tm_b, &bars[0], 0, 0);
      tma_load_2d(sB + N * 128, &tm_b, &bars[0], 64, 0);
    } else {
#pragma unroll
      for (int r = 0; r < N / 64; ++r) tma_load_2d(sB + r * 16384, &tm_b, &bars[0], 64 * r, 0);
    }
  }
  if (MODE == 1) {
    // Thread t owns row t of A; store it as packed bf16 pairs into TMEM
    // columns [128, 192) of its lane (column c holds K = 2c, 2c+1).
    const uint32_t* row = reinterpret_cast<const uint32_t*>(a_gmem + threadIdx.x * 128);
    uint32_t regs[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) regs[c] = row[c];
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16) + 128;
    tmem_st32(taddr, regs);
    tmem_st32(taddr + 32, regs + 32);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (threadIdx.x == 0) {
    if (mbar_wait(&bars[0], 0, &abort_flag, status, kDevTimeoutTma)) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_bf16_f32(128, N, false, MODE != 0);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint64_t bdesc;
        if (MODE == 0)
          bdesc = sdesc_sw128(smem_u32(sB) + (k / 4) * (N * 128) + (k % 4) * 32, 16, 1024);
        else
          bdesc = sdesc_sw128(smem_u32(sB) + k * 2048, 16384, 1024);
        if (MODE == 1) {
          umma_ts(tmem, tmem + 128 + k * 8, bdesc, idesc, k > 0);
        } else {
          const uint64_t adesc = sdesc_sw128(smem_u32(sA) + (k / 4) * 16384 + (k % 4) * 32, 16, 1024);
          umma_ss(tmem, adesc, bdesc, idesc, k > 0);
        }
      }
      umma_commit(&bars[1]);
    }
  }
  bool ok = mbar_wait(&bars[1], 0, &abort_flag, status, kDevTimeoutMma);
  ok = __all_sync(0xffffffffu, ok);
  tc_fence_after();
  if (ok) {
#pragma unroll 1
    for (int c = 0; c < N; c += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c, r);
      tmem_wait_ld();
      float* out = d + static_cast<size_t>(threadIdx.x) * N + c;
#pragma unroll
      for (int j = 0; j < 32; ++j) out[j] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <int N, int MODE>
int launch_selftest(aex_ctx* ctx, const uint16_t* a, const uint16_t* b, float* d, cudaStream_t s) {
  CUtensorMap tma, tmb;
  {
    uint64_t dims[2] = {128, 128}, strides[1] = {256};
    uint32_t box[2] = {64, 128};
    if (int r = make_tmap(ctx, &tma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, 2, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  if (MODE == 0) {
    uint64_t dims[2] = {128, N}, strides[1] = {256};
    uint32_t box[2] = {64, N};
    if (int r = make_tmap(ctx, &tmb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, 2, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  } else {
    uint64_t dims[2] = {N, 128}, strides[1] = {N * 2};
    uint32_t box[2] = {64, 128};
    if (int r = make_tmap(ctx, &tmb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, 2, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
  }
  auto kern = umma_selftest_kernel<N, MODE>;
  AEX_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSelftestSmem));
  kern<<<1, 128, kSelftestSmem, s>>>(tma, tmb, a, d, ctx->d_status);
  return check_launch(ctx, "umma_selftest_kernel");
}

// One warp waits on an mbarrier that nothing arrives on, with the same bounded
// loop the library's kernels use but a caller-chosen limit: after limit_ns of
// %globaltimer time it records kDevTimeoutSelftest in the status word and
// returns. Nothing else is in flight (no copies, no tensor memory), so the
// kernel ends cleanly and the context stays usable.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const uint32_t a = smem_u32(&bar);
  const uint64_t t0 = globaltimer_ns();
  bool done = false;
  while (!done) {
    done = mbar_try_wait(a, 0);
    if (!done && globaltimer_ns() - t0 > limit_ns) {
      if (threadIdx.x == 0) atomicCAS(status, 0, kDevTimeoutSelftest);
      break;
    }
  }
}

}  // namespace
}  // namespace aex

extern "C" int aex_selftest_wait(aex_ctx* ctx, int timeout_us, aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (timeout_us < 1 || timeout_us > 1000000)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "selftest wait: timeout_us %d outside [1, 1000000]", timeout_us);
  if (int r = bind_device(ctx)) return r;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(timeout_us) * 1000ull,
                                                                        ctx->d_status);
  return check_launch(ctx, "wait_selftest_kernel");
}

extern "C" int aex_selftest_umma(aex_ctx* ctx, int mode, const uint16_t* a, const uint16_t* b, int n, float* d,
                                 aex_stream stream) {
  using namespace aex;
  if (!ctx) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (!a || !b || !d) return set_error(ctx, AEX_ERR_INVALID_ARG, "NULL pointer");
  if (int r = bind_device(ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  if (mode == 0 && n == 128) return launch_selftest<128, 0>(ctx, a, b, d, s);
  if (mode == 0 && n == 256) return launch_selftest<256, 0>(ctx, a, b, d, s);
  if (mode == 1 && n == 128) return launch_selftest<128, 1>(ctx, a, b, d, s);
  if (mode == 2 && n == 128) return launch_selftest<128, 2>(ctx, a, b, d, s);
  if (mode == 2 && n == 256) return launch_selftest<256, 2>(ctx, a, b, d, s);
  return set_error(ctx, AEX_ERR_INVALID_ARG, "selftest: unsupported mode %d / n %d", mode, n);
}
