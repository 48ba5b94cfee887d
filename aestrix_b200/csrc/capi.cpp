// capi.cpp — context lifetime, error strings, synchronisation and TMA
// descriptor encoding for libaestrix_cuda.
#include <cudaTypedefs.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "internal.h"

namespace {
thread_local std::string g_create_error;

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

namespace aex {

int set_error(aex_ctx* ctx, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx)
    ctx->last_error = buf;
  else
    g_create_error = buf;
  return code;
}

int cuda_error(aex_ctx* ctx, cudaError_t e, const char* what) {
  const int code = (e == cudaErrorMemoryAllocation) ? AEX_ERR_OOM : AEX_ERR_CUDA;
  return set_error(ctx, code, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int bind_device(aex_ctx* ctx) {
  int cur = -1;
  AEX_CUDA_TRY(ctx, cudaGetDevice(&cur));
  if (cur != ctx->device) AEX_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  return AEX_OK;
}

int ensure_scratch(aex_ctx* ctx, size_t bytes, void** out) {
  if (bytes == 0) {
    *out = nullptr;
    return AEX_OK;
  }
  if (ctx->scratch_bytes < bytes) {
    if (ctx->scratch) {
      // The previous scratch may still be in use by queued work on any stream.
      AEX_CUDA_TRY(ctx, cudaDeviceSynchronize());
      cudaFree(ctx->scratch);
      ctx->scratch = nullptr;
      ctx->scratch_bytes = 0;
    }
    void* p = nullptr;
    AEX_CUDA_TRY(ctx, cudaMalloc(&p, bytes));
    ctx->scratch = p;
    ctx->scratch_bytes = bytes;
  }
  *out = ctx->scratch;
  return AEX_OK;
}

int make_tmap(aex_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dtype, const void* base, int rank,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swizzle) {
  auto fn = encode_tiled_fn();
  if (!fn) return set_error(ctx, AEX_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(ctx, AEX_ERR_INVALID_ARG, "TMA base pointer %p is not 16-byte aligned", base);
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0)
      return set_error(ctx, AEX_ERR_INVALID_ARG, "TMA stride %llu bytes (dim %d) is not a multiple of 16",
                       (unsigned long long)strides_bytes[i], i + 1);
  cuuint32_t elem_str[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(out, dtype, rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box),
                  elem_str, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, AEX_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return AEX_OK;
}

int check_launch(aex_ctx* ctx, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(ctx, e, what);
  return AEX_OK;
}

}  // namespace aex

extern "C" {

int aex_abi_version(void) { return AEX_ABI_VERSION; }

int aex_ctx_create(int device, aex_ctx** out) {
  if (!out) return aex::set_error(nullptr, AEX_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return aex::cuda_error(nullptr, e, "cudaGetDeviceCount");
  if (device < 0 || device >= n)
    return aex::set_error(nullptr, AEX_ERR_INVALID_ARG, "device %d out of range [0,%d)", device, n);
  cudaDeviceProp prop{};
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return aex::cuda_error(nullptr, e, "cudaGetDeviceProperties");
  if (prop.major != 10 || prop.minor != 0)
    return aex::set_error(nullptr, AEX_ERR_UNSUPPORTED,
                          "device %d is sm_%d%d; libaestrix_cuda is built for sm_100a (B200) only", device,
                          prop.major, prop.minor);
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return aex::cuda_error(nullptr, e, "cudaSetDevice");
  auto* ctx = new aex_ctx();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  e = cudaMalloc(&ctx->d_status, sizeof(int));
  if (e != cudaSuccess) {
    delete ctx;
    return aex::cuda_error(nullptr, e, "cudaMalloc(status)");
  }
  e = cudaMemset(ctx->d_status, 0, sizeof(int));
  if (e != cudaSuccess) {
    cudaFree(ctx->d_status);
    delete ctx;
    return aex::cuda_error(nullptr, e, "cudaMemset(status)");
  }
  *out = ctx;
  return AEX_OK;
}

void aex_ctx_destroy(aex_ctx* ctx) {
  if (!ctx) return;
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (cur >= 0) cudaSetDevice(cur);
  delete ctx;
}

const char* aex_last_error_string(const aex_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : g_create_error.c_str();
}

int aex_device_sm_count(const aex_ctx* ctx) { return ctx ? ctx->sm_count : 0; }

int aex_device_status(aex_ctx* ctx, int* code) {
  if (!ctx || !code) return aex::set_error(ctx, AEX_ERR_INVALID_ARG, "NULL argument");
  if (int r = aex::bind_device(ctx)) return r;
  AEX_CUDA_TRY(ctx, cudaDeviceSynchronize());
  int v = 0;
  AEX_CUDA_TRY(ctx, cudaMemcpy(&v, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) AEX_CUDA_TRY(ctx, cudaMemset(ctx->d_status, 0, sizeof(int)));
  *code = v;
  return AEX_OK;
}

int aex_sync(aex_ctx* ctx, aex_stream stream, int timeout_ms) {
  if (!ctx) return aex::set_error(ctx, AEX_ERR_INVALID_ARG, "NULL ctx");
  if (int r = aex::bind_device(ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return aex::cuda_error(ctx, e, "cudaStreamQuery");
    if (timeout_ms > 0 && std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
      return aex::set_error(ctx, AEX_ERR_TIMEOUT, "stream still busy after %d ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int v = 0;
  AEX_CUDA_TRY(ctx, cudaMemcpy(&v, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) {
    cudaMemset(ctx->d_status, 0, sizeof(int));
    return aex::set_error(ctx, AEX_ERR_DEVICE, "a kernel reported device status %d (bounded wait expired)", v);
  }
  return AEX_OK;
}

}  // extern "C"
