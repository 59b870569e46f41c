// ctx.cu — library status, error reporting and the per-domain device context.
#include <cstdio>
#include <string>

#include "common.cuh"

namespace clm {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  const int code = (e == cudaErrorMemoryAllocation) ? CLM_RESOURCE_EXHAUSTED
                   : (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice || e == cudaErrorInsufficientDriver ||
                      e == cudaErrorNoKernelImageForDevice)
                       ? CLM_HARDWARE_UNAVAILABLE
                       : CLM_INTERNAL;
  return fail(code, std::string(what) + ": " + cudaGetErrorString(e));
}

int ctx_enter(clm_b200_ctx* ctx) {
  CLM_CHECK(ctx != nullptr, CLM_INVALID_ARGUMENT, "null context");
  CLM_CUDA(cudaSetDevice(ctx->device));
  return CLM_OK;
}

void ctx_retain(clm_b200_ctx* ctx) {
  if (ctx) ++ctx->refs;
}

static void ctx_free(clm_b200_ctx* ctx) {
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch) cudaFree(ctx->scratch);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
}

void ctx_release(clm_b200_ctx* ctx) {
  if (ctx && --ctx->refs <= 0 && ctx->closed) ctx_free(ctx);
}

int ctx_scratch(clm_b200_ctx* ctx, size_t bytes, void** out) {
  if (bytes > ctx->scratch_bytes) {
    CLM_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->scratch) CLM_CUDA(cudaFree(ctx->scratch));
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    CLM_CUDA(cudaMalloc(&ctx->scratch, want));
    ctx->scratch_bytes = want;
  }
  *out = ctx->scratch;
  return CLM_OK;
}

}  // namespace clm

using namespace clm;

extern "C" {

int clm_b200_abi_version(void) { return CLM_B200_ABI_VERSION; }

const char* clm_b200_last_error(void) { return g_last_error.c_str(); }

int clm_b200_device_count(int* n) {
  CLM_CHECK(n != nullptr, CLM_INVALID_ARGUMENT, "null output");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *n = 0;
    return CLM_OK;
  }
  *n = c;
  return CLM_OK;
}

int clm_b200_ctx_create(int device, clm_b200_ctx** out) {
  CLM_CHECK(out != nullptr, CLM_INVALID_ARGUMENT, "null output");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(CLM_HARDWARE_UNAVAILABLE, "no CUDA device is visible");
  }
  CLM_CHECK(device >= 0 && device < n, CLM_HARDWARE_UNAVAILABLE, "device index " + std::to_string(device) +
                                                                      " is not visible (" + std::to_string(n) +
                                                                      " devices)");
  cudaDeviceProp prop;
  CLM_CUDA(cudaGetDeviceProperties(&prop, device));
  CLM_CHECK(prop.major == 10 && prop.minor == 0, CLM_HARDWARE_UNAVAILABLE,
            std::string("device ") + prop.name + " is not sm_100 (this build contains sm_100a code only)");
  CLM_CUDA(cudaSetDevice(device));
  auto* c = new clm_b200_ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return cuda_fail(e, "cudaStreamCreate");
  }
  *out = c;
  return CLM_OK;
}

int clm_b200_ctx_destroy(clm_b200_ctx* ctx) {
  if (ctx == nullptr || ctx->closed) return CLM_OK;
  ctx->closed = true;
  if (ctx->refs <= 0) ctx_free(ctx);  // else the last object created on it frees it
  return CLM_OK;
}

int clm_b200_ctx_stream(clm_b200_ctx* ctx, void** stream) {
  CLM_CHECK(ctx != nullptr && stream != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  *stream = ctx->stream;
  return CLM_OK;
}

int clm_b200_ctx_synchronize(clm_b200_ctx* ctx) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CUDA(cudaStreamSynchronize(ctx->stream));
  return CLM_OK;
}

}  // extern "C"
