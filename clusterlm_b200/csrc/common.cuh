// common.cuh — shared host/device helpers for libclm_b200 (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/clm_b200.h"

namespace clm {

// ---- error model: int status + thread-local message (the ABI's clm_b200_last_error) ----
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define CLM_CUDA(call)                                  \
  do {                                                  \
    cudaError_t clm_e_ = (call);                        \
    if (clm_e_ != cudaSuccess) return ::clm::cuda_fail(clm_e_, #call); \
  } while (0)

#define CLM_CHECK(cond, code, msg)             \
  do {                                         \
    if (!(cond)) return ::clm::fail((code), (msg)); \
  } while (0)

#define CLM_TRY(expr)              \
  do {                             \
    int clm_s_ = (expr);           \
    if (clm_s_ != CLM_OK) return clm_s_; \
  } while (0)

// Launch-error check after a kernel launch.
#define CLM_LAUNCHED(what) CLM_CUDA(cudaGetLastError())

}  // namespace clm

// Context: one device, one stream, and a scratch arena reused by calls that need temporaries.
struct clm_b200_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  // Grow-only device scratch for temporaries of a single call (row statistics, partial sums).
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // Objects created on this context (engines, matrices, links) that are still alive.  clm_b200_ctx_destroy
  // while some are alive only marks the context closed; the last object's destruction frees it.
  int refs = 0;
  bool closed = false;
};

namespace clm {

// Ensures ctx->scratch holds at least `bytes`; synchronises the stream before growing.
int ctx_scratch(clm_b200_ctx* ctx, size_t bytes, void** out);
// Makes ctx->device current for the calling thread.
int ctx_enter(clm_b200_ctx* ctx);
// An object created on ctx holds it (retain) until it is destroyed (release frees a closed, unused context).
void ctx_retain(clm_b200_ctx* ctx);
void ctx_release(clm_b200_ctx* ctx);
inline cudaStream_t pick_stream(clm_b200_ctx* ctx, void* s) { return s ? static_cast<cudaStream_t>(s) : ctx->stream; }

// ---- device helpers ----
__host__ __device__ inline uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

// Philox4x32-10 (Salmon et al., SC'11).
__host__ __device__ inline void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                              uint32_t k1, uint32_t out[4]) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)p1;
    c3 = (uint32_t)p0;
    c0 = n0;
    c2 = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

// Uniform double in [0,1): top 53 bits of (o0:o1), the construction of the reference Rng::uniform()
// (runtime/domain/src/sampling.cpp:33) applied to a Philox block.
__host__ __device__ inline double philox_uniform(uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
  uint32_t o[4];
  philox4x32_10(c0, c1, c2, c3, (uint32_t)key, (uint32_t)(key >> 32), o);
  const uint64_t bits = ((uint64_t)o[0] << 32) | o[1];
  return (double)(bits >> 11) * 0x1.0p-53;
}

}  // namespace clm
