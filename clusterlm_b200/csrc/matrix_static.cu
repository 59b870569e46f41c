// matrix_static.cu — clm_b200_matmul_rows_static: the q-row GEMM of clm_b200_matmul_rows with every byte of its
// scratch in one fixed device array compiled into this library, so that the call allocates no device memory.
//
// Scratch layout inside g_matmul_scratch (offsets 256-byte aligned):
//   [0, kCounterBytes)   split-reduction counters, one int per 128-row group, and after them one error word.  They
//                        must be zero when the product starts, so every call clears them first (an asynchronous
//                        memset of the array, no allocation): a call whose bounded wait gave up leaves arrivals
//                        behind, and the next call must not pass its waits on them.
//   then                 activation fragments, sub-block sums, split partials (written before they are read
//                        within the same call).
// A row group whose split reduction gave up is written as NaN (the call itself has already returned CLM_OK: it
// only enqueues work).
// One array per device: two calls whose kernels overlap on the same device (different streams, or different
// threads without ordering) race on it and give wrong results.  Callers serialise calls per device.
// The first call on a device resolves the array's address with cudaGetSymbolAddress (with that device current)
// and caches it; make that first call before any stream capture that should contain later calls.
#include <mutex>

#include "gemv2.cuh"
#include "matrix.cuh"

namespace clm {
namespace {

constexpr size_t kStaticScratchBytes = CLM_B200_STATIC_SCRATCH_BYTES;
constexpr size_t kCounterBytes = 16 * 1024;
constexpr size_t kMaxGroups = kCounterBytes / sizeof(int) - 64;  // 4032 row groups = 516,096 rows; then the error word
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_matmul_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

size_t align256(size_t n) { return (n + 255) & ~size_t{255}; }

// Address of g_matmul_scratch on `device`, which must be the current device.
int static_scratch(int device, void** out) {
  CLM_CHECK(device >= 0 && device < kMaxDevices, CLM_OUT_OF_RANGE, "device ordinal beyond the static scratch table");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_matmul_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static matmul scratch)");
    CLM_CHECK(p != nullptr, CLM_INTERNAL, "static matmul scratch has no device address");
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return CLM_OK;
}

int matmul_rows_static(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x, int q, float* d_y,
                       cudaStream_t st) {
  if (w->quant == CLM_QUANT_F32 || w->quant == CLM_QUANT_Q8_FIXTURE)
    return launch_gemv_f32(static_cast<const float*>(w->data), w->rows, w->cols, d_x, q, d_y, st);
  const GemvShape& s = w->shape;
  const GemvPlan p = gemv_plan(s, q, ctx->sm_count);
  CLM_CHECK((size_t)s.ng <= kMaxGroups, CLM_OUT_OF_RANGE,
            "matrix has more row groups than the static scratch's counters cover (rows <= 516096)");
  const size_t fb = align256(xfrag_bytes((int)s.cols, p.nt)), sb = align256(xsum_bytes((int)s.cols));
  const size_t pb = align256((size_t)s.ng * p.ksplit * q * 128 * sizeof(float));
  const size_t need = kCounterBytes + fb + sb + pb;
  CLM_CHECK(need <= kStaticScratchBytes, CLM_RESOURCE_EXHAUSTED,
            "matmul_rows_static needs " + std::to_string(need) + " bytes of scratch; the static scratch holds " +
                std::to_string(kStaticScratchBytes) + " (use clm_b200_matmul_rows)");
  void* scratch = nullptr;
  CLM_TRY(static_scratch(ctx->device, &scratch));
  uint8_t* base = static_cast<uint8_t*>(scratch);
  int* counters = reinterpret_cast<int*>(base);
  CLM_CUDA(cudaMemsetAsync(counters, 0, (kMaxGroups + 1) * sizeof(int), st));
  XBuf in;
  in.frag = reinterpret_cast<uint2*>(base + kCounterBytes);
  in.sum = reinterpret_cast<float*>(base + kCounterBytes + fb);
  float* part = reinterpret_cast<float*>(base + kCounterBytes + fb + sb);
  const float hi = w->quant == CLM_QUANT_Q4_K ? 0.0625f : 1.0f;
  CLM_TRY(launch_prep_rows(d_x, s.cols, q, (int)s.cols, nullptr, p.nt, hi, in, false, st));
  Epi e;
  e.kind = EPI_STORE;
  e.out = d_y;
  e.out_ld = s.rows;
  e.err = counters + kMaxGroups;
  return launch_gemv(s, p, static_cast<const uint8_t*>(w->data), in, q, e, part, counters, st);
}

}  // namespace
}  // namespace clm

using namespace clm;

extern "C" int clm_b200_matmul_rows_static(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x,
                                           uint32_t positions, float* d_y, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(w != nullptr && d_x != nullptr && d_y != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  CLM_CHECK(w->ctx == ctx, CLM_INVALID_ARGUMENT, "matrix belongs to another context");
  CLM_CHECK(positions >= 1 && positions <= 16, CLM_OUT_OF_RANGE, "positions must be in [1, 16]");
  return matmul_rows_static(ctx, w, d_x, (int)positions, d_y, pick_stream(ctx, stream));
}
