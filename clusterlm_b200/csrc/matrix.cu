// matrix.cu — resident weight matrices and the q-row GEMM entry point (clm_b200_matmul_rows).
#include <algorithm>
#include <string>

#include "codec.cuh"
#include "gemv.cuh"
#include "gemv2.cuh"
#include "gemm_tc.cuh"
#include "matrix.cuh"

namespace clm {

// f32 rows: one warp per output row, lanes stride the columns, positions in registers (q <= 16).
__global__ void __launch_bounds__(256) gemv_f32_kernel(const float* __restrict__ w, uint32_t rows, uint32_t cols,
                                                       const float* __restrict__ x, int q, float* __restrict__ y) {
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= rows) return;
  const float* wr = w + (size_t)warp * cols;
  float acc[16];
#pragma unroll
  for (int p = 0; p < 16; ++p) acc[p] = 0.0f;
  for (uint32_t k = lane; k < cols; k += 32) {
    const float wv = wr[k];
#pragma unroll
    for (int p = 0; p < 16; ++p)
      if (p < q) acc[p] = fmaf(wv, x[(size_t)p * cols + k], acc[p]);
  }
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    if (p >= q) break;
    float v = acc[p];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) y[(size_t)p * rows + warp] = v;
  }
}

int launch_gemv_f32(const float* d_w, uint32_t rows, uint32_t cols, const float* d_x, int q, float* d_y,
                    cudaStream_t st) {
  const uint64_t threads = (uint64_t)rows * 32;
  gemv_f32_kernel<<<(unsigned)ceil_div(threads, 256), 256, 0, st>>>(d_w, rows, cols, d_x, q, d_y);
  CLM_LAUNCHED("gemv_f32_kernel");
  return CLM_OK;
}

int matrix_create(clm_b200_ctx* ctx, int quant, const void* bytes, bool device_src, uint64_t nbytes, uint32_t rows,
                  uint32_t cols, clm_b200_matrix** out, uint32_t half_rows) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(out != nullptr, CLM_INVALID_ARGUMENT, "null output");
  *out = nullptr;
  CLM_CHECK(rows > 0 && cols > 0, CLM_INVALID_ARGUMENT, "empty matrix");
  const uint64_t want = clm_b200_tensor_bytes(quant, (uint64_t)rows * cols);
  CLM_CHECK(want != 0, CLM_INVALID_ARGUMENT, "unsupported representation or partial block");
  CLM_CHECK(nbytes == want, CLM_DATA_LOSS, "matrix byte size does not match rows x cols in its representation");
  CLM_CHECK(bytes != nullptr, CLM_INVALID_ARGUMENT, "null bytes");
  const bool tiled = quant == CLM_QUANT_Q4_K || quant == CLM_QUANT_Q8_0;
  if (tiled) {
    CLM_CHECK(rows % 16 == 0, CLM_INVALID_ARGUMENT, "Q4_K/Q8_0 matrices need rows % 16 == 0");
    CLM_CHECK(cols % 256 == 0, CLM_INVALID_ARGUMENT, "Q4_K/Q8_0 matrices need cols % 256 == 0");
  }
  cudaStream_t st = ctx->stream;
  auto* m = new clm_b200_matrix();
  m->ctx = ctx;
  m->quant = quant;
  m->rows = rows;
  m->cols = cols;
  void* staging = nullptr;
  int status = CLM_OK;
  do {
    const void* src = bytes;
    if (device_src) {
      // the bytes may still be in flight on another stream of the caller (an encode, a copy): wait for the device
      cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) {
        status = cuda_fail(e, "cudaDeviceSynchronize(matrix upload)");
        break;
      }
    } else {
      cudaError_t e = cudaMalloc(&staging, nbytes);
      if (e != cudaSuccess) {
        status = cuda_fail(e, "cudaMalloc(matrix staging)");
        break;
      }
      e = cudaMemcpyAsync(staging, bytes, nbytes, cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) {
        status = cuda_fail(e, "cudaMemcpyAsync(matrix upload)");
        break;
      }
      src = staging;
    }
    if (tiled) {
      m->shape = gemv_shape(quant, rows, cols);
      m->bytes = m->shape.bytes();
      cudaError_t e = cudaMalloc(&m->data, m->bytes);
      if (e != cudaSuccess) {
        status = cuda_fail(e, "cudaMalloc(matrix tiles)");
        break;
      }
      status = launch_repack(m->shape, static_cast<const uint8_t*>(src), static_cast<uint8_t*>(m->data), st, half_rows);
    } else {
      m->bytes = (uint64_t)rows * cols * 4;
      cudaError_t e = cudaMalloc(&m->data, m->bytes);
      if (e != cudaSuccess) {
        status = cuda_fail(e, "cudaMalloc(matrix f32)");
        break;
      }
      status = launch_decode(quant, src, static_cast<float*>(m->data), (uint64_t)rows * cols, st);
    }
    if (status != CLM_OK) break;
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) status = cuda_fail(e, "matrix upload");
  } while (false);
  if (staging) cudaFree(staging);
  if (status != CLM_OK) {
    if (m->data) cudaFree(m->data);
    delete m;
    return status;
  }
  ctx_retain(ctx);
  *out = m;
  return CLM_OK;
}

int matmul_rows(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x, int q, float* d_y, cudaStream_t st) {
  if (w->quant == CLM_QUANT_F32 || w->quant == CLM_QUANT_Q8_FIXTURE)
    return launch_gemv_f32(static_cast<const float*>(w->data), w->rows, w->cols, d_x, q, d_y, st);
  const GemvShape& s = w->shape;
  if (q > 16) {
    // wide windows: tcgen05 tensor-core GEMM (gemm_tc.cu)
    CLM_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0, CLM_INVALID_ARGUMENT, "x must be 16-byte aligned");
    const TcPlan tp = gemm_tc_plan(s, q, ctx->sm_count);
    const size_t xb = (tp.xh_bytes + 255) / 256 * 256;
    void* scratch = nullptr;
    CLM_TRY(ctx_scratch(ctx, xb + tp.part_floats * sizeof(float), &scratch));
    uint8_t* base = static_cast<uint8_t*>(scratch);
    return launch_gemm_tc(s, tp, static_cast<const uint8_t*>(w->data), d_x, q, d_y, base,
                          reinterpret_cast<float*>(base + xb), nullptr, st);
  }
  const GemvPlan p = gemv_plan(s, q, ctx->sm_count);
  const size_t fb = xfrag_bytes((int)s.cols, p.nt), sb = xsum_bytes((int)s.cols);
  const size_t pb = (size_t)s.ng * p.ksplit * q * 128 * sizeof(float), cb = (size_t)s.ng * sizeof(int);
  void* scratch = nullptr;
  CLM_TRY(ctx_scratch(ctx, fb + sb + pb + cb + 1024, &scratch));
  uint8_t* base = static_cast<uint8_t*>(scratch);
  XBuf in;
  in.frag = reinterpret_cast<uint2*>(base);
  in.sum = reinterpret_cast<float*>(base + fb);
  float* part = reinterpret_cast<float*>(base + fb + sb);
  int* counters = reinterpret_cast<int*>(base + fb + sb + pb);
  CLM_CUDA(cudaMemsetAsync(counters, 0, cb, st));
  const float hi = w->quant == CLM_QUANT_Q4_K ? 0.0625f : 1.0f;
  CLM_TRY(launch_prep_rows(d_x, s.cols, q, (int)s.cols, nullptr, p.nt, hi, in, false, st));
  Epi e;
  e.kind = EPI_STORE;
  e.out = d_y;
  e.out_ld = s.rows;
  return launch_gemv(s, p, static_cast<const uint8_t*>(w->data), in, q, e, part, counters, st);
}

}  // namespace clm

using namespace clm;

extern "C" {

int clm_b200_matrix_upload(clm_b200_ctx* ctx, int quant, const void* h_bytes, uint64_t nbytes, uint32_t rows,
                           uint32_t cols, clm_b200_matrix** out) {
  return matrix_create(ctx, quant, h_bytes, false, nbytes, rows, cols, out);
}

int clm_b200_matrix_upload_device(clm_b200_ctx* ctx, int quant, const void* d_bytes, uint64_t nbytes, uint32_t rows,
                                  uint32_t cols, clm_b200_matrix** out) {
  return matrix_create(ctx, quant, d_bytes, true, nbytes, rows, cols, out);
}

int clm_b200_matrix_free(clm_b200_matrix* m) {
  if (m == nullptr) return CLM_OK;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  if (m->data) cudaFree(m->data);
  clm_b200_ctx* ctx = m->ctx;
  delete m;
  ctx_release(ctx);
  return CLM_OK;
}

int clm_b200_matrix_info(const clm_b200_matrix* m, int* quant, uint32_t* rows, uint32_t* cols, uint64_t* bytes) {
  CLM_CHECK(m != nullptr, CLM_INVALID_ARGUMENT, "null matrix");
  if (quant) *quant = m->quant;
  if (rows) *rows = m->rows;
  if (cols) *cols = m->cols;
  if (bytes) *bytes = m->bytes;
  return CLM_OK;
}

int clm_b200_matmul_rows(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x, uint32_t positions, float* d_y,
                         void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(w != nullptr && d_x != nullptr && d_y != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  CLM_CHECK(w->ctx == ctx, CLM_INVALID_ARGUMENT, "matrix belongs to another context");
  CLM_CHECK(positions >= 1 && positions <= 256, CLM_OUT_OF_RANGE, "positions must be in [1, 256]");
  CLM_CHECK(positions <= 16 || w->quant == CLM_QUANT_Q4_K || w->quant == CLM_QUANT_Q8_0, CLM_OUT_OF_RANGE,
            "more than 16 positions need a Q4_K or Q8_0 matrix");
  return matmul_rows(ctx, w, d_x, (int)positions, d_y, pick_stream(ctx, stream));
}

}  // extern "C"
