// matrix.cuh — the resident matrix object shared by the API and the engines.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

struct clm_b200_matrix {
  clm_b200_ctx* ctx = nullptr;
  int quant = 0;
  uint32_t rows = 0, cols = 0;
  void* data = nullptr;  // tiled layout (Q4_K / Q8_0) or f32 row-major (f32 / q8_0-fixture decoded)
  uint64_t bytes = 0;
  clm::GemvShape shape;  // tiled only
};

namespace clm {
// half_rows > 0: the tensor is a stacked [gate; up] pair of half_rows rows each, tiled with 64 gate rows and the
// matching 64 up rows per 128-row group (the SwiGLU epilogue's layout).
int matrix_create(clm_b200_ctx* ctx, int quant, const void* bytes, bool device_src, uint64_t nbytes, uint32_t rows,
                  uint32_t cols, clm_b200_matrix** out, uint32_t half_rows = 0);
// y[p][i] = W[i] . x[p] (q <= 16) on stream st; uses ctx scratch for staging and split partials.
int matmul_rows(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x, int q, float* d_y, cudaStream_t st);
int launch_gemv_f32(const float* d_w, uint32_t rows, uint32_t cols, const float* d_x, int q, float* d_y,
                    cudaStream_t st);
}  // namespace clm
