// gemm_tc.cuh — wide-window (17..256 rows) dequantising GEMM on tcgen05 tensor cores (kernel in gemm_tc.cu).
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace clm {

struct TcPlan {
  int P = 0;              // window rows rounded up to a multiple of 16 (the MMA's N)
  int ksplit = 1;         // K splits (grid y); > 1 sums f32 partials in split order
  int stages = 0;         // (A tile, B tile) stages in shared memory
  int kc = 64;            // columns per stage (64, or 128 when two such stages fit next to the raw ring)
  size_t smem = 0;        // dynamic shared memory of one CTA
  size_t part_floats = 0; // f32 partials needed when ksplit > 1
  size_t xh_bytes = 0;    // fp16 activation tiles (P x cols)
};

TcPlan gemm_tc_plan(const GemvShape& s, int q, int sm_count);

// y[p][n] = W[n] . x[p] (x: q x cols f32 row-major, 16-byte aligned; y: q x rows f32) for 17 <= q <= 256 with W
// in the tile layout of gemv.cuh (Q4_K or Q8_0).  d_xh holds p.xh_bytes (16-byte aligned) for the fp16 activation
// tiles, d_part p.part_floats floats when p.ksplit > 1; a bounded wait that gives up stores kErrWaitTimeout in
// *d_err (if not null).
int launch_gemm_tc(const GemvShape& s, const TcPlan& p, const uint8_t* d_tiles, const float* d_x, int q, float* d_y,
                   uint8_t* d_xh, float* d_part, int* d_err, cudaStream_t st);

// The GEMM alone, over activation tiles already in d_xh (written by launch_tc_xprep or a fused producer).  With
// sum_splits false and p.ksplit > 1 the K-split partials stay in d_part ([ksplit][q][rows], summed in split order
// by the consumer) and d_y is not written.
int launch_gemm_tc_tiles(const GemvShape& s, const TcPlan& p, const uint8_t* d_tiles, const uint8_t* d_xh, int q,
                         float* d_y, float* d_part, int* d_err, cudaStream_t st, bool sum_splits = true);

// Activation tiles of the GEMM: x (q x K f32, row-major) -> fp16, K-major 128-byte-swizzled tiles of 64 columns,
// tile c at d_xh + c * P * 128 with row p's 16-byte chunk j at tc_tile_off(p, j); rows q..P-1 are zero.
int launch_tc_xprep(const float* d_x, int q, int K, int P, uint8_t* d_xh, cudaStream_t st);

// Byte offset of row r's 16-byte chunk c (8 fp16 columns) inside one 64-column activation tile.
__host__ __device__ __forceinline__ uint32_t tc_tile_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

}  // namespace clm
