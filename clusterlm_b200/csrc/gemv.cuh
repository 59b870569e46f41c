// gemv.cuh — tiled, fused-dequant q-row GEMV for GGUF Q4_K / Q8_0 weights on sm_100a.
//
// The computation is the reference's reference_matmul_rows (runtime/domain/src/reference_kernels.cpp:24-30):
// y[p][i] = W[i] . x[p] for a window of q <= 16 positions, each weight row read once.  At q <= 16 it is
// HBM-bound, so the design minimises instructions per weight byte:
//
//  * Weights are repacked once at upload into tiles of 16 rows x 256 columns (one Q4_K superblock or eight
//    Q8_0 blocks per row).  The repack is a lossless byte permutation: every byte of the GGUF tensor lands in
//    exactly one tile word, ordered so that one 32-bit word is one thread's share of one m16n8k16 A fragment.
//    Eight tiles of consecutive row tiles at the same superblock are contiguous ("row group" of 128 rows).
//  * Thread (g = lane/4, t = lane%4) owns sub-blocks 2t and 2t+1 of rows g and g+8 for the whole tile, so it
//    decodes exactly four scales and four mins per tile and no scale is decoded twice in a warp.
//  * Nibbles/bytes become fp16 with one LOP3 (or PRMT) into the 0x6400 exponent (value 1024 + n) and one
//    HFMA2 h*s - 1024*s = s*n (exact product, one rounding).  High Q4_K nibbles give 16*n; the activation
//    fragments of those k are pre-scaled by 1/16, so no extra shift is needed.
//  * The Q4_K min (and the +128 bias of the unsigned Q8_0 view) is one extra mma pair per superblock:
//    A = -m[row][sub-block] for both 16-column halves, B = the halves' activation sums split into fp16 hi + lo,
//    written by the producer directly in B-fragment order (gemv2.cuh).
//  * Activations reach the consumer warps through shared memory in fragment order (one LDS.64 per mma).
#pragma once
#include "common.cuh"

namespace clm {

constexpr int kQ4kTileBytes = 2304;  // 2048 B nibbles + 16 rows x 16 B scale records
constexpr int kQ80TileBytes = 4352;  // 4096 B int8 + 16 rows x 8 half scales
constexpr int kGemvWarps = 8;        // row tiles per row group / warps per CTA
constexpr int kXfragSbBytes = 16 * 32 * 8;  // one superblock of B fragments for one n8 column tile
constexpr size_t kGemvSmemBudget = 210 * 1024;  // dynamic shared memory of one persistent GEMV CTA

// n-tiles of the min / bias B fragments per superblock in an activation hand-off (two for up to 16 window rows,
// four for up to 32)
__host__ __device__ constexpr int sum_tiles(int nt) { return nt < 2 ? 2 : nt; }
// window rows per group of sum-of-squares partials (XBuf::ss is [nss][kSsRows])
constexpr int kSsRows = 32;

// Superblocks per unit of the stream-K GEMV: pairs, or single superblocks for 4 n-tiles (whose activation fragments
// would otherwise leave room for only two ring stages).
__host__ __device__ constexpr int gemv_unit_sb(int nt) { return nt >= 4 ? 1 : 2; }

struct GemvShape {
  int quant = 0;
  uint32_t rows = 0, cols = 0;
  uint32_t rt = 0;  // row tiles (rows / 16)
  uint32_t ng = 0;  // row groups (ceil(rt / 8))
  uint32_t sb = 0;  // superblocks per row (cols / 256)
  int tile_bytes = 0;
  uint64_t bytes() const { return (uint64_t)ng * sb * kGemvWarps * tile_bytes; }
};

struct GemvPlan {
  int nt = 1;        // n8 column tiles (1: q <= 8, 2: q <= 16)
  int grid = 0;      // persistent CTAs (one per SM)
  int stages = 0;    // shared-memory ring stages per CTA
  int ksplit = 1;    // partial slots per row group (the most CTA ranges one group can span)
  size_t smem = 0;   // dynamic shared memory bytes
  uint64_t xfrag_bytes = 0, xs_bytes = 0;
};

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);  // one paired conversion, lo in the low half
  return *reinterpret_cast<const uint32_t*>(&h);
}

GemvShape gemv_shape(int quant, uint32_t rows, uint32_t cols);
GemvPlan gemv_plan(const GemvShape& s, int q, int sm_count);

// Repack a GGUF-layout tensor (device memory) into the tiled layout (device memory, s.bytes()).
// half_rows > 0 interleaves a stacked [gate; up] tensor of 2*half_rows rows in 64-row halves per 128-row group.
int launch_repack(const GemvShape& s, const uint8_t* d_src, uint8_t* d_tiles, cudaStream_t st, uint32_t half_rows = 0);
}  // namespace clm
