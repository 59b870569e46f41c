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
//  * The Q4_K min (and the +128 bias of the unsigned Q8_0 view) is one extra mma per tile pair:
//    A = -m[row][sub-block], B = per-sub-block activation sums split into fp16 hi + lo.
//  * Activations reach the consumer warps through shared memory in fragment order (one LDS.64 per mma).
#pragma once
#include "common.cuh"

namespace clm {

constexpr int kQ4kTileBytes = 2304;  // 2048 B nibbles + 16 rows x 16 B scale records
constexpr int kQ80TileBytes = 4352;  // 4096 B int8 + 16 rows x 8 half scales
constexpr int kGemvWarps = 8;        // row tiles per row group / warps per CTA
constexpr int kXfragSbBytes = 16 * 32 * 8;  // one superblock of B fragments for one n8 column tile
constexpr int kXsPairBytes = 32 * 16;       // one superblock pair of sub-block sums (hi, lo) per column tile
constexpr size_t kGemvSmemBudget = 210 * 1024;  // dynamic shared memory of one persistent GEMV CTA

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

// Writes activation row p (x[cols] in shared memory, fp32) in the GEMV's fragment order:
//   xfrag[sb][nt][s][lane], lane = (p%8)*4 + t: {half2(x[k0], x[k0+1]), half2(x[k1], x[k1+1]) * hi_scale}
//   xs[pair][nt][lane]: fp16 hi/lo split of the 32-element sub-block sums
// hi_scale is 1/16 for Q4_K (high-nibble sub-blocks) and 1 for Q8_0.  `sums` is shared scratch of cols/32
// floats.  x == nullptr writes zeros (rows beyond the window).  All threads of the block must call.
__device__ inline void write_xfrag_row(const float* x, int p, uint32_t cols, int nt_count, float hi_scale,
                                       uint2* __restrict__ xfrag, uint4* __restrict__ xs, float* sums) {
  const uint32_t sb_count = cols / 256, nt = (uint32_t)p / 8, g = (uint32_t)p % 8;
  for (uint32_t it = threadIdx.x; it < sb_count * 64; it += blockDim.x) {
    const uint32_t sb = it / 64, s = (it / 4) % 16, t = it % 4;
    uint2 v = make_uint2(0, 0);
    if (x) {
      const uint32_t k0 = sb * 256 + 64 * t + 2 * s, k1 = k0 + 32;
      v.x = pack_half2(x[k0], x[k0 + 1]);
      v.y = pack_half2(x[k1] * hi_scale, x[k1 + 1] * hi_scale);
    }
    xfrag[((size_t)sb * nt_count + nt) * 512 + s * 32 + g * 4 + t] = v;
  }
  for (uint32_t j = threadIdx.x; j < cols / 32; j += blockDim.x) {
    float a = 0.0f;
    if (x)
      for (int l = 0; l < 32; ++l) a += x[32 * j + l];
    sums[j] = a;
  }
  __syncthreads();
  const uint32_t pairs = (sb_count + 1) / 2;
  for (uint32_t it = threadIdx.x; it < pairs * 4; it += blockDim.x) {
    const uint32_t pr = it / 4, t = it % 4;
    float v[4];
    for (int h = 0; h < 2; ++h)
      for (int e = 0; e < 2; ++e) {
        const uint32_t sb = 2 * pr + h;
        v[2 * h + e] = sb < sb_count ? sums[sb * 8 + 2 * t + e] : 0.0f;
      }
    float hi[4], lo[4];
    for (int i = 0; i < 4; ++i) {
      hi[i] = __half2float(__float2half_rn(v[i]));
      lo[i] = v[i] - hi[i];
    }
    xs[((size_t)pr * nt_count + nt) * 32 + g * 4 + t] =
        make_uint4(pack_half2(hi[0], hi[1]), pack_half2(hi[2], hi[3]), pack_half2(lo[0], lo[1]), pack_half2(lo[2], lo[3]));
  }
  __syncthreads();
}

GemvShape gemv_shape(int quant, uint32_t rows, uint32_t cols);
GemvPlan gemv_plan(const GemvShape& s, int q, int sm_count);

// Repack a GGUF-layout tensor (device memory) into the tiled layout (device memory, s.bytes()).
// half_rows > 0 interleaves a stacked [gate; up] tensor of 2*half_rows rows in 64-row halves per 128-row group.
int launch_repack(const GemvShape& s, const uint8_t* d_src, uint8_t* d_tiles, cudaStream_t st, uint32_t half_rows = 0);
}  // namespace clm
