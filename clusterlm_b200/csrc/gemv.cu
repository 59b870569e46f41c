// gemv.cu — repack, activation staging and the tiled fused-dequant GEMV (see gemv.cuh for the design).
#include <algorithm>

#include "gemv.cuh"
#include "gemv_tile.cuh"
#include "pdl.cuh"

namespace clm {

// ---------------------------------------------------------------------------------------------------
// repack: GGUF row-major blocks -> fragment-ordered tiles
// ---------------------------------------------------------------------------------------------------
// Tiled row r -> source row.  half_rows = 0: identity.  half_rows = F > 0 (a stacked [gate; up] tensor of 2F
// rows): each 128-row group g holds gate rows 64g..64g+63 then up rows F+64g..F+64g+63, so one group carries
// both operands of SwiGLU for 64 consecutive ffn indices.
__device__ __forceinline__ uint32_t interleaved_row(uint32_t r, uint32_t half_rows) {
  if (half_rows == 0) return r;
  const uint32_t grp = r / 128, k = r % 128;
  return k < 64 ? grp * 64 + k : half_rows + grp * 64 + (k - 64);
}

// One thread per output 32-bit word of a tile's quant region, plus the scale records.
__global__ void repack_q4k_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint32_t rows,
                                  uint32_t sb_per_row, uint32_t ng, uint32_t half_rows) {
  const uint64_t tiles = (uint64_t)ng * sb_per_row * kGemvWarps;
  const uint64_t per_tile = 512 + 16;  // 512 qs words + 16 scale records
  const uint64_t gid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (gid >= tiles * per_tile) return;
  const uint64_t tile = gid / per_tile;
  const uint32_t item = (uint32_t)(gid % per_tile);
  const uint32_t r8 = (uint32_t)(tile % kGemvWarps);
  const uint64_t gs = tile / kGemvWarps;
  const uint32_t sb = (uint32_t)(gs % sb_per_row), grp = (uint32_t)(gs / sb_per_row);
  const uint32_t rt = grp * kGemvWarps + r8;
  uint8_t* t = dst + tile * kQ4kTileBytes;
  auto block_of = [&](uint32_t row) -> const uint8_t* {
    row = interleaved_row(row, half_rows);
    return row < rows ? src + ((uint64_t)row * sb_per_row + sb) * 144 : nullptr;
  };
  if (item < 512) {
    // word index = (s/4)*128 + lane*4 + (s%4)
    const uint32_t s = (item / 128) * 4 + (item % 4), lane = (item % 128) / 4;
    const uint32_t g = lane / 4, tq = lane % 4;
    const uint8_t* b0 = block_of(rt * 16 + g);
    const uint8_t* b1 = block_of(rt * 16 + g + 8);
    const uint32_t off = 16 + 32 * tq + 2 * s;
    const uint32_t x0 = b0 ? b0[off] : 0, x1 = b1 ? b1[off] : 0, x2 = b0 ? b0[off + 1] : 0,
                   x3 = b1 ? b1[off + 1] : 0;
    reinterpret_cast<uint32_t*>(t)[item] = x0 | (x1 << 8) | (x2 << 16) | (x3 << 24);
  } else {
    const uint32_t r = item - 512;
    const uint8_t* b = block_of(rt * 16 + r);
    uint8_t* rec = t + 2048 + 16 * r;
    if (!b) {
      for (int i = 0; i < 16; ++i) rec[i] = 0;
      return;
    }
    rec[0] = b[0];
    rec[1] = b[1];
    rec[2] = b[2];
    rec[3] = b[3];
    // 96-bit field: entry j (sc_j | m_j << 6) at bit 12*j
    uint32_t w[3] = {0, 0, 0};
    const uint8_t* sc = b + 4;
    for (int j = 0; j < 8; ++j) {
      int s6, m6;
      if (j < 4) {
        s6 = sc[j] & 63;
        m6 = sc[j + 4] & 63;
      } else {
        s6 = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m6 = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      const uint32_t e = (uint32_t)s6 | ((uint32_t)m6 << 6);
      const int bit = 12 * j;
      w[bit / 32] |= e << (bit % 32);
      if (bit % 32 > 20) w[bit / 32 + 1] |= e >> (32 - bit % 32);
    }
    for (int i = 0; i < 3; ++i)
      for (int k = 0; k < 4; ++k) rec[4 + 4 * i + k] = (uint8_t)(w[i] >> (8 * k));
  }
}

__global__ void repack_q80_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint32_t rows,
                                  uint32_t sb_per_row, uint32_t ng, uint32_t half_rows) {
  const uint64_t tiles = (uint64_t)ng * sb_per_row * kGemvWarps;
  const uint64_t per_tile = 1024 + 16 * 8;  // 1024 q words + 16 rows x 8 half scales
  const uint64_t gid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (gid >= tiles * per_tile) return;
  const uint64_t tile = gid / per_tile;
  const uint32_t item = (uint32_t)(gid % per_tile);
  const uint32_t r8 = (uint32_t)(tile % kGemvWarps);
  const uint64_t gs = tile / kGemvWarps;
  const uint32_t sb = (uint32_t)(gs % sb_per_row), grp = (uint32_t)(gs / sb_per_row);
  const uint32_t rt = grp * kGemvWarps + r8;
  const uint32_t blocks_per_row = sb_per_row * 8;
  uint8_t* t = dst + tile * kQ80TileBytes;
  auto block_of = [&](uint32_t row, uint32_t j) -> const uint8_t* {
    row = interleaved_row(row, half_rows);
    return row < rows ? src + ((uint64_t)row * blocks_per_row + (uint64_t)sb * 8 + j) * 34 : nullptr;
  };
  if (item < 1024) {
    // word index = (s/4)*256 + lane*8 + (s%4)*2 + e
    const uint32_t e = item % 2, s = (item / 256) * 4 + (item % 8) / 2, lane = (item % 256) / 8;
    const uint32_t g = lane / 4, tq = lane % 4, j = 2 * tq + e;
    const uint8_t* b0 = block_of(rt * 16 + g, j);
    const uint8_t* b1 = block_of(rt * 16 + g + 8, j);
    const uint32_t o = 2 + 2 * s;
    const uint32_t x0 = b0 ? b0[o] : 0, x1 = b0 ? b0[o + 1] : 0, x2 = b1 ? b1[o] : 0, x3 = b1 ? b1[o + 1] : 0;
    reinterpret_cast<uint32_t*>(t)[item] = x0 | (x1 << 8) | (x2 << 16) | (x3 << 24);
  } else {
    const uint32_t r = (item - 1024) / 8, j = (item - 1024) % 8;
    const uint8_t* b = block_of(rt * 16 + r, j);
    uint8_t* rec = t + 4096 + 16 * r + 2 * j;
    rec[0] = b ? b[0] : 0;
    rec[1] = b ? b[1] : 0;
  }
}

// ---------------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------------
GemvShape gemv_shape(int quant, uint32_t rows, uint32_t cols) {
  GemvShape s;
  s.quant = quant;
  s.rows = rows;
  s.cols = cols;
  s.rt = (rows + 15) / 16;
  s.ng = (s.rt + kGemvWarps - 1) / kGemvWarps;
  s.sb = cols / 256;
  s.tile_bytes = quant == CLM_QUANT_Q4_K ? kQ4kTileBytes : kQ80TileBytes;
  return s;
}

GemvPlan gemv_plan(const GemvShape& s, int q, int sm_count) {
  // The persistent GEMV (gemv4.cu): one CTA per SM over a ring of `stages` superblock-pair stages, each holding
  // the pair's weights (2 x 8 tiles), activation fragments (2 x nt x 4 KB) and sub-block sums (2 x sum tiles x
  // 512 B); nt = 1, 2 or 4 n-tiles of 8 window rows.
  GemvPlan p;
  p.nt = q <= 8 ? 1 : (q <= 16 ? 2 : 4);
  const int usb = gemv_unit_sb(p.nt);
  const long long units = (long long)s.ng * ((s.sb + usb - 1) / usb);
  p.grid = (int)std::min<long long>(units, sm_count > 0 ? sm_count : 148);
  const size_t stage = (size_t)usb * kGemvWarps * s.tile_bytes + (size_t)usb * p.nt * kXfragSbBytes +
                       (size_t)usb * 512 * sum_tiles(p.nt);
  const size_t y_bytes = (size_t)(p.nt >= 4 ? 32 : 16) * 128 * sizeof(float);
  p.stages = usb == 1 ? 8 : 4;
  while (p.stages > 2 && p.stages * stage + y_bytes > kGemvSmemBudget) --p.stages;
  p.smem = p.stages * stage + y_bytes;
  // row-group segments: a group of ppr units spans at most ceil(ppr * grid / units) + 1 CTA ranges
  const long long ppr = (s.sb + usb - 1) / usb;
  p.ksplit = (int)((ppr * p.grid + units - 1) / units + 1);
  p.xfrag_bytes = (uint64_t)p.nt * s.sb * kXfragSbBytes;
  p.xs_bytes = 0;
  return p;
}

int launch_repack(const GemvShape& s, const uint8_t* d_src, uint8_t* d_tiles, cudaStream_t st, uint32_t half_rows) {
  const uint64_t tiles = (uint64_t)s.ng * s.sb * kGemvWarps;
  const uint64_t items = tiles * (s.quant == CLM_QUANT_Q4_K ? 528 : 1152);
  const uint64_t blocks = ceil_div(items, 256);
  CLM_CHECK(blocks < (1ull << 31), CLM_RESOURCE_EXHAUSTED, "matrix too large to repack");
  if (s.quant == CLM_QUANT_Q4_K)
    repack_q4k_kernel<<<(unsigned)blocks, 256, 0, st>>>(d_src, d_tiles, s.rows, s.sb, s.ng, half_rows);
  else
    repack_q80_kernel<<<(unsigned)blocks, 256, 0, st>>>(d_src, d_tiles, s.rows, s.sb, s.ng, half_rows);
  CLM_LAUNCHED("repack");
  return CLM_OK;
}

}  // namespace clm
