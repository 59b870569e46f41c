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
// activation staging
// ---------------------------------------------------------------------------------------------------
// xfrag[sb][nt][s][lane] = {half2(x[p][k0], x[p][k0+1]), half2(x[p][k1], x[p][k1+1]) * hi_scale}
//   p = nt*8 + lane/4, k0 = 256 sb + 64 t + 2 s, k1 = k0 + 32, t = lane%4
// xs[pair][nt][lane] = {hi(sum sb0 sub 2t, 2t+1), hi(sum sb1 ...), lo(...), lo(...)}
// (superblock-major, so one CTA's k-range is one contiguous span of each array)
__global__ void prep_x_kernel(const float* __restrict__ x, int q, uint32_t cols, uint32_t sb_per_row, int nt_count,
                              float hi_scale, uint2* __restrict__ xfrag, uint4* __restrict__ xs) {
  const uint32_t n_frag = (uint32_t)nt_count * sb_per_row * 512;
  const uint32_t pairs = (sb_per_row + 1) / 2;
  const uint32_t n_xs = (uint32_t)nt_count * pairs * 32;
  const uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x;
  griddep_wait();
  griddep_launch();
  if (gid < n_frag) {
    const uint32_t lane = gid % 32, s = (gid / 32) % 16, nt = (gid / 512) % nt_count, sb = gid / (512 * nt_count);
    const int p = (int)nt * 8 + (int)(lane / 4);
    const uint32_t t = lane % 4;
    uint2 v = make_uint2(0, 0);
    if (p < q) {
      const float* xr = x + (size_t)p * cols;
      const uint32_t k0 = sb * 256 + 64 * t + 2 * s, k1 = k0 + 32;
      v.x = pack_half2(xr[k0], xr[k0 + 1]);
      v.y = pack_half2(xr[k1] * hi_scale, xr[k1 + 1] * hi_scale);
    }
    xfrag[gid] = v;
  } else if (gid < n_frag + n_xs) {
    const uint32_t i = gid - n_frag;
    const uint32_t lane = i % 32, nt = (i / 32) % nt_count, pr = i / (32 * nt_count);
    const int p = (int)nt * 8 + (int)(lane / 4);
    const uint32_t t = lane % 4;
    float sums[4] = {0, 0, 0, 0};  // sb0 sub 2t, sb0 sub 2t+1, sb1 sub 2t, sb1 sub 2t+1
    if (p < q) {
      const float* xr = x + (size_t)p * cols;
      for (int h = 0; h < 2; ++h) {
        const uint32_t sb = 2 * pr + h;
        if (sb >= sb_per_row) continue;
        for (int e = 0; e < 2; ++e) {
          const uint32_t k = sb * 256 + 32 * (2 * t + e);
          float a = 0.0f;
          for (int l = 0; l < 32; ++l) a += xr[k + l];
          sums[2 * h + e] = a;
        }
      }
    }
    uint4 v;
    float hi[4], lo[4];
    for (int i2 = 0; i2 < 4; ++i2) {
      hi[i2] = __half2float(__float2half_rn(sums[i2]));
      lo[i2] = sums[i2] - hi[i2];
    }
    v.x = pack_half2(hi[0], hi[1]);
    v.y = pack_half2(hi[2], hi[3]);
    v.z = pack_half2(lo[0], lo[1]);
    v.w = pack_half2(lo[2], lo[3]);
    xs[i] = v;
  }
}

template <typename Raw, int NT>
__global__ void __launch_bounds__(256) gemv_tiled_kernel(const uint8_t* __restrict__ tiles, uint32_t rows,
                                                        uint32_t sb_per_row, int tile_bytes, int ksplit, int sbps,
                                                        const uint2* __restrict__ xfrag,
                                                        const uint4* __restrict__ xsg, int q,
                                                        float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int grp = blockIdx.x / ksplit, ks = blockIdx.x % ksplit;
  const int sb0 = ks * sbps;
  const int sb1 = min((int)sb_per_row, sb0 + sbps);
  const int nsb = sb1 - sb0;
  const int pairs_local = (nsb + 1) / 2;
  uint2* xf = reinterpret_cast<uint2*>(smem);
  uint4* xs = reinterpret_cast<uint4*>(smem + (size_t)NT * nsb * kXfragSbBytes);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, t = lane % 4, g = lane / 4;
  const uint8_t* tile0 = tiles + ((size_t)(grp * sb_per_row + sb0) * kGemvWarps + warp) * tile_bytes;
  const size_t sb_stride = (size_t)kGemvWarps * tile_bytes;

  // Issue the first weight loads before waiting for the producer of the activations (weights are immutable).
  Raw cur, nxt;
  load_raw(cur, tile0, lane);
  griddep_wait();
  griddep_launch();

  // Stage this CTA's activation fragments (one contiguous span each; sb0 is even).
  {
    const uint4* src = reinterpret_cast<const uint4*>(xfrag + (size_t)sb0 * NT * 512);
    uint4* dst = reinterpret_cast<uint4*>(xf);
    for (int i = threadIdx.x; i < nsb * NT * 256; i += blockDim.x) dst[i] = __ldg(src + i);
    const uint4* xsrc = xsg + (size_t)(sb0 / 2) * NT * 32;
    for (int i = threadIdx.x; i < pairs_local * NT * 32; i += blockDim.x) xs[i] = __ldg(xsrc + i);
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;

  for (int i = 0; i < nsb; i += 2) {
    uint32_t m0g, m0g8, m1g = 0, m1g8 = 0;
    if (i + 1 < nsb) load_raw(nxt, tile0 + (i + 1) * sb_stride, lane);
    tile_mmas<NT>(cur, t, xf + (size_t)i * NT * 512, lane, acc, m0g, m0g8);
    if (i + 1 < nsb) {
      if (i + 2 < nsb) load_raw(cur, tile0 + (i + 2) * sb_stride, lane);
      tile_mmas<NT>(nxt, t, xf + (size_t)(i + 1) * NT * 512, lane, acc, m1g, m1g8);
    }
    min_mma<NT>(acc, m0g, m0g8, m1g, m1g8, xs, i / 2, lane);
  }

  const uint32_t row_base = (uint32_t)(grp * kGemvWarps + warp) * 16;
  float* o = out + (size_t)ks * q * rows;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int p0 = nt * 8 + 2 * t;
    const uint32_t r0 = row_base + g, r1 = row_base + g + 8;
    if (p0 < q) {
      if (r0 < rows) o[(size_t)p0 * rows + r0] = acc[nt][0];
      if (r1 < rows) o[(size_t)p0 * rows + r1] = acc[nt][2];
    }
    if (p0 + 1 < q) {
      if (r0 < rows) o[(size_t)(p0 + 1) * rows + r0] = acc[nt][1];
      if (r1 < rows) o[(size_t)(p0 + 1) * rows + r1] = acc[nt][3];
    }
  }
}

__global__ void reduce_splits_kernel(const float* __restrict__ part, int ksplit, uint64_t n, float* __restrict__ y) {
  griddep_wait();
  griddep_launch();
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float a = 0.0f;
    for (int k = 0; k < ksplit; ++k) a += part[(uint64_t)k * n + i];
    y[i] = a;
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
  GemvPlan p;
  p.nt = q <= 8 ? 1 : 2;
  const int cap = p.nt == 1 ? 22 : 10;  // superblocks of staged activations per CTA (~100 KB)
  const int target = 2 * (sm_count > 0 ? sm_count : 148);
  const int sb = (int)s.sb;
  int best_split = 1, best_sbps = sb + (sb & 1);
  for (int ks = 1; ks <= sb; ++ks) {
    int sbps = (sb + ks - 1) / ks;
    sbps += sbps & 1;
    const int splits = (sb + sbps - 1) / sbps;
    best_split = splits;
    best_sbps = sbps;
    if (sbps > cap) continue;
    if ((long)s.ng * splits >= target || sbps <= 2) break;
  }
  p.ksplit = best_split;
  p.sbps = best_sbps;
  const int pairs_local = (p.sbps + 1) / 2;
  p.smem = (size_t)p.nt * p.sbps * kXfragSbBytes + (size_t)p.nt * pairs_local * kXsPairBytes;
  p.xfrag_bytes = (uint64_t)p.nt * s.sb * kXfragSbBytes;
  p.xs_bytes = (uint64_t)p.nt * ((s.sb + 1) / 2) * kXsPairBytes;
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

int launch_prep_x(const GemvShape& s, const GemvPlan& p, const float* d_x, int q, void* d_xfrag, void* d_xs,
                  cudaStream_t st) {
  const uint32_t n = (uint32_t)p.nt * s.sb * 512 + (uint32_t)p.nt * ((s.sb + 1) / 2) * 32;
  const float hi_scale = s.quant == CLM_QUANT_Q4_K ? 0.0625f : 1.0f;
  return launch_pdl(prep_x_kernel, dim3((n + 255) / 256), dim3(256), 0, st, d_x, q, s.cols, s.sb, p.nt, hi_scale,
                    static_cast<uint2*>(d_xfrag), static_cast<uint4*>(d_xs));
}

template <typename Raw, int NT>
static int launch_gemv_t(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const void* d_xfrag,
                         const void* d_xs, int q, float* d_out, cudaStream_t st) {
  auto kern = gemv_tiled_kernel<Raw, NT>;
  CLM_TRY(ensure_smem(kern, p.smem));
  const unsigned blocks = s.ng * (unsigned)p.ksplit;
  return launch_pdl(kern, dim3(blocks), dim3(256), p.smem, st, d_tiles, s.rows, s.sb, s.tile_bytes, p.ksplit, p.sbps,
                    static_cast<const uint2*>(d_xfrag), static_cast<const uint4*>(d_xs), q, d_out);
}

int launch_gemv(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const void* d_xfrag, const void* d_xs,
                int q, float* d_out, cudaStream_t st) {
  if (s.quant == CLM_QUANT_Q4_K)
    return p.nt == 1 ? launch_gemv_t<RawQ4k, 1>(s, p, d_tiles, d_xfrag, d_xs, q, d_out, st)
                     : launch_gemv_t<RawQ4k, 2>(s, p, d_tiles, d_xfrag, d_xs, q, d_out, st);
  return p.nt == 1 ? launch_gemv_t<RawQ80, 1>(s, p, d_tiles, d_xfrag, d_xs, q, d_out, st)
                   : launch_gemv_t<RawQ80, 2>(s, p, d_tiles, d_xfrag, d_xs, q, d_out, st);
}

int launch_reduce_splits(const float* d_part, int ksplit, int q, uint32_t rows, float* d_y, cudaStream_t st) {
  const uint64_t n = (uint64_t)q * rows;
  const uint64_t blocks = std::min<uint64_t>(ceil_div(n, 256), 4096);
  return launch_pdl(reduce_splits_kernel, dim3((unsigned)blocks), dim3(256), 0, st, d_part, ksplit, n, d_y);
}

}  // namespace clm
