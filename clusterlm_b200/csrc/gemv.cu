// gemv.cu — repack, activation staging and the tiled fused-dequant GEMV (see gemv.cuh for the design).
#include <algorithm>

#include "gemv.cuh"
#include "pdl.cuh"

namespace clm {

// ---------------------------------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void mma16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t lo_bcast(uint32_t x) { return __byte_perm(x, x, 0x1010); }
__device__ __forceinline__ uint32_t hi_bcast(uint32_t x) { return __byte_perm(x, x, 0x3232); }

constexpr uint32_t kHalfNeg1024x2 = 0xE400E400u;
constexpr uint32_t kHalfNeg128x2 = 0xD800D800u;
constexpr uint32_t kMagic = 0x64006400u;  // fp16 pair (1024, 1024)

// ---------------------------------------------------------------------------------------------------
// repack: GGUF row-major blocks -> fragment-ordered tiles
// ---------------------------------------------------------------------------------------------------
// One thread per output 32-bit word of a tile's quant region, plus the scale records.
__global__ void repack_q4k_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint32_t rows,
                                  uint32_t sb_per_row, uint32_t ng) {
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
                                  uint32_t sb_per_row, uint32_t ng) {
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

// ---------------------------------------------------------------------------------------------------
// the GEMV kernel
// ---------------------------------------------------------------------------------------------------
struct RawQ4k {
  uint4 q[4];
  uint4 rg, rg8;
};
struct RawQ80 {
  uint4 q[8];
  uint32_t sg, sg8;
};

__device__ __forceinline__ void load_raw(RawQ4k& r, const uint8_t* tile, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(tile);
#pragma unroll
  for (int j = 0; j < 4; ++j) r.q[j] = __ldg(p + j * 32 + lane);
  const int g = lane / 4;
  r.rg = __ldg(reinterpret_cast<const uint4*>(tile + 2048 + 16 * g));
  r.rg8 = __ldg(reinterpret_cast<const uint4*>(tile + 2048 + 16 * (g + 8)));
}
__device__ __forceinline__ void load_raw(RawQ80& r, const uint8_t* tile, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(tile);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r.q[2 * j] = __ldg(p + j * 64 + lane * 2);
    r.q[2 * j + 1] = __ldg(p + j * 64 + lane * 2 + 1);
  }
  const int g = lane / 4, t = lane % 4;
  r.sg = __ldg(reinterpret_cast<const uint32_t*>(tile + 4096 + 16 * g + 4 * t));
  r.sg8 = __ldg(reinterpret_cast<const uint32_t*>(tile + 4096 + 16 * (g + 8) + 4 * t));
}

__device__ __forceinline__ uint32_t q4k_entries(const uint4& r, int t) {
  const uint32_t a = t < 2 ? r.y : (t == 2 ? r.z : r.w);
  const uint32_t b = t < 2 ? r.z : (t == 2 ? r.w : 0u);
  return __funnelshift_r(a, b, (24 * t) & 31) & 0xFFFFFFu;
}

// Per-row dequant constants: sA/sB = scale broadcast for sub-blocks 2t / 2t+1, nA/nB = -1024 * scale,
// negm = (-m(2t), -m(2t+1)) for the min mma.
struct RowDq {
  uint32_t sA, sB, nA, nB, negm;
};

__device__ __forceinline__ RowDq q4k_row(const uint4& r, int t) {
  const uint32_t v = q4k_entries(r, t);
  const uint32_t e0 = v & 0xFFFu, e1 = v >> 12;
  const uint32_t scw = kMagic | (e0 & 63u) | ((e1 & 63u) << 16);
  const uint32_t mw = kMagic | (e0 >> 6) | ((e1 >> 6) << 16);
  const uint32_t d2 = lo_bcast(r.x), dm2 = hi_bcast(r.x);
  const uint32_t S = hfma2u(scw, d2, hmul2u(d2, kHalfNeg1024x2));            // (d*sc_a, d*sc_b)
  const uint32_t negdm2 = dm2 ^ 0x80008000u;
  const uint32_t negM = hfma2u(mw, negdm2, hmul2u(negdm2, kHalfNeg1024x2));  // -(dmin*m_a), -(dmin*m_b)
  RowDq o;
  o.sA = lo_bcast(S);
  o.sB = hi_bcast(S);
  o.nA = hmul2u(o.sA, kHalfNeg1024x2);
  o.nB = hmul2u(o.sB, kHalfNeg1024x2);
  o.negm = negM;
  return o;
}

__device__ __forceinline__ RowDq q80_row(uint32_t S) {
  RowDq o;
  o.sA = lo_bcast(S);
  o.sB = hi_bcast(S);
  o.nA = hmul2u(o.sA, kHalfNeg1024x2);
  o.nB = hmul2u(o.sB, kHalfNeg1024x2);
  o.negm = hmul2u(S, kHalfNeg128x2);  // the unsigned view adds 128 per byte: subtract 128*s*sum(x)
  return o;
}

template <int NT>
__device__ __forceinline__ void tile_mmas(const RawQ4k& r, int t, const uint2* __restrict__ xf, int lane,
                                          float (&acc)[NT][4], uint32_t& negm_g, uint32_t& negm_g8) {
  const RowDq dg = q4k_row(r.rg, t), dg8 = q4k_row(r.rg8, t);
  negm_g = dg.negm;
  negm_g8 = dg8.negm;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const uint4& qq = r.q[s / 4];
    const uint32_t w = (s % 4 == 0) ? qq.x : (s % 4 == 1) ? qq.y : (s % 4 == 2) ? qq.z : qq.w;
    const uint32_t w8 = w >> 8;
    const uint32_t a0 = hfma2u((w & 0x000F000Fu) | kMagic, dg.sA, dg.nA);
    const uint32_t a1 = hfma2u((w8 & 0x000F000Fu) | kMagic, dg8.sA, dg8.nA);
    const uint32_t a2 = hfma2u((w & 0x00F000F0u) | kMagic, dg.sB, dg.nB);
    const uint32_t a3 = hfma2u((w8 & 0x00F000F0u) | kMagic, dg8.sB, dg8.nB);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint2 b = xf[(nt * 16 + s) * 32 + lane];
      mma16816(acc[nt], a0, a1, a2, a3, b.x, b.y);
    }
  }
}

template <int NT>
__device__ __forceinline__ void tile_mmas(const RawQ80& r, int t, const uint2* __restrict__ xf, int lane,
                                          float (&acc)[NT][4], uint32_t& negm_g, uint32_t& negm_g8) {
  const RowDq dg = q80_row(r.sg), dg8 = q80_row(r.sg8);
  negm_g = dg.negm;
  negm_g8 = dg8.negm;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const uint4& qq = r.q[2 * (s / 4) + (s % 4) / 2];
    const uint32_t w0 = ((s % 2) == 0 ? qq.x : qq.z) ^ 0x80808080u;
    const uint32_t w1 = ((s % 2) == 0 ? qq.y : qq.w) ^ 0x80808080u;
    const uint32_t a0 = hfma2u(__byte_perm(w0, 0x64646464u, 0x4140), dg.sA, dg.nA);
    const uint32_t a1 = hfma2u(__byte_perm(w0, 0x64646464u, 0x4342), dg8.sA, dg8.nA);
    const uint32_t a2 = hfma2u(__byte_perm(w1, 0x64646464u, 0x4140), dg.sB, dg.nB);
    const uint32_t a3 = hfma2u(__byte_perm(w1, 0x64646464u, 0x4342), dg8.sB, dg8.nB);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint2 b = xf[(nt * 16 + s) * 32 + lane];
      mma16816(acc[nt], a0, a1, a2, a3, b.x, b.y);
    }
  }
}

// xs points at the CTA's staged sub-block sums, layout [pair][nt][lane].
template <int NT>
__device__ __forceinline__ void min_mma(float (&acc)[NT][4], uint32_t m0g, uint32_t m0g8, uint32_t m1g, uint32_t m1g8,
                                        const uint4* __restrict__ xs, int pl, int lane) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint4 v = xs[(pl * NT + nt) * 32 + lane];
    mma16816(acc[nt], m0g, m0g8, m1g, m1g8, v.x, v.y);
    mma16816(acc[nt], m0g, m0g8, m1g, m1g8, v.z, v.w);
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

int launch_repack(const GemvShape& s, const uint8_t* d_src, uint8_t* d_tiles, cudaStream_t st) {
  const uint64_t tiles = (uint64_t)s.ng * s.sb * kGemvWarps;
  const uint64_t items = tiles * (s.quant == CLM_QUANT_Q4_K ? 528 : 1152);
  const uint64_t blocks = ceil_div(items, 256);
  CLM_CHECK(blocks < (1ull << 31), CLM_RESOURCE_EXHAUSTED, "matrix too large to repack");
  if (s.quant == CLM_QUANT_Q4_K)
    repack_q4k_kernel<<<(unsigned)blocks, 256, 0, st>>>(d_src, d_tiles, s.rows, s.sb, s.ng);
  else
    repack_q80_kernel<<<(unsigned)blocks, 256, 0, st>>>(d_src, d_tiles, s.rows, s.sb, s.ng);
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
