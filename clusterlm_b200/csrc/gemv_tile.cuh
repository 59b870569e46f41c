// gemv_tile.cuh — device building blocks of the tiled fused-dequant GEMV (see gemv.cuh for the design):
// fp16x2 helpers, per-tile register images, scale decoding and the per-tile mma sequences.
#pragma once
#include "gemv.cuh"

namespace clm {

// ---------------------------------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------------------------------
static __device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
static __device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
static __device__ __forceinline__ void mma16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// (a & MASK) | c in one LOP3 (c held in a register, so the mask can be the instruction's immediate).
template <uint32_t MASK>
static __device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "n"(MASK), "r"(c));
  return d;
}
static __device__ __forceinline__ uint32_t lo_bcast(uint32_t x) { return __byte_perm(x, x, 0x1010); }
static __device__ __forceinline__ uint32_t hi_bcast(uint32_t x) { return __byte_perm(x, x, 0x3232); }

static constexpr uint32_t kHalfNeg1024x2 = 0xE400E400u;
static constexpr uint32_t kHalfNeg128x2 = 0xD800D800u;
static constexpr uint32_t kMagic = 0x64006400u;  // fp16 pair (1024, 1024)

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

static __device__ __forceinline__ void load_raw(RawQ4k& r, const uint8_t* tile, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(tile);
#pragma unroll
  for (int j = 0; j < 4; ++j) r.q[j] = __ldg(p + j * 32 + lane);
  const int g = lane / 4;
  r.rg = __ldg(reinterpret_cast<const uint4*>(tile + 2048 + 16 * g));
  r.rg8 = __ldg(reinterpret_cast<const uint4*>(tile + 2048 + 16 * (g + 8)));
}
static __device__ __forceinline__ void load_raw(RawQ80& r, const uint8_t* tile, int lane) {
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

// Raw tile image from shared memory (the bulk-copied k-chunk); same lane mapping as load_raw.
static __device__ __forceinline__ void load_raw_s(RawQ4k& r, const uint8_t* tile, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(tile);
#pragma unroll
  for (int j = 0; j < 4; ++j) r.q[j] = p[j * 32 + lane];
  const int g = lane / 4;
  r.rg = *reinterpret_cast<const uint4*>(tile + 2048 + 16 * g);
  r.rg8 = *reinterpret_cast<const uint4*>(tile + 2048 + 16 * (g + 8));
}
static __device__ __forceinline__ void load_raw_s(RawQ80& r, const uint8_t* tile, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(tile);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r.q[2 * j] = p[j * 64 + lane * 2];
    r.q[2 * j + 1] = p[j * 64 + lane * 2 + 1];
  }
  const int g = lane / 4, t = lane % 4;
  r.sg = *reinterpret_cast<const uint32_t*>(tile + 4096 + 16 * g + 4 * t);
  r.sg8 = *reinterpret_cast<const uint32_t*>(tile + 4096 + 16 * (g + 8) + 4 * t);
}

static __device__ __forceinline__ uint32_t q4k_entries(const uint4& r, int t) {
  const uint32_t a = t < 2 ? r.y : (t == 2 ? r.z : r.w);
  const uint32_t b = t < 2 ? r.z : (t == 2 ? r.w : 0u);
  return __funnelshift_r(a, b, (24 * t) & 31) & 0xFFFFFFu;
}

// Per-row dequant constants: sA/sB = scale broadcast for sub-blocks 2t / 2t+1, nA/nB = -1024 * scale,
// negm = (-m(2t), -m(2t+1)) for the min mma.
struct RowDq {
  uint32_t sA, sB, nA, nB, negm;
};

static __device__ __forceinline__ RowDq q4k_row(const uint4& r, int t) {
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

static __device__ __forceinline__ RowDq q80_row(uint32_t S) {
  RowDq o;
  o.sA = lo_bcast(S);
  o.sB = hi_bcast(S);
  o.nA = hmul2u(o.sA, kHalfNeg1024x2);
  o.nB = hmul2u(o.sB, kHalfNeg1024x2);
  o.negm = hmul2u(S, kHalfNeg128x2);  // the unsigned view adds 128 per byte: subtract 128*s*sum(x)
  return o;
}

// acc[s & 1]: even and odd k-steps accumulate into separate registers, two independent mma chains.
template <int NT>
static __device__ __forceinline__ void tile_mmas(const RawQ4k& r, int t, const uint2* __restrict__ xf, int lane,
                                          float (&acc)[2][NT][4], uint32_t& negm_g, uint32_t& negm_g8) {
  const RowDq dg = q4k_row(r.rg, t), dg8 = q4k_row(r.rg8, t);
  negm_g = dg.negm;
  negm_g8 = dg8.negm;
  uint32_t magic;  // the exponent pattern in a register: each nibble pair is then one LOP3
  asm volatile("mov.b32 %0, %1;" : "=r"(magic) : "n"(kMagic));
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const uint4& qq = r.q[s / 4];
    const uint32_t w = (s % 4 == 0) ? qq.x : (s % 4 == 1) ? qq.y : (s % 4 == 2) ? qq.z : qq.w;
    const uint32_t w8 = w >> 8;
    const uint32_t a0 = hfma2u(and_or<0x000F000Fu>(w, magic), dg.sA, dg.nA);
    const uint32_t a1 = hfma2u(and_or<0x000F000Fu>(w8, magic), dg8.sA, dg8.nA);
    const uint32_t a2 = hfma2u(and_or<0x00F000F0u>(w, magic), dg.sB, dg.nB);
    const uint32_t a3 = hfma2u(and_or<0x00F000F0u>(w8, magic), dg8.sB, dg8.nB);
    if (NT >= 4) {
      // 4 n-tiles, interleaved in pairs: one 16-byte load per pair; the chains are already independent, so one
      // accumulator set (registers for the 32-row GEMV)
      const uint4* xf4 = reinterpret_cast<const uint4*>(xf);
#pragma unroll
      for (int pr = 0; pr < NT / 2; ++pr) {
        const uint4 b = xf4[(pr * 16 + s) * 32 + lane];
        mma16816(acc[0][2 * pr], a0, a1, a2, a3, b.x, b.y);
        mma16816(acc[0][2 * pr + 1], a0, a1, a2, a3, b.z, b.w);
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b = xf[(nt * 16 + s) * 32 + lane];
        mma16816(acc[s & 1][nt], a0, a1, a2, a3, b.x, b.y);
      }
    }
  }
}

template <int NT>
static __device__ __forceinline__ void tile_mmas(const RawQ80& r, int t, const uint2* __restrict__ xf, int lane,
                                          float (&acc)[2][NT][4], uint32_t& negm_g, uint32_t& negm_g8) {
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
    if (NT >= 4) {
      const uint4* xf4 = reinterpret_cast<const uint4*>(xf);
#pragma unroll
      for (int pr = 0; pr < NT / 2; ++pr) {
        const uint4 b = xf4[(pr * 16 + s) * 32 + lane];
        mma16816(acc[0][2 * pr], a0, a1, a2, a3, b.x, b.y);
        mma16816(acc[0][2 * pr + 1], a0, a1, a2, a3, b.z, b.w);
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b = xf[(nt * 16 + s) * 32 + lane];
        mma16816(acc[s & 1][nt], a0, a1, a2, a3, b.x, b.y);
      }
    }
  }
}


}  // namespace clm
