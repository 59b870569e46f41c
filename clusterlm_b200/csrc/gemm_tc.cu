// gemm_tc.cu — wide-window dequantising GEMM on the 5th-generation tensor cores (tcgen05 / TMEM), sm_100a.
//
// Y[p][n] = W[n] . X[p] for p < P window rows (17 <= P <= 256: tree windows of several sequences, prefill chunks),
// W in GGUF Q4_K / Q8_0, repacked in the group-major tile layout of gemv.cuh.  The q <= 16 windows use the
// bandwidth-bound q-row GEMV (gemv4.cu); from P > 16 on the tensor-core work per weight byte grows with P and the
// tcgen05 path takes over:
//
//  * A first kernel converts the window's activations (f32) to fp16 tiles already in the MMA's layout (K-major,
//    128-byte swizzle: 8-row atoms of 1024 B, 16-byte chunk c of row r stored at chunk c ^ (r % 8)), one
//    P x 64 tile per 64-column chunk.
//  * Grid (row group of 128 weight rows, K split).  A CTA walks its K range in chunks of KC = 128 columns (64 when
//    two 128-column stages do not fit next to the raw ring, i.e. above 128 window rows): every stage hands the MMA
//    warp KC / 64 swizzled 64-column A and B tiles at once, which halves the per-stage hand-offs that bound this
//    kernel (a dequantising warp spends a fixed ~0.25 us between stages).  Warp 9 bulk-copies (cp.async.bulk, no
//    multicast) the group's raw superblocks (8 repacked tiles, issued before griddepcontrol.wait) into a 2-slot
//    ring and each chunk's activation tiles (contiguous in xh) into the chunk's stage.  For every chunk eight warps
//    dequantise the group's 128 x KC weights (row tile w of warp w) from the staged superblock into the stage's fp16
//    A tiles, in the same swizzled layout.  Up to four stages keep the copies and the dequantisation ahead of the
//    MMAs.
//  * Warp 8 owns the accumulator: it allocates P (rounded up to a power of two, >= 32) TMEM columns, and one of
//    its lanes issues the KC / 16 K = 16 tcgen05.mma.cta_group::1.kind::f16 (M = 128 weight rows, N = P window
//    rows, f32 accumulate in TMEM) per chunk once the stage's "full" mbarrier has the eight warps' arrivals and
//    the activation tile's bytes, then
//    tcgen05.commit releases the stage ("free" mbarrier) when those MMAs have read it.
//  * After the last chunk a commit on the "done" mbarrier hands the accumulator to the epilogue: warp w reads TMEM
//    lanes 32 (w % 4) .. +31 (its weight rows) and half of the columns with tcgen05.ld and stores the f32 partial
//    of its K range; a second kernel sums the K splits in split order (deterministic) into Y.
//  * Every mbarrier wait is bounded (bulk.cuh) and records an error instead of hanging; the TMEM columns are
//    freed by the CTA that allocated them on every path.
//
// Weights are dequantised as GGUF decodes them (Q4_K: q * (d*sc) - dmin*m, Q8_0: q * d), rounded to fp16 once
// (d*sc and dmin*m are themselves fp16); the activations are rounded to fp16; products accumulate in f32.
#include <cstdlib>

#include "bulk.cuh"
#include "gemm_tc.cuh"
#include "gemv_tile.cuh"
#include "pdl.cuh"

namespace clm {

namespace {

constexpr int kTcWarps = 8;                      // dequant / epilogue warps
constexpr int kTcThreads = 32 * (kTcWarps + 2);  // + the MMA warp + the copy warp
constexpr int kTcMaxStages = 4;
constexpr int kTcRawSlots = 2;                   // raw superblock stages (8 repacked tiles each)
constexpr int kTcKc = 64;                     // columns per chunk (one 128-byte swizzle row of fp16)
constexpr uint32_t kATileBytes = 128 * kTcKc * 2;  // 16 KB

// Byte offset of element chunk (row r, 16-byte chunk c) in a K-major SW128 tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return tc_tile_off(r, c); }

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 B apart (SBO), LBO unused (1).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address
  d |= (uint64_t)1u << 16;                          // leading byte offset (16-byte units), unused for SW128 K-major
  d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset: next 8-row atom
  d |= (uint64_t)1u << 46;                          // descriptor version (sm100)
  d |= (uint64_t)2u << 61;                          // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16: A, B fp16 (K-major), D f32, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
constexpr uint32_t kMagic1152 = 0x64806480u;  // fp16 pair (1152, 1152) = 1024 + 128

// fp16 pairs of 8 consecutive weights of one row, two sub-blocks: `lo` for columns [8q, 8q+8) of the chunk's
// first sub-block, `hi` for the same columns of the second.
struct Dq8 {
  uint4 lo, hi;
};

// Q4_K: the thread's four nibble words (k-steps 4q..4q+3 of the quarter j of the superblock) for rows g and g+8,
// from the tile staged in shared memory.
__device__ __forceinline__ void dq_q4k(const uint8_t* tile, int j, int g, int qq, Dq8& r0, Dq8& r8) {
  const uint4 raw = lds128(tile + (size_t)(qq * 32 + 4 * g + j) * 16);
  const uint4 rg = lds128(tile + 2048 + 16 * g), rg8 = lds128(tile + 2048 + 16 * (g + 8));
  const RowDq d = q4k_row(rg, j), d8 = q4k_row(rg8, j);
  const uint32_t mA = lo_bcast(d.negm), mB = hi_bcast(d.negm), mA8 = lo_bcast(d8.negm), mB8 = hi_bcast(d8.negm);
  uint32_t magic;
  asm volatile("mov.b32 %0, %1;" : "=r"(magic) : "n"(kMagic));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o0[4], o1[4], o8[4], o9[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t x = w[s], x4 = x >> 4, x8 = x >> 8, x12 = x >> 12;
    // q exactly (1024 + q - 1024), then q * (d*sc) - dmin*m with one rounding
    o0[s] = hfma2u(hsub2u(and_or<0x000F000Fu>(x, magic), kMagic), d.sA, mA);
    o1[s] = hfma2u(hsub2u(and_or<0x000F000Fu>(x4, magic), kMagic), d.sB, mB);
    o8[s] = hfma2u(hsub2u(and_or<0x000F000Fu>(x8, magic), kMagic), d8.sA, mA8);
    o9[s] = hfma2u(hsub2u(and_or<0x000F000Fu>(x12, magic), kMagic), d8.sB, mB8);
  }
  r0.lo = make_uint4(o0[0], o0[1], o0[2], o0[3]);
  r0.hi = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  r8.lo = make_uint4(o8[0], o8[1], o8[2], o8[3]);
  r8.hi = make_uint4(o9[0], o9[1], o9[2], o9[3]);
}

// Q8_0: the thread's eight int8 words (k-steps 4q..4q+3, blocks 2j and 2j+1) for rows g and g+8, from shared
// memory.
__device__ __forceinline__ void dq_q80(const uint8_t* tile, int j, int g, int qq, Dq8& r0, Dq8& r8) {
  const uint8_t* base = tile + (size_t)(qq * 256 + (4 * g + j) * 8) * 4;
  const uint4 a = lds128(base), b = lds128(base + 16);
  const uint32_t sg = *reinterpret_cast<const uint32_t*>(tile + 4096 + 16 * g + 4 * j);
  const uint32_t sg8 = *reinterpret_cast<const uint32_t*>(tile + 4096 + 16 * (g + 8) + 4 * j);
  const uint32_t sA = lo_bcast(sg), sB = hi_bcast(sg), sA8 = lo_bcast(sg8), sB8 = hi_bcast(sg8);
  // words in order (s, e): a = {(0,0),(0,1),(1,0),(1,1)}, b = {(2,0),(2,1),(3,0),(3,1)}
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t o0[4], o1[4], o8[4], o9[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t x0 = w[2 * s] ^ 0x80808080u, x1 = w[2 * s + 1] ^ 0x80808080u;
    // the signed byte exactly (1024 + (b + 128) - 1152), then b * d with one rounding
    o0[s] = hmul2u(hsub2u(__byte_perm(x0, 0x64646464u, 0x4140), kMagic1152), sA);
    o8[s] = hmul2u(hsub2u(__byte_perm(x0, 0x64646464u, 0x4342), kMagic1152), sA8);
    o1[s] = hmul2u(hsub2u(__byte_perm(x1, 0x64646464u, 0x4140), kMagic1152), sB);
    o9[s] = hmul2u(hsub2u(__byte_perm(x1, 0x64646464u, 0x4342), kMagic1152), sB8);
  }
  r0.lo = make_uint4(o0[0], o0[1], o0[2], o0[3]);
  r0.hi = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  r8.lo = make_uint4(o8[0], o8[1], o8[2], o8[3]);
  r8.hi = make_uint4(o9[0], o9[1], o9[2], o9[3]);
}

// x (q x K f32) -> fp16 activation tiles in the MMA's layout: [K / 64 chunks][P rows, SW128 K-major], rows >= q zero,
// so that each chunk's B tile is one contiguous bulk copy.
__global__ void tc_xprep_kernel(const float* __restrict__ x, int q, int K, int P, uint8_t* __restrict__ xh) {
  griddep_wait();
  griddep_launch();
  const uint64_t n = (uint64_t)(K / kTcKc) * P * 8;  // 16-byte chunks
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const int ch = (int)(i % 8), p = (int)((i / 8) % P), c = (int)(i / ((uint64_t)8 * P));
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (p < q) {
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)p * K + (size_t)c * kTcKc + 8 * ch);
      const float4 u0 = __ldg(src), u1 = __ldg(src + 1);
      v = make_uint4(pack_half2(u0.x, u0.y), pack_half2(u0.z, u0.w), pack_half2(u1.x, u1.y), pack_half2(u1.z, u1.w));
    }
    *reinterpret_cast<uint4*>(xh + (size_t)c * P * 128 + sw128_off(p, ch)) = v;
  }
}

template <int QUANT, int KC>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const uint8_t* __restrict__ tiles, int sb_count,
                                                                 int tile_bytes, const uint8_t* __restrict__ xh, int q,
                                                                 int K, int P, int ksplit, int stages,
                                                                 float* __restrict__ part, uint32_t rows_total,
                                                                 int* __restrict__ err, int ahead) {
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  __shared__ __align__(8) uint64_t full[kTcMaxStages], freeb[kTcMaxStages], raw_full[kTcRawSlots],
      raw_free[kTcRawSlots], done;
  __shared__ uint32_t s_tmem;
  // 1024-byte aligned area (the dynamic allocation carries 1 KB of slack): [stages x (A tile, B tile)][raw slots]
  uint8_t* tc_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int SUB = KC / kTcKc;  // 64-column tiles per stage
  constexpr int CPS = 256 / KC;    // stages per raw superblock
  const uint32_t btile = (uint32_t)P * 128u * SUB;
  const uint32_t atile = kATileBytes * SUB;
  const uint32_t stage_bytes = atile + btile;
  const uint32_t raw_bytes = (uint32_t)kGemvWarps * (uint32_t)tile_bytes;
  uint8_t* raw_base = tc_smem + (size_t)stages * stage_bytes;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int grp = blockIdx.x, split = blockIdx.y;
  const int chunks = K / KC;
  const int c0 = split * chunks / ksplit, c1 = (split + 1) * chunks / ksplit;
  const int ncols = P <= 32 ? 32 : (P <= 64 ? 64 : (P <= 128 ? 128 : 256));

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], kTcWarps + 1);  // eight dequant warps + the copy warp's expect_tx of the B tile
      mbar_init(&freeb[s], 1);
    }
    for (int s = 0; s < kTcRawSlots; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_free[s], kTcWarps);
    }
    mbar_init(&done, 1);
    mbar_fence_init();
  }
  if (warp == kTcWarps) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == kTcWarps + 1) {
    // ---------------- copy warp: raw superblocks (weights, before griddepcontrol.wait) and B tiles ----------------
    if (lane == 0) {
      const uint64_t policy = evict_first_policy();
      int rslot = 0, slot = 0;
      uint32_t rphase = 0, phase = 0;
      bool waited = false;
      // L2 lookahead: the raw ring holds two superblocks, so the superblocks after them are prefetched into L2
      // (`ahead` of them), which keeps more of the weight stream in flight than the ring's shared memory holds
      const int sb_end = (c1 + CPS - 1) / CPS;
      int l2sb = c0 / CPS + kTcRawSlots;
      auto l2_until = [&](int upto) {
        for (; l2sb < sb_end && l2sb < upto; ++l2sb)
          l2_prefetch_share(tiles + ((size_t)grp * sb_count + l2sb) * (size_t)raw_bytes, raw_bytes, 0, 1, raw_bytes);
      };
      l2_until(c0 / CPS + kTcRawSlots + ahead);
      for (int c = c0; c < c1; ++c) {
        if (c == c0 || c % CPS == 0) {
          if (!mbar_wait_backoff(&raw_free[rslot], rphase ^ 1u, err, 64)) break;
          const int sb = c / CPS;
          l2_until(sb + 1 + kTcRawSlots + ahead);
          mbar_expect_tx(&raw_full[rslot], raw_bytes);
          bulk_g2s_stream(raw_base + (size_t)rslot * raw_bytes,
                          tiles + ((size_t)grp * sb_count + sb) * (size_t)raw_bytes, raw_bytes, &raw_full[rslot],
                          policy);
          if (++rslot == kTcRawSlots) {
            rslot = 0;
            rphase ^= 1u;
          }
        }
        if (!waited) {  // the activations are the previous kernel's output
          griddep_wait();
          griddep_launch();
          waited = true;
        }
        if (!mbar_wait_backoff(&freeb[slot], phase ^ 1u, err, 64)) break;
        mbar_expect_tx(&full[slot], btile);
        bulk_g2s(tc_smem + (size_t)slot * stage_bytes + atile, xh + (size_t)c * btile, btile, &full[slot]);
        if (++slot == stages) {
          slot = 0;
          phase ^= 1u;
        }
      }
      if (!waited) {
        griddep_wait();
        griddep_launch();
      }
    } else {
      griddep_wait();
      griddep_launch();
    }
  } else if (warp == kTcWarps) {
    // ---------------- MMA issuer ----------------
    griddep_wait();
    griddep_launch();
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(P);
      const uint32_t sbase = smem_addr(tc_smem);
      int slot = 0;
      uint32_t phase = 0;
      for (int c = c0; c < c1; ++c) {
        mbar_wait(&full[slot], phase, err);
        tc_fence_after();
        const uint32_t a = sbase + (uint32_t)slot * stage_bytes, b = a + atile;
#pragma unroll
        for (int sub = 0; sub < SUB; ++sub)
#pragma unroll
          for (int kk = 0; kk < kTcKc / 16; ++kk)
            umma_f16(tmem, umma_desc_sw128(a + sub * kATileBytes + 32 * kk),
                     umma_desc_sw128(b + sub * (uint32_t)P * 128u + 32 * kk), idesc,
                     (c > c0 || sub > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&freeb[slot]);  // the stage is free once these MMAs have read it
        if (++slot == stages) {
          slot = 0;
          phase ^= 1u;
        }
      }
      umma_commit(&done);  // all MMAs of the CTA complete: the accumulator is final
    }
    __syncwarp();
  } else {
    // ---------------- dequant warps ----------------
    griddep_wait();
    griddep_launch();
    const int rt = warp, g = lane / 4, qq = lane % 4;
    int slot = 0, rslot = 0;
    uint32_t phase = 0, rphase = 0;
    for (int c = c0; c < c1; ++c) {
      if (c == c0 || c % CPS == 0) mbar_wait(&raw_full[rslot], rphase, err);
      // the slot's previous MMAs have read it (a fresh barrier passes the parity-1 wait at once)
      mbar_wait(&freeb[slot], phase ^ 1u, err);
      uint8_t* A = tc_smem + (size_t)slot * stage_bytes;
      const uint8_t* tile = raw_base + (size_t)rslot * raw_bytes + (size_t)rt * tile_bytes;
#pragma unroll
      for (int sub = 0; sub < SUB; ++sub) {  // quarter j of the superblock -> 64-column A tile `sub`
        const int j = (c % CPS) * SUB + sub;
        Dq8 r0, r8;
        if (QUANT == CLM_QUANT_Q4_K)
          dq_q4k(tile, j, g, qq, r0, r8);
        else
          dq_q80(tile, j, g, qq, r0, r8);
        const int row = rt * 16 + g;
        uint8_t* As = A + sub * kATileBytes;
        *reinterpret_cast<uint4*>(As + sw128_off(row, qq)) = r0.lo;
        *reinterpret_cast<uint4*>(As + sw128_off(row, 4 + qq)) = r0.hi;
        *reinterpret_cast<uint4*>(As + sw128_off(row + 8, qq)) = r8.lo;
        *reinterpret_cast<uint4*>(As + sw128_off(row + 8, 4 + qq)) = r8.hi;
      }
      fence_async_smem();  // generic-proxy writes -> visible to the tensor core's async reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[slot]);
      if (c % CPS == CPS - 1 || c == c1 - 1) {  // done with this raw superblock
        if (lane == 0) mbar_arrive(&raw_free[rslot]);
        if (++rslot == kTcRawSlots) {
          rslot = 0;
          rphase ^= 1u;
        }
      }
      if (++slot == stages) {
        slot = 0;
        phase ^= 1u;
      }
    }
    // ---------------- epilogue: TMEM -> f32 partial ----------------
    mbar_wait(&done, 0, err);
    tc_fence_after();
    const int quarter = warp % 4, colhalf = warp / 4;
    const uint32_t row = (uint32_t)grp * 128 + 32 * quarter + lane;
    float* out = part + (size_t)split * q * rows_total;
    for (int cb = colhalf * 32; cb < P; cb += 64) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)cb, v);
      if (row < rows_total) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (cb + i < q) out[(size_t)(cb + i) * rows_total + row] = v[i];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcWarps) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

__global__ void split_sum_kernel(const float* __restrict__ part, int ksplit, uint64_t n, float* __restrict__ y) {
  griddep_wait();
  griddep_launch();
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float a = part[i];
    for (int s = 1; s < ksplit; ++s) a += part[(uint64_t)s * n + i];
    y[i] = a;
  }
}

// Raw superblocks prefetched into L2 beyond the ring (CLM_B200_TC_AHEAD).  Off by default: at 128 and 256 rows
// the GEMM is bound by the per-chunk hand-offs between its warps, and 4 or 8 superblocks ahead measured slower.
int tc_l2_ahead() {
  static const int v = [] {
    const char* e = getenv("CLM_B200_TC_AHEAD");
    return e ? atoi(e) : 0;
  }();
  return v;
}

}  // namespace

TcPlan gemm_tc_plan(const GemvShape& s, int q, int sm_count) {
  TcPlan p;
  p.P = ((q + 15) / 16) * 16;
  const size_t raw = (size_t)kTcRawSlots * kGemvWarps * s.tile_bytes;
  const size_t stage64 = kATileBytes + (size_t)p.P * 128;
  constexpr size_t kSmemMax = 227 * 1024;
  // 128-column stages when two of them fit next to the raw ring (up to 128 window rows)
  p.kc = 1024 + 2 * 2 * stage64 + raw <= kSmemMax ? 128 : 64;
  const size_t stage = stage64 * (p.kc / kTcKc);
  const int chunks = (int)s.cols / p.kc;
  // K splits: as many as keep the grid within one wave of CTAs (one per SM), at least two chunks per CTA.  (Splits
  // that balance a second wave, e.g. 3 for 224 row groups, measured slower: their partials cost more than the wave.)
  const int sms = sm_count > 0 ? sm_count : 148;
  int ks = (int)(s.ng < (uint32_t)sms ? sms / s.ng : 1);
  if (ks > chunks / 2) ks = chunks / 2;
  if (ks < 1) ks = 1;
  p.ksplit = ks;
  p.stages = kTcMaxStages;
  while (p.stages > 2 && 1024 + p.stages * stage + raw > kSmemMax) --p.stages;
  p.smem = 1024 + (size_t)p.stages * stage + raw;
  p.part_floats = (size_t)ks * q * s.rows;
  p.xh_bytes = (size_t)p.P * s.cols * 2;
  return p;
}

int launch_tc_xprep(const float* d_x, int q, int K, int P, uint8_t* d_xh, cudaStream_t st) {
  CLM_CHECK(K % kTcKc == 0 && q >= 1 && q <= P && P % 16 == 0, CLM_INVALID_ARGUMENT, "activation tile shape");
  CLM_CHECK((reinterpret_cast<uintptr_t>(d_x) & 15) == 0 && (reinterpret_cast<uintptr_t>(d_xh) & 15) == 0,
            CLM_INTERNAL, "activation rows and tiles must be 16-byte aligned");
  const uint64_t n = (uint64_t)(K / kTcKc) * P * 8;
  return launch_pdl(tc_xprep_kernel, dim3((unsigned)std::min<uint64_t>((n + 255) / 256, 4096)), dim3(256), 0, st,
                    d_x, q, K, P, d_xh);
}

int launch_gemm_tc(const GemvShape& s, const TcPlan& p, const uint8_t* d_tiles, const float* d_x, int q, float* d_y,
                   uint8_t* d_xh, float* d_part, int* d_err, cudaStream_t st) {
  CLM_TRY(launch_tc_xprep(d_x, q, (int)s.cols, p.P, d_xh, st));
  return launch_gemm_tc_tiles(s, p, d_tiles, d_xh, q, d_y, d_part, d_err, st);
}

int launch_gemm_tc_tiles(const GemvShape& s, const TcPlan& p, const uint8_t* d_tiles, const uint8_t* d_xh, int q,
                         float* d_y, float* d_part, int* d_err, cudaStream_t st, bool sum_splits) {
  CLM_CHECK(q > 16 && q <= 256 && p.P == ((q + 15) / 16) * 16, CLM_OUT_OF_RANGE,
            "tensor-core GEMM covers 17..256 window rows");
  CLM_CHECK(s.cols % 256 == 0, CLM_INVALID_ARGUMENT, "columns must be a multiple of 256");
  CLM_CHECK(s.quant == CLM_QUANT_Q4_K || s.quant == CLM_QUANT_Q8_0, CLM_UNIMPLEMENTED, "tensor-core GEMM: Q4_K / Q8_0");
  CLM_CHECK(p.smem <= 227 * 1024, CLM_RESOURCE_EXHAUSTED, "tensor-core GEMM: shared memory");
  CLM_CHECK((reinterpret_cast<uintptr_t>(d_xh) & 15) == 0, CLM_INTERNAL, "activation tiles must be 16-byte aligned");
  CLM_CHECK(p.ksplit == 1 || d_part != nullptr, CLM_INTERNAL, "split-K partials need a buffer");
  CLM_CHECK(p.kc == 64 || p.kc == 128, CLM_INTERNAL, "tensor-core GEMM: stage width");
  const dim3 grid(s.ng, (unsigned)p.ksplit);
  float* out = p.ksplit > 1 ? d_part : d_y;
  auto go = [&](auto kern) -> int {
    CLM_TRY(ensure_smem(kern, p.smem));
    return launch_pdl(kern, grid, dim3(kTcThreads), p.smem, st, d_tiles, (int)s.sb, s.tile_bytes, d_xh, q,
                      (int)s.cols, p.P, p.ksplit, p.stages, out, s.rows, d_err, tc_l2_ahead());
  };
  if (s.quant == CLM_QUANT_Q4_K)
    CLM_TRY(p.kc == 128 ? go(gemm_tc_kernel<CLM_QUANT_Q4_K, 128>) : go(gemm_tc_kernel<CLM_QUANT_Q4_K, 64>));
  else
    CLM_TRY(p.kc == 128 ? go(gemm_tc_kernel<CLM_QUANT_Q8_0, 128>) : go(gemm_tc_kernel<CLM_QUANT_Q8_0, 64>));
  if (p.ksplit > 1 && sum_splits) {
    const uint64_t n = (uint64_t)q * s.rows;
    CLM_TRY(launch_pdl(split_sum_kernel, dim3((unsigned)std::min<uint64_t>((n + 255) / 256, 4096)), dim3(256), 0, st,
                       (const float*)d_part, p.ksplit, n, d_y));
  }
  return CLM_OK;
}

}  // namespace clm
