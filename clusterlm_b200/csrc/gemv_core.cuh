// gemv_core.cuh — building blocks of the persistent q-row GEMV shared by the single-matrix kernel (gemv4.cu)
// and the verify-window dataflow kernel (flow.cu): consumer warp roles, the per-unit tensor-core step, row-group
// flush (segment partials reduced by the group's first segment) and the fused epilogues.
#pragma once
#include "bulk.cuh"
#include "gemv2.cuh"
#include "gemv_tile.cuh"
#include "llama.cuh"

namespace clm {

constexpr int kG4Consumers = 512;              // 16 consumer warps: 8 row tiles x 2 superblocks
constexpr int kG4Threads = kG4Consumers + 32;  // + the producer warp
constexpr int kG4MaxStages = 10;
constexpr int kG4SbSumBytes = 8 * 16 * 4;      // one half of one superblock's sub-block sums: [8 sub-blocks][16 p] f32

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

template <int EPI = 0>
__device__ __forceinline__ long long tree_depth4(const int32_t* parent, int i) {
  long long d = 0;
  for (int a = parent[i]; a >= 0 && d < 64; a = parent[a]) ++d;
  return d;
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// CTA whose stream-K range holds unit x.
__device__ __forceinline__ int cta_of_unit(long long x, long long U, int G) { return (int)(((x + 1) * G - 1) / U); }

// Segments of the group of units [x, y] (the CTA ranges that hold any of them) and this CTA's ordinal among them;
// u0 = first unit of this CTA's range.  With U >= G every CTA owns at least one unit, so consecutive CTAs are
// consecutive segments; with U < G every CTA owns at most one unit and CTAs without units sit between them.
__device__ __forceinline__ void group_segments(long long x, long long y, long long U, int G, long long u0, int* seg,
                                               int* nseg) {
  if (U >= G) {
    const int c_first = cta_of_unit(x, U, G);
    *seg = (int)blockIdx.x - c_first;
    *nseg = cta_of_unit(y, U, G) - c_first + 1;
  } else {
    *seg = (int)((u0 > x ? u0 : x) - x);
    *nseg = (int)(y - x + 1);
  }
}

struct G4Geom {
  int sb;          // superblocks per row
  int usb;         // superblocks per unit (2 in both the single-matrix GEMV and the dataflow kernel)
  int ppr;         // units per row group
  int tile_bytes;  // one 16-row x 256-column tile
  int sb_bytes;    // 8 tiles of one superblock
  int stage_bytes;
  int sum_half;    // bytes of one half of a unit's sub-block sums (usb x kG4SbSumBytes)
  int frag_off, sum_off;  // offsets inside a stage: [weights usb sb][fragments usb sb x NT][sums half 0][half 1]
};

// Position in a CTA's unit range without divisions in the loops: (row group, superblock pair) of the unit and
// (ring slot, phase parity) of its stage.
struct UnitCursor {
  int grp = 0, pr = 0, slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int ppr, int stages) {
    if (++pr == ppr) {
      pr = 0;
      ++grp;
    }
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Epilogue operands that do not depend on this kernel's products (the residual rows and the next norm's weights,
// or the position, page and RoPE factors), loaded when a CTA starts a row group so that their latency overlaps the
// group's tensor-core work and the segment exchange.  Element i = tid + kG4Consumers * k of the epilogue's loops.
// QM: the most window rows the launch serves (16, or 32 for the 4-n-tile GEMV); the loops below run QM / 4 (residual)
// and QM / 8 (RoPE) elements per thread.
struct EpiPre {
  float h[8];       // EPI_RESID_PREP: h[p][row0 + r], i = p * 128 + r
  float w;          // EPI_RESID_PREP: wnext[row0 + tid] (tid < 128)
  long long base;   // EPI_ROPE_KV: committed position
  float2 cs[4];     // EPI_ROPE_KV: RoPE (cos, sin) of element i = p * (hd / 2) + pair
  int32_t page[4];  // EPI_ROPE_KV: KV page of window row p
};

template <int EPI, int QM = 16>
__device__ __forceinline__ void epi_preload(EpiPre& pre, int grp, uint32_t rows, int q, const Epi& epi) {
  const int tid = threadIdx.x, row0 = grp * 128;
  if (EPI == EPI_RESID_PREP) {
#pragma unroll
    for (int k = 0; k < QM / 4; ++k) {
      const int i = tid + kG4Consumers * k, p = i / 128, r = i % 128;
      pre.h[k] = (i < q * 128 && row0 + r < (int)rows) ? __ldcg(epi.h + (size_t)p * epi.H + row0 + r) : 0.0f;
    }
    pre.w = (tid < 128 && row0 + tid < (int)rows) ? epi.wnext[row0 + tid] : 0.0f;
  } else if (EPI == EPI_ROPE_KV) {
    if (epi.seg_q > 0) return;  // several sessions: the epilogue reads its operands itself
    const int hd = epi.hd, head = grp;
    pre.base = *epi.pos;
#pragma unroll
    for (int k = 0; k < QM / 8; ++k) {
      const int i = tid + kG4Consumers * k, p = i / (hd / 2), pr = i % (hd / 2);
      pre.cs[k] = make_float2(0.0f, 0.0f);
      pre.page[k] = 0;
      if (i < q * (hd / 2)) {
        const long long slot = pre.base + p;
        pre.page[k] = epi.pages[slot / 64];
        if (head < epi.nh + epi.nkv) {
          const long long rope_pos = epi.parent ? pre.base + tree_depth4<0>(epi.parent, p) : slot;
          pre.cs[k] = epi.rope[(size_t)rope_pos * (hd / 2) + pr];
        }
      }
    }
  }
}

// Epilogue over y[p][r] (128 rows of group grp) in shared memory; consumer threads only.  `pre` holds the operands
// preloaded by epi_preload (or null: they are read here); s_aux is shared scratch of at least 128 floats.
template <int EPI, int QM = 16>
__device__ void g4_epilogue(float* y, const float* s_scale, int grp, uint32_t rows, int q, const Epi& epi,
                            float* s_aux, const EpiPre* pre) {
  const int tid = threadIdx.x;
  const int row0 = grp * 128;
  if (EPI == EPI_STORE) {
    for (int i = tid; i < q * 128; i += kG4Consumers) {
      const int p = i / 128, r = i % 128;
      if (row0 + r < (int)rows) epi.out[(size_t)p * epi.out_ld + row0 + r] = y[i] * s_scale[p];
    }
  } else if (EPI == EPI_RESID_PREP) {
#pragma unroll
    for (int k = 0; k < QM / 4; ++k) {
      const int i = tid + kG4Consumers * k, p = i / 128, r = i % 128;
      if (i >= q * 128 || row0 + r >= (int)rows) continue;
      float* hp = epi.h + (size_t)p * epi.H + row0 + r;
      const float hn = (pre ? pre->h[k] : __ldcg(hp)) + y[i] * s_scale[p];  // h is written by other CTAs
      *hp = hn;
      y[i] = hn;
    }
    if (tid < 128) s_aux[tid] = pre ? pre->w : (row0 + tid < (int)rows ? epi.wnext[row0 + tid] : 0.0f);
    consumer_sync();
    const int nt_out = (q + 7) / 8 == 3 ? 4 : (q + 7) / 8;
    for (int i = tid; i < 8 * 8 * nt_out; i += kG4Consumers) {
      const int gg = i % 8, p = i / 8;
      float vals[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int r = 16 * gg + k;
        vals[k] = p < q ? y[p * 128 + r] * s_aux[r] : 0.0f;
      }
      prep16(vals, nullptr, p, q, (row0 + 16 * gg) / 16, nt_out, epi.hi_scale, epi.next.frag, epi.next.sum, nullptr,
             epi.H);
    }
    // the next consumer's row scale: sum of squares of this group's 128 new residual values, per row
    if (epi.next.ss) {
      const int ln = tid % 32;
#pragma unroll
      for (int p = tid / 32; p < QM; p += kG4Consumers / 32) {  // one warp per row
        float a = 0.0f;
        if (p < q && row0 + ln < (int)rows) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float v = y[p * 128 + ln + 32 * k];
            a += v * v;
          }
        }
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (ln == 0) epi.next.ss[(size_t)grp * kSsRows + p] = a;
      }
    }
  } else if (EPI == EPI_ROPE_KV) {
    const int head = grp, hd = epi.hd;
    const bool seg = epi.seg_q > 0;
    if (seg) pre = nullptr;
    const long long base = seg ? 0 : (pre ? pre->base : *epi.pos);
#pragma unroll
    for (int k = 0; k < QM / 8; ++k) {
      const int i = tid + kG4Consumers * k;
      if (i >= q * (hd / 2)) continue;
      const int p = i / (hd / 2), pr = i % (hd / 2);
      const float a = y[p * 128 + 2 * pr] * s_scale[p], b = y[p * 128 + 2 * pr + 1] * s_scale[p];
      // several sessions: row p is row p % seg_q of session p / seg_q
      const int sg = seg ? p / epi.seg_q : 0;
      const long long slot = seg ? *epi.seg_pos[sg] + (p - sg * epi.seg_q) : base + p;
      const int32_t page = pre ? pre->page[k] : (seg ? epi.seg_pages[sg] : epi.pages)[slot / 64];
      if (head < epi.nh + epi.nkv) {
        float2 cs;
        if (pre) {
          cs = pre->cs[k];
        } else {
          const long long rope_pos = (!seg && epi.parent) ? base + tree_depth4(epi.parent, p) : slot;
          cs = epi.rope[(size_t)rope_pos * (hd / 2) + pr];
        }
        const float c = cs.x, s = cs.y;
        const float ra = a * c - b * s, rb = a * s + b * c;
        __half* dst;
        if (head < epi.nh) {
          dst = epi.q16 + ((size_t)p * epi.nh + head) * hd + 2 * pr;
        } else {
          const int pos = (int)(slot % 64), d0 = 2 * pr;
          dst = epi.kpool + (((size_t)page * epi.nkv + (head - epi.nh)) * 64 + pos) * hd +
                8 * kv_k_chunk(d0 >> 3, pos) + (d0 & 7);
        }
        dst[0] = __float2half_rn(ra);
        dst[1] = __float2half_rn(rb);
      } else {
        const int pos = (int)(slot % 64), d0 = 2 * pr;
        __half* vt = epi.vpool + (((size_t)page * epi.nkv + (head - epi.nh - epi.nkv)) * hd + d0) * 64;
        vt[8 * kv_v_chunk(pos >> 3, d0) + (pos & 7)] = __float2half_rn(a);
        vt[64 + 8 * kv_v_chunk(pos >> 3, d0 + 1) + (pos & 7)] = __float2half_rn(b);
      }
    }
  } else if (EPI == EPI_SWIGLU_PREP) {
    // rows [0, 64) gate, [64, 128) up of ffn indices grp*64 + [0, 64)
    for (int i = tid; i < q * 64; i += kG4Consumers) {
      const int p = i / 64, k = i % 64;
      const float gv = y[p * 128 + k] * s_scale[p], uv = y[p * 128 + 64 + k] * s_scale[p];
      y[p * 128 + k] = gv / (1.0f + expf(-gv)) * uv;
    }
    consumer_sync();
    const int nt_out = (q + 7) / 8 == 3 ? 4 : (q + 7) / 8;
    for (int i = tid; i < 4 * 8 * nt_out; i += kG4Consumers) {
      const int gg = i % 4, p = i / 4;
      float vals[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) vals[k] = p < q ? y[p * 128 + 16 * gg + k] : 0.0f;
      prep16(vals, nullptr, p, q, (grp * 64 + 16 * gg) / 16, nt_out, epi.hi_scale, epi.next.frag, epi.next.sum,
             nullptr, epi.ffn);
    }
  }
  consumer_sync();  // y is reused by the next group
}


// Epilogue kind chosen at run time (the dataflow kernel's phases, the flush of a row group).
template <int QM = 16>
__device__ __forceinline__ void g4_epilogue_rt(int kind, float* y, const float* s_scale, int grp, uint32_t rows,
                                               int q, const Epi& epi, float* s_aux, const EpiPre* pre) {
  switch (kind) {
    case EPI_STORE: g4_epilogue<EPI_STORE, QM>(y, s_scale, grp, rows, q, epi, s_aux, pre); break;
    case EPI_RESID_PREP: g4_epilogue<EPI_RESID_PREP, QM>(y, s_scale, grp, rows, q, epi, s_aux, pre); break;
    case EPI_ROPE_KV: g4_epilogue<EPI_ROPE_KV, QM>(y, s_scale, grp, rows, q, epi, s_aux, pre); break;
    default: g4_epilogue<EPI_SWIGLU_PREP, QM>(y, s_scale, grp, rows, q, epi, s_aux, pre); break;
  }
}

// epi_preload with the kind chosen at run time.
template <int QM = 16>
__device__ __forceinline__ void epi_preload_rt(int kind, EpiPre& pre, int grp, uint32_t rows, int q, const Epi& epi) {
  if (kind == EPI_RESID_PREP) epi_preload<EPI_RESID_PREP, QM>(pre, grp, rows, q, epi);
  if (kind == EPI_ROPE_KV) epi_preload<EPI_ROPE_KV, QM>(pre, grp, rows, q, epi);
}

// Row scale (folded rmsnorm) 1/sqrt(sum(ss)/ss_n + eps) per window row from the input's sum-of-squares partials
// (1 without partials), in two steps so that the partials' load latency overlaps the first units: g4_ss_load at
// the start of a GEMV (registers only), g4_ss_finish before the first flush.  Consumer threads only; s_red holds
// kG4Consumers floats, s_scale kSsRows.  Thread tid adds partials c = tid / 32 + 16 k (k ascending) of row tid % 32;
// the first two are loaded ahead, any further ones (partials per 16 columns of the strip GEMV) in g4_ss_finish.
struct G4SsPre {
  float a = 0.0f, b = 0.0f;
};
__device__ __forceinline__ G4SsPre g4_ss_load(const XBuf& in) {
  G4SsPre r;
  const int tid = threadIdx.x, p = tid % kSsRows, c = tid / kSsRows;
  constexpr int kStride = kG4Consumers / kSsRows;
  if (in.ss) {
    if (c < in.nss) r.a = __ldcg(in.ss + (size_t)c * kSsRows + p);
    if (c + kStride < in.nss) r.b = __ldcg(in.ss + (size_t)(c + kStride) * kSsRows + p);
  }
  return r;
}
__device__ __forceinline__ void g4_ss_finish(const G4SsPre& pre, const XBuf& in, const Epi& epi, int q, float* s_red,
                                             float* s_scale) {
  const int tid = threadIdx.x;
  constexpr int kStride = kG4Consumers / kSsRows;
  {
    float a = pre.a + pre.b;
    if (in.ss)
      for (int c0 = tid / kSsRows + 2 * kStride; c0 < in.nss; c0 += 8 * kStride) {
        // eight loads in flight, added in partial order
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = c0 + k * kStride;
          v[k] = c < in.nss ? __ldcg(in.ss + (size_t)c * kSsRows + tid % kSsRows) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) a += v[k];
      }
    s_red[tid] = a;
  }
  consumer_sync();
  if (tid < kSsRows) {
    float sc = 1.0f;
    if (in.ss && tid < q) {
      float tot = 0.0f;
      for (int c = 0; c < kStride; ++c) tot += s_red[c * kSsRows + tid];
      sc = 1.0f / sqrtf(tot / epi.ss_n + epi.eps);
    }
    s_scale[tid] = sc;
  }
  consumer_sync();
}

// Accumulators of one consumer warp: row tile rt = warp % 8, superblock hh = warp / 8 of each unit, even and
// odd k-steps in separate registers.
template <int NT>
struct G4Acc {
  float v[2][NT][4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) v[a][nt][i] = 0.0f;
  }
  // dst[p][r] (+)= this warp's sums for its rows
  __device__ __forceinline__ void put(float* dst, bool add, int q, int rt, int lane) const {
    const int t = lane % 4, g = lane / 4, r0 = rt * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int p0 = nt * 8 + 2 * t;
      const float v0 = v[0][nt][0] + v[1][nt][0], v1 = v[0][nt][1] + v[1][nt][1];
      const float v2 = v[0][nt][2] + v[1][nt][2], v3 = v[0][nt][3] + v[1][nt][3];
      if (p0 < q) {
        dst[p0 * 128 + r0] = add ? dst[p0 * 128 + r0] + v0 : v0;
        dst[p0 * 128 + r1] = add ? dst[p0 * 128 + r1] + v2 : v2;
      }
      if (p0 + 1 < q) {
        dst[(p0 + 1) * 128 + r0] = add ? dst[(p0 + 1) * 128 + r0] + v1 : v1;
        dst[(p0 + 1) * 128 + r1] = add ? dst[(p0 + 1) * 128 + r1] + v3 : v3;
      }
    }
  }
};

// Row tile rt of superblock hh of the unit staged at `st` (nsb superblocks in the unit): dequantised tensor-core
// products into acc, then the unit's min / bias term for this superblock.
template <typename Raw, int NT>
__device__ __forceinline__ void g4_consume_tile(const uint8_t* st, const G4Geom& geo, int hh, int nsb, int rt,
                                                int lane, G4Acc<NT>& acc) {
  const int t = lane % 4;
  const uint2* xf = reinterpret_cast<const uint2*>(st + geo.frag_off) + hh * NT * 512;
  uint32_t mg, mg8;
  Raw r;
  load_raw_s(r, st + (size_t)hh * geo.sb_bytes + (size_t)rt * geo.tile_bytes, lane);
  tile_mmas<NT>(r, t, xf, lane, acc.v, mg, mg8);
  // min / bias term of this superblock: A = -m per (row, sub-block) for both 16-column halves, B = the staged
  // fp16 hi / lo half sums (prep16's fragment layout)
  const uint4* sf = reinterpret_cast<const uint4*>(st + geo.sum_off) + hh * 32 * sum_tiles(NT);
  (void)nsb;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint4 b = sf[nt * 32 + lane];
    mma16816(acc.v[0][nt], mg, mg8, mg, mg8, b.x, b.y);
    mma16816(acc.v[1][nt], mg, mg8, mg, mg8, b.z, b.w);
  }
}

// Both superblocks of the unit staged at `st` (nsb of them) for row tile rt: one warp's whole share of the unit.
template <typename Raw, int NT>
__device__ __forceinline__ void g4_consume_pair(const uint8_t* st, const G4Geom& geo, int nsb, int rt, int lane,
                                                G4Acc<NT>& acc) {
  const int t = lane % 4;
  const uint2* xf = reinterpret_cast<const uint2*>(st + geo.frag_off);
  const uint4* sf = reinterpret_cast<const uint4*>(st + geo.sum_off);
  uint32_t m0 = 0u, m08 = 0u, m1 = 0u, m18 = 0u;
  {
    Raw r;
    load_raw_s(r, st + (size_t)rt * geo.tile_bytes, lane);
    tile_mmas<NT>(r, t, xf, lane, acc.v, m0, m08);
  }
  if (nsb > 1) {
    Raw r;
    load_raw_s(r, st + (size_t)geo.sb_bytes + (size_t)rt * geo.tile_bytes, lane);
    tile_mmas<NT>(r, t, xf + NT * 512, lane, acc.v, m1, m18);
  }
  // min / bias terms: A = -m per (row, sub-block) for both 16-column halves, B = the staged hi / lo half sums
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    if (hh >= nsb) break;
    const uint32_t a = hh ? m1 : m0, a8 = hh ? m18 : m08;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint4 b = sf[hh * 32 * sum_tiles(NT) + nt * 32 + lane];
      mma16816(acc.v[0][nt], a, a8, a, a8, b.x, b.y);
      mma16816(acc.v[NT >= 4 ? 0 : 1][nt], a, a8, a, a8, b.z, b.w);
    }
  }
}

// One unit (superblock pair of a row group) staged at `st`: this warp's tile of superblock hh = warp / 8.
template <typename Raw, int NT>
__device__ __forceinline__ void g4_consume_unit(const uint8_t* st, const G4Geom& geo, int nsb, int warp, int lane,
                                                G4Acc<NT>& acc) {
  const int rt = warp % kGemvWarps, hh = warp / kGemvWarps;
  if (hh >= nsb) return;
  g4_consume_tile<Raw, NT>(st, geo, hh, nsb, rt, lane, acc);
}

// Dataflow signal of a finished row group (one thread, after the consumer barrier that ends the epilogue, so the
// release covers every consumer's stores): its chunk counter (a QKV head signals its kv head) and the phase's
// finished-group count.
__device__ __forceinline__ void g4_signal(const Epi& epi, int grp) {
  if (epi.sig != nullptr) {
    int c = grp / epi.sig_div;
    if (epi.sig_qkv) {
      const int group = epi.nh / epi.nkv;
      c = grp < epi.nh ? grp / group : (grp < epi.nh + epi.nkv ? grp - epi.nh : grp - epi.nh - epi.nkv);
    }
    red_release_add(epi.sig + c, 1);
  }
  if (epi.done != nullptr) red_release_add(epi.done, 1);
}

// Flush row group `grp` of a stream-K range: fold the two superblock warps into y (fixed order); a group owned by
// this CTA alone goes to the epilogue.  Otherwise a later segment publishes its partial (release-add on the group's
// counter by one thread after the consumer barrier) and continues without waiting, and the group's first segment
// waits (bounded acquire spin) for the other nseg-1 partials, sums them in segment order, resets the counter and
// runs the epilogue.  Every CTA of the grid is resident (one per SM), so the wait always ends.  Consumer threads
// only.  Returns true in the CTA that ran the group's epilogue.
template <int NT>
__device__ bool g4_flush(int grp, const G4Acc<NT>& acc, float* y, float* part, int* counters, int maxseg,
                         long long U, int G, long long u0, int ppr, int q, uint32_t rows, int epi_kind, const Epi& epi,
                         float* s_scale, int* s_last, const G4SsPre& ss_pre, const XBuf& in, bool& scale_ready,
                         float* s_red, const EpiPre* pre = nullptr, EpiPre* lazy = nullptr) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  if (!scale_ready) {
    G4SsPre sp = ss_pre;
    if (epi.ss_done != nullptr) {
      // dataflow: the row scale needs every sum-of-squares partial of the residual phase that wrote the input
      if (tid == 0) (void)dep_wait(epi.ss_done, epi.ss_target, epi.err);
      consumer_sync();
      sp = g4_ss_load(in);
    }
    g4_ss_finish(sp, in, epi, q, s_red, s_scale);
    scale_ready = true;
  }
  const int rt = warp % kGemvWarps, hh = warp / kGemvWarps;
  if (hh == 1) acc.put(y, false, q, rt, lane);
  consumer_sync();
  if (hh == 0) acc.put(y, true, q, rt, lane);
  consumer_sync();
  int seg = 0, nseg = 1;
  group_segments((long long)grp * ppr, (long long)grp * ppr + ppr - 1, U, G, u0, &seg, &nseg);
  // A row group that cannot be reduced (too few partial slots, or a wait that gave up) raises the error flag; a
  // plain product (EPI_STORE) also writes its rows as NaN, so a caller without an error flag never reads stale or
  // partial sums as a result.
  auto fail_group = [&](int code) {
    if (tid == 0 && epi.err && code) atomicExch(epi.err, code);
    if (epi_kind == EPI_STORE)
      for (int i = tid; i < q * 128; i += kG4Consumers) {
        const int p = i / 128, r = i % 128;
        if (grp * 128 + r < (int)rows) epi.out[(size_t)p * epi.out_ld + grp * 128 + r] = __int_as_float(0x7fc00000);
      }
  };
  if (nseg > maxseg) {  // partial slots too few for this launch shape: never write past them
    fail_group(kErrPartialSlots);
    return false;
  }
  if (nseg > 1) {
    if (seg > 0) {
      // a later segment publishes its partial and moves on; the group's first segment (whose CTA reaches the
      // group at the end of its range) reduces it
      float* mine = part + ((size_t)grp * maxseg + seg) * q * 128;
      for (int i = tid; i < q * 128; i += kG4Consumers) mine[i] = y[i];
      consumer_sync();
      if (tid == 0) red_release_add(&counters[grp], 1);
      return false;
    }
    if (lazy != nullptr) {  // the epilogue's operands load while the other segments' partials arrive
      epi_preload_rt<NT >= 4 ? 32 : 16>(epi_kind, *lazy, grp, rows, q, epi);
      pre = lazy;
    }
    if (tid == 0) {
      const bool ok = wait_count(&counters[grp], nseg - 1, epi.err);
      if (ok) counters[grp] = 0;  // every arrival of this launch is in: ready for the next launch
      *s_last = ok;
    }
    consumer_sync();
    if (!*s_last) {
      fail_group(0);  // wait_count raised the flag
      return false;
    }
    const float* all = part + (size_t)grp * maxseg * q * 128;
    for (int i = tid; i < q * 128; i += kG4Consumers) {
      float a = y[i];
      int k = 1;
      for (; k + 4 <= nseg; k += 4) {
        const float v0 = __ldcg(all + (size_t)k * q * 128 + i), v1 = __ldcg(all + (size_t)(k + 1) * q * 128 + i);
        const float v2 = __ldcg(all + (size_t)(k + 2) * q * 128 + i), v3 = __ldcg(all + (size_t)(k + 3) * q * 128 + i);
        a += v0;
        a += v1;
        a += v2;
        a += v3;
      }
      for (; k < nseg; ++k) a += __ldcg(all + (size_t)k * q * 128 + i);
      y[i] = a;
    }
    consumer_sync();
  }
  g4_epilogue_rt<NT >= 4 ? 32 : 16>(epi_kind, y, s_scale, grp, rows, q, epi, s_red, pre);  // ends with a barrier
  if (tid == 0) g4_signal(epi, grp);
  return true;
}

// Geometry of a tiled matrix in the persistent GEMV for `nt` column tiles and units of `usb` superblocks.
inline G4Geom g4_geom(const GemvShape& s, int nt, int usb = 2) {
  G4Geom geo;
  geo.sb = (int)s.sb;
  geo.usb = usb;
  geo.ppr = (int)(s.sb + usb - 1) / usb;
  geo.tile_bytes = s.tile_bytes;
  geo.sb_bytes = kGemvWarps * s.tile_bytes;
  geo.sum_half = usb * 256 * sum_tiles(nt);  // the stage's sum region is 2 * sum_half = usb x 512 B x sum tiles
  geo.frag_off = usb * geo.sb_bytes;
  geo.sum_off = geo.frag_off + usb * nt * kXfragSbBytes;
  geo.stage_bytes = geo.sum_off + 2 * geo.sum_half;
  return geo;
}

}  // namespace clm
