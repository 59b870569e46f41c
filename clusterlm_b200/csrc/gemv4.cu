// gemv4.cu — persistent, warp-specialised, stream-K q-row GEMV with fused epilogues (sm_100a).
//
// y[p][row] = W[row] . x[p] for q <= 16 window rows, W in the group-major tile layout of gemv.cuh
// ([128-row group][superblock][8 row tiles]).  The work is the sequence of "units" (row group, superblock pair),
// U = ng * ceil(SB / 2) of them, split into gridDim.x contiguous ranges (stream-K): CTA c owns units
// [c*U/G, (c+1)*U/G).  Every unit is ~37 KB (Q4_K) / ~70 KB (Q8_0) of weights, so every CTA streams the same
// number of bytes whatever the matrix shape.
//
//  * Warp 8 is the producer: one lane keeps a ring of `stages` shared-memory slots full with cp.async.bulk
//    copies (no multicast) of the unit's weights, activation fragments and sub-block sums, completing on the
//    slot's "full" mbarrier.  The first `stages` weight copies are issued before griddepcontrol.wait (weights are
//    immutable), so under programmatic dependent launch they stream in while the previous kernel finishes.
//  * Warps 0..15 consume: warp w dequantises row tile w % 8 of superblock w / 8 of the unit in registers
//    (gemv_tile.cuh) and issues m16n8k16 tensor-core products against the staged fragments (even and odd
//    k-steps on separate accumulators), then releases the slot ("empty" mbarrier).  The two warps of a row
//    tile fold their accumulators through shared memory when the CTA flushes a row group.
//  * When a CTA's range leaves a row group it flushes the group: a group owned by one CTA goes straight to the
//    epilogue; otherwise each CTA writes its segment's partial and the last one to arrive (atomic counter) sums
//    the segments in index order (deterministic) and runs the epilogue.
//  * Every mbarrier wait is bounded (bulk.cuh); a timeout raises the epilogue's error flag.
#include "bulk.cuh"
#include "gemv2.cuh"
#include "gemv_tile.cuh"
#include "llama.cuh"
#include "pdl.cuh"

namespace clm {

constexpr int kG4Consumers = 512;              // 16 consumer warps: 8 row tiles x 2 superblocks
constexpr int kG4Threads = kG4Consumers + 32;  // + the producer warp
constexpr int kG4MaxStages = 4;
constexpr int kG4SumBytes = 16 * 16 * 4;       // one half of a unit's sub-block sums: [16 sub-blocks][16 p] f32

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

__device__ __forceinline__ long long tree_depth4(const int32_t* parent, int i) {
  long long d = 0;
  for (int a = parent[i]; a >= 0 && d < 64; a = parent[a]) ++d;
  return d;
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// CTA whose stream-K range holds unit x.
__device__ __forceinline__ int cta_of_unit(long long x, long long U, int G) { return (int)(((x + 1) * G - 1) / U); }

struct G4Geom {
  int sb;          // superblocks per row
  int ppr;         // units (superblock pairs) per row group
  int tile_bytes;  // one 16-row x 256-column tile
  int sb_bytes;    // 8 tiles of one superblock
  int stage_bytes;
  int frag_off, sum_off;  // offsets inside a stage: [weights 2 sb][fragments 2 sb x NT][sums half 0][half 1]
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

// Epilogue over y[p][r] (128 rows of group grp) in shared memory; consumer threads only.
template <int EPI>
__device__ void g4_epilogue(float* y, const float* s_scale, int grp, uint32_t rows, int q, const Epi& epi,
                            float* s_ss) {
  const int tid = threadIdx.x;
  const int row0 = grp * 128;
  if (EPI == EPI_STORE) {
    for (int i = tid; i < q * 128; i += kG4Consumers) {
      const int p = i / 128, r = i % 128;
      if (row0 + r < (int)rows) epi.out[(size_t)p * epi.out_ld + row0 + r] = y[i] * s_scale[p];
    }
  } else if (EPI == EPI_RESID_PREP) {
    for (int i = tid; i < q * 128; i += kG4Consumers) {
      const int p = i / 128, r = i % 128;
      if (row0 + r >= (int)rows) continue;
      float* hp = epi.h + (size_t)p * epi.H + row0 + r;
      const float hn = *hp + y[i] * s_scale[p];
      *hp = hn;
      y[i] = hn;
    }
    consumer_sync();
    const int nt_out = q <= 8 ? 1 : 2;
    for (int i = tid; i < 8 * 8 * nt_out; i += kG4Consumers) {
      const int gg = i % 8, p = i / 8;
      float vals[16], raw[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int r = 16 * gg + k;
        raw[k] = p < q ? y[p * 128 + r] : 0.0f;
        vals[k] = raw[k] * epi.wnext[row0 + r];
      }
      prep16(vals, raw, p, q, (row0 + 16 * gg) / 16, nt_out, epi.hi_scale, epi.next.frag, epi.next.sum, epi.next.ss,
             epi.H);
    }
  } else if (EPI == EPI_ROPE_KV) {
    const int head = grp, hd = epi.hd;
    const long long base = *epi.pos;
    for (int i = tid; i < q * (hd / 2); i += kG4Consumers) {
      const int p = i / (hd / 2), pr = i % (hd / 2);
      const float a = y[p * 128 + 2 * pr] * s_scale[p], b = y[p * 128 + 2 * pr + 1] * s_scale[p];
      const long long slot = base + p;
      const long long rope_pos = epi.parent ? base + tree_depth4(epi.parent, p) : slot;
      const int32_t page = epi.pages[slot / 64];
      if (head < epi.nh + epi.nkv) {
        const double inv = exp2(-(double)(2 * pr) / (double)hd * log2((double)epi.theta));
        double sn, cs;
        sincos((double)rope_pos * inv, &sn, &cs);
        const float c = (float)cs, s = (float)sn;
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
    const int nt_out = q <= 8 ? 1 : 2;
    for (int i = tid; i < 4 * 8 * nt_out; i += kG4Consumers) {
      const int gg = i % 4, p = i / 4;
      float vals[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) vals[k] = p < q ? y[p * 128 + 16 * gg + k] : 0.0f;
      prep16(vals, nullptr, p, q, (grp * 64 + 16 * gg) / 16, nt_out, epi.hi_scale, epi.next.frag, epi.next.sum,
             nullptr, epi.ffn);
    }
  }
  (void)s_ss;
  consumer_sync();  // y is reused by the next group
}

template <typename Raw, int NT, int EPI>
__global__ void __launch_bounds__(kG4Threads, 1) gemv4_kernel(const uint8_t* __restrict__ tiles, uint32_t rows,
                                                             int ng, G4Geom geo, int stages, XBuf in, int q, Epi epi,
                                                             float* __restrict__ part, int* __restrict__ counters,
                                                             int maxseg) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kG4MaxStages], empty[kG4MaxStages];
  __shared__ float s_scale[16];
  __shared__ float s_red[kG4Consumers];
  __shared__ int s_last;
  float* y = reinterpret_cast<float*>(smem + (size_t)stages * geo.stage_bytes);  // [16][128]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long U = (long long)ng * geo.ppr;
  const int G = gridDim.x;
  const long long u0 = (long long)blockIdx.x * U / G, u1 = (long long)(blockIdx.x + 1) * U / G;
  const int n = (int)(u1 - u0);
  UnitCursor start;
  start.grp = (int)(u0 / geo.ppr);
  start.pr = (int)(u0 - (long long)start.grp * geo.ppr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kG4Consumers / 32);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kG4Consumers / 32) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t policy = evict_first_policy();
      const int nsub = geo.sb * 8;
      auto issue_weights = [&](const UnitCursor& c) {
        const int nsb = min(2, geo.sb - 2 * c.pr);
        uint8_t* st = smem + (size_t)c.slot * geo.stage_bytes;
        const uint32_t wb = (uint32_t)(nsb * geo.sb_bytes);
        const uint32_t ab = (uint32_t)(nsb * NT * kXfragSbBytes + 2 * nsb * 512);
        mbar_expect_tx(&full[c.slot], wb + ab);
        bulk_g2s_stream(st, tiles + ((size_t)c.grp * geo.sb + 2 * c.pr) * geo.sb_bytes, wb, &full[c.slot], policy);
      };
      auto issue_acts = [&](const UnitCursor& c) {
        const int nsb = min(2, geo.sb - 2 * c.pr);
        uint8_t* st = smem + (size_t)c.slot * geo.stage_bytes;
        bulk_g2s(st + geo.frag_off, in.frag + (size_t)2 * c.pr * NT * 512, (uint32_t)(nsb * NT * kXfragSbBytes),
                 &full[c.slot]);
        for (int h = 0; h < 2; ++h)
          bulk_g2s(st + geo.sum_off + h * kG4SumBytes, in.sum + ((size_t)h * nsub + 16 * c.pr) * 16,
                   (uint32_t)(nsb * 512), &full[c.slot]);
      };
      const int pre = min(n, stages);
      UnitCursor w = start, a = start;
      for (int i = 0; i < pre; ++i, w.next(geo.ppr, stages)) issue_weights(w);
      griddep_wait();
      griddep_launch();
      for (int i = 0; i < pre; ++i, a.next(geo.ppr, stages)) issue_acts(a);
      for (int i = pre; i < n; ++i, w.next(geo.ppr, stages)) {
        if (!mbar_wait(&empty[w.slot], w.phase ^ 1u, epi.err)) break;  // the slot's previous use is consumed
        issue_weights(w);
        issue_acts(w);
      }
    } else {
      griddep_wait();
      griddep_launch();
    }
    return;
  }

  // ---------------- consumers ----------------
  griddep_wait();
  griddep_launch();
  const int t = lane % 4, g = lane / 4;
  const int tid = threadIdx.x;
  // row scale (folded rmsnorm) from the producer's sum-of-squares partials
  {
    const int p = tid % 16, c0 = tid / 16;
    float a = 0.0f;
    if (in.ss)
      for (int c = c0; c < in.nss; c += kG4Consumers / 16) a += in.ss[(size_t)c * 16 + p];
    s_red[tid] = a;
    consumer_sync();
    if (tid < 16) {
      float sc = 1.0f;
      if (in.ss && tid < q) {
        float tot = 0.0f;
        for (int c = 0; c < kG4Consumers / 16; ++c) tot += s_red[c * 16 + tid];
        sc = 1.0f / sqrtf(tot / epi.ss_n + epi.eps);
      }
      s_scale[tid] = sc;
    }
    consumer_sync();
  }

  const int rt = warp % kGemvWarps, hh = warp / kGemvWarps;  // row tile, superblock of the unit
  float acc[2][NT][4];
  auto zero_acc = [&]() {
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[a][nt][i] = 0.0f;
  };
  const int r0 = rt * 16 + g, r1 = r0 + 8;
  // y[p][r] (+)= this warp's accumulators (both chains)
  auto put = [&](float* dst, bool add) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int p0 = nt * 8 + 2 * t;
      const float v0 = acc[0][nt][0] + acc[1][nt][0], v1 = acc[0][nt][1] + acc[1][nt][1];
      const float v2 = acc[0][nt][2] + acc[1][nt][2], v3 = acc[0][nt][3] + acc[1][nt][3];
      if (p0 < q) {
        dst[p0 * 128 + r0] = add ? dst[p0 * 128 + r0] + v0 : v0;
        dst[p0 * 128 + r1] = add ? dst[p0 * 128 + r1] + v2 : v2;
      }
      if (p0 + 1 < q) {
        dst[(p0 + 1) * 128 + r0] = add ? dst[(p0 + 1) * 128 + r0] + v1 : v1;
        dst[(p0 + 1) * 128 + r1] = add ? dst[(p0 + 1) * 128 + r1] + v3 : v3;
      }
    }
  };
  auto flush = [&](int grp) {
    // this CTA's segment of the group: superblock-1 warps first, then superblock-0 warps add (fixed order)
    if (hh == 1) put(y, false);
    consumer_sync();
    if (hh == 0) put(y, true);
    consumer_sync();
    const int c_first = cta_of_unit((long long)grp * geo.ppr, U, G);
    const int c_last = cta_of_unit((long long)grp * geo.ppr + geo.ppr - 1, U, G);
    const int nseg = c_last - c_first + 1;
    if (nseg > 1) {
      const int seg = (int)blockIdx.x - c_first;
      float* mine = part + ((size_t)grp * maxseg + seg) * q * 128;
      for (int i = tid; i < q * 128; i += kG4Consumers) mine[i] = y[i];
      __threadfence();
      consumer_sync();
      if (tid == 0) s_last = atomicAdd(&counters[grp], 1) == nseg - 1;
      consumer_sync();
      if (!s_last) return;
      __threadfence();
      const float* all = part + (size_t)grp * maxseg * q * 128;
      for (int i = tid; i < q * 128; i += kG4Consumers) {
        float a = 0.0f;
        int k = 0;
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
      if (tid == 0) counters[grp] = 0;
      consumer_sync();
    }
    g4_epilogue<EPI>(y, s_scale, grp, rows, q, epi, nullptr);
  };

  zero_acc();
  int cur = n > 0 ? start.grp : -1;
  UnitCursor c = start;
  for (int i = 0; i < n; ++i, c.next(geo.ppr, stages)) {
    const int grp = c.grp, pr = c.pr, slot = c.slot;
    if (grp != cur) {
      flush(cur);
      cur = grp;
      zero_acc();
    }
    const int nsb = min(2, geo.sb - 2 * pr);
    mbar_wait(&full[slot], c.phase, epi.err);
    const uint8_t* st = smem + (size_t)slot * geo.stage_bytes;
    if (hh < nsb) {
      const uint2* xf = reinterpret_cast<const uint2*>(st + geo.frag_off) + hh * NT * 512;
      const float* s0 = reinterpret_cast<const float*>(st + geo.sum_off);
      const float* s1 = s0 + kG4SumBytes / 4;
      uint32_t mg, mg8;
      Raw r;
      load_raw_s(r, st + (size_t)hh * geo.sb_bytes + (size_t)rt * geo.tile_bytes, lane);
      tile_mmas<NT>(r, t, xf, lane, acc, mg, mg8);
      // min / bias term of this superblock: A = -m per (row, sub-block) in this warp's k-half of the pair,
      // B = fp16 hi + lo of the pair's sub-block sums
      const uint32_t a0 = hh == 0 ? mg : 0u, a1 = hh == 0 ? mg8 : 0u, a2 = hh == 1 ? mg : 0u, a3 = hh == 1 ? mg8 : 0u;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int p = nt * 8 + g;
        float v[4];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int sub = h2 * 8 + 2 * t + e;
            v[2 * h2 + e] = h2 < nsb ? s0[sub * 16 + p] + s1[sub * 16 + p] : 0.0f;
          }
        // fp16 hi + lo split of each sum (paired conversions)
        const __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(v[0] - f01.x, v[1] - f01.y);
        const __half2 l23 = __floats2half2_rn(v[2] - f23.x, v[3] - f23.y);
        mma16816(acc[0][nt], a0, a1, a2, a3, h2u(h01), h2u(h23));
        mma16816(acc[1][nt], a0, a1, a2, a3, h2u(l01), h2u(l23));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (cur >= 0) flush(cur);
}

// x[p][0:cols] (row stride ld) * w -> fragments / sums (+ ss); one thread per (16-column group, row).
__global__ void prep_rows_kernel(const float* __restrict__ x, long long ld, int q, int cols,
                                 const float* __restrict__ w, int nt, float hi_scale, uint2* __restrict__ frag,
                                 float* __restrict__ sum, float* __restrict__ ss) {
  griddep_wait();
  griddep_launch();
  const int groups = cols / 16;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= groups * 8 * nt) return;
  const int c = i % groups, p = i / groups;
  float vals[16], raw[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    raw[k] = p < q ? x[(size_t)p * ld + 16 * c + k] : 0.0f;
    vals[k] = w ? raw[k] * w[16 * c + k] : raw[k];
  }
  prep16(vals, ss ? raw : nullptr, p, q, c, nt, hi_scale, frag, sum, ss, cols);
}

int launch_prep_rows(const float* d_x, long long ld, int q, int cols, const float* d_w, int nt, float hi_scale,
                     const XBuf& out, bool with_ss, cudaStream_t st) {
  const int n = cols / 16 * 8 * nt;
  return launch_pdl(prep_rows_kernel, dim3((n + 127) / 128), dim3(128), 0, st, d_x, ld, q, cols, d_w, nt, hi_scale,
                    out.frag, out.sum, with_ss ? out.ss : nullptr);
}

template <typename Raw, int NT, int EPI>
static int launch4(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q,
                   const Epi& epi, float* part, int* counters, cudaStream_t st) {
  auto kern = gemv4_kernel<Raw, NT, EPI>;
  CLM_TRY(ensure_smem(kern, p.smem));
  G4Geom geo;
  geo.sb = (int)s.sb;
  geo.ppr = (int)(s.sb + 1) / 2;
  geo.tile_bytes = s.tile_bytes;
  geo.sb_bytes = kGemvWarps * s.tile_bytes;
  geo.frag_off = 2 * geo.sb_bytes;
  geo.sum_off = geo.frag_off + 2 * NT * kXfragSbBytes;
  geo.stage_bytes = geo.sum_off + 2 * kG4SumBytes;
  return launch_pdl(kern, dim3((unsigned)p.grid), dim3(kG4Threads), p.smem, st, d_tiles, s.rows, (int)s.ng, geo,
                    p.stages, in, q, epi, part, counters, p.ksplit);
}

template <typename Raw, int NT>
static int launch4_epi(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q,
                       const Epi& epi, float* part, int* counters, cudaStream_t st) {
  switch (epi.kind) {
    case EPI_STORE: return launch4<Raw, NT, EPI_STORE>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_RESID_PREP: return launch4<Raw, NT, EPI_RESID_PREP>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_ROPE_KV: return launch4<Raw, NT, EPI_ROPE_KV>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_SWIGLU_PREP: return launch4<Raw, NT, EPI_SWIGLU_PREP>(s, p, d_tiles, in, q, epi, part, counters, st);
  }
  return fail(CLM_INTERNAL, "unknown GEMV epilogue");
}

int launch_gemv(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi,
                float* part, int* counters, cudaStream_t st) {
  CLM_CHECK(q >= 1 && q <= 8 * p.nt, CLM_INTERNAL, "GEMV plan does not cover the window width");
  if (s.quant == CLM_QUANT_Q4_K)
    return p.nt == 1 ? launch4_epi<RawQ4k, 1>(s, p, d_tiles, in, q, epi, part, counters, st)
                     : launch4_epi<RawQ4k, 2>(s, p, d_tiles, in, q, epi, part, counters, st);
  return p.nt == 1 ? launch4_epi<RawQ80, 1>(s, p, d_tiles, in, q, epi, part, counters, st)
                   : launch4_epi<RawQ80, 2>(s, p, d_tiles, in, q, epi, part, counters, st);
}

}  // namespace clm
