// gemv3.cu — the fused-epilogue q-row GEMV used by the engines (design notes in gemv2.cuh / gemv.cuh).
//
// A CTA computes 128 rows (8 row tiles, one per warp) over a k-chunk of superblocks, exactly like the tiled
// kernel of gemv.cu, then:
//  * with one k-chunk per row group it keeps the 128 x q results in shared memory;
//  * with several it writes its partial, and the LAST CTA to finish a row group (atomic counter) sums the
//    partials in k-chunk order (deterministic) — no separate reduction kernel;
// and that CTA runs the epilogue on the 128 rows: a row scale folded from the previous producer's
// sum-of-squares partials (rmsnorm), then store / residual + next-input preparation / RoPE + paged KV append /
// SwiGLU + next-input preparation.
#include "gemv2.cuh"
#include "gemv_tile.cuh"
#include "pdl.cuh"

namespace clm {

__device__ __forceinline__ long long tree_depth3(const int32_t* parent, int i) {
  long long d = 0;
  for (int a = parent[i]; a >= 0 && d < 64; a = parent[a]) ++d;
  return d;
}

template <typename Raw, int NT, int EPI>
__global__ void __launch_bounds__(256) gemv3_kernel(const uint8_t* __restrict__ tiles, uint32_t rows,
                                                   uint32_t sb_per_row, int tile_bytes, int ksplit, int sbps,
                                                   XBuf in, int q, Epi epi, float* __restrict__ part,
                                                   int* __restrict__ counters) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int grp = blockIdx.x / ksplit, ks = blockIdx.x % ksplit;
  const int sb0 = ks * sbps;
  const int sb1 = min((int)sb_per_row, sb0 + sbps);
  const int nsb = sb1 - sb0;
  const int pairs_local = (nsb + 1) / 2;
  uint2* xf = reinterpret_cast<uint2*>(smem);
  uint4* xs = reinterpret_cast<uint4*>(smem + (size_t)NT * sbps * kXfragSbBytes);
  float* y = reinterpret_cast<float*>(smem + (size_t)NT * sbps * kXfragSbBytes + (size_t)NT * ((sbps + 1) / 2) * kXsPairBytes);
  __shared__ float s_scale[16];
  __shared__ int s_last;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, t = lane % 4, g = lane / 4;
  const uint8_t* tile0 = tiles + ((size_t)(grp * sb_per_row + sb0) * kGemvWarps + warp) * tile_bytes;
  const size_t sb_stride = (size_t)kGemvWarps * tile_bytes;

  Raw cur, nxt;
  load_raw(cur, tile0, lane);  // weights are immutable: fetched before waiting for the producer
  griddep_wait();
  griddep_launch();

  // stage the activation fragments of this k-chunk and the sub-block sums (f32 halves -> fp16 hi/lo)
  {
    const uint4* src = reinterpret_cast<const uint4*>(in.frag + (size_t)sb0 * NT * 512);
    uint4* dst = reinterpret_cast<uint4*>(xf);
    for (int i = threadIdx.x; i < nsb * NT * 256; i += blockDim.x) dst[i] = __ldg(src + i);
    const int nsub = (int)sb_per_row * 8;
    for (int i = threadIdx.x; i < pairs_local * NT * 32; i += blockDim.x) {
      const int ln = i % 32, nt = (i / 32) % NT, pl = i / (32 * NT);
      const int p = nt * 8 + ln / 4, tt = ln % 4;
      float v[4];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int sb = sb0 + 2 * pl + hh;
          float a = 0.0f;
          if (sb < sb1) {
            const int j = sb * 8 + 2 * tt + e;
            a = in.sum[(size_t)j * 16 + p] + in.sum[((size_t)nsub + j) * 16 + p];
          }
          v[2 * hh + e] = a;
        }
      float hi[4], lo[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        hi[k] = __half2float(__float2half_rn(v[k]));
        lo[k] = v[k] - hi[k];
      }
      xs[i] = make_uint4(pack_half2(hi[0], hi[1]), pack_half2(hi[2], hi[3]), pack_half2(lo[0], lo[1]),
                         pack_half2(lo[2], lo[3]));
    }
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

  // results of this CTA for its 128 rows: y[p][r]
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  auto put = [&](float* dst) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int p0 = nt * 8 + 2 * t;
      if (p0 < q) {
        dst[p0 * 128 + r0] = acc[nt][0];
        dst[p0 * 128 + r1] = acc[nt][2];
      }
      if (p0 + 1 < q) {
        dst[(p0 + 1) * 128 + r0] = acc[nt][1];
        dst[(p0 + 1) * 128 + r1] = acc[nt][3];
      }
    }
  };
  if (ksplit == 1) {
    put(y);
  } else {
    float* mine = part + ((size_t)grp * ksplit + ks) * q * 128;
    put(mine);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[grp], 1) == ksplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* all = part + (size_t)grp * ksplit * q * 128;
    for (int i = threadIdx.x; i < q * 128; i += blockDim.x) {
      float a = 0.0f;
      for (int k = 0; k < ksplit; ++k) a += __ldcg(all + (size_t)k * q * 128 + i);
      y[i] = a;
    }
    if (threadIdx.x == 0) counters[grp] = 0;
  }
  // row scale (folded rmsnorm)
  if (threadIdx.x < 16) {
    float sc = 1.0f;
    if (in.ss && (int)threadIdx.x < q) {
      float a = 0.0f;
      for (int c = 0; c < in.nss; ++c) a += in.ss[(size_t)c * 16 + threadIdx.x];
      sc = 1.0f / sqrtf(a / epi.ss_n + epi.eps);
    }
    s_scale[threadIdx.x] = sc;
  }
  __syncthreads();

  const int row0 = grp * 128;
  if (EPI == EPI_STORE) {
    for (int i = threadIdx.x; i < q * 128; i += blockDim.x) {
      const int p = i / 128, r = i % 128;
      if (row0 + r < (int)rows) epi.out[(size_t)p * epi.out_ld + row0 + r] = y[i] * s_scale[p];
    }
  } else if (EPI == EPI_RESID_PREP) {
    for (int i = threadIdx.x; i < q * 128; i += blockDim.x) {
      const int p = i / 128, r = i % 128;
      if (row0 + r >= (int)rows) continue;
      float* hp = epi.h + (size_t)p * epi.H + row0 + r;
      const float hn = *hp + y[i] * s_scale[p];
      *hp = hn;
      y[i] = hn;
    }
    __syncthreads();
    const int nt_out = q <= 8 ? 1 : 2;
    for (int i = threadIdx.x; i < 8 * 8 * nt_out; i += blockDim.x) {
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
    const int head = grp, hd = epi.hd, qd = epi.nh * hd;
    (void)qd;
    const long long base = *epi.pos;
    for (int i = threadIdx.x; i < q * (hd / 2); i += blockDim.x) {
      const int p = i / (hd / 2), pr = i % (hd / 2);
      const float a = y[p * 128 + 2 * pr] * s_scale[p], b = y[p * 128 + 2 * pr + 1] * s_scale[p];
      const long long slot = base + p;
      const long long rope_pos = epi.parent ? base + tree_depth3(epi.parent, p) : slot;
      const int32_t page = epi.pages[slot / 64];
      if (head < epi.nh + epi.nkv) {
        const double inv = exp2(-(double)(2 * pr) / (double)hd * log2((double)epi.theta));
        double sn, cs;
        sincos((double)rope_pos * inv, &sn, &cs);
        const float c = (float)cs, s = (float)sn;
        const float ra = a * c - b * s, rb = a * s + b * c;
        __half* dst;
        if (head < epi.nh)
          dst = epi.q16 + ((size_t)p * epi.nh + head) * hd + 2 * pr;
        else
          dst = epi.kpool + (((size_t)page * epi.nkv + (head - epi.nh)) * 64 + slot % 64) * hd + 2 * pr;
        dst[0] = __float2half_rn(ra);
        dst[1] = __float2half_rn(rb);
      } else {
        __half* vt = epi.vpool + (((size_t)page * epi.nkv + (head - epi.nh - epi.nkv)) * hd + 2 * pr) * 64 + slot % 64;
        vt[0] = __float2half_rn(a);
        vt[64] = __float2half_rn(b);
      }
    }
  } else if (EPI == EPI_SWIGLU_PREP) {
    // rows [0, 64) gate, [64, 128) up of ffn indices grp*64 + [0, 64)
    for (int i = threadIdx.x; i < q * 64; i += blockDim.x) {
      const int p = i / 64, k = i % 64;
      const float gv = y[p * 128 + k] * s_scale[p], uv = y[p * 128 + 64 + k] * s_scale[p];
      y[p * 128 + k] = gv / (1.0f + expf(-gv)) * uv;
    }
    __syncthreads();
    const int nt_out = q <= 8 ? 1 : 2;
    for (int i = threadIdx.x; i < 4 * 8 * nt_out; i += blockDim.x) {
      const int gg = i % 4, p = i / 4;
      float vals[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) vals[k] = p < q ? y[p * 128 + 16 * gg + k] : 0.0f;
      prep16(vals, nullptr, p, q, (grp * 64 + 16 * gg) / 16, nt_out, epi.hi_scale, epi.next.frag, epi.next.sum,
             nullptr, epi.ffn);
    }
  }
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

size_t gemv3_smem(const GemvPlan& p) {
  return (size_t)p.nt * p.sbps * kXfragSbBytes + (size_t)p.nt * ((p.sbps + 1) / 2) * kXsPairBytes +
         (size_t)16 * 128 * sizeof(float);
}

template <typename Raw, int NT, int EPI>
static int launch3(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q,
                   const Epi& epi, float* part, int* counters, cudaStream_t st) {
  auto kern = gemv3_kernel<Raw, NT, EPI>;
  const size_t smem = gemv3_smem(p);
  CLM_TRY(ensure_smem(kern, smem));
  return launch_pdl(kern, dim3(s.ng * (unsigned)p.ksplit), dim3(256), smem, st, d_tiles, s.rows, s.sb, s.tile_bytes,
                    p.ksplit, p.sbps, in, q, epi, part, counters);
}

template <typename Raw, int NT>
static int launch3_epi(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q,
                       const Epi& epi, float* part, int* counters, cudaStream_t st) {
  switch (epi.kind) {
    case EPI_STORE: return launch3<Raw, NT, EPI_STORE>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_RESID_PREP: return launch3<Raw, NT, EPI_RESID_PREP>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_ROPE_KV: return launch3<Raw, NT, EPI_ROPE_KV>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_SWIGLU_PREP: return launch3<Raw, NT, EPI_SWIGLU_PREP>(s, p, d_tiles, in, q, epi, part, counters, st);
  }
  return fail(CLM_INTERNAL, "unknown GEMV epilogue");
}

int launch_gemv3(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi,
                 float* part, int* counters, cudaStream_t st) {
  if (s.quant == CLM_QUANT_Q4_K)
    return p.nt == 1 ? launch3_epi<RawQ4k, 1>(s, p, d_tiles, in, q, epi, part, counters, st)
                     : launch3_epi<RawQ4k, 2>(s, p, d_tiles, in, q, epi, part, counters, st);
  return p.nt == 1 ? launch3_epi<RawQ80, 1>(s, p, d_tiles, in, q, epi, part, counters, st)
                   : launch3_epi<RawQ80, 2>(s, p, d_tiles, in, q, epi, part, counters, st);
}

}  // namespace clm
