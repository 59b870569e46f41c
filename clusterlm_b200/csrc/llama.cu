// llama.cu — per-layer kernels of the Llama-shaped decoder family (see llama.cuh).
#include <cfloat>

#include "gemv2.cuh"
#include "llama.cuh"
#include "pdl.cuh"

namespace clm {

// ---------------------------------------------------------------------------------------------------
// embedding: exact dequantisation of one GGUF row per window position
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ float ld_half_le(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__global__ void embed_kernel(const uint8_t* __restrict__ embd, int quant, const int32_t* __restrict__ tokens, int H,
                             float* __restrict__ h) {
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x;
  const int32_t tok = tokens[p];
  float* out = h + (size_t)p * H;
  if (quant == CLM_QUANT_Q4_K) {
    const uint8_t* row = embd + (size_t)tok * (H / 256) * 144;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const uint8_t* b = row + (i / 256) * 144;
      const int e = i % 256, j = e / 32, l = e % 32;
      const uint8_t* sc = b + 4;
      int s, m;
      if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      const float ds = __fmul_rn(ld_half_le(b), (float)s), dm = __fmul_rn(ld_half_le(b + 2), (float)m);
      const int qv = (b[16 + 32 * (j / 2) + l] >> ((j & 1) ? 4 : 0)) & 0xF;
      out[i] = __fsub_rn(__fmul_rn(ds, (float)qv), dm);
    }
  } else {
    const uint8_t* row = embd + (size_t)tok * (H / 32) * 34;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const uint8_t* b = row + (i / 32) * 34;
      out[i] = __fmul_rn(ld_half_le(b), (float)(int8_t)b[2 + i % 32]);
    }
  }
}

int launch_embed(const uint8_t* d_embd, int quant, const int32_t* d_tokens, int q, int H, float* d_h, cudaStream_t st) {
  return launch_pdl(embed_kernel, dim3(q), dim3(256), 0, st, d_embd, quant, d_tokens, H, d_h);
}

// ---------------------------------------------------------------------------------------------------
// residual + RMSNorm -> GEMV fragments
// ---------------------------------------------------------------------------------------------------
__device__ float block_sum_f(float v) {
  __shared__ float sm[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x / 32) ? sm[lane] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  v = sm[0];
  __syncthreads();
  return v;
}

__global__ void __launch_bounds__(512) norm_kernel(const float* __restrict__ part, int nsplit, int part_rows, int q,
                                                   int H, const float* __restrict__ w, float eps, float* h, int nt,
                                                   float hi_scale, uint2* __restrict__ xfrag, uint4* __restrict__ xs) {
  extern __shared__ float smem[];
  float* x = smem;           // H
  float* sums = smem + H;    // H / 32
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x;
  if (p >= q) {
    write_xfrag_row(nullptr, p, H, nt, hi_scale, xfrag, xs, sums);
    return;
  }
  float* hr = h + (size_t)p * H;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = hr[i];
    for (int s = 0; s < nsplit; ++s) v += part[((size_t)s * q + p) * part_rows + i];
    hr[i] = v;
    x[i] = v;
    ss += v * v;
  }
  ss = block_sum_f(ss);
  const float denom = sqrtf(ss / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) x[i] = x[i] * w[i] / denom;
  __syncthreads();
  write_xfrag_row(x, p, H, nt, hi_scale, xfrag, xs, sums);
}

int launch_norm(const float* d_part, int nsplit, int part_rows, int q, int H, const float* d_w, float eps, float* d_h,
                int nt, float hi_scale, void* d_xfrag, void* d_xs, cudaStream_t st) {
  const size_t smem = (size_t)H * 4 + (size_t)H / 32 * 4;
  CLM_TRY(ensure_smem(norm_kernel, smem));
  return launch_pdl(norm_kernel, dim3(8 * nt), dim3(512), smem, st, d_part, nsplit, part_rows, q, H, d_w, eps, d_h, nt,
                    hi_scale, static_cast<uint2*>(d_xfrag), static_cast<uint4*>(d_xs));
}

// ---------------------------------------------------------------------------------------------------
// RoPE + paged KV append
// ---------------------------------------------------------------------------------------------------
// K pool: [page][nkv][64][hd] fp16; V pool (transposed): [page][nkv][hd][64] fp16.
__device__ __forceinline__ long long tree_depth(const int32_t* parent, int i) {
  long long d = 0;
  for (int a = parent[i]; a >= 0 && d < 64; a = parent[a]) ++d;
  return d;
}

__global__ void rope_kv_kernel(const float* __restrict__ part, int nsplit, int q, int nh, int nkv, int hd, float theta,
                               const long long* __restrict__ d_pos, const int32_t* __restrict__ parent,
                               const int32_t* __restrict__ pages, __half* __restrict__ kpool,
                               __half* __restrict__ vpool, __half* __restrict__ q16) {
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x, head = blockIdx.y, i = threadIdx.x;  // pair (2i, 2i+1)
  if (2 * i >= hd) return;
  const int qd = nh * hd, kvd = nkv * hd, cols = qd + 2 * kvd;
  const long long base = *d_pos;
  const long long slot = base + p;
  const long long rope_pos = parent ? base + tree_depth(parent, p) : slot;
  auto val = [&](int c) {
    float v = 0.0f;
    for (int s = 0; s < nsplit; ++s) v += part[((size_t)s * q + p) * cols + c];
    return v;
  };
  if (head < nh + nkv) {
    const int col = head < nh ? head * hd : qd + (head - nh) * hd;
    const float a = val(col + 2 * i), b = val(col + 2 * i + 1);
    const double inv = exp2(-(double)(2 * i) / (double)hd * log2((double)theta));
    double sn, cs;
    sincos((double)rope_pos * inv, &sn, &cs);
    const float c = (float)cs, s = (float)sn;
    const float ra = a * c - b * s, rb = a * s + b * c;
    if (head < nh) {
      __half* dst = q16 + ((size_t)p * nh + head) * hd + 2 * i;
      dst[0] = __float2half_rn(ra);
      dst[1] = __float2half_rn(rb);
    } else {
      const int j = head - nh;
      const int32_t page = pages[slot / kPageTokens];
      __half* dst = kpool + (((size_t)page * nkv + j) * kPageTokens + slot % kPageTokens) * hd + 2 * i;
      dst[0] = __float2half_rn(ra);
      dst[1] = __float2half_rn(rb);
    }
  } else {
    const int j = head - nh - nkv;
    const int col = qd + kvd + j * hd;
    const int32_t page = pages[slot / kPageTokens];
    __half* vt = vpool + (((size_t)page * nkv + j) * hd + 2 * i) * kPageTokens + slot % kPageTokens;
    vt[0] = __float2half_rn(val(col + 2 * i));
    vt[kPageTokens] = __float2half_rn(val(col + 2 * i + 1));
  }
}

int launch_rope_kv(const float* d_part, int nsplit, int q, const LlamaDims& d, const long long* d_pos,
                   const int32_t* d_parent, const int32_t* d_pages, __half* d_k, __half* d_v, __half* d_q,
                   cudaStream_t st) {
  return launch_pdl(rope_kv_kernel, dim3(q, d.nh + 2 * d.nkv), dim3(d.hd / 2), 0, st, d_part, nsplit, q, d.nh, d.nkv,
                    d.hd, d.theta, d_pos, d_parent, d_pages, d_k, d_v, d_q);
}

// ---------------------------------------------------------------------------------------------------
// attention over the paged fp16 cache: one warp per (m-tile of 16 query rows, kv head, page of 64 positions)
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word_of(const uint4 (&v)[4], int w) {
  const uint4& u = v[w / 4];
  return (w % 4 == 0) ? u.x : (w % 4 == 1) ? u.y : (w % 4 == 2) ? u.z : u.w;
}

// Visibility of absolute position `pos` to window row i.
__device__ __forceinline__ bool visible(long long pos, long long base, int i, const int32_t* parent) {
  if (pos < base) return true;
  const long long rel = pos - base;
  if (!parent) return rel <= i;
  for (int a = i, guard = 0; a >= 0 && guard < 64; a = parent[a], ++guard)
    if (a == rel) return true;
  return false;
}

template <int HD>
__global__ void __launch_bounds__(32 * kAttnWarps) attention_kernel(
    const __half* __restrict__ q16, const __half* __restrict__ kpool, const __half* __restrict__ vpool,
    const int32_t* __restrict__ pages, const long long* __restrict__ d_pos, const int32_t* __restrict__ parent, int q,
    int nh, int nkv, float scale_log2, int max_pages, float* __restrict__ part, int* __restrict__ counters, int nt_out,
    float hi_scale, uint2* __restrict__ out_frag, float* __restrict__ out_sum) {
  static_assert(HD == 128, "head_dim 128 layout");
  constexpr int RW = HD + 2;  // one partial row: O[HD], m, l
  __shared__ float sp[kAttnWarps][16][RW];
  __shared__ int s_last;
  griddep_wait();
  griddep_launch();
  const int kvh = blockIdx.x, mt = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, t = lane % 4;
  const int pg = blockIdx.y * kAttnWarps + warp;
  const int group = nh / nkv;
  const long long base = *d_pos;
  const long long nvis = base + q;
  const int npages = (int)((nvis + kPageTokens - 1) / kPageTokens);
  const int ngroups = (npages + kAttnWarps - 1) / kAttnWarps;
  const int r0 = mt * 16 + g, r1 = r0 + 8;
  const int i0 = r0 / group, i1 = r1 / group;
  const bool v0 = i0 < q, v1 = i1 < q;
  const bool active = pg < npages && pg < max_pages;

  if (active) {
    const int32_t page = pages[pg];
    // Q fragments: thread t holds head dims [32t, 32t+32) of rows r0 and r1.
    uint4 qw0[4], qw1[4];
    {
      const uint4 z = make_uint4(0, 0, 0, 0);
      const uint4* a = reinterpret_cast<const uint4*>(q16 + ((size_t)i0 * nh + kvh * group + r0 % group) * HD + 32 * t);
      const uint4* b = reinterpret_cast<const uint4*>(q16 + ((size_t)i1 * nh + kvh * group + r1 % group) * HD + 32 * t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qw0[j] = v0 ? a[j] : z;
        qw1[j] = v1 ? b[j] : z;
      }
    }
    // S = Q K^T over the 64 positions of the page; n-tile j column c <-> position 16*(c/2) + 2j + c%2.
    const __half* kpage = kpool + ((size_t)page * nkv + kvh) * kPageTokens * HD;
    float S[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.0f;
      const int pos = 16 * (g / 2) + 2 * j + (g % 2);
      const uint4* kr = reinterpret_cast<const uint4*>(kpage + (size_t)pos * HD + 32 * t);
      uint4 kw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) kw[u] = kr[u];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        mma_f16(S[j], word_of(qw0, 2 * ks), word_of(qw1, 2 * ks), word_of(qw0, 2 * ks + 1), word_of(qw1, 2 * ks + 1),
                word_of(kw, 2 * ks), word_of(kw, 2 * ks + 1));
    }
    float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const long long pos = (long long)pg * kPageTokens + 16 * t + 2 * j + e;
        S[j][e] = (v0 && visible(pos, base, i0, parent)) ? S[j][e] * scale_log2 : -INFINITY;
        S[j][2 + e] = (v1 && visible(pos, base, i1, parent)) ? S[j][2 + e] * scale_log2 : -INFINITY;
        m0 = fmaxf(m0, S[j][e]);
        m1 = fmaxf(m1, S[j][2 + e]);
      }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    float l0 = 0.0f, l1 = 0.0f;
    uint32_t pa[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p00 = m0 == -INFINITY ? 0.0f : exp2f(S[j][0] - m0);
      const float p01 = m0 == -INFINITY ? 0.0f : exp2f(S[j][1] - m0);
      const float p10 = m1 == -INFINITY ? 0.0f : exp2f(S[j][2] - m1);
      const float p11 = m1 == -INFINITY ? 0.0f : exp2f(S[j][3] - m1);
      l0 += p00 + p01;
      l1 += p10 + p11;
      pa[j][0] = pack_half2(p00, p01);
      pa[j][1] = pack_half2(p10, p11);
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    const __half* vpage = vpool + ((size_t)page * nkv + kvh) * HD * kPageTokens;
#pragma unroll 4
    for (int jn = 0; jn < HD / 8; ++jn) {
      float O[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint4* vr = reinterpret_cast<const uint4*>(vpage + (size_t)(8 * jn + g) * kPageTokens + 16 * t);
      const uint4 va = vr[0], vb = vr[1];
      const uint32_t vw[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16(O, pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1], vw[2 * kk], vw[2 * kk + 1]);
      sp[warp][g][8 * jn + 2 * t] = O[0];
      sp[warp][g][8 * jn + 2 * t + 1] = O[1];
      sp[warp][g + 8][8 * jn + 2 * t] = O[2];
      sp[warp][g + 8][8 * jn + 2 * t + 1] = O[3];
    }
    if (t == 0) {
      sp[warp][g][HD] = m0;
      sp[warp][g][HD + 1] = l0;
      sp[warp][g + 8][HD] = m1;
      sp[warp][g + 8][HD + 1] = l1;
    }
  } else {
    for (int i = lane; i < 16; i += 32) {
      sp[warp][i][HD] = -INFINITY;
      sp[warp][i][HD + 1] = 0.0f;
    }
  }
  __syncthreads();
  // combine the CTA's pages into one partial per (m-tile, kv head, page group)
  float* mine = part + (((size_t)mt * nkv + kvh) * max_pages + blockIdx.y) * 16 * RW;
  if ((int)blockIdx.y < ngroups) {
    for (int i = threadIdx.x; i < 16 * RW; i += blockDim.x) {
      const int r = i / RW, c = i % RW;
      float M = -INFINITY;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sp[w][r][HD]);
      float a = 0.0f;
      if (c == HD) {
        a = M;
      } else {
        for (int w = 0; w < kAttnWarps; ++w) {
          const float m = sp[w][r][HD];
          if (m == -INFINITY) continue;
          a += sp[w][r][c] * exp2f(m - M);
        }
      }
      mine[i] = a;
    }
  }
  // the last CTA of this (m-tile, kv head) combines the page groups and writes W_o's input fragments
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[mt * nkv + kvh], 1) == (int)gridDim.y - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* allp = part + ((size_t)mt * nkv + kvh) * max_pages * 16 * RW;
  __shared__ float o_s[16][HD];
  __shared__ float wmax[16], wsum[16];
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float M = -INFINITY;
    for (int gi = 0; gi < ngroups; ++gi) M = fmaxf(M, __ldcg(allp + ((size_t)gi * 16 + r) * RW + HD));
    float L = 0.0f;
    for (int gi = 0; gi < ngroups; ++gi) {
      const float m = __ldcg(allp + ((size_t)gi * 16 + r) * RW + HD);
      if (m != -INFINITY) L += __ldcg(allp + ((size_t)gi * 16 + r) * RW + HD + 1) * exp2f(m - M);
    }
    wmax[r] = M;
    wsum[r] = L > 0.0f ? 1.0f / L : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * HD; i += blockDim.x) {
    const int r = i / HD, c = i % HD;
    float a = 0.0f;
    for (int gi = 0; gi < ngroups; ++gi) {
      const float m = __ldcg(allp + ((size_t)gi * 16 + r) * RW + HD);
      if (m != -INFINITY) a += __ldcg(allp + ((size_t)gi * 16 + r) * RW + c) * exp2f(m - wmax[r]);
    }
    o_s[r][c] = a * wsum[r];
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[mt * nkv + kvh] = 0;
  // fragments: query vector r = window row i, head kvh*group + r%group; 8 column groups of 16 per head
  const int qd = nh * HD;
  for (int it = threadIdx.x; it < 16 * (HD / 16); it += blockDim.x) {
    const int r = it / (HD / 16), gg = it % (HD / 16);
    const int i = (mt * 16 + r) / group, head = kvh * group + (mt * 16 + r) % group;
    if (i >= q) continue;
    prep16(&o_s[r][16 * gg], nullptr, i, q, (head * HD + 16 * gg) / 16, nt_out, hi_scale, out_frag, out_sum, nullptr,
           qd);
  }
}

int launch_attention(const __half* d_q, const __half* d_k, const __half* d_v, const int32_t* d_pages,
                     const long long* d_pos, const int32_t* d_parent, int q, const LlamaDims& d, int max_pages,
                     float* d_part, int* d_counters, int nt_out, float hi_scale, void* d_frag, float* d_sum,
                     cudaStream_t st) {
  CLM_CHECK(d.hd == 128, CLM_UNIMPLEMENTED, "attention kernel supports head_dim 128");
  const int group = d.nh / d.nkv;
  const int mtiles = (q * group + 15) / 16;
  const float scale_log2 = (float)(1.4426950408889634 / sqrt((double)d.hd));
  return launch_pdl(attention_kernel<128>, dim3(d.nkv, (max_pages + kAttnWarps - 1) / kAttnWarps, mtiles),
                    dim3(32 * kAttnWarps), 0, st, d_q, d_k, d_v, d_pages, d_pos, d_parent, q, d.nh, d.nkv, scale_log2,
                    max_pages, d_part, d_counters, nt_out, hi_scale, static_cast<uint2*>(d_frag), d_sum);
}

// ---------------------------------------------------------------------------------------------------
// combine page partials -> attention output row -> GEMV fragments for W_o
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) attn_combine_kernel(const float* __restrict__ part,
                                                           const long long* __restrict__ d_pos, int q, int nh, int nkv,
                                                           int hd, int max_pages, int nt, float hi_scale,
                                                           uint2* __restrict__ xfrag, uint4* __restrict__ xs) {
  extern __shared__ float smem[];
  const int qd = nh * hd;
  float* o = smem;              // qd
  float* sums = smem + qd;      // qd / 32
  float* wts = sums + qd / 32;  // nh * max_pages weights
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x;
  if (p >= q) {
    write_xfrag_row(nullptr, p, qd, nt, hi_scale, xfrag, xs, sums);
    return;
  }
  const int group = nh / nkv;
  const long long nvis = *d_pos + q;
  const int npages = (int)((nvis + kPageTokens - 1) / kPageTokens);
  // per head: weights exp2(m_pg - M) / L
  for (int h = threadIdx.x; h < nh; h += blockDim.x) {
    const int kvh = h / group, r = p * group + h % group, mt = r / 16, rr = r % 16;
    const float* base = part + ((size_t)mt * nkv + kvh) * max_pages * 16 * (hd + 2) + (size_t)rr * (hd + 2);
    float M = -INFINITY;
    for (int pg = 0; pg < npages; ++pg) M = fmaxf(M, base[(size_t)pg * 16 * (hd + 2) + hd]);
    float L = 0.0f;
    for (int pg = 0; pg < npages; ++pg) {
      const float m = base[(size_t)pg * 16 * (hd + 2) + hd];
      const float w = m == -INFINITY ? 0.0f : exp2f(m - M);
      wts[h * max_pages + pg] = w;
      L += w * base[(size_t)pg * 16 * (hd + 2) + hd + 1];
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int pg = 0; pg < npages; ++pg) wts[h * max_pages + pg] *= inv;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < qd; c += blockDim.x) {
    const int h = c / hd, dd = c % hd;
    const int kvh = h / group, r = p * group + h % group, mt = r / 16, rr = r % 16;
    const float* base = part + ((size_t)mt * nkv + kvh) * max_pages * 16 * (hd + 2) + (size_t)rr * (hd + 2) + dd;
    float a = 0.0f;
    for (int pg = 0; pg < npages; ++pg) a += wts[h * max_pages + pg] * base[(size_t)pg * 16 * (hd + 2)];
    o[c] = a;
  }
  __syncthreads();
  write_xfrag_row(o, p, qd, nt, hi_scale, xfrag, xs, sums);
}

int launch_attn_combine(const float* d_part, const long long* d_pos, int q, const LlamaDims& d, int max_pages, int nt,
                        float hi_scale, void* d_xfrag, void* d_xs, cudaStream_t st) {
  const size_t smem = (size_t)d.qd() * 4 + (size_t)d.qd() / 32 * 4 + (size_t)d.nh * max_pages * 4;
  CLM_CHECK(smem <= 200 * 1024, CLM_RESOURCE_EXHAUSTED, "attention combine needs too much shared memory");
  CLM_TRY(ensure_smem(attn_combine_kernel, smem));
  return launch_pdl(attn_combine_kernel, dim3(8 * nt), dim3(512), smem, st, d_part, d_pos, q, d.nh, d.nkv, d.hd,
                    max_pages, nt, hi_scale, static_cast<uint2*>(d_xfrag), static_cast<uint4*>(d_xs));
}

// ---------------------------------------------------------------------------------------------------
// SwiGLU: a = silu(gate) * up (reference_math.hpp:32 silu = z / (1 + exp(-z)))
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) swiglu_kernel(const float* __restrict__ part, int nsplit, int q, int F, int nt,
                                                      float hi_scale, uint2* __restrict__ xfrag,
                                                      uint4* __restrict__ xs) {
  extern __shared__ float smem[];
  float* a = smem;
  float* sums = smem + F;
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x;
  if (p >= q) {
    write_xfrag_row(nullptr, p, F, nt, hi_scale, xfrag, xs, sums);
    return;
  }
  for (int i = threadIdx.x; i < F; i += blockDim.x) {
    float gsum = 0.0f, usum = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
      const float* row = part + ((size_t)s * q + p) * 2 * F;
      gsum += row[i];
      usum += row[F + i];
    }
    a[i] = gsum / (1.0f + expf(-gsum)) * usum;
  }
  __syncthreads();
  write_xfrag_row(a, p, F, nt, hi_scale, xfrag, xs, sums);
}

int launch_swiglu(const float* d_part, int nsplit, int q, int F, int nt, float hi_scale, void* d_xfrag, void* d_xs,
                  cudaStream_t st) {
  const size_t smem = (size_t)F * 4 + (size_t)F / 32 * 4;
  CLM_CHECK(smem <= 200 * 1024, CLM_RESOURCE_EXHAUSTED, "SwiGLU row does not fit in shared memory");
  CLM_TRY(ensure_smem(swiglu_kernel, smem));
  return launch_pdl(swiglu_kernel, dim3(8 * nt), dim3(1024), smem, st, d_part, nsplit, q, F, nt, hi_scale,
                    static_cast<uint2*>(d_xfrag), static_cast<uint4*>(d_xs));
}

// ---------------------------------------------------------------------------------------------------
// stage boundary records (hc = 1): {S[H], P[H], g}
// ---------------------------------------------------------------------------------------------------
__global__ void pack_boundary_kernel(const float* __restrict__ h, const float* __restrict__ part, int nsplit, int q,
                                     int H, float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.y;
  float* rec = out + (size_t)p * (2 * H + 1);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) {
    float v = h[(size_t)p * H + i];
    for (int s = 0; s < nsplit; ++s) v += part[((size_t)s * q + p) * H + i];
    rec[i] = v;
    rec[H + i] = 0.0f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) rec[2 * H] = 1.0f;
}

int launch_pack_boundary(const float* d_h, const float* d_part, int nsplit, int q, int H, float* d_out,
                         cudaStream_t st) {
  return launch_pdl(pack_boundary_kernel, dim3(8, q), dim3(256), 0, st, d_h, d_part, nsplit, q, H, d_out);
}

__global__ void unpack_boundary_kernel(const float* __restrict__ in, int H, float* __restrict__ h) {
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.y;
  const float* rec = in + (size_t)p * (2 * H + 1);
  const float g = rec[2 * H];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x)
    h[(size_t)p * H + i] = rec[i] + g * rec[H + i];
}

int launch_unpack_boundary(const float* d_in, int q, int H, float* d_h, cudaStream_t st) {
  return launch_pdl(unpack_boundary_kernel, dim3(8, q), dim3(256), 0, st, d_in, H, d_h);
}

}  // namespace clm
