// llama.cu — per-layer kernels of the Llama-shaped decoder family (see llama.cuh).
#include <cfloat>

#include "bulk.cuh"
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

// Shared memory of one attention CTA: kAttnPages pages of K [64][HD] and V^T [HD][64] (fp16), staged by bulk copies.
constexpr size_t attn_page_bytes(int hd) { return (size_t)kPageTokens * hd * sizeof(__half); }
constexpr size_t attn_smem_bytes(int hd) { return (size_t)kAttnPages * 2 * attn_page_bytes(hd); }

// One CTA = kAttnPages consecutive pages of one kv head for one m-tile of 16 query rows; two warps per page, warp
// w taking positions [32*(w%2), 32*(w%2)+32) of page w/2.  Each page (K and V^T, 2 x 16 KB) is fetched with two
// cp.async.bulk copies into shared memory; pages that hold only committed positions (all < base) are requested
// BEFORE griddepcontrol.wait, because the preceding QKV GEMV writes only positions >= base, so under
// programmatic dependent launch the bulk of the KV stream overlaps the previous kernel.  The page holding the
// window's own positions is requested after the wait.
//
// Fragment mapping (mma m16n8k16, lane = 4g + t): in S = Q K^T, n-tile j column n is half-page position
// p(j, n) = 8*(n/2) + 2j + n%2, so the C fragment of n-tile j holds positions 8t + 2j + {0, 1}; the P fragments
// of S's n-tiles 2kk and 2kk+1 are then exactly the A fragment of the P.V k-step kk over positions
// 8t + 4kk + {0..3}, whose B fragment is the lane's single V^T chunk (positions 8t..8t+7 of the half page).
template <int HD>
__global__ void __launch_bounds__(32 * kAttnWarps) attention_kernel(
    const __half* __restrict__ q16, const __half* __restrict__ kpool, const __half* __restrict__ vpool,
    const int32_t* __restrict__ pages, const long long* __restrict__ d_pos, const int32_t* __restrict__ parent, int q,
    int nh, int nkv, float scale_log2, int max_pages, float* __restrict__ part, int* __restrict__ counters, int nt_out,
    float hi_scale, uint2* __restrict__ out_frag, float* __restrict__ out_sum, int* __restrict__ err) {
  static_assert(HD == 128, "head_dim 128 layout");
  constexpr int RW = kAttnRowFloats;  // one partial row: O[HD], m, l, padding (16-byte aligned rows)
  constexpr uint32_t kPageBytes = (uint32_t)attn_page_bytes(HD);
  extern __shared__ __align__(128) uint8_t attn_smem[];
  __shared__ __align__(8) uint64_t bar[kAttnPages];
  __shared__ int s_last;
  const int kvh = blockIdx.x, mt = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, t = lane % 4;
  const int wp = warp / 2, half = warp % 2;  // page within the CTA, half of that page
  const int pg = blockIdx.y * kAttnPages + wp;
  __half* ks = reinterpret_cast<__half*>(attn_smem + (size_t)wp * 2 * kPageBytes);
  __half* vs = ks + kPageTokens * HD;
  // this warp's partial [16][RW], written over its page once both warps of the page are done with it
  float* sp = reinterpret_cast<float*>(attn_smem + (size_t)wp * 2 * kPageBytes) + half * 16 * RW;

  if (threadIdx.x == 0) {
    for (int w = 0; w < kAttnPages; ++w) mbar_init(&bar[w], 1);
    mbar_fence_init();
  }
  __syncthreads();
  // committed position and page table do not depend on the preceding kernel
  const long long base = *d_pos;
  const long long nvis = base + q;
  const int npages = (int)((nvis + kPageTokens - 1) / kPageTokens);
  const int ngroups = (npages + kAttnPages - 1) / kAttnPages;
  const bool active = pg < npages && pg < max_pages;
  const bool committed_page = (long long)(pg + 1) * kPageTokens <= base;
  auto request = [&]() {
    const int32_t page = pages[pg];
    const size_t off = ((size_t)page * nkv + kvh) * kPageTokens * HD;
    mbar_expect_tx(&bar[wp], 2 * kPageBytes);
    bulk_g2s(ks, kpool + off, kPageBytes, &bar[wp]);
    bulk_g2s(vs, vpool + off, kPageBytes, &bar[wp]);
  };
  const bool requester = active && half == 0 && lane == 0;
  if (requester && committed_page) request();
  griddep_wait();
  griddep_launch();
  if (requester && !committed_page) request();

  const int group = nh / nkv;
  const int r0 = mt * 16 + g, r1 = r0 + 8;
  const int i0 = r0 / group, i1 = r1 / group;
  const bool v0 = i0 < q, v1 = i1 < q;
  bool ok = active;
  float O[HD / 8][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  if (active) {
    // Q fragments: thread t holds head dims [32t, 32t+32) of rows r0 and r1 (the same k permutation as K below).
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
    ok = mbar_wait(&bar[wp], 0, err);
    if (ok) {
      float S[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.0f;
        const int pos = 32 * half + 8 * (g / 2) + 2 * j + (g % 2);
        const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)pos * HD);
        uint4 kw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) kw[u] = kr[kv_k_chunk(4 * t + u, pos)];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(S[j], word_of(qw0, 2 * kk), word_of(qw1, 2 * kk), word_of(qw0, 2 * kk + 1), word_of(qw1, 2 * kk + 1),
                  word_of(kw, 2 * kk), word_of(kw, 2 * kk + 1));
      }
      if (committed_page) {  // every position is visible to every window row
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            S[j][e] = v0 ? S[j][e] * scale_log2 : -INFINITY;
            S[j][2 + e] = v1 ? S[j][2 + e] * scale_log2 : -INFINITY;
            m0 = fmaxf(m0, S[j][e]);
            m1 = fmaxf(m1, S[j][2 + e]);
          }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const long long pos = (long long)pg * kPageTokens + 32 * half + 8 * t + 2 * j + e;
            S[j][e] = (v0 && visible(pos, base, i0, parent)) ? S[j][e] * scale_log2 : -INFINITY;
            S[j][2 + e] = (v1 && visible(pos, base, i1, parent)) ? S[j][2 + e] * scale_log2 : -INFINITY;
            m0 = fmaxf(m0, S[j][e]);
            m1 = fmaxf(m1, S[j][2 + e]);
          }
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
      }
      uint32_t pa[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
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
#pragma unroll
      for (int jn = 0; jn < HD / 8; ++jn) {
        O[jn][0] = O[jn][1] = O[jn][2] = O[jn][3] = 0.0f;
        const int vrow = 8 * jn + g;
        const uint4 va = reinterpret_cast<const uint4*>(vs + (size_t)vrow * kPageTokens)[kv_v_chunk(4 * half + t, vrow)];
        mma_f16(O[jn], pa[0][0], pa[0][1], pa[1][0], pa[1][1], va.x, va.y);
        mma_f16(O[jn], pa[2][0], pa[2][1], pa[3][0], pa[3][1], va.z, va.w);
      }
    } else {
      // the copy never completed (error flag raised): give it one more bounded wait before the CTA can exit
      mbar_wait(&bar[wp], 0, err);
    }
  }
  // both warps of the page are done reading it: its space takes their partials
  asm volatile("bar.sync %0, 64;" ::"r"(1 + wp) : "memory");
  if (active && ok) {
#pragma unroll
    for (int jn = 0; jn < HD / 8; ++jn) {
      *reinterpret_cast<float2*>(sp + g * RW + 8 * jn + 2 * t) = make_float2(O[jn][0], O[jn][1]);
      *reinterpret_cast<float2*>(sp + (g + 8) * RW + 8 * jn + 2 * t) = make_float2(O[jn][2], O[jn][3]);
    }
    if (t == 0) {
      sp[g * RW + HD] = m0;
      sp[g * RW + HD + 1] = l0;
      sp[(g + 8) * RW + HD] = m1;
      sp[(g + 8) * RW + HD + 1] = l1;
    }
  } else if (lane < 16) {
    sp[lane * RW + HD] = -INFINITY;
    sp[lane * RW + HD + 1] = 0.0f;
  }
  __syncthreads();
  auto spw = [&](int w) {
    return reinterpret_cast<const float*>(attn_smem + (size_t)(w / 2) * 2 * kPageBytes) + (w % 2) * 16 * RW;
  };
  // combine the CTA's warps into one partial per (m-tile, kv head, page group)
  float* mine = part + (((size_t)mt * nkv + kvh) * max_pages + blockIdx.y) * 16 * RW;
  if ((int)blockIdx.y < ngroups) {
    for (int i = threadIdx.x; i < 16 * (HD + 2); i += blockDim.x) {
      const int r = i / (HD + 2), c = i % (HD + 2);
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, spw(w)[r * RW + HD]);
      float a = 0.0f;
      if (c == HD) {
        a = M;
      } else {
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
          const float m = spw(w)[r * RW + HD];
          if (m == -INFINITY) continue;
          a += spw(w)[r * RW + c] * exp2f(m - M);
        }
      }
      mine[r * RW + c] = a;
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
  // combine weights w[gi][r] = exp2(m_gi - M) / L, staged in shared memory (after o_s)
  float* o_s = reinterpret_cast<float*>(attn_smem);  // [16][HD], reusing the page buffers
  float* wgt = o_s + 16 * HD;                         // [ngroups][16]
  float* lsum = wgt + ngroups * 16;                    // [ngroups][16]
  for (int i = threadIdx.x; i < ngroups * 16; i += blockDim.x) {
    wgt[i] = __ldcg(allp + (size_t)i * RW + HD);
    lsum[i] = __ldcg(allp + (size_t)i * RW + HD + 1);
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float M = -INFINITY;
    for (int gi = 0; gi < ngroups; ++gi) M = fmaxf(M, wgt[gi * 16 + r]);
    float L = 0.0f;
    for (int gi = 0; gi < ngroups; ++gi) {
      const float m = wgt[gi * 16 + r];
      const float e = m == -INFINITY ? 0.0f : exp2f(m - M);
      L += lsum[gi * 16 + r] * e;
      wgt[gi * 16 + r] = e;
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int gi = 0; gi < ngroups; ++gi) wgt[gi * 16 + r] *= inv;
  }
  __syncthreads();
  {
    // thread (row r, 8 columns c8): 16-byte loads, four page groups in flight
    const int r = threadIdx.x / (HD / 8), c8 = threadIdx.x % (HD / 8);
    float a[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = 0.0f;
    const float* col = allp + (size_t)r * RW + 8 * c8;
    int gi = 0;
    for (; gi + 4 <= ngroups; gi += 4) {
      float4 v[4][2];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4* p4 = reinterpret_cast<const float4*>(col + (size_t)(gi + u) * 16 * RW);
        v[u][0] = __ldcg(p4);
        v[u][1] = __ldcg(p4 + 1);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = wgt[(gi + u) * 16 + r];
        a[0] += v[u][0].x * w;
        a[1] += v[u][0].y * w;
        a[2] += v[u][0].z * w;
        a[3] += v[u][0].w * w;
        a[4] += v[u][1].x * w;
        a[5] += v[u][1].y * w;
        a[6] += v[u][1].z * w;
        a[7] += v[u][1].w * w;
      }
    }
    for (; gi < ngroups; ++gi) {
      const float4* p4 = reinterpret_cast<const float4*>(col + (size_t)gi * 16 * RW);
      const float4 x0 = __ldcg(p4), x1 = __ldcg(p4 + 1);
      const float w = wgt[gi * 16 + r];
      a[0] += x0.x * w;
      a[1] += x0.y * w;
      a[2] += x0.z * w;
      a[3] += x0.w * w;
      a[4] += x1.x * w;
      a[5] += x1.y * w;
      a[6] += x1.z * w;
      a[7] += x1.w * w;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) o_s[r * HD + 8 * c8 + k] = a[k];
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[mt * nkv + kvh] = 0;
  // fragments: query vector r = window row i, head kvh*group + r%group; 8 column groups of 16 per head
  const int qd = nh * HD;
  for (int it = threadIdx.x; it < 16 * (HD / 16); it += blockDim.x) {
    const int r = it / (HD / 16), gg = it % (HD / 16);
    const int i = (mt * 16 + r) / group, head = kvh * group + (mt * 16 + r) % group;
    if (i >= q) continue;
    prep16(&o_s[r * HD + 16 * gg], nullptr, i, q, (head * HD + 16 * gg) / 16, nt_out, hi_scale, out_frag, out_sum,
           nullptr, qd);
  }
}

int launch_attention(const __half* d_q, const __half* d_k, const __half* d_v, const int32_t* d_pages,
                     const long long* d_pos, const int32_t* d_parent, int q, const LlamaDims& d, int max_pages,
                     float* d_part, int* d_counters, int nt_out, float hi_scale, void* d_frag, float* d_sum, int* d_err,
                     cudaStream_t st) {
  CLM_CHECK(d.hd == 128, CLM_UNIMPLEMENTED, "attention kernel supports head_dim 128");
  const int group = d.nh / d.nkv;
  const int mtiles = (q * group + 15) / 16;
  const float scale_log2 = (float)(1.4426950408889634 / sqrt((double)d.hd));
  const size_t smem = attn_smem_bytes(128);
  CLM_CHECK((size_t)16 * 128 * 4 + (size_t)((max_pages + kAttnPages - 1) / kAttnPages) * 32 * 4 <= smem,
            CLM_RESOURCE_EXHAUSTED, "attention: max_context too large for the page-group combine");
  CLM_TRY(ensure_smem(attention_kernel<128>, smem));
  return launch_pdl(attention_kernel<128>, dim3(d.nkv, (max_pages + kAttnPages - 1) / kAttnPages, mtiles),
                    dim3(32 * kAttnWarps), smem, st, d_q, d_k, d_v, d_pages, d_pos, d_parent, q, d.nh, d.nkv,
                    scale_log2, max_pages, d_part, d_counters, nt_out, hi_scale, static_cast<uint2*>(d_frag), d_sum,
                    d_err);
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
