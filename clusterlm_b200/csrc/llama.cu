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
  // the token's row is staged in shared memory with 16-byte loads (one round trip), then decoded from there
  constexpr int kRowMax = 9216;  // a Q4_K row of H <= 16384 or a Q8_0 row of H <= 8448
  __shared__ __align__(16) uint8_t srow[kRowMax];
  const size_t row_bytes = quant == CLM_QUANT_Q4_K ? (size_t)(H / 256) * 144 : (size_t)(H / 32) * 34;
  const uint8_t* grow = embd + (size_t)tok * row_bytes;
  const bool staged = row_bytes <= kRowMax && row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(grow) & 15) == 0;
  if (staged) {
    for (int i = threadIdx.x; i < (int)(row_bytes / 16); i += blockDim.x)
      reinterpret_cast<uint4*>(srow)[i] = __ldg(reinterpret_cast<const uint4*>(grow) + i);
    __syncthreads();
  }
  const uint8_t* row = staged ? srow : grow;
  if (quant == CLM_QUANT_Q4_K) {
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
  for (int a = i, guard = 0; a >= 0 && guard < 256; a = parent[a], ++guard)
    if (a == rel) return true;
  return false;
}

// Shared memory of one attention CTA: kAttnPages page buffers of K [64][HD] and V^T [HD][64] (fp16), staged by bulk
// copies.
constexpr size_t attn_page_bytes(int hd) { return (size_t)kPageTokens * hd * sizeof(__half); }
constexpr size_t attn_smem_bytes(int hd) { return (size_t)kAttnPages * 2 * attn_page_bytes(hd); }

// Split-KV decode attention.  Grid (kv head, split, m-tile); the S = gridDim.y splits of a (kv head, m-tile) own
// contiguous page ranges of the visible positions [0, pos + q).
//
//  * Page buffer b (of kAttnPages) serves the CTA's pages b, b + kAttnPages, ...; warps 2b and 2b+1 take
//    positions [0, 32) and [32, 64) of each and keep a running (max, sum, O) per query row (online softmax), so a
//    warp's state stays in registers however many pages the split holds.  Committed pages (every position
//    < pos) are requested before griddepcontrol.wait: the preceding QKV GEMV writes only positions >= pos, so the
//    bulk of the KV stream overlaps the previous kernel.  A buffer is refilled once both of its warps are done
//    with it (named barrier of the pair).
//  * The CTA folds its eight warps into one partial (per-row weights computed once), writes it, and publishes it
//    with one release-add on the (m-tile, kv head) arrival counter.
//  * Every split waits (bounded acquire spin) until all S partials are in, then combines a 1/S slice of the
//    16 rows x HD/16 column groups over the S partials and writes W_o's input fragments for it.  All splits of
//    the grid are resident together (at most one CTA per SM and the grid is no larger than the SM count), so
//    the wait ends.  The last split to leave resets the counters for the next launch.
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
    float hi_scale, uint2* __restrict__ out_frag, float* __restrict__ out_sum, int* __restrict__ err,
    const uint8_t* __restrict__ pf, unsigned long long pf_bytes, float* __restrict__ out_f32, AttnLink link,
    int row_off, int q_frag) {
  static_assert(HD == 128, "head_dim 128 layout");
  static_assert(kAttnWarps == 2 * kAttnPages, "two warps per page buffer");
  constexpr int RW = kAttnRowFloats;  // one partial row: O[HD], m, l, padding (16-byte aligned rows)
  constexpr uint32_t kPageBytes = (uint32_t)attn_page_bytes(HD);
  constexpr int kItems = 16 * (HD / 16);  // (row, 16-column group) items of the final combine
  extern __shared__ __align__(128) uint8_t attn_smem[];
  __shared__ __align__(8) uint64_t bar[kAttnPages];
  __shared__ float s_wt[16][kAttnWarps];
  __shared__ float s_ml[16][2];
  __shared__ float s_out[kAttnWarps * 32 / 16][16];
  const int kvh = blockIdx.x, split = blockIdx.y, S = gridDim.y, mt = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, t = lane % 4;
  const int wp = warp / 2, half = warp % 2;  // page buffer of this warp, half of each page
  __half* ks = reinterpret_cast<__half*>(attn_smem + (size_t)wp * 2 * kPageBytes);
  __half* vs = ks + kPageTokens * HD;

  if (threadIdx.x == 0) {
    for (int w = 0; w < kAttnPages; ++w) mbar_init(&bar[w], 1);
    mbar_fence_init();
  }
  __syncthreads();
  // committed position and page table do not depend on the preceding kernel
  const long long base = *d_pos;
  const long long nvis = base + q;
  const long long np_l = (nvis + kPageTokens - 1) / kPageTokens;
  const int npages = (int)(np_l < max_pages ? np_l : max_pages);
  const int p_begin = (int)((long long)split * npages / S), p_end = (int)((long long)(split + 1) * npages / S);
  const bool owner = half == 0 && lane == 0;  // requests the pages of buffer wp
  auto request = [&](int pg) {
    const size_t off = ((size_t)pages[pg] * nkv + kvh) * kPageTokens * HD;
    mbar_expect_tx(&bar[wp], 2 * kPageBytes);
    bulk_g2s(ks, kpool + off, kPageBytes, &bar[wp]);
    bulk_g2s(vs, vpool + off, kPageBytes, &bar[wp]);
  };
  const int first = p_begin + wp;
  const bool first_committed = (long long)(first + 1) * kPageTokens <= base;
  if (owner && first < p_end && first_committed) request(first);
  // L2 lookahead: this CTA's share of the next kernel's weights (W_o), read while the attention runs
  if (threadIdx.x == 32 * (kAttnWarps - 1))
    l2_prefetch_share(pf, pf_bytes, (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)),
                      (int)(gridDim.x * gridDim.y * gridDim.z), ~0ull);
  const bool linked = link.wait != nullptr;
  if (!linked) griddep_wait();
  griddep_launch();
  if (linked) {
    // dataflow: this kv head's query, key and value rows are written
    __shared__ int s_dep;
    if (threadIdx.x == 0) s_dep = dep_wait(link.wait + kvh, link.target, err);
    __syncthreads();
    (void)s_dep;                 // on failure the flag is raised; the window's outputs are not used
    fence_proxy_async_global();  // the window's page is bulk-copied after other CTAs' stores into it
  }
  if (owner && first < p_end && !first_committed) request(first);

  const int group = nh / nkv;
  const int r0 = mt * 16 + g, r1 = r0 + 8;
  const int i0 = r0 / group, i1 = r1 / group;
  const bool v0 = i0 < q, v1 = i1 < q;
  // Q fragments: thread t holds head dims [32t, 32t+32) of rows r0 and r1 (the same k permutation as K below).
  uint4 qw0[4], qw1[4];
  {
    const uint4 z = make_uint4(0, 0, 0, 0);
    const uint4* a = reinterpret_cast<const uint4*>(q16 + ((size_t)i0 * nh + kvh * group + r0 % group) * HD + 32 * t);
    const uint4* b = reinterpret_cast<const uint4*>(q16 + ((size_t)i1 * nh + kvh * group + r1 % group) * HD + 32 * t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // L2 reads: the rows may have been written by other SMs during this launch
      qw0[j] = v0 ? __ldcg(a + j) : z;
      qw1[j] = v1 ? __ldcg(b + j) : z;
    }
  }
  float O[HD / 8][4];
#pragma unroll
  for (int jn = 0; jn < HD / 8; ++jn) O[jn][0] = O[jn][1] = O[jn][2] = O[jn][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  uint32_t phase = 0;
  for (int pg = first; pg < p_end; pg += kAttnPages, phase ^= 1u) {
    // every issued copy is waited for (bounded), so no copy is in flight when the CTA leaves
    const bool ok = mbar_wait(&bar[wp], phase, err);
    if (ok) {
      float Sx[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Sx[j][0] = Sx[j][1] = Sx[j][2] = Sx[j][3] = 0.0f;
        const int pos = 32 * half + 8 * (g / 2) + 2 * j + (g % 2);
        const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)pos * HD);
        uint4 kw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) kw[u] = kr[kv_k_chunk(4 * t + u, pos)];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16(Sx[j], word_of(qw0, 2 * kk), word_of(qw1, 2 * kk), word_of(qw0, 2 * kk + 1), word_of(qw1, 2 * kk + 1),
                  word_of(kw, 2 * kk), word_of(kw, 2 * kk + 1));
      }
      float mx0 = m0, mx1 = m1;
      if ((long long)(pg + 1) * kPageTokens <= base) {  // every position is visible to every window row
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            Sx[j][e] = v0 ? Sx[j][e] * scale_log2 : -INFINITY;
            Sx[j][2 + e] = v1 ? Sx[j][2 + e] * scale_log2 : -INFINITY;
            mx0 = fmaxf(mx0, Sx[j][e]);
            mx1 = fmaxf(mx1, Sx[j][2 + e]);
          }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const long long pos = (long long)pg * kPageTokens + 32 * half + 8 * t + 2 * j + e;
            Sx[j][e] = (v0 && visible(pos, base, i0, parent)) ? Sx[j][e] * scale_log2 : -INFINITY;
            Sx[j][2 + e] = (v1 && visible(pos, base, i1, parent)) ? Sx[j][2 + e] * scale_log2 : -INFINITY;
            mx0 = fmaxf(mx0, Sx[j][e]);
            mx1 = fmaxf(mx1, Sx[j][2 + e]);
          }
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      // rescale the running state to the new maxima
      const float c0 = mx0 == -INFINITY ? 1.0f : exp2f(m0 - mx0), c1 = mx1 == -INFINITY ? 1.0f : exp2f(m1 - mx1);
      m0 = mx0;
      m1 = mx1;
      l0 *= c0;
      l1 *= c1;
#pragma unroll
      for (int jn = 0; jn < HD / 8; ++jn) {
        O[jn][0] *= c0;
        O[jn][1] *= c0;
        O[jn][2] *= c1;
        O[jn][3] *= c1;
      }
      uint32_t pa[4][2];
      float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p00 = m0 == -INFINITY ? 0.0f : exp2f(Sx[j][0] - m0);
        const float p01 = m0 == -INFINITY ? 0.0f : exp2f(Sx[j][1] - m0);
        const float p10 = m1 == -INFINITY ? 0.0f : exp2f(Sx[j][2] - m1);
        const float p11 = m1 == -INFINITY ? 0.0f : exp2f(Sx[j][3] - m1);
        ps0 += p00 + p01;
        ps1 += p10 + p11;
        pa[j][0] = pack_half2(p00, p01);
        pa[j][1] = pack_half2(p10, p11);
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, o);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, o);
      }
      l0 += ps0;
      l1 += ps1;
#pragma unroll
      for (int jn = 0; jn < HD / 8; ++jn) {
        const int vrow = 8 * jn + g;
        const uint4 va = reinterpret_cast<const uint4*>(vs + (size_t)vrow * kPageTokens)[kv_v_chunk(4 * half + t, vrow)];
        mma_f16(O[jn], pa[0][0], pa[0][1], pa[1][0], pa[1][1], va.x, va.y);
        mma_f16(O[jn], pa[2][0], pa[2][1], pa[3][0], pa[3][1], va.z, va.w);
      }
    }
    // both warps of the buffer are done with this page: refill it with the buffer's next page
    asm volatile("bar.sync %0, 64;" ::"r"(1 + wp) : "memory");
    if (owner && pg + kAttnPages < p_end) request(pg + kAttnPages);
  }

  // this warp's partial [16][RW] over the first half of its buffer's space (its pages are all consumed)
  float* sp = reinterpret_cast<float*>(attn_smem + (size_t)wp * 2 * kPageBytes) + half * 16 * RW;
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
  __syncthreads();
  auto spw = [&](int w) {
    return reinterpret_cast<const float*>(attn_smem + (size_t)(w / 2) * 2 * kPageBytes) + (w % 2) * 16 * RW;
  };
  // per-row weights of the eight warps, once
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, spw(w)[r * RW + HD]);
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float m = spw(w)[r * RW + HD];
      const float e = m == -INFINITY ? 0.0f : exp2f(m - M);
      s_wt[r][w] = e;
      L += spw(w)[r * RW + HD + 1] * e;
    }
    s_ml[r][0] = M;
    s_ml[r][1] = L;
  }
  __syncthreads();
  // this split's partial, in global memory
  const size_t head_slot = (size_t)mt * nkv + kvh;
  float* allp = part + head_slot * S * 16 * RW;
  float* mine = allp + (size_t)split * 16 * RW;
  for (int i = threadIdx.x; i < 16 * (HD / 4); i += blockDim.x) {
    const int r = i / (HD / 4), c4 = i % (HD / 4);
    float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float e = s_wt[r][w];
      const float4 v = *reinterpret_cast<const float4*>(spw(w) + r * RW + 4 * c4);
      a.x += v.x * e;
      a.y += v.y * e;
      a.z += v.z * e;
      a.w += v.w * e;
    }
    *reinterpret_cast<float4*>(mine + r * RW + 4 * c4) = a;
  }
  if (threadIdx.x < 16) {
    mine[threadIdx.x * RW + HD] = s_ml[threadIdx.x][0];
    mine[threadIdx.x * RW + HD + 1] = s_ml[threadIdx.x][1];
  }
  __syncthreads();
  int* arrive = counters + head_slot;
  int* depart = counters + (size_t)gridDim.z * nkv + head_slot;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    red_release_add(arrive, 1);
    s_ok = wait_count(arrive, S, err);
    // every split has passed the wait once all have departed: the last one resets both counters
    if (atomicAdd(depart, 1) == S - 1) {
      *arrive = 0;
      *depart = 0;
    }
  }
  __syncthreads();
  if (!s_ok) return;

  // final combine of this split's slice of the (row, column group) items over the S partials
  const int it_begin = split * kItems / S, it_end = (split + 1) * kItems / S;
  const int lanes = blockDim.x / 16;  // items in flight per pass
  const int qd = nh * HD;
  for (int it0 = it_begin; it0 < it_end; it0 += lanes) {
    const int li = threadIdx.x / 16, c = threadIdx.x % 16, it = it0 + li;
    const bool live = it < it_end;
    const int r = live ? it / (HD / 16) : 0, cg = live ? it % (HD / 16) : 0;
    // all of a thread's loads are issued before any is used (kAttnMaxSplits at a time)
    float M = -INFINITY, L = 0.0f, a = 0.0f;
    for (int k0 = 0; k0 < S; k0 += kAttnMaxSplits) {
      float mk[kAttnMaxSplits], lk[kAttnMaxSplits], vk[kAttnMaxSplits];
#pragma unroll
      for (int k = 0; k < kAttnMaxSplits; ++k) {
        const float* row = allp + ((size_t)(k0 + k) * 16 + r) * RW;
        const bool in = k0 + k < S;
        mk[k] = in ? __ldcg(row + HD) : -INFINITY;
        lk[k] = in ? __ldcg(row + HD + 1) : 0.0f;
        vk[k] = in ? __ldcg(row + 16 * cg + c) : 0.0f;
      }
      float Mn = M;
#pragma unroll
      for (int k = 0; k < kAttnMaxSplits; ++k) Mn = fmaxf(Mn, mk[k]);
      const float cr = Mn == -INFINITY ? 1.0f : exp2f(M - Mn);  // rescale what earlier batches summed
      L *= cr;
      a *= cr;
      M = Mn;
#pragma unroll
      for (int k = 0; k < kAttnMaxSplits; ++k) {
        const float e = mk[k] == -INFINITY ? 0.0f : exp2f(mk[k] - M);
        L += lk[k] * e;
        a += vk[k] * e;
      }
    }
    s_out[li][c] = L > 0.0f ? a / L : 0.0f;
    if (out_f32 != nullptr) {  // f32 rows [q][nh * HD] (the wide window's W_o input)
      const int i = (mt * 16 + r) / group, head = kvh * group + (mt * 16 + r) % group;
      if (live && i < q) out_f32[(size_t)i * qd + head * HD + 16 * cg + c] = s_out[li][c];
      continue;
    }
    __syncthreads();
    if (live && c == 0) {
      // query vector r = window row i, head kvh*group + r%group; 16 columns 16cg.. of that head
      const int i = (mt * 16 + r) / group, head = kvh * group + (mt * 16 + r) % group;
      if (i < q)
        prep16(s_out[li], nullptr, row_off + i, q_frag, (head * HD + 16 * cg) / 16, nt_out, hi_scale, out_frag, out_sum,
               nullptr, qd);
    }
    __syncthreads();
  }
  if (link.sig != nullptr) {
    __syncthreads();  // every thread's fragments are stored before the release
    if (threadIdx.x == 0) {
      if (link.span > 1) {
        for (int c = 0; c < link.span; ++c) red_release_add(link.sig + kvh * link.span + c, 1);
      } else {
        red_release_add(link.sig + kvh / link.kvh_div, 1);
      }
    }
  }
}

int launch_attention(const __half* d_q, const __half* d_k, const __half* d_v, const int32_t* d_pages,
                     const long long* d_pos, const int32_t* d_parent, int q, const LlamaDims& d, int max_pages,
                     float* d_part, int* d_counters, int nt_out, float hi_scale, void* d_frag, float* d_sum, int* d_err,
                     const uint8_t* d_prefetch, unsigned long long prefetch_bytes, int sm_count, cudaStream_t st,
                     float* d_out_f32, const AttnLink& link, int row_off, int q_frag) {
  CLM_CHECK(d.hd == 128, CLM_UNIMPLEMENTED, "attention kernel supports head_dim 128");
  if (q_frag <= 0) q_frag = q;
  CLM_CHECK(d_out_f32 != nullptr || (row_off >= 0 && row_off + q <= q_frag && q_frag <= 8 * nt_out && nt_out <= 4),
            CLM_OUT_OF_RANGE, "W_o input fragments: rows outside the window's n-tiles");
  const int group = d.nh / d.nkv;
  const int mtiles = (q * group + 15) / 16;
  const float scale_log2 = (float)(1.4426950408889634 / sqrt((double)d.hd));
  const size_t smem = attn_smem_bytes(128);
  // splits per (kv head, m-tile): enough for the pages, no more CTAs than SMs (the splits wait for each other).
  // With more (kv head, m-tile) pairs than SMs there is one split each, whose wait is on its own arrival only.
  const int splits = attention_splits(q, d, max_pages, sm_count);
  CLM_TRY(ensure_smem(attention_kernel<128>, smem));
  return launch_pdl(attention_kernel<128>, dim3(d.nkv, splits, mtiles), dim3(32 * kAttnWarps), smem, st, d_q, d_k,
                    d_v, d_pages, d_pos, d_parent, q, d.nh, d.nkv, scale_log2, max_pages, d_part, d_counters, nt_out,
                    hi_scale, static_cast<uint2*>(d_frag), d_sum, d_err, d_prefetch, prefetch_bytes, d_out_f32, link,
                    row_off, q_frag);
}

int attention_splits(int q, const LlamaDims& d, int max_pages, int sm_count) {
  const int mtiles = (q * (d.nh / d.nkv) + 15) / 16;
  const int heads = d.nkv * mtiles;
  int splits = (max_pages + kAttnPages - 1) / kAttnPages;
  if (splits > sm_count / heads) splits = sm_count / heads;
  if (splits < 1) splits = 1;
  return splits;
}

// ---------------------------------------------------------------------------------------------------
// wide-window attention: every KV page read once per (kv head, 16-row block, segment)
// ---------------------------------------------------------------------------------------------------
constexpr int kWideAttnPages = 3;        // page ring depth (K page + V^T page per slot)
constexpr int kWideAttnMaxGroup = 8;     // query heads per kv head
constexpr int kWideAttnHeads = 4;        // query heads per CTA (a larger group is split over group / 4 CTAs)
constexpr int kWideAttnMaxSplits = 8;    // KV splits per (kv head, 16-row block, segment)

template <int HD>
__global__ void __launch_bounds__(32 * (2 * kWideAttnHeads + 1), 1) attention_wide_kernel(
    const __half* __restrict__ q16, const __half* __restrict__ kpool, const __half* __restrict__ vpool,
    const __grid_constant__ AttnSegs segs, const int32_t* __restrict__ parent, int qs, int nh, int nkv, float scale_log2,
    int max_pages, int nsplit, float* __restrict__ gpart, int* __restrict__ counters, float* __restrict__ out,
    int* __restrict__ err) {
  static_assert(HD == 128, "head_dim 128 layout");
  constexpr int RW = kAttnRowFloats;
  constexpr uint32_t kPageBytes = (uint32_t)attn_page_bytes(HD);
  extern __shared__ __align__(128) uint8_t wa_smem[];
  __shared__ __align__(8) uint64_t full[kWideAttnPages], empty[kWideAttnPages];
  const int group = nh / nkv, hg = group < kWideAttnHeads ? group : kWideAttnHeads, nsub = group / hg;
  const int kvh = blockIdx.x / nsub, h0 = kvh * group + (blockIdx.x % nsub) * hg;  // this CTA's first query head
  const int blk = blockIdx.y, seg = blockIdx.z / nsplit, split = blockIdx.z % nsplit;
  const int nw = 2 * hg;  // consumer warps
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, t = lane % 4;
  const long long* d_pos = segs.pos[seg];
  const int32_t* pages = segs.pages[seg];
  const int row0 = segs.row0[seg];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWideAttnPages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nw);
    }
    mbar_fence_init();
  }
  __syncthreads();
  // committed position and page table do not depend on the preceding kernel
  const long long base = *d_pos;
  const int last_row = min(16 * blk + 15, qs - 1);
  const long long np_l = (base + last_row + 1 + kPageTokens - 1) / kPageTokens;
  const int np_all = (int)(np_l < max_pages ? np_l : max_pages);
  // this split's contiguous share of the visible pages
  const int pg_begin = (int)((long long)split * np_all / nsplit), pg_end = (int)((long long)(split + 1) * np_all / nsplit);
  auto kbuf = [&](int s) { return reinterpret_cast<__half*>(wa_smem + (size_t)s * 2 * kPageBytes); };
  // the consumers' final states, after the page ring: [warp][16 rows][RW]
  float* parts = reinterpret_cast<float*>(wa_smem + (size_t)kWideAttnPages * 2 * kPageBytes);

  if (warp == nw) {
    // ---------------- producer: committed pages before griddepcontrol.wait, the window's after ----------------
    bool waited = false;
    if (lane == 0) {
      int slot = 0;
      uint32_t phase = 0;
      for (int pg = pg_begin; pg < pg_end; ++pg) {
        if (!waited && (long long)(pg + 1) * kPageTokens > base) {
          griddep_wait();  // this page holds rows the preceding kernel wrote
          waited = true;
        }
        if (!mbar_wait(&empty[slot], phase ^ 1u, err)) break;
        const size_t off = ((size_t)pages[pg] * nkv + kvh) * kPageTokens * HD;
        mbar_expect_tx(&full[slot], 2 * kPageBytes);
        bulk_g2s(kbuf(slot), kpool + off, kPageBytes, &full[slot]);
        bulk_g2s(kbuf(slot) + kPageTokens * HD, vpool + off, kPageBytes, &full[slot]);
        if (++slot == kWideAttnPages) {
          slot = 0;
          phase ^= 1u;
        }
      }
    }
    if (!waited) griddep_wait();
    griddep_launch();
  } else if (warp < nw) {
    // ---------------- consumers: m-tile j (16 of the block's 16 x group rows), half of every page ----------------
    griddep_wait();
    griddep_launch();
    const int j = warp / 2, half = warp % 2;
    const int r0 = j * 16 + g, r1 = r0 + 8;  // rows of the block: window row 16 blk + r / hg, head h0 + r % hg
    const int i0 = 16 * blk + r0 / hg, i1 = 16 * blk + r1 / hg;
    const bool v0 = i0 < qs, v1 = i1 < qs;
    float O[HD / 8][4];
#pragma unroll
    for (int jn = 0; jn < HD / 8; ++jn) O[jn][0] = O[jn][1] = O[jn][2] = O[jn][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    uint4 qw0[4], qw1[4];
    {
      const uint4 z = make_uint4(0, 0, 0, 0);
      const uint4* a = reinterpret_cast<const uint4*>(
          q16 + ((size_t)(row0 + (v0 ? i0 : 0)) * nh + h0 + r0 % hg) * HD + 32 * t);
      const uint4* b = reinterpret_cast<const uint4*>(
          q16 + ((size_t)(row0 + (v1 ? i1 : 0)) * nh + h0 + r1 % hg) * HD + 32 * t);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        qw0[u] = v0 ? a[u] : z;
        qw1[u] = v1 ? b[u] : z;
      }
    }
    int slot = 0;
    uint32_t phase = 0;
    for (int pg = pg_begin; pg < pg_end; ++pg) {
      const bool ok = mbar_wait(&full[slot], phase, err);
      const __half* ks = kbuf(slot);
      const __half* vs = ks + kPageTokens * HD;
      if (ok) {
        float Sx[4][4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          Sx[jj][0] = Sx[jj][1] = Sx[jj][2] = Sx[jj][3] = 0.0f;
          const int pos = 32 * half + 8 * (g / 2) + 2 * jj + (g % 2);
          const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)pos * HD);
          uint4 kw[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) kw[u] = kr[kv_k_chunk(4 * t + u, pos)];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16(Sx[jj], word_of(qw0, 2 * kk), word_of(qw1, 2 * kk), word_of(qw0, 2 * kk + 1),
                    word_of(qw1, 2 * kk + 1), word_of(kw, 2 * kk), word_of(kw, 2 * kk + 1));
        }
        float mx0 = m0, mx1 = m1;
        if ((long long)(pg + 1) * kPageTokens <= base) {  // every position is visible to every window row
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              Sx[jj][e] = v0 ? Sx[jj][e] * scale_log2 : -INFINITY;
              Sx[jj][2 + e] = v1 ? Sx[jj][2 + e] * scale_log2 : -INFINITY;
              mx0 = fmaxf(mx0, Sx[jj][e]);
              mx1 = fmaxf(mx1, Sx[jj][2 + e]);
            }
        } else {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const long long pos = (long long)pg * kPageTokens + 32 * half + 8 * t + 2 * jj + e;
              Sx[jj][e] = (v0 && visible(pos, base, i0, parent)) ? Sx[jj][e] * scale_log2 : -INFINITY;
              Sx[jj][2 + e] = (v1 && visible(pos, base, i1, parent)) ? Sx[jj][2 + e] * scale_log2 : -INFINITY;
              mx0 = fmaxf(mx0, Sx[jj][e]);
              mx1 = fmaxf(mx1, Sx[jj][2 + e]);
            }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float c0 = mx0 == -INFINITY ? 1.0f : exp2f(m0 - mx0), c1 = mx1 == -INFINITY ? 1.0f : exp2f(m1 - mx1);
        m0 = mx0;
        m1 = mx1;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int jn = 0; jn < HD / 8; ++jn) {
          O[jn][0] *= c0;
          O[jn][1] *= c0;
          O[jn][2] *= c1;
          O[jn][3] *= c1;
        }
        uint32_t pa[4][2];
        float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float p00 = m0 == -INFINITY ? 0.0f : exp2f(Sx[jj][0] - m0);
          const float p01 = m0 == -INFINITY ? 0.0f : exp2f(Sx[jj][1] - m0);
          const float p10 = m1 == -INFINITY ? 0.0f : exp2f(Sx[jj][2] - m1);
          const float p11 = m1 == -INFINITY ? 0.0f : exp2f(Sx[jj][3] - m1);
          ps0 += p00 + p01;
          ps1 += p10 + p11;
          pa[jj][0] = pack_half2(p00, p01);
          pa[jj][1] = pack_half2(p10, p11);
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          ps0 += __shfl_xor_sync(0xffffffffu, ps0, o);
          ps1 += __shfl_xor_sync(0xffffffffu, ps1, o);
        }
        l0 += ps0;
        l1 += ps1;
#pragma unroll
        for (int jn = 0; jn < HD / 8; ++jn) {
          const int vrow = 8 * jn + g;
          const uint4 va =
              reinterpret_cast<const uint4*>(vs + (size_t)vrow * kPageTokens)[kv_v_chunk(4 * half + t, vrow)];
          mma_f16(O[jn], pa[0][0], pa[0][1], pa[1][0], pa[1][1], va.x, va.y);
          mma_f16(O[jn], pa[2][0], pa[2][1], pa[3][0], pa[3][1], va.z, va.w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == kWideAttnPages) {
        slot = 0;
        phase ^= 1u;
      }
    }
    float* sp = parts + (size_t)warp * 16 * RW;
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
  }
  __syncthreads();
  const int qd = nh * HD;
  const int rows = hg * 16;  // this CTA's rows: m-tile j = row / 16
  constexpr int C4 = HD / 4;
  // per row, once: the weights of the two halves (and, for a split, the combined max and sum)
  __shared__ float s_wa[kWideAttnHeads * 16], s_wb[kWideAttnHeads * 16], s_M[kWideAttnHeads * 16],
      s_L[kWideAttnHeads * 16];
  __shared__ float s_wk[kWideAttnMaxSplits][kWideAttnHeads * 16];
  if (threadIdx.x < rows) {
    const int rr = threadIdx.x, j = rr / 16, r = rr % 16;
    const float* a = parts + (size_t)(2 * j) * 16 * RW + r * RW;
    const float* b = a + 16 * RW;
    const float ma = a[HD], mb = b[HD];
    const float M = fmaxf(ma, mb);
    const float ea = ma == -INFINITY ? 0.0f : exp2f(ma - M), eb = mb == -INFINITY ? 0.0f : exp2f(mb - M);
    const float L = a[HD + 1] * ea + b[HD + 1] * eb;
    const bool norm = nsplit == 1;
    s_wa[rr] = norm ? (L > 0.0f ? ea / L : 0.0f) : ea;
    s_wb[rr] = norm ? (L > 0.0f ? eb / L : 0.0f) : eb;
    s_M[rr] = M;
    s_L[rr] = L;
  }
  __syncthreads();
  auto half_sum = [&](int rr, int c4) {
    const int j = rr / 16, r = rr % 16;
    const float4 x = *reinterpret_cast<const float4*>(parts + (size_t)(2 * j) * 16 * RW + r * RW + 4 * c4);
    const float4 y = *reinterpret_cast<const float4*>(parts + (size_t)(2 * j + 1) * 16 * RW + r * RW + 4 * c4);
    const float wa = s_wa[rr], wb = s_wb[rr];
    return make_float4(x.x * wa + y.x * wb, x.y * wa + y.y * wb, x.z * wa + y.z * wb, x.w * wa + y.w * wb);
  };
  auto out_at = [&](int rr, int c4) -> float4* {
    const int i = 16 * blk + rr / hg;
    return reinterpret_cast<float4*>(out + (size_t)(row0 + i) * qd + (h0 + rr % hg) * HD + 4 * c4);
  };
  if (nsplit == 1) {
    for (int idx = threadIdx.x; idx < rows * C4; idx += blockDim.x) {
      const int rr = idx / C4, c4 = idx % C4;
      if (16 * blk + rr / hg < qs) *out_at(rr, c4) = half_sum(rr, c4);
    }
    return;
  }
  // split KV: this split's partial (unnormalised O, max, sum) to global memory; the last split of the tile to
  // arrive (counter) combines all of them, so no CTA waits for another
  const int tile = (blockIdx.x * gridDim.y + blk) * (gridDim.z / nsplit) + seg;
  float* tp = gpart + (size_t)tile * nsplit * rows * RW;
  float* mine = tp + (size_t)split * rows * RW;
  for (int idx = threadIdx.x; idx < rows * C4; idx += blockDim.x) {
    const int rr = idx / C4, c4 = idx % C4;
    *reinterpret_cast<float4*>(mine + (size_t)rr * RW + 4 * c4) = half_sum(rr, c4);
  }
  if (threadIdx.x < rows) {
    mine[(size_t)threadIdx.x * RW + HD] = s_M[threadIdx.x];
    mine[(size_t)threadIdx.x * RW + HD + 1] = s_L[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&counters[tile], 1);
    s_last = prev == nsplit - 1;
    if (s_last) {
      counters[tile] = 0;  // every split of this launch has arrived: ready for the next launch
      __threadfence();
    }
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x < rows) {  // per row: the splits' weights e_k / sum_k(L_k e_k)
    const int rr = threadIdx.x;
    float M = -INFINITY;
    for (int k = 0; k < nsplit; ++k) M = fmaxf(M, __ldcg(tp + ((size_t)k * rows + rr) * RW + HD));
    float L = 0.0f;
    for (int k = 0; k < nsplit; ++k) {
      const float* row = tp + ((size_t)k * rows + rr) * RW;
      const float mk = __ldcg(row + HD);
      const float e = mk == -INFINITY ? 0.0f : exp2f(mk - M);
      s_wk[k][rr] = e;
      L += __ldcg(row + HD + 1) * e;
    }
    for (int k = 0; k < nsplit; ++k) s_wk[k][rr] = L > 0.0f ? s_wk[k][rr] / L : 0.0f;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < rows * C4; idx += blockDim.x) {
    const int rr = idx / C4, c4 = idx % C4;
    if (16 * blk + rr / hg >= qs) continue;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int k = 0; k < nsplit; ++k) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(tp + ((size_t)k * rows + rr) * RW) + c4);
      const float w = s_wk[k][rr];
      acc = make_float4(acc.x + v.x * w, acc.y + v.y * w, acc.z + v.z * w, acc.w + v.w * w);
    }
    *out_at(rr, c4) = acc;
  }
}

int launch_attention_wide(const __half* d_q, const __half* d_k, const __half* d_v, const AttnSegs& segs, int nseg,
                          const int32_t* d_parent, int qs, const LlamaDims& d, int max_pages, float* d_part,
                          size_t part_floats, int* d_counters, int n_counters, int sm_count, float* d_out, int* d_err,
                          cudaStream_t st) {
  CLM_CHECK(d.hd == 128, CLM_UNIMPLEMENTED, "attention kernel supports head_dim 128");
  const int group = d.nh / d.nkv;
  const int hg = group < kWideAttnHeads ? group : kWideAttnHeads;
  CLM_CHECK(group >= 1 && group <= kWideAttnMaxGroup && group * d.nkv == d.nh && group % hg == 0, CLM_UNIMPLEMENTED,
            "wide attention: 1, 2, 4 or 8 query heads per kv head");
  CLM_CHECK(nseg >= 1 && nseg <= kWideAttnMaxSegs && qs >= 1, CLM_INVALID_ARGUMENT, "wide attention: segments");
  const size_t ring = (size_t)kWideAttnPages * 2 * attn_page_bytes(128);
  const size_t parts = (size_t)2 * hg * 16 * kAttnRowFloats * sizeof(float);
  const size_t smem = ring + parts;
  CLM_TRY(ensure_smem(attention_wide_kernel<128>, smem));
  const float scale_log2 = (float)(1.4426950408889634 / sqrt((double)d.hd));
  // KV splits only while the tiles leave SMs idle: as many as fit in one wave (a 256-row prefill window has 128
  // tiles and runs unsplit, which measured faster than splitting it), at least four pages per split
  const int tiles = d.nkv * (group / hg) * ((qs + 15) / 16) * nseg;
  int nsplit = (sm_count > 0 ? sm_count : 148) / tiles;
  if (nsplit > max_pages / 4) nsplit = max_pages / 4;
  if (nsplit > kWideAttnMaxSplits) nsplit = kWideAttnMaxSplits;
  if (nsplit < 1) nsplit = 1;
  const size_t per_split = (size_t)hg * 16 * kAttnRowFloats;
  while (nsplit > 1 && ((size_t)tiles * nsplit * per_split > part_floats || tiles > n_counters)) --nsplit;
  return launch_pdl(attention_wide_kernel<128>, dim3(d.nkv * (group / hg), (qs + 15) / 16, nseg * nsplit),
                    dim3(32 * (2 * hg + 1)), smem, st, d_q, d_k, d_v, segs, d_parent, qs, d.nh, d.nkv, scale_log2,
                    max_pages, nsplit, d_part, d_counters, d_out, d_err);
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
