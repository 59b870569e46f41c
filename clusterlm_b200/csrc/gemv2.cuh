// gemv2.cuh — activation hand-off and fused epilogues of the q-row GEMV chain (kernel in gemv4.cu).
//
// y[p][row] = W[row] . x[p] for q <= 16 window rows, W in GGUF Q4_K / Q8_0 repacked into the group-major tile
// layout of gemv.cuh.
//
//  * Activations come from the producer kernel as fp16 fragments xfrag[sb][nt][16 s][32 lanes] (uint2) and the
//    sums of every 16-column half of every 32-column sub-block, split into fp16 hi + lo and stored directly as the
//    B fragments of the Q4_K min / Q8_0 bias mma: xsum[sb][n-tile (2)][32 lanes] of four words {hi half 0,
//    hi half 1, lo half 0, lo half 1}, each word the pair (sub-block 2t, 2t+1) of lane (g, t) = window row g of
//    the n-tile.  Both written by prep16 below.
//  * Optional row scale 1/sqrt(mean(h^2) + eps) from sum-of-squares partials: rmsnorm(h) * w is folded as
//    (W . (h * w)) / denom, so no separate normalisation kernel runs between layers.
//  * Epilogues: store; residual add + next-norm preparation; RoPE + paged KV append; SwiGLU + down preparation.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace clm {

enum { EPI_STORE = 0, EPI_RESID_PREP = 1, EPI_ROPE_KV = 2, EPI_SWIGLU_PREP = 3 };

// Activation hand-off between a producer and a consuming GEMV.
struct XBuf {
  uint2* frag = nullptr;   // [SB][nt][16 s][32 lanes]
  float* sum = nullptr;    // [SB][sum_tiles(nt) n-tiles][32 lanes][4 words] min / bias mma B fragments (512 B each)
  float* ss = nullptr;     // [nss][kSsRows p] sum-of-squares partials, one per 128 (or 16) columns, or null
  int nss = 0;
};

struct Epi {
  int kind = EPI_STORE;
  // row scale: 1 / sqrtf(sum(ss) / ss_n + eps), from the input XBuf's ss partials
  float ss_n = 0.0f, eps = 0.0f;
  // EPI_STORE: out[p * out_ld + row]
  float* out = nullptr;
  long long out_ld = 0;
  // EPI_RESID_PREP: h[p * H + row] += y; next input = h * wnext (fragments for a consumer with hi_scale)
  float* h = nullptr;
  int H = 0;
  const float* wnext = nullptr;
  XBuf next;
  float hi_scale = 1.0f;
  // EPI_ROPE_KV
  int nh = 0, nkv = 0, hd = 0;
  const float2* rope = nullptr;  // [position][hd/2] (cos, sin) of position * theta^(-2i/hd)
  const long long* pos = nullptr;
  const int32_t* parent = nullptr;
  const int32_t* pages = nullptr;
  __half* kpool = nullptr;
  __half* vpool = nullptr;
  __half* q16 = nullptr;
  // EPI_ROPE_KV over a window of several sessions (seg_q > 0): rows [s * seg_q, (s + 1) * seg_q) belong to session
  // s, at its committed position *seg_pos[s] with its page table seg_pages[s] (linear windows; pos / pages unused)
  int seg_q = 0;
  const long long* seg_pos[4] = {};
  const int32_t* seg_pages[4] = {};
  // EPI_SWIGLU_PREP: rows of the CTA's first tile are gate rows, second tile the matching up rows
  int ffn = 0;
  int* err = nullptr;  // set to 1 if a bounded wait gave up
  // L2 lookahead: once a CTA's producer has issued its own copies it prefetches into L2 the first pf_cap bytes of
  // its share of the next kernel's weights [pf, pf + pf_bytes) (split like the next kernel's stream-K ranges), so
  // the next kernel's first copies hit L2 while this kernel drains.  With EPI_ROPE_KV and pf_kv the prefetch is
  // instead this layer's KV pages [0, ceil((pos + q) / 64)) for the attention that follows.
  const uint8_t* pf = nullptr;
  unsigned long long pf_bytes = 0, pf_cap = 0;
  bool pf_kv = false;
  int pf_max_pages = 0;
  // Dataflow inside a window chain (gemv4.cu, gemv_strip.cu).  wait == null: the kernel reads what its predecessor
  // wrote after griddepcontrol.wait.  Otherwise input chunk c (the 512 columns of the units' superblock pair c) is
  // ready once wait[c] >= wait_target and the row scale's sums of squares once *ss_done >= ss_target, and the kernel
  // never waits for its predecessor's completion: everything it reads is published by release-adds that it acquires,
  // and no CTA of a linked launch touches memory after its last signal, so a plain launch that waits for the chain's
  // last kernel sees all of the chain's results.  A finished row group g adds 1 to sig[g / sig_div] (sig_qkv: to its
  // kv head's counter) and to *done (either may be null).
  const int* wait = nullptr;
  int wait_target = 0;
  const int* ss_done = nullptr;
  int ss_target = 0;
  int* sig = nullptr;
  int sig_div = 1;
  int sig_qkv = 0;
  int* done = nullptr;
};

// The fused GEMV (gemv4.cu) over the group-major tile layout of gemv.cuh.  `part` holds ng*p.ksplit*q*128 f32
// segment partials and `counters` ng zero-initialised ints (left zero after every launch).
int launch_gemv(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi,
                float* part, int* counters, cudaStream_t st);
// Units (or strip stages) that the GEMVs prefetch into L2 beyond their shared-memory ring (CLM_B200_L2AHEAD).  Off
// by default: the stream is bound by the consumers' dequantisation, and prefetching ahead measured slower.
constexpr int kL2Ahead = 0;
int gemv_l2_ahead();

// Producer helpers.
// x[q][cols] fp32 (row stride ld) times optional w[cols] -> fragments + sums (+ ss partials over 16-column
// groups when with_ss).  Rows p in [q, 8*nt) are written as zeros.
int launch_prep_rows(const float* d_x, long long ld, int q, int cols, const float* d_w, int nt, float hi_scale,
                     const XBuf& out, bool with_ss, cudaStream_t st);
// Bytes of the fragment / sum buffers for `cols` columns.
inline size_t xfrag_bytes(int cols, int nt) { return (size_t)(cols / 256) * nt * 32 * 16 * sizeof(uint2); }
inline size_t xsum_bytes(int cols, int nt = 2) { return (size_t)(cols / 256) * 512 * sum_tiles(nt); }

// Device helper shared by producers: writes the fragments / half sums of one 16-column group [16c, 16c+16)
// of activation row p from `vals` (16 floats, already multiplied by the next norm's weight if any) and, when
// ss_out is set, the sum of squares of `raw` (the values being normalised).  p >= q writes zeros.  One
// thread per (group, p).
__device__ __forceinline__ void prep16(const float* vals, const float* raw, int p, int q, int c, int nt,
                                       float hi_scale, uint2* __restrict__ frag, float* __restrict__ xsum,
                                       float* ss_out, int total_cols) {
  const int k = 16 * c, sb = k / 256, o = k % 256, t = o / 64, part = (o % 64) / 32, s0 = (o % 32) / 2;
  const int ntile = p / 8, g = p % 8;
  // fragment layout [sb][nt][s][lane] (gemv.cuh): word (s, lane) at ((sb*nt + ntile)*16 + s)*32 + lane; with 4 n-tiles
  // the n-tiles are interleaved in pairs, [sb][nt / 2][s][lane][2], so that one 16-byte load reads two n-tiles
  uint32_t* w;
  int sstride;  // u32 words between consecutive k-steps s
  if (nt == 4) {
    w = reinterpret_cast<uint32_t*>(frag + (((size_t)sb * 2 + ntile / 2) * 16 * 32 + g * 4 + t) * 2 + (ntile & 1));
    sstride = 128;
  } else {
    w = reinterpret_cast<uint32_t*>(frag + ((size_t)sb * nt + ntile) * 512 + g * 4 + t);
    sstride = 64;
  }
  float sum = 0.0f, ss = 0.0f;
  const bool live = p < q;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = live ? vals[2 * i] : 0.0f, b = live ? vals[2 * i + 1] : 0.0f;
    sum += a + b;
    if (raw && live) ss += raw[2 * i] * raw[2 * i] + raw[2 * i + 1] * raw[2 * i + 1];
    const float sa = part ? a * hi_scale : a, sbv = part ? b * hi_scale : b;
    w[(s0 + i) * sstride + part] =
        (uint32_t)__half_as_ushort(__float2half_rn(sa)) | ((uint32_t)__half_as_ushort(__float2half_rn(sbv)) << 16);
  }
  const int j = o / 32, half = (o % 32) / 16;
  const int ns = sum_tiles(nt);
  if (p < 8 * ns) {
    // B fragment words of the min / bias mma (k = half * 8 + sub-block): lane (p % 8, j / 2), element j % 2
    const __half hi = __float2half_rn(sum);
    const __half lo = __float2half_rn(sum - __half2float(hi));
    __half* wq = reinterpret_cast<__half*>(xsum) + ((((size_t)sb * ns + ntile) * 32 + g * 4 + (j >> 1)) * 4) * 2;
    wq[half * 2 + (j & 1)] = hi;
    wq[(2 + half) * 2 + (j & 1)] = lo;
  }
  if (ss_out && p < kSsRows) ss_out[(size_t)c * kSsRows + p] = ss;
  (void)total_cols;
}

}  // namespace clm
