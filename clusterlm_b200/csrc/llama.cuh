// llama.cuh — kernels of the Llama-shaped decoder family (dense GQA attention with RoPE, SwiGLU FFN,
// GGUF Q4_K / Q8_0 weights, paged fp16 KV cache).  The reference has no implementation of this family
// (its llama path is the un-vendored llama.cpp); the per-layer math is the oracle's orc_llama_layer.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace clm {

constexpr int kPageTokens = 64;  // KV page: 64 positions of one KV head
constexpr int kAttnPages = 4;    // page buffers per attention CTA
constexpr int kAttnWarps = 8;    // warps per attention CTA (two per page buffer, half a page each)
constexpr int kAttnMaxSplits = 24;  // partials a thread of the final attention combine loads at once
constexpr int kAttnRowFloats = 132;  // one partial row: O[128], m, l, 2 floats of padding (16-byte aligned rows)

struct LlamaDims {
  int H = 0, nh = 0, nkv = 0, hd = 0, F = 0, V = 0;
  float theta = 500000.0f, eps = 1e-5f;
  int quant = CLM_QUANT_Q4_K;
  int qd() const { return nh * hd; }
  int kvd() const { return nkv * hd; }
};

// Swizzled 16-byte chunks of a KV page (bank-conflict-free shared-memory reads of the attention kernel):
//   K page [64 positions][128 head dims] fp16: head-dim chunk c (8 dims) of position pos is stored at chunk
//     kv_k_chunk(c, pos) of that position's row;
//   V^T page [128 head dims][64 positions] fp16: position chunk c (8 positions) of head dim d is stored at chunk
//     kv_v_chunk(c, d) of that dim's row.
__host__ __device__ __forceinline__ int kv_k_chunk(int c, int pos) { return c ^ (((c >> 3) & 1) << 1) ^ (pos & 1); }
__host__ __device__ __forceinline__ int kv_v_chunk(int c, int d) { return c ^ (d & 1); }

// Attention partials of one (m-tile, kv head, page): 16 rows x (hd values + m + l).
inline size_t attn_partial_floats(int hd) { return (size_t)16 * (hd + 4); }

int launch_embed(const uint8_t* d_embd, int quant, const int32_t* d_tokens, int q, int H, float* d_h, cudaStream_t st);
// Paged split-KV attention for q window rows: per (kv head, m-tile of 16 query rows) S splits own contiguous page
// ranges (pages staged in shared memory by bulk copies, committed pages before griddepcontrol.wait, online softmax
// per warp), write one partial each, and every split then combines a slice of the outputs over all partials and
// writes W_o's input fragments (out_frag / out_sum, qd columns).  S is chosen so that the grid fits the SM count.
// d_part holds mtiles*nkv*max_pages*attn_partial_floats(hd) floats; d_counters 2*mtiles*nkv zeroed ints (left zero);
// a bounded wait that gives up stores kErrWaitTimeout in *d_err.  [d_prefetch, d_prefetch + prefetch_bytes) (the next
// kernel's weights, or null) is prefetched into L2, split over the CTAs.  With d_out_f32 (wide windows, any q) the
// outputs go to f32 rows d_out_f32[q][qd] instead of the fragments; when the (kv head, m-tile) pairs outnumber the
// SMs each pair has one split.
//
// Dataflow inside a window chain (link.wait non-null): kv head h's inputs (its query heads, k and v rows from the
// QKV GEMV) are ready once link.wait[h] >= link.target; the kernel does not wait for its predecessor's completion.
// Every CTA adds 1, once its share of the W_o fragments is written, to link.sig[h * span + i] for i < span (a kv
// head's query heads cover `span` 512-column chunks) or to link.sig[h / kvh_div] (kv heads sharing a chunk).
struct AttnLink {
  const int* wait = nullptr;
  int target = 0;
  int* sig = nullptr;
  int span = 1, kvh_div = 1;
};
int launch_attention(const __half* d_q, const __half* d_k, const __half* d_v, const int32_t* d_pages,
                     const long long* d_pos, const int32_t* d_parent, int q, const LlamaDims& d, int max_pages,
                     float* d_part, int* d_counters, int nt_out, float hi_scale, void* d_frag, float* d_sum,
                     int* d_err, const uint8_t* d_prefetch, unsigned long long prefetch_bytes, int sm_count,
                     cudaStream_t st, float* d_out_f32 = nullptr, const AttnLink& link = AttnLink{},
                     int row_off = 0, int q_frag = 0);
// row_off / q_frag: the window's rows are rows row_off .. row_off + q - 1 of a batched window of q_frag rows (the W_o
// fragments of every session of the batch; q_frag 0 = q).
// Splits per (kv head, m-tile) that launch_attention uses for these arguments (its grid is nkv x splits x mtiles).
int attention_splits(int q, const LlamaDims& d, int max_pages, int sm_count);
// Wide-window attention (windows of more than 16 rows, and batched windows of several sessions): one CTA per
// (kv head, block of 16 window rows, session segment) holds the block's rows of every query head of the kv head
// (16 x group rows; a group of 8 is split over two CTAs of 4 heads) and streams the segment's visible KV pages once through a 3-page ring (bulk copies by a
// producer warp); two warps per 16-row m-tile take the two halves of each page with an online softmax, and the CTA
// combines them into f32 rows out[row0 + i][nh * hd].  Segment s: window rows row0[s] .. row0[s] + qs - 1 of
// q16 / out, committed position *pos[s], page table pages[s]; parent (shared tree shape, or null for linear
// windows) as in launch_attention.  group = nh / nkv <= 8, hd = 128, at most kWideAttnMaxSegs segments.
constexpr int kWideAttnMaxSegs = 16;
struct AttnSegs {
  const long long* pos[kWideAttnMaxSegs];
  const int32_t* pages[kWideAttnMaxSegs];
  int row0[kWideAttnMaxSegs];
};
// With fewer (kv head, block, segment) tiles than SMs the visible pages are split over up to 8 CTAs per tile (as
// many as fit in one wave): each writes its partial to d_part (part_floats floats) and the last to arrive on the tile's
// counter (d_counters: n_counters zeroed ints, left zero) combines them; no CTA waits for another.
int launch_attention_wide(const __half* d_q, const __half* d_k, const __half* d_v, const AttnSegs& segs, int nseg,
                          const int32_t* d_parent, int qs, const LlamaDims& d, int max_pages, float* d_part,
                          size_t part_floats, int* d_counters, int n_counters, int sm_count, float* d_out, int* d_err,
                          cudaStream_t st);
// Copies h[p][0:H] of rows into the boundary records out[p] = {S = h, P = 0, g = 1} (hc = 1).
int launch_pack_boundary(const float* d_h, const float* d_part, int nsplit, int q, int H, float* d_out,
                         cudaStream_t st);
// Folds boundary records (S + g*P) into h (hc = 1).
int launch_unpack_boundary(const float* d_in, int q, int H, float* d_h, cudaStream_t st);

}  // namespace clm
