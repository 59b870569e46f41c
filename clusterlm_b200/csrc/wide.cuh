// wide.cuh — the elementwise steps of a wide verify window (17..256 rows: prefill chunks and large tree windows)
// around the tensor-core GEMMs of gemm_tc.cuh.  Each step reads the previous GEMM's f32 rows and writes the next
// GEMM's fp16 activation tiles (tc_tile_off layout), or the attention's inputs (q16 rows, paged KV).
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"
#include "llama.cuh"

namespace clm {

// A GEMM's f32 output as the wide steps read it: y[i] = sum over k < nsplit of p[k * stride + i], in split order
// (nsplit = 1: the GEMM wrote y itself).
struct WideIn {
  const float* p = nullptr;
  int nsplit = 1;
  unsigned long long stride = 0;
};

// h[p] (+= y[p] when y.p is not null), then the next GEMM's tiles of rmsnorm(h[p]) * w:
// x = h * w / sqrt(mean(h^2) + eps), p < q, K = H columns, tiles of P rows.  H % 8 == 0, H <= 8192.
int launch_wide_norm_prep(WideIn y, float* d_h, int q, int H, const float* d_w, float eps, int P,
                          uint8_t* d_xh, cudaStream_t st);

// The QKV rows y[p][(nh + 2 nkv) * hd] of window row p at KV slot base + p (base = *d_pos): RoPE of the q and k
// heads at position base + p (linear) or base + depth(p) (tree, parent[p] < p or -1), q heads -> q16[p][nh][hd],
// k / v heads -> the paged fp16 pools (kv_k_chunk / kv_v_chunk layout of llama.cuh).
int launch_wide_rope_kv(WideIn y, int q, const LlamaDims& d, const float2* d_rope, const long long* d_pos,
                        const int32_t* d_pages, const int32_t* d_parent, __half* d_q16, __half* d_kpool,
                        __half* d_vpool, cudaStream_t st);

// SwiGLU of the gate|up rows y[p][2F] (row group g of 128: gate of ffn indices 64g..64g+63, then their up rows)
// -> the down GEMM's tiles of silu(gate) * up, K = F columns.
int launch_wide_swiglu_prep(WideIn y, int q, int F, int P, uint8_t* d_xh, cudaStream_t st);

}  // namespace clm
