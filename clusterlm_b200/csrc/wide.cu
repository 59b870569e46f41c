// wide.cu — elementwise steps of a wide verify window (see wide.cuh).
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "pdl.cuh"
#include "wide.cuh"

namespace clm {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormUnits = 4;  // 8-column units per thread: H <= 8 * 256 * 4

__device__ __forceinline__ float4 ld_in4(const WideIn& y, size_t i) {
  float4 a = *reinterpret_cast<const float4*>(y.p + i);
  for (int k = 1; k < y.nsplit; ++k) {
    const float4 b = *reinterpret_cast<const float4*>(y.p + k * y.stride + i);
    a = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  }
  return a;
}
__device__ __forceinline__ float ld_in(const WideIn& y, size_t i) {
  float a = y.p[i];
  for (int k = 1; k < y.nsplit; ++k) a += y.p[k * y.stride + i];
  return a;
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
}

// One CTA per window row: the residual update, the row's sum of squares, then its normalised fp16 tile chunks.
__global__ void __launch_bounds__(kNormThreads) wide_norm_prep_kernel(const WideIn y, float* __restrict__ h, int H,
                                                                      const float* __restrict__ w, float eps, int P,
                                                                      uint8_t* __restrict__ xh) {
  griddep_wait();
  griddep_launch();
  __shared__ float s_red[kNormThreads / 32];
  const int p = blockIdx.x, tid = threadIdx.x, units = H / 8;
  float* hp = h + (size_t)p * H;
  const size_t yrow = (size_t)p * H;
  float v[kNormUnits][8];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kNormUnits; ++k) {
    const int u = tid + kNormThreads * k;
    if (u >= units) continue;
    float4 a = *reinterpret_cast<const float4*>(hp + 8 * u), b = *reinterpret_cast<const float4*>(hp + 8 * u + 4);
    if (y.p) {
      const float4 c = ld_in4(y, yrow + 8 * u), e = ld_in4(y, yrow + 8 * u + 4);
      a = make_float4(a.x + c.x, a.y + c.y, a.z + c.z, a.w + c.w);
      b = make_float4(b.x + e.x, b.y + e.y, b.z + e.z, b.w + e.w);
      *reinterpret_cast<float4*>(hp + 8 * u) = a;
      *reinterpret_cast<float4*>(hp + 8 * u + 4) = b;
    }
    v[k][0] = a.x; v[k][1] = a.y; v[k][2] = a.z; v[k][3] = a.w;
    v[k][4] = b.x; v[k][5] = b.y; v[k][6] = b.z; v[k][7] = b.w;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (tid % 32 == 0) s_red[tid / 32] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += s_red[i];
  const float sc = 1.0f / sqrtf(tot / (float)H + eps);
#pragma unroll
  for (int k = 0; k < kNormUnits; ++k) {
    const int u = tid + kNormThreads * k;
    if (u >= units) continue;
    const float4 a = *reinterpret_cast<const float4*>(w + 8 * u), b = *reinterpret_cast<const float4*>(w + 8 * u + 4);
    const float wv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[k][i] * sc * wv[i];
    *reinterpret_cast<uint4*>(xh + (size_t)(u / 8) * P * 128 + tc_tile_off(p, u % 8)) = pack8(o);
  }
}

// Depth of tree node i (its ancestors in the window), at most 255.
__device__ __forceinline__ int node_depth(const int32_t* parent, int i) {
  int d = 0;
  for (int a = parent[i]; a >= 0 && d < 256; a = parent[a]) ++d;
  return d;
}

// Grid (window row, head of the QKV rows), hd / 2 threads: one RoPE pair (or two V dims) each.
__global__ void wide_rope_kv_kernel(const WideIn y, int nh, int nkv, int hd,
                                    const float2* __restrict__ rope, const long long* __restrict__ d_pos,
                                    const int32_t* __restrict__ pages, const int32_t* __restrict__ parent,
                                    __half* __restrict__ q16, __half* __restrict__ kpool, __half* __restrict__ vpool) {
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x, head = blockIdx.y, pr = threadIdx.x;
  const int rows = (nh + 2 * nkv) * hd;
  const float a = ld_in(y, (size_t)p * rows + head * hd + 2 * pr), b = ld_in(y, (size_t)p * rows + head * hd + 2 * pr + 1);
  const long long base = *d_pos, slot = base + p;
  const int32_t page = pages[slot / kPageTokens];
  const int pos = (int)(slot % kPageTokens), d0 = 2 * pr;
  if (head < nh + nkv) {
    const long long rope_pos = parent ? base + node_depth(parent, p) : slot;
    const float2 cs = rope[(size_t)rope_pos * (hd / 2) + pr];
    const float ra = a * cs.x - b * cs.y, rb = a * cs.y + b * cs.x;
    __half* dst;
    if (head < nh)
      dst = q16 + ((size_t)p * nh + head) * hd + d0;
    else
      dst = kpool + (((size_t)page * nkv + (head - nh)) * kPageTokens + pos) * hd + 8 * kv_k_chunk(d0 >> 3, pos) +
            (d0 & 7);
    dst[0] = __float2half_rn(ra);
    dst[1] = __float2half_rn(rb);
  } else {
    __half* vt = vpool + (((size_t)page * nkv + (head - nh - nkv)) * hd + d0) * kPageTokens;
    vt[8 * kv_v_chunk(pos >> 3, d0) + (pos & 7)] = __float2half_rn(a);
    vt[kPageTokens + 8 * kv_v_chunk(pos >> 3, d0 + 1) + (pos & 7)] = __float2half_rn(b);
  }
}

// Grid (window row, F / 512), 64 threads: eight consecutive ffn indices each.
__global__ void wide_swiglu_prep_kernel(const WideIn y, int F, int P, uint8_t* __restrict__ xh) {
  griddep_wait();
  griddep_launch();
  const int p = blockIdx.x;
  const int j0 = (blockIdx.y * 64 + threadIdx.x) * 8;
  if (j0 >= F) return;
  const size_t g = (size_t)p * 2 * F + (size_t)(j0 / 64) * 128 + j0 % 64;
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float gv = ld_in(y, g + i), uv = ld_in(y, g + 64 + i);
    o[i] = gv / (1.0f + expf(-gv)) * uv;
  }
  *reinterpret_cast<uint4*>(xh + (size_t)(j0 / 64) * P * 128 + tc_tile_off(p, (j0 % 64) / 8)) = pack8(o);
}

}  // namespace

int launch_wide_norm_prep(WideIn d_y, float* d_h, int q, int H, const float* d_w, float eps, int P,
                          uint8_t* d_xh, cudaStream_t st) {
  CLM_CHECK(H % 64 == 0 && H <= 8 * kNormThreads * kNormUnits, CLM_UNIMPLEMENTED, "wide window: hidden size");
  CLM_CHECK(q >= 1 && q <= P && P % 16 == 0, CLM_INVALID_ARGUMENT, "wide window: row count");
  return launch_pdl(wide_norm_prep_kernel, dim3(q), dim3(kNormThreads), 0, st, d_y, d_h, H, d_w, eps, P, d_xh);
}

int launch_wide_rope_kv(WideIn d_y, int q, const LlamaDims& d, const float2* d_rope, const long long* d_pos,
                        const int32_t* d_pages, const int32_t* d_parent, __half* d_q16, __half* d_kpool,
                        __half* d_vpool, cudaStream_t st) {
  CLM_CHECK(d.hd % 16 == 0 && d.hd <= 256, CLM_UNIMPLEMENTED, "wide window: head dim");
  return launch_pdl(wide_rope_kv_kernel, dim3(q, d.nh + 2 * d.nkv), dim3(d.hd / 2), 0, st, d_y, d.nh, d.nkv, d.hd,
                    d_rope, d_pos, d_pages, d_parent, d_q16, d_kpool, d_vpool);
}

int launch_wide_swiglu_prep(WideIn d_y, int q, int F, int P, uint8_t* d_xh, cudaStream_t st) {
  CLM_CHECK(F % 64 == 0, CLM_UNIMPLEMENTED, "wide window: ffn size");
  return launch_pdl(wide_swiglu_prep_kernel, dim3(q, (F + 511) / 512), dim3(64), 0, st, d_y, F, P, d_xh);
}

}  // namespace clm
