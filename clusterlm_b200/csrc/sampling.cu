// sampling.cu — greedy/stochastic sampling and speculative acceptance on the device.
//
// Reference semantics: runtime/domain/src/sampling.cpp:44-131.
//  * argmax: first index of the maximum (ties to the lowest index).
//  * distribution: e_i = exp(double(l_i - max) / T), P_i = float(e_i / sum e).
//  * sample_from: total = serial double sum; r = u * total; first nonzero i with r < acc_i where acc_i is the
//    serial double prefix sum; else the last nonzero index.
//  * verify_speculative: accept draft j if u < min(1, p/q) (u drawn only when q > 0); on the first rejection
//    sample float(max(0, P - Q)) (or P when that mass is zero); if all are accepted sample the bonus row.
//
// sample_from is reproduced bit for bit without a serial walk.  Every positive f32 value is an integer
// multiple of 2^-149, so prefix sums are computed EXACTLY in 192-bit fixed point.  The serial double sums
// differ from the exact ones by at most g*S (recursive summation bound, g ~ V*2^-53), and r likewise.  The
// index is taken from the exact prefixes only when that bound proves the serial comparisons give the same
// index; otherwise (probability ~V*g per draw) one thread re-walks the row serially.
//
// Every row operation is spread over ceil(V / kSampleChunk) CTAs per row ("chunks"): per-chunk partial results
// go to scratch, and the last CTA of a row (atomic counter, left at zero afterwards) combines them in chunk
// order, so results are deterministic and independent of scheduling.
#include <cfloat>

#include "common.cuh"
#include "pdl.cuh"
#include "sampling.cuh"
#include "exp2_table.cuh"

namespace clm {

// ---------------------------------------------------------------------------------------------------
// 192-bit unsigned fixed point, unit 2^-149
// ---------------------------------------------------------------------------------------------------
struct U192 {
  unsigned long long w[3];
};

__device__ __forceinline__ U192 u192_zero() { return U192{{0ull, 0ull, 0ull}}; }

__device__ __forceinline__ void u192_add(U192& a, const U192& b) {
  asm("add.cc.u64 %0, %0, %3;\n\taddc.cc.u64 %1, %1, %4;\n\taddc.u64 %2, %2, %5;"
      : "+l"(a.w[0]), "+l"(a.w[1]), "+l"(a.w[2])
      : "l"(b.w[0]), "l"(b.w[1]), "l"(b.w[2]));
}

__device__ __forceinline__ bool u192_gt(const U192& a, const U192& b) {
  if (a.w[2] != b.w[2]) return a.w[2] > b.w[2];
  if (a.w[1] != b.w[1]) return a.w[1] > b.w[1];
  return a.w[0] > b.w[0];
}

// x must be finite, >= 0 and < 2^20 (checked by the caller).
__device__ __forceinline__ U192 u192_from_float(float x) {
  const uint32_t bits = __float_as_uint(x);
  const uint32_t e = bits >> 23;
  const unsigned long long m = e == 0 ? (bits & 0x7FFFFFu) : ((bits & 0x7FFFFFu) | 0x800000u);
  const int shift = e == 0 ? 0 : (int)e - 1;  // value = m * 2^(shift) units of 2^-149
  U192 r = u192_zero();
  const int wi = shift / 64, bi = shift % 64;
  r.w[wi] = m << bi;
  if (bi > 40 && wi < 2) r.w[wi + 1] = m >> (64 - bi);
  return r;
}

// Approximate value in units of 1 (relative error < 2^-52).
__device__ __forceinline__ double u192_to_double(const U192& a) {
  return ((double)a.w[2] * 0x1.0p128 + (double)a.w[1] * 0x1.0p64 + (double)a.w[0]) * 0x1.0p-149;
}

// ceil (up = true) or floor of v * 2^149 as U192; v >= 0.  Returns false if it does not fit.
__device__ bool u192_from_double(double v, bool up, U192* out) {
  *out = u192_zero();
  if (!(v > 0.0)) return v == 0.0;
  int e;
  const double f = frexp(v, &e);                                 // v = f * 2^e, f in [0.5, 1)
  const unsigned long long m = (unsigned long long)ldexp(f, 53);  // exact 53-bit integer
  int sh = e - 53 + 149;                                         // V = m * 2^sh
  if (sh + 53 > 191) return false;
  if (sh >= 0) {
    const int wi = sh / 64, bi = sh % 64;
    out->w[wi] = m << bi;
    if (bi > 11 && wi < 2) out->w[wi + 1] = m >> (64 - bi);
    return true;
  }
  const int rs = -sh;
  unsigned long long q = rs >= 64 ? 0ull : (m >> rs);
  const bool frac = rs >= 64 ? (m != 0) : ((m & ((1ull << rs) - 1ull)) != 0);
  if (up && frac) q += 1;
  out->w[0] = q;
  return true;
}

__device__ __forceinline__ U192 shfl_up_u192(const U192& v, int d) {
  U192 r;
#pragma unroll
  for (int i = 0; i < 3; ++i) r.w[i] = __shfl_up_sync(0xffffffffu, v.w[i], d);
  return r;
}

// Block-wide exclusive scan of U192 (blockDim.x multiple of 32, <= 1024).  Returns the exclusive prefix for
// the calling thread and writes the block total to *total (all threads).
__device__ U192 block_exclusive_scan(const U192& v, U192* total) {
  __shared__ U192 warp_sums[32];
  __shared__ U192 tot;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  U192 inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    U192 o = shfl_up_u192(inc, d);
    if (lane >= d) u192_add(inc, o);
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    U192 ws = lane < nw ? warp_sums[lane] : u192_zero();
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      U192 o = shfl_up_u192(ws, d);
      if (lane >= d) u192_add(ws, o);
    }
    if (lane < nw) warp_sums[lane] = ws;  // inclusive warp prefix
    if (lane == nw - 1) tot = ws;
  }
  __syncthreads();
  U192 before = warp > 0 ? warp_sums[warp - 1] : u192_zero();
  // exclusive prefix of this thread = before + (inc - v); compute as before + exclusive within the warp
  U192 excl = shfl_up_u192(inc, 1);
  if (lane == 0) excl = u192_zero();
  u192_add(before, excl);
  *total = tot;
  __syncthreads();
  return before;
}

// Block-wide exclusive max-scan of ints (identity -1); *all_max receives the block maximum.
__device__ int32_t block_exclusive_max(int32_t v, int32_t* all_max) {
  __shared__ int32_t wmax[32];
  __shared__ int32_t s_all;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  int32_t inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int32_t o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc = max(inc, o);
  }
  if (lane == 31) wmax[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int32_t w = lane < nw ? wmax[lane] : -1;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t o = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w = max(w, o);
    }
    if (lane < nw) wmax[lane] = w;
    if (lane == nw - 1) s_all = w;
  }
  __syncthreads();
  int32_t excl = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) excl = -1;
  if (warp > 0) excl = max(excl, wmax[warp - 1]);
  *all_max = s_all;
  __syncthreads();
  return excl;
}

__device__ __forceinline__ bool fast_ok(float x) { return x >= 0.0f && x < 1048576.0f; }  // false for NaN / inf

// The reference's serial sample_from over values fx(0..n-1) with uniform u (one thread).
template <typename F>
__device__ int32_t serial_sample(const F& fx, uint32_t n, double u) {
  double total = 0;
  for (uint32_t i = 0; i < n; ++i) total += (double)fx(i);
  const double r = u * total;
  double acc = 0;
  int32_t last = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const float v = fx(i);
    if (v <= 0.0f) continue;
    acc += (double)v;
    last = (int32_t)i;
    if (r < acc) return last;
  }
  return last;
}


// ---------------------------------------------------------------------------------------------------
// scratch
// ---------------------------------------------------------------------------------------------------
namespace {
size_t al(size_t n) { return (n + 255) & ~size_t{255}; }
}  // namespace

size_t SampleScratch::bytes(uint32_t rows, uint32_t seqs, uint32_t V) {
  const size_t C = sample_chunks(V);
  return al((rows + seqs) * sizeof(int)) + al(rows * C * 4) + al(rows * C * 8) + al(rows * 4) + al(rows * 8) +
         al(rows * C * 4) + al(rows * C * 4) + al(seqs * 2 * C * 24) + al(seqs * 2 * C * 4) + al(seqs * C * 4) +
         al(seqs * 8) + al(seqs * 4);
}

SampleScratch SampleScratch::carve(void* base, uint32_t rows, uint32_t seqs, uint32_t V) {
  const size_t C = sample_chunks(V);
  uint8_t* p = static_cast<uint8_t*>(base);
  SampleScratch s;
  s.rows = rows;
  s.seqs = seqs;
  s.chunks = (uint32_t)C;
  auto take = [&](size_t n) {
    uint8_t* r = p;
    p += al(n);
    return r;
  };
  s.rcnt = reinterpret_cast<int*>(take((rows + seqs) * sizeof(int)));
  s.scnt = s.rcnt + rows;
  s.counter_bytes = al((rows + seqs) * sizeof(int));
  s.cmax = reinterpret_cast<float*>(take(rows * C * 4));
  s.csum = reinterpret_cast<double*>(take(rows * C * 8));
  s.mx = reinterpret_cast<float*>(take(rows * 4));
  s.kept = reinterpret_cast<double*>(take(rows * 8));
  s.cval = reinterpret_cast<float*>(take(rows * C * 4));
  s.cidx = reinterpret_cast<int32_t*>(take(rows * C * 4));
  s.c192 = reinterpret_cast<unsigned long long*>(take(seqs * 2 * C * 24));
  s.clast = reinterpret_cast<int32_t*>(take(seqs * 2 * C * 4));
  s.cflag = reinterpret_cast<int*>(take(seqs * C * 4));
  s.u = reinterpret_cast<double*>(take(seqs * 8));
  s.sel = reinterpret_cast<int32_t*>(take(seqs * 4));
  return s;
}

// ---------------------------------------------------------------------------------------------------
// block reductions
// ---------------------------------------------------------------------------------------------------
constexpr int kSampleThreads = 256;
constexpr int kPerThread = kSampleChunk / kSampleThreads;  // 8 contiguous entries per thread

__device__ float block_max(float v) {
  __shared__ float sm[32];
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x / 32) ? sm[lane] : -FLT_MAX;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  v = sm[0];
  __syncthreads();
  return v;
}

__device__ double block_sum_d(double v) {
  __shared__ double sm[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x / 32) ? sm[lane] : 0.0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  v = sm[0];
  __syncthreads();
  return v;
}

// (value, index) maximum with ties to the lower index; NaN values never win.
__device__ __forceinline__ void argmax_merge(float& bv, int32_t& bi, float v, int32_t i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__device__ void block_argmax_pair(float& bv, int32_t& bi) {
  __shared__ float sv[32];
  __shared__ int32_t si[32];
  for (int o = 16; o > 0; o >>= 1) argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = lane < (int)(blockDim.x / 32) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x / 32) ? si[lane] : INT32_MAX;
    for (int o = 16; o > 0; o >>= 1)
      argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) {
      sv[0] = bv;
      si[0] = bi;
    }
  }
  __syncthreads();
  bv = sv[0];
  bi = si[0];
  __syncthreads();
}

// The last CTA of row r (of `total` CTAs) gets true; the counter is left at zero.
__device__ bool last_of(int* cnt, int total) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(cnt, 1) == total - 1;
    if (s_last) *cnt = 0;
  }
  __syncthreads();
  const bool r = s_last;
  if (r) __threadfence();
  return r;
}

__device__ __forceinline__ float read_temperature(float T, const RoundCtl* ctl) { return ctl ? ctl->temperature : T; }

// exp(x) for x <= 0 in double precision by Tang's table-driven method (P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point arithmetic", ACM TOMS 15(2), 1989), with a
// 2048-entry table (exp2_table.cuh): x = (k + r') ln2 / 2048 with k = round(x * 2048 / ln2), taken from the low bits
// of x * 2048 / ln2 + 1.5 * 2^52 (no conversion instructions), and |r| <= ln2 / 4096 (ln2 / 2048 split into a
// 29-bit head, so that k * head is exact, and a tail); exp(x) = 2^(k >> 11) * T[k & 2047] * (1 + p(r)) with p the
// degree-4 Taylor polynomial of exp(r) - 1 (truncation below 1e-20 relative).  Within 1 ulp of exp, like a library
// exp; results that would be subnormal, -inf and NaN take the library exp.
__device__ __forceinline__ double exp_nonpos(double x) {
  if (!(x > -707.0)) return exp(x);
  constexpr double kShift = 0x1.8p52;
  double kd = fma(x, k2048ByLn2, kShift);
  const int k = (int)(unsigned)__double_as_longlong(kd);  // the rounded integer sits in the low bits
  kd -= kShift;
  double r = fma(kd, -kLn2By2048Head, x);
  r = fma(kd, -kLn2By2048Tail, r);
  double t = fma(r, 1.0 / 24.0, 1.0 / 6.0);
  t = fma(r, t, 0.5);
  const double p = fma(r * r, t, r);
  const double tab = __ldg(&kExp2Tab2048[k & 2047]);
  const double y = fma(tab, p, tab);
  return __longlong_as_double(__double_as_longlong(y) + ((long long)(k >> 11) << 52));
}

// e = exp(double(l - m) / T), the reference's softmax term (sampling.cpp:64); at T = 1 the division is the
// identity and is skipped (same value, no double division).  l <= m for every entry of a row, so x <= 0.
__device__ __forceinline__ double soft_term(float l, float m, float T) {
  const double x = (double)__fsub_rn(l, m);
  return exp_nonpos(T == 1.0f ? x : x / (double)T);
}

// float(e / kept), the reference's probability of a softmax term (sampling.cpp:64-83: a double quotient rounded to
// float), through a multiplication by inv = 1 / kept: the double product differs from the correctly rounded quotient
// by at most 2 ulps, so it rounds to the same float unless it lies within a few ulps of a float rounding boundary
// (a double whose 29 bits below the float mantissa are 1 << 28); there, and outside the normal float range of a
// probability, the quotient itself is computed.  Same float as (float)(e / kept) for every input.
__device__ __forceinline__ float prob_of(double e, double kept, double inv) {
  const double q = e * inv;
  if (!(q > 0x1p-125 && q < 1.0)) return (float)(e / kept);
  const long long d = (long long)(__double_as_longlong(q) & 0x1FFFFFFFll) - (1ll << 28);
  if (d > -16 && d < 16) return (float)(e / kept);
  return (float)q;
}

// ---------------------------------------------------------------------------------------------------
// argmax rows (sampling.cpp:44-49): first index of the maximum; a NaN at index 0 pins the answer to 0 and
// NaNs elsewhere are never chosen (the reference's `logits[i] > logits[best]` scan)
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kSampleThreads) argmax_chunks_kernel(const float* __restrict__ logits, uint32_t V,
                                                                       float* __restrict__ cval,
                                                                       int32_t* __restrict__ cidx, int* __restrict__ cnt,
                                                                       int32_t* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const uint32_t c = blockIdx.x, r = blockIdx.y, C = gridDim.x;
  const float* l = logits + (size_t)r * V;
  const uint32_t lo = c * kSampleChunk, hi = min(V, lo + kSampleChunk);
  float bv = -INFINITY;
  int32_t bi = INT32_MAX;
  for (uint32_t i = lo + threadIdx.x; i < hi; i += kSampleThreads) argmax_merge(bv, bi, l[i], (int32_t)i);
  block_argmax_pair(bv, bi);
  if (threadIdx.x == 0) {
    cval[(size_t)r * C + c] = bv;
    cidx[(size_t)r * C + c] = bi;
  }
  if (!last_of(&cnt[r], (int)C)) return;
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    int32_t ix = INT32_MAX;
    for (uint32_t k = 0; k < C; ++k) argmax_merge(v, ix, __ldcg(cval + (size_t)r * C + k), __ldcg(cidx + (size_t)r * C + k));
    out[r] = (isnan(l[0]) || ix == INT32_MAX) ? 0 : ix;
  }
}

// ---------------------------------------------------------------------------------------------------
// distribution rows (sampling.cpp:51-86, temperature only): P_i = float(exp(double(l_i - max) / T) / kept)
// ---------------------------------------------------------------------------------------------------
// Row statistics use larger chunks than the sampling kernels (kStatsChunk entries per CTA, 64 per thread, four
// independent accumulators), so that a CTA's fixed cost (reduction, arrival counter) is spread over more bytes.
constexpr uint32_t kStatsChunk = 16384;
inline uint32_t stats_chunks(uint32_t V) { return (V + kStatsChunk - 1) / kStatsChunk; }

// One chunk's statistics in one launch: the chunk maximum m_c (from -FLT_MAX, like the row maximum of the
// reference's scan) and the double sum s_c of exp(double(l - m_c) / T) in one fixed order (thread-strided float4
// lanes, four accumulators, block reduction).  The CTA reads its 64 KB chunk twice; the second pass finds it in
// L1 / L2, so DRAM sees the logits once.  Every thread of the block returns both.  The whole-row statistics and the
// vocab-shard statistics share it, so a shard that starts at a chunk boundary reproduces the whole row's chunk
// statistics bit for bit.
struct ChunkStats {
  float m;
  double s;
};
__device__ __forceinline__ ChunkStats chunk_stats(const float* __restrict__ l, uint32_t V, uint32_t c, float T) {
  const uint32_t lo = c * kStatsChunk, hi = min(V, lo + kStatsChunk);
  ChunkStats r;
  if ((V & 3u) == 0) {  // rows start 16-byte aligned: float4 loads
    const float4* l4 = reinterpret_cast<const float4*>(l);
    float m0 = -FLT_MAX, m1 = -FLT_MAX, m2 = -FLT_MAX, m3 = -FLT_MAX;
#pragma unroll 4
    for (uint32_t i = lo / 4 + threadIdx.x; i < hi / 4; i += kSampleThreads) {
      const float4 v = l4[i];
      m0 = fmaxf(m0, v.x);
      m1 = fmaxf(m1, v.y);
      m2 = fmaxf(m2, v.z);
      m3 = fmaxf(m3, v.w);
    }
    r.m = block_max(fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)));
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    // unrolled so that several iterations' loads and exps are in flight (the additions keep their order)
#pragma unroll 4
    for (uint32_t i = lo / 4 + threadIdx.x; i < hi / 4; i += kSampleThreads) {
      const float4 v = l4[i];
      a0 += soft_term(v.x, r.m, T);
      a1 += soft_term(v.y, r.m, T);
      a2 += soft_term(v.z, r.m, T);
      a3 += soft_term(v.w, r.m, T);
    }
    r.s = block_sum_d((a0 + a1) + (a2 + a3));
  } else {
    float m0 = -FLT_MAX;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += kSampleThreads) m0 = fmaxf(m0, l[i]);
    r.m = block_max(m0);
    double a0 = 0.0;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += kSampleThreads) a0 += soft_term(l[i], r.m, T);
    r.s = block_sum_d(a0);
  }
  return r;
}

// Row maximum M (the chunk maxima in chunk order) and kept = sum over chunks of s_c * exp(double(m_c - M) / T), in
// chunk order: exp((l - M) / T) = exp((l - m_c) / T) * exp((m_c - M) / T), so kept is the whole row's softmax
// denominator with one extra rounding per chunk.  n chunks at cm / cs (stride 1).
__device__ __forceinline__ void combine_chunks(const float* cm, const double* cs, uint32_t n, float T, float* M_out,
                                               double* kept_out) {
  float M = -FLT_MAX;
  for (uint32_t k = 0; k < n; ++k) M = fmaxf(M, __ldcg(cm + k));
  double kept = 0.0;
  for (uint32_t k = 0; k < n; ++k) kept += __ldcg(cs + k) * soft_term(__ldcg(cm + k), M, T);
  *M_out = M;
  *kept_out = kept;
}

// Row statistics in one pass over the logits: per chunk (m_c, s_c), then the row's last CTA combines them.
__global__ void __launch_bounds__(kSampleThreads) stats_kernel(const float* __restrict__ logits, uint32_t V,
                                                               uint32_t off, float T, const RoundCtl* __restrict__ ctl,
                                                               float* __restrict__ cmax, double* __restrict__ csum,
                                                               float* __restrict__ mx, double* __restrict__ kept,
                                                               int* __restrict__ cnt) {
  griddep_wait();
  griddep_launch();
  T = read_temperature(T, ctl);
  const uint32_t c = blockIdx.x, C = gridDim.x;
  const uint32_t r = blockIdx.y + off;  // statistics row
  const ChunkStats cs = chunk_stats(logits + (size_t)blockIdx.y * V, V, c, T);
  if (threadIdx.x == 0) {
    cmax[(size_t)r * C + c] = cs.m;
    csum[(size_t)r * C + c] = cs.s;
  }
  if (!last_of(&cnt[r], (int)C)) return;
  if (threadIdx.x == 0) combine_chunks(cmax + (size_t)r * C, csum + (size_t)r * C, C, T, &mx[r], &kept[r]);
}

// Vocab shard statistics: the chunk statistics of the rows of a shard (entries [first, first + Vs) of each row, first
// a multiple of kStatsChunk), without the combine: om[r][c], os[r][c] for the shard's chunks.
__global__ void __launch_bounds__(kSampleThreads) shard_chunk_stats_kernel(const float* __restrict__ logits,
                                                                           uint32_t Vs, float T, float* __restrict__ om,
                                                                           double* __restrict__ os) {
  griddep_wait();
  griddep_launch();
  const uint32_t c = blockIdx.x, C = gridDim.x;
  const ChunkStats cs = chunk_stats(logits + (size_t)blockIdx.y * Vs, Vs, c, T);
  if (threadIdx.x == 0) {
    om[(size_t)blockIdx.y * C + c] = cs.m;
    os[(size_t)blockIdx.y * C + c] = cs.s;
  }
}

// The whole rows' (max, kept) from the ranks' gathered chunk statistics gm / gs [world][rows][cmax] (rank w holds
// counts.n[w] chunks of each row), combined in column order exactly as combine_chunks does for a whole row.
struct ShardCounts {
  uint32_t n[64];
};
__global__ void shard_combine_kernel(const float* __restrict__ gm, const double* __restrict__ gs, ShardCounts counts,
                                     uint32_t world, uint32_t rows, uint32_t cmax, float T, float* __restrict__ mx,
                                     double* __restrict__ kept) {
  griddep_wait();
  griddep_launch();
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float M = -FLT_MAX;
  for (uint32_t w = 0; w < world; ++w)
    for (uint32_t k = 0; k < counts.n[w]; ++k) M = fmaxf(M, gm[((size_t)w * rows + r) * cmax + k]);
  double a = 0.0;
  for (uint32_t w = 0; w < world; ++w)
    for (uint32_t k = 0; k < counts.n[w]; ++k) {
      const size_t i = ((size_t)w * rows + r) * cmax + k;
      a += gs[i] * soft_term(gm[i], M, T);
    }
  mx[r] = M;
  kept[r] = a;
}

__global__ void __launch_bounds__(kSampleThreads) probs_kernel(const float* __restrict__ logits, uint32_t V, float T,
                                                               const RoundCtl* __restrict__ ctl,
                                                               const float* __restrict__ mx,
                                                               const double* __restrict__ kept,
                                                               float* __restrict__ probs) {
  griddep_wait();
  griddep_launch();
  T = read_temperature(T, ctl);
  const uint32_t c = blockIdx.x, r = blockIdx.y;
  const float* l = logits + (size_t)r * V;
  float* o = probs + (size_t)r * V;
  const float m = mx[r];
  const double k = kept[r], inv = 1.0 / k;
  const uint32_t lo = c * kSampleChunk, hi = min(V, lo + kSampleChunk);
  for (uint32_t i = lo + threadIdx.x; i < hi; i += kSampleThreads) o[i] = prob_of(soft_term(l[i], m, T), k, inv);
}

__global__ void onehot_kernel(const int32_t* __restrict__ idx, uint32_t vocab, float* __restrict__ probs) {
  const size_t row = blockIdx.y;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    probs[row * vocab + i] = (int32_t)i == idx[row] ? 1.0f : 0.0f;
}

// ---------------------------------------------------------------------------------------------------
// exact sample_from over chunks
// ---------------------------------------------------------------------------------------------------
// What sequence b samples from.  Plain jobs: row P + b*row_stride.  Acceptance jobs (sel[b] = j written by
// accept_decide_kernel): j == k -> the bonus row P[b][k]; else the residual float(max(0, P[b][j] - Q[b][j]))
// (Q one-hot at the draft when Q is null), or P[b][j] when no residual is positive (sampling.cpp:117-126).
struct SampleJob {
  // target rows P [seq][k+1][V] and draft rows Q [seq][k][V]: materialised probabilities, or (P / Q null) logits
  // LP / LQ whose statistics (launch_row_stats) are at scratch rows 0.. and qoff..; no Q and no LQ: one-hot drafts
  const float* P = nullptr;
  const float* Q = nullptr;
  const float* LP = nullptr;
  const float* LQ = nullptr;
  const float* mx = nullptr;
  const double* kept = nullptr;
  uint32_t qoff = 0;
  float T = 1.0f;  // logits-mode temperature (ctl's when given)
  const int32_t* drafts = nullptr;
  uint64_t row_stride = 0;  // plain jobs
  uint32_t k = 0;
  bool accept = false;
  const int32_t* sel = nullptr;
  // the uniform of sequence b: uniforms[b] (or u_dev[b]) else Philox(seed, draw, stream, *d_counter) under ctl's seed
  const double* uniforms = nullptr;
  uint64_t seed = 0;
  uint32_t draw = 0, stream = 0;
  const unsigned long long* d_counter = nullptr;
  const RoundCtl* ctl = nullptr;
};

// One probability row: materialised (p), or distribution(logits row, T) evaluated per entry from the row's
// (max, kept) exactly as probs_kernel writes it.
struct ProbRow {
  const float* p = nullptr;
  const float* l = nullptr;
  float m = 0.0f;
  double kept = 1.0;
  float T = 1.0f;
  double inv = 1.0;  // 1 / kept
  __device__ __forceinline__ float operator()(uint32_t i) const {
    return p ? p[i] : prob_of(soft_term(l[i], m, T), kept, inv);
  }
};

struct RowFx {
  ProbRow P;
  ProbRow Q;  // residual against Q, or one-hot at d when hasQ is false and residual is set
  bool hasQ;
  int32_t d;
  bool residual;
  __device__ __forceinline__ double q_at(uint32_t i) const { return hasQ ? (double)Q(i) : ((int32_t)i == d ? 1.0 : 0.0); }
  __device__ float operator()(uint32_t i) const {
    if (!residual) return P(i);
    const double r = (double)P(i) - q_at(i);
    return (float)(r > 0.0 ? r : 0.0);
  }
};

__device__ __forceinline__ float job_temperature(const SampleJob& job) { return job.ctl ? job.ctl->temperature : job.T; }

// Target row `row` ([seq][k+1] numbering) and draft row `row` ([seq][k]) of an acceptance job.
__device__ __forceinline__ ProbRow target_row(const SampleJob& job, size_t row, uint32_t V, float T) {
  if (job.P) return ProbRow{job.P + row * V};
  return ProbRow{nullptr, job.LP + row * V, job.mx[row], job.kept[row], T, 1.0 / job.kept[row]};
}
__device__ __forceinline__ ProbRow draft_row(const SampleJob& job, size_t row, uint32_t V, float T) {
  if (job.Q) return ProbRow{job.Q + row * V};
  if (job.LQ) {
    const double kq = job.kept[job.qoff + row];
    return ProbRow{nullptr, job.LQ + row * V, job.mx[job.qoff + row], kq, T, 1.0 / kq};
  }
  return ProbRow{};
}

// fx of sequence b: variant 0 = main (bonus / residual / plain row), 1 = fallback P[b][j] (acceptance, j < k)
__device__ __forceinline__ RowFx job_fx(const SampleJob& job, uint32_t b, uint32_t V, int variant, float T) {
  if (!job.accept) return RowFx{ProbRow{job.P + (size_t)b * job.row_stride}, ProbRow{}, false, 0, false};
  const uint32_t j = (uint32_t)job.sel[b];
  const ProbRow Pj = target_row(job, (size_t)b * (job.k + 1) + j, V, T);
  if (j >= job.k || variant == 1) return RowFx{Pj, ProbRow{}, false, 0, false};
  const bool hasQ = job.Q != nullptr || job.LQ != nullptr;
  return RowFx{Pj, hasQ ? draft_row(job, (size_t)b * job.k + j, V, T) : ProbRow{}, hasQ,
               job.drafts[(size_t)b * job.k + j], true};
}

__device__ __forceinline__ double job_uniform(const SampleJob& job, const double* u_dev, uint32_t b) {
  if (u_dev) return u_dev[b];
  if (job.uniforms) return job.uniforms[b];
  const uint64_t seed = job.ctl ? job.ctl->seed : job.seed;
  const unsigned long long c = job.d_counter ? *job.d_counter : 0ull;
  return philox_uniform(seed, job.draw, job.stream, (uint32_t)c, (uint32_t)(c >> 32));
}

// Per-chunk exact sums of fx over this thread's kPerThread contiguous entries.
template <typename F>
__device__ __forceinline__ void thread_sums(const F& fx, uint32_t lo, uint32_t hi, U192& sum, int32_t& last, bool& bad) {
  sum = u192_zero();
  last = -1;
  bad = false;
  for (uint32_t i = lo; i < hi; ++i) {
    const float x = fx(i);
    if (!fast_ok(x)) {
      bad = true;
      continue;
    }
    if (x > 0.0f) {
      u192_add(sum, u192_from_float(x));
      last = (int32_t)i;
    }
  }
}

__global__ void __launch_bounds__(kSampleThreads) sample_chunks_kernel(SampleJob job, uint32_t V,
                                                                       unsigned long long* __restrict__ c192,
                                                                       int32_t* __restrict__ clast,
                                                                       int* __restrict__ cflag, int* __restrict__ cnt,
                                                                       const double* __restrict__ u_dev,
                                                                       int32_t* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const uint32_t c = blockIdx.x, b = blockIdx.y, C = gridDim.x, tid = threadIdx.x;
  const uint32_t clo = c * kSampleChunk, chi = min(V, clo + kSampleChunk);
  const bool two = job.accept && (uint32_t)job.sel[b] < job.k;  // residual with a P fallback
  const float T = job_temperature(job);
  __shared__ int s_flags;
  if (tid == 0) s_flags = 0;
  __syncthreads();
  const uint32_t lo = min(chi, clo + tid * kPerThread), hi = min(chi, lo + kPerThread);
  // the main pass sums the main row only; the fallback P[b][j] of a residual is needed only when no entry of the
  // whole residual is positive, which the last CTA alone learns, so that CTA sums the fallback's chunks itself
  {
    const int variant = 0;
    const RowFx fx = job_fx(job, b, V, variant, T);
    U192 sum;
    int32_t last;
    bool bad;
    thread_sums(fx, lo, hi, sum, last, bad);
    // residual mass test of sampling.cpp:121-123 (some double residual > 0).  A residual is the difference of two
    // floats (or of a float and 1), so when positive it is at least 2^-149 and its float is positive too: with every
    // entry finite the test is "a positive entry was summed".  Non-finite entries take the double test itself.
    bool anypos = false;
    if (variant == 0 && two) {
      anypos = last >= 0;
      if (bad && !anypos)
        for (uint32_t i = lo; i < hi; ++i) anypos |= ((double)fx.P(i) - fx.q_at(i)) > 0.0;
    }
    U192 total;
    (void)block_exclusive_scan(sum, &total);
    int32_t lmax;
    (void)block_exclusive_max(last, &lmax);
    if (bad) atomicOr(&s_flags, variant == 0 ? 1 : 4);
    if (anypos) atomicOr(&s_flags, 2);
    __syncthreads();
    if (tid == 0) {
      unsigned long long* o = c192 + (((size_t)b * 2 + variant) * C + c) * 3;
      o[0] = total.w[0];
      o[1] = total.w[1];
      o[2] = total.w[2];
      clast[((size_t)b * 2 + variant) * C + c] = lmax;
    }
  }
  if (tid == 0) cflag[(size_t)b * C + c] = s_flags;
  if (!last_of(&cnt[b], (int)C)) return;

  // ---- last CTA of sequence b: pick the row variant, locate the chunk, then the entry ----
  __shared__ int s_variant, s_state, s_chunk, s_fl;
  __shared__ int32_t s_result, s_prev_nz;
  __shared__ U192 s_th_true, s_th_false, s_prefix;
  if (tid == 0) {
    int fl = 0;
    for (uint32_t k = 0; k < C; ++k) fl |= __ldcg(cflag + (size_t)b * C + k);
    s_fl = fl;
    s_variant = (two && !(fl & 2)) ? 1 : 0;
  }
  __syncthreads();
  if (s_variant == 1) {
    // the residual has no positive entry: the chunk sums of the fallback row, chunk after chunk
    const RowFx fx1 = job_fx(job, b, V, 1, T);
    for (uint32_t k = 0; k < C; ++k) {
      const uint32_t klo = k * kSampleChunk, khi = min(V, klo + kSampleChunk);
      const uint32_t lo1 = min(khi, klo + tid * kPerThread), hi1 = min(khi, lo1 + kPerThread);
      U192 sum;
      int32_t last;
      bool bad;
      thread_sums(fx1, lo1, hi1, sum, last, bad);
      U192 total;
      (void)block_exclusive_scan(sum, &total);
      int32_t lmax;
      (void)block_exclusive_max(last, &lmax);
      if (bad) atomicOr(&s_fl, 4);
      if (tid == 0) {
        unsigned long long* o = c192 + (((size_t)b * 2 + 1) * C + k) * 3;
        o[0] = total.w[0];
        o[1] = total.w[1];
        o[2] = total.w[2];
        clast[((size_t)b * 2 + 1) * C + k] = lmax;
        __threadfence();  // read back below through L2 (__ldcg) by other threads of the CTA
      }
    }
  }
  __syncthreads();
  if (tid == 0) s_state = (s_fl & (s_variant == 0 ? 1 : 4)) ? 2 : 0;  // a non-finite or huge value: serial walk
  __syncthreads();
  const int variant = s_variant;
  const RowFx fx = job_fx(job, b, V, variant, T);
  const double u = job_uniform(job, u_dev, b);
  // chunk prefix sums (C <= kSampleThreads chunks per row)
  U192 csum = u192_zero();
  int32_t cl = -1;
  if (tid < C) {
    const unsigned long long* o = c192 + (((size_t)b * 2 + variant) * C + tid) * 3;
    csum.w[0] = __ldcg(o);
    csum.w[1] = __ldcg(o + 1);
    csum.w[2] = __ldcg(o + 2);
    cl = __ldcg(clast + ((size_t)b * 2 + variant) * C + tid);
  }
  U192 total;
  const U192 cprefix = block_exclusive_scan(csum, &total);
  int32_t overall_last;
  const int32_t cprev = block_exclusive_max(cl, &overall_last);
  if (tid == 0 && s_state == 0) {
    if (overall_last < 0) {
      s_result = 0;
      s_state = 1;
    } else {
      const double S = u192_to_double(total);
      const double g = ((double)V + 8.0) * 0x1.0p-52 + 16.0 * 0x1.0p-53;
      const double r_lo = u * S * (1.0 - g), r_hi = u * S * (1.0 + g);
      bool ok = u192_from_double(r_hi * (1.0 + 2.0 * g), true, &s_th_true);
      ok = ok && u192_from_double(r_lo * (1.0 - 2.0 * g), false, &s_th_false);
      if (!ok) {
        s_state = 2;
      } else if (!u192_gt(total, s_th_true)) {
        // no certainly-true index: answer the last nonzero if every prefix is certainly false
        if (!u192_gt(total, s_th_false)) {
          s_result = overall_last;
          s_state = 1;
        } else {
          s_state = 2;
        }
      }
    }
  }
  __syncthreads();
  if (s_state == 0 && tid < C) {
    U192 end = cprefix;
    u192_add(end, csum);
    if (!u192_gt(cprefix, s_th_true) && u192_gt(end, s_th_true)) {
      s_chunk = (int)tid;
      s_prefix = cprefix;
      s_prev_nz = cprev;
    }
  }
  __syncthreads();
  const int state = s_state;  // every thread branches on the same value
  __syncthreads();
  if (state == 0) {
    // entry level inside the crossing chunk
    const uint32_t xlo = (uint32_t)s_chunk * kSampleChunk, xhi = min(V, xlo + kSampleChunk);
    const uint32_t lo2 = min(xhi, xlo + tid * kPerThread), hi2 = min(xhi, lo2 + kPerThread);
    U192 sum;
    int32_t last;
    bool bad;
    thread_sums(fx, lo2, hi2, sum, last, bad);
    U192 ctot;
    U192 prefix = block_exclusive_scan(sum, &ctot);
    u192_add(prefix, s_prefix);
    int32_t lm;
    int32_t prev = block_exclusive_max(last, &lm);
    if (prev < 0) prev = s_prev_nz;
    U192 end = prefix;
    u192_add(end, sum);
    if (!u192_gt(prefix, s_th_true) && u192_gt(end, s_th_true)) {
      U192 run = prefix;
      int32_t prev_nz = prev;
      U192 prev_prefix = prefix;
      for (uint32_t i = lo2; i < hi2; ++i) {
        const float x = fx(i);
        if (!(x > 0.0f)) continue;
        u192_add(run, u192_from_float(x));
        if (u192_gt(run, s_th_true)) {
          const bool prev_false = prev_nz < 0 || !u192_gt(prev_prefix, s_th_false);
          s_result = (int32_t)i;
          s_state = prev_false ? 1 : 2;
          break;
        }
        prev_nz = (int32_t)i;
        prev_prefix = run;
      }
    }
    __syncthreads();
  }
  if (tid == 0) out[b] = s_state == 1 ? s_result : serial_sample(fx, V, u);
}

// ---------------------------------------------------------------------------------------------------
// speculative acceptance decisions (sampling.cpp:103-116): one thread per sequence
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ double draw_uniform(const double* uniforms, uint64_t seed, uint64_t counter_base,
                                               uint32_t seq, uint32_t k, uint32_t n) {
  // Philox counter (draw, sequence, counter_base lo, counter_base hi) under key `seed`.
  if (uniforms) return uniforms[(size_t)seq * (k + 1) + n];
  return philox_uniform(seed, n, seq, (uint32_t)counter_base, (uint32_t)(counter_base >> 32));
}

__global__ void accept_decide_kernel(SampleJob job, uint32_t batch, uint32_t V, const double* __restrict__ uniforms,
                                     uint64_t seed, uint64_t counter_base, int32_t* __restrict__ sel,
                                     double* __restrict__ u_out, uint32_t* __restrict__ accepted) {
  griddep_wait();
  griddep_launch();
  const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const uint32_t k = job.k;
  if (job.d_counter) counter_base = *job.d_counter;
  if (job.ctl) seed = job.ctl->seed;
  const float T = job_temperature(job);
  const bool hasQ = job.Q != nullptr || job.LQ != nullptr;
  const int32_t* d = job.drafts + (size_t)b * k;
  uint32_t used = 0, j = 0;
  for (; j < k; ++j) {
    const uint32_t dj = (uint32_t)d[j];
    const double p = dj < V ? (double)target_row(job, (size_t)b * (k + 1) + j, V, T)(dj) : 0.0;
    const double q = hasQ ? (dj < V ? (double)draft_row(job, (size_t)b * k + j, V, T)(dj) : 0.0) : 1.0;
    if (q > 0.0) {
      const double ratio = p / q;
      const double lim = ratio < 1.0 ? ratio : 1.0;
      if (draw_uniform(uniforms, seed, counter_base, b, k, used++) < lim) continue;
    }
    break;
  }
  sel[b] = (int32_t)j;
  accepted[b] = j;
  u_out[b] = draw_uniform(uniforms, seed, counter_base, b, k, used);
}

__global__ void philox_uniforms_kernel(uint64_t seed, uint64_t first, uint32_t c2, uint32_t c3, uint64_t n,
                                       double* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t c = first + i;
    out[i] = philox_uniform(seed, (uint32_t)c, (uint32_t)(c >> 32), c2, c3);
  }
}

// ---------------------------------------------------------------------------------------------------
// distribution() with top-k / top-p (sampling.cpp:51-86) exactly as the reference orders it: the sum of e in
// index order, a stable descending sort of e, the top-p cumulative and the kept sum in sorted order.  One CTA per
// row; the sort is a stable LSD radix sort on 4-bit digits of ~bits(e) (descending e, ties by ascending index).
// ---------------------------------------------------------------------------------------------------
constexpr int kTruncThreads = 512;

// Block-wide exclusive sum of one uint32 per thread.
__device__ uint32_t block_exclusive_sum_u32(uint32_t v) {
  __shared__ uint32_t ws[32];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  uint32_t inc = v;
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += o;
  }
  if (lane == 31) ws[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nw ? ws[lane] : 0u;
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t o = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += o;
    }
    if (lane < nw) ws[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  const uint32_t r = (warp > 0 ? ws[warp - 1] : 0u) + inc - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kTruncThreads) truncated_distribution_kernel(
    const float* __restrict__ logits, uint32_t V, float T, uint32_t top_k, float top_p, double* __restrict__ e_all,
    unsigned long long* __restrict__ key_a, unsigned long long* __restrict__ key_b, uint32_t* __restrict__ idx_a,
    uint32_t* __restrict__ idx_b, float* __restrict__ probs) {
  __shared__ uint32_t cnt[16][kTruncThreads];  // per-thread digit counts, then scatter offsets
  __shared__ uint32_t s_keep;
  __shared__ double s_sum, s_kept;
  const uint32_t row = blockIdx.x, tid = threadIdx.x;
  const float* l = logits + (size_t)row * V;
  double* e = e_all + (size_t)row * V;
  unsigned long long* ka = key_a + (size_t)row * V;
  unsigned long long* kb = key_b + (size_t)row * V;
  uint32_t* ia = idx_a + (size_t)row * V;
  uint32_t* ib = idx_b + (size_t)row * V;
  float* out = probs + (size_t)row * V;
  // max (std::max_element: NaNs never win unless first; finite logits expected)
  float m = -FLT_MAX;
  for (uint32_t i = tid; i < V; i += kTruncThreads) m = fmaxf(m, l[i]);
  m = block_max(m);
  for (uint32_t i = tid; i < V; i += kTruncThreads) {
    const double v = soft_term(l[i], m, T);
    e[i] = v;
    ka[i] = ~(unsigned long long)__double_as_longlong(v);  // ascending ~bits = descending e (e >= 0)
    ia[i] = i;
    out[i] = 0.0f;
  }
  __syncthreads();
  if (tid == 0) {
    double sum = 0.0;
    for (uint32_t i = 0; i < V; ++i) sum += e[i];
    s_sum = sum;
  }
  // stable LSD radix sort: each thread owns a contiguous chunk, so equal digits keep their order
  const uint32_t chunk = (V + kTruncThreads - 1) / kTruncThreads;
  const uint32_t c0 = min(V, tid * chunk), c1 = min(V, c0 + chunk);
  for (int pass = 0; pass < 16; ++pass) {
    const int shift = 4 * pass;
    for (int d = 0; d < 16; ++d) cnt[d][tid] = 0;
    for (uint32_t i = c0; i < c1; ++i) ++cnt[(ka[i] >> shift) & 15][tid];
    __syncthreads();
    {  // exclusive scan in (digit, thread) order: thread t scans linear entries [16t, 16t + 16)
      uint32_t* lin = &cnt[0][0];
      uint32_t local = 0;
      for (int j = 0; j < 16; ++j) local += lin[16 * tid + j];
      const uint32_t before = block_exclusive_sum_u32(local);
      uint32_t run = before;
      for (int j = 0; j < 16; ++j) {
        const uint32_t c = lin[16 * tid + j];
        lin[16 * tid + j] = run;
        run += c;
      }
    }
    __syncthreads();
    for (uint32_t i = c0; i < c1; ++i) {
      const unsigned long long k = ka[i];
      const uint32_t dst = cnt[(k >> shift) & 15][tid]++;
      kb[dst] = k;
      ib[dst] = ia[i];
    }
    __syncthreads();
    unsigned long long* tk = ka;
    ka = kb;
    kb = tk;
    uint32_t* ti = ia;
    ia = ib;
    ib = ti;
  }
  // ia is the stable descending order
  if (tid == 0) {
    uint32_t keep = V;
    if (top_k > 0 && top_k < keep) keep = top_k;
    if (top_p < 1.0f) {
      double acc = 0.0;
      for (uint32_t i = 0; i < keep; ++i) {
        acc += e[ia[i]] / s_sum;
        if (acc >= (double)top_p) {
          keep = i + 1;
          break;
        }
      }
    }
    double kept = 0.0;
    for (uint32_t i = 0; i < keep; ++i) kept += e[ia[i]];
    s_keep = keep;
    s_kept = kept;
  }
  __syncthreads();
  for (uint32_t i = tid; i < s_keep; i += kTruncThreads) out[ia[i]] = (float)(e[ia[i]] / s_kept);
}

// ---------------------------------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------------------------------
int launch_argmax_rows(const float* d_logits, uint32_t rows, uint32_t V, int32_t* d_out, const SampleScratch& s,
                       cudaStream_t st) {
  if (rows == 0) return CLM_OK;
  CLM_CHECK(rows <= s.rows, CLM_INTERNAL, "sampling scratch too small");
  return launch_pdl(argmax_chunks_kernel, dim3(sample_chunks(V), rows), dim3(kSampleThreads), 0, st, d_logits, V,
                    s.cval, s.cidx, s.rcnt, d_out);
}

int launch_row_stats(const float* d_logits, uint32_t rows, uint32_t V, float T, const RoundCtl* ctl, uint32_t off,
                     const SampleScratch& s, cudaStream_t st) {
  if (rows == 0) return CLM_OK;
  CLM_CHECK(off + rows <= s.rows, CLM_INTERNAL, "sampling scratch too small");
  const dim3 grid(stats_chunks(V), rows);
  return launch_pdl(stats_kernel, grid, dim3(kSampleThreads), 0, st, d_logits, V, off, T, ctl, s.cmax, s.csum, s.mx,
                    s.kept, s.rcnt);
}

int launch_probs(const float* d_logits, uint32_t rows, uint32_t V, float T, const RoundCtl* ctl, float* d_probs,
                 const SampleScratch& s, cudaStream_t st) {
  if (rows == 0) return CLM_OK;
  CLM_TRY(launch_row_stats(d_logits, rows, V, T, ctl, 0, s, st));
  const dim3 grid(sample_chunks(V), rows);
  return launch_pdl(probs_kernel, grid, dim3(kSampleThreads), 0, st, d_logits, V, T, ctl, (const float*)s.mx,
                    (const double*)s.kept, d_probs);
}

static int launch_sample_job(const SampleJob& job, uint32_t seqs, uint32_t V, const double* u_dev, int32_t* d_out,
                             const SampleScratch& s, cudaStream_t st) {
  CLM_CHECK(seqs <= s.seqs, CLM_INTERNAL, "sampling scratch too small");
  CLM_CHECK(sample_chunks(V) <= (uint32_t)kSampleThreads, CLM_OUT_OF_RANGE, "vocabulary too large for sampling");
  return launch_pdl(sample_chunks_kernel, dim3(sample_chunks(V), seqs), dim3(kSampleThreads), 0, st, job, V, s.c192,
                    s.clast, s.cflag, s.scnt, u_dev, d_out);
}

int launch_sample_rows(const float* d_probs, uint32_t rows, uint64_t row_stride, uint32_t V, const double* d_uniforms,
                       uint64_t seed, uint32_t draw, uint32_t stream_id, const unsigned long long* d_counter,
                       const RoundCtl* ctl, int32_t* d_out, const SampleScratch& s, cudaStream_t st) {
  if (rows == 0) return CLM_OK;
  SampleJob job;
  job.P = d_probs;
  job.row_stride = row_stride;
  job.uniforms = d_uniforms;
  job.seed = seed;
  job.draw = draw;
  job.stream = stream_id;
  job.d_counter = d_counter;
  job.ctl = ctl;
  return launch_sample_job(job, rows, V, nullptr, d_out, s, st);
}

int launch_accept(const AcceptRows& rows, const int32_t* d_drafts, uint32_t batch, uint32_t k, uint32_t V,
                  const double* d_uniforms, uint64_t seed, uint64_t counter_base,
                  const unsigned long long* d_counter, const RoundCtl* ctl, uint32_t* d_accepted, int32_t* d_next,
                  const SampleScratch& s, cudaStream_t st) {
  if (batch == 0) return CLM_OK;
  CLM_CHECK(batch <= s.seqs, CLM_INTERNAL, "sampling scratch too small");
  CLM_CHECK((rows.P != nullptr) != (rows.LP != nullptr), CLM_INTERNAL, "acceptance needs one target row source");
  SampleJob job;
  job.P = rows.P;
  job.Q = rows.Q;
  job.LP = rows.LP;
  job.LQ = rows.Q ? nullptr : rows.LQ;
  job.mx = s.mx;
  job.kept = s.kept;
  job.qoff = rows.q_stats_off;
  job.T = rows.T;
  job.ctl = ctl;
  job.d_counter = d_counter;
  job.drafts = d_drafts;
  job.k = k;
  job.accept = true;
  job.sel = s.sel;
  CLM_TRY(launch_pdl(accept_decide_kernel, dim3((batch + 127) / 128), dim3(128), 0, st, job, batch, V, d_uniforms,
                     seed, counter_base, s.sel, s.u, d_accepted));
  job.d_counter = nullptr;  // the sample kernel takes the uniforms accept_decide_kernel stored
  return launch_sample_job(job, batch, V, s.u, d_next, s, st);
}


// One stochastic draft step: probs = distribution(logits, T, top_k, top_p) for T > 0 (with top-k / top-p the exact
// reference truncation order, scratch from the context), then out = sample_from(probs, *d_u).
int launch_draft_sample(clm_b200_ctx* ctx, const float* d_logits, uint32_t V, float T, uint32_t top_k, float top_p,
                        const double* d_u, float* d_probs, int32_t* d_out, const SampleScratch& s, cudaStream_t st) {
  if (top_k > 0 || top_p < 1.0f) {
    void* scr = nullptr;
    const size_t n = V;
    CLM_TRY(ctx_scratch(ctx, n * (8 + 8 + 8 + 4 + 4) + 1024, &scr));
    double* e = static_cast<double*>(scr);
    unsigned long long* ka = reinterpret_cast<unsigned long long*>(e + n);
    unsigned long long* kb = ka + n;
    uint32_t* ia = reinterpret_cast<uint32_t*>(kb + n);
    uint32_t* ib = ia + n;
    truncated_distribution_kernel<<<1, kTruncThreads, 0, st>>>(d_logits, V, T, top_k, top_p, e, ka, kb, ia, ib,
                                                               d_probs);
    CLM_LAUNCHED("truncated_distribution_kernel");
  } else {
    CLM_TRY(launch_probs(d_logits, 1, V, T, nullptr, d_probs, s, st));
  }
  return launch_sample_rows(d_probs, 1, V, V, d_u, 0, 0, 0, nullptr, nullptr, d_out, s, st);
}

}  // namespace clm

using namespace clm;

namespace {

// Scratch for a C-ABI call from the context's scratch buffer, counters zeroed on the call's stream.
int abi_scratch(clm_b200_ctx* ctx, uint32_t rows, uint32_t seqs, uint32_t V, size_t extra, cudaStream_t st,
                SampleScratch* out, void** extra_ptr) {
  const size_t sb = SampleScratch::bytes(rows, seqs, V);
  void* base = nullptr;
  CLM_TRY(ctx_scratch(ctx, sb + extra + 256, &base));
  *out = SampleScratch::carve(base, rows, seqs, V);
  CLM_CUDA(cudaMemsetAsync(base, 0, out->counter_bytes, st));
  if (extra_ptr) *extra_ptr = static_cast<uint8_t*>(base) + ((sb + 255) & ~size_t{255});
  return CLM_OK;
}

}  // namespace

extern "C" {

int clm_b200_argmax_rows(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab, int32_t* d_out,
                         void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_logits && d_out, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  SampleScratch s;
  CLM_TRY(abi_scratch(ctx, rows, 0, vocab, 0, st, &s, nullptr));
  return launch_argmax_rows(d_logits, rows, vocab, d_out, s, st);
}

int clm_b200_distribution_rows(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab,
                               float temperature, uint32_t top_k, float top_p, float* d_probs, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_logits && d_probs, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  if (temperature <= 0.0f) {
    SampleScratch s;
    void* idx = nullptr;
    CLM_TRY(abi_scratch(ctx, rows, 0, vocab, (size_t)rows * 4, st, &s, &idx));
    CLM_TRY(launch_argmax_rows(d_logits, rows, vocab, static_cast<int32_t*>(idx), s, st));
    const unsigned gx = (unsigned)std::min<uint64_t>(ceil_div(vocab, 256), 64);
    onehot_kernel<<<dim3(gx, rows), 256, 0, st>>>(static_cast<const int32_t*>(idx), vocab, d_probs);
    CLM_LAUNCHED("onehot_kernel");
    return CLM_OK;
  }
  if (top_k > 0 || top_p < 1.0f) {
    // exact reference ordering (sort + serial sums): one CTA per row, scratch 28 bytes per entry
    void* scr = nullptr;
    const size_t n = (size_t)rows * vocab;
    CLM_TRY(ctx_scratch(ctx, n * (8 + 8 + 8 + 4 + 4) + 1024, &scr));
    double* e = static_cast<double*>(scr);
    unsigned long long* ka = reinterpret_cast<unsigned long long*>(e + n);
    unsigned long long* kb = ka + n;
    uint32_t* ia = reinterpret_cast<uint32_t*>(kb + n);
    uint32_t* ib = ia + n;
    truncated_distribution_kernel<<<rows, kTruncThreads, 0, st>>>(d_logits, vocab, temperature, top_k, top_p, e, ka,
                                                                   kb, ia, ib, d_probs);
    CLM_LAUNCHED("truncated_distribution_kernel");
    return CLM_OK;
  }
  SampleScratch s;
  CLM_TRY(abi_scratch(ctx, rows, 0, vocab, 0, st, &s, nullptr));
  return launch_probs(d_logits, rows, vocab, temperature, nullptr, d_probs, s, st);
}

int clm_b200_sample_rows(clm_b200_ctx* ctx, const float* d_probs, uint32_t rows, uint32_t vocab,
                         const double* d_uniforms, int32_t* d_out, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_probs && d_uniforms && d_out, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  SampleScratch s;
  CLM_TRY(abi_scratch(ctx, 0, rows, vocab, 0, st, &s, nullptr));
  return launch_sample_rows(d_probs, rows, vocab, vocab, d_uniforms, 0, 0, 0, nullptr, nullptr, d_out, s, st);
}

int clm_b200_verify_speculative(clm_b200_ctx* ctx, const float* d_target, const int32_t* d_drafts,
                                const float* d_draft_probs, uint32_t batch, uint32_t k, uint32_t vocab,
                                const double* d_uniforms, uint64_t seed, uint64_t counter_base, uint32_t* d_accepted,
                                int32_t* d_next, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (batch == 0) return CLM_OK;
  CLM_CHECK(d_target && (k == 0 || d_drafts) && d_accepted && d_next, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  SampleScratch s;
  CLM_TRY(abi_scratch(ctx, 0, batch, vocab, 0, st, &s, nullptr));
  AcceptRows src;
  src.P = d_target;
  src.Q = d_draft_probs;
  return launch_accept(src, d_drafts, batch, k, vocab, d_uniforms, seed, counter_base, nullptr, nullptr, d_accepted,
                       d_next, s, st);
}

int clm_b200_accept_logits(clm_b200_ctx* ctx, const float* d_tl, const float* d_dl, const int32_t* d_drafts,
                           uint32_t batch, uint32_t k, uint32_t vocab, float temperature, const double* d_uniforms,
                           uint64_t seed, uint64_t counter_base, uint32_t* d_accepted, int32_t* d_next, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  CLM_CHECK(temperature > 0.0f, CLM_INVALID_ARGUMENT, "fused acceptance needs temperature > 0");
  if (batch == 0) return CLM_OK;
  CLM_CHECK(d_tl && (k == 0 || d_drafts) && d_accepted && d_next, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  const uint32_t trows = batch * (k + 1), drows = d_dl ? batch * k : 0, rows = trows + drows;
  SampleScratch s;
  CLM_TRY(abi_scratch(ctx, rows, batch, vocab, 0, st, &s, nullptr));
  // row statistics only (target rows at 0.., draft rows at trows..); probabilities are evaluated where used
  CLM_TRY(launch_row_stats(d_tl, trows, vocab, temperature, nullptr, 0, s, st));
  if (drows) CLM_TRY(launch_row_stats(d_dl, drows, vocab, temperature, nullptr, trows, s, st));
  AcceptRows src;
  src.LP = d_tl;
  src.LQ = d_dl;
  src.q_stats_off = trows;
  src.T = temperature;
  return launch_accept(src, d_drafts, batch, k, vocab, d_uniforms, seed, counter_base, nullptr, nullptr, d_accepted,
                       d_next, s, st);
}

int clm_b200_shard_stats(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab_shard,
                         uint64_t first_col, float temperature, float* d_chunk_max, double* d_chunk_sum, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab_shard > 0 && temperature > 0.0f, CLM_INVALID_ARGUMENT, "empty shard or temperature <= 0");
  CLM_CHECK(first_col % kStatsChunk == 0, CLM_INVALID_ARGUMENT,
            "a vocab shard must start at a multiple of 16384 columns (the statistics chunk)");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_logits && d_chunk_max && d_chunk_sum, CLM_INVALID_ARGUMENT, "null buffer");
  return launch_pdl(shard_chunk_stats_kernel, dim3(stats_chunks(vocab_shard), rows), dim3(kSampleThreads), 0,
                    pick_stream(ctx, stream), d_logits, vocab_shard, temperature, d_chunk_max, d_chunk_sum);
}

int clm_b200_shard_combine(clm_b200_ctx* ctx, const float* d_chunk_max, const double* d_chunk_sum, uint32_t world,
                           const uint32_t* h_counts, uint32_t rows, uint32_t max_chunks, float temperature,
                           float* d_max, double* d_kept, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(world >= 1 && world <= 64 && h_counts != nullptr && temperature > 0.0f, CLM_INVALID_ARGUMENT,
            "1..64 shards with their chunk counts, temperature > 0");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_chunk_max && d_chunk_sum && d_max && d_kept, CLM_INVALID_ARGUMENT, "null buffer");
  ShardCounts c{};
  for (uint32_t w = 0; w < world; ++w) {
    CLM_CHECK(h_counts[w] <= max_chunks, CLM_INVALID_ARGUMENT, "a shard's chunk count exceeds max_chunks");
    c.n[w] = h_counts[w];
  }
  return launch_pdl(shard_combine_kernel, dim3((unsigned)ceil_div(rows, 128)), dim3(128), 0, pick_stream(ctx, stream),
                    d_chunk_max, d_chunk_sum, c, world, rows, max_chunks, temperature, d_max, d_kept);
}

int clm_b200_shard_probs(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab_shard,
                         float temperature, const float* d_global_max, const double* d_kept, float* d_probs,
                         void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab_shard > 0 && temperature > 0.0f, CLM_INVALID_ARGUMENT, "empty shard or temperature <= 0");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_logits && d_global_max && d_kept && d_probs, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  const dim3 grid(sample_chunks(vocab_shard), rows);
  return launch_pdl(probs_kernel, grid, dim3(kSampleThreads), 0, st, d_logits, vocab_shard, temperature,
                    (const RoundCtl*)nullptr, d_global_max, d_kept, d_probs);
}

int clm_b200_philox_uniforms(clm_b200_ctx* ctx, uint64_t seed, uint64_t first, uint32_t c2, uint32_t c3, uint64_t n,
                             double* d_out, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  if (n == 0) return CLM_OK;
  CLM_CHECK(d_out != nullptr, CLM_INVALID_ARGUMENT, "null output");
  const uint64_t blocks = std::min<uint64_t>(ceil_div(n, 256), 4096);
  philox_uniforms_kernel<<<(unsigned)blocks, 256, 0, pick_stream(ctx, stream)>>>(seed, first, c2, c3, n, d_out);
  CLM_LAUNCHED("philox_uniforms_kernel");
  return CLM_OK;
}

}  // extern "C"
