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
// multiple of 2^-149, so prefix sums are computed EXACTLY in 192-bit fixed point with a block scan.  The
// serial double sums differ from the exact ones by at most g*S (recursive summation bound, g ~ V*2^-53), and
// r likewise.  The index is taken from the exact prefixes only when that bound proves the serial comparisons
// give the same index; otherwise (probability ~V*g per draw) one thread re-walks the row serially.
#include <cfloat>

#include "common.cuh"
#include "pdl.cuh"
#include "sampling.cuh"

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

// Block-cooperative exact sample_from.  All threads must call; all threads get the result.
// *fell_back (optional) reports whether the serial walk was needed.
template <typename F>
__device__ int32_t exact_sample(const F& fx, uint32_t n, double u, bool* fell_back = nullptr) {
  __shared__ int32_t s_result;
  __shared__ int s_state;  // 0 undecided, 1 decided, 2 fallback
  __shared__ U192 s_th_true, s_th_false;
  const uint32_t nt = blockDim.x, tid = threadIdx.x;
  const uint32_t chunk = (n + nt - 1) / nt;
  const uint32_t c0 = min(n, tid * chunk), c1 = min(n, c0 + chunk);
  U192 sum = u192_zero();
  int32_t last_nz = -1;
  bool bad = false;
  for (uint32_t i = c0; i < c1; ++i) {
    const float x = fx(i);
    if (!fast_ok(x)) {
      bad = true;
      continue;
    }
    if (x > 0.0f) {
      u192_add(sum, u192_from_float(x));
      last_nz = (int32_t)i;
    }
  }
  if (tid == 0) s_state = 0;
  bad = __syncthreads_or(bad);
  U192 total;
  const U192 prefix = block_exclusive_scan(sum, &total);
  // last nonzero index strictly before this chunk (chunks are ordered, so a max-scan), and overall
  int32_t overall_last;
  const int32_t prev_before_chunk = block_exclusive_max(last_nz, &overall_last);
  if (bad) {
    if (tid == 0) {
      s_state = 2;
    }
  } else if (overall_last < 0) {
    if (tid == 0) {
      s_result = 0;
      s_state = 1;
    }
  } else if (tid == 0) {
    const double S = u192_to_double(total);
    const double g = ((double)n + 8.0) * 0x1.0p-52 + 16.0 * 0x1.0p-53;
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
  __syncthreads();
  if (s_state == 0) {
    // the chunk whose exact prefix crosses th_true holds the first certainly-true index
    U192 end = prefix;
    u192_add(end, sum);
    if (!u192_gt(prefix, s_th_true) && u192_gt(end, s_th_true)) {
      U192 run = prefix;
      int32_t prev_nz = prev_before_chunk;
      U192 prev_prefix = prefix;
      for (uint32_t i = c0; i < c1; ++i) {
        const float x = fx(i);
        if (!(x > 0.0f)) continue;
        u192_add(run, u192_from_float(x));
        if (u192_gt(run, s_th_true)) {
          const bool prev_false = prev_nz < 0 || !u192_gt(prev_prefix, s_th_false);
          if (prev_false) {
            s_result = (int32_t)i;
            s_state = 1;
          } else {
            s_state = 2;
          }
          break;
        }
        prev_nz = (int32_t)i;
        prev_prefix = run;
      }
    }
  }
  __syncthreads();
  if (s_state != 1) {
    if (tid == 0) s_result = serial_sample(fx, n, u);
    __syncthreads();
  }
  if (fell_back) *fell_back = s_state != 1;
  const int32_t r = s_result;
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------------------------------
// value providers
// ---------------------------------------------------------------------------------------------------
struct RowValues {
  const float* p;
  __device__ float operator()(uint32_t i) const { return p[i]; }
};

// float(max(0, double(P_i) - Q_i)), Q one-hot at d when q == nullptr (sampling.cpp:117-123)
struct ResidualArrays {
  const float* P;
  const float* Q;
  int32_t d;
  __device__ float operator()(uint32_t i) const {
    const double qi = Q ? (double)Q[i] : ((int32_t)i == d ? 1.0 : 0.0);
    const double r = (double)P[i] - qi;
    return (float)(r > 0.0 ? r : 0.0);
  }
};

// distribution() value of one logit row: float(exp(double(l - mx)/T) / kept)
__device__ __forceinline__ float dist_value(float l, float mx, double inv_t_div, double kept, float T) {
  (void)inv_t_div;
  const double e = exp((double)__fsub_rn(l, mx) / (double)T);
  return (float)(e / kept);
}

struct LogitRow {
  const float* l;
  float mx;
  double kept;
  float T;
  __device__ float operator()(uint32_t i) const { return dist_value(l[i], mx, 0.0, kept, T); }
};

struct ResidualLogits {
  LogitRow P;
  const float* ql;  // draft logits row or nullptr (one-hot)
  float qmx;
  double qkept;
  int32_t d;
  __device__ float operator()(uint32_t i) const {
    const double pi = (double)P(i);
    const double qi = ql ? (double)dist_value(ql[i], qmx, 0.0, qkept, P.T) : ((int32_t)i == d ? 1.0 : 0.0);
    const double r = pi - qi;
    return (float)(r > 0.0 ? r : 0.0);
  }
};

// ---------------------------------------------------------------------------------------------------
// block reductions
// ---------------------------------------------------------------------------------------------------
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

// ---------------------------------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------------------------------
// First index of the maximum of l[0..vocab); a NaN at index 0 pins the answer to 0 and NaNs elsewhere are never
// chosen (the reference's `logits[i] > logits[best]` scan).  All threads get the result.
__device__ int32_t block_argmax(const float* __restrict__ l, uint32_t vocab) {
  __shared__ float sv[32];
  __shared__ int32_t si[32];
  __shared__ int32_t s_res;
  float best = -INFINITY;
  int32_t bi = INT32_MAX;
  for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = l[i];
    if (v > best || (v == best && (int32_t)i < bi)) {
      best = v;
      bi = (int32_t)i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < (int)(blockDim.x / 32) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x / 32) ? si[lane] : INT32_MAX;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) s_res = (isnan(l[0]) || bi == INT32_MAX) ? 0 : bi;
  }
  __syncthreads();
  const int32_t r = s_res;
  __syncthreads();
  return r;
}

__global__ void argmax_rows_kernel(const float* __restrict__ logits, uint32_t vocab, int32_t* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int32_t r = block_argmax(logits + (size_t)blockIdx.x * vocab, vocab);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

// Row statistics for distribution(): max and kept = sum exp(double(l - max)/T).
__global__ void row_stats_kernel(const float* __restrict__ logits, uint32_t vocab, float T, float* __restrict__ mx_out,
                                 double* __restrict__ kept_out, const RoundCtl* __restrict__ ctl) {
  griddep_wait();
  griddep_launch();
  if (ctl) T = ctl->temperature;
  const float* l = logits + (size_t)blockIdx.x * vocab;
  float m = -FLT_MAX;
  for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) m = fmaxf(m, l[i]);
  m = block_max(m);
  double s = 0.0;
  for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) s += exp((double)__fsub_rn(l[i], m) / (double)T);
  s = block_sum_d(s);
  if (threadIdx.x == 0) {
    mx_out[blockIdx.x] = m;
    kept_out[blockIdx.x] = s;
  }
}

__global__ void distribution_kernel(const float* __restrict__ logits, uint32_t vocab, float T,
                                    const float* __restrict__ mx, const double* __restrict__ kept,
                                    float* __restrict__ probs) {
  const size_t row = blockIdx.y;
  const float* l = logits + row * vocab;
  float* o = probs + row * vocab;
  const float m = mx[row];
  const double k = kept[row];
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    o[i] = dist_value(l[i], m, 0.0, k, T);
}

__global__ void onehot_kernel(const int32_t* __restrict__ idx, uint32_t vocab, float* __restrict__ probs) {
  const size_t row = blockIdx.y;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    probs[row * vocab + i] = (int32_t)i == idx[row] ? 1.0f : 0.0f;
}

__global__ void __launch_bounds__(1024) sample_rows_kernel(const float* __restrict__ probs, uint32_t vocab,
                                                           const double* __restrict__ uniforms,
                                                           int32_t* __restrict__ out) {
  RowValues f{probs + (size_t)blockIdx.x * vocab};
  const int32_t r = exact_sample(f, vocab, uniforms[blockIdx.x]);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
}

__device__ __forceinline__ double draw_uniform(const double* uniforms, uint64_t seed, uint64_t counter_base,
                                               uint32_t seq, uint32_t k, uint32_t n) {
  // Philox counter (draw, sequence, counter_base lo, counter_base hi) under key `seed`.
  if (uniforms) return uniforms[(size_t)seq * (k + 1) + n];
  return philox_uniform(seed, n, seq, (uint32_t)counter_base, (uint32_t)(counter_base >> 32));
}

// One CTA per sequence: sequential acceptance tests, then a block-cooperative exact resample.
__global__ void __launch_bounds__(1024) verify_kernel(const float* __restrict__ target, const int32_t* __restrict__ drafts,
                                                      const float* __restrict__ draft_probs, uint32_t k, uint32_t vocab,
                                                      const double* __restrict__ uniforms, uint64_t seed,
                                                      uint64_t counter_base, uint32_t* __restrict__ accepted,
                                                      int32_t* __restrict__ next) {
  const uint32_t b = blockIdx.x;
  const float* T = target + (size_t)b * (k + 1) * vocab;
  const int32_t* d = drafts + (size_t)b * k;
  const float* Q = draft_probs ? draft_probs + (size_t)b * k * vocab : nullptr;
  __shared__ uint32_t s_j, s_used;
  if (threadIdx.x == 0) {
    uint32_t used = 0, j = 0;
    for (; j < k; ++j) {
      const uint32_t dj = (uint32_t)d[j];
      const double p = dj < vocab ? (double)T[(size_t)j * vocab + dj] : 0.0;
      const double q = Q ? (dj < vocab ? (double)Q[(size_t)j * vocab + dj] : 0.0) : 1.0;
      if (q > 0.0) {
        const double ratio = p / q;
        const double lim = ratio < 1.0 ? ratio : 1.0;
        if (draw_uniform(uniforms, seed, counter_base, b, k, used++) < lim) continue;
      }
      break;
    }
    s_j = j;
    s_used = used;
  }
  __syncthreads();
  const uint32_t j = s_j;
  const double u = draw_uniform(uniforms, seed, counter_base, b, k, s_used);
  int32_t tok;
  if (j == k) {
    tok = exact_sample(RowValues{T + (size_t)k * vocab}, vocab, u);
  } else {
    ResidualArrays res{T + (size_t)j * vocab, Q ? Q + (size_t)j * vocab : nullptr, d[j]};
    // mass > 0 iff some residual (in double) is positive
    bool any = false;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) {
      const double qi = res.Q ? (double)res.Q[i] : ((int32_t)i == res.d ? 1.0 : 0.0);
      any |= ((double)res.P[i] - qi) > 0.0;
    }
    any = __syncthreads_or(any);
    tok = any ? exact_sample(res, vocab, u) : exact_sample(RowValues{res.P}, vocab, u);
  }
  if (threadIdx.x == 0) {
    accepted[b] = j;
    next[b] = tok;
  }
}

// Fused acceptance from logits (row statistics precomputed by row_stats_kernel).
// Stats layout: target row j of sequence b at b*(k+1) + j; draft row j at batch*(k+1) + b*k + j.
__global__ void __launch_bounds__(1024) accept_logits_kernel(
    const float* __restrict__ tl, const float* __restrict__ dl, const int32_t* __restrict__ drafts, uint32_t k,
    uint32_t vocab, float T, const float* __restrict__ mx, const double* __restrict__ kept,
    const double* __restrict__ uniforms, uint64_t seed, uint64_t counter_base,
    const unsigned long long* __restrict__ d_counter, uint32_t* __restrict__ accepted, int32_t* __restrict__ next,
    const RoundCtl* __restrict__ ctl) {
  griddep_wait();
  griddep_launch();
  if (d_counter) counter_base = *d_counter;
  if (ctl) {
    T = ctl->temperature;
    seed = ctl->seed;
  }
  const uint32_t b = blockIdx.x;
  const float* tb = tl + (size_t)b * (k + 1) * vocab;
  const float* db = dl ? dl + (size_t)b * k * vocab : nullptr;
  const int32_t* d = drafts + (size_t)b * k;
  const float* smx = mx + (size_t)b * (k + 1);  // target row j: smx[j]
  const double* skept = kept + (size_t)b * (k + 1);
  const float* qmx = mx + (size_t)gridDim.x * (k + 1) + (size_t)b * k;  // draft row j: qmx[j]
  const double* qkept = kept + (size_t)gridDim.x * (k + 1) + (size_t)b * k;
  __shared__ uint32_t s_j, s_used;
  if (threadIdx.x == 0) {
    uint32_t used = 0, j = 0;
    for (; j < k; ++j) {
      const uint32_t dj = (uint32_t)d[j];
      const double p = dj < vocab ? (double)dist_value(tb[(size_t)j * vocab + dj], smx[j], 0.0, skept[j], T) : 0.0;
      const double q =
          db ? (dj < vocab ? (double)dist_value(db[(size_t)j * vocab + dj], qmx[j], 0.0, qkept[j], T) : 0.0) : 1.0;
      if (q > 0.0) {
        const double ratio = p / q;
        const double lim = ratio < 1.0 ? ratio : 1.0;
        if (draw_uniform(uniforms, seed, counter_base, b, k, used++) < lim) continue;
      }
      break;
    }
    s_j = j;
    s_used = used;
  }
  __syncthreads();
  const uint32_t j = s_j;
  const double u = draw_uniform(uniforms, seed, counter_base, b, k, s_used);
  int32_t tok;
  if (j == k) {
    tok = exact_sample(LogitRow{tb + (size_t)k * vocab, smx[k], skept[k], T}, vocab, u);
  } else {
    ResidualLogits res{LogitRow{tb + (size_t)j * vocab, smx[j], skept[j], T},
                       db ? db + (size_t)j * vocab : nullptr, db ? qmx[j] : 0.0f, db ? qkept[j] : 1.0, d[j]};
    bool any = false;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) {
      const double pi = (double)res.P(i);
      const double qi = res.ql ? (double)dist_value(res.ql[i], res.qmx, 0.0, res.qkept, T)
                               : ((int32_t)i == res.d ? 1.0 : 0.0);
      any |= (pi - qi) > 0.0;
    }
    any = __syncthreads_or(any);
    tok = any ? exact_sample(res, vocab, u) : exact_sample(res.P, vocab, u);
  }
  if (threadIdx.x == 0) {
    accepted[b] = j;
    next[b] = tok;
  }
}

__global__ void philox_uniforms_kernel(uint64_t seed, uint64_t first, uint32_t c2, uint32_t c3, uint64_t n,
                                       double* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t c = first + i;
    out[i] = philox_uniform(seed, (uint32_t)c, (uint32_t)(c >> 32), c2, c3);
  }
}

// ---------------------------------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------------------------------
int launch_argmax(const float* d_logits, uint32_t rows, uint32_t vocab, int32_t* d_out, cudaStream_t st) {
  if (rows == 0) return CLM_OK;
  return launch_pdl(argmax_rows_kernel, dim3(rows), dim3(1024), 0, st, d_logits, vocab, d_out);
}

int launch_row_stats(const float* d_logits, uint32_t rows, uint32_t vocab, float T, float* d_mx, double* d_kept,
                     cudaStream_t st, const RoundCtl* ctl) {
  if (rows == 0) return CLM_OK;
  return launch_pdl(row_stats_kernel, dim3(rows), dim3(512), 0, st, d_logits, vocab, T, d_mx, d_kept, ctl);
}

int launch_accept_logits(const float* d_tl, const float* d_dl, const int32_t* d_drafts, uint32_t batch, uint32_t k,
                         uint32_t vocab, float T, const float* d_mx, const double* d_kept, const double* d_uniforms,
                         uint64_t seed, uint64_t counter_base, const unsigned long long* d_counter,
                         uint32_t* d_accepted, int32_t* d_next, cudaStream_t st, const RoundCtl* ctl) {
  return launch_pdl(accept_logits_kernel, dim3(batch), dim3(1024), 0, st, d_tl, d_dl, d_drafts, k, vocab, T, d_mx,
                    d_kept, d_uniforms, seed, counter_base, d_counter, d_accepted, d_next, ctl);
}

// One row of logits -> one token: argmax (T <= 0) or sample_from(distribution(row, T)) with the Philox
// uniform (draw, stream, counter lo, counter hi), counter read from *d_counter.
__global__ void __launch_bounds__(1024) sample_logits_kernel(const float* __restrict__ logits, uint32_t vocab, float T,
                                                             uint64_t seed, uint32_t draw, uint32_t stream_id,
                                                             const unsigned long long* __restrict__ d_counter,
                                                             int32_t* __restrict__ out, const RoundCtl* __restrict__ ctl) {
  griddep_wait();
  griddep_launch();
  if (ctl) {
    T = ctl->temperature;
    seed = ctl->seed;
  }
  if (T <= 0.0f) {
    const int32_t r = block_argmax(logits, vocab);
    if (threadIdx.x == 0) *out = r;
    return;
  }
  float m = -FLT_MAX;
  for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) m = fmaxf(m, logits[i]);
  m = block_max(m);
  double s = 0.0;
  for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) s += exp((double)__fsub_rn(logits[i], m) / (double)T);
  s = block_sum_d(s);
  const unsigned long long c = d_counter ? *d_counter : 0ull;
  const double u = philox_uniform(seed, draw, stream_id, (uint32_t)c, (uint32_t)(c >> 32));
  const int32_t tok = exact_sample(LogitRow{logits, m, s, T}, vocab, u);
  if (threadIdx.x == 0) *out = tok;
}

int launch_sample_logits(const float* d_logits, uint32_t vocab, float T, uint64_t seed, uint32_t draw,
                         uint32_t stream_id, const unsigned long long* d_counter, int32_t* d_out, cudaStream_t st,
                         const RoundCtl* ctl) {
  return launch_pdl(sample_logits_kernel, dim3(1), dim3(1024), 0, st, d_logits, vocab, T, seed, draw, stream_id,
                    d_counter, d_out, ctl);
}

}  // namespace clm

using namespace clm;

extern "C" {

int clm_b200_argmax_rows(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab, int32_t* d_out,
                         void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  CLM_CHECK(rows == 0 || (d_logits && d_out), CLM_INVALID_ARGUMENT, "null buffer");
  return launch_argmax(d_logits, rows, vocab, d_out, pick_stream(ctx, stream));
}

int clm_b200_distribution_rows(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab,
                               float temperature, uint32_t top_k, float top_p, float* d_probs, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_logits && d_probs, CLM_INVALID_ARGUMENT, "null buffer");
  cudaStream_t st = pick_stream(ctx, stream);
  const unsigned gx = (unsigned)std::min<uint64_t>(ceil_div(vocab, 256), 64);
  if (temperature <= 0.0f) {
    void* scr = nullptr;
    CLM_TRY(ctx_scratch(ctx, (size_t)rows * 4, &scr));
    int32_t* idx = static_cast<int32_t*>(scr);
    CLM_TRY(launch_argmax(d_logits, rows, vocab, idx, st));
    onehot_kernel<<<dim3(gx, rows), 256, 0, st>>>(idx, vocab, d_probs);
    CLM_LAUNCHED("onehot_kernel");
    return CLM_OK;
  }
  CLM_CHECK(top_k == 0 && top_p >= 1.0f, CLM_UNIMPLEMENTED,
            "top-k / top-p truncation is not implemented on the device yet (temperature-only distributions)");
  void* scr = nullptr;
  CLM_TRY(ctx_scratch(ctx, (size_t)rows * 16, &scr));
  double* kept = static_cast<double*>(scr);
  float* mx = reinterpret_cast<float*>(kept + rows);
  CLM_TRY(launch_row_stats(d_logits, rows, vocab, temperature, mx, kept, st));
  distribution_kernel<<<dim3(gx, rows), 256, 0, st>>>(d_logits, vocab, temperature, mx, kept, d_probs);
  CLM_LAUNCHED("distribution_kernel");
  return CLM_OK;
}

int clm_b200_sample_rows(clm_b200_ctx* ctx, const float* d_probs, uint32_t rows, uint32_t vocab,
                         const double* d_uniforms, int32_t* d_out, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (rows == 0) return CLM_OK;
  CLM_CHECK(d_probs && d_uniforms && d_out, CLM_INVALID_ARGUMENT, "null buffer");
  sample_rows_kernel<<<rows, 1024, 0, pick_stream(ctx, stream)>>>(d_probs, vocab, d_uniforms, d_out);
  CLM_LAUNCHED("sample_rows_kernel");
  return CLM_OK;
}

int clm_b200_verify_speculative(clm_b200_ctx* ctx, const float* d_target, const int32_t* d_drafts,
                                const float* d_draft_probs, uint32_t batch, uint32_t k, uint32_t vocab,
                                const double* d_uniforms, uint64_t seed, uint64_t counter_base, uint32_t* d_accepted,
                                int32_t* d_next, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(vocab > 0, CLM_INVALID_ARGUMENT, "empty vocabulary");
  if (batch == 0) return CLM_OK;
  CLM_CHECK(d_target && (k == 0 || d_drafts) && d_accepted && d_next, CLM_INVALID_ARGUMENT, "null buffer");
  verify_kernel<<<batch, 1024, 0, pick_stream(ctx, stream)>>>(d_target, d_drafts, d_draft_probs, k, vocab, d_uniforms,
                                                              seed, counter_base, d_accepted, d_next);
  CLM_LAUNCHED("verify_kernel");
  return CLM_OK;
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
  void* scr = nullptr;
  CLM_TRY(ctx_scratch(ctx, (size_t)rows * 16, &scr));
  double* kept = static_cast<double*>(scr);
  float* mx = reinterpret_cast<float*>(kept + rows);
  CLM_TRY(launch_row_stats(d_tl, trows, vocab, temperature, mx, kept, st));
  if (drows) CLM_TRY(launch_row_stats(d_dl, drows, vocab, temperature, mx + trows, kept + trows, st));
  return launch_accept_logits(d_tl, d_dl, d_drafts, batch, k, vocab, temperature, mx, kept, d_uniforms, seed,
                              counter_base, nullptr, d_accepted, d_next, st);
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
