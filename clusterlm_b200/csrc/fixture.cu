// fixture.cu — the clusterlm-fixture family on the device: the reference's own fixture model
// (runtime/domain/src/reference_domain.cpp:452-585) as one CTA per stage window.
//
// The model is tiny (H = 64), so a window is latency-bound: one CTA holds every activation of the window in
// shared memory and walks the local layers.  The arithmetic reproduces the reference's order: every dot
// product is one thread's ascending loop, and this file is compiled with --fmad=false so no multiply-add is
// contracted (the reference builds with -ffp-contract=off, runtime/domain/CMakeLists.txt:9-14).  exp and
// tanh are evaluated in double and rounded to f32, which agrees with a correctly rounded libm in all but
// rare last-bit cases.
#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "codec.cuh"
#include "engine.cuh"
#include "pdl.cuh"
#include "sampling.cuh"

namespace clm {

struct FixLayerW {  // weights of one local layer (device pointers)
  int kind;         // 0 recurrent, 1 attention
  const float* dense;
  const float* shared;   // [gate sff*H][up sff*H][down H*sff] or null
  const float* experts;  // E x [gate ff*H][up ff*H][down H*ff]
};

struct FixLayerS {  // sequence state of one local layer for one session (device pointers)
  float* rec;   // committed recurrent state [H]
  float* snap;  // window snapshots [max_window][H]
  float* kc;    // [max_context][kvd]
  float* vc;
};

struct FixParams {
  int H, hc, E, K, ff, sff, nh, nkv, hd, V, ple_layer, ngram, ple_rows;
  int nlayers, layer_begin, max_context;
  int score_ld;  // max_context + 1: a row of attention scores plus the stashed softmax sum
  int q;
  long long base;
  int has_tokens, has_head;
  // dense layout offsets (fixture_model.cpp dense_layout): recurrent / attention
  int o_norm, o_win, o_decay, o_wout, o_router_r, o_inj_r;
  int o_wq, o_wk, o_wv, o_wo, o_router_a, o_inj_a;
};

__device__ __forceinline__ float fexp(float z) { return (float)exp((double)z); }
__device__ __forceinline__ float ftanh(float z) { return (float)tanh((double)z); }
__device__ __forceinline__ float fsilu(float z) { return z / (1.0f + fexp(-z)); }
__device__ __forceinline__ float fsigmoid(float z) { return 1.0f / (1.0f + fexp(-z)); }

// refmath::dot order (reference_math.hpp): acc += a[i] * b[i] for ascending i, each product and sum rounded
// (this file is built without contraction).  The operands (global or shared) are fetched 16 at a time ahead of
// the sums, so a row costs one memory latency per 16 elements instead of one per element; the arithmetic and its
// order are unchanged.
__device__ __forceinline__ float dotf(const float* a, const float* b, int n) {
  float acc = 0.0f;
  int i = 0;
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0) {
    for (; i + 16 <= n; i += 16) {
      float4 wa[4], wb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        wa[j] = reinterpret_cast<const float4*>(a + i)[j];
        wb[j] = reinterpret_cast<const float4*>(b + i)[j];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc += wa[j].x * wb[j].x;
        acc += wa[j].y * wb[j].y;
        acc += wa[j].z * wb[j].z;
        acc += wa[j].w * wb[j].w;
      }
    }
  }
  for (; i < n; ++i) acc += a[i] * b[i];
  return acc;
}

__device__ __forceinline__ uint64_t mix64d(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// One stage window.  `rec_io` holds the q boundary records (in: from the previous stage or zero + embedding;
// out: this stage's records).  scratch: [q][nh][max_context + 1] attention scores (+ softmax sum).
__global__ void __launch_bounds__(256) fixture_window_kernel(FixParams P, const FixLayerW* __restrict__ W,
                                                             const FixLayerS* __restrict__ S,
                                                             const float* __restrict__ embd,
                                                             const float* __restrict__ ple,
                                                             const float* __restrict__ head_norm,
                                                             const float* __restrict__ head_w,
                                                             const int32_t* __restrict__ tokens,
                                                             const int32_t* __restrict__ history,
                                                             float* __restrict__ rec_io, float* __restrict__ logits,
                                                             float* __restrict__ scores) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float sm[];
  const int H = P.H, hc = P.hc, q = P.q, tid = threadIdx.x, nt = blockDim.x;
  const int fpp = hc * H + H + hc;
  const int qd = P.nh * P.hd, kvd = P.nkv * P.hd, ffmax = max(P.ff, P.sff);
  float* rec = sm;                   // q * fpp
  float* x = rec + q * fpp;          // q * H
  float* u = x + q * H;              // q * H (mean / tanh(r) / attention out source)
  float* t = u + q * H;              // q * H (pre-activation) / q * qd attention q
  float* m = t + q * max(H, qd);     // q * H
  float* h = m + q * H;              // q * H
  float* y = h + q * H;              // q * H
  float* d = y + q * H;              // q * H
  float* kv = d + q * H;             // q * 2 kvd
  float* o = kv + q * 2 * kvd;       // q * qd
  float* ab = o + q * qd;            // q * 2 ffmax
  float* z = ab + q * 2 * ffmax;     // q * ffmax
  float* router = z + q * ffmax;     // q * E
  float* wts = router + q * P.E;     // q * K
  float* denom = wts + q * P.K;      // q
  int* sel = reinterpret_cast<int*>(denom + q);  // q * K

  // load / build the input records
  for (int i = tid; i < q * fpp; i += nt) {
    if (P.has_tokens) {
      const int p = i / fpp, c = i % fpp;
      rec[i] = c < hc * H ? embd[(size_t)tokens[p] * H + c % H] : 0.0f;  // P and g stay 0
    } else {
      rec[i] = rec_io[i];
    }
  }
  __syncthreads();

  for (int li = 0; li < P.nlayers; ++li) {
    const FixLayerW lw = W[li];
    const FixLayerS ls = S[li];
    const int L = P.layer_begin + li;
    const float* dn = lw.dense;
    const bool recur = lw.kind == 0;
    const float* wnorm = dn + P.o_norm;
    // 1. fold S_j += g_j * P ; u = mean over streams ; x = rmsnorm(u)
    for (int i = tid; i < q * hc * H; i += nt) {
      const int p = i / (hc * H), jc = i % (hc * H), j = jc / H, c = jc % H;
      float* r = rec + p * fpp;
      r[jc] += r[hc * H + H + j] * r[hc * H + c];
    }
    __syncthreads();
    const float inv = 1.0f / (float)hc;
    for (int i = tid; i < q * H; i += nt) {
      const int p = i / H, c = i % H;
      const float* r = rec + p * fpp;
      float acc = 0.0f;
      for (int j = 0; j < hc; ++j) acc += r[j * H + c];
      u[i] = acc * inv;
    }
    __syncthreads();
    for (int p = tid; p < q; p += nt) {
      float ss = 0.0f;
      for (int c = 0; c < H; ++c) ss += u[p * H + c] * u[p * H + c];
      denom[p] = sqrtf(ss / (float)H + 1e-6f);
    }
    __syncthreads();
    for (int i = tid; i < q * H; i += nt) x[i] = u[i] * wnorm[i % H] / denom[i / H];
    __syncthreads();
    // 2. PLE: n-gram hash over committed history + window tokens (prefix only)
    if (L == P.ple_layer) {
      for (int i = tid; i < q * H; i += nt) {
        const int p = i / H, c = i % H;
        const long long pos = P.base + p;
        uint64_t hsh = 0x243F6A8885A308D3ull;
        for (int k = P.ngram - 1; k >= 0; --k) {
          const int32_t tok =
              pos >= k ? (pos - k < P.base ? history[pos - k] : tokens[pos - k - P.base]) : -1;
          hsh = mix64d(hsh ^ (uint64_t)(uint32_t)tok);
        }
        x[i] += 0.1f * ple[(size_t)(hsh % (uint64_t)P.ple_rows) * H + c];
      }
      __syncthreads();
    }
    // 3. mixer
    if (recur) {
      const float* win = dn + P.o_win;
      const float* wout = dn + P.o_wout;
      const float* decay = dn + P.o_decay;
      for (int i = tid; i < q * H; i += nt) t[i] = dotf(win + (i % H) * H, x + (i / H) * H, H);
      __syncthreads();
      for (int c = tid; c < H; c += nt) {
        float prev = ls.rec[c];
        for (int p = 0; p < q; ++p) {
          const float r = decay[c] * prev + t[p * H + c];
          ls.snap[p * H + c] = r;
          u[p * H + c] = ftanh(r);
          prev = r;
        }
      }
      __syncthreads();
      for (int i = tid; i < q * H; i += nt) m[i] = dotf(wout + (i % H) * H, u + (i / H) * H, H);
      __syncthreads();
    } else {
      const float* wq = dn + P.o_wq;
      const float* wk = dn + P.o_wk;
      const float* wv = dn + P.o_wv;
      const float* wo = dn + P.o_wo;
      for (int i = tid; i < q * qd; i += nt) t[i] = dotf(wq + (i % qd) * H, x + (i / qd) * H, H);
      for (int i = tid; i < q * 2 * kvd; i += nt) {
        const int p = i / (2 * kvd), r = i % (2 * kvd);
        const float v = r < kvd ? dotf(wk + r * H, x + p * H, H) : dotf(wv + (r - kvd) * H, x + p * H, H);
        kv[i] = v;
        float* dst = r < kvd ? ls.kc : ls.vc;
        dst[(size_t)(P.base + p) * kvd + (r % kvd)] = v;
      }
      __syncthreads();
      const float scale = 1.0f / sqrtf((float)P.hd);
      const int group = P.nh / P.nkv;
      // scores[p][head][t] = dot(q_h, k_t) * scale
      for (int p = 0; p < q; ++p) {
        const long long npos = P.base + p + 1;
        for (long long i = tid; i < (long long)P.nh * npos; i += nt) {
          const int head = (int)(i / npos);
          const long long tt = i % npos;
          const float* kt = ls.kc + (size_t)tt * kvd + (head / group) * P.hd;
          scores[((size_t)p * P.nh + head) * P.score_ld + tt] = dotf(t + p * qd + head * P.hd, kt, P.hd) * scale;
        }
      }
      __syncthreads();
      // per (p, head): max, exp, ascending sum (one thread each)
      for (int i = tid; i < q * P.nh; i += nt) {
        const int p = i / P.nh;
        float* sc = scores + (size_t)i * P.score_ld;
        const long long npos = P.base + p + 1;
        float mx = 0.0f;
        for (long long tt = 0; tt < npos; ++tt)
          if (tt == 0 || sc[tt] > mx) mx = sc[tt];
        float sum = 0.0f;
        for (long long tt = 0; tt < npos; ++tt) {
          sc[tt] = fexp(sc[tt] - mx);
          sum += sc[tt];
        }
        sc[P.score_ld - 1] = sum;  // stash the sum past the row (npos <= max_context)
      }
      __syncthreads();
      for (int i = tid; i < q * qd; i += nt) {
        const int p = i / qd, hd_i = i % qd, head = hd_i / P.hd, dd = hd_i % P.hd;
        const float* sc = scores + ((size_t)p * P.nh + head) * P.score_ld;
        const float sum = sc[P.score_ld - 1];
        const long long npos = P.base + p + 1;
        float acc = 0.0f;
        for (long long tt = 0; tt < npos; ++tt) {
          const float wt = sc[tt] / sum;
          acc += wt * ls.vc[(size_t)tt * kvd + (head / group) * P.hd + dd];
        }
        o[i] = acc;
      }
      __syncthreads();
      for (int i = tid; i < q * H; i += nt) m[i] = dotf(wo + (i % H) * qd, o + (i / H) * qd, qd);
      __syncthreads();
    }
    // 4. h = x + m ; router logits
    for (int i = tid; i < q * H; i += nt) h[i] = x[i] + m[i];
    __syncthreads();
    const float* wr = dn + (recur ? P.o_router_r : P.o_router_a);
    const float* winj = dn + (recur ? P.o_inj_r : P.o_inj_a);
    for (int i = tid; i < q * P.E; i += nt) router[i] = dotf(wr + (i % P.E) * H, h + (i / P.E) * H, H);
    __syncthreads();
    // 5. top-K (ties to the lower expert index), sorted, softmax over the selected logits
    for (int p = tid; p < q; p += nt) {
      const float* rl = router + p * P.E;
      int* sp = sel + p * P.K;
      uint64_t used = 0;  // E <= 64
      for (int k = 0; k < P.K; ++k) {
        int best = P.E;
        for (int e = 0; e < P.E; ++e)
          if (!((used >> e) & 1ull) && (best == P.E || rl[e] > rl[best])) best = e;
        used |= 1ull << best;
        sp[k] = best;
      }
      for (int a = 1; a < P.K; ++a)  // insertion sort ascending
        for (int b = a; b > 0 && sp[b - 1] > sp[b]; --b) {
          const int tmp = sp[b];
          sp[b] = sp[b - 1];
          sp[b - 1] = tmp;
        }
      float mx = rl[sp[0]];
      for (int k = 0; k < P.K; ++k) mx = fmaxf(mx, rl[sp[k]]);
      float* wp = wts + p * P.K;
      float wsum = 0.0f;
      for (int k = 0; k < P.K; ++k) {
        wp[k] = fexp(rl[sp[k]] - mx);
        wsum += wp[k];
      }
      for (int k = 0; k < P.K; ++k) wp[k] /= wsum;
    }
    for (int i = tid; i < q * H; i += nt) y[i] = 0.0f;
    __syncthreads();
    // 6. routed experts in selection order, then the shared expert
    const size_t esz = (size_t)2 * P.ff * H + (size_t)H * P.ff;
    for (int k = 0; k <= P.K; ++k) {
      const bool shared = k == P.K;
      if (shared && (P.sff == 0 || lw.shared == nullptr)) break;
      const int ff = shared ? P.sff : P.ff;
      for (int i = tid; i < q * 2 * ff; i += nt) {
        const int p = i / (2 * ff), r = i % (2 * ff);
        const float* base = shared ? lw.shared : lw.experts + esz * sel[p * P.K + k];
        ab[p * 2 * ffmax + r] = dotf(base + (size_t)r * H, h + p * H, H);  // gate rows then up rows
      }
      __syncthreads();
      for (int i = tid; i < q * ff; i += nt) {
        const int p = i / ff, c = i % ff;
        z[p * ffmax + c] = fsilu(ab[p * 2 * ffmax + c]) * ab[p * 2 * ffmax + ff + c];
      }
      __syncthreads();
      for (int i = tid; i < q * H; i += nt) {
        const int p = i / H, c = i % H;
        const float* base = shared ? lw.shared : lw.experts + esz * sel[p * P.K + k];
        const float dv = dotf(base + (size_t)2 * ff * H + (size_t)c * ff, z + p * ffmax, ff);
        y[i] += shared ? dv : wts[p * P.K + k] * dv;
      }
      __syncthreads();
    }
    // 7. P = m + y ; g_j = sigmoid(inj_j . x)
    for (int i = tid; i < q * (H + hc); i += nt) {
      const int p = i / (H + hc), c = i % (H + hc);
      float* r = rec + p * fpp;
      if (c < H)
        r[hc * H + c] = m[p * H + c] + y[p * H + c];
      else
        r[hc * H + H + (c - H)] = fsigmoid(dotf(winj + (c - H) * H, x + p * H, H));
    }
    __syncthreads();
  }

  // this stage's output records (a tail's run_window returns them too, reference_domain.cpp:408-427)
  for (int i = tid; i < q * fpp; i += nt) rec_io[i] = rec[i];
  if (P.has_head) {
    // head_position (reference_domain.cpp:577-585): fold a copy of the streams, mean, rmsnorm(head_norm), logits
    for (int i = tid; i < q * H; i += nt) {
      const int p = i / H, c = i % H;
      const float* r = rec + p * fpp;
      float acc = 0.0f;
      for (int j = 0; j < hc; ++j) acc += r[j * H + c] + r[hc * H + H + j] * r[hc * H + c];
      u[i] = acc * (1.0f / (float)hc);
    }
    __syncthreads();
    for (int p = tid; p < q; p += nt) {
      float ss = 0.0f;
      for (int c = 0; c < H; ++c) ss += u[p * H + c] * u[p * H + c];
      denom[p] = sqrtf(ss / (float)H + 1e-6f);
    }
    __syncthreads();
    for (int i = tid; i < q * H; i += nt) x[i] = u[i] * head_norm[i % H] / denom[i / H];
    __syncthreads();
    for (int i = tid; i < q * P.V; i += nt) logits[i] = dotf(head_w + (size_t)(i % P.V) * H, x + (i / P.V) * H, H);
  }
}

// MTP fixture drafter step (drafter.cpp:39-55): logits = head . rmsnorm(embd[prev], norm).
__global__ void fixture_mtp_kernel(const float* __restrict__ embd, const float* __restrict__ norm,
                                   const float* __restrict__ head, int H, int V, const int32_t* __restrict__ prev,
                                   float* __restrict__ logits) {
  griddep_wait();
  griddep_launch();
  __shared__ float xs[1024];
  __shared__ float den;
  const int tok = *prev;
  const float* e = embd + (size_t)tok * H;
  if (threadIdx.x == 0) {
    float ss = 0.0f;
    for (int c = 0; c < H; ++c) ss += e[c] * e[c];
    den = sqrtf(ss / (float)H + 1e-6f);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) xs[c] = e[c] * norm[c] / den;
  __syncthreads();
  for (int v = threadIdx.x; v < V; v += blockDim.x) logits[v] = dotf(head + (size_t)v * H, xs, H);
}

__global__ void fixture_commit_kernel(float* __restrict__ rec, const float* __restrict__ snap, int H, int n) {
  for (int c = threadIdx.x; c < H; c += blockDim.x) rec[c] = snap[(size_t)(n - 1) * H + c];
}

}  // namespace clm

using namespace clm;

struct FixSession {
  uint64_t id = 0;
  long long pos = 0;
  uint32_t outstanding = 0;
  std::vector<float*> bufs;
  FixLayerS* d_layers = nullptr;
  int32_t* history = nullptr;  // prefix: committed tokens
};

struct FixtureEngine : clm_b200_engine {
  clm_b200_fixture_geometry g{};
  std::vector<uint8_t> kinds;
  clm_b200_stage_spec spec{};
  FixParams P{};
  bool prepared = false;
  std::map<std::string, float*> objects;  // name -> decoded f32 (device)
  std::vector<void*> allocations;
  uint64_t weight_bytes = 0;
  FixLayerW* d_w = nullptr;
  float *rec_io = nullptr, *logits = nullptr, *scores = nullptr, *mtp_logits = nullptr, *mtp_probs = nullptr;
  SampleScratch samp;  // chunked sampling scratch of the MTP drafter (1 row, 1 sequence)
  int32_t *tokens = nullptr, *prev = nullptr;
  std::map<uint64_t, std::unique_ptr<FixSession>> sessions;
  size_t smem = 0;

  int fpp() const { return (int)(g.residual_streams * g.hidden + g.hidden + g.residual_streams); }
  bool has_tokens() const { return spec.role == CLM_ROLE_PREFIX || spec.role == CLM_ROLE_WHOLE; }
  bool has_head() const { return spec.role == CLM_ROLE_TAIL || spec.role == CLM_ROLE_WHOLE; }
  int alloc(void** p, size_t bytes) {
    CLM_CUDA(cudaMalloc(p, bytes));
    allocations.push_back(*p);
    return CLM_OK;
  }
  float* obj(const std::string& n) const {
    auto it = objects.find(n);
    return it == objects.end() ? nullptr : it->second;
  }
  uint64_t dense_floats(int kind) const {
    const uint64_t H = g.hidden, qd = (uint64_t)g.n_heads * g.head_dim, kvd = (uint64_t)g.n_kv_heads * g.head_dim;
    const uint64_t mix = kind == 0 ? 2 * H * H + H : 2 * qd * H + 2 * kvd * H;
    return H + mix + (uint64_t)g.n_experts * H + (uint64_t)g.residual_streams * H;
  }
  // expected f32 element count of a named object, 0 if the name is not one of this stage's objects
  uint64_t expected_elems(const std::string& n) const {
    const uint64_t H = g.hidden, V = g.vocab;
    if (n == "token_embd") return V * H;
    if (n == "ple_lookup") return (uint64_t)g.ple_rows * H;
    if (n == "output_head" || n == "mtp_drafter") return H + V * H;
    unsigned L = 0, e = 0;
    char tail[32] = {0};
    if (sscanf(n.c_str(), "blk.%u.%31s", &L, tail) == 2 && L < g.n_layers) {
      const std::string t(tail);
      if (t == "dense") return dense_floats(kinds[L]);
      if (t == "shared") return 3ull * g.shared_expert_ff * H;
      if (sscanf(tail, "exp.%u", &e) == 1 && e < g.n_experts) return 3ull * g.expert_ff * H;
    }
    return 0;
  }
  ~FixtureEngine() override {
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto& kv : sessions)
      for (float* b : kv.second->bufs) cudaFree(b);
    for (void* p : allocations) cudaFree(p);
  }
};

namespace clm {

FixtureEngine* as_fixture(clm_b200_engine* e) { return static_cast<FixtureEngine*>(e); }

int fixture_create(clm_b200_ctx* ctx, const clm_b200_fixture_geometry* g, const clm_b200_stage_spec* spec,
                   clm_b200_engine** out) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(g && spec && out && g->layer_kinds, CLM_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  CLM_CHECK(g->n_layers > 0 && g->hidden > 0 && g->residual_streams > 0 && g->n_experts > 0 &&
                g->n_active_experts > 0 && g->n_active_experts <= g->n_experts && g->expert_ff > 0 &&
                g->n_heads > 0 && g->n_kv_heads > 0 && g->head_dim > 0 && g->vocab > 0 && g->ple_rows > 0,
            CLM_INVALID_ARGUMENT, "geometry: zero or inconsistent dimension");
  CLM_CHECK(g->n_heads % g->n_kv_heads == 0, CLM_INVALID_ARGUMENT, "geometry: n_heads must be a multiple of n_kv_heads");
  CLM_CHECK(g->ple_layer < g->n_layers && g->ple_ngram >= 1 && g->ple_ngram <= 16, CLM_INVALID_ARGUMENT,
            "geometry: PLE layer / n-gram out of range");
  CLM_CHECK(g->n_experts <= 64 && g->hidden <= 1024 && g->n_active_experts <= 16, CLM_UNIMPLEMENTED,
            "fixture engine supports E <= 64, H <= 1024, K <= 16");
  CLM_CHECK(spec->layer_end <= g->n_layers && spec->layer_begin <= spec->layer_end, CLM_INVALID_ARGUMENT,
            "layer range outside the model");
  CLM_CHECK(spec->max_context >= 1 && spec->max_window >= 1 && spec->max_sessions >= 1 &&
                spec->max_window <= spec->max_context && spec->max_window <= 16,
            CLM_INVALID_ARGUMENT, "domain spec needs max_context >= max_window >= 1, max_window <= 16");
  // role rules (reference_domain.cpp:67-85)
  const bool has_ple = g->ple_layer >= spec->layer_begin && g->ple_layer < spec->layer_end;
  switch (spec->role) {
    case CLM_ROLE_PREFIX:
      CLM_CHECK(spec->layer_begin == 0 && has_ple, CLM_INVALID_ARGUMENT,
                "prefix domain must start at layer 0 and contain the PLE layer");
      break;
    case CLM_ROLE_MIDDLE:
      CLM_CHECK(spec->layer_end > spec->layer_begin, CLM_INVALID_ARGUMENT, "middle domain needs at least one layer");
      CLM_CHECK(!has_ple, CLM_INVALID_ARGUMENT, "only the prefix domain may contain the PLE layer");
      break;
    case CLM_ROLE_TAIL:
      CLM_CHECK(!has_ple, CLM_INVALID_ARGUMENT, "only the prefix domain may contain the PLE layer");
      CLM_CHECK(spec->layer_end == g->n_layers, CLM_INVALID_ARGUMENT, "tail domain must end at the last layer");
      break;
    case CLM_ROLE_WHOLE:
      CLM_CHECK(spec->layer_begin == 0 && spec->layer_end == g->n_layers, CLM_INVALID_ARGUMENT,
                "a whole-model domain holds every layer");
      break;
    default:
      return fail(CLM_INVALID_ARGUMENT, "unknown role");
  }
  auto* e = new FixtureEngine();
  e->ctx = ctx;
  e->family = CLM_FAMILY_FIXTURE;
  e->g = *g;
  e->kinds.assign(g->layer_kinds, g->layer_kinds + g->n_layers);
  e->g.layer_kinds = nullptr;
  e->spec = *spec;
  for (uint8_t k : e->kinds)
    if (k > 1) {
      delete e;
      return fail(CLM_INVALID_ARGUMENT, "geometry: unknown layer kind");
    }
  ctx_retain(ctx);
  FixParams& P = e->P;
  P.H = (int)g->hidden;
  P.hc = (int)g->residual_streams;
  P.E = (int)g->n_experts;
  P.K = (int)g->n_active_experts;
  P.ff = (int)g->expert_ff;
  P.sff = (int)g->shared_expert_ff;
  P.nh = (int)g->n_heads;
  P.nkv = (int)g->n_kv_heads;
  P.hd = (int)g->head_dim;
  P.V = (int)g->vocab;
  P.ple_layer = (int)g->ple_layer;
  P.ngram = (int)g->ple_ngram;
  P.ple_rows = (int)g->ple_rows;
  P.nlayers = (int)(spec->layer_end - spec->layer_begin);
  P.layer_begin = (int)spec->layer_begin;
  P.max_context = (int)spec->max_context;
  P.score_ld = P.max_context + 1;
  P.has_tokens = e->has_tokens();
  P.has_head = e->has_head();
  const int H = P.H, qd = P.nh * P.hd, kvd = P.nkv * P.hd;
  P.o_norm = 0;
  P.o_win = H;
  P.o_decay = H + H * H;
  P.o_wout = 2 * H + H * H;
  P.o_router_r = 2 * H + 2 * H * H;
  P.o_inj_r = P.o_router_r + P.E * H;
  P.o_wq = H;
  P.o_wk = H + qd * H;
  P.o_wv = P.o_wk + kvd * H;
  P.o_wo = P.o_wv + kvd * H;
  P.o_router_a = P.o_wo + H * qd;
  P.o_inj_a = P.o_router_a + P.E * H;
  *out = e;
  return CLM_OK;
}

int fixture_set_object(FixtureEngine* e, const char* name, int quant, const void* h_bytes, uint64_t nbytes) {
  CLM_TRY(ctx_enter(e->ctx));
  CLM_CHECK(name && h_bytes, CLM_INVALID_ARGUMENT, "null argument");
  CLM_CHECK(!e->prepared, CLM_FAILED_PRECONDITION, "objects are bound before prepare");
  CLM_CHECK(quant == CLM_QUANT_F32 || quant == CLM_QUANT_Q8_FIXTURE, CLM_INVALID_ARGUMENT,
            "fixture objects are f32 or q8_0-fixture");
  const std::string n(name);
  const uint64_t elems = e->expected_elems(n);
  CLM_CHECK(elems != 0, CLM_NOT_FOUND, "'" + n + "' is not an object of this model");
  // routed experts are three whole-block tensors; everything else is one tensor
  const bool expert = n.find(".exp.") != std::string::npos;
  const uint64_t want = expert ? 3 * clm_b200_tensor_bytes(quant, elems / 3) : clm_b200_tensor_bytes(quant, elems);
  CLM_CHECK(want != 0 && nbytes == want, CLM_DATA_LOSS, "object '" + n + "' has the wrong size for its representation");
  void* staging = nullptr;
  CLM_CUDA(cudaMalloc(&staging, nbytes));
  float* dst = e->obj(n);
  int rc = CLM_OK;
  if (!dst) rc = e->alloc((void**)&dst, elems * sizeof(float));
  cudaStream_t st = e->ctx->stream;
  if (rc == CLM_OK) {
    cudaError_t err = cudaMemcpyAsync(staging, h_bytes, nbytes, cudaMemcpyHostToDevice, st);
    if (err != cudaSuccess) rc = cuda_fail(err, "object upload");
  }
  if (rc == CLM_OK) {
    if (expert) {
      const uint64_t per = elems / 3, pb = want / 3;
      for (int i = 0; i < 3 && rc == CLM_OK; ++i)
        rc = launch_decode(quant, static_cast<uint8_t*>(staging) + i * pb, dst + i * per, per, st);
    } else {
      rc = launch_decode(quant, staging, dst, elems, st);
    }
  }
  cudaStreamSynchronize(st);
  cudaFree(staging);
  if (rc != CLM_OK) return rc;
  if (!e->objects.count(n)) e->weight_bytes += nbytes;
  e->objects[n] = dst;
  return CLM_OK;
}

int fixture_prepare(FixtureEngine* e) {
  CLM_TRY(ctx_enter(e->ctx));
  CLM_CHECK(!e->prepared, CLM_FAILED_PRECONDITION, "domain already prepared; release() first");
  const FixParams& P = e->P;
  auto need = [&](const std::string& n) -> int {
    return e->obj(n) ? CLM_OK : fail(CLM_NOT_FOUND, "required object '" + n + "' is not bound");
  };
  std::vector<FixLayerW> w;
  for (int li = 0; li < P.nlayers; ++li) {
    const int L = P.layer_begin + li;
    const std::string b = "blk." + std::to_string(L) + ".";
    CLM_TRY(need(b + "dense"));
    if (P.sff > 0) CLM_TRY(need(b + "shared"));
    for (int x = 0; x < P.E; ++x) CLM_TRY(need(b + "exp." + std::to_string(x)));
    FixLayerW lw;
    lw.kind = e->kinds[L];
    lw.dense = e->obj(b + "dense");
    lw.shared = P.sff > 0 ? e->obj(b + "shared") : nullptr;
    // experts must be contiguous for the kernel: gather into one array
    const size_t esz = (size_t)3 * P.ff * P.H;
    float* all = nullptr;
    CLM_TRY(e->alloc((void**)&all, esz * P.E * sizeof(float)));
    for (int x = 0; x < P.E; ++x)
      CLM_CUDA(cudaMemcpyAsync(all + esz * x, e->obj(b + "exp." + std::to_string(x)), esz * sizeof(float),
                               cudaMemcpyDeviceToDevice, e->ctx->stream));
    lw.experts = all;
    w.push_back(lw);
  }
  if (e->has_tokens()) {
    CLM_TRY(need("token_embd"));
    CLM_TRY(need("ple_lookup"));
  }
  if (e->has_head()) CLM_TRY(need("output_head"));
  const int W = (int)e->spec.max_window, fpp = e->fpp();
  if (!w.empty()) {
    CLM_TRY(e->alloc((void**)&e->d_w, w.size() * sizeof(FixLayerW)));
    CLM_CUDA(cudaMemcpy(e->d_w, w.data(), w.size() * sizeof(FixLayerW), cudaMemcpyHostToDevice));
  }
  CLM_TRY(e->alloc((void**)&e->rec_io, (size_t)W * fpp * sizeof(float)));
  CLM_TRY(e->alloc((void**)&e->tokens, (size_t)(W + 1) * sizeof(int32_t)));
  CLM_TRY(e->alloc((void**)&e->prev, sizeof(int32_t)));
  CLM_TRY(e->alloc((void**)&e->scores, (size_t)W * P.nh * P.score_ld * sizeof(float)));
  if (e->has_head()) CLM_TRY(e->alloc((void**)&e->logits, (size_t)W * P.V * sizeof(float)));
  if (e->obj("mtp_drafter")) {
    CLM_TRY(e->alloc((void**)&e->mtp_logits, (size_t)W * P.V * sizeof(float)));
    CLM_TRY(e->alloc((void**)&e->mtp_probs, (size_t)W * P.V * sizeof(float)));  // one row per draft step
    void* sbase = nullptr;
    CLM_TRY(e->alloc(&sbase, SampleScratch::bytes(1, 1, (uint32_t)P.V)));
    e->samp = SampleScratch::carve(sbase, 1, 1, (uint32_t)P.V);
    CLM_CUDA(cudaMemset(sbase, 0, e->samp.counter_bytes));
  }
  const int qd = P.nh * P.hd, kvd = P.nkv * P.hd, ffmax = std::max(P.ff, P.sff);
  const size_t floats = (size_t)W * fpp + (size_t)W * P.H * 7 + (size_t)W * std::max(P.H, qd) + (size_t)W * 2 * kvd +
                        (size_t)W * qd + (size_t)W * 3 * ffmax + (size_t)W * P.E + (size_t)W * P.K + W;
  e->smem = floats * sizeof(float) + (size_t)W * P.K * sizeof(int);
  CLM_CHECK(e->smem <= 200 * 1024, CLM_RESOURCE_EXHAUSTED, "fixture window does not fit in shared memory");
  CLM_TRY(ensure_smem(fixture_window_kernel, e->smem));
  CLM_CUDA(cudaStreamSynchronize(e->ctx->stream));
  e->prepared = true;
  return CLM_OK;
}

int fixture_info(const FixtureEngine* e, uint64_t* weight_bytes, uint64_t* state_bytes, uint32_t* fpp) {
  if (weight_bytes) *weight_bytes = e->weight_bytes;
  if (state_bytes) {
    uint64_t n = 0;
    const uint64_t kvd = (uint64_t)e->P.nkv * e->P.hd;
    for (int li = 0; li < e->P.nlayers; ++li)
      n += e->kinds[e->P.layer_begin + li] == 0 ? (uint64_t)e->P.H * 4 : 2 * kvd * e->P.max_context * 4;
    if (e->has_tokens()) n += (uint64_t)e->P.max_context * 4;
    *state_bytes = n;
  }
  if (fpp) *fpp = (uint32_t)e->fpp();
  return CLM_OK;
}

int fixture_session_open(FixtureEngine* e, uint64_t id) {
  CLM_TRY(ctx_enter(e->ctx));
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "domain not prepared");
  CLM_CHECK(!e->sessions.count(id), CLM_ALREADY_EXISTS, "session already open");
  CLM_CHECK(e->sessions.size() < e->spec.max_sessions, CLM_RESOURCE_EXHAUSTED, "max_sessions reached");
  auto s = std::make_unique<FixSession>();
  s->id = id;
  const FixParams& P = e->P;
  const size_t kvd = (size_t)P.nkv * P.hd;
  std::vector<FixLayerS> ls(P.nlayers);
  auto mk = [&](float** p, size_t n) -> int {
    CLM_CUDA(cudaMalloc(p, n * sizeof(float)));
    s->bufs.push_back(*p);
    CLM_CUDA(cudaMemset(*p, 0, n * sizeof(float)));
    return CLM_OK;
  };
  int rc = CLM_OK;
  for (int li = 0; li < P.nlayers && rc == CLM_OK; ++li) {
    if (e->kinds[P.layer_begin + li] == 0) {
      rc = mk(&ls[li].rec, P.H);
      if (rc == CLM_OK) rc = mk(&ls[li].snap, (size_t)e->spec.max_window * P.H);
    } else {
      rc = mk(&ls[li].kc, (size_t)P.max_context * kvd);
      if (rc == CLM_OK) rc = mk(&ls[li].vc, (size_t)P.max_context * kvd);
    }
  }
  if (rc == CLM_OK && P.nlayers > 0) rc = mk(reinterpret_cast<float**>(&s->d_layers), ls.size() * sizeof(FixLayerS) / 4 + 1);
  if (rc == CLM_OK && P.nlayers > 0) {
    cudaError_t err = cudaMemcpy(s->d_layers, ls.data(), ls.size() * sizeof(FixLayerS), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) rc = cuda_fail(err, "session state");
  }
  if (rc == CLM_OK) rc = mk(reinterpret_cast<float**>(&s->history), (size_t)P.max_context);
  if (rc != CLM_OK) {
    for (float* b : s->bufs) cudaFree(b);
    return rc;
  }
  e->sessions[id] = std::move(s);
  return CLM_OK;
}

int fixture_session_close(FixtureEngine* e, uint64_t id) {
  CLM_TRY(ctx_enter(e->ctx));
  auto it = e->sessions.find(id);
  if (it == e->sessions.end()) return CLM_OK;
  CLM_CUDA(cudaStreamSynchronize(e->ctx->stream));
  for (float* b : it->second->bufs) cudaFree(b);
  e->sessions.erase(it);
  return CLM_OK;
}

int fixture_run_window(FixtureEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* tokens,
                       const float* in, float* out, float* logits, bool device, void* stream) {
  CLM_TRY(ctx_enter(e->ctx));
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "domain not prepared");
  auto it = e->sessions.find(id);
  CLM_CHECK(it != e->sessions.end(), CLM_NOT_FOUND, "session not open");
  FixSession& s = *it->second;
  CLM_CHECK(s.outstanding == 0, CLM_FAILED_PRECONDITION, "a window is already outstanding for this session");
  CLM_CHECK(q >= 1, CLM_INVALID_ARGUMENT, "window must have at least one position");
  CLM_CHECK(q <= e->spec.max_window, CLM_RESOURCE_EXHAUSTED, "window exceeds max_window");
  CLM_CHECK(base + q <= e->spec.max_context, CLM_RESOURCE_EXHAUSTED, "window exceeds max_context");
  CLM_CHECK((long long)base == s.pos, CLM_FAILED_PRECONDITION, "window base position != committed position");
  cudaStream_t st = device ? pick_stream(e->ctx, stream) : e->ctx->stream;
  const cudaMemcpyKind h2d = device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const cudaMemcpyKind d2h = device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
  const size_t rec = (size_t)q * e->fpp() * sizeof(float);
  if (e->has_tokens()) {
    CLM_CHECK(tokens != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes tokens");
    if (!device)
      for (uint32_t i = 0; i < q; ++i)
        CLM_CHECK(tokens[i] >= 0 && tokens[i] < e->P.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
    CLM_CUDA(cudaMemcpyAsync(e->tokens, tokens, q * sizeof(int32_t), h2d, st));
  } else {
    CLM_CHECK(in != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes activations");
    CLM_CUDA(cudaMemcpyAsync(e->rec_io, in, rec, h2d, st));
  }
  FixParams P = e->P;
  P.q = (int)q;
  P.base = (long long)base;
  P.has_head = e->has_head() && logits != nullptr;  // a tail's run_window without the head returns records only
  const unsigned long long l0 = t_kernel_launches;
  CLM_TRY(launch_pdl(fixture_window_kernel, dim3(1), dim3(256), e->smem, st, P, (const FixLayerW*)e->d_w,
                     (const FixLayerS*)s.d_layers, (const float*)e->obj("token_embd"),
                     (const float*)e->obj("ple_lookup"),
                     e->has_head() ? (const float*)e->obj("output_head") : nullptr,
                     e->has_head() ? (const float*)e->obj("output_head") + P.H : nullptr, (const int32_t*)e->tokens,
                     (const int32_t*)s.history, e->rec_io, e->logits, e->scores));
  e->last_launches = t_kernel_launches - l0;
  if (P.has_head) CLM_CUDA(cudaMemcpyAsync(logits, e->logits, (size_t)q * P.V * sizeof(float), d2h, st));
  if (out) CLM_CUDA(cudaMemcpyAsync(out, e->rec_io, rec, d2h, st));
  if (!device) CLM_CUDA(cudaStreamSynchronize(st));
  s.outstanding = q;
  return CLM_OK;
}

int fixture_commit(FixtureEngine* e, uint64_t id, uint32_t n) {
  CLM_TRY(ctx_enter(e->ctx));
  auto it = e->sessions.find(id);
  CLM_CHECK(it != e->sessions.end(), CLM_NOT_FOUND, "session not open");
  FixSession& s = *it->second;
  CLM_CHECK(s.outstanding > 0, CLM_FAILED_PRECONDITION, "no outstanding window");
  CLM_CHECK(n >= 1 && n <= s.outstanding, CLM_INVALID_ARGUMENT, "accepted must be in [1, q]");
  cudaStream_t st = e->ctx->stream;
  // keep exactly the first n positions: r = snapshot[n-1]; history += the first n tokens
  std::vector<FixLayerS> ls(e->P.nlayers);
  if (e->P.nlayers > 0)
    CLM_CUDA(cudaMemcpy(ls.data(), s.d_layers, ls.size() * sizeof(FixLayerS), cudaMemcpyDeviceToHost));
  for (int li = 0; li < e->P.nlayers; ++li)
    if (e->kinds[e->P.layer_begin + li] == 0) fixture_commit_kernel<<<1, 64, 0, st>>>(ls[li].rec, ls[li].snap, e->P.H, (int)n);
  if (e->has_tokens())
    CLM_CUDA(cudaMemcpyAsync(s.history + s.pos, e->tokens, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  CLM_CUDA(cudaStreamSynchronize(st));
  s.pos += n;
  s.outstanding = 0;
  return CLM_OK;
}

int fixture_abort(FixtureEngine* e, uint64_t id) {
  auto it = e->sessions.find(id);
  CLM_CHECK(it != e->sessions.end(), CLM_NOT_FOUND, "session not open");
  it->second->outstanding = 0;  // snapshots, tentative KV rows and window tokens are temporary by construction
  return CLM_OK;
}

int fixture_session_position(const FixtureEngine* e, uint64_t id, uint64_t* committed) {
  auto it = e->sessions.find(id);
  CLM_CHECK(it != e->sessions.end(), CLM_NOT_FOUND, "session not open");
  *committed = (uint64_t)it->second->pos;
  return CLM_OK;
}

int fixture_mtp_draft(FixtureEngine* e, int32_t prev, uint32_t count, float T, uint64_t seed, uint64_t counter,
                      int32_t* h_tokens, float* h_logits) {
  CLM_TRY(ctx_enter(e->ctx));
  CLM_CHECK(e->prepared && e->obj("mtp_drafter") && e->obj("token_embd"), CLM_FAILED_PRECONDITION,
            "the MTP drafter needs the mtp_drafter and token_embd objects");
  CLM_CHECK(count >= 1 && count <= e->spec.max_window, CLM_OUT_OF_RANGE, "count must be in [1, max_window]");
  CLM_CHECK(h_tokens != nullptr, CLM_INVALID_ARGUMENT, "null output");
  const FixParams& P = e->P;
  CLM_CHECK(prev >= 0 && prev < P.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
  cudaStream_t st = e->ctx->stream;
  unsigned long long* ctr = nullptr;
  CLM_CUDA(cudaMalloc(&ctr, sizeof(unsigned long long)));
  unsigned long long cv = counter;
  CLM_CUDA(cudaMemcpyAsync(ctr, &cv, sizeof(cv), cudaMemcpyHostToDevice, st));
  CLM_CUDA(cudaMemcpyAsync(e->tokens, &prev, sizeof(int32_t), cudaMemcpyHostToDevice, st));
  const float* mtp = e->obj("mtp_drafter");
  int rc = CLM_OK;
  for (uint32_t j = 0; j < count && rc == CLM_OK; ++j) {
    rc = launch_pdl(fixture_mtp_kernel, dim3(1), dim3(256), 0, st, (const float*)e->obj("token_embd"), mtp, mtp + P.H,
                    P.H, P.V, (const int32_t*)(e->tokens + j), e->mtp_logits + (size_t)j * P.V);
    if (rc == CLM_OK) {
      const float* row = e->mtp_logits + (size_t)j * P.V;
      if (T > 0.0f) {
        rc = launch_probs(row, 1, (uint32_t)P.V, T, nullptr, e->mtp_probs, e->samp, st);
        if (rc == CLM_OK)
          rc = launch_sample_rows(e->mtp_probs, 1, (uint64_t)P.V, (uint32_t)P.V, nullptr, seed, j, 1u, ctr, nullptr,
                                  e->tokens + j + 1, e->samp, st);
      } else {
        rc = launch_argmax_rows(row, 1, (uint32_t)P.V, e->tokens + j + 1, e->samp, st);
      }
    }
  }
  if (rc == CLM_OK) {
    cudaMemcpyAsync(h_tokens, e->tokens + 1, count * sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (h_logits) cudaMemcpyAsync(h_logits, e->mtp_logits, (size_t)count * P.V * sizeof(float), cudaMemcpyDeviceToHost, st);
  }
  cudaStreamSynchronize(st);
  cudaFree(ctr);
  return rc;
}

// Stochastic MTP proposal (clm_b200_mtp_propose; MtpFixtureDrafter::propose, drafter.cpp:72-86): each draft is
// sampled from distribution(step logits, T, top-k, top-p) with the caller's uniform; the rows are returned.
int fixture_mtp_propose(FixtureEngine* e, int32_t prev, uint32_t count, float T, uint32_t top_k, float top_p,
                        const double* h_uniforms, int32_t* h_tokens, float* h_probs) {
  if (T <= 0.0f) {  // greedy drafts (argmax chain), one-hot rows
    const int rc = fixture_mtp_draft(e, prev, count, 0.0f, 0, 0, h_tokens, nullptr);
    if (rc == CLM_OK && h_probs != nullptr) {
      const size_t V = (size_t)e->P.V;
      std::memset(h_probs, 0, count * V * sizeof(float));
      for (uint32_t j = 0; j < count; ++j) h_probs[j * V + (uint32_t)h_tokens[j]] = 1.0f;
    }
    return rc;
  }
  CLM_TRY(ctx_enter(e->ctx));
  CLM_CHECK(e->prepared && e->obj("mtp_drafter") && e->obj("token_embd"), CLM_FAILED_PRECONDITION,
            "the MTP drafter needs the mtp_drafter and token_embd objects");
  CLM_CHECK(count >= 1 && count <= e->spec.max_window, CLM_OUT_OF_RANGE, "count must be in [1, max_window]");
  CLM_CHECK(h_tokens != nullptr && h_uniforms != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  const FixParams& P = e->P;
  CLM_CHECK(prev >= 0 && prev < P.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
  cudaStream_t st = e->ctx->stream;
  double* du = nullptr;
  CLM_CUDA(cudaMalloc(&du, count * sizeof(double)));
  int rc = CLM_OK;
  if (cudaMemcpyAsync(du, h_uniforms, count * sizeof(double), cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(e->tokens, &prev, sizeof(int32_t), cudaMemcpyHostToDevice, st) != cudaSuccess)
    rc = fail(CLM_INTERNAL, "uniform / token upload failed");
  const float* mtp = e->obj("mtp_drafter");
  for (uint32_t j = 0; j < count && rc == CLM_OK; ++j) {
    rc = launch_pdl(fixture_mtp_kernel, dim3(1), dim3(256), 0, st, (const float*)e->obj("token_embd"), mtp, mtp + P.H,
                    P.H, P.V, (const int32_t*)(e->tokens + j), e->mtp_logits + (size_t)j * P.V);
    if (rc == CLM_OK)
      rc = launch_draft_sample(e->ctx, e->mtp_logits + (size_t)j * P.V, (uint32_t)P.V, T, top_k, top_p, du + j,
                               e->mtp_probs + (size_t)j * P.V, e->tokens + j + 1, e->samp, st);
  }
  if (rc == CLM_OK) {
    cudaMemcpyAsync(h_tokens, e->tokens + 1, count * sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (h_probs) cudaMemcpyAsync(h_probs, e->mtp_probs, (size_t)count * P.V * sizeof(float), cudaMemcpyDeviceToHost, st);
  }
  const cudaError_t se = cudaStreamSynchronize(st);
  cudaFree(du);
  if (rc == CLM_OK && se != cudaSuccess) rc = cuda_fail(se, "mtp propose");
  return rc;
}

}  // namespace clm
