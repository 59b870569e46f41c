// engine.cu — the Llama-family execution engine: one stage (layer range) of a model on one GPU, its sessions,
// window execution (CUDA graphs of PDL-chained kernels), commit/abort, the MTP draft head and the
// device-resident speculative round.
//
// Window semantics follow ReferenceDomainImpl::execute / commit_window / abort_window
// (runtime/domain/src/reference_domain.cpp:297-445): a window writes KV rows at positions base..base+q-1
// tentatively; commit(n) advances the committed position by n (rows past it are rewritten before any later
// read, as in the reference); abort drops the window.
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "codec.cuh"
#include "bulk.cuh"
#include "engine.cuh"
#include "gemv_strip.cuh"
#include "link.cuh"
#include "flow.cuh"
#include "gemv.cuh"
#include "gemv2.cuh"
#include "llama.cuh"
#include "matrix.cuh"
#include "pdl.cuh"
#include "sampling.cuh"
#include "gemm_tc.cuh"
#include "wide.cuh"

namespace clm {

struct SessionState {  // device-resident, one per session
  long long pos;               // committed position
  unsigned long long round;    // speculative rounds completed (Philox counter)
  int next_token;              // token to feed at `pos`
  unsigned accepted;           // drafts accepted in the last round
  int count;                   // tokens emitted by the last round
  unsigned commit_in;          // pipeline: positions committed at the start of the current round (from the link)
};

struct Gemv {
  clm_b200_matrix* m = nullptr;
  GemvPlan plan[3];  // nt = 1, 2, 4
  const GemvPlan& for_q(int q) const { return plan[q <= 8 ? 0 : (q <= 16 ? 1 : 2)]; }
};

struct Session {
  uint64_t id = 0;
  std::vector<int32_t> pages;
  int32_t* d_pages = nullptr;
  SessionState* d_state = nullptr;
  long long pos = 0;          // committed position as known to the host
  long long pos_bound = 0;    // upper bound while device-driven rounds are in flight
  bool pos_stale = false;     // device rounds ran since the last read of d_state->pos
  uint32_t outstanding = 0;  // q of the outstanding window, 0 = none
  bool tree = false;         // the outstanding window is a tree (commit with clm_b200_commit_path)
  std::vector<int32_t> tree_parents;  // the outstanding tree's parents when given by the host (else in e->parents)
  std::map<std::tuple<int, int, int>, cudaGraphExec_t> graphs;  // (kind, q, flag) -> executable graph
  std::map<std::tuple<int, int, int>, int> seen;
  std::map<std::tuple<int, int, int>, unsigned long long> launches;  // kernels per graph
  std::map<int, FlowPhase*> flow_phases;  // dataflow window kernel phase tables by q (device arrays)
  int32_t* d_win = nullptr;    // pipeline tail: this session's current window tokens [W + 1]
  float* d_dprobs = nullptr;   // pipeline tail: draft distributions of the current window [W][V]
  bool own_links = false;      // pipeline: the session's messages use lin / lout below (clm_b200_pipe_attach_session)
  LinkDev lin, lout;
};

// Zeroes the dataflow counters of a window chain before its first linked launch (after the previous window ended).
__global__ void zero_ints_kernel(int* __restrict__ p, int n) {
  griddep_wait();
  griddep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = 0;
}

__global__ void fill_kernel(float* p, float v, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// rope[pos][i] = (cos, sin)(pos * theta^(-2i/hd)), evaluated in double and rounded to f32.
__global__ void rope_table_kernel(float2* __restrict__ out, uint32_t npos, int hd, float theta) {
  const uint64_t n = (uint64_t)npos * (hd / 2);
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n; k += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t pos = k / (hd / 2);
    const int i = (int)(k % (hd / 2));
    const double inv = exp2(-(double)(2 * i) / (double)hd * log2((double)theta));
    double sn, cs;
    sincos((double)pos * inv, &sn, &cs);
    out[k] = make_float2((float)cs, (float)sn);
  }
}

// Keeps the accepted tree path: the KV rows of window nodes path[i] move to window slot i (base + i), in every
// layer and kv head.  One CTA per (layer, kv head); all sources are read before any row is written (a path is
// increasing, but a destination can be a later move's source).  K rows are swizzled by position parity and V^T
// columns by head-dim parity (llama.cuh), so elements are moved one by one with both layouts' index maps.
__global__ void kv_compact_kernel(__half* const* __restrict__ kpools, __half* const* __restrict__ vpools,
                                  const int32_t* __restrict__ pages, const long long* __restrict__ d_pos,
                                  const int32_t* __restrict__ path, int n, int nkv, int hd) {
  extern __shared__ __half kv_rows[];  // [n][2][hd]
  const int layer = blockIdx.x, kvh = blockIdx.y;
  __half* K = kpools[layer];
  __half* Vt = vpools[layer];
  const long long base = *d_pos;
  auto k_at = [&](long long slot, int dd) -> __half* {
    const int pos = (int)(slot % 64);
    return K + (((size_t)pages[slot / 64] * nkv + kvh) * 64 + pos) * hd + 8 * kv_k_chunk(dd >> 3, pos) + (dd & 7);
  };
  auto v_at = [&](long long slot, int dd) -> __half* {
    const int pos = (int)(slot % 64);
    return Vt + (((size_t)pages[slot / 64] * nkv + kvh) * hd + dd) * 64 + 8 * kv_v_chunk(pos >> 3, dd) + (pos & 7);
  };
  for (int j = threadIdx.x; j < n * hd; j += blockDim.x) {
    const int i = j / hd, dd = j % hd;
    const long long src = base + path[i];
    kv_rows[(2 * i) * hd + dd] = *k_at(src, dd);
    kv_rows[(2 * i + 1) * hd + dd] = *v_at(src, dd);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < n * hd; j += blockDim.x) {
    const int i = j / hd, dd = j % hd;
    if (path[i] == i) continue;
    *k_at(base + i, dd) = kv_rows[(2 * i) * hd + dd];
    *v_at(base + i, dd) = kv_rows[(2 * i + 1) * hd + dd];
  }
}

__global__ void round_head_kernel(const SessionState* __restrict__ st, int32_t* __restrict__ win) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) win[0] = st->next_token;
}

// Greedy acceptance (coordinator.cpp:1295-1298) from the window's row argmaxes: accepted = longest prefix with
// argmax(logits[i]) == window[i+1]; next = argmax(logits[accepted]).
__global__ void greedy_decide_kernel(const int32_t* __restrict__ am, int q, const int32_t* __restrict__ win,
                                     uint32_t* __restrict__ acc, int32_t* __restrict__ nxt) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x != 0) return;
  uint32_t a = 0;
  while ((int)a + 1 < q && am[a] == win[a + 1]) ++a;
  *acc = a;
  *nxt = am[a];
}

// Emits win[1..a] and the next token, advances the session (commit of a+1 positions).
__global__ void round_commit_kernel(SessionState* __restrict__ st, const int32_t* __restrict__ win,
                                    const uint32_t* __restrict__ acc, const int32_t* __restrict__ nxt,
                                    int32_t* __restrict__ emitted, uint32_t* __restrict__ count) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x != 0) return;
  const uint32_t a = *acc;
  for (uint32_t i = 0; i < a; ++i) emitted[i] = win[1 + i];
  emitted[a] = *nxt;
  *count = a + 1;
  st->pos += a + 1;
  st->next_token = *nxt;
  st->accepted = a;
  st->count = (int)(a + 1);
  st->round += 1;
}

// Commits a prefill chunk of q positions (auto_commit).
__global__ void pos_advance_kernel(SessionState* __restrict__ st, int q) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) st->pos += q;
}

__global__ void set_next_kernel(SessionState* __restrict__ st, const int32_t* __restrict__ tok) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x == 0) st->next_token = *tok;
}

// Copies a device tree's parent array, replacing any entry that is not -1 or an earlier node by -1 and flagging
// the window (kErrBadTree), so no ancestor walk can leave the window.
constexpr int kErrBadTree = 6;
__global__ void tree_guard_kernel(const int32_t* __restrict__ in, int q, int32_t* __restrict__ out, int* __restrict__ bad) {
  const int i = threadIdx.x;
  if (i < q) {
    const int32_t p = in[i];
    const bool ok = p >= -1 && p < i;
    out[i] = ok ? p : -1;
    if (!ok) atomicExch(bad, kErrBadTree);
  }
}

__global__ void embed_guard_kernel(const int32_t* __restrict__ tokens, int q, int vocab, int32_t* __restrict__ out,
                                   int* __restrict__ bad) {
  griddep_wait();
  griddep_launch();
  const int p = threadIdx.x;
  if (p < q) {
    const int32_t t = tokens[p];
    const bool ok = t >= 0 && t < vocab;
    out[p] = ok ? t : 0;
    if (!ok) atomicExch(bad, 1);
  }
}

}  // namespace clm

using namespace clm;

struct LlamaEngine : clm_b200_engine {
  LlamaDims d;
  clm_b200_llama_geometry geo{};
  clm_b200_stage_spec spec{};
  bool has_embd = false, has_head = false, has_mtp = false, has_tokens = false;
  bool prepared = false, weights_ready = false;
  int max_pages = 0;  // pages per session
  int pages_total = 0;
  std::vector<int32_t> free_pages;
  // weights
  struct Layer {
    Gemv qkv, o, gu, down;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
  };
  std::vector<Layer> layers;
  uint8_t* embd = nullptr;
  uint64_t embd_bytes = 0;
  Gemv head, mtp_gu, mtp_down;
  float *out_norm = nullptr, *mtp_ffn_norm = nullptr, *mtp_out_norm = nullptr;
  // KV pools per layer
  std::vector<__half*> kpool, vpool;
  __half** d_kpools = nullptr;  // device copies of the pool pointers (tree-path KV compaction)
  __half** d_vpools = nullptr;
  // window buffers
  float* h = nullptr;
  float* part = nullptr;     // GEMV split partials (last-CTA reduction)
  int* gcount = nullptr;     // GEMV row-group counters
  // the second partial region of the linked chain: consecutive GEMVs alternate between the two (a GEMV's partials
  // may still be read by its first segments while the next GEMV's later segments write theirs)
  float* part2 = nullptr;
  int* gcount2 = nullptr;
  // dataflow counters of a linked window chain (LinkLayout per layer), zeroed at the start of every window
  int* link_ctr = nullptr;
  int link_n = 0;
  bool link_ok = false;  // the linked chain is on (CLM_B200_LINK=1) and the geometry fits it
  // the strip GEMV (gemv_strip.cu) for the layers' QKV (1), W_o (2), gate|up (4) (CLM_B200_STRIP): measured faster
  // for QKV and W_o, whose stream-K reductions dominate their time, slower for the longer gate|up stream
  int strip_mask = 3;
  unsigned long long pf_cap = 64 * 1024;  // L2 lookahead bytes per CTA of the next GEMV (CLM_B200_PF_KB)
  int* acount = nullptr;     // attention (m-tile, kv head) counters
  size_t gcount_n = 0, acount_n = 0;  // their lengths (reset_counters)
  void* samp_counters = nullptr;      // the sampling scratch's arrival counters and their bytes
  size_t samp_counter_bytes = 0;
  XBuf xa, xb;               // activation hand-offs, alternated along the chain
  float* ones_h = nullptr;   // norm weight 1 for stage ends without a following norm
  __half* q16 = nullptr;
  float* attn_part = nullptr;
  float2* rope = nullptr;    // RoPE (cos, sin) table [max_context][hd/2]
  // dataflow verify-window kernel (flow.cu): grid / ring stages per column-tile count (index nt - 1), attention
  // segment partials, per-kind GEMV partials, readiness counters
  int flow_grid_n[2] = {0, 0}, flow_stage_count[2] = {0, 0}, flow_stage_bytes[2] = {0, 0};
  int flow_attn_maxseg = 0;
  float* flow_attn_part = nullptr;
  enum { FK_QKV = 0, FK_O, FK_GU, FK_DOWN, FK_HEAD, FK_KINDS };
  float* flow_part[FK_KINDS] = {};  // stream-K partials per matrix kind (phases of one kind never overlap)
  int* flow_gcount[FK_KINDS] = {};  // their row-group counters
  size_t flow_gcount_n[FK_KINDS] = {};
  int* flow_ctr = nullptr;          // readiness counters of one window, zeroed before every launch
  size_t flow_ctr_n = 0;
  // wide windows (17..max_window rows when max_window > 16): tensor-core GEMMs (gemm_tc.cu) between the elementwise
  // steps of wide.cu
  float* wy = nullptr;       // GEMM outputs [W][largest row count of a layer matrix]
  float* wpart = nullptr;    // split-K partials of the tensor-core GEMMs
  size_t wpart_floats = 0;
  float* wattn = nullptr;    // attention outputs [W][qd]
  float* wattn_part = nullptr;  // wide attention: KV-split partials and their tile counters
  size_t wattn_part_floats = 0;
  int* wattn_cnt = nullptr;
  int wattn_tiles = 0;
  uint8_t* wxh = nullptr;    // fp16 activation tiles of the next GEMM
  float* logits = nullptr;
  int32_t* tokens = nullptr;
  float* bin = nullptr;
  float* bout = nullptr;
  float* h_mtp = nullptr;
  float* draft_logits = nullptr;
  int32_t* win = nullptr;
  int32_t* parents = nullptr;  // tree window: parent node of each window row (-1: the committed context)
  float* tprobs = nullptr;    // distribution rows of the window's logits [W][V]
  float* dprobs = nullptr;    // distribution rows of the MTP drafts [W][V]
  int32_t* am = nullptr;      // row argmaxes [W]
  SampleScratch samp;         // chunked sampling scratch (2W rows, 1 sequence)
  uint32_t* acc = nullptr;
  int32_t* nxt = nullptr;
  int32_t* emitted = nullptr;
  uint32_t* count = nullptr;
  int* bad = nullptr;
  unsigned long long* zero_counter = nullptr;
  RoundCtl* ctl = nullptr;               // temperature / seed of the current round (device)
  double* propose_u = nullptr;           // clm_b200_mtp_propose's uniforms [max_window]
  // stage pipeline (link.cuh): input and output links and their device views
  clm_b200_link* pipe_in = nullptr;
  clm_b200_link* pipe_out = nullptr;
  LinkDev lin, lout;
  std::map<uint64_t, std::unique_ptr<Session>> sessions;
  // batched windows: CUDA graphs per session set (the Session objects hold only graphs), dropped whenever a session
  // closes (the graphs hold its position and page-table addresses)
  std::map<std::vector<uint64_t>, std::unique_ptr<Session>> batch_graphs;
  std::vector<void*> allocations;
  uint64_t weight_bytes = 0;

  int floats_per_position() const { return 2 * d.H + 1; }
  float hi_scale() const { return d.quant == CLM_QUANT_Q4_K ? 0.0625f : 1.0f; }
  int wmax() const { return (int)spec.max_window; }

  // pinned host staging of the host-buffer window calls (grown on demand, freed with the engine)
  void* pin_in = nullptr;
  void* pin_out = nullptr;
  size_t pin_in_bytes = 0, pin_out_bytes = 0;
  int pinned(void** buf, size_t* cap, size_t bytes) {
    if (bytes <= *cap) return CLM_OK;
    if (*buf) CLM_CUDA(cudaFreeHost(*buf));
    *buf = nullptr;
    *cap = 0;
    CLM_CUDA(cudaHostAlloc(buf, bytes, cudaHostAllocDefault));
    *cap = bytes;
    return CLM_OK;
  }

  int alloc(void** p, size_t bytes) {
    CLM_CUDA(cudaMalloc(p, bytes));
    allocations.push_back(*p);
    return CLM_OK;
  }
  template <typename T>
  int alloc_t(T** p, size_t count) {
    void* v = nullptr;
    CLM_TRY(alloc(&v, count * sizeof(T)));
    *p = static_cast<T*>(v);
    return CLM_OK;
  }

  int make_gemv(Gemv& g, const void* d_src, uint64_t nbytes, uint32_t rows, uint32_t cols, uint32_t half_rows = 0) {
    CLM_TRY(matrix_create(ctx, d.quant, d_src, true, nbytes, rows, cols, &g.m, half_rows));
    g.plan[0] = gemv_plan(g.m->shape, 8, ctx->sm_count);
    g.plan[1] = gemv_plan(g.m->shape, 16, ctx->sm_count);
    g.plan[2] = gemv_plan(g.m->shape, 32, ctx->sm_count);
    weight_bytes += g.m->bytes;
    return CLM_OK;
  }

  int ones(float** p, size_t n) {
    CLM_TRY(alloc_t(p, n));
    fill_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, ctx->stream>>>(*p, 1.0f, n);
    CLM_LAUNCHED("fill_kernel");
    return CLM_OK;
  }

  // ---- one fused GEMV of the chain
  int gemv_strip(const Gemv& g, int q, const XBuf& in, const Epi& epi, cudaStream_t st) {
    return launch_gemv_strip(g.m->shape, static_cast<const uint8_t*>(g.m->data), in, q, epi, ctx->sm_count, st);
  }
  // Whether matrix `bit` of a layer (1 QKV, 2 W_o, 4 gate|up) runs on the strip GEMV for q rows.
  bool strip_for(const Gemv& g, int bit, int q, int kind) const {
    return (strip_mask & bit) && gemv_strip_ok(g.m->shape, q, kind);
  }
  int gemv(const Gemv& g, int q, const XBuf& in, const Epi& epi, cudaStream_t st, bool alt = false) {
    const GemvPlan& p = g.for_q(q);
    return launch_gemv(g.m->shape, p, static_cast<const uint8_t*>(g.m->data), in, q, epi, alt ? part2 : part,
                       alt ? gcount2 : gcount, st);
  }

  // Counters of one layer of a linked chain (ints at link_ctr + layer * per_layer): the attention's wait per kv
  // head, W_o's input chunks, gate|up's input chunks + W_o's finished groups, down's input chunks, the next QKV's
  // (or the head's) input chunks + down's finished groups.
  struct LinkLayout {
    int attn, o, gu, o_done, down, next, down_done, per_layer;
  };
  LinkLayout link_layout() const {
    LinkLayout L;
    const int ch_h = d.H / 512, ch_q = d.qd() / 512, ch_f = d.F / 512;
    L.attn = 0;
    L.o = L.attn + d.nkv;
    L.gu = L.o + ch_q;
    L.o_done = L.gu + ch_h;
    L.down = L.o_done + 1;
    L.next = L.down + ch_f;
    L.down_done = L.next + ch_h;
    L.per_layer = L.down_done + 1;
    return L;
  }
  bool link_shape_ok() const {
    const int group = d.nh / d.nkv;
    return d.hd == 128 && d.H % 512 == 0 && d.qd() % 512 == 0 && d.F % 512 == 0 &&
           (group % 4 == 0 || 4 % group == 0);
  }
  Epi epi_base(int kind) const {
    Epi e;
    e.kind = kind;
    e.ss_n = (float)d.H;
    e.eps = d.eps;
    e.hi_scale = hi_scale();
    e.err = bad;
    return e;
  }
  Epi epi_resid(float* hbuf, const float* wnext, const XBuf& next) const {
    Epi e = epi_base(EPI_RESID_PREP);
    e.h = hbuf;
    e.H = d.H;
    e.wnext = wnext;
    e.next = next;
    return e;
  }

  // L2 lookahead of the next GEMV of the chain: each CTA prefetches the first bytes of the matching CTA range of
  // `next` (its first units) once its own copies are issued
  void lookahead(Epi& e, const Gemv& next) const {
    e.pf = static_cast<const uint8_t*>(next.m->data);
    e.pf_bytes = next.m->shape.bytes();
    e.pf_cap = pf_cap;
  }

  // ---- the layer range over q rows; h holds the stage input and xa its first norm's preparation
  int enqueue_layers(Session& s, int q, const int32_t* parent, cudaStream_t st) {
    const int nt = q <= 8 ? 1 : 2;
    const long long* pos = &s.d_state->pos;
    // linked chain: every launch after the first waits on per-chunk readiness counters instead of on its
    // predecessor's completion (gemv4.cu, llama.cu); the partial regions alternate between consecutive GEMVs
    const bool linked = link_ok;
    const LinkLayout LL = link_layout();
    const int group = d.nh / d.nkv;
    const int mtiles = (q * group + 15) / 16;
    const int splits = attention_splits(q, d, max_pages, ctx->sm_count);
    auto ctr = [&](size_t li, int off) { return link_ctr + li * LL.per_layer + off; };
    for (size_t li = 0; li < layers.size(); ++li) {
      Layer& L = layers[li];
      const bool sq = strip_for(L.qkv, 1, q, EPI_ROPE_KV), so = strip_for(L.o, 2, q, EPI_RESID_PREP),
                 sg = strip_for(L.gu, 4, q, EPI_SWIGLU_PREP);
      const int strips_per_head = d.hd / 16;
      // q, k, v with RoPE and the paged KV append fused into the epilogue (input: xa = h * attn_norm)
      Epi ek = epi_base(EPI_ROPE_KV);
      ek.nh = d.nh;
      ek.nkv = d.nkv;
      ek.hd = d.hd;
      ek.rope = rope;
      ek.pos = pos;
      ek.pages = s.d_pages;
      ek.kpool = kpool[li];
      ek.vpool = vpool[li];
      ek.q16 = q16;
      ek.parent = parent;
      ek.pf_kv = true;  // the attention's KV pages into L2 while the QKV GEMV drains
      ek.pf_max_pages = max_pages;
      AttnLink al;
      if (linked) {
        if (li > 0) link_in(ek, li - 1, LL.next, 4, LL.down_done, d.H / 128);
        ek.sig = ctr(li, LL.attn);
        ek.sig_qkv = 1;
        al.wait = ctr(li, LL.attn);
        // the kv head's query heads, its k head and its v head (each in 8 strips on the strip GEMV)
        al.target = (group + 2) * (sq ? strips_per_head : 1);
        al.sig = ctr(li, LL.o);
        if (group >= 4) {
          al.span = group / 4;
        } else {
          al.kvh_div = 4 / group;
        }
      }
      if (sq) {
        CLM_TRY(gemv_strip(L.qkv, q, xa, ek, st));
      } else {
        CLM_TRY(gemv(L.qkv, q, xa, ek, st));
      }
      // attention -> xb (W_o input); W_o into L2 meanwhile
      CLM_TRY(launch_attention(q16, kpool[li], vpool[li], s.d_pages, pos, parent, q, d, max_pages, attn_part, acount,
                               nt, hi_scale(), xb.frag, xb.sum, bad, static_cast<const uint8_t*>(L.o.m->data),
                               L.o.m->shape.bytes(), ctx->sm_count, st, nullptr, al));
      XBuf ob = xb;
      ob.ss = nullptr;
      // h += W_o o ; xa = h * ffn_norm (+ sum of squares)
      Epi eo = epi_resid(h, L.ffn_norm, xa);
      lookahead(eo, L.gu);
      if (linked) {
        eo.wait = ctr(li, LL.o);
        eo.wait_target = splits * mtiles * (group >= 4 ? 1 : 4 / group);
        eo.sig = ctr(li, LL.gu);
        eo.sig_div = 4;
        eo.done = ctr(li, LL.o_done);
      }
      if (so) {
        CLM_TRY(gemv_strip(L.o, q, ob, eo, st));
      } else {
        CLM_TRY(gemv(L.o, q, ob, eo, st, linked));
      }
      // SwiGLU of the gate/up rows -> xb (W_down input)
      Epi es = epi_base(EPI_SWIGLU_PREP);
      es.ffn = d.F;
      es.next = xb;
      lookahead(es, L.down);
      XBuf gin = xa;
      if (so) gin.nss = d.H / 16;  // W_o's strips wrote sum-of-squares partials per 16 columns
      if (linked) {
        // a chunk of gate|up's input: 4 row groups of W_o, or 32 of its strips
        link_in(es, li, LL.gu, so ? 32 : 4, LL.o_done, so ? d.H / 16 : d.H / 128);
        es.sig = ctr(li, LL.down);
        es.sig_div = 8;  // 64 SwiGLU outputs per row group, 512 per chunk of down's input
      }
      if (sg) {
        CLM_TRY(gemv_strip(L.gu, q, gin, es, st));
      } else {
        CLM_TRY(gemv(L.gu, q, gin, es, st));
      }
      // h += W_down a ; xa = h * (next layer's attn_norm | output norm | 1)
      const float* wnext = li + 1 < layers.size() ? layers[li + 1].attn_norm : (has_head ? out_norm : ones_h);
      XBuf db = xb;
      db.ss = nullptr;
      Epi ed = epi_resid(h, wnext, xa);
      if (li + 1 < layers.size())
        lookahead(ed, layers[li + 1].qkv);
      else if (has_head)
        lookahead(ed, head);
      if (linked) {
        ed.wait = ctr(li, LL.down);
        ed.wait_target = sg ? 32 : 8;  // gate|up units (16 outputs) or row groups (64 outputs) per chunk
        ed.sig = ctr(li, LL.next);
        ed.sig_div = 4;
        ed.done = ctr(li, LL.down_done);
      }
      CLM_TRY(gemv(L.down, q, db, ed, st, linked));
    }
    return CLM_OK;
  }
  // A linked GEMV whose input is a residual phase's preparation (4 row groups per chunk) with the folded rmsnorm:
  // chunk counters at layer li's offset `chunks`, the phase's finished groups at `done`.
  void link_in(Epi& e, size_t li, int chunks, int per_chunk, int done, int done_target) const {
    e.wait = link_ctr + li * link_layout().per_layer + chunks;
    e.wait_target = per_chunk;
    e.ss_done = link_ctr + li * link_layout().per_layer + done;
    e.ss_target = done_target;
  }

  // ---- the layers (+ head) of a window as phases of the dataflow kernel: the same chain as enqueue_layers
  FlowGemv flow_gemv(const Gemv& g, int nt, const XBuf& in, const Epi& epi, int kind) const {
    FlowGemv m;
    m.tiles = static_cast<const uint8_t*>(g.m->data);
    m.rows = g.m->shape.rows;
    m.ng = (int)g.m->shape.ng;
    m.geo = g4_geom(g.m->shape, nt);
    m.maxseg = g.plan[nt - 1].ksplit;
    m.in = in;
    m.epi = epi;
    m.epi_kind = epi.kind;
    m.part = flow_part[kind];
    m.counters = flow_gcount[kind];
    return m;
  }

  // Readiness counters of one window (offsets into flow_ctr): per layer the 512-column chunks of the QKV, W_o,
  // gate|up and down inputs, the kv heads of the attention, and the finished-row-group counts of W_o and down;
  // then the head's input chunks.
  struct FlowCtr {
    int per_layer = 0, qkv = 0, attn = 0, o = 0, gu = 0, down = 0, done_o = 0, done_down = 0, head = 0;
  };
  FlowCtr flow_ctr_layout() const {
    FlowCtr c;
    c.qkv = 0;
    c.attn = c.qkv + d.H / 512;
    c.o = c.attn + d.nkv;
    c.gu = c.o + d.qd() / 512;
    c.down = c.gu + d.H / 512;
    c.done_o = c.down + d.F / 512;
    c.done_down = c.done_o + 1;
    c.per_layer = c.done_down + 1;
    c.head = (int)layers.size() * c.per_layer;
    return c;
  }
  bool flow_shape_ok() const {
    return d.hd == 128 && d.H % 512 == 0 && d.F % 512 == 0 && d.qd() % 512 == 0 && !layers.empty();
  }

  int enqueue_window_flow(Session& s, int q, cudaStream_t st) {
    const int nt = q <= 8 ? 1 : 2;
    auto it = s.flow_phases.find(q);
    FlowPhase* d_ph = nullptr;
    const int nph = (int)layers.size() * 5 + (has_head ? 1 : 0);
    if (it != s.flow_phases.end()) {
      d_ph = it->second;
    } else {
      const FlowCtr C = flow_ctr_layout();
      std::vector<FlowPhase> ph;
      const long long* pos = &s.d_state->pos;
      const int group = d.nh / d.nkv;
      const int mtiles = (q * group + 15) / 16;
      const int ng_h = d.H / 128;  // row groups of a residual GEMV (W_o, down)
      for (size_t li = 0; li < layers.size(); ++li) {
        const Layer& L = layers[li];
        int* lc = flow_ctr + li * C.per_layer;
        Epi ek = epi_base(EPI_ROPE_KV);
        ek.nh = d.nh;
        ek.nkv = d.nkv;
        ek.hd = d.hd;
        ek.rope = rope;
        ek.pos = pos;
        ek.pages = s.d_pages;
        ek.kpool = kpool[li];
        ek.vpool = vpool[li];
        ek.q16 = q16;
        FlowPhase p0;
        p0.kind = FLOW_GEMV;
        p0.g = flow_gemv(L.qkv, nt, xa, ek, FK_QKV);
        if (li > 0) {
          p0.wait = lc + C.qkv;
          p0.wait_target = 4;
          p0.ss_done = lc - C.per_layer + C.done_down;
          p0.ss_target = ng_h;
        }
        p0.sig = lc + C.attn;
        p0.sig_qkv = 1;
        ph.push_back(p0);
        FlowPhase pa;
        pa.kind = FLOW_ATTN;
        pa.a.q16 = q16;
        pa.a.kpool = kpool[li];
        pa.a.vpool = vpool[li];
        pa.a.pages = s.d_pages;
        pa.a.nh = d.nh;
        pa.a.nkv = d.nkv;
        pa.a.mtiles = mtiles;
        pa.a.maxseg = flow_attn_maxseg;
        pa.a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)d.hd));
        pa.a.part = flow_attn_part;
        pa.a.counters = acount;
        pa.a.out = xb;
        pa.a.out.ss = nullptr;
        pa.a.hi_scale = hi_scale();
        pa.a.nt_out = nt;
        pa.wait = lc + C.attn;
        pa.wait_target = group + 2;
        pa.sig = lc + C.o;
        // a W_o unit reads 512 columns = 4 query heads: a kv head's outputs cover group / 4 chunks, or 4 / group kv
        // heads share one chunk
        pa.sig_span = group >= 4 ? group / 4 : 1;
        pa.sig_kvh_div = group >= 4 ? 1 : 4 / group;
        ph.push_back(pa);
        XBuf ob = xb;
        ob.ss = nullptr;
        FlowPhase po;
        po.kind = FLOW_GEMV;
        po.g = flow_gemv(L.o, nt, ob, epi_resid(h, L.ffn_norm, xa), FK_O);
        po.wait = lc + C.o;
        po.wait_target = mtiles * pa.sig_kvh_div;
        po.sig = lc + C.gu;
        po.sig_div = 4;
        po.done = lc + C.done_o;
        ph.push_back(po);
        Epi es = epi_base(EPI_SWIGLU_PREP);
        es.ffn = d.F;
        es.next = xb;
        FlowPhase pg;
        pg.kind = FLOW_GEMV;
        pg.g = flow_gemv(L.gu, nt, xa, es, FK_GU);
        pg.wait = lc + C.gu;
        pg.wait_target = 4;
        pg.ss_done = lc + C.done_o;
        pg.ss_target = ng_h;
        pg.sig = lc + C.down;
        pg.sig_div = 8;  // a gate|up row group gives 64 SwiGLU columns
        ph.push_back(pg);
        const float* wnext = li + 1 < layers.size() ? layers[li + 1].attn_norm : (has_head ? out_norm : ones_h);
        XBuf db = xb;
        db.ss = nullptr;
        FlowPhase pd;
        pd.kind = FLOW_GEMV;
        pd.g = flow_gemv(L.down, nt, db, epi_resid(h, wnext, xa), FK_DOWN);
        pd.wait = lc + C.down;
        pd.wait_target = 8;
        pd.sig = li + 1 < layers.size() ? lc + C.per_layer + C.qkv : (has_head ? flow_ctr + C.head : nullptr);
        pd.sig_div = 4;
        pd.done = lc + C.done_down;
        ph.push_back(pd);
      }
      if (has_head) {
        Epi eo = epi_base(EPI_STORE);
        eo.out = logits;
        eo.out_ld = d.V;
        FlowPhase pho;
        pho.kind = FLOW_GEMV;
        pho.g = flow_gemv(head, nt, xa, eo, FK_HEAD);
        pho.wait = flow_ctr + C.head;
        pho.wait_target = 4;
        pho.ss_done = flow_ctr + (layers.size() - 1) * C.per_layer + C.done_down;
        pho.ss_target = ng_h;
        ph.push_back(pho);
      }
      CLM_CHECK((int)ph.size() == nph, CLM_INTERNAL, "flow kernel phase count");
      CLM_CUDA(cudaMalloc(&d_ph, ph.size() * sizeof(FlowPhase)));
      CLM_CUDA(cudaMemcpy(d_ph, ph.data(), ph.size() * sizeof(FlowPhase), cudaMemcpyHostToDevice));
      s.flow_phases[q] = d_ph;
    }
    FlowParams P;
    P.phases = d_ph;
    P.nphases = nph;
    P.q = q;
    P.pos = &s.d_state->pos;
    P.err = bad;
    P.stages = flow_stage_count[nt - 1];
    P.stage_bytes = flow_stage_bytes[nt - 1];
    return launch_flow(P, d.quant, nt, flow_grid_n[nt - 1], flow_ctr, flow_ctr_n * sizeof(int), st);
  }

  // ---- one tensor-core GEMM of a wide window: y[p] = W . x[p] over the tiles in wxh.  `out` tells the next step
  // where the product is: y itself, or the K-split partials it sums (no separate reduction launch).
  int gemm_wide(const Gemv& g, int q, float* y, cudaStream_t st, WideIn* out = nullptr) {
    const TcPlan p = gemm_tc_plan(g.m->shape, q, ctx->sm_count);
    CLM_CHECK(p.ksplit == 1 || p.part_floats <= wpart_floats, CLM_INTERNAL, "wide window: split-K partials");
    const bool defer = out != nullptr && p.ksplit > 1;
    if (out != nullptr) {
      out->p = defer ? wpart : y;
      out->nsplit = defer ? p.ksplit : 1;
      out->stride = (unsigned long long)q * g.m->shape.rows;
    }
    return launch_gemm_tc_tiles(g.m->shape, p, static_cast<const uint8_t*>(g.m->data), wxh, q, y, wpart, bad, st,
                                !defer);
  }

  // ---- a wide window (17..256 rows: prefill chunks, large trees, or the windows of several sessions stacked):
  // per layer the QKV, W_o, gate|up and down GEMMs on tensor cores over all rows, each followed by its
  // elementwise step (RoPE + KV append, residual + rmsnorm, SwiGLU) that writes the next GEMM's fp16 tiles; the
  // RoPE/KV step and the attention run per session segment (its own position, pages and cache rows)
  struct WideSeg {
    Session* s;
    int row0, q;
  };
  int enqueue_window_wide(Session& s, int q, const int32_t* d_tok, const int32_t* parent, cudaStream_t st) {
    const WideSeg seg{&s, 0, q};
    return enqueue_window_wide(&seg, 1, q, d_tok, parent, st);
  }
  int enqueue_window_wide(const WideSeg* segs, int nseg, int q, const int32_t* d_tok, const int32_t* parent,
                          cudaStream_t st) {
    const int P = (q + 15) / 16 * 16;
    const size_t qkv_rows = (size_t)d.qd() + 2 * d.kvd();
    CLM_CHECK(nseg >= 1 && nseg <= kWideAttnMaxSegs, CLM_OUT_OF_RANGE, "wide window: at most 16 sessions");
    AttnSegs attn_segs{};
    for (int k = 0; k < nseg; ++k) {
      CLM_CHECK(segs[k].q == segs[0].q && segs[k].row0 == k * segs[0].q, CLM_INTERNAL, "wide window: segment rows");
      attn_segs.pos[k] = &segs[k].s->d_state->pos;
      attn_segs.pages[k] = segs[k].s->d_pages;
      attn_segs.row0[k] = segs[k].row0;
    }
    if (has_tokens) {
      CLM_TRY(launch_pdl(embed_guard_kernel, dim3(1), dim3(256), 0, st, d_tok, q, (int)d.V, tokens, bad));
      CLM_TRY(launch_embed(embd, d.quant, tokens, q, d.H, h, st));
    } else {
      CLM_TRY(launch_unpack_boundary(bin, q, d.H, h, st));
    }
    const float* w0 = layers.empty() ? (has_head ? out_norm : ones_h) : layers[0].attn_norm;
    CLM_TRY(launch_wide_norm_prep(WideIn{}, h, q, d.H, w0, d.eps, P, wxh, st));
    for (size_t li = 0; li < layers.size(); ++li) {
      const Layer& L = layers[li];
      WideIn y;
      CLM_TRY(gemm_wide(L.qkv, q, wy, st, &y));
      for (int k = 0; k < nseg; ++k) {
        const WideSeg& g = segs[k];
        const long long* pos = &g.s->d_state->pos;
        __half* qs = q16 + (size_t)g.row0 * d.qd();
        WideIn ys = y;
        ys.p += (size_t)g.row0 * qkv_rows;
        CLM_TRY(launch_wide_rope_kv(ys, g.q, d, rope, pos, g.s->d_pages, parent, qs, kpool[li], vpool[li], st));
      }
      // one attention launch over every segment (all segments have segs[0].q rows)
      CLM_TRY(launch_attention_wide(q16, kpool[li], vpool[li], attn_segs, nseg, parent, segs[0].q, d, max_pages,
                                    wattn_part, wattn_part_floats, wattn_cnt, wattn_tiles, ctx->sm_count, wattn, bad,
                                    st));
      CLM_TRY(launch_tc_xprep(wattn, q, d.qd(), P, wxh, st));
      CLM_TRY(gemm_wide(L.o, q, wy, st, &y));
      CLM_TRY(launch_wide_norm_prep(y, h, q, d.H, L.ffn_norm, d.eps, P, wxh, st));
      CLM_TRY(gemm_wide(L.gu, q, wy, st, &y));
      CLM_TRY(launch_wide_swiglu_prep(y, q, d.F, P, wxh, st));
      CLM_TRY(gemm_wide(L.down, q, wy, st, &y));
      const float* wnext = li + 1 < layers.size() ? layers[li + 1].attn_norm : (has_head ? out_norm : ones_h);
      CLM_TRY(launch_wide_norm_prep(y, h, q, d.H, wnext, d.eps, P, wxh, st));
    }
    if (has_head) return gemm_wide(head, q, logits, st);
    return launch_pack_boundary(h, nullptr, 0, q, d.H, bout, st);
  }

  // ---- one window over several sessions on the q-row GEMV chain (n sessions x qs <= 32 rows, linear windows): every
  // matrix streams once for all rows (the 4-n-tile GEMV), the QKV epilogue places each row's K / V at its own
  // session's position, and the attention runs once per session into that session's rows of W_o's input
  int enqueue_batch_chain(const WideSeg* segs, int nseg, int Q, const int32_t* d_tok, cudaStream_t st) {
    const int qs = segs[0].q;
    CLM_CHECK(nseg >= 1 && nseg <= 4 && Q == nseg * qs && Q <= 32, CLM_OUT_OF_RANGE,
              "batched GEMV window: at most 4 sessions and 32 rows");
    const int nt = Q <= 8 ? 1 : (Q <= 16 ? 2 : 4);
    if (has_tokens) {
      CLM_TRY(launch_pdl(embed_guard_kernel, dim3(1), dim3(64), 0, st, d_tok, Q, (int)d.V, tokens, bad));
      CLM_TRY(launch_embed(embd, d.quant, tokens, Q, d.H, h, st));
    } else {
      CLM_TRY(launch_unpack_boundary(bin, Q, d.H, h, st));
    }
    const float* w0 = layers.empty() ? (has_head ? out_norm : ones_h) : layers[0].attn_norm;
    CLM_TRY(launch_prep_rows(h, d.H, Q, d.H, w0, nt, hi_scale(), xa, true, st));
    for (size_t li = 0; li < layers.size(); ++li) {
      Layer& L = layers[li];
      Epi ek = epi_base(EPI_ROPE_KV);
      ek.nh = d.nh;
      ek.nkv = d.nkv;
      ek.hd = d.hd;
      ek.rope = rope;
      ek.kpool = kpool[li];
      ek.vpool = vpool[li];
      ek.q16 = q16;
      ek.seg_q = qs;
      for (int k = 0; k < nseg; ++k) {
        ek.seg_pos[k] = &segs[k].s->d_state->pos;
        ek.seg_pages[k] = segs[k].s->d_pages;
      }
      CLM_TRY(gemv(L.qkv, Q, xa, ek, st));
      for (int k = 0; k < nseg; ++k)
        CLM_TRY(launch_attention(q16 + (size_t)segs[k].row0 * d.qd(), kpool[li], vpool[li], segs[k].s->d_pages,
                                 &segs[k].s->d_state->pos, nullptr, qs, d, max_pages, attn_part, acount, nt, hi_scale(),
                                 xb.frag, xb.sum, bad, k + 1 == nseg ? static_cast<const uint8_t*>(L.o.m->data) : nullptr,
                                 L.o.m->shape.bytes(), ctx->sm_count, st, nullptr, AttnLink{}, segs[k].row0, Q));
      XBuf ob = xb;
      ob.ss = nullptr;
      Epi eo = epi_resid(h, L.ffn_norm, xa);
      lookahead(eo, L.gu);
      CLM_TRY(gemv(L.o, Q, ob, eo, st));
      Epi es = epi_base(EPI_SWIGLU_PREP);
      es.ffn = d.F;
      es.next = xb;
      lookahead(es, L.down);
      CLM_TRY(gemv(L.gu, Q, xa, es, st));
      const float* wnext = li + 1 < layers.size() ? layers[li + 1].attn_norm : (has_head ? out_norm : ones_h);
      XBuf db = xb;
      db.ss = nullptr;
      Epi ed = epi_resid(h, wnext, xa);
      if (li + 1 < layers.size())
        lookahead(ed, layers[li + 1].qkv);
      else if (has_head)
        lookahead(ed, head);
      CLM_TRY(gemv(L.down, Q, db, ed, st));
    }
    if (has_head) {
      Epi eo = epi_base(EPI_STORE);
      eo.out = logits;
      eo.out_ld = d.V;
      return gemv(head, Q, xa, eo, st);
    }
    return launch_pack_boundary(h, nullptr, 0, Q, d.H, bout, st);
  }

  // ---- a full window: input (tokens or records) -> layers -> logits or records
  int enqueue_window(Session& s, int q, const int32_t* d_tok, cudaStream_t st, const int32_t* parent = nullptr) {
    if (q > 16) return enqueue_window_wide(s, q, d_tok, parent, st);
    const int nt = q <= 8 ? 1 : 2;
    if (has_tokens) {
      CLM_TRY(launch_pdl(embed_guard_kernel, dim3(1), dim3(64), 0, st, d_tok, q, (int)d.V, tokens, bad));
      CLM_TRY(launch_embed(embd, d.quant, tokens, q, d.H, h, st));
    } else {
      CLM_TRY(launch_unpack_boundary(bin, q, d.H, h, st));
    }
    const float* w0 = layers.empty() ? (has_head ? out_norm : ones_h) : layers[0].attn_norm;
    if (link_ok && !layers.empty())
      CLM_TRY(launch_pdl(zero_ints_kernel, dim3((unsigned)ceil_div(link_n, 256)), dim3(256), 0, st, link_ctr, link_n));
    CLM_TRY(launch_prep_rows(h, d.H, q, d.H, w0, nt, hi_scale(), xa, true, st));
    if (flow_grid_n[nt - 1] > 0 && parent == nullptr) {
      // layers (and the head) in one cooperative launch
      CLM_TRY(enqueue_window_flow(s, q, st));
      if (!has_head) CLM_TRY(launch_pack_boundary(h, nullptr, 0, q, d.H, bout, st));
      return CLM_OK;
    }
    CLM_TRY(enqueue_layers(s, q, parent, st));
    if (has_head) {
      Epi eo = epi_base(EPI_STORE);
      eo.out = logits;
      eo.out_ld = d.V;
      if (link_ok && !layers.empty())
        link_in(eo, layers.size() - 1, link_layout().next, 4, link_layout().down_done, d.H / 128);
      CLM_TRY(gemv(head, q, xa, eo, st));
    } else {
      CLM_TRY(launch_pack_boundary(h, nullptr, 0, q, d.H, bout, st));
    }
    return CLM_OK;
  }

  // ---- one MTP step: prev token (device) -> draft logits row
  int enqueue_mtp_step(const int32_t* d_prev, float* d_logits_row, cudaStream_t st) {
    CLM_TRY(launch_embed(embd, d.quant, d_prev, 1, d.H, h_mtp, st));
    CLM_TRY(launch_prep_rows(h_mtp, d.H, 1, d.H, mtp_ffn_norm, 1, hi_scale(), xa, true, st));
    Epi es = epi_base(EPI_SWIGLU_PREP);
    es.ffn = d.F;
    es.next = xb;
    CLM_TRY(gemv(mtp_gu, 1, xa, es, st));
    XBuf db = xb;
    db.ss = nullptr;
    CLM_TRY(gemv(mtp_down, 1, db, epi_resid(h_mtp, mtp_out_norm, xa), st));
    Epi eo = epi_base(EPI_STORE);
    eo.out = d_logits_row;
    eo.out_ld = d.V;
    CLM_TRY(gemv(head, 1, xa, eo, st));
    return CLM_OK;
  }

  // ---- one speculative round on a WHOLE engine
  // Temperature and seed are read from `ctl` (device); `stochastic` selects the acceptance kernels.
  int enqueue_round(Session& s, int q, bool stochastic, cudaStream_t st) {
    CLM_TRY(enqueue_drafts(s, q, stochastic, win, dprobs, st));
    CLM_TRY(enqueue_window(s, q, win, st));
    return enqueue_accept(s, q, stochastic, win, dprobs, st);
  }

  // The window's tokens: w[0] = the session's next token, w[1..q-1] = MTP drafts chained from it (greedy, or
  // sampled with Philox draws (draw j, stream 1, session round) from distribution rows kept in dp[j]).
  int enqueue_drafts(Session& s, int q, bool stochastic, int32_t* w, float* dp, cudaStream_t st) {
    const unsigned long long* ctr = &s.d_state->round;
    CLM_TRY(launch_pdl(round_head_kernel, dim3(1), dim3(32), 0, st, (const SessionState*)s.d_state, w));
    for (int j = 0; j + 1 < q; ++j) {
      CLM_TRY(enqueue_mtp_step(w + j, draft_logits + (size_t)j * d.V, st));
      CLM_TRY(sample_token(draft_logits + (size_t)j * d.V, stochastic, 1.0f, 0, (uint32_t)j, 1u, ctr, ctl,
                           dp + (size_t)j * d.V, w + j + 1, st));
    }
    return CLM_OK;
  }

  // Acceptance of the window w (logits in `logits`, draft distributions dp) and the round's commit.
  int enqueue_accept(Session& s, int q, bool stochastic, const int32_t* w, const float* dp, cudaStream_t st) {
    const unsigned long long* ctr = &s.d_state->round;
    if (stochastic) {
      // the window's distributions are evaluated from its logits where acceptance reads them
      CLM_TRY(launch_row_stats(logits, q, d.V, 1.0f, ctl, 0, samp, st));
      AcceptRows src;
      src.LP = logits;
      src.Q = q > 1 ? dp : nullptr;
      CLM_TRY(launch_accept(src, w + 1, 1, q - 1, d.V, nullptr, 0, 0, ctr, ctl, acc, nxt, samp, st));
    } else {
      CLM_TRY(launch_argmax_rows(logits, q, d.V, am, samp, st));
      CLM_TRY(launch_pdl(greedy_decide_kernel, dim3(1), dim3(32), 0, st, (const int32_t*)am, q, w, acc, nxt));
    }
    return launch_pdl(round_commit_kernel, dim3(1), dim3(32), 0, st, s.d_state, w, (const uint32_t*)acc,
                      (const int32_t*)nxt, emitted, count);
  }

  // ---- stage pipeline (clm_b200_pipe_*)
  uint32_t record_bytes(int q) const { return (uint32_t)(((size_t)q * floats_per_position() * 4 + 15) / 16 * 16); }
  static uint32_t token_bytes(int q) { return (uint32_t)((q * 4 + 15) / 16 * 16); }

  // The links of session s's messages: its own (clm_b200_pipe_attach_session) or the engine's.
  const LinkDev& link_in(const Session& s) const { return s.own_links ? s.lin : lin; }
  const LinkDev& link_out(const Session& s) const { return s.own_links ? s.lout : lout; }

  // One round of session s on this stage (see clm_b200_pipe_round).
  int enqueue_pipe_round(Session& s, int q, bool stochastic, cudaStream_t st) {
    long long* pos = &s.d_state->pos;
    unsigned* cin = &s.d_state->commit_in;
    const LinkDev &li = link_in(s), &lo = link_out(s);
    if (spec.role == CLM_ROLE_PREFIX) {
      CLM_TRY(launch_link_recv(li, win, (uint32_t)((wmax() + 1) * 4), (uint32_t)q, pos, cin, bad, st));
    } else {
      // the tail committed its own previous round at acceptance
      CLM_TRY(launch_link_recv(li, bin, record_bytes(wmax()), (uint32_t)q,
                               spec.role == CLM_ROLE_TAIL ? nullptr : pos, cin, bad, st));
    }
    if (spec.role != CLM_ROLE_TAIL) {
      CLM_TRY(enqueue_window(s, q, win, st));
      return launch_link_send(lo, bout, record_bytes(q), cin, (uint32_t)q, LINK_MSG_WINDOW, bad, st);
    }
    CLM_TRY(enqueue_window(s, q, s.d_win, st));
    CLM_TRY(enqueue_accept(s, q, stochastic, s.d_win, s.d_dprobs, st));
    CLM_TRY(enqueue_drafts(s, q, stochastic, s.d_win, s.d_dprobs, st));
    return launch_link_send(lo, s.d_win, token_bytes(q), count, (uint32_t)q, LINK_MSG_WINDOW, bad, st);
  }

  // One prompt chunk of session s on this stage, committed at once (the prefix's tokens are already in win).
  int enqueue_pipe_prefill(Session& s, int q, cudaStream_t st) {
    if (spec.role != CLM_ROLE_PREFIX)
      CLM_TRY(launch_link_recv(link_in(s), bin, record_bytes(wmax()), (uint32_t)q, nullptr, nullptr, bad, st));
    CLM_TRY(enqueue_window(s, q, win, st));
    if (spec.role != CLM_ROLE_TAIL)
      CLM_TRY(launch_link_send(link_out(s), bout, record_bytes(q), nullptr, (uint32_t)q, LINK_MSG_PREFILL, bad, st));
    return launch_pdl(pos_advance_kernel, dim3(1), dim3(32), 0, st, s.d_state, q);
  }

  // One token from one logits row: argmax, or sample_from(distribution(row, T)) with the Philox uniform
  // (draw, stream, *ctr) under the seed (ctl's when given); the distribution row goes to probs_row.
  int sample_token(const float* row, bool stochastic, float T, uint64_t seed, uint32_t draw, uint32_t stream,
                   const unsigned long long* ctr, const RoundCtl* rctl, float* probs_row, int32_t* out,
                   cudaStream_t st) {
    if (!stochastic) return launch_argmax_rows(row, 1, d.V, out, samp, st);
    CLM_TRY(launch_probs(row, 1, d.V, T, rctl, probs_row, samp, st));
    return launch_sample_rows(probs_row, 1, d.V, d.V, nullptr, seed, draw, stream, ctr, rctl, out, samp, st);
  }

  // Runs `enq` for (kind, q, flag) as a CUDA graph: eager on first use, captured on the second, replayed after.
  template <typename F>
  int run_graph(Session& s, int kind, int q, int flag, cudaStream_t st, F&& enq) {
    const auto key = std::make_tuple(kind, q, flag);
    auto it = s.graphs.find(key);
    if (it != s.graphs.end()) {
      CLM_CUDA(cudaGraphLaunch(it->second, st));
      last_launches = s.launches[key];
      return CLM_OK;
    }
    const unsigned long long l0 = t_kernel_launches;
    if (s.seen[key]++ == 0) {
      const int rc0 = enq(st);
      last_launches = t_kernel_launches - l0;
      return rc0;
    }
    cudaGraph_t g = nullptr;
    CLM_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    const int rc = enq(st);
    s.launches[key] = t_kernel_launches - l0;
    last_launches = s.launches[key];
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc != CLM_OK) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    s.graphs[key] = ex;
    CLM_CUDA(cudaGraphLaunch(ex, st));
    return CLM_OK;
  }

  // Zeroes every arrival counter of the split reductions.  A reduction resets its counter only after a wait that
  // succeeded, so after a bounded wait gave up the counters may hold arrivals of the failed launch; without this a
  // later window (or graph replay) would pass its waits early and sum stale partials.  The stream is idle here.
  int reset_counters() {
    if (gcount) CLM_CUDA(cudaMemset(gcount, 0, gcount_n * sizeof(int)));
    if (gcount2) CLM_CUDA(cudaMemset(gcount2, 0, gcount_n * sizeof(int)));
    if (link_ctr) CLM_CUDA(cudaMemset(link_ctr, 0, (size_t)link_n * sizeof(int)));
    if (acount) CLM_CUDA(cudaMemset(acount, 0, acount_n * sizeof(int)));
    if (wattn_cnt) CLM_CUDA(cudaMemset(wattn_cnt, 0, (size_t)wattn_tiles * sizeof(int)));
    if (samp_counters) CLM_CUDA(cudaMemset(samp_counters, 0, samp_counter_bytes));
    for (int k = 0; k < FK_KINDS; ++k)
      if (flow_gcount[k]) CLM_CUDA(cudaMemset(flow_gcount[k], 0, flow_gcount_n[k] * sizeof(int)));
    return CLM_OK;
  }

  int check_bad(cudaStream_t st) {
    int b = 0;
    CLM_CUDA(cudaMemcpyAsync(&b, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
    CLM_CUDA(cudaStreamSynchronize(st));
    if (b) {
      CLM_CUDA(cudaMemset(bad, 0, sizeof(int)));
      CLM_TRY(reset_counters());
      if (b == kErrWaitTimeout) return fail(CLM_DEADLINE_EXCEEDED, "a bounded device wait gave up (copy never completed)");
      if (b == kErrPartialSlots) return fail(CLM_INTERNAL, "a split reduction needed more partial slots than planned");
      if (b == kErrLinkTimeout)
        return fail(CLM_DEADLINE_EXCEEDED, "a stage link wait gave up (the peer stage stopped or fell behind)");
      if (b == kErrLinkMismatch) return fail(CLM_VERSION_MISMATCH, "a stage link message has another window width");
      if (b == kErrBadTree)
        return fail(CLM_INVALID_ARGUMENT, "tree window: parent[i] must be -1 or an earlier node");
      return fail(CLM_INVALID_ARGUMENT, "token outside the vocabulary");
    }
    return CLM_OK;
  }

  void release_session(Session& s) {
    for (auto& kv : s.graphs) cudaGraphExecDestroy(kv.second);
    s.graphs.clear();
    for (auto& kv : s.flow_phases) cudaFree(kv.second);
    s.flow_phases.clear();
    if (s.d_pages) cudaFree(s.d_pages);
    if (s.d_state) cudaFree(s.d_state);
    if (s.d_win) cudaFree(s.d_win);
    if (s.d_dprobs) cudaFree(s.d_dprobs);
    s.d_win = nullptr;
    s.d_dprobs = nullptr;
    for (int32_t p : s.pages) free_pages.push_back(p);
    s.pages.clear();
    s.d_pages = nullptr;
    s.d_state = nullptr;
  }

  void drop_batch_graphs() {
    for (auto& kv : batch_graphs) release_session(*kv.second);
    batch_graphs.clear();
  }

  ~LlamaEngine() override {
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    drop_batch_graphs();
    for (auto& kv : sessions) release_session(*kv.second);
    sessions.clear();
    auto free_m = [](Gemv& g) {
      if (g.m) clm_b200_matrix_free(g.m);
      g.m = nullptr;
    };
    for (auto& L : layers) {
      free_m(L.qkv);
      free_m(L.o);
      free_m(L.gu);
      free_m(L.down);
    }
    free_m(head);
    free_m(mtp_gu);
    free_m(mtp_down);
    for (void* p : allocations) cudaFree(p);
    if (pin_in) cudaFreeHost(pin_in);
    if (pin_out) cudaFreeHost(pin_out);
  }
};

namespace {

int engine_enter(LlamaEngine* e) {
  CLM_CHECK(e != nullptr, CLM_INVALID_ARGUMENT, "null engine");
  return ctx_enter(e->ctx);
}

Session* find_session(LlamaEngine* e, uint64_t id) {
  auto it = e->sessions.find(id);
  return it == e->sessions.end() ? nullptr : it->second.get();
}

}  // namespace

namespace clm {

LlamaEngine* as_llama(clm_b200_engine* e) { return static_cast<LlamaEngine*>(e); }

int llama_create(clm_b200_ctx* ctx, const clm_b200_llama_geometry* g, const clm_b200_stage_spec* spec,
                          clm_b200_engine** out) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(g && spec && out, CLM_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  CLM_CHECK(g->n_layers > 0 && g->hidden > 0 && g->n_heads > 0 && g->n_kv_heads > 0 && g->vocab > 0 && g->ffn > 0,
            CLM_INVALID_ARGUMENT, "geometry has a zero dimension");
  CLM_CHECK(g->n_heads % g->n_kv_heads == 0, CLM_INVALID_ARGUMENT, "n_heads must be a multiple of n_kv_heads");
  CLM_CHECK(g->head_dim == 128, CLM_UNIMPLEMENTED, "head_dim must be 128");
  CLM_CHECK(g->quant == CLM_QUANT_Q4_K || g->quant == CLM_QUANT_Q8_0, CLM_INVALID_ARGUMENT, "quant must be Q4_K or Q8_0");
  CLM_CHECK(g->hidden % 256 == 0 && g->ffn % 256 == 0 && (g->n_heads * g->head_dim) % 256 == 0, CLM_INVALID_ARGUMENT,
            "hidden, ffn and n_heads*head_dim must be multiples of 256");
  CLM_CHECK(g->vocab % 16 == 0 && (g->n_kv_heads * g->head_dim) % 16 == 0, CLM_INVALID_ARGUMENT,
            "vocab and kv width must be multiples of 16");
  CLM_CHECK(spec->layer_end <= g->n_layers && spec->layer_begin <= spec->layer_end, CLM_INVALID_ARGUMENT,
            "layer range outside the model");
  CLM_CHECK(spec->role >= CLM_ROLE_PREFIX && spec->role <= CLM_ROLE_WHOLE, CLM_INVALID_ARGUMENT, "unknown role");
  CLM_CHECK(spec->max_context > 0 && spec->max_window > 0 && spec->max_sessions > 0 &&
                spec->max_window <= spec->max_context,
            CLM_INVALID_ARGUMENT, "domain spec needs max_context >= max_window >= 1 and max_sessions >= 1");
  CLM_CHECK(spec->max_window <= 256, CLM_OUT_OF_RANGE, "max_window must be <= 256");
  if (spec->role == CLM_ROLE_PREFIX || spec->role == CLM_ROLE_WHOLE)
    CLM_CHECK(spec->layer_begin == 0, CLM_INVALID_ARGUMENT, "prefix domain must start at layer 0");
  if (spec->role == CLM_ROLE_TAIL || spec->role == CLM_ROLE_WHOLE)
    CLM_CHECK(spec->layer_end == g->n_layers, CLM_INVALID_ARGUMENT, "tail domain must end at the last layer");
  if (spec->role == CLM_ROLE_MIDDLE)
    CLM_CHECK(spec->layer_end > spec->layer_begin, CLM_INVALID_ARGUMENT, "middle domain needs at least one layer");
  auto* e = new LlamaEngine();
  e->ctx = ctx;
  ctx_retain(ctx);
  e->family = CLM_FAMILY_LLAMA;
  e->geo = *g;
  e->spec = *spec;
  e->d.H = (int)g->hidden;
  e->d.nh = (int)g->n_heads;
  e->d.nkv = (int)g->n_kv_heads;
  e->d.hd = (int)g->head_dim;
  e->d.F = (int)g->ffn;
  e->d.V = (int)g->vocab;
  e->d.theta = g->rope_theta;
  e->d.eps = g->rms_eps;
  e->d.quant = g->quant;
  e->has_tokens = spec->role == CLM_ROLE_PREFIX || spec->role == CLM_ROLE_WHOLE;
  e->has_head = spec->role == CLM_ROLE_TAIL || spec->role == CLM_ROLE_WHOLE;
  e->has_mtp = e->has_head && g->mtp != 0;
  e->has_embd = e->has_tokens || e->has_mtp;
  e->max_pages = (int)ceil_div(spec->max_context, kPageTokens);
  *out = e;
  return CLM_OK;
}


int llama_generate_weights(LlamaEngine* e, uint64_t seed, float stddev) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(!e->weights_ready, CLM_FAILED_PRECONDITION, "weights already bound");
  const LlamaDims& d = e->d;
  cudaStream_t st = e->ctx->stream;
  auto tbytes = [&](uint64_t n) { return clm_b200_tensor_bytes(d.quant, n); };
  uint64_t biggest = std::max<uint64_t>(tbytes((uint64_t)(d.qd() + 2 * d.kvd()) * d.H), tbytes((uint64_t)2 * d.F * d.H));
  biggest = std::max<uint64_t>(biggest, tbytes((uint64_t)d.H * d.F));
  if (e->has_head || e->has_embd) biggest = std::max<uint64_t>(biggest, tbytes((uint64_t)d.V * d.H));
  uint8_t* tmp = nullptr;
  CLM_CUDA(cudaMalloc(&tmp, biggest));
  int rc = CLM_OK;
  auto gen = [&](uint32_t id, uint64_t n, uint8_t* dst) { return launch_gen_encode(d.quant, seed, id, n, stddev, dst, st); };
  do {
    for (uint32_t L = e->spec.layer_begin; L < e->spec.layer_end && rc == CLM_OK; ++L) {
      LlamaEngine::Layer lay;
      const uint64_t H = d.H, qd = d.qd(), kvd = d.kvd(), F = d.F;
      const uint32_t id = 16 * L;
      if ((rc = gen(id + 0, qd * H, tmp)) || (rc = gen(id + 1, kvd * H, tmp + tbytes(qd * H))) ||
          (rc = gen(id + 2, kvd * H, tmp + tbytes((qd + kvd) * H))))
        break;
      if ((rc = e->make_gemv(lay.qkv, tmp, tbytes((qd + 2 * kvd) * H), (uint32_t)(qd + 2 * kvd), (uint32_t)H))) break;
      if ((rc = gen(id + 3, H * qd, tmp)) || (rc = e->make_gemv(lay.o, tmp, tbytes(H * qd), (uint32_t)H, (uint32_t)qd)))
        break;
      if ((rc = gen(id + 4, F * H, tmp)) || (rc = gen(id + 5, F * H, tmp + tbytes(F * H))) ||
          (rc = e->make_gemv(lay.gu, tmp, tbytes(2 * F * H), (uint32_t)(2 * F), (uint32_t)H, (uint32_t)F)))
        break;
      if ((rc = gen(id + 6, H * F, tmp)) || (rc = e->make_gemv(lay.down, tmp, tbytes(H * F), (uint32_t)H, (uint32_t)F)))
        break;
      if ((rc = e->ones(&lay.attn_norm, H)) || (rc = e->ones(&lay.ffn_norm, H))) break;
      e->layers.push_back(lay);
    }
    if (rc) break;
    const uint64_t VH = (uint64_t)d.V * d.H;
    if (e->has_embd) {
      e->embd_bytes = tbytes(VH);
      if ((rc = e->alloc((void**)&e->embd, e->embd_bytes)) || (rc = gen(1000, VH, e->embd))) break;
      e->weight_bytes += e->embd_bytes;
    }
    if (e->has_head) {
      if ((rc = gen(1001, VH, tmp)) || (rc = e->make_gemv(e->head, tmp, tbytes(VH), (uint32_t)d.V, (uint32_t)d.H))) break;
      if ((rc = e->ones(&e->out_norm, d.H))) break;
    }
    if (e->has_mtp) {
      const uint64_t FH = (uint64_t)d.F * d.H;
      if ((rc = gen(1002, FH, tmp)) || (rc = gen(1003, FH, tmp + tbytes(FH))) ||
          (rc = e->make_gemv(e->mtp_gu, tmp, tbytes(2 * FH), (uint32_t)(2 * d.F), (uint32_t)d.H, (uint32_t)d.F)))
        break;
      if ((rc = gen(1004, FH, tmp)) || (rc = e->make_gemv(e->mtp_down, tmp, tbytes(FH), (uint32_t)d.H, (uint32_t)d.F)))
        break;
      if ((rc = e->ones(&e->mtp_ffn_norm, d.H)) || (rc = e->ones(&e->mtp_out_norm, d.H))) break;
    }
  } while (false);
  cudaStreamSynchronize(st);
  cudaFree(tmp);
  if (rc == CLM_OK) e->weights_ready = true;
  return rc;
}

// Binds this stage's weights from named host tensors in GGUF naming and block layout (llama.cpp's tensor names:
// token_embd, blk.L.{attn_q,attn_k,attn_v,attn_output,ffn_gate,ffn_up,ffn_down,attn_norm,ffn_norm}, output_norm,
// output, each with the ".weight" suffix; the MTP head as mtp.{ffn_gate,ffn_up,ffn_down,ffn_norm,output_norm}).
// Matrices are in the engine's quantisation, norms f32; the same matrices are built as by llama_generate_weights.
int llama_load_tensors(LlamaEngine* e, const clm_b200_tensor* t, uint32_t n) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(!e->weights_ready, CLM_FAILED_PRECONDITION, "weights already bound");
  CLM_CHECK(t != nullptr || n == 0, CLM_INVALID_ARGUMENT, "null tensor list");
  const LlamaDims& d = e->d;
  cudaStream_t st = e->ctx->stream;
  std::map<std::string, const clm_b200_tensor*> by;
  for (uint32_t i = 0; i < n; ++i) {
    CLM_CHECK(t[i].name != nullptr && (t[i].data != nullptr || t[i].bytes == 0), CLM_INVALID_ARGUMENT,
              "tensor without a name or data");
    by[t[i].name] = &t[i];
  }
  auto tbytes = [&](uint64_t m) { return clm_b200_tensor_bytes(d.quant, m); };
  // one required tensor of `elems` elements in the engine's quantisation (f32 when `norm`)
  auto find = [&](const std::string& name, uint64_t elems, bool norm, const clm_b200_tensor** out) -> int {
    auto it = by.find(name);
    if (it == by.end()) return fail(CLM_NOT_FOUND, ("tensor missing: " + name).c_str());
    const clm_b200_tensor* x = it->second;
    const int want = norm ? CLM_QUANT_F32 : d.quant;
    if (x->quant < 0)  // a ggml type without a CLM representation (ggml type -1 - quant), e.g. Q6_K
      return fail(CLM_UNIMPLEMENTED, ("tensor " + name + " is in ggml type " + std::to_string(-1 - x->quant) +
                                      ", which the engine does not bind (Q4_K, Q8_0 matrices; f32 norms)")
                                         .c_str());
    if (x->quant != want)
      return fail(CLM_UNIMPLEMENTED, ("tensor " + name + " is not in the engine's quantisation (norms: f32)").c_str());
    const uint64_t want_bytes = norm ? elems * 4 : tbytes(elems);
    if (x->bytes != want_bytes) return fail(CLM_DATA_LOSS, ("tensor " + name + " has the wrong size").c_str());
    *out = x;
    return CLM_OK;
  };
  uint64_t biggest = std::max<uint64_t>(tbytes((uint64_t)(d.qd() + 2 * d.kvd()) * d.H), tbytes((uint64_t)2 * d.F * d.H));
  biggest = std::max<uint64_t>(biggest, tbytes((uint64_t)d.H * d.F));
  if (e->has_head) biggest = std::max<uint64_t>(biggest, tbytes((uint64_t)d.V * d.H));
  uint8_t* tmp = nullptr;
  CLM_CUDA(cudaMalloc(&tmp, biggest));
  int rc = CLM_OK;
  // host bytes of tensors `parts` one after another into tmp
  auto stage = [&](std::initializer_list<const clm_b200_tensor*> parts) -> int {
    uint64_t off = 0;
    for (const clm_b200_tensor* x : parts) {
      const cudaError_t err = cudaMemcpyAsync(tmp + off, x->data, x->bytes, cudaMemcpyHostToDevice, st);
      if (err != cudaSuccess) return cuda_fail(err, "tensor upload");
      off += x->bytes;
    }
    const cudaError_t err = cudaStreamSynchronize(st);
    return err == cudaSuccess ? CLM_OK : cuda_fail(err, "tensor upload");
  };
  auto norm = [&](const std::string& name, float** dst) -> int {
    const clm_b200_tensor* x = nullptr;
    int r = find(name, (uint64_t)d.H, true, &x);
    if (r == CLM_OK) r = e->alloc_t(dst, (size_t)d.H);
    if (r == CLM_OK) {
      const cudaError_t err = cudaMemcpy(*dst, x->data, (size_t)d.H * 4, cudaMemcpyHostToDevice);
      if (err != cudaSuccess) r = cuda_fail(err, "norm upload");
    }
    return r;
  };
  do {
    const uint64_t H = d.H, qd = d.qd(), kvd = d.kvd(), F = d.F;
    for (uint32_t L = e->spec.layer_begin; L < e->spec.layer_end && rc == CLM_OK; ++L) {
      LlamaEngine::Layer lay;
      const std::string b = "blk." + std::to_string(L) + ".";
      const clm_b200_tensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *g = nullptr, *u = nullptr,
                            *dn = nullptr;
      if ((rc = find(b + "attn_q.weight", qd * H, false, &q)) || (rc = find(b + "attn_k.weight", kvd * H, false, &k)) ||
          (rc = find(b + "attn_v.weight", kvd * H, false, &v)) ||
          (rc = find(b + "attn_output.weight", H * qd, false, &o)) ||
          (rc = find(b + "ffn_gate.weight", F * H, false, &g)) || (rc = find(b + "ffn_up.weight", F * H, false, &u)) ||
          (rc = find(b + "ffn_down.weight", H * F, false, &dn)))
        break;
      if ((rc = stage({q, k, v})) ||
          (rc = e->make_gemv(lay.qkv, tmp, tbytes((qd + 2 * kvd) * H), (uint32_t)(qd + 2 * kvd), (uint32_t)H)))
        break;
      if ((rc = stage({o})) || (rc = e->make_gemv(lay.o, tmp, tbytes(H * qd), (uint32_t)H, (uint32_t)qd))) break;
      if ((rc = stage({g, u})) ||
          (rc = e->make_gemv(lay.gu, tmp, tbytes(2 * F * H), (uint32_t)(2 * F), (uint32_t)H, (uint32_t)F)))
        break;
      if ((rc = stage({dn})) || (rc = e->make_gemv(lay.down, tmp, tbytes(H * F), (uint32_t)H, (uint32_t)F))) break;
      if ((rc = norm(b + "attn_norm.weight", &lay.attn_norm)) || (rc = norm(b + "ffn_norm.weight", &lay.ffn_norm)))
        break;
      e->layers.push_back(lay);
    }
    if (rc) break;
    const uint64_t VH = (uint64_t)d.V * d.H;
    if (e->has_embd) {
      const clm_b200_tensor* x = nullptr;
      if ((rc = find("token_embd.weight", VH, false, &x))) break;
      e->embd_bytes = x->bytes;
      if ((rc = e->alloc((void**)&e->embd, e->embd_bytes))) break;
      const cudaError_t err = cudaMemcpy(e->embd, x->data, x->bytes, cudaMemcpyHostToDevice);
      if (err != cudaSuccess) {
        rc = cuda_fail(err, "embedding upload");
        break;
      }
      e->weight_bytes += e->embd_bytes;
    }
    if (e->has_head) {
      const clm_b200_tensor* x = nullptr;
      // files whose head shares the token embedding's weights have no output.weight (llama.cpp then uses
      // token_embd.weight as the head)
      const char* head_name = by.count("output.weight") ? "output.weight" : "token_embd.weight";
      if ((rc = find(head_name, VH, false, &x)) || (rc = stage({x})) ||
          (rc = e->make_gemv(e->head, tmp, tbytes(VH), (uint32_t)d.V, (uint32_t)d.H)))
        break;
      if ((rc = norm("output_norm.weight", &e->out_norm))) break;
    }
    if (e->has_mtp) {
      const uint64_t FH = (uint64_t)d.F * d.H;
      const clm_b200_tensor *g = nullptr, *u = nullptr, *dn = nullptr;
      if ((rc = find("mtp.ffn_gate.weight", FH, false, &g)) || (rc = find("mtp.ffn_up.weight", FH, false, &u)) ||
          (rc = find("mtp.ffn_down.weight", FH, false, &dn)))
        break;
      if ((rc = stage({g, u})) ||
          (rc = e->make_gemv(e->mtp_gu, tmp, tbytes(2 * FH), (uint32_t)(2 * d.F), (uint32_t)d.H, (uint32_t)d.F)))
        break;
      if ((rc = stage({dn})) || (rc = e->make_gemv(e->mtp_down, tmp, tbytes(FH), (uint32_t)d.H, (uint32_t)d.F)))
        break;
      if ((rc = norm("mtp.ffn_norm.weight", &e->mtp_ffn_norm)) || (rc = norm("mtp.output_norm.weight", &e->mtp_out_norm)))
        break;
    }
  } while (false);
  cudaStreamSynchronize(st);
  cudaFree(tmp);
  if (rc == CLM_OK) e->weights_ready = true;
  return rc;
}

int llama_prepare(LlamaEngine* e) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->weights_ready, CLM_FAILED_PRECONDITION, "weights are not bound");
  CLM_CHECK(!e->prepared, CLM_FAILED_PRECONDITION, "engine already prepared");
  const LlamaDims& d = e->d;
  const int W = e->wmax();
  // largest split-partial buffer over every GEMV of this stage at nt = 1 and 2
  uint64_t part_floats = 1, max_ng = 1;
  auto account = [&](const Gemv& g) {
    if (!g.m) return;
    for (int i = 0; i < 3; ++i)
      part_floats = std::max<uint64_t>(part_floats, (uint64_t)g.m->shape.ng * g.plan[i].ksplit * W * 128);
    max_ng = std::max<uint64_t>(max_ng, g.m->shape.ng);
  };
  for (auto& L : e->layers) {
    account(L.qkv);
    account(L.o);
    account(L.gu);
    account(L.down);
  }
  account(e->head);
  account(e->mtp_gu);
  account(e->mtp_down);
  e->pages_total = (int)e->spec.max_sessions * e->max_pages;
  const size_t page_bytes = (size_t)d.nkv * kPageTokens * d.hd * sizeof(__half);
  const int mtiles = (W * (d.nh / d.nkv) + 15) / 16;
  const int mtiles_q16 = (std::min(W, 16) * (d.nh / d.nkv) + 15) / 16;  // windows on the GEMV chain
  const int maxcols = std::max(std::max(d.H, d.F), d.qd());
  CLM_TRY(e->alloc_t(&e->h, (size_t)W * d.H));
  CLM_TRY(e->alloc_t(&e->part, part_floats));
  CLM_TRY(e->alloc_t(&e->gcount, max_ng));
  CLM_CUDA(cudaMemset(e->gcount, 0, max_ng * sizeof(int)));
  e->gcount_n = max_ng;
  {
    const char* env = getenv("CLM_B200_LINK");
    e->link_ok = env && env[0] == '1' && e->link_shape_ok() && !e->layers.empty();
    const char* senv = getenv("CLM_B200_STRIP");
    if (senv) e->strip_mask = atoi(senv);
    const char* penv = getenv("CLM_B200_PF_KB");
    if (penv && atoi(penv) > 0) e->pf_cap = (unsigned long long)atoi(penv) * 1024;
  }
  if (e->link_ok) {
    CLM_TRY(e->alloc_t(&e->part2, part_floats));
    CLM_TRY(e->alloc_t(&e->gcount2, max_ng));
    CLM_CUDA(cudaMemset(e->gcount2, 0, max_ng * sizeof(int)));
    e->link_n = (int)(e->layers.size() * e->link_layout().per_layer);
    CLM_TRY(e->alloc_t(&e->link_ctr, (size_t)e->link_n));
    CLM_CUDA(cudaMemset(e->link_ctr, 0, (size_t)e->link_n * sizeof(int)));
  }
  CLM_TRY(e->alloc_t(&e->acount, (size_t)2 * mtiles * d.nkv));  // attention arrival + departure counters
  CLM_CUDA(cudaMemset(e->acount, 0, (size_t)2 * mtiles * d.nkv * sizeof(int)));
  e->acount_n = (size_t)2 * mtiles * d.nkv;
  for (XBuf* x : {&e->xa, &e->xb}) {
    // fragments and sums for up to 32 window rows (the batched GEMV chain's 4 n-tiles)
    CLM_TRY(e->alloc((void**)&x->frag, xfrag_bytes(maxcols, 4)));
    CLM_CUDA(cudaMemset(x->frag, 0, xfrag_bytes(maxcols, 4)));
    CLM_TRY(e->alloc((void**)&x->sum, xsum_bytes(maxcols, 4)));
    CLM_CUDA(cudaMemset(x->sum, 0, xsum_bytes(maxcols, 4)));
    CLM_TRY(e->alloc_t(&x->ss, (size_t)(d.H / 16) * 16));  // partials per 128 columns, or per 16 (strip GEMV)
    x->nss = d.H / 128;
  }
  CLM_TRY(e->ones(&e->ones_h, d.H));
  CLM_TRY(e->alloc_t(&e->q16, (size_t)W * d.qd()));
  // split partials, one per CTA: a launch has (m-tiles x kv heads) x splits CTAs with splits <= max_pages, and
  // more than one split only while that product stays within the SM count
  {
    const size_t narrow = (size_t)mtiles_q16 * d.nkv * e->max_pages;
    const size_t wide = std::max((size_t)e->ctx->sm_count, (size_t)mtiles * d.nkv);
    CLM_TRY(e->alloc_t(&e->attn_part, std::max(narrow, wide) * attn_partial_floats(d.hd)));
  }
  if (W > 16) {
    size_t rows = (size_t)d.H, part_max = 0;
    auto wide_account = [&](const Gemv& g) {
      if (!g.m) return;
      rows = std::max<size_t>(rows, g.m->shape.rows);
      const TcPlan p = gemm_tc_plan(g.m->shape, W, e->ctx->sm_count);
      if (p.ksplit > 1) part_max = std::max(part_max, p.part_floats);
    };
    for (auto& L : e->layers) {
      wide_account(L.qkv);
      wide_account(L.o);
      wide_account(L.gu);
      wide_account(L.down);
    }
    wide_account(e->head);
    const size_t P = (size_t)(W + 15) / 16 * 16;
    CLM_TRY(e->alloc_t(&e->wy, (size_t)W * rows));
    e->wpart_floats = part_max;
    if (part_max) CLM_TRY(e->alloc_t(&e->wpart, part_max));
    CLM_TRY(e->alloc_t(&e->wattn, (size_t)W * d.qd()));
    {
      // tiles of a wide attention launch: (kv head, head subgroup) x (16-row blocks, or sessions of <= 16 rows)
      const int group = d.nh / d.nkv, hg = group < 4 ? group : 4;
      e->wattn_tiles = d.nkv * (group / hg) * std::max((W + 15) / 16, 16);
      e->wattn_part_floats = (size_t)e->wattn_tiles * 8 * hg * 16 * kAttnRowFloats;
      CLM_TRY(e->alloc_t(&e->wattn_part, e->wattn_part_floats));
      CLM_TRY(e->alloc_t(&e->wattn_cnt, (size_t)e->wattn_tiles));
      CLM_CUDA(cudaMemset(e->wattn_cnt, 0, (size_t)e->wattn_tiles * sizeof(int)));
    }
    CLM_TRY(e->alloc((void**)&e->wxh, P * maxcols * sizeof(__half)));
  }
  {
    const size_t n = (size_t)e->spec.max_context * (d.hd / 2);
    CLM_TRY(e->alloc_t(&e->rope, n));
    rope_table_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, e->ctx->stream>>>(e->rope, e->spec.max_context, d.hd,
                                                                               d.theta);
    CLM_LAUNCHED("rope_table_kernel");
  }
  // dataflow window kernel (windows of <= 16 rows without a tree): one cooperative grid per column-tile count;
  // opt-in with CLM_B200_FLOW=1 (the per-kernel chain is faster on the measured shapes)
  {
    const char* env = getenv("CLM_B200_FLOW");
    const bool want = env && env[0] == '1' && e->flow_shape_ok();
    const int G = e->ctx->sm_count;
    e->flow_attn_maxseg = (G + d.nkv - 1) / d.nkv + 1;  // bound for one m-tile (more m-tiles: fewer segments)
    if (want && e->flow_attn_maxseg <= 64) {
      for (int nt = 1; nt <= 2; ++nt) {
        const GemvShape sh = e->layers[0].qkv.m->shape;
        const int sbytes = g4_geom(sh, nt).stage_bytes;
        const int stages = flow_stages(sbytes);
        e->flow_stage_bytes[nt - 1] = sbytes;
        e->flow_stage_count[nt - 1] = stages;
        e->flow_grid_n[nt - 1] = stages ? flow_grid(e->ctx->device, stages, sbytes, d.quant, nt) : 0;
        if (e->flow_grid_n[nt - 1] != G) e->flow_grid_n[nt - 1] = 0;  // the stream-K bounds assume one CTA per SM
      }
      const int wq = std::min(W, 16);
      auto region = [&](int kind, std::initializer_list<const Gemv*> gs) -> int {
        uint64_t floats = 1, ng = 1;
        for (const Gemv* g : gs) {
          if (!g->m) continue;
          for (int i = 0; i < 2; ++i)
            floats = std::max<uint64_t>(floats, (uint64_t)g->m->shape.ng * g->plan[i].ksplit * wq * 128);
          ng = std::max<uint64_t>(ng, g->m->shape.ng);
        }
        CLM_TRY(e->alloc_t(&e->flow_part[kind], floats));
        CLM_TRY(e->alloc_t(&e->flow_gcount[kind], ng));
        CLM_CUDA(cudaMemset(e->flow_gcount[kind], 0, ng * sizeof(int)));
        e->flow_gcount_n[kind] = ng;
        return CLM_OK;
      };
      const auto& L0 = e->layers[0];  // every layer's matrices have the same shapes
      CLM_TRY(region(LlamaEngine::FK_QKV, {&L0.qkv}));
      CLM_TRY(region(LlamaEngine::FK_O, {&L0.o}));
      CLM_TRY(region(LlamaEngine::FK_GU, {&L0.gu}));
      CLM_TRY(region(LlamaEngine::FK_DOWN, {&L0.down}));
      CLM_TRY(region(LlamaEngine::FK_HEAD, {&e->head}));
      CLM_TRY(e->alloc_t(&e->flow_attn_part,
                         (size_t)mtiles_q16 * d.nkv * e->flow_attn_maxseg * 16 * kFlowAttnRowFloats));
      const auto C = e->flow_ctr_layout();
      e->flow_ctr_n = (size_t)C.head + d.H / 512;
      CLM_TRY(e->alloc_t(&e->flow_ctr, e->flow_ctr_n));
    }
  }
  CLM_TRY(e->alloc_t(&e->tokens, (size_t)W));
  // (+4 floats: link messages are whole 16-byte units)
  CLM_TRY(e->alloc_t(&e->bin, (size_t)W * e->floats_per_position() + 4));
  CLM_TRY(e->alloc_t(&e->bout, (size_t)W * e->floats_per_position() + 4));
  CLM_CUDA(cudaMemset(e->bin, 0, ((size_t)W * e->floats_per_position() + 4) * sizeof(float)));
  CLM_CUDA(cudaMemset(e->bout, 0, ((size_t)W * e->floats_per_position() + 4) * sizeof(float)));
  CLM_TRY(e->alloc_t(&e->bad, 1));
  CLM_CUDA(cudaMemset(e->bad, 0, sizeof(int)));
  if (e->has_head) CLM_TRY(e->alloc_t(&e->logits, (size_t)W * d.V));
  if (e->has_mtp) {
    CLM_TRY(e->alloc_t(&e->h_mtp, (size_t)d.H));
    CLM_TRY(e->alloc_t(&e->draft_logits, (size_t)W * d.V));
  }
  CLM_TRY(e->alloc_t(&e->win, (size_t)W + 1));
  CLM_TRY(e->alloc_t(&e->parents, (size_t)W));
  if (e->has_head) {
    CLM_TRY(e->alloc_t(&e->tprobs, (size_t)W * d.V));
    CLM_TRY(e->alloc_t(&e->dprobs, (size_t)W * d.V));
    CLM_TRY(e->alloc_t(&e->am, (size_t)W));
    void* sbase = nullptr;
    const size_t sbytes = SampleScratch::bytes(2 * W, 1, d.V);
    CLM_TRY(e->alloc(&sbase, sbytes));
    e->samp = SampleScratch::carve(sbase, 2 * W, 1, d.V);
    CLM_CUDA(cudaMemset(sbase, 0, e->samp.counter_bytes));
    e->samp_counters = sbase;
    e->samp_counter_bytes = e->samp.counter_bytes;
  }
  CLM_TRY(e->alloc_t(&e->acc, 1));
  CLM_TRY(e->alloc_t(&e->nxt, 1));
  CLM_TRY(e->alloc_t(&e->emitted, (size_t)W + 1));
  CLM_TRY(e->alloc_t(&e->count, 1));
  CLM_TRY(e->alloc_t(&e->zero_counter, 1));
  CLM_TRY(e->alloc_t(&e->ctl, 1));
  CLM_CUDA(cudaMemset(e->ctl, 0, sizeof(RoundCtl)));
  CLM_CUDA(cudaMemset(e->zero_counter, 0, sizeof(unsigned long long)));
  for (size_t li = 0; li < e->layers.size(); ++li) {
    __half *k = nullptr, *v = nullptr;
    CLM_TRY(e->alloc_t(&k, page_bytes / sizeof(__half) * e->pages_total));
    CLM_TRY(e->alloc_t(&v, page_bytes / sizeof(__half) * e->pages_total));
    CLM_CUDA(cudaMemset(k, 0, page_bytes * e->pages_total));
    CLM_CUDA(cudaMemset(v, 0, page_bytes * e->pages_total));
    e->kpool.push_back(k);
    e->vpool.push_back(v);
  }
  for (int p = e->pages_total - 1; p >= 0; --p) e->free_pages.push_back(p);
  CLM_CUDA(cudaStreamSynchronize(e->ctx->stream));
  e->prepared = true;
  return CLM_OK;
}

int llama_info(const LlamaEngine* e, uint64_t* weight_bytes, uint64_t* state_bytes, uint32_t* fpp) {
  CLM_CHECK(e != nullptr, CLM_INVALID_ARGUMENT, "null engine");
  if (weight_bytes) *weight_bytes = e->weight_bytes;
  if (state_bytes)
    *state_bytes = (uint64_t)e->layers.size() * 2 * e->max_pages * e->d.nkv * kPageTokens * e->d.hd * sizeof(__half);
  if (fpp) *fpp = (uint32_t)e->floats_per_position();
  return CLM_OK;
}

int llama_session_open(LlamaEngine* e, uint64_t id) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "engine not prepared");
  CLM_CHECK(find_session(e, id) == nullptr, CLM_ALREADY_EXISTS, "session already open");
  CLM_CHECK((int)e->free_pages.size() >= e->max_pages, CLM_RESOURCE_EXHAUSTED, "max_sessions reached");
  auto s = std::make_unique<Session>();
  s->id = id;
  for (int i = 0; i < e->max_pages; ++i) {
    s->pages.push_back(e->free_pages.back());
    e->free_pages.pop_back();
  }
  cudaError_t err = cudaMalloc(&s->d_pages, s->pages.size() * sizeof(int32_t));
  if (err == cudaSuccess) err = cudaMalloc(&s->d_state, sizeof(SessionState));
  if (err == cudaSuccess)
    err = cudaMemcpy(s->d_pages, s->pages.data(), s->pages.size() * sizeof(int32_t), cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cudaMemset(s->d_state, 0, sizeof(SessionState));
  if (err == cudaSuccess && e->spec.role == CLM_ROLE_TAIL && e->has_mtp) {
    // a pipeline tail keeps each session's window and draft distributions across rounds
    err = cudaMalloc(&s->d_win, (size_t)(e->wmax() + 1) * sizeof(int32_t));
    if (err == cudaSuccess) err = cudaMemset(s->d_win, 0, (size_t)(e->wmax() + 1) * sizeof(int32_t));
    if (err == cudaSuccess) err = cudaMalloc(&s->d_dprobs, (size_t)e->wmax() * e->d.V * sizeof(float));
  }
  if (err != cudaSuccess) {
    e->release_session(*s);
    return cuda_fail(err, "session_open");
  }
  e->sessions[id] = std::move(s);
  return CLM_OK;
}

int llama_session_close(LlamaEngine* e, uint64_t id) {
  CLM_TRY(engine_enter(e));
  Session* s = find_session(e, id);
  if (!s) return CLM_OK;  // idempotent cleanup (WindowLedger::abort_session)
  CLM_CUDA(cudaStreamSynchronize(e->ctx->stream));
  e->drop_batch_graphs();
  e->release_session(*s);
  e->sessions.erase(id);
  return CLM_OK;
}

// Re-reads the committed position after device-driven rounds.
static int sync_pos(LlamaEngine* e, Session* s) {
  if (!s->pos_stale) return CLM_OK;
  long long p = 0;
  CLM_CUDA(cudaMemcpyAsync(&p, &s->d_state->pos, sizeof(p), cudaMemcpyDeviceToHost, e->ctx->stream));
  CLM_CUDA(cudaStreamSynchronize(e->ctx->stream));
  s->pos = s->pos_bound = p;
  s->pos_stale = false;
  return CLM_OK;
}

static int run_window_common(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, cudaStream_t st,
                             Session** out) {
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "engine not prepared");
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_TRY(sync_pos(e, s));
  CLM_CHECK(s->outstanding == 0, CLM_FAILED_PRECONDITION, "a window is already outstanding for this session");
  CLM_CHECK(q >= 1, CLM_INVALID_ARGUMENT, "window must have at least one position");
  CLM_CHECK(q <= e->spec.max_window, CLM_RESOURCE_EXHAUSTED, "window exceeds max_window");
  CLM_CHECK(base + q <= e->spec.max_context, CLM_RESOURCE_EXHAUSTED, "window exceeds max_context");
  CLM_CHECK((long long)base == s->pos, CLM_FAILED_PRECONDITION, "window base position != committed position");
  (void)st;
  *out = s;
  return CLM_OK;
}

int llama_run_window_device(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* d_tokens,
                               const float* d_in, float* d_out, float* d_logits, void* stream) {
  CLM_TRY(engine_enter(e));
  cudaStream_t st = pick_stream(e->ctx, stream);
  Session* s = nullptr;
  CLM_TRY(run_window_common(e, id, base, q, st, &s));
  const size_t rec = (size_t)q * e->floats_per_position() * sizeof(float);
  if (e->has_tokens) {
    CLM_CHECK(d_tokens != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes tokens");
  } else {
    CLM_CHECK(d_in != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes activations");
    CLM_CUDA(cudaMemcpyAsync(e->bin, d_in, rec, cudaMemcpyDeviceToDevice, st));
  }
  if (e->has_tokens) CLM_CUDA(cudaMemcpyAsync(e->win, d_tokens, q * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  CLM_TRY(e->run_graph(*s, 0, (int)q, 0, st, [&](cudaStream_t cs) { return e->enqueue_window(*s, (int)q, e->win, cs); }));
  if (e->has_head) {
    if (d_logits)
      CLM_CUDA(cudaMemcpyAsync(d_logits, e->logits, (size_t)q * e->d.V * sizeof(float), cudaMemcpyDeviceToDevice, st));
  } else if (d_out) {
    CLM_CUDA(cudaMemcpyAsync(d_out, e->bout, rec, cudaMemcpyDeviceToDevice, st));
  }
  s->outstanding = q;  // out-of-range device tokens embed as zeros and are reported by llama_commit
  return CLM_OK;
}

int llama_run_tree_device(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* d_parents,
                          const int32_t* d_tokens, const float* d_in, float* d_out, float* d_logits, void* stream) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(d_parents != nullptr, CLM_INVALID_ARGUMENT, "null parents");
  cudaStream_t st = pick_stream(e->ctx, stream);
  Session* s = nullptr;
  CLM_TRY(run_window_common(e, id, base, q, st, &s));
  const size_t rec = (size_t)q * e->floats_per_position() * sizeof(float);
  if (e->has_tokens) {
    CLM_CHECK(d_tokens != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes tokens");
    CLM_CUDA(cudaMemcpyAsync(e->win, d_tokens, q * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  } else {
    CLM_CHECK(d_in != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes activations");
    CLM_CUDA(cudaMemcpyAsync(e->bin, d_in, rec, cudaMemcpyDeviceToDevice, st));
  }
  // device parents are validated on the device (a bad entry becomes -1 and the window reports an error at commit)
  tree_guard_kernel<<<1, 32 * ((q + 31) / 32), 0, st>>>(d_parents, (int)q, e->parents, e->bad);
  CLM_LAUNCHED("tree_guard_kernel");
  CLM_TRY(e->run_graph(*s, 4, (int)q, 0, st,
                       [&](cudaStream_t cs) { return e->enqueue_window(*s, (int)q, e->win, cs, e->parents); }));
  if (e->has_head) {
    if (d_logits)
      CLM_CUDA(cudaMemcpyAsync(d_logits, e->logits, (size_t)q * e->d.V * sizeof(float), cudaMemcpyDeviceToDevice, st));
  } else if (d_out) {
    CLM_CUDA(cudaMemcpyAsync(d_out, e->bout, rec, cudaMemcpyDeviceToDevice, st));
  }
  s->outstanding = q;
  s->tree = true;
  s->tree_parents.clear();  // validated on the device: commit_path reads them there
  return CLM_OK;
}

static int run_window_host(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_parents,
                           const int32_t* h_tokens, const float* h_in, float* h_out, float* h_logits) {
  CLM_TRY(engine_enter(e));
  cudaStream_t st = e->ctx->stream;
  Session* s = nullptr;
  if (h_parents != nullptr) {
    // a tree: every node's parent is an earlier node or -1 (the committed context)
    for (uint32_t i = 0; i < q; ++i)
      CLM_CHECK(h_parents[i] >= -1 && h_parents[i] < (int32_t)i, CLM_INVALID_ARGUMENT,
                "tree window: parent[i] must be -1 or an earlier node");
  }
  CLM_TRY(run_window_common(e, id, base, q, st, &s));
  const size_t rec = (size_t)q * e->floats_per_position() * sizeof(float);
  const size_t out_bytes = e->has_head ? (size_t)q * e->d.V * sizeof(float) : rec;
  // the caller's buffers are pageable (records arriving from another host, logits for the acceptance): they pass
  // through pinned staging buffers of the engine, so both copies are DMA transfers at full link speed
  CLM_TRY(e->pinned(&e->pin_in, &e->pin_in_bytes, std::max(rec, (size_t)q * sizeof(int32_t))));
  CLM_TRY(e->pinned(&e->pin_out, &e->pin_out_bytes, out_bytes));
  if (e->has_tokens) {
    CLM_CHECK(h_tokens != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes tokens");
    for (uint32_t i = 0; i < q; ++i)
      CLM_CHECK(h_tokens[i] >= 0 && h_tokens[i] < e->d.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
    std::memcpy(e->pin_in, h_tokens, q * sizeof(int32_t));
    CLM_CUDA(cudaMemcpyAsync(e->win, e->pin_in, q * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  } else {
    CLM_CHECK(h_in != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes activations");
    std::memcpy(e->pin_in, h_in, rec);
    CLM_CUDA(cudaMemcpyAsync(e->bin, e->pin_in, rec, cudaMemcpyHostToDevice, st));
  }
  if (h_parents != nullptr) {
    CLM_CUDA(cudaMemcpyAsync(e->parents, h_parents, q * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    CLM_TRY(e->run_graph(*s, 4, (int)q, 0, st,
                         [&](cudaStream_t cs) { return e->enqueue_window(*s, (int)q, e->win, cs, e->parents); }));
  } else {
    CLM_TRY(e->run_graph(*s, 0, (int)q, 0, st,
                         [&](cudaStream_t cs) { return e->enqueue_window(*s, (int)q, e->win, cs); }));
  }
  float* h_dst = e->has_head ? h_logits : h_out;
  if (h_dst)
    CLM_CUDA(cudaMemcpyAsync(e->pin_out, e->has_head ? e->logits : e->bout, out_bytes, cudaMemcpyDeviceToHost, st));
  CLM_CUDA(cudaStreamSynchronize(st));
  if (h_dst) std::memcpy(h_dst, e->pin_out, out_bytes);
  s->outstanding = q;
  s->tree = h_parents != nullptr;
  if (h_parents)
    s->tree_parents.assign(h_parents, h_parents + q);
  else
    s->tree_parents.clear();
  return CLM_OK;
}

int llama_run_batch(LlamaEngine* e, uint32_t n, const uint64_t* ids, const uint64_t* bases, uint32_t q,
                    const int32_t* h_parents, const int32_t* h_tokens, float* h_logits) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "engine not prepared");
  CLM_CHECK(e->spec.role == CLM_ROLE_WHOLE, CLM_FAILED_PRECONDITION, "batched windows need a whole-model engine");
  CLM_CHECK(ids != nullptr && bases != nullptr && h_tokens != nullptr && n >= 1 && q >= 1, CLM_INVALID_ARGUMENT,
            "batched window: null or empty argument");
  CLM_CHECK((uint64_t)n * q <= e->spec.max_window, CLM_RESOURCE_EXHAUSTED, "batched window exceeds max_window");
  CLM_CHECK(q <= 16, CLM_OUT_OF_RANGE, "batched window: at most 16 rows per session");
  const uint32_t Q = n * q;
  CLM_CHECK(Q > 16, CLM_OUT_OF_RANGE, "batched window: more than 16 rows in all (fewer: one window per session)");
  if (h_parents != nullptr)
    for (uint32_t i = 0; i < q; ++i)
      CLM_CHECK(h_parents[i] >= -1 && h_parents[i] < (int32_t)i, CLM_INVALID_ARGUMENT,
                "tree window: parent[i] must be -1 or an earlier node");
  for (uint32_t i = 0; i < Q; ++i)
    CLM_CHECK(h_tokens[i] >= 0 && h_tokens[i] < e->d.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
  cudaStream_t st = e->ctx->stream;
  std::vector<LlamaEngine::WideSeg> segs;
  for (uint32_t b = 0; b < n; ++b) {
    for (uint32_t c = 0; c < b; ++c) CLM_CHECK(ids[c] != ids[b], CLM_INVALID_ARGUMENT, "a session appears twice");
    Session* s = nullptr;
    CLM_TRY(run_window_common(e, ids[b], bases[b], q, st, &s));
    segs.push_back({s, (int)(b * q), (int)q});
  }
  CLM_CUDA(cudaMemcpyAsync(e->win, h_tokens, Q * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  if (h_parents != nullptr)
    CLM_CUDA(cudaMemcpyAsync(e->parents, h_parents, q * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  // one CUDA graph per session set (eager on first use, captured on the second, replayed after)
  std::vector<uint64_t> key(ids, ids + n);
  auto& holder = e->batch_graphs[key];
  if (!holder) holder = std::make_unique<Session>();
  const int32_t* par = h_parents ? e->parents : nullptr;
  CLM_TRY(e->run_graph(*holder, 7, (int)Q, h_parents ? 1 : 0, st, [&](cudaStream_t cs) {
    return e->enqueue_window_wide(segs.data(), (int)n, (int)Q, e->win, par, cs);
  }));
  if (h_logits)
    CLM_CUDA(cudaMemcpyAsync(h_logits, e->logits, (size_t)Q * e->d.V * sizeof(float), cudaMemcpyDeviceToHost, st));
  CLM_CUDA(cudaStreamSynchronize(st));
  for (auto& g : segs) {
    g.s->outstanding = q;
    g.s->tree = h_parents != nullptr;
    if (h_parents)
      g.s->tree_parents.assign(h_parents, h_parents + q);
    else
      g.s->tree_parents.clear();
  }
  return CLM_OK;
}

int llama_run_batch_device(LlamaEngine* e, uint32_t n, const uint64_t* ids, const uint64_t* bases, uint32_t q,
                           const int32_t* d_tokens, const float* d_in, float* d_out, float* d_logits, void* stream) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "engine not prepared");
  CLM_CHECK(ids != nullptr && bases != nullptr && n >= 1 && n <= 4 && q >= 1 && q <= 8, CLM_INVALID_ARGUMENT,
            "batched GEMV window: 1..4 sessions of 1..8 rows");
  const uint32_t Q = n * q;
  CLM_CHECK(Q <= e->spec.max_window, CLM_RESOURCE_EXHAUSTED, "batched window exceeds max_window");
  if (e->has_tokens)
    CLM_CHECK(d_tokens != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes tokens");
  else
    CLM_CHECK(d_in != nullptr, CLM_INVALID_ARGUMENT, "this stage consumes activations");
  cudaStream_t st = pick_stream(e->ctx, stream);
  std::vector<LlamaEngine::WideSeg> segs;
  for (uint32_t b = 0; b < n; ++b) {
    for (uint32_t c = 0; c < b; ++c) CLM_CHECK(ids[c] != ids[b], CLM_INVALID_ARGUMENT, "a session appears twice");
    Session* s = nullptr;
    CLM_TRY(run_window_common(e, ids[b], bases[b], q, st, &s));
    segs.push_back({s, (int)(b * q), (int)q});
  }
  const size_t rec = (size_t)Q * e->floats_per_position() * sizeof(float);
  if (e->has_tokens)
    CLM_CUDA(cudaMemcpyAsync(e->win, d_tokens, Q * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  else
    CLM_CUDA(cudaMemcpyAsync(e->bin, d_in, rec, cudaMemcpyDeviceToDevice, st));
  std::vector<uint64_t> key(ids, ids + n);
  auto& holder = e->batch_graphs[key];
  if (!holder) holder = std::make_unique<Session>();
  CLM_TRY(e->run_graph(*holder, 8, (int)Q, 0, st, [&](cudaStream_t cs) {
    return e->enqueue_batch_chain(segs.data(), (int)n, (int)Q, e->win, cs);
  }));
  if (e->has_head) {
    if (d_logits)
      CLM_CUDA(cudaMemcpyAsync(d_logits, e->logits, (size_t)Q * e->d.V * sizeof(float), cudaMemcpyDeviceToDevice, st));
  } else if (d_out) {
    CLM_CUDA(cudaMemcpyAsync(d_out, e->bout, rec, cudaMemcpyDeviceToDevice, st));
  }
  for (auto& g : segs) {
    g.s->outstanding = q;
    g.s->tree = false;
    g.s->tree_parents.clear();
  }
  return CLM_OK;
}

int llama_run_window(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_tokens,
                     const float* h_in, float* h_out, float* h_logits) {
  return run_window_host(e, id, base, q, nullptr, h_tokens, h_in, h_out, h_logits);
}

int llama_run_tree(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_parents,
                   const int32_t* h_tokens, const float* h_in, float* h_out, float* h_logits) {
  CLM_CHECK(h_parents != nullptr, CLM_INVALID_ARGUMENT, "null parents");
  return run_window_host(e, id, base, q, h_parents, h_tokens, h_in, h_out, h_logits);
}

int llama_commit_path(LlamaEngine* e, uint64_t id, const int32_t* h_path, uint32_t n) {
  CLM_TRY(engine_enter(e));
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_CHECK(s->outstanding > 0, CLM_FAILED_PRECONDITION, "no outstanding window");
  CLM_CHECK(h_path != nullptr && n >= 1 && n <= s->outstanding, CLM_INVALID_ARGUMENT, "path must hold 1..q nodes");
  std::vector<int32_t> parents(s->outstanding, -1);
  if (s->tree && s->tree_parents.size() == s->outstanding)
    parents = s->tree_parents;
  else if (s->tree)
    CLM_CUDA(cudaMemcpy(parents.data(), e->parents, s->outstanding * sizeof(int32_t), cudaMemcpyDeviceToHost));
  else
    for (uint32_t i = 0; i < s->outstanding; ++i) parents[i] = (int32_t)i - 1;
  for (uint32_t i = 0; i < n; ++i) {
    CLM_CHECK(h_path[i] >= 0 && (uint32_t)h_path[i] < s->outstanding, CLM_INVALID_ARGUMENT, "path node out of range");
    CLM_CHECK(parents[h_path[i]] == (i == 0 ? -1 : h_path[i - 1]), CLM_INVALID_ARGUMENT,
              "path must run from a root (parent -1) along parent links");
  }
  {
    const int rc = e->check_bad(e->ctx->stream);
    if (rc != CLM_OK) {
      s->outstanding = 0;
      return rc;
    }
  }
  cudaStream_t st = e->ctx->stream;
  bool moved = false;
  for (uint32_t i = 0; i < n; ++i) moved |= h_path[i] != (int32_t)i;
  if (moved && !e->layers.empty()) {
    if (e->d_kpools == nullptr) {
      CLM_TRY(e->alloc_t(&e->d_kpools, e->layers.size()));
      CLM_TRY(e->alloc_t(&e->d_vpools, e->layers.size()));
      CLM_CUDA(cudaMemcpy(e->d_kpools, e->kpool.data(), e->layers.size() * sizeof(__half*), cudaMemcpyHostToDevice));
      CLM_CUDA(cudaMemcpy(e->d_vpools, e->vpool.data(), e->layers.size() * sizeof(__half*), cudaMemcpyHostToDevice));
    }
    CLM_CUDA(cudaMemcpyAsync(e->parents, h_path, n * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    const size_t smem = (size_t)n * 2 * e->d.hd * sizeof(__half);
    CLM_TRY(ensure_smem(kv_compact_kernel, smem));
    kv_compact_kernel<<<dim3((unsigned)e->layers.size(), (unsigned)e->d.nkv), 256, smem, st>>>(
        e->d_kpools, e->d_vpools, s->d_pages, &s->d_state->pos, e->parents, (int)n, e->d.nkv, e->d.hd);
    CLM_LAUNCHED("kv_compact_kernel");
  }
  s->pos += n;
  s->pos_bound = s->pos;
  s->outstanding = 0;
  s->tree = false;
  CLM_CUDA(cudaMemcpyAsync(&s->d_state->pos, &s->pos, sizeof(long long), cudaMemcpyHostToDevice, st));
  CLM_CUDA(cudaStreamSynchronize(st));
  return CLM_OK;
}

int llama_commit(LlamaEngine* e, uint64_t id, uint32_t accepted) {
  CLM_TRY(engine_enter(e));
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_CHECK(s->outstanding > 0, CLM_FAILED_PRECONDITION, "no outstanding window");
  CLM_CHECK(accepted >= 1 && accepted <= s->outstanding, CLM_INVALID_ARGUMENT, "accepted must be in [1, q]");
  {
    const int rc = e->check_bad(e->ctx->stream);
    if (rc != CLM_OK) {
      s->outstanding = 0;  // the window is dropped, as the ledger's fail_window does
      return rc;
    }
  }
  CLM_CHECK(!s->tree, CLM_FAILED_PRECONDITION, "a tree window is committed with clm_b200_commit_path");
  s->pos += accepted;
  s->pos_bound = s->pos;
  s->outstanding = 0;
  // the device copy of the committed position is read by the next window's kernels (stream-ordered)
  CLM_CUDA(cudaMemcpyAsync(&s->d_state->pos, &s->pos, sizeof(long long), cudaMemcpyHostToDevice, e->ctx->stream));
  CLM_CUDA(cudaStreamSynchronize(e->ctx->stream));
  return CLM_OK;
}

int llama_abort(LlamaEngine* e, uint64_t id) {
  CLM_TRY(engine_enter(e));
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  s->outstanding = 0;  // KV rows past the committed position are rewritten before any read
  return CLM_OK;
}

int llama_session_position(const LlamaEngine* e, uint64_t id, uint64_t* committed) {
  CLM_CHECK(e != nullptr && committed != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  auto it = e->sessions.find(id);
  CLM_CHECK(it != e->sessions.end(), CLM_NOT_FOUND, "session not open");
  // device-resident rounds advance the position on the device: read it back (waits for the engine's stream)
  CLM_TRY(sync_pos(const_cast<LlamaEngine*>(e), it->second.get()));
  *committed = (uint64_t)it->second->pos;
  return CLM_OK;
}

int llama_mtp_draft(LlamaEngine* e, int32_t prev, uint32_t count, float T, uint64_t seed, uint64_t counter,
                       int32_t* h_tokens, float* h_logits) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->prepared && e->has_mtp, CLM_FAILED_PRECONDITION, "engine has no MTP head");
  CLM_CHECK(count >= 1 && count < e->spec.max_window, CLM_OUT_OF_RANGE, "count must be in [1, max_window)");
  CLM_CHECK(prev >= 0 && prev < e->d.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
  CLM_CHECK(h_tokens != nullptr, CLM_INVALID_ARGUMENT, "null output");
  cudaStream_t st = e->ctx->stream;
  unsigned long long ctr = counter;
  CLM_CUDA(cudaMemcpyAsync(e->zero_counter, &ctr, sizeof(ctr), cudaMemcpyHostToDevice, st));
  CLM_CUDA(cudaMemcpyAsync(e->win, &prev, sizeof(int32_t), cudaMemcpyHostToDevice, st));
  for (uint32_t j = 0; j < count; ++j) {
    CLM_TRY(e->enqueue_mtp_step(e->win + j, e->draft_logits + (size_t)j * e->d.V, st));
    CLM_TRY(e->sample_token(e->draft_logits + (size_t)j * e->d.V, T > 0.0f, T, seed, j, 1u, e->zero_counter, nullptr,
                            e->dprobs + (size_t)j * e->d.V, e->win + j + 1, st));
  }
  CLM_CUDA(cudaMemcpyAsync(h_tokens, e->win + 1, count * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  if (h_logits)
    CLM_CUDA(cudaMemcpyAsync(h_logits, e->draft_logits, (size_t)count * e->d.V * sizeof(float), cudaMemcpyDeviceToHost,
                             st));
  ctr = 0;
  CLM_CUDA(cudaMemcpyAsync(e->zero_counter, &ctr, sizeof(ctr), cudaMemcpyHostToDevice, st));
  CLM_CUDA(cudaStreamSynchronize(st));
  return CLM_OK;
}

// Stochastic MTP proposal (clm_b200_mtp_propose): each draft sampled from distribution(step logits, T, top-k,
// top-p) with the caller's uniform, its distribution row returned.
int llama_mtp_propose(LlamaEngine* e, int32_t prev, uint32_t count, float T, uint32_t top_k, float top_p,
                      const double* h_uniforms, int32_t* h_tokens, float* h_probs) {
  if (T <= 0.0f) {  // greedy drafts (argmax chain), one-hot rows
    const int rc = llama_mtp_draft(e, prev, count, 0.0f, 0, 0, h_tokens, nullptr);
    if (rc == CLM_OK && h_probs != nullptr) {
      const size_t V = (size_t)e->d.V;
      std::memset(h_probs, 0, count * V * sizeof(float));
      for (uint32_t j = 0; j < count; ++j) h_probs[j * V + (uint32_t)h_tokens[j]] = 1.0f;
    }
    return rc;
  }
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->prepared && e->has_mtp, CLM_FAILED_PRECONDITION, "engine has no MTP head");
  CLM_CHECK(count >= 1 && count < e->spec.max_window, CLM_OUT_OF_RANGE, "count must be in [1, max_window)");
  CLM_CHECK(prev >= 0 && prev < e->d.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
  CLM_CHECK(h_tokens != nullptr && h_uniforms != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  cudaStream_t st = e->ctx->stream;
  if (e->propose_u == nullptr) CLM_TRY(e->alloc_t(&e->propose_u, (size_t)e->wmax()));
  CLM_CUDA(cudaMemcpyAsync(e->propose_u, h_uniforms, count * sizeof(double), cudaMemcpyHostToDevice, st));
  CLM_CUDA(cudaMemcpyAsync(e->win, &prev, sizeof(int32_t), cudaMemcpyHostToDevice, st));
  const size_t V = (size_t)e->d.V;
  for (uint32_t j = 0; j < count; ++j) {
    CLM_TRY(e->enqueue_mtp_step(e->win + j, e->draft_logits + j * V, st));
    CLM_TRY(launch_draft_sample(e->ctx, e->draft_logits + j * V, (uint32_t)V, T, top_k, top_p, e->propose_u + j,
                                e->dprobs + j * V, e->win + j + 1, e->samp, st));
  }
  CLM_CUDA(cudaMemcpyAsync(h_tokens, e->win + 1, count * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  if (h_probs) CLM_CUDA(cudaMemcpyAsync(h_probs, e->dprobs, count * V * sizeof(float), cudaMemcpyDeviceToHost, st));
  return e->check_bad(st);
}

int llama_spec_begin(LlamaEngine* e, uint64_t id, const int32_t* h_prompt, uint32_t n,
                        const clm_b200_spec_params* p) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->spec.role == CLM_ROLE_WHOLE, CLM_FAILED_PRECONDITION, "speculative rounds need a whole-model engine");
  CLM_CHECK(h_prompt != nullptr && n >= 1 && p != nullptr, CLM_INVALID_ARGUMENT, "empty prompt");
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_TRY(sync_pos(e, s));
  uint32_t off = 0;
  while (off < n) {
    const uint32_t q = std::min<uint32_t>(e->spec.max_window, n - off);
    CLM_TRY(llama_run_window(e, id, (uint64_t)s->pos, q, h_prompt + off, nullptr, nullptr, nullptr));
    CLM_TRY(llama_commit(e, id, q));
    off += q;
  }
  // first token from the last prompt position (argmax, or a sample with Philox draw (0, stream 2, 0))
  cudaStream_t st = e->ctx->stream;
  const uint32_t last = (n - 1) % e->spec.max_window;
  CLM_TRY(e->sample_token(e->logits + (size_t)last * e->d.V, p->temperature > 0.0f, p->temperature, p->seed, 0u, 2u,
                          e->zero_counter, nullptr, e->tprobs, e->nxt, st));
  CLM_TRY(launch_pdl(set_next_kernel, dim3(1), dim3(32), 0, st, s->d_state, (const int32_t*)e->nxt));
  CLM_CUDA(cudaStreamSynchronize(st));
  return CLM_OK;
}

int llama_spec_round_device(LlamaEngine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* d_tokens,
                               uint32_t* d_count, void* stream) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(p != nullptr, CLM_INVALID_ARGUMENT, "null params");
  CLM_CHECK(e->spec.role == CLM_ROLE_WHOLE && e->has_mtp, CLM_FAILED_PRECONDITION,
            "speculative rounds need a whole-model engine with an MTP head");
  CLM_CHECK(p->q >= 1 && p->q <= e->spec.max_window, CLM_OUT_OF_RANGE, "q must be in [1, max_window]");
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_CHECK(s->outstanding == 0, CLM_FAILED_PRECONDITION, "a window is outstanding");
  if ((uint64_t)s->pos_bound + p->q > e->spec.max_context) CLM_TRY(sync_pos(e, s));
  CLM_CHECK((uint64_t)s->pos_bound + p->q <= e->spec.max_context, CLM_RESOURCE_EXHAUSTED,
            "speculative round would exceed max_context");
  cudaStream_t st = pick_stream(e->ctx, stream);
  const bool stochastic = p->temperature > 0.0f;
  // the round's inputs (temperature, seed) go host -> device each round; the graph reads them there
  RoundCtl c{p->temperature, 0u, (unsigned long long)p->seed};
  CLM_CUDA(cudaMemcpyAsync(e->ctl, &c, sizeof(c), cudaMemcpyHostToDevice, st));
  CLM_TRY(e->run_graph(*s, 1, (int)p->q, stochastic ? 1 : 0, st,
                       [&](cudaStream_t cs) { return e->enqueue_round(*s, (int)p->q, stochastic, cs); }));
  if (d_tokens) CLM_CUDA(cudaMemcpyAsync(d_tokens, e->emitted, (p->q + 1) * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  if (d_count) CLM_CUDA(cudaMemcpyAsync(d_count, e->count, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
  s->pos_bound += p->q;
  s->pos_stale = true;
  return CLM_OK;
}

// ---- stage pipeline ------------------------------------------------------------------------------

// Device views of a stage's input and output links, checked against the largest message this stage exchanges.
static int pipe_links(const LlamaEngine* e, clm_b200_link* in, clm_b200_link* out, LinkDev* li, LinkDev* lo) {
  CLM_TRY(link_dev(in, false, li));
  CLM_TRY(link_dev(out, true, lo));
  const uint32_t need_in = e->spec.role == CLM_ROLE_PREFIX ? LlamaEngine::token_bytes(e->wmax()) : e->record_bytes(e->wmax());
  const uint32_t need_out = e->spec.role == CLM_ROLE_TAIL ? LlamaEngine::token_bytes(e->wmax()) : e->record_bytes(e->wmax());
  CLM_CHECK(li->slot_bytes >= need_in + kLinkHeaderBytes && lo->slot_bytes >= need_out + kLinkHeaderBytes,
            CLM_RESOURCE_EXHAUSTED, "link slots are smaller than a max_window message");
  return CLM_OK;
}

int llama_pipe_attach(LlamaEngine* e, clm_b200_link* in, clm_b200_link* out) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "engine not prepared");
  CLM_CHECK(e->spec.role != CLM_ROLE_WHOLE, CLM_FAILED_PRECONDITION, "a whole-model engine is not a pipeline stage");
  CLM_CHECK(e->spec.role != CLM_ROLE_TAIL || e->has_mtp, CLM_FAILED_PRECONDITION,
            "a pipeline tail drafts the next window: it needs an MTP head");
  LinkDev li, lo;
  CLM_TRY(pipe_links(e, in, out, &li, &lo));
  e->pipe_in = in;
  e->pipe_out = out;
  e->lin = li;
  e->lout = lo;
  return CLM_OK;
}

int llama_pipe_attach_session(LlamaEngine* e, uint64_t id, clm_b200_link* in, clm_b200_link* out) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(e->pipe_in != nullptr, CLM_FAILED_PRECONDITION, "engine is not attached to a pipeline");
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_CHECK(s->outstanding == 0, CLM_FAILED_PRECONDITION, "a window is outstanding");
  LinkDev li, lo;
  CLM_TRY(pipe_links(e, in ? in : e->pipe_in, out ? out : e->pipe_out, &li, &lo));
  // the session's captured rounds hold the links they were captured with
  for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);
  s->graphs.clear();
  s->seen.clear();
  s->launches.clear();
  s->lin = li;
  s->lout = lo;
  s->own_links = true;
  return CLM_OK;
}

static int pipe_session(LlamaEngine* e, uint64_t id, uint32_t q, Session** out) {
  CLM_CHECK(e->prepared, CLM_FAILED_PRECONDITION, "engine not prepared");
  CLM_CHECK(e->pipe_in != nullptr, CLM_FAILED_PRECONDITION, "engine is not attached to a pipeline");
  Session* s = find_session(e, id);
  CLM_CHECK(s != nullptr, CLM_NOT_FOUND, "session not open");
  CLM_CHECK(s->outstanding == 0, CLM_FAILED_PRECONDITION, "a window is outstanding");
  CLM_CHECK(q >= 1 && q <= e->spec.max_window, CLM_OUT_OF_RANGE, "window must be in [1, max_window]");
  CLM_CHECK((uint64_t)s->pos_bound + q <= e->spec.max_context, CLM_RESOURCE_EXHAUSTED,
            "pipeline round would exceed max_context");
  *out = s;
  return CLM_OK;
}

int llama_pipe_prefill(LlamaEngine* e, uint64_t id, const int32_t* h_tokens, uint32_t q, void* stream) {
  CLM_TRY(engine_enter(e));
  Session* s = nullptr;
  CLM_TRY(pipe_session(e, id, q, &s));
  cudaStream_t st = pick_stream(e->ctx, stream);
  if (e->spec.role == CLM_ROLE_PREFIX) {
    CLM_CHECK(h_tokens != nullptr, CLM_INVALID_ARGUMENT, "the prefix consumes tokens");
    for (uint32_t i = 0; i < q; ++i)
      CLM_CHECK(h_tokens[i] >= 0 && h_tokens[i] < e->d.V, CLM_INVALID_ARGUMENT, "token outside the vocabulary");
    CLM_CUDA(cudaMemcpyAsync(e->win, h_tokens, q * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  }
  CLM_TRY(e->run_graph(*s, 6, (int)q, 0, st, [&](cudaStream_t cs) { return e->enqueue_pipe_prefill(*s, (int)q, cs); }));
  s->pos_bound += q;
  s->pos_stale = true;
  return CLM_OK;
}

int llama_pipe_begin(LlamaEngine* e, uint64_t id, uint32_t row, const clm_b200_spec_params* p, void* stream) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(p != nullptr, CLM_INVALID_ARGUMENT, "null params");
  CLM_CHECK(e->spec.role == CLM_ROLE_TAIL, CLM_FAILED_PRECONDITION, "only the pipeline tail begins the rounds");
  Session* s = nullptr;
  CLM_TRY(pipe_session(e, id, p->q, &s));
  CLM_CHECK(row < e->spec.max_window, CLM_OUT_OF_RANGE, "row outside the last window");
  cudaStream_t st = pick_stream(e->ctx, stream);
  const bool stochastic = p->temperature > 0.0f;
  RoundCtl c{p->temperature, 0u, (unsigned long long)p->seed};
  CLM_CUDA(cudaMemcpyAsync(e->ctl, &c, sizeof(c), cudaMemcpyHostToDevice, st));
  CLM_TRY(e->sample_token(e->logits + (size_t)row * e->d.V, stochastic, p->temperature, p->seed, 0u, 2u,
                          e->zero_counter, nullptr, e->tprobs, e->nxt, st));
  CLM_TRY(launch_pdl(set_next_kernel, dim3(1), dim3(32), 0, st, s->d_state, (const int32_t*)e->nxt));
  CLM_TRY(e->enqueue_drafts(*s, (int)p->q, stochastic, s->d_win, s->d_dprobs, st));
  return launch_link_send(e->link_out(*s), s->d_win, LlamaEngine::token_bytes((int)p->q), nullptr, p->q,
                          LINK_MSG_WINDOW, e->bad, st);
}

int llama_pipe_round(LlamaEngine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* d_tokens, uint32_t* d_count,
                     void* stream) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(p != nullptr, CLM_INVALID_ARGUMENT, "null params");
  Session* s = nullptr;
  CLM_TRY(pipe_session(e, id, p->q, &s));
  cudaStream_t st = pick_stream(e->ctx, stream);
  const bool stochastic = p->temperature > 0.0f;
  if (e->spec.role == CLM_ROLE_TAIL) {
    RoundCtl c{p->temperature, 0u, (unsigned long long)p->seed};
    CLM_CUDA(cudaMemcpyAsync(e->ctl, &c, sizeof(c), cudaMemcpyHostToDevice, st));
  }
  CLM_TRY(e->run_graph(*s, 5, (int)p->q, stochastic ? 1 : 0, st,
                       [&](cudaStream_t cs) { return e->enqueue_pipe_round(*s, (int)p->q, stochastic, cs); }));
  if (e->spec.role == CLM_ROLE_TAIL) {
    if (d_tokens)
      CLM_CUDA(cudaMemcpyAsync(d_tokens, e->emitted, (p->q + 1) * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    if (d_count) CLM_CUDA(cudaMemcpyAsync(d_count, e->count, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
  }
  s->pos_bound += p->q;
  s->pos_stale = true;
  return CLM_OK;
}

int llama_pipe_status(LlamaEngine* e, void* stream) {
  CLM_TRY(engine_enter(e));
  return e->check_bad(pick_stream(e->ctx, stream));
}

int llama_spec_round(LlamaEngine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* h_tokens,
                        uint32_t* h_count) {
  CLM_TRY(engine_enter(e));
  CLM_CHECK(h_tokens != nullptr && h_count != nullptr, CLM_INVALID_ARGUMENT, "null output");
  cudaStream_t st = e->ctx->stream;
  CLM_TRY(llama_spec_round_device(e, id, p, nullptr, nullptr, st));
  CLM_CUDA(cudaMemcpyAsync(h_count, e->count, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  CLM_CUDA(cudaMemcpyAsync(h_tokens, e->emitted, (p->q + 1) * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  CLM_CUDA(cudaStreamSynchronize(st));
  Session* s = find_session(e, id);
  s->pos += *h_count;
  s->pos_bound = s->pos;
  s->pos_stale = false;
  return CLM_OK;
}

}  // namespace clm
