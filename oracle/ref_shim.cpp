// ref_shim.cpp — extern "C" entry points over the REFERENCE's own compiled code (TEST INFRASTRUCTURE).
//
// oracle/Makefile compiles this file together with the reference's runtime sources, unmodified and in
// place, into oracle/_ref/libclm_ref.so.  Tests use it to pin the C restatement (oracle.c) and to produce
// golden vectors; bench.py's reference arm times it.  Nothing in the product links it.
//
// Each wrapper calls exactly one reference API and converts plain pointers to the reference's types.
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "clusterlm/domain/drafter.hpp"
#include "clusterlm/domain/reference_domain.hpp"
#include "clusterlm/domain/reference_kernels.hpp"
#include "clusterlm/domain/sampling.hpp"
#include "clusterlm/objects/canonical_store.hpp"
#include "clusterlm/objects/fixture_model.hpp"
#include "clusterlm/objects/tensor_codec.hpp"

using namespace clusterlm;

namespace {
thread_local std::string g_err;
int fail(const Status& st) {
  g_err = st.to_string();
  return static_cast<int>(st.code()) == 0 ? 17 : static_cast<int>(st.code());
}
const char* quant_name(int q) {
  switch (q) {
    case 0: return "f32";
    case 1: return "q8_0-fixture";
    case 2: return "q8_0";
    default: return "unknown";
  }
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// ---- codecs: runtime/objects/src/tensor_codec.cpp ----
float ref_half_to_float(std::uint16_t h) { return objects::half_to_float(h); }
std::uint16_t ref_float_to_half(float f) { return objects::float_to_half(f); }
std::uint64_t ref_tensor_bytes(int quant, std::uint64_t n) { return objects::tensor_bytes(quant_name(quant), n); }
int ref_decode_tensor(int quant, const std::uint8_t* bytes, std::uint64_t nbytes, float* out, std::uint64_t n) {
  Status st = objects::decode_tensor(quant_name(quant), ByteSpan(bytes, nbytes), std::span<float>(out, n));
  return st.is_ok() ? 0 : fail(st);
}
int ref_encode(int quant, const float* v, std::uint64_t n, std::uint8_t* out, std::uint64_t out_cap) {
  Bytes b;
  Status st = quant == 1 ? objects::encode_q8_fixture(std::span<const float>(v, n), b)
                         : objects::encode_q8_0_ggml(std::span<const float>(v, n), b);
  if (!st.is_ok()) return fail(st);
  if (b.size() > out_cap) return 6;
  std::memcpy(out, b.data(), b.size());
  return 0;
}

// ---- reference kernels: runtime/domain/src/reference_kernels.cpp ----
void ref_matmul_rows(const float* w, std::uint64_t rows, std::uint64_t cols, const float* x, std::uint64_t positions,
                     float* y) {
  domain::reference_matmul_rows(w, rows, cols, x, positions, y);
}
void ref_matvec(const float* w, std::uint64_t rows, std::uint64_t cols, const float* x, float* y) {
  domain::reference_matvec(w, rows, cols, x, y);
}

// ---- sampling: runtime/domain/src/sampling.cpp ----
void ref_rng_uniforms(std::uint64_t seed, std::uint64_t n, double* out) {
  domain::Rng r(seed);
  for (std::uint64_t i = 0; i < n; ++i) out[i] = r.uniform();
}
std::uint64_t ref_mix_seed(std::uint64_t a, std::uint64_t b) { return domain::mix_seed(a, b); }
std::int32_t ref_argmax(const float* logits, std::uint64_t n) {
  return domain::argmax_token(std::span<const float>(logits, n));
}
void ref_distribution(const float* logits, std::uint64_t n, float temperature, std::uint32_t top_k, float top_p,
                      float* out) {
  domain::SamplingParams p;
  p.temperature = temperature;
  p.top_k = top_k;
  p.top_p = top_p;
  auto d = domain::distribution(std::span<const float>(logits, n), p);
  std::memcpy(out, d.data(), n * sizeof(float));
}
std::int32_t ref_sample_from(const float* probs, std::uint64_t n, std::uint64_t seed) {
  domain::Rng r(seed);
  return domain::sample_from(std::span<const float>(probs, n), r);
}
// verify_speculative for `batch` sequences; sequence b uses Rng(seeds[b]).
void ref_verify_speculative(const float* target, const std::int32_t* drafts, const float* draft_probs,
                            std::uint32_t batch, std::uint32_t k, std::uint64_t vocab, const std::uint64_t* seeds,
                            std::uint32_t* accepted, std::int32_t* next) {
  for (std::uint32_t b = 0; b < batch; ++b) {
    std::vector<std::vector<float>> t, q;
    const float* tb = target + std::uint64_t{b} * (k + 1) * vocab;
    for (std::uint32_t j = 0; j <= k; ++j) t.emplace_back(tb + j * vocab, tb + (j + 1) * vocab);
    if (draft_probs != nullptr) {
      const float* qb = draft_probs + std::uint64_t{b} * k * vocab;
      for (std::uint32_t j = 0; j < k; ++j) q.emplace_back(qb + j * vocab, qb + (j + 1) * vocab);
    }
    domain::Rng r(seeds[b]);
    auto o = domain::verify_speculative(t, std::span<const std::int32_t>(drafts + std::uint64_t{b} * k, k), q, r);
    accepted[b] = o.accepted_drafts;
    next[b] = o.next_token;
  }
}
// ScriptedDrafter::draft (runtime/domain/src/drafter.cpp:91-109).
void ref_scripted_draft(const std::int32_t* ref, std::uint64_t ref_len, std::uint32_t vocab, std::uint64_t seed,
                        double rate, std::uint64_t committed_len, std::uint32_t count, std::int32_t* out) {
  domain::ScriptedDrafter::Config c;
  c.vocab = vocab;
  c.seed = seed;
  c.corruption_rate = rate;
  domain::ScriptedDrafter d(std::vector<std::int32_t>(ref, ref + ref_len), c);
  std::vector<std::int32_t> committed(committed_len, 0);
  auto r = d.draft(committed, 0, count);
  std::memcpy(out, r.data(), r.size() * sizeof(std::int32_t));
}

// ---- fixture model: runtime/objects/src/fixture_model.cpp ----
int ref_write_fixture(const char* dir, int tiny, std::uint32_t layers, std::uint64_t seed) {
  objects::FixtureSpec s = tiny ? objects::FixtureSpec::tiny() : objects::FixtureSpec{};
  if (layers) s.n_layers = layers;
  s.seed = seed;
  auto m = objects::write_fixture_model(s, dir);
  return m.is_ok() ? 0 : fail(m.status());
}

// ---- canonical model store: object bytes by manifest name (runtime/objects/src/canonical_store.cpp)
void* ref_store_open(const char* dir) {
  auto st = objects::CanonicalModelStore::open(dir);
  if (!st.is_ok()) {
    fail(st.status());
    return nullptr;
  }
  return std::move(st).value().release();
}
void ref_store_close(void* h) { delete static_cast<objects::CanonicalModelStore*>(h); }
// quant: 0 f32, 1 q8_0-fixture, 2 q8_0, -1 other.  Returns 0 and the byte count; copies when cap suffices.
int ref_store_object(void* h, const char* name, std::uint8_t* buf, std::uint64_t cap, int* quant,
                     std::uint64_t* nbytes) {
  auto* s = static_cast<objects::CanonicalModelStore*>(h);
  auto p = s->resolve(name);
  if (!p.is_ok()) return fail(p.status());
  const std::string& qt = p->entry->representation.quant_type;
  *quant = qt == "f32" ? 0 : qt == "q8_0-fixture" ? 1 : qt == "q8_0" ? 2 : -1;
  *nbytes = p->bytes.size();
  if (buf && cap >= p->bytes.size()) std::memcpy(buf, p->bytes.data(), p->bytes.size());
  return 0;
}
// geometry: 15 u32 fields then layer kinds (n_layers bytes)
int ref_store_geometry(void* h, std::uint32_t* dims, std::uint8_t* kinds, std::uint32_t kinds_cap) {
  auto* s = static_cast<objects::CanonicalModelStore*>(h);
  const auto& g = s->manifest().geometry;
  const std::uint32_t v[15] = {g.n_layers, g.hidden_size, g.residual_streams, g.n_experts, g.n_active_experts,
                               g.expert_ff, g.shared_expert_ff, g.n_heads, g.n_kv_heads, g.head_dim,
                               g.vocab_size, g.ple_layer, g.ple_ngram, g.ple_rows, g.mtp_layers};
  std::memcpy(dims, v, sizeof v);
  for (std::uint32_t i = 0; i < g.n_layers && i < kinds_cap; ++i) kinds[i] = static_cast<std::uint8_t>(g.layer_kinds[i]);
  return 0;
}

// ---- in-process pipeline over ReferenceDomain (the pattern of tests/domain/pipeline_harness.hpp) ----
struct RefPipeline {
  std::unique_ptr<objects::CanonicalModelStore> store;
  std::vector<std::unique_ptr<domain::ReferenceDomain>> stages;
  std::unique_ptr<domain::MtpFixtureDrafter> mtp;
  std::uint32_t max_window = 0;
  std::uint64_t epoch = 1, session = 1;
};

void* ref_pipeline_create(const char* dir, const std::uint32_t* bounds, std::uint32_t nbounds,
                          std::uint32_t max_context, std::uint32_t max_window) {
  auto p = std::make_unique<RefPipeline>();
  auto st = objects::CanonicalModelStore::open(dir);
  if (!st.is_ok()) {
    fail(st.status());
    return nullptr;
  }
  p->store = std::move(st).value();
  p->max_window = max_window;
  const std::size_t n = nbounds - 1;
  for (std::size_t i = 0; i < n; ++i) {
    domain::DomainSpec spec;
    spec.stage = StageId{static_cast<std::uint32_t>(i)};
    spec.role = i == 0 ? domain::StageRole::kPrefix : (i + 1 == n ? domain::StageRole::kTail : domain::StageRole::kMiddle);
    spec.layers = {bounds[i], bounds[i + 1]};
    spec.max_context = max_context;
    spec.max_window = max_window;
    spec.max_sessions = 4;
    auto d = domain::ReferenceDomain::create(p->store->manifest(), spec);
    if (!d.is_ok()) {
      fail(d.status());
      return nullptr;
    }
    Status s = (*d)->prepare(*p->store);
    if (!s.is_ok()) {
      fail(s);
      return nullptr;
    }
    if (!(*d)->open_session(Epoch{p->epoch}, SessionId{p->session}).is_ok()) return nullptr;
    p->stages.push_back(std::move(d).value());
  }
  auto m = domain::MtpFixtureDrafter::create(p->store->manifest(), *p->store);
  if (m.is_ok()) p->mtp = std::move(m).value();
  return p.release();
}

void ref_pipeline_destroy(void* h) { delete static_cast<RefPipeline*>(h); }

// Runs one window through every stage (activations copied between stages as values, exactly as the wire
// would carry them).  stage_out (optional) receives each stage's output record, stage-major.
int ref_pipeline_run(void* h, std::uint64_t window_id, std::uint64_t base, std::uint64_t state,
                     const std::int32_t* tokens, std::uint32_t q, float* logits, float* stage_out) {
  auto* p = static_cast<RefPipeline*>(h);
  domain::WindowRequest req;
  req.epoch = Epoch{p->epoch};
  req.session = SessionId{p->session};
  req.window = WindowId{window_id};
  req.base_position = base;
  req.expected_state = StateVersion{state};
  req.positions = q;
  auto act = p->stages.front()->run_prefix(req, std::span<const std::int32_t>(tokens, q));
  if (!act.is_ok()) return fail(act.status());
  domain::StageActivations cur = std::move(act).value();
  std::size_t off = 0;
  auto keep = [&](const domain::StageActivations& a) {
    if (stage_out) std::memcpy(stage_out + off, a.data.data(), a.data.size() * sizeof(float));
    off += a.data.size();
  };
  keep(cur);
  for (std::size_t i = 1; i + 1 < p->stages.size(); ++i) {
    auto next = p->stages[i]->run_window(req, cur);
    if (!next.is_ok()) return fail(next.status());
    cur = std::move(next).value();
    keep(cur);
  }
  auto l = p->stages.back()->run_tail(req, cur);
  if (!l.is_ok()) return fail(l.status());
  std::memcpy(logits, l->data.data(), l->data.size() * sizeof(float));
  return 0;
}

int ref_pipeline_commit(void* h, std::uint64_t window_id, std::uint64_t state, std::uint32_t accepted) {
  auto* p = static_cast<RefPipeline*>(h);
  domain::CommitRequest c;
  c.epoch = Epoch{p->epoch};
  c.session = SessionId{p->session};
  c.window = WindowId{window_id};
  c.accepted = accepted;
  c.expected_state = StateVersion{state};
  for (auto& s : p->stages) {
    auto a = s->commit_window(c);
    if (!a.is_ok()) return fail(a.status());
  }
  return 0;
}

int ref_pipeline_abort(void* h, std::uint64_t window_id) {
  auto* p = static_cast<RefPipeline*>(h);
  for (auto& s : p->stages) {
    auto a = s->abort_window(Epoch{p->epoch}, SessionId{p->session}, WindowId{window_id});
    if (!a.is_ok()) return fail(a.status());
  }
  return 0;
}

std::int32_t ref_pipeline_mtp_step(void* h, std::int32_t prev) {
  auto* p = static_cast<RefPipeline*>(h);
  return p->mtp ? p->mtp->step(prev) : -1;
}

int ref_pipeline_mtp_logits(void* h, std::int32_t prev, float* out) {
  auto* p = static_cast<RefPipeline*>(h);
  if (!p->mtp) return 5;
  auto l = p->mtp->step_logits(prev);
  std::memcpy(out, l.data(), l.size() * sizeof(float));
  return 0;
}

}  // extern "C"
