// Drop-in parity driver: the reference's ReferenceDomain pipeline and the b200 backend's pipeline over the same
// fixture model, plan and requests, through the reference's own BackendAdapter / ExecutionDomain / Drafter
// interfaces (runtime/domain/include/clusterlm/domain/backend_adapter.hpp:14-27, execution_domain.hpp:143-174).
//
//   backend_parity <scratch dir> [--bench]
//   backend_parity <scratch dir> --llama <model.gguf>
//
// Checks (each prints PASS/FAIL; the exit status is the number of failures):
//   * greedy speculative generation (ScriptedDrafter, corruption 0.3, q = 4, 32 new tokens; plan 0-4|4-10|10-13|13-16)
//     gives the same windows, accepted counts and tokens; logits within 1e-4 (absolute) with the same argmax;
//   * stage-level drop-in: mixed pipelines (reference prefix + b200 middles + reference tail and the converse);
//   * a tail's run_window returns the same activation records as the reference;
//   * admission, commit and abort rules (ledger errors, idempotent commit replay, abort then re-run);
//   * the GPU MTP drafter drafts the same tokens as MtpFixtureDrafter.
// With --bench it also times windows per second of both pipelines (q = 4 windows, 1 thread each).
// With --llama, a llama GGUF file's ModelManifest (the reference's build_llama_manifest) drives a 3-stage pipeline of
// b200 domains (prefix, middle, tail; tensors named from the file's directory, bytes from an ObjectResolver over the
// file) whose logits must equal, bit for bit, a whole-model engine loaded from the same file through the C ABI; plus
// the domains' requirements and the stochastic MTP proposal when the file has an MTP head.
// Activations cross every stage boundary through the wire encoding (StageActivations::encode / decode).
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "clusterlm/common/bytes.hpp"
#include "clusterlm/domain/backend_adapter.hpp"
#include "clusterlm/domain/drafter.hpp"
#include "clusterlm/domain/sampling.hpp"
#include "clusterlm/backends/llama_manifest.hpp"
#include "clusterlm/objects/canonical_store.hpp"
#include "clusterlm/objects/fixture_model.hpp"
#include "clusterlm/objects/gguf.hpp"
#include "../../include/clm_b200.h"
#include "../../clusterlm_b200/backend/b200_backend.hpp"

using namespace clusterlm;
using namespace clusterlm::domain;

namespace {

int g_failures = 0;

void check(bool ok, const std::string& name, const std::string& detail = "") {
  std::printf("%s %s%s%s\n", ok ? "PASS" : "FAIL", name.c_str(), detail.empty() ? "" : ": ", detail.c_str());
  std::fflush(stdout);
  if (!ok) ++g_failures;
}

std::int32_t argmax_row(const float* row, std::uint32_t n) {
  std::uint32_t best = 0;
  for (std::uint32_t i = 1; i < n; ++i)
    if (row[i] > row[best]) best = i;
  return static_cast<std::int32_t>(best);
}

StageActivations wire(const StageActivations& a, std::uint32_t max_positions) {
  ByteWriter w;
  a.encode(w);
  ByteReader r(w.bytes());
  auto back = StageActivations::decode(r, max_positions);
  if (!back.is_ok()) {
    check(false, "wire decode", back.status().to_string());
    return a;
  }
  return std::move(back).value();
}

struct Pipeline {
  std::vector<std::unique_ptr<ExecutionDomain>> stages;
  std::uint32_t max_window = 8;
  Epoch epoch{1};
  SessionId session{1};

  // backends[i] builds stage i.
  static std::unique_ptr<Pipeline> build(const objects::ModelManifest& m, const objects::ObjectResolver& store,
                                         const std::vector<std::uint32_t>& bounds,
                                         const std::vector<BackendAdapter*>& backends, std::uint32_t max_context,
                                         std::uint32_t max_window) {
    auto p = std::make_unique<Pipeline>();
    p->max_window = max_window;
    const std::size_t n = bounds.size() - 1;
    for (std::size_t i = 0; i < n; ++i) {
      DomainSpec spec;
      spec.stage = StageId{static_cast<std::uint32_t>(i)};
      spec.role = i == 0 ? StageRole::kPrefix : (i + 1 == n ? StageRole::kTail : StageRole::kMiddle);
      spec.layers = {bounds[i], bounds[i + 1]};
      spec.max_context = max_context;
      spec.max_window = max_window;
      spec.max_sessions = 4;
      auto d = backends[i]->create_domain(m, spec);
      if (!d.is_ok()) {
        check(false, "create_domain stage " + std::to_string(i), d.status().to_string());
        return nullptr;
      }
      const Status st = (*d)->prepare(store);
      if (!st.is_ok()) {
        check(false, "prepare stage " + std::to_string(i), st.to_string());
        return nullptr;
      }
      p->stages.push_back(std::move(d).value());
    }
    return p;
  }

  Status open() {
    for (auto& s : stages) CLM_RETURN_IF_ERROR(s->open_session(epoch, session));
    return Status::ok();
  }

  Result<Logits> run(const WindowRequest& req, std::span<const std::int32_t> tokens,
                     std::vector<StageActivations>* hops = nullptr) {
    auto act = stages.front()->run_prefix(req, tokens);
    if (!act.is_ok()) return act.status();
    StageActivations cur = wire(*act, max_window);
    if (hops) hops->push_back(cur);
    for (std::size_t i = 1; i + 1 < stages.size(); ++i) {
      auto next = stages[i]->run_window(req, cur);
      if (!next.is_ok()) return next.status();
      cur = wire(*next, max_window);
      if (hops) hops->push_back(cur);
    }
    return stages.back()->run_tail(req, cur);
  }

  Result<CommitAck> commit(const CommitRequest& c) {
    Result<CommitAck> last = make_error(ErrorCode::kInternal, "no stages");
    for (auto& s : stages) {
      last = s->commit_window(c);
      if (!last.is_ok()) return last;
    }
    return last;
  }
};

struct Trace {
  std::vector<std::vector<std::int32_t>> windows;
  std::vector<std::uint32_t> accepted;
  std::vector<std::vector<float>> logits;
  std::vector<std::int32_t> generated;
  bool ok = true;
  std::string error;
};

// Greedy speculative generation (Coordinator::generate's acceptance rule, coordinator.cpp:1295-1298): prefill the
// prompt in chunks of max_window, then windows [next, drafts...] with accepted = 1 + longest matching prefix.
Trace generate(Pipeline& p, const std::vector<std::int32_t>& prompt, std::uint32_t n_new, Drafter* drafter,
               std::uint32_t q, std::uint32_t vocab) {
  Trace t;
  if (Status st = p.open(); !st.is_ok()) {
    t.ok = false;
    t.error = st.to_string();
    return t;
  }
  std::uint64_t wid = 0, base = 0, state = 0;
  std::vector<std::int32_t> committed;
  std::int32_t next = 0;
  auto step = [&](const std::vector<std::int32_t>& toks, bool prefill) -> bool {
    WindowRequest req;
    req.epoch = p.epoch;
    req.session = p.session;
    req.window = WindowId{++wid};
    req.base_position = base;
    req.expected_state = StateVersion{state};
    req.positions = static_cast<std::uint32_t>(toks.size());
    auto l = p.run(req, toks);
    if (!l.is_ok()) {
      t.ok = false;
      t.error = l.status().to_string();
      return false;
    }
    std::uint32_t acc = req.positions;
    if (!prefill) {
      acc = 1;
      for (std::uint32_t i = 0; i + 1 < toks.size(); ++i) {
        if (argmax_row(l->data.data() + std::size_t{i} * vocab, vocab) != toks[i + 1]) break;
        ++acc;
      }
    }
    CommitRequest c;
    c.epoch = p.epoch;
    c.session = p.session;
    c.window = req.window;
    c.accepted = acc;
    c.expected_state = StateVersion{state};
    auto ack = p.commit(c);
    if (!ack.is_ok()) {
      t.ok = false;
      t.error = ack.status().to_string();
      return false;
    }
    state = ack->state.value;
    base += acc;
    committed.insert(committed.end(), toks.begin(), toks.begin() + acc);
    next = argmax_row(l->data.data() + std::size_t{acc - 1} * vocab, vocab);
    t.windows.push_back(toks);
    t.accepted.push_back(acc);
    t.logits.push_back(l->data);
    return true;
  };
  for (std::size_t i = 0; i < prompt.size(); i += p.max_window) {
    const std::size_t n = std::min<std::size_t>(p.max_window, prompt.size() - i);
    if (!step(std::vector<std::int32_t>(prompt.begin() + i, prompt.begin() + i + n), true)) return t;
  }
  while (t.generated.size() < n_new) {
    std::vector<std::int32_t> w{next};
    if (drafter != nullptr && q > 1) {
      auto d = drafter->draft(committed, next, q - 1);
      w.insert(w.end(), d.begin(), d.end());
    }
    const std::size_t before = committed.size();
    if (!step(w, false)) return t;
    for (std::size_t i = before; i < committed.size() && t.generated.size() < n_new; ++i)
      t.generated.push_back(committed[i]);
  }
  return t;
}

void compare_traces(const Trace& a, const Trace& b, std::uint32_t vocab, const std::string& name) {
  if (!a.ok || !b.ok) {
    check(false, name, "generation failed: " + a.error + " | " + b.error);
    return;
  }
  bool same_windows = a.windows == b.windows && a.accepted == b.accepted && a.generated == b.generated;
  double worst = 0.0;
  bool same_argmax = true;
  for (std::size_t w = 0; w < std::min(a.logits.size(), b.logits.size()); ++w) {
    const auto& x = a.logits[w];
    const auto& y = b.logits[w];
    if (x.size() != y.size()) {
      same_windows = false;
      continue;
    }
    for (std::size_t i = 0; i < x.size(); ++i) worst = std::max(worst, (double)std::fabs(x[i] - y[i]));
    for (std::size_t r = 0; r < x.size() / vocab; ++r)
      same_argmax &= argmax_row(x.data() + r * vocab, vocab) == argmax_row(y.data() + r * vocab, vocab);
  }
  char buf[160];
  std::snprintf(buf, sizeof buf, "%zu windows, %zu tokens, max |dlogit| %.3g", a.windows.size(), a.generated.size(), worst);
  check(same_windows && same_argmax && worst <= 1e-4, name, buf);
}

WindowRequest request(std::uint64_t window, std::uint64_t base, std::uint64_t state, std::uint32_t q,
                      std::uint64_t epoch = 1) {
  WindowRequest r;
  r.epoch = Epoch{epoch};
  r.session = SessionId{1};
  r.window = WindowId{window};
  r.base_position = base;
  r.expected_state = StateVersion{state};
  r.positions = q;
  return r;
}

void admission_rules(BackendAdapter& b200, const objects::ModelManifest& m, const objects::ObjectResolver& store,
                     BackendAdapter& ref) {
  const std::vector<std::uint32_t> bounds{0, 4, 10, 13, 16};
  auto p = Pipeline::build(m, store, bounds, {&b200, &b200, &b200, &b200}, 64, 8);
  auto r = Pipeline::build(m, store, bounds, {&ref, &ref, &ref, &ref}, 64, 8);
  if (!p || !r) return;
  check(p->open().is_ok() && r->open().is_ok(), "open sessions");
  const std::vector<std::int32_t> toks{1, 2, 3, 4};
  auto& prefix = *p->stages.front();
  auto& middle = *p->stages[1];
  auto& tail = *p->stages.back();

  // role errors
  auto e1 = middle.run_prefix(request(1, 0, 0, 4), toks);
  check(!e1.is_ok() && e1.status().code() == ErrorCode::kFailedPrecondition, "run_prefix on a middle stage refused");
  // stale epoch
  auto e2 = prefix.run_prefix(request(1, 0, 0, 4, 7), toks);
  check(!e2.is_ok() && e2.status().code() == ErrorCode::kStaleEpoch, "stale epoch refused",
        e2.is_ok() ? "accepted" : e2.status().to_string());
  // window larger than max_window
  std::vector<std::int32_t> big(9, 1);
  auto e3 = prefix.run_prefix(request(2, 0, 0, 9), big);
  check(!e3.is_ok() && e3.status().code() == ErrorCode::kResourceExhausted, "window > max_window refused");
  // token outside the vocabulary
  std::vector<std::int32_t> bad{1, 2, 999, 4};
  auto e4 = prefix.run_prefix(request(3, 0, 0, 4), bad);
  check(!e4.is_ok() && e4.status().code() == ErrorCode::kInvalidArgument, "token outside vocabulary refused");

  // a good window through all stages, same logits as the reference
  std::vector<StageActivations> hops_b, hops_r;
  auto lb = p->run(request(4, 0, 0, 4), toks, &hops_b);
  auto lr = r->run(request(4, 0, 0, 4), toks, &hops_r);
  check(lb.is_ok() && lr.is_ok(), "window 4 runs", lb.is_ok() ? "" : lb.status().to_string());
  if (lb.is_ok() && lr.is_ok()) {
    double worst = 0;
    for (std::size_t i = 0; i < lb->data.size(); ++i) worst = std::max(worst, (double)std::fabs(lb->data[i] - lr->data[i]));
    double hop = 0;
    for (std::size_t h = 0; h < hops_b.size(); ++h)
      for (std::size_t i = 0; i < hops_b[h].data.size(); ++i)
        hop = std::max(hop, (double)std::fabs(hops_b[h].data[i] - hops_r[h].data[i]));
    char buf[96];
    std::snprintf(buf, sizeof buf, "max |dlogit| %.3g, max |drecord| %.3g", worst, hop);
    check(worst <= 1e-4 && hop <= 1e-4, "window logits and stage records match the reference", buf);
  }
  // a second window while one is outstanding
  auto e5 = prefix.run_prefix(request(5, 0, 0, 4), toks);
  check(!e5.is_ok(), "second outstanding window refused");
  // a repeated (old) window id after the failed one
  auto e6 = prefix.run_prefix(request(4, 0, 0, 4), toks);
  check(!e6.is_ok(), "repeated window id refused");

  // commit 2 of 4 on every stage; replay is idempotent with the identical ack
  CommitRequest c;
  c.epoch = Epoch{1};
  c.session = SessionId{1};
  c.window = WindowId{4};
  c.accepted = 2;
  c.expected_state = StateVersion{0};
  auto a1 = p->commit(c);
  auto a2 = p->commit(c);
  check(a1.is_ok() && a2.is_ok() && *a1 == *a2 && a1->committed_position == 2, "commit and idempotent replay",
        a1.is_ok() ? "" : a1.status().to_string());
  auto rc1 = r->commit(c);
  check(rc1.is_ok() && a1.is_ok() && *rc1 == *a1, "commit ack equals the reference's ack");
  const std::uint64_t st = a1.is_ok() ? a1->state.value : 0;
  // wrong base position after commit
  auto e7 = prefix.run_prefix(request(6, 0, st, 2), std::vector<std::int32_t>{5, 6});
  check(!e7.is_ok(), "window at a stale base refused");

  // abort a window, then run the same positions again: same logits as running them directly (reference)
  std::vector<std::int32_t> t2{7, 8, 9};
  auto x1 = p->run(request(7, 2, st, 3), t2);
  bool aborted = x1.is_ok();
  for (auto& s : p->stages) aborted &= s->abort_window(Epoch{1}, SessionId{1}, WindowId{7}).is_ok();
  for (auto& s : p->stages) aborted &= s->abort_window(Epoch{1}, SessionId{1}, WindowId{7}).is_ok();  // harmless repeat
  check(aborted, "abort_window (and its repeat)");
  auto x2 = p->run(request(8, 2, st, 3), t2);
  auto y2 = r->run(request(8, 2, st, 3), t2);
  if (x2.is_ok() && y2.is_ok()) {
    double worst = 0;
    for (std::size_t i = 0; i < x2->data.size(); ++i) worst = std::max(worst, (double)std::fabs(x2->data[i] - y2->data[i]));
    check(worst <= 1e-4, "re-run after abort matches the reference", std::to_string(worst));
  } else {
    check(false, "re-run after abort", x2.is_ok() ? y2.status().to_string() : x2.status().to_string());
  }
  auto metrics = tail.read_metrics();
  check(metrics.windows_run >= 2 && metrics.windows_committed >= 1, "metrics count windows");
  check(prefix.abort_session(Epoch{1}, SessionId{1}).is_ok(), "abort_session");
  auto e8 = prefix.run_prefix(request(10, 0, 0, 1), std::vector<std::int32_t>{1});
  check(!e8.is_ok(), "window on an aborted session refused");
  check(prefix.release().is_ok() && !prefix.open_session(Epoch{1}, SessionId{1}).is_ok(), "release drops the domain");
  check(prefix.prepare(store).is_ok() && prefix.open_session(Epoch{2}, SessionId{1}).is_ok(), "prepare again after release");
}

void tail_records(BackendAdapter& b200, BackendAdapter& ref, const objects::ModelManifest& m,
                  const objects::ObjectResolver& store) {
  // prefix (reference) -> tail stage 4..16 run_window on both backends: identical records expected within 1e-4
  auto p = Pipeline::build(m, store, {0, 4, 16}, {&ref, &ref}, 64, 8);
  auto tb = Pipeline::build(m, store, {0, 4, 16}, {&ref, &b200}, 64, 8);
  if (!p || !tb) return;
  check(p->open().is_ok() && tb->open().is_ok(), "open tail sessions");
  const std::vector<std::int32_t> toks{3, 1, 4, 1, 5};
  auto a = p->stages[0]->run_prefix(request(1, 0, 0, 5), toks);
  if (!a.is_ok()) return check(false, "tail prefix", a.status().to_string());
  auto rr = p->stages[1]->run_window(request(1, 0, 0, 5), *a);
  auto rb = tb->stages[1]->run_window(request(1, 0, 0, 5), *a);
  if (!rr.is_ok() || !rb.is_ok()) return check(false, "tail run_window", rb.is_ok() ? rr.status().to_string() : rb.status().to_string());
  double worst = 0;
  for (std::size_t i = 0; i < rr->data.size(); ++i) worst = std::max(worst, (double)std::fabs(rr->data[i] - rb->data[i]));
  check(rr->data.size() == rb->data.size() && worst <= 1e-4, "tail run_window returns the reference's records",
        std::to_string(worst));
}

double time_windows(Pipeline& p, int n) {
  if (!p.open().is_ok()) return 0.0;
  std::vector<std::int32_t> toks{1, 2, 3, 4};
  std::uint64_t base = 0, state = 0;
  const auto t0 = std::chrono::steady_clock::now();
  for (int i = 0; i < n; ++i) {
    auto l = p.run(request(i + 1, base, state, 4), toks);
    if (!l.is_ok()) return 0.0;
    CommitRequest c;
    c.epoch = p.epoch;
    c.session = p.session;
    c.window = WindowId{static_cast<std::uint64_t>(i + 1)};
    c.accepted = 4;
    c.expected_state = StateVersion{state};
    auto ack = p.commit(c);
    if (!ack.is_ok()) return 0.0;
    state = ack->state.value;
    base += 4;
  }
  return n / std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// ObjectResolver over a model's GGUF files: each object is its source ranges read and concatenated (what a
// Node's lease store provisions for the manifest).
class GgufResolver final : public objects::ObjectResolver {
 public:
  GgufResolver(const objects::ModelManifest& m, const std::filesystem::path& dir) : m_(m), dir_(dir) {}
  Result<objects::ProvisionedObject> resolve(std::string_view name) const override {
    const objects::ManifestObject* o = m_.find(name);
    if (o == nullptr) return make_error(ErrorCode::kNotFound, "no object " + std::string(name));
    auto& buf = cache_[std::string(name)];
    if (buf.empty()) {
      for (const auto& r : o->source_ranges) {
        std::ifstream f(dir_ / m_.shards[r.shard].file_name, std::ios::binary);
        f.seekg(static_cast<std::streamoff>(r.offset));
        const std::size_t at = buf.size();
        buf.resize(at + r.length);
        f.read(reinterpret_cast<char*>(buf.data() + at), static_cast<std::streamsize>(r.length));
        if (!f) return make_error(ErrorCode::kDataLoss, "short read of " + std::string(name));
      }
    }
    objects::ProvisionedObject p;
    p.entry = o;
    p.bytes = std::span<const std::uint8_t>(buf.data(), buf.size());
    return p;
  }

 private:
  const objects::ModelManifest& m_;
  std::filesystem::path dir_;
  mutable std::map<std::string, std::vector<std::uint8_t>> cache_;
};

int llama_mode(const std::filesystem::path& gguf) {
  auto mm = backends::build_llama_manifest({gguf});
  if (!mm.is_ok()) {
    std::fprintf(stderr, "manifest: %s\n", mm.status().to_string().c_str());
    return 2;
  }
  const objects::ModelManifest m = std::move(mm).value();
  const auto& g = m.geometry;
  const std::uint32_t V = g.vocab_size, L = g.n_layers;
  check(g.family == "llama.cpp:llama" && g.residual_streams == 1 && L >= 3, "llama manifest geometry",
        g.family + " layers " + std::to_string(L));
  GgufResolver store(m, gguf.parent_path());
  backends::B200BackendOptions opt;
  opt.model_dir = gguf.parent_path();
  auto b200 = backends::make_b200_backend(opt);
  // the same domains without model_dir are refused at create_domain
  {
    auto plain = backends::make_b200_backend();
    DomainSpec spec;
    spec.role = StageRole::kPrefix;
    spec.layers = {0, 1};
    spec.max_context = 64;
    spec.max_window = 8;
    auto d = plain->create_domain(m, spec);
    check(!d.is_ok() && d.status().code() == ErrorCode::kFailedPrecondition, "llama domain without model_dir refused");
  }
  const std::vector<std::uint32_t> plan{0, 1, L - 1, L};
  auto bp = Pipeline::build(m, store, plan, {b200.get(), b200.get(), b200.get()}, 128, 8);
  if (!bp) return g_failures;
  {  // requirements of the middle stage: its layers' objects, the KV pages of its layers
    const auto req = bp->stages[1]->describe_requirements();
    std::uint64_t want = 0;
    for (std::uint32_t l = 1; l + 1 < L; ++l) want += m.find(objects::dense_object_name(l))->byte_size;
    const std::uint64_t kv = std::uint64_t{L - 2} * 2 * 128 * g.n_kv_heads * g.head_dim * 2 * 4;
    check(req.is_ok() && req->gpu_weight_bytes == want && req->state_bytes == kv &&
              req->required_objects.size() == L - 2,
          "llama middle-stage requirements (weights, KV pages, objects)");
  }
  // the whole model through the C ABI from the same file
  auto files = objects::open_gguf_model({gguf});
  if (!files.is_ok()) return 2;
  std::vector<std::vector<std::uint8_t>> data;
  std::vector<clm_b200_tensor> tensors;
  std::ifstream f(gguf, std::ios::binary);
  for (const auto& t : files->shards[0].tensors) {
    data.emplace_back(t.n_bytes);
    f.seekg(static_cast<std::streamoff>(t.file_offset));
    f.read(reinterpret_cast<char*>(data.back().data()), static_cast<std::streamsize>(t.n_bytes));
    const int ty = static_cast<int>(t.type);
    tensors.push_back(clm_b200_tensor{t.name.c_str(), ty == 0 ? CLM_QUANT_F32 : ty == 8 ? CLM_QUANT_Q8_0 : ty == 12 ? CLM_QUANT_Q4_K : -1 - ty,
                                      nullptr, t.n_bytes});
  }
  for (std::size_t i = 0; i < tensors.size(); ++i) tensors[i].data = data[i].data();
  clm_b200_ctx* cx = nullptr;
  clm_b200_engine* whole = nullptr;
  clm_b200_llama_geometry lg{};
  lg.n_layers = L;
  lg.hidden = g.hidden_size;
  lg.n_heads = g.n_heads;
  lg.n_kv_heads = g.n_kv_heads;
  lg.head_dim = g.head_dim;
  lg.ffn = g.expert_ff;
  lg.vocab = V;
  const objects::GgufValue* th = files->meta().find("llama.rope.freq_base");
  lg.rope_theta = th ? static_cast<float>(*th->as_double()) : 10000.0f;
  const objects::GgufValue* ep = files->meta().find("llama.attention.layer_norm_rms_epsilon");
  lg.rms_eps = ep ? static_cast<float>(*ep->as_double()) : 1e-5f;
  const auto qt = files->find_tensor("blk.0.attn_q.weight");
  lg.quant = qt && static_cast<int>(qt->info->type) == 8 ? CLM_QUANT_Q8_0 : CLM_QUANT_Q4_K;
  lg.mtp = files->find_tensor("mtp.ffn_gate.weight") ? 1 : 0;
  clm_b200_stage_spec ws{0, L, CLM_ROLE_WHOLE, 128, 8, 1};
  bool ok = clm_b200_ctx_create(0, &cx) == CLM_OK && clm_b200_llama_create(cx, &lg, &ws, &whole) == CLM_OK &&
            clm_b200_llama_load_tensors(whole, tensors.data(), static_cast<std::uint32_t>(tensors.size())) == CLM_OK &&
            clm_b200_engine_prepare(whole) == CLM_OK && clm_b200_session_open(whole, 1) == CLM_OK;
  check(ok, "whole-model engine from the GGUF file", ok ? "" : clm_b200_last_error());
  if (!ok) return g_failures;
  // windows through the pipeline and the whole engine: prefill 8, then q = 4 windows keeping 4, 2, 1, 3
  check(bp->open().is_ok(), "open llama pipeline sessions");
  Rng rng(7);
  std::uint64_t base = 0, state = 0, wid = 0;
  bool same = true;
  std::size_t windows = 0;
  const std::vector<std::pair<std::uint32_t, std::uint32_t>> steps{{8, 8}, {4, 4}, {4, 2}, {4, 1}, {4, 3}};
  for (auto [q, keep] : steps) {
    std::vector<std::int32_t> toks(q);
    for (auto& t : toks) t = static_cast<std::int32_t>(rng.uniform() * V);
    auto l = bp->run(request(++wid, base, state, q), toks);
    std::vector<float> want(std::size_t{q} * V);
    const int rc = clm_b200_run_window(whole, 1, base, q, toks.data(), nullptr, nullptr, want.data());
    if (!l.is_ok() || rc != CLM_OK) {
      check(false, "llama window", l.is_ok() ? clm_b200_last_error() : l.status().to_string());
      return g_failures;
    }
    same &= l->data == want;
    ++windows;
    CommitRequest c;
    c.epoch = bp->epoch;
    c.session = bp->session;
    c.window = WindowId{wid};
    c.accepted = keep;
    c.expected_state = StateVersion{state};
    auto ack = bp->commit(c);
    if (!ack.is_ok() || clm_b200_commit(whole, 1, keep) != CLM_OK) {
      check(false, "llama commit", ack.is_ok() ? clm_b200_last_error() : ack.status().to_string());
      return g_failures;
    }
    state = ack->state.value;
    base += keep;
  }
  check(same, "3-stage llama pipeline (b200 ExecutionDomain over the GGUF manifest) == whole-model engine, bitwise",
        std::to_string(windows) + " windows");
  if (lg.mtp) {  // the drafter bound to the llama tail: greedy draft and stochastic proposal rows
    auto drafter = backends::make_b200_mtp_drafter(*bp->stages.back());
    check(drafter.is_ok(), "MTP drafter bound to the llama tail", drafter.is_ok() ? "" : drafter.status().to_string());
    if (drafter.is_ok()) {
      SamplingParams sp;
      sp.temperature = 1.0f;
      Rng r1(11);
      auto prop = (*drafter)->propose({}, 5, 3, sp, r1);
      bool rows = prop.tokens.size() == 3 && prop.probs.size() == 3;
      for (std::size_t j = 0; rows && j < 3; ++j) {
        double tot = 0.0;
        for (float v : prop.probs[j]) tot += v;
        rows &= prop.probs[j].size() == V && std::fabs(tot - 1.0) < 1e-3 && prop.probs[j][prop.tokens[j]] > 0.0f;
      }
      check(rows, "llama MTP proposal: 3 drafts with their distributions");
    }
  }
  clm_b200_engine_destroy(whole);
  clm_b200_ctx_destroy(cx);
  std::printf("%d failure(s)\n", g_failures);
  return g_failures;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: backend_parity <scratch dir> [--bench]\n");
    return 2;
  }
  if (argc > 3 && std::strcmp(argv[2], "--llama") == 0) return llama_mode(argv[3]);
  const std::filesystem::path dir = std::filesystem::path(argv[1]) / "fixture";
  const bool bench = argc > 2 && std::strcmp(argv[2], "--bench") == 0;
  std::filesystem::create_directories(dir);
  objects::FixtureSpec spec;  // the default fixture (16 layers, H 64, hc 4, 32 experts top-4, V 256), seed "CLM1"
  auto wm = objects::write_fixture_model(spec, dir);
  if (!wm.is_ok()) {
    std::fprintf(stderr, "fixture: %s\n", wm.status().to_string().c_str());
    return 2;
  }
  auto so = objects::CanonicalModelStore::open(dir);
  if (!so.is_ok()) {
    std::fprintf(stderr, "store: %s\n", so.status().to_string().c_str());
    return 2;
  }
  auto store = std::move(so).value();
  const auto& m = store->manifest();
  const std::uint32_t V = m.geometry.vocab_size;

  auto ref = make_reference_backend();
  auto b200 = backends::make_b200_backend();
  const BackendInfo info = b200->info();
  check(info.name == "b200" && info.supports_gpu && info.hardware_available, "backend info",
        info.name + " " + info.build_hash);

  // the reference prompt: 16 ids uniform in [0, 256) from Rng(0)
  Rng rng(0);
  std::vector<std::int32_t> prompt(16);
  for (auto& t : prompt) t = static_cast<std::int32_t>(rng.uniform() * V);
  const std::vector<std::uint32_t> plan{0, 4, 10, 13, 16};

  {  // ScriptedDrafter needs the greedy continuation: run the reference once without a drafter
    auto rp = Pipeline::build(m, *store, plan, {ref.get(), ref.get(), ref.get(), ref.get()}, 128, 8);
    auto bp = Pipeline::build(m, *store, plan, {b200.get(), b200.get(), b200.get(), b200.get()}, 128, 8);
    if (!rp || !bp) return 1;
    Trace greedy_r = generate(*rp, prompt, 32, nullptr, 1, V);
    Trace greedy_b = generate(*bp, prompt, 32, nullptr, 1, V);
    compare_traces(greedy_r, greedy_b, V, "plain greedy generation (q = 1) equals the reference");

    std::vector<std::int32_t> seq = prompt;
    seq.insert(seq.end(), greedy_r.generated.begin(), greedy_r.generated.end());
    ScriptedDrafter::Config cfg;
    cfg.vocab = V;
    cfg.seed = 1;
    cfg.corruption_rate = 0.3;
    ScriptedDrafter d1(seq, cfg), d2(seq, cfg);
    auto rp2 = Pipeline::build(m, *store, plan, {ref.get(), ref.get(), ref.get(), ref.get()}, 128, 8);
    auto bp2 = Pipeline::build(m, *store, plan, {b200.get(), b200.get(), b200.get(), b200.get()}, 128, 8);
    Trace spec_r = generate(*rp2, prompt, 32, &d1, 4, V);
    Trace spec_b = generate(*bp2, prompt, 32, &d2, 4, V);
    compare_traces(spec_r, spec_b, V, "speculative generation q = 4 scripted:0.3 equals the reference");
    check(spec_b.generated == greedy_r.generated, "speculative output == plain greedy output");

    // stage-level drop-in: heterogeneous pipelines
    ScriptedDrafter d3(seq, cfg), d4(seq, cfg);
    auto mix1 = Pipeline::build(m, *store, plan, {ref.get(), b200.get(), b200.get(), ref.get()}, 128, 8);
    auto mix2 = Pipeline::build(m, *store, plan, {b200.get(), ref.get(), ref.get(), b200.get()}, 128, 8);
    compare_traces(spec_r, generate(*mix1, prompt, 32, &d3, 4, V), V, "mixed pipeline ref|b200|b200|ref");
    compare_traces(spec_r, generate(*mix2, prompt, 32, &d4, 4, V), V, "mixed pipeline b200|ref|ref|b200");
  }

  admission_rules(*b200, m, *store, *ref);
  tail_records(*b200, *ref, m, *store);

  {  // GPU MTP drafters (standalone and bound to a b200 tail) == MtpFixtureDrafter
    auto md = MtpFixtureDrafter::create(m, *store);
    auto bd = backends::make_b200_mtp_drafter(m, *store, 0, 8);
    if (!md.is_ok() || !bd.is_ok()) {
      check(false, "MTP drafters", md.is_ok() ? bd.status().to_string() : md.status().to_string());
    } else {
      bool same = true;
      for (std::int32_t prev = 0; prev < 16; ++prev) {
        auto a = (*md)->draft({}, prev * 13 % static_cast<std::int32_t>(V), 11);
        auto b = (*bd)->draft({}, prev * 13 % static_cast<std::int32_t>(V), 11);
        same &= a == b && a.size() == 11;
      }
      check(same, "standalone GPU MTP drafter drafts the reference's tokens (16 starts x 11 steps)");
      // stochastic proposals (MtpFixtureDrafter::propose, drafter.cpp:72-86) from the same Rng: the same tokens, and
      // distribution rows within one ulp (the double exp and kept-sum order of the device's distribution)
      bool same_tokens = true;
      std::size_t entries = 0, off_by_one = 0, worse = 0;
      for (int variant = 0; variant < 2; ++variant) {
        SamplingParams sp;
        sp.temperature = variant == 0 ? 1.0f : 0.8f;
        sp.top_k = variant == 0 ? 0 : 40;
        sp.top_p = variant == 0 ? 1.0f : 0.9f;
        for (std::int32_t start = 0; start < 8; ++start) {
          Rng ra(100 + start), rb(100 + start);
          auto a = (*md)->propose({}, start * 29 % static_cast<std::int32_t>(V), 7, sp, ra);
          auto b = (*bd)->propose({}, start * 29 % static_cast<std::int32_t>(V), 7, sp, rb);
          same_tokens &= a.tokens == b.tokens && a.probs.size() == b.probs.size();
          for (std::size_t j = 0; j < std::min(a.probs.size(), b.probs.size()); ++j)
            for (std::size_t i = 0; i < a.probs[j].size() && i < b.probs[j].size(); ++i) {
              std::int32_t x, y;
              std::memcpy(&x, &a.probs[j][i], 4);
              std::memcpy(&y, &b.probs[j][i], 4);
              const std::int64_t d = std::llabs(static_cast<std::int64_t>(x) - y);
              ++entries;
              off_by_one += d == 1;
              worse += d > 1;
            }
        }
      }
      char pb[160];
      std::snprintf(pb, sizeof pb, "%zu entries, %zu off by 1 ulp, %zu by more", entries, off_by_one, worse);
      check(same_tokens && worse == 0, "GPU MTP proposal == MtpFixtureDrafter::propose (T=1; T=0.8 top-k 40 top-p 0.9)",
            pb);

      // speculative generation with MTP drafts: reference pipeline + MtpFixtureDrafter against the b200 pipeline +
      // the drafter bound to its tail
      auto rp = Pipeline::build(m, *store, plan, {ref.get(), ref.get(), ref.get(), ref.get()}, 128, 8);
      auto bp = Pipeline::build(m, *store, plan, {b200.get(), b200.get(), b200.get(), b200.get()}, 128, 8);
      if (rp && bp) {
        auto bound = backends::make_b200_mtp_drafter(*bp->stages.back());
        check(bound.is_ok(), "drafter bound to the b200 tail", bound.is_ok() ? "" : bound.status().to_string());
        auto not_b200 = backends::make_b200_mtp_drafter(*rp->stages.back());
        check(!not_b200.is_ok() && not_b200.status().code() == ErrorCode::kInvalidArgument,
              "binding to a reference tail refused");
        auto middle = backends::make_b200_mtp_drafter(*bp->stages[1]);
        check(!middle.is_ok(), "binding to a middle stage refused");
        if (bound.is_ok()) {
          Trace tr = generate(*rp, prompt, 32, md->get(), 4, V);
          Trace tb = generate(*bp, prompt, 32, bound->get(), 4, V);
          compare_traces(tr, tb, V, "MTP speculative generation q = 4 equals the reference");
        }
      }
    }
  }

  if (bench) {
    auto rp = Pipeline::build(m, *store, plan, {ref.get(), ref.get(), ref.get(), ref.get()}, 2048, 8);
    auto bp = Pipeline::build(m, *store, plan, {b200.get(), b200.get(), b200.get(), b200.get()}, 2048, 8);
    if (rp && bp) {
      const double wr = time_windows(*rp, 100), wb = time_windows(*bp, 400);
      // the C1 workload end to end: speculative generation of 32 new tokens, q = 4, ScriptedDrafter with
      // corruption 0.3, from the 16-token prompt; decode tokens per second over `reps` generations (prefill
      // included, as the reference's clusterlm-bench reports decode tok/s of whole requests)
      std::vector<std::int32_t> seq = prompt;
      {
        auto gp = Pipeline::build(m, *store, plan, {ref.get(), ref.get(), ref.get(), ref.get()}, 128, 8);
        Trace g = gp ? generate(*gp, prompt, 32, nullptr, 1, V) : Trace{};
        seq.insert(seq.end(), g.generated.begin(), g.generated.end());
      }
      auto gen_rate = [&](BackendAdapter* be, int reps, double* accepted_per_round) {
        ScriptedDrafter::Config cfg;
        cfg.vocab = V;
        cfg.seed = 1;
        cfg.corruption_rate = 0.3;
        double secs = 0.0;
        std::size_t tokens = 0, rounds = 0;
        for (int r = 0; r < reps; ++r) {
          ScriptedDrafter d(seq, cfg);
          auto p = Pipeline::build(m, *store, plan, {be, be, be, be}, 128, 8);
          if (!p) return 0.0;
          const auto t0 = std::chrono::steady_clock::now();
          Trace t = generate(*p, prompt, 32, &d, 4, V);
          secs += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
          if (!t.ok) return 0.0;
          tokens += t.generated.size();
          rounds += t.accepted.size();
        }
        *accepted_per_round = rounds ? static_cast<double>(tokens) / rounds : 0.0;
        return tokens / secs;
      };
      double apr_r = 0.0, apr_b = 0.0;
      gen_rate(b200.get(), 2, &apr_b);  // warm-up: CUDA graphs captured on first use
      const double tr = gen_rate(ref.get(), 5, &apr_r), tb = gen_rate(b200.get(), 20, &apr_b);
      std::printf("{\"bench\": \"fixture q=4 windows (4 stages in one process, wire encoding between stages)\", "
                  "\"reference_windows_per_s\": %.2f, \"b200_windows_per_s\": %.2f, "
                  "\"reference_decode_tok_s\": %.2f, \"b200_decode_tok_s\": %.2f, "
                  "\"reference_tokens_per_round\": %.3f, \"b200_tokens_per_round\": %.3f}\n",
                  wr, wb, tr, tb, apr_r, apr_b);
    }
  }
  std::printf("%d failure(s)\n", g_failures);
  return g_failures;
}
