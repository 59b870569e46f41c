// B200 backend: BackendAdapter / ExecutionDomain / Drafter of ClusterLM over the libclm_b200 C ABI.
//
// One B200Domain = one clm_b200 engine (a stage's layer range on one GPU, its own CUDA context handle and
// stream) plus a windows::WindowLedger that admits every request exactly as the reference domain does
// (runtime/domain/src/reference_domain.cpp:376-445 for execute, :297-337 for commit/abort).  The engine holds
// weights, sequence state and window buffers in device memory; activations and logits cross the C ABI as host
// arrays in the StageActivations record layout (boundary.hpp:29-42), so a middle stage on another machine sees
// exactly the reference's wire records.
#include "b200_backend.hpp"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>

#include "../../include/clm_b200.h"
#include "clusterlm/domain/drafter.hpp"
#include "clusterlm/objects/gguf.hpp"
#include "clusterlm/windows/window_ledger.hpp"

namespace clusterlm::backends {
namespace {

using domain::CommitAck;
using domain::CommitRequest;
using domain::DomainMetrics;
using domain::DomainRequirements;
using domain::DomainSpec;
using domain::Logits;
using domain::StageActivations;
using domain::StageRole;
using domain::WindowAbortAck;
using domain::WindowRequest;
using objects::LayerKind;
using objects::ModelGeometry;
using objects::ModelManifest;

constexpr std::string_view kFixtureFamily = "clusterlm-fixture";
// Manifests built from llama.cpp GGUF files name their family "llama.cpp:<architecture>"
// (runtime/backends/llama/src/llama_manifest.cpp:77); the b200 engine runs the dense "llama" architecture.
constexpr std::string_view kLlamaFamilyPrefix = "llama.cpp:";

bool is_llama_family(const ModelGeometry& g) { return g.family.rfind(kLlamaFamilyPrefix, 0) == 0; }

// ggml tensor type -> clm_b200 quant id (GGML_TYPE_F32 = 0, Q8_0 = 8, Q4_K = 12); other types pass as -1 - type,
// which clm_b200_llama_load_tensors refuses by name when the stage needs the tensor.
int quant_of_ggml(objects::GgmlType t) {
  switch (static_cast<int>(t)) {
    case 0: return CLM_QUANT_F32;
    case 8: return CLM_QUANT_Q8_0;
    case 12: return CLM_QUANT_Q4_K;
    default: return -1 - static_cast<int>(t);
  }
}

// clm_b200 status codes are ErrorCode values (include/clm_b200.h); the message is the library's thread-local text.
Status from_clm(int rc, std::string_view what) {
  if (rc == CLM_OK) return Status::ok();
  const char* msg = clm_b200_last_error();
  return make_error(static_cast<ErrorCode>(rc), std::string(what) + ": " + (msg ? msg : ""));
}

Status invalid(std::string m) { return make_error(ErrorCode::kInvalidArgument, std::move(m)); }
Status precondition(std::string m) { return make_error(ErrorCode::kFailedPrecondition, std::move(m)); }

// Representation::quant_type -> clm_b200 quant id (-1: not served by this backend).
int quant_of(const objects::Representation& r) {
  if (r.quant_type == "f32") return CLM_QUANT_F32;
  if (r.quant_type == "q8_0-fixture") return CLM_QUANT_Q8_FIXTURE;
  if (r.quant_type == "q8_0") return CLM_QUANT_Q8_0;
  if (r.quant_type == "q4_k" || r.quant_type == "Q4_K") return CLM_QUANT_Q4_K;
  return -1;
}

// Process-wide device contexts, one per CUDA device, shared by the domains placed on it (a context is only a
// device binding and a stream; every domain keeps its own engine, buffers and state).
class DeviceContexts {
 public:
  static Result<std::shared_ptr<clm_b200_ctx>> get(int device) {
    static std::mutex mu;
    static std::unordered_map<int, std::weak_ptr<clm_b200_ctx>> live;
    std::lock_guard<std::mutex> lock(mu);
    if (auto p = live[device].lock()) return p;
    int n = 0;
    if (clm_b200_device_count(&n) != CLM_OK || n == 0)
      return make_error(ErrorCode::kHardwareUnavailable, "b200 backend: no CUDA device");
    if (device < 0 || device >= n) return invalid("b200 backend: device " + std::to_string(device) + " does not exist");
    clm_b200_ctx* raw = nullptr;
    CLM_RETURN_IF_ERROR(from_clm(clm_b200_ctx_create(device, &raw), "clm_b200_ctx_create"));
    std::shared_ptr<clm_b200_ctx> p(raw, [](clm_b200_ctx* c) { clm_b200_ctx_destroy(c); });
    live[device] = p;
    return p;
  }
};

clm_b200_fixture_geometry fixture_geometry(const ModelGeometry& g, std::vector<std::uint8_t>& kinds) {
  kinds.resize(g.layer_kinds.size());
  for (std::size_t i = 0; i < kinds.size(); ++i) kinds[i] = static_cast<std::uint8_t>(g.layer_kinds[i]);
  clm_b200_fixture_geometry c{};
  c.n_layers = g.n_layers;
  c.hidden = g.hidden_size;
  c.residual_streams = g.residual_streams;
  c.n_experts = g.n_experts;
  c.n_active_experts = g.n_active_experts;
  c.expert_ff = g.expert_ff;
  c.shared_expert_ff = g.shared_expert_ff;
  c.n_heads = g.n_heads;
  c.n_kv_heads = g.n_kv_heads;
  c.head_dim = g.head_dim;
  c.vocab = g.vocab_size;
  c.ple_layer = g.ple_layer;
  c.ple_ngram = g.ple_ngram;
  c.ple_rows = g.ple_rows;
  c.layer_kinds = kinds.data();
  return c;
}

class B200Domain final : public domain::ExecutionDomain {
 public:
  B200Domain(ModelManifest manifest, DomainSpec spec, int device, std::filesystem::path model_dir)
      : manifest_(std::move(manifest)), g_(manifest_.geometry), spec_(spec), device_(device),
        layout_(domain::BoundaryLayout::for_geometry(g_)), model_dir_(std::move(model_dir)) {}
  ~B200Domain() override { destroy_engine(); }

  Status init() {
    CLM_RETURN_IF_ERROR(manifest_.validate());
    llama_ = is_llama_family(g_);
    if (g_.family != kFixtureFamily && !llama_)
      return make_error(ErrorCode::kUnimplemented, "b200 backend serves the clusterlm-fixture and llama.cpp:llama "
                                                   "families; family '" + g_.family + "' is not implemented");
    if (llama_) CLM_RETURN_IF_ERROR(init_llama());
    if (spec_.max_context == 0 || spec_.max_window == 0 || spec_.max_sessions == 0 || spec_.max_window > spec_.max_context)
      return invalid("domain spec needs max_context >= max_window >= 1 and max_sessions >= 1");
    if (spec_.layers.end > g_.n_layers || spec_.layers.end < spec_.layers.begin)
      return invalid("layer range outside the model");
    CLM_ASSIGN_OR_RETURN(ctx_, DeviceContexts::get(device_));
    // the engine validates role rules (prefix owns layer 0 and the PLE layer, tail ends at the last layer)
    return create_engine();
  }

  const DomainSpec& spec() const override { return spec_; }
  domain::BoundaryLayout boundary() const override { return layout_; }

  Result<DomainRequirements> describe_requirements() const override {
    if (llama_) return llama_requirements();
    DomainRequirements r;
    r.required_objects = required_object_names();
    std::uint64_t largest = 0;
    for (const auto& name : r.required_objects) {
      const objects::ManifestObject* o = manifest_.find(name);
      if (o == nullptr) return make_error(ErrorCode::kNotFound, "manifest has no object '" + name + "'");
      // resident form: f32 (q8_0-fixture is decoded exactly at prepare: 36 bytes -> 32 floats)
      const std::uint64_t resident =
          o->representation.quant_type == "q8_0-fixture" ? o->byte_size / 36 * 32 * 4 : o->byte_size;
      r.gpu_weight_bytes += resident;
      largest = std::max(largest, o->byte_size);
    }
    std::uint64_t weight = 0, state = 0;
    std::uint32_t fpp = 0;
    if (engine_ != nullptr) {
      CLM_RETURN_IF_ERROR(from_clm(clm_b200_engine_info(engine_, &weight, &state, &fpp), "clm_b200_engine_info"));
    }
    r.state_bytes = state * spec_.max_sessions;
    r.window_bytes = window_bytes_per_session() * spec_.max_sessions;
    const std::uint64_t qd = std::uint64_t{g_.n_heads} * g_.head_dim;
    r.scratch_bytes = std::uint64_t{spec_.max_window} *
                      (layout_.floats_per_position() + g_.n_heads * (spec_.max_context + 1ull) + qd +
                       (has_head() ? g_.vocab_size : 0)) * 4;
    r.staging_bytes = largest;  // one object at a time through a device staging buffer
    return r;
  }

  Status prepare(const objects::ObjectResolver& resolver) override {
    if (prepared_) return precondition("domain already prepared; release() first");
    if (engine_ == nullptr) CLM_RETURN_IF_ERROR(create_engine());
    Status st = bind_and_prepare(resolver);
    if (!st.is_ok()) {
      destroy_engine();  // a failed prepare releases everything
      return st;
    }
    prepared_ = true;
    return Status::ok();
  }

  Status open_session(Epoch epoch, SessionId session) override {
    if (!prepared_) return precondition("domain not prepared");
    if (!sessions_.contains(session) && sessions_.size() >= spec_.max_sessions)
      return make_error(ErrorCode::kResourceExhausted, "max_sessions reached");
    CLM_RETURN_IF_ERROR(ledger_.open_session(epoch, session));
    // re-opening replaces the session's state (reference_domain.cpp:258-276)
    if (sessions_.contains(session)) {
      CLM_RETURN_IF_ERROR(from_clm(clm_b200_session_close(engine_, session.value), "clm_b200_session_close"));
      windows_.erase(session);
    }
    CLM_RETURN_IF_ERROR(from_clm(clm_b200_session_open(engine_, session.value), "clm_b200_session_open"));
    sessions_.insert(session);
    return Status::ok();
  }

  Result<StageActivations> run_prefix(const WindowRequest& request, std::span<const std::int32_t> tokens) override {
    if (spec_.role != StageRole::kPrefix) return precondition("run_prefix is only valid on a prefix domain");
    return execute(request, nullptr, tokens, nullptr);
  }

  Result<StageActivations> run_window(const WindowRequest& request, const StageActivations& input) override {
    if (spec_.role == StageRole::kPrefix) return precondition("a prefix domain consumes tokens, not activations");
    return execute(request, &input, {}, nullptr);
  }

  Result<Logits> run_tail(const WindowRequest& request, const StageActivations& input) override {
    if (spec_.role != StageRole::kTail) return precondition("run_tail is only valid on a tail domain");
    Logits logits;
    auto r = execute(request, &input, {}, &logits);
    if (!r.is_ok()) return r.status();
    return logits;
  }

  Result<CommitAck> commit_window(const CommitRequest& request) override {
    if (!prepared_) return precondition("domain not prepared");
    CLM_ASSIGN_OR_RETURN(windows::WindowLedger::CommitDecision decision, ledger_.begin_commit(request));
    if (decision.kind == windows::WindowLedger::CommitDecision::Kind::kReplay) return decision.ack;
    auto w = windows_.find(request.session);
    if (w == windows_.end() || w->second != request.window)
      return make_error(ErrorCode::kInternal, "ledger and domain window state disagree");
    CLM_RETURN_IF_ERROR(
        from_clm(clm_b200_commit(engine_, request.session.value, request.accepted), "clm_b200_commit"));
    windows_.erase(w);
    ++metrics_.windows_committed;
    metrics_.positions_committed += request.accepted;
    return ledger_.finish_commit(request);
  }

  Result<WindowAbortAck> abort_window(Epoch epoch, SessionId session, WindowId window) override {
    CLM_ASSIGN_OR_RETURN(WindowAbortAck ack, ledger_.abort_window(epoch, session, window));
    auto w = windows_.find(session);
    if (w != windows_.end() && w->second == window) {
      CLM_RETURN_IF_ERROR(from_clm(clm_b200_abort(engine_, session.value), "clm_b200_abort"));
      windows_.erase(w);
      ++metrics_.windows_aborted;
    }
    return ack;
  }

  Status abort_session(Epoch epoch, SessionId session) override {
    CLM_RETURN_IF_ERROR(ledger_.abort_session(epoch, session));
    if (windows_.erase(session) != 0) ++metrics_.windows_aborted;
    if (sessions_.erase(session) != 0 && engine_ != nullptr)
      CLM_RETURN_IF_ERROR(from_clm(clm_b200_session_close(engine_, session.value), "clm_b200_session_close"));
    return Status::ok();
  }

  Status release() override {
    ledger_.clear();
    sessions_.clear();
    windows_.clear();
    destroy_engine();
    prepared_ = false;
    return Status::ok();
  }

  // The engine and the draft width of a prepared tail that holds the MTP drafter objects (nullptr otherwise).
  clm_b200_engine* drafter_engine() const { return prepared_ && drafter_ready_ ? engine_ : nullptr; }
  // Drafts per device call: the fixture engine drafts up to max_window tokens, the llama engine max_window - 1.
  std::uint32_t max_draft() const { return llama_ ? std::max<std::uint32_t>(spec_.max_window, 2) - 1 : spec_.max_window; }
  std::uint32_t vocab() const { return g_.vocab_size; }

  DomainMetrics read_metrics() const override {
    DomainMetrics m = metrics_;
    std::uint64_t weight = 0, state = 0;
    if (engine_ != nullptr && clm_b200_engine_info(engine_, &weight, &state, nullptr) == CLM_OK) {
      m.resident_weight_bytes = prepared_ ? weight : 0;
      m.state_bytes = state * sessions_.size();
    }
    m.window_bytes = window_bytes_per_session() * sessions_.size();
    m.stale_rejections = ledger_.stale_rejections();
    return m;
  }

 private:
  bool has_head() const { return spec_.role == StageRole::kTail; }

  std::vector<std::string> required_object_names() const {
    if (llama_) return llama_object_names();
    std::vector<std::string> names;
    if (spec_.role == StageRole::kPrefix) {
      names.emplace_back(objects::kEmbeddingObjectName);
      names.emplace_back(objects::kPleObjectName);
    }
    for (std::uint32_t L = spec_.layers.begin; L < spec_.layers.end; ++L) {
      names.push_back(objects::dense_object_name(L));
      if (g_.shared_expert_ff > 0) names.push_back(objects::shared_expert_object_name(L));
      for (std::uint32_t e = 0; e < g_.n_experts; ++e) names.push_back(objects::expert_object_name(L, e));
    }
    if (spec_.role == StageRole::kTail) names.emplace_back(objects::kHeadObjectName);
    return names;
  }

  std::uint64_t window_bytes_per_session() const {
    if (llama_) return 0;  // no per-window state beyond the KV rows the window writes into its pages
    std::uint64_t rec = 0;
    for (std::uint32_t L = spec_.layers.begin; L < spec_.layers.end; ++L)
      rec += g_.layer_kinds[L] == LayerKind::kRecurrent ? 1 : 0;
    return rec * spec_.max_window * g_.hidden_size * 4;
  }

  Status create_engine() {
    clm_b200_stage_spec cs{};
    cs.layer_begin = spec_.layers.begin;
    cs.layer_end = spec_.layers.end;
    cs.role = static_cast<int>(spec_.role);
    cs.max_context = spec_.max_context;
    cs.max_window = spec_.max_window;
    cs.max_sessions = spec_.max_sessions;
    if (llama_) return from_clm(clm_b200_llama_create(ctx_.get(), &lgeo_, &cs, &engine_), "clm_b200_llama_create");
    std::vector<std::uint8_t> kinds;
    const clm_b200_fixture_geometry cg = fixture_geometry(g_, kinds);
    return from_clm(clm_b200_fixture_create(ctx_.get(), &cg, &cs, &engine_), "clm_b200_fixture_create");
  }

  void destroy_engine() {
    if (engine_ != nullptr) clm_b200_engine_destroy(engine_);
    engine_ = nullptr;
  }

  Status bind(const objects::ObjectResolver& resolver, const std::string& name) {
    CLM_ASSIGN_OR_RETURN(objects::ProvisionedObject obj, resolver.resolve(name));
    if (obj.entry == nullptr) return make_error(ErrorCode::kInternal, "resolver returned no manifest entry");
    const int quant = quant_of(obj.entry->representation);
    if (quant < 0)
      return make_error(ErrorCode::kUnimplemented, "object '" + name + "' is stored as " +
                                                       obj.entry->representation.quant_type +
                                                       ", which the b200 backend does not execute");
    return from_clm(clm_b200_engine_set_object(engine_, name.c_str(), quant, obj.bytes.data(), obj.bytes.size()),
                    "binding '" + name + "'");
  }

  Status bind_and_prepare(const objects::ObjectResolver& resolver) {
    if (llama_) return llama_bind_and_prepare(resolver);
    for (const std::string& name : required_object_names()) CLM_RETURN_IF_ERROR(bind(resolver, name));
    // A Father tail also binds the MTP drafter and the embedding when they are provisioned to it, so that a
    // drafter bound to this domain (make_b200_mtp_drafter(tail)) runs on the same GPU as the head.
    drafter_ready_ = false;
    if (spec_.role == StageRole::kTail && manifest_.find(objects::kMtpObjectName) != nullptr &&
        manifest_.find(objects::kEmbeddingObjectName) != nullptr &&
        resolver.resolve(objects::kMtpObjectName).is_ok() && resolver.resolve(objects::kEmbeddingObjectName).is_ok()) {
      CLM_RETURN_IF_ERROR(bind(resolver, std::string(objects::kMtpObjectName)));
      CLM_RETURN_IF_ERROR(bind(resolver, std::string(objects::kEmbeddingObjectName)));
      drafter_ready_ = true;
    }
    return from_clm(clm_b200_engine_prepare(engine_), "clm_b200_engine_prepare");
  }

  // ---- the llama.cpp family (dense "llama" architecture)
  // Reads the GGUF tensor directory and metadata of the manifest's shards (model_dir / ShardInfo::file_name) to name
  // the byte ranges of each object and to complete the engine geometry (RoPE base, RMS epsilon, quantisation).
  Status init_llama() {
    if (model_dir_.empty())
      return precondition("b200 backend: a llama.cpp manifest needs B200BackendOptions::model_dir (the GGUF directory)");
    std::vector<std::filesystem::path> paths;
    for (const auto& sh : manifest_.shards) paths.push_back(model_dir_ / sh.file_name);
    auto files = objects::open_gguf_model(paths);
    if (!files.is_ok()) return files.status();
    gguf_ = std::make_unique<objects::GgufModelFiles>(std::move(files).value());
    const objects::GgufFile& meta = gguf_->meta();
    auto meta_str = [&](const std::string& k) {
      const objects::GgufValue* v = meta.find(k);
      return v != nullptr && v->is_string() ? v->s : std::string{};
    };
    auto meta_num = [&](const std::string& k, double dflt) {
      const objects::GgufValue* v = meta.find(k);
      if (v == nullptr) return dflt;
      auto d = v->as_double();
      return d ? *d : dflt;
    };
    const std::string arch = meta_str("general.architecture");
    if (arch != "llama" || g_.n_experts != 1 || g_.shared_expert_ff != 0)
      return make_error(ErrorCode::kUnimplemented,
                        "b200 backend: llama.cpp architecture '" + arch + "' (dense llama only)");
    for (auto k : g_.layer_kinds)
      if (k != LayerKind::kFullAttention) return make_error(ErrorCode::kUnimplemented, "b200 backend: recurrent layers");
    if (gguf_->find_tensor("rope_freqs.weight"))
      return make_error(ErrorCode::kUnimplemented, "b200 backend: rope_freqs.weight (RoPE frequency factors)");
    const std::string scaling = meta_str(arch + ".rope.scaling.type");
    if (!scaling.empty() && scaling != "none")
      return make_error(ErrorCode::kUnimplemented, "b200 backend: RoPE scaling '" + scaling + "'");
    auto q = gguf_->find_tensor("blk.0.attn_q.weight");
    if (!q) return make_error(ErrorCode::kNotFound, "b200 backend: blk.0.attn_q.weight missing");
    lgeo_.quant = quant_of_ggml(q->info->type);
    if (lgeo_.quant != CLM_QUANT_Q4_K && lgeo_.quant != CLM_QUANT_Q8_0)
      return make_error(ErrorCode::kUnimplemented, "b200 backend: matrices must be Q4_K or Q8_0 (llama-quantize --pure)");
    lgeo_.n_layers = g_.n_layers;
    lgeo_.hidden = g_.hidden_size;
    lgeo_.n_heads = g_.n_heads;
    lgeo_.n_kv_heads = g_.n_kv_heads;
    lgeo_.head_dim = g_.head_dim;
    lgeo_.ffn = g_.expert_ff;
    lgeo_.vocab = g_.vocab_size;
    lgeo_.rope_theta = static_cast<float>(meta_num(arch + ".rope.freq_base", 10000.0));
    lgeo_.rms_eps = static_cast<float>(meta_num(arch + ".attention.layer_norm_rms_epsilon", 1e-5));
    lgeo_.mtp = gguf_->find_tensor("mtp.ffn_gate.weight") ? 1u : 0u;
    for (std::uint32_t sh = 0; sh < gguf_->shards.size(); ++sh)
      for (const auto& t : gguf_->shards[sh].tensors) by_offset_[{sh, t.file_offset}] = &t;
    return Status::ok();
  }

  // token_embd on the prefix (and on a tail whose head shares it, or whose MTP head needs it), blk.L.dense per
  // layer, output_head on the tail (llama_manifest.hpp:9-11).
  std::vector<std::string> llama_object_names() const {
    std::vector<std::string> names;
    const bool tail = spec_.role == StageRole::kTail;
    const bool tied = !gguf_->find_tensor("output.weight");
    if (spec_.role == StageRole::kPrefix || (tail && (tied || lgeo_.mtp)))
      names.emplace_back(objects::kEmbeddingObjectName);
    for (std::uint32_t L = spec_.layers.begin; L < spec_.layers.end; ++L) names.push_back(objects::dense_object_name(L));
    if (tail) names.emplace_back(objects::kHeadObjectName);
    return names;
  }

  Result<DomainRequirements> llama_requirements() const {
    DomainRequirements r;
    r.required_objects = llama_object_names();
    std::uint64_t largest = 0;
    for (const auto& name : r.required_objects) {
      const objects::ManifestObject* o = manifest_.find(name);
      if (o == nullptr) return make_error(ErrorCode::kNotFound, "manifest has no object '" + name + "'");
      r.gpu_weight_bytes += o->byte_size;  // Q4_K / Q8_0 blocks are repacked losslessly: the same bytes resident
      largest = std::max(largest, o->byte_size);
    }
    // paged fp16 KV cache: every layer of the stage, K and V, max_context positions in 64-position pages
    const std::uint64_t kvd = std::uint64_t{g_.n_kv_heads} * g_.head_dim;
    const std::uint64_t ctx_pages = (std::uint64_t{spec_.max_context} + 63) / 64;
    r.state_bytes = std::uint64_t{spec_.layers.end - spec_.layers.begin} * 2 * ctx_pages * 64 * kvd * 2 *
                    spec_.max_sessions;
    r.window_bytes = 0;
    // window buffers: residual rows, records in and out, the widest activation hand-off, logits and draft rows
    const std::uint64_t W = spec_.max_window, H = g_.hidden_size, V = g_.vocab_size;
    const std::uint64_t wide = std::max<std::uint64_t>({H, std::uint64_t{g_.expert_ff}, std::uint64_t{g_.n_heads} * g_.head_dim});
    r.scratch_bytes = W * (H + 2 * layout_.floats_per_position() + 4 * wide) * 4 +
                      (spec_.role == StageRole::kTail ? 3 * W * V * 4 : 0);
    r.staging_bytes = largest;
    return r;
  }

  // Binds the stage's tensors from the resolver's object bytes: each source range of an object is one GGUF tensor,
  // named from the tensor directory by (shard, file offset); the engine repacks them on the device.
  Status llama_bind_and_prepare(const objects::ObjectResolver& resolver) {
    std::vector<objects::ProvisionedObject> held;
    std::vector<clm_b200_tensor> tensors;
    std::vector<std::string> names;
    names.reserve(4096);
    for (const std::string& name : llama_object_names()) {
      CLM_ASSIGN_OR_RETURN(objects::ProvisionedObject obj, resolver.resolve(name));
      if (obj.entry == nullptr) return make_error(ErrorCode::kInternal, "resolver returned no manifest entry");
      if (obj.bytes.size() != obj.entry->byte_size)
        return make_error(ErrorCode::kDataLoss, "object '" + name + "' has " + std::to_string(obj.bytes.size()) +
                                                    " bytes, the manifest says " + std::to_string(obj.entry->byte_size));
      std::uint64_t off = 0;
      for (const auto& r : obj.entry->source_ranges) {
        auto it = by_offset_.find({r.shard, r.offset});
        if (it == by_offset_.end() || it->second->n_bytes != r.length)
          return make_error(ErrorCode::kVersionMismatch,
                            "object '" + name + "': a source range is not a tensor of the model directory's GGUF files");
        names.push_back(it->second->name);
        tensors.push_back(clm_b200_tensor{nullptr, quant_of_ggml(it->second->type), obj.bytes.data() + off, r.length});
        off += r.length;
      }
      held.push_back(obj);
    }
    for (std::size_t i = 0; i < tensors.size(); ++i) tensors[i].name = names[i].c_str();
    CLM_RETURN_IF_ERROR(from_clm(clm_b200_llama_load_tensors(engine_, tensors.data(), static_cast<std::uint32_t>(tensors.size())),
                                 "clm_b200_llama_load_tensors"));
    drafter_ready_ = spec_.role == StageRole::kTail && lgeo_.mtp != 0;
    return from_clm(clm_b200_engine_prepare(engine_), "clm_b200_engine_prepare");
  }

  Result<StageActivations> execute(const WindowRequest& req, const StageActivations* input,
                                   std::span<const std::int32_t> tokens, Logits* logits_out) {
    if (!prepared_) return precondition("domain not prepared");
    const Status admitted = ledger_.begin_window(req);
    if (!admitted.is_ok()) return admitted;
    auto reject = [&](Status st) -> Result<StageActivations> {
      ledger_.fail_window(req.session);
      return st;
    };
    if (req.positions > spec_.max_window) return reject(make_error(ErrorCode::kResourceExhausted, "window exceeds max_window"));
    if (req.base_position + req.positions > spec_.max_context)
      return reject(make_error(ErrorCode::kResourceExhausted, "window exceeds max_context"));
    if (input != nullptr) {
      const Status v = input->validate();
      if (!v.is_ok()) return reject(v);
      if (input->layout != layout_) return reject(make_error(ErrorCode::kVersionMismatch, "activation layout mismatch"));
      if (input->positions != req.positions || input->first_position != req.base_position)
        return reject(invalid("activations do not match the window request"));
    } else {
      if (tokens.size() != req.positions) return reject(invalid("tokens.size() != request.positions"));
      for (std::int32_t t : tokens)
        if (t < 0 || static_cast<std::uint32_t>(t) >= g_.vocab_size) return reject(invalid("token outside the vocabulary"));
    }
    const auto t0 = std::chrono::steady_clock::now();
    StageActivations out;
    out.layout = layout_;
    out.first_position = req.base_position;
    out.positions = req.positions;
    float* h_out = nullptr;
    float* h_logits = nullptr;
    if (logits_out != nullptr) {
      logits_out->positions = req.positions;
      logits_out->vocab = g_.vocab_size;
      logits_out->data.assign(std::size_t{req.positions} * g_.vocab_size, 0.0f);
      h_logits = logits_out->data.data();
    } else {
      out.data.assign(std::size_t{req.positions} * layout_.floats_per_position(), 0.0f);
      h_out = out.data.data();
    }
    const int rc = clm_b200_run_window(engine_, req.session.value, req.base_position, req.positions,
                                       input == nullptr ? tokens.data() : nullptr,
                                       input != nullptr ? input->data.data() : nullptr, h_out, h_logits);
    if (rc != CLM_OK) return reject(from_clm(rc, "clm_b200_run_window"));
    windows_[req.session] = req.window;
    ++metrics_.windows_run;
    metrics_.compute_ns_total += static_cast<std::uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
    return out;
  }

  ModelManifest manifest_;
  const ModelGeometry& g_;
  DomainSpec spec_;
  int device_;
  domain::BoundaryLayout layout_;
  std::filesystem::path model_dir_;
  bool llama_ = false;
  std::unique_ptr<objects::GgufModelFiles> gguf_;  // llama family: tensor directory of the model's GGUF files
  std::map<std::pair<std::uint32_t, std::uint64_t>, const objects::GgufTensorInfo*> by_offset_;
  clm_b200_llama_geometry lgeo_{};
  std::shared_ptr<clm_b200_ctx> ctx_;
  clm_b200_engine* engine_ = nullptr;
  bool prepared_ = false;
  bool drafter_ready_ = false;
  windows::WindowLedger ledger_;
  std::unordered_set<SessionId> sessions_;
  std::unordered_map<SessionId, WindowId> windows_;  // the outstanding window of each session
  DomainMetrics metrics_;
};

class B200Backend final : public domain::BackendAdapter {
 public:
  explicit B200Backend(B200BackendOptions options) : options_(std::move(options)) {}

  domain::BackendInfo info() const override {
    domain::BackendInfo i;
    i.name = "b200";
    i.build_hash = kB200BuildHash;
    i.supports_gpu = true;
    int n = 0;
    i.hardware_available = clm_b200_device_count(&n) == CLM_OK && n > 0;
    return i;
  }

  Result<std::unique_ptr<domain::ExecutionDomain>> create_domain(const ModelManifest& manifest,
                                                                 const DomainSpec& spec) override {
    const std::uint32_t s = spec.stage.value;
    const int device = s < options_.stage_devices.size() ? options_.stage_devices[s] : options_.default_device;
    auto d = std::make_unique<B200Domain>(manifest, spec, device, options_.model_dir);
    CLM_RETURN_IF_ERROR(d->init());
    return std::unique_ptr<domain::ExecutionDomain>(std::move(d));
  }

 private:
  B200BackendOptions options_;
};

// MTP drafter on the GPU (MtpFixtureDrafter's step chained count times, drafter.cpp:39-89).  Either bound to a
// prepared b200 tail domain that holds the drafter (the fixture's mtp_drafter + token_embd objects, or a llama
// file's mtp.* tensors; it then borrows the tail's engine, so the tail must outlive it), or standalone over a
// zero-layer fixture tail engine of its own that holds token_embd, output_head and mtp_drafter.  draft() is greedy
// (argmax, lowest index on ties).  propose() is MtpFixtureDrafter::propose (drafter.cpp:72-86): with sampling
// parameters each draft is sampled from distribution(step logits, params) on the device with one uniform of the
// caller's Rng, drawn in the reference's order, and the proposal carries every draft's distribution (the Q rows
// of stochastic verification); greedy parameters give the greedy draft without rows.
class B200MtpDrafter final : public domain::Drafter {
 public:
  static Result<std::unique_ptr<domain::Drafter>> bound(domain::ExecutionDomain& tail) {
    auto* d = dynamic_cast<B200Domain*>(&tail);
    if (d == nullptr) return invalid("make_b200_mtp_drafter: the tail domain was not created by the b200 backend");
    if (d->spec().role != StageRole::kTail) return invalid("make_b200_mtp_drafter: the domain is not a tail");
    if (d->drafter_engine() == nullptr)
      return precondition("the b200 tail holds no MTP drafter (mtp_drafter and token_embd not provisioned, or not prepared)");
    auto out = std::unique_ptr<B200MtpDrafter>(new B200MtpDrafter());
    out->engine_ = d->drafter_engine();
    out->max_draft_ = d->max_draft();
    out->vocab_ = d->vocab();
    return std::unique_ptr<domain::Drafter>(std::move(out));
  }

  static Result<std::unique_ptr<domain::Drafter>> standalone(const ModelManifest& manifest,
                                                             const objects::ObjectResolver& resolver, int device,
                                                             std::uint32_t max_draft) {
    const ModelGeometry& g = manifest.geometry;
    if (g.family != kFixtureFamily)
      return make_error(ErrorCode::kUnimplemented, "b200 MTP drafter serves the clusterlm-fixture family");
    auto d = std::unique_ptr<B200MtpDrafter>(new B200MtpDrafter());
    CLM_ASSIGN_OR_RETURN(d->ctx_, DeviceContexts::get(device));
    std::vector<std::uint8_t> kinds;
    const clm_b200_fixture_geometry cg = fixture_geometry(g, kinds);
    clm_b200_stage_spec cs{};
    cs.layer_begin = g.n_layers;
    cs.layer_end = g.n_layers;
    cs.role = CLM_ROLE_TAIL;
    cs.max_context = std::max<std::uint32_t>(max_draft, 1);
    cs.max_window = std::max<std::uint32_t>(max_draft, 1);
    cs.max_sessions = 1;
    CLM_RETURN_IF_ERROR(from_clm(clm_b200_fixture_create(d->ctx_.get(), &cg, &cs, &d->owned_), "clm_b200_fixture_create"));
    d->engine_ = d->owned_;
    for (std::string_view name : {objects::kEmbeddingObjectName, objects::kHeadObjectName, objects::kMtpObjectName}) {
      CLM_ASSIGN_OR_RETURN(objects::ProvisionedObject obj, resolver.resolve(name));
      const int quant = obj.entry ? quant_of(obj.entry->representation) : -1;
      if (quant < 0) return make_error(ErrorCode::kUnimplemented, "unsupported representation of " + std::string(name));
      CLM_RETURN_IF_ERROR(from_clm(clm_b200_engine_set_object(d->owned_, std::string(name).c_str(), quant,
                                                              obj.bytes.data(), obj.bytes.size()),
                                   "binding " + std::string(name)));
    }
    CLM_RETURN_IF_ERROR(from_clm(clm_b200_engine_prepare(d->owned_), "clm_b200_engine_prepare"));
    d->max_draft_ = cs.max_window;
    d->vocab_ = g.vocab_size;
    return std::unique_ptr<domain::Drafter>(std::move(d));
  }

  ~B200MtpDrafter() override {
    if (owned_ != nullptr) clm_b200_engine_destroy(owned_);
  }

  // Drafter::draft has no error channel: a failed device call yields an empty draft (a plain q = 1 window).
  std::vector<std::int32_t> draft(std::span<const std::int32_t> /*committed_tokens*/, std::int32_t next_token,
                                  std::uint32_t count) override {
    std::vector<std::int32_t> out;
    std::int32_t prev = next_token;
    while (out.size() < count) {
      const std::uint32_t n = std::min<std::uint32_t>(count - static_cast<std::uint32_t>(out.size()), max_draft_);
      std::vector<std::int32_t> chunk(n, 0);
      if (clm_b200_mtp_draft(engine_, prev, n, 0.0f, 0, 0, chunk.data(), nullptr) != CLM_OK) return {};
      out.insert(out.end(), chunk.begin(), chunk.end());
      prev = out.back();
    }
    return out;
  }

  // Drafter::propose has no error channel either: a failed device call yields an empty proposal.
  domain::DraftProposal propose(std::span<const std::int32_t> committed, std::int32_t next_token, std::uint32_t count,
                                const domain::SamplingParams& params, domain::Rng& rng) override {
    if (params.greedy()) return domain::DraftProposal{draft(committed, next_token, count), {}};
    domain::DraftProposal out;
    std::int32_t prev = next_token;
    while (out.tokens.size() < count) {
      const std::uint32_t n = std::min<std::uint32_t>(count - static_cast<std::uint32_t>(out.tokens.size()), max_draft_);
      std::vector<double> u(n);
      for (double& x : u) x = rng.uniform();  // one uniform per draft, as sample_from draws them
      std::vector<std::int32_t> toks(n, 0);
      std::vector<float> probs(std::size_t{n} * vocab_);
      if (clm_b200_mtp_propose(engine_, prev, n, params.temperature, params.top_k, params.top_p, u.data(), toks.data(),
                               probs.data()) != CLM_OK)
        return {};
      for (std::uint32_t j = 0; j < n; ++j) {
        out.tokens.push_back(toks[j]);
        out.probs.emplace_back(probs.begin() + std::size_t{j} * vocab_, probs.begin() + std::size_t{j + 1} * vocab_);
      }
      prev = out.tokens.back();
    }
    return out;
  }

 private:
  B200MtpDrafter() = default;
  std::shared_ptr<clm_b200_ctx> ctx_;
  clm_b200_engine* owned_ = nullptr;   // standalone drafters own their engine
  clm_b200_engine* engine_ = nullptr;  // the engine drafted on (owned_ or a tail domain's)
  std::uint32_t max_draft_ = 1;
  std::uint32_t vocab_ = 0;
};

}  // namespace

std::unique_ptr<domain::BackendAdapter> make_b200_backend(const B200BackendOptions& options) {
  return std::make_unique<B200Backend>(options);
}

Result<std::unique_ptr<domain::Drafter>> make_b200_mtp_drafter(domain::ExecutionDomain& tail) {
  return B200MtpDrafter::bound(tail);
}

Result<std::unique_ptr<domain::Drafter>> make_b200_mtp_drafter(const objects::ModelManifest& manifest,
                                                               const objects::ObjectResolver& resolver, int device,
                                                               std::uint32_t max_draft) {
  return B200MtpDrafter::standalone(manifest, resolver, device, max_draft);
}

}  // namespace clusterlm::backends
