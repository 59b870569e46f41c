// engine_api.cu — the C ABI of the execution engines, dispatched on the engine family.
#include "engine.cuh"

using namespace clm;

namespace {

int enter(clm_b200_engine* e) {
  CLM_CHECK(e != nullptr, CLM_INVALID_ARGUMENT, "null engine");
  return ctx_enter(e->ctx);
}
LlamaEngine* llama(clm_b200_engine* e) { return as_llama(e); }
FixtureEngine* fixture(clm_b200_engine* e) { return as_fixture(e); }
const LlamaEngine* llama(const clm_b200_engine* e) { return as_llama(const_cast<clm_b200_engine*>(e)); }
const FixtureEngine* fixture(const clm_b200_engine* e) { return as_fixture(const_cast<clm_b200_engine*>(e)); }

}  // namespace

extern "C" {

int clm_b200_llama_create(clm_b200_ctx* ctx, const clm_b200_llama_geometry* g, const clm_b200_stage_spec* spec,
                          clm_b200_engine** out) {
  return llama_create(ctx, g, spec, out);
}

int clm_b200_fixture_create(clm_b200_ctx* ctx, const clm_b200_fixture_geometry* g, const clm_b200_stage_spec* spec,
                            clm_b200_engine** out) {
  return fixture_create(ctx, g, spec, out);
}

int clm_b200_engine_destroy(clm_b200_engine* e) {
  if (e == nullptr) return CLM_OK;
  clm_b200_ctx* ctx = e->ctx;
  delete e;
  ctx_release(ctx);
  return CLM_OK;
}

int clm_b200_engine_generate_weights(clm_b200_engine* e, uint64_t seed, float stddev) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED,
            "synthetic weights are generated for the Llama family; fixture objects come from the fixture generator");
  return llama_generate_weights(llama(e), seed, stddev);
}

int clm_b200_llama_load_tensors(clm_b200_engine* e, const clm_b200_tensor* tensors, uint32_t n) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "GGUF tensors bind to Llama-family engines");
  return llama_load_tensors(llama(e), tensors, n);
}

int clm_b200_engine_set_object(clm_b200_engine* e, const char* name, int quant, const void* h_bytes, uint64_t nbytes) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_FIXTURE, CLM_UNIMPLEMENTED, "object binding is implemented for the fixture family");
  return fixture_set_object(fixture(e), name, quant, h_bytes, nbytes);
}

int clm_b200_engine_prepare(clm_b200_engine* e) {
  CLM_TRY(enter(e));
  return e->family == CLM_FAMILY_LLAMA ? llama_prepare(llama(e)) : fixture_prepare(fixture(e));
}

int clm_b200_engine_info(const clm_b200_engine* e, uint64_t* weight_bytes, uint64_t* state_bytes, uint32_t* fpp) {
  CLM_CHECK(e != nullptr, CLM_INVALID_ARGUMENT, "null engine");
  return e->family == CLM_FAMILY_LLAMA ? llama_info(llama(e), weight_bytes, state_bytes, fpp)
                                       : fixture_info(fixture(e), weight_bytes, state_bytes, fpp);
}

int clm_b200_session_open(clm_b200_engine* e, uint64_t id) {
  CLM_TRY(enter(e));
  return e->family == CLM_FAMILY_LLAMA ? llama_session_open(llama(e), id) : fixture_session_open(fixture(e), id);
}

int clm_b200_session_close(clm_b200_engine* e, uint64_t id) {
  CLM_TRY(enter(e));
  return e->family == CLM_FAMILY_LLAMA ? llama_session_close(llama(e), id) : fixture_session_close(fixture(e), id);
}

int clm_b200_run_window(clm_b200_engine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_tokens,
                        const float* h_in, float* h_out, float* h_logits) {
  CLM_TRY(enter(e));
  if (e->family == CLM_FAMILY_LLAMA) return llama_run_window(llama(e), id, base, q, h_tokens, h_in, h_out, h_logits);
  return fixture_run_window(fixture(e), id, base, q, h_tokens, h_in, h_out, h_logits, false, nullptr);
}

int clm_b200_run_window_device(clm_b200_engine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* d_tokens,
                               const float* d_in, float* d_out, float* d_logits, void* stream) {
  CLM_TRY(enter(e));
  if (e->family == CLM_FAMILY_LLAMA)
    return llama_run_window_device(llama(e), id, base, q, d_tokens, d_in, d_out, d_logits, stream);
  return fixture_run_window(fixture(e), id, base, q, d_tokens, d_in, d_out, d_logits, true, stream);
}

int clm_b200_commit(clm_b200_engine* e, uint64_t id, uint32_t accepted) {
  CLM_TRY(enter(e));
  return e->family == CLM_FAMILY_LLAMA ? llama_commit(llama(e), id, accepted) : fixture_commit(fixture(e), id, accepted);
}

int clm_b200_run_tree_window(clm_b200_engine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_parents,
                             const int32_t* h_tokens, const float* h_in, float* h_out, float* h_logits) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "tree windows are served by the Llama-family engine");
  return llama_run_tree(llama(e), id, base, q, h_parents, h_tokens, h_in, h_out, h_logits);
}

int clm_b200_commit_path(clm_b200_engine* e, uint64_t id, const int32_t* h_path, uint32_t n) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "tree windows are served by the Llama-family engine");
  return llama_commit_path(llama(e), id, h_path, n);
}

int clm_b200_abort(clm_b200_engine* e, uint64_t id) {
  CLM_TRY(enter(e));
  return e->family == CLM_FAMILY_LLAMA ? llama_abort(llama(e), id) : fixture_abort(fixture(e), id);
}

int clm_b200_session_position(const clm_b200_engine* e, uint64_t id, uint64_t* committed) {
  CLM_CHECK(e != nullptr && committed != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  return e->family == CLM_FAMILY_LLAMA ? llama_session_position(llama(e), id, committed)
                                       : fixture_session_position(fixture(e), id, committed);
}

int clm_b200_engine_last_launches(const clm_b200_engine* e, uint64_t* launches) {
  CLM_CHECK(e != nullptr && launches != nullptr, CLM_INVALID_ARGUMENT, "null argument");
  *launches = e->last_launches;
  return CLM_OK;
}

int clm_b200_mtp_draft(clm_b200_engine* e, int32_t prev, uint32_t count, float T, uint64_t seed, uint64_t counter,
                       int32_t* h_tokens, float* h_logits) {
  CLM_TRY(enter(e));
  if (e->family == CLM_FAMILY_LLAMA) return llama_mtp_draft(llama(e), prev, count, T, seed, counter, h_tokens, h_logits);
  return fixture_mtp_draft(fixture(e), prev, count, T, seed, counter, h_tokens, h_logits);
}

int clm_b200_mtp_propose(clm_b200_engine* e, int32_t prev, uint32_t count, float temperature, uint32_t top_k,
                         float top_p, const double* h_uniforms, int32_t* h_tokens, float* h_probs) {
  CLM_TRY(enter(e));
  if (e->family == CLM_FAMILY_LLAMA)
    return llama_mtp_propose(llama(e), prev, count, temperature, top_k, top_p, h_uniforms, h_tokens, h_probs);
  return fixture_mtp_propose(fixture(e), prev, count, temperature, top_k, top_p, h_uniforms, h_tokens, h_probs);
}

int clm_b200_spec_begin(clm_b200_engine* e, uint64_t id, const int32_t* h_prompt, uint32_t n,
                        const clm_b200_spec_params* p) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "device-resident rounds are implemented for the Llama family");
  return llama_spec_begin(llama(e), id, h_prompt, n, p);
}

int clm_b200_spec_round(clm_b200_engine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* h_tokens,
                        uint32_t* h_count) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "device-resident rounds are implemented for the Llama family");
  return llama_spec_round(llama(e), id, p, h_tokens, h_count);
}

int clm_b200_spec_round_device(clm_b200_engine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* d_tokens,
                               uint32_t* d_count, void* stream) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "device-resident rounds are implemented for the Llama family");
  return llama_spec_round_device(llama(e), id, p, d_tokens, d_count, stream);
}

int clm_b200_run_tree_window_device(clm_b200_engine* e, uint64_t id, uint64_t base, uint32_t positions,
                                    const int32_t* d_parents, const int32_t* d_tokens, const float* d_in, float* d_out,
                                    float* d_logits, void* stream) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "tree windows are implemented for the Llama family");
  return llama_run_tree_device(llama(e), id, base, positions, d_parents, d_tokens, d_in, d_out, d_logits, stream);
}

int clm_b200_run_batch_window(clm_b200_engine* e, uint32_t n_sessions, const uint64_t* sessions, const uint64_t* bases,
                              uint32_t positions, const int32_t* h_parents, const int32_t* h_tokens, float* h_logits) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "batched windows are implemented for the Llama family");
  return llama_run_batch(llama(e), n_sessions, sessions, bases, positions, h_parents, h_tokens, h_logits);
}

int clm_b200_run_batch_window_device(clm_b200_engine* e, uint32_t n_sessions, const uint64_t* sessions,
                                     const uint64_t* bases, uint32_t positions, const int32_t* d_tokens,
                                     const float* d_in, float* d_out, float* d_logits, void* stream) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "batched windows are implemented for the Llama family");
  return llama_run_batch_device(llama(e), n_sessions, sessions, bases, positions, d_tokens, d_in, d_out, d_logits,
                                stream);
}

static int llama_only(clm_b200_engine* e) {
  CLM_TRY(enter(e));
  CLM_CHECK(e->family == CLM_FAMILY_LLAMA, CLM_UNIMPLEMENTED, "stage pipelines are implemented for the Llama family");
  return CLM_OK;
}

int clm_b200_pipe_attach(clm_b200_engine* e, clm_b200_link* in, clm_b200_link* out) {
  CLM_TRY(llama_only(e));
  return llama_pipe_attach(llama(e), in, out);
}

int clm_b200_pipe_prefill(clm_b200_engine* e, uint64_t id, const int32_t* h_tokens, uint32_t positions, void* stream) {
  CLM_TRY(llama_only(e));
  return llama_pipe_prefill(llama(e), id, h_tokens, positions, stream);
}

int clm_b200_pipe_begin(clm_b200_engine* e, uint64_t id, uint32_t row, const clm_b200_spec_params* p, void* stream) {
  CLM_TRY(llama_only(e));
  return llama_pipe_begin(llama(e), id, row, p, stream);
}

int clm_b200_pipe_round(clm_b200_engine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* d_tokens,
                        uint32_t* d_count, void* stream) {
  CLM_TRY(llama_only(e));
  return llama_pipe_round(llama(e), id, p, d_tokens, d_count, stream);
}

int clm_b200_pipe_status(clm_b200_engine* e, void* stream) {
  CLM_TRY(llama_only(e));
  return llama_pipe_status(llama(e), stream);
}

int clm_b200_pipe_attach_session(clm_b200_engine* e, uint64_t id, clm_b200_link* in, clm_b200_link* out) {
  CLM_TRY(llama_only(e));
  return llama_pipe_attach_session(llama(e), id, in, out);
}

}  // extern "C"
