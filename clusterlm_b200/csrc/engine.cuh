// engine.cuh — the opaque engine behind clm_b200_engine*: a Llama-family engine (engine.cu) or a
// clusterlm-fixture-family engine (fixture.cu); engine_api.cu dispatches the C ABI on `family`.
#pragma once
#include "common.cuh"

enum { CLM_FAMILY_LLAMA = 0, CLM_FAMILY_FIXTURE = 1 };

struct clm_b200_engine {
  clm_b200_ctx* ctx = nullptr;
  int family = CLM_FAMILY_LLAMA;
  unsigned long long last_launches = 0;  // kernels in the last window / round
  virtual ~clm_b200_engine() = default;
};

struct LlamaEngine;
struct FixtureEngine;

namespace clm {
LlamaEngine* as_llama(clm_b200_engine* e);      // static_cast, defined where the type is complete
FixtureEngine* as_fixture(clm_b200_engine* e);
// Llama family (engine.cu)
int llama_create(clm_b200_ctx* ctx, const clm_b200_llama_geometry* g, const clm_b200_stage_spec* spec,
                 clm_b200_engine** out);
int llama_generate_weights(LlamaEngine* e, uint64_t seed, float stddev);
int llama_load_tensors(LlamaEngine* e, const clm_b200_tensor* t, uint32_t n);
int llama_prepare(LlamaEngine* e);
int llama_info(const LlamaEngine* e, uint64_t* weight_bytes, uint64_t* state_bytes, uint32_t* fpp);
int llama_session_open(LlamaEngine* e, uint64_t id);
int llama_session_close(LlamaEngine* e, uint64_t id);
int llama_run_window_device(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* d_tokens,
                            const float* d_in, float* d_out, float* d_logits, void* stream);
int llama_run_window(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_tokens, const float* h_in,
                     float* h_out, float* h_logits);
int llama_commit(LlamaEngine* e, uint64_t id, uint32_t accepted);
int llama_run_tree(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* h_parents,
                   const int32_t* h_tokens, const float* h_in, float* h_out, float* h_logits);
int llama_commit_path(LlamaEngine* e, uint64_t id, const int32_t* h_path, uint32_t n);
int llama_run_tree_device(LlamaEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* d_parents,
                          const int32_t* d_tokens, const float* d_in, float* d_out, float* d_logits, void* stream);
int llama_run_batch_device(LlamaEngine* e, uint32_t n, const uint64_t* ids, const uint64_t* bases, uint32_t q,
                           const int32_t* d_tokens, const float* d_in, float* d_out, float* d_logits, void* stream);
int llama_run_batch(LlamaEngine* e, uint32_t n, const uint64_t* ids, const uint64_t* bases, uint32_t q,
                    const int32_t* h_parents, const int32_t* h_tokens, float* h_logits);
int llama_abort(LlamaEngine* e, uint64_t id);
int llama_session_position(const LlamaEngine* e, uint64_t id, uint64_t* committed);
int llama_mtp_draft(LlamaEngine* e, int32_t prev, uint32_t count, float T, uint64_t seed, uint64_t counter,
                    int32_t* h_tokens, float* h_logits);
int llama_mtp_propose(LlamaEngine* e, int32_t prev, uint32_t count, float T, uint32_t top_k, float top_p,
                      const double* h_uniforms, int32_t* h_tokens, float* h_probs);
int llama_spec_begin(LlamaEngine* e, uint64_t id, const int32_t* h_prompt, uint32_t n, const clm_b200_spec_params* p);
int llama_spec_round_device(LlamaEngine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* d_tokens,
                            uint32_t* d_count, void* stream);
int llama_spec_round(LlamaEngine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* h_tokens, uint32_t* h_count);
int llama_pipe_attach(LlamaEngine* e, clm_b200_link* in, clm_b200_link* out);
int llama_pipe_prefill(LlamaEngine* e, uint64_t id, const int32_t* h_tokens, uint32_t q, void* stream);
int llama_pipe_begin(LlamaEngine* e, uint64_t id, uint32_t row, const clm_b200_spec_params* p, void* stream);
int llama_pipe_round(LlamaEngine* e, uint64_t id, const clm_b200_spec_params* p, int32_t* d_tokens, uint32_t* d_count,
                     void* stream);
int llama_pipe_status(LlamaEngine* e, void* stream);
int llama_pipe_attach_session(LlamaEngine* e, uint64_t id, clm_b200_link* in, clm_b200_link* out);
// fixture family (fixture.cu)
int fixture_create(clm_b200_ctx* ctx, const clm_b200_fixture_geometry* g, const clm_b200_stage_spec* spec,
                   clm_b200_engine** out);
int fixture_set_object(FixtureEngine* e, const char* name, int quant, const void* h_bytes, uint64_t nbytes);
int fixture_prepare(FixtureEngine* e);
int fixture_info(const FixtureEngine* e, uint64_t* weight_bytes, uint64_t* state_bytes, uint32_t* fpp);
int fixture_session_open(FixtureEngine* e, uint64_t id);
int fixture_session_close(FixtureEngine* e, uint64_t id);
int fixture_run_window(FixtureEngine* e, uint64_t id, uint64_t base, uint32_t q, const int32_t* tokens,
                       const float* in, float* out, float* logits, bool device, void* stream);
int fixture_commit(FixtureEngine* e, uint64_t id, uint32_t accepted);
int fixture_abort(FixtureEngine* e, uint64_t id);
int fixture_session_position(const FixtureEngine* e, uint64_t id, uint64_t* committed);
int fixture_mtp_draft(FixtureEngine* e, int32_t prev, uint32_t count, float T, uint64_t seed, uint64_t counter,
                      int32_t* h_tokens, float* h_logits);
int fixture_mtp_propose(FixtureEngine* e, int32_t prev, uint32_t count, float T, uint32_t top_k, float top_p,
                        const double* h_uniforms, int32_t* h_tokens, float* h_probs);
}  // namespace clm
