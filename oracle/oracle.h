/*
 * oracle.h — CPU restatement of ClusterLM's speculative-window hot path (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the checker for the B200 kernels.  Only the test suite, the smoke check and the
 * CPU-baseline leg of the benchmark may load it; the product library never links or calls it.
 *
 * Every function restates a reference algorithm and names the reference file:line it follows
 * (paths are relative to the clusterlm repository root).  Where the reference has no implementation
 * (Q4_K, Philox, the Llama-shaped decoder, tree attention) the function says so and the parity of
 * that piece is pinned by other means (gguf-py decode, published Philox known-answer vectors) or is
 * marked "parity unpinned".
 *
 * Arithmetic conventions (match the reference's reference_math.hpp:1-6): single-threaded fixed
 * ascending-order float reductions, compiled with -ffp-contract=off so no FMA changes rounding.
 */
#ifndef CLM_ORACLE_H
#define CLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Quant identifiers shared with the product ABI (clm_b200.h). */
enum { ORC_F32 = 0, ORC_Q8_FIXTURE = 1, ORC_Q8_0 = 2, ORC_Q4_K = 3 };

/* ---- binary16 (runtime/objects/src/tensor_codec.cpp:16-73) ---------------------------------- */
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);

/* ---- tensor codecs (tensor_codec.cpp:9-14 sizes, :75-99 decode, :110-141 encoders) ----------- */
uint64_t orc_tensor_bytes(int quant, uint64_t n_elems);
/* 0 ok, 1 bad type/count, 7 size mismatch (the reference's kInvalidArgument / kDataLoss codes). */
int orc_decode_tensor(int quant, const uint8_t* bytes, uint64_t nbytes, float* out, uint64_t n);
int orc_encode_q8_fixture(const float* v, uint64_t n, uint8_t* out);
int orc_encode_q8_0(const float* v, uint64_t n, uint8_t* out);
/* Q4_K: not in the reference's code (only its size, runtime/objects/src/ggml_types.cpp:26).  The
 * encoder is this project's own deterministic min/max quantiser over the public ggml block format;
 * decode follows the published format (pinned bit-exactly against gguf-py 0.19.0 by the tests). */
int orc_encode_q4_k(const float* v, uint64_t n, uint8_t* out);

/* ---- reference_math / reference_kernels (reference_math.hpp:12-48, reference_kernels.cpp:9-30) */
float orc_dot(const float* a, const float* b, uint64_t n);
void orc_matvec(const float* w, uint64_t rows, uint64_t cols, const float* x, float* y);
void orc_rmsnorm(const float* x, const float* w, uint64_t n, float eps, float* out);
float orc_silu(float z);
float orc_sigmoid(float z);
/* y[p][i] = W[i] . x[p], output p-major (reference_kernels.cpp:24-30). */
void orc_matmul_rows(const float* w, uint64_t rows, uint64_t cols, const float* x, uint64_t positions, float* y);
/* Same, with W given as quantised rows that are decoded one row at a time, spread over `threads`
 * POSIX threads by row ranges (each output element is still one ascending-order dot). */
int orc_matmul_rows_quant(int quant, const uint8_t* wbytes, uint64_t rows, uint64_t cols, const float* x,
                          uint64_t positions, float* y, int threads);

/* ---- RNG ------------------------------------------------------------------------------------ */
/* xoshiro256** seeded by splitmix64 (runtime/domain/src/sampling.cpp:10-35). */
typedef struct { uint64_t s[4]; } orc_rng;
void orc_rng_seed(orc_rng* r, uint64_t seed);
uint64_t orc_rng_next(orc_rng* r);
double orc_rng_uniform(orc_rng* r);
uint64_t orc_mix_seed(uint64_t a, uint64_t b); /* sampling.cpp:37-42 */
uint64_t orc_mix64(uint64_t z);                /* drafter.cpp:10-15, reference_domain.cpp:24-29 */
/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11).  Not in the reference (it names Philox only as a
 * comment, runtime/backends/strata-core/src/mtp_drafter.cpp:29). */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
/* Uniform double in [0,1) from counter (c0..c3) under a 64-bit key, built like Rng::uniform()
 * (sampling.cpp:33): the top 53 bits of (out0:out1). */
double orc_philox_uniform(uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3);

/* ---- sampling (sampling.cpp:44-131) --------------------------------------------------------- */
int32_t orc_argmax(const float* logits, uint64_t n);
void orc_distribution(const float* logits, uint64_t n, float temperature, uint32_t top_k, float top_p, float* out);
/* sample_from with the uniform supplied by the caller (the reference draws it from its Rng). */
int32_t orc_sample_from(const float* probs, uint64_t n, double u);
/* verify_speculative over one sequence: target is (k+1) x V, draft_probs is k x V or NULL (one-hot
 * drafter).  Uniforms are consumed from `uniforms` in the reference's order (one per acceptance test
 * with q > 0, then one for the final sample); *used receives how many were consumed. */
void orc_verify_speculative(const float* target, const int32_t* drafts, const float* draft_probs, uint32_t k,
                            uint64_t vocab, const double* uniforms, uint32_t* accepted, int32_t* next_token,
                            uint32_t* used);

/* ---- drafters (runtime/domain/src/drafter.cpp:39-109) ---------------------------------------- */
/* One MTP fixture step: argmax(head . rmsnorm(embd[prev], norm)), ties to the lowest index. */
int32_t orc_mtp_fixture_step(const float* embd, const float* norm, const float* head, uint32_t hidden, uint32_t vocab,
                             int32_t prev);
/* ScriptedDrafter::draft: replay `ref` with deterministic corruption. */
void orc_scripted_draft(const int32_t* ref, uint64_t ref_len, uint32_t vocab, uint64_t seed, double corruption_rate,
                        uint64_t committed_len, uint32_t count, int32_t* out);

/* ---- synthetic weights (counter-based; identical bits on host and device) --------------------- */
/* w[i] = std * IH4(i) / sqrt(1/3), IH4 = Irwin-Hall sum of four 22-bit Philox uniforms centred on 0,
 * keyed (seed, tensor_id, element index).  Integer sums are exact; one float multiply rounds. */
void orc_gen_weights(uint64_t seed, uint32_t tensor_id, uint64_t first, uint64_t n, float stddev, float* out);

/* ---- Llama-shaped decoder layer (no reference implementation: parity unpinned) ---------------- */
typedef struct {
  uint32_t hidden, n_heads, n_kv_heads, head_dim, ffn;
  float rope_theta, rms_eps;
} orc_llama_dims;
/* One decoder layer for `q` consecutive positions starting at `base`, in place on h[q][hidden].
 * Weights are quantised rows (quant) for wq|wk|wv (stacked rows), wo, wg|wu (stacked), wd.
 * kcache/vcache are [max_ctx][n_kv*head_dim] f32; positions base..base+q-1 are written.
 * Attention: row i attends slots 0..base+i (causal), or, when `parent` is non-NULL, the committed
 * prefix 0..base-1 plus its own ancestors inside the window (tree drafts: parent[i] < i or -1). */
/* K / V cache rows of one layer for q positions (rmsnorm, k|v rows of the q|k|v matrix, RoPE on k). */
int orc_llama_kv_rows(const orc_llama_dims* d, int quant, const uint8_t* wqkv, const float* attn_norm,
                      const float* h, uint64_t base, uint32_t q, float* kc, float* vc, int threads);
int orc_llama_layer(const orc_llama_dims* d, int quant, const uint8_t* wqkv, const uint8_t* wo, const uint8_t* wgu,
                    const uint8_t* wd, const float* attn_norm, const float* ffn_norm, float* kcache, float* vcache,
                    uint64_t base, uint32_t q, const int32_t* parent, float* h, int threads);

#ifdef __cplusplus
}
#endif
#endif
