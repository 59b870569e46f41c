/*
 * clm_b200.h — C ABI of the B200-native ClusterLM speculative-window backend (libclm_b200.so).
 *
 * Plain pointers and sizes only.  Every call returns an int status whose values equal
 * clusterlm::ErrorCode (runtime/common/include/clusterlm/common/status.hpp:15-36); the message of the
 * last failure on the calling thread is clm_b200_last_error().  No exception crosses this boundary.
 *
 * Pointer conventions: `d_` = device memory on the context's GPU, `h_` = host memory (pageable or pinned).
 * `stream` is a cudaStream_t (NULL = the context's own stream).  Calls that take device pointers are
 * asynchronous on that stream; calls that take host pointers synchronise before returning.
 *
 * Threading: a context, its matrices and engines are driven by one caller at a time
 * (runtime/domain/include/clusterlm/domain/reference_domain.hpp:4 "Not thread-safe").
 */
#ifndef CLM_B200_H
#define CLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CLM_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define CLM_API __attribute__((visibility("default")))
#else
#define CLM_API
#endif

/* Status codes: the numeric values of clusterlm::ErrorCode (status.hpp:15-36). */
enum {
  CLM_OK = 0,
  CLM_INVALID_ARGUMENT = 1,
  CLM_OUT_OF_RANGE = 2,
  CLM_NOT_FOUND = 3,
  CLM_ALREADY_EXISTS = 4,
  CLM_FAILED_PRECONDITION = 5,
  CLM_RESOURCE_EXHAUSTED = 6,
  CLM_DATA_LOSS = 7,
  CLM_STALE_EPOCH = 10,
  CLM_ABORTED = 11,
  CLM_DEADLINE_EXCEEDED = 13,
  CLM_VERSION_MISMATCH = 15,
  CLM_INTERNAL = 17,
  CLM_UNIMPLEMENTED = 18,
  CLM_HARDWARE_UNAVAILABLE = 19
};

/* Tensor representations (runtime/objects/include/clusterlm/objects/tensor_codec.hpp:23-28 for the
 * first three; Q4_K is the ggml 256-element / 144-byte superblock, ggml_types.cpp:26). */
enum { CLM_QUANT_F32 = 0, CLM_QUANT_Q8_FIXTURE = 1, CLM_QUANT_Q8_0 = 2, CLM_QUANT_Q4_K = 3 };

/* ---- library / context ------------------------------------------------------------------------ */
CLM_API int clm_b200_abi_version(void);
CLM_API const char* clm_b200_last_error(void);
/* Number of visible CUDA devices (0 without a GPU: the backend's BackendInfo::hardware_available). */
CLM_API int clm_b200_device_count(int* n);

typedef struct clm_b200_ctx clm_b200_ctx;
/* One context per (domain, GPU): owns a stream and every device allocation made through it
 * (runtime/domain/include/clusterlm/domain/execution_domain.hpp:4-7: a domain never shares pointers,
 * streams or allocators).  CLM_HARDWARE_UNAVAILABLE when the device is absent or not sm_100. */
CLM_API int clm_b200_ctx_create(int device, clm_b200_ctx** out);
CLM_API int clm_b200_ctx_destroy(clm_b200_ctx* ctx);
CLM_API int clm_b200_ctx_stream(clm_b200_ctx* ctx, void** stream);
CLM_API int clm_b200_ctx_synchronize(clm_b200_ctx* ctx);

/* ---- codecs (replaces objects::tensor_bytes / decode_tensor, tensor_codec.cpp:9-99) ------------ */
CLM_API uint64_t clm_b200_tensor_bytes(int quant, uint64_t n_elems);
/* Exact dequantisation on the device: f32 copy, q8_0-fixture f32(scale)*q, q8_0 f32(half scale)*q, and
 * Q4_K (d*sc)*q - (dmin*m) with each product and the difference rounded once in f32 (bit-identical to
 * the reference decoder for the first three and to gguf-py for Q4_K).  CLM_DATA_LOSS on a byte-count
 * mismatch, CLM_INVALID_ARGUMENT on an unknown type or a count that is not whole blocks. */
CLM_API int clm_b200_decode_tensor(clm_b200_ctx* ctx, int quant, const void* d_bytes, uint64_t nbytes, float* d_out,
                           uint64_t n_elems, void* stream);
/* Deterministic Q4_K / Q8_0 encoders on the device (Q8_0 follows tensor_codec.cpp:127-141; Q4_K is this
 * project's min/max quantiser).  n_elems must be whole blocks. */
CLM_API int clm_b200_encode(clm_b200_ctx* ctx, int quant, const float* d_in, uint64_t n_elems, void* d_out, void* stream);
/* Counter-based synthetic weights: out[i] = stddev * sqrt(3) * IH4(seed, tensor_id, first+i) / 2^22 where
 * IH4 is the centred sum of four 22-bit Philox4x32-10 outputs (no reference counterpart). */
CLM_API int clm_b200_generate_weights(clm_b200_ctx* ctx, uint64_t seed, uint32_t tensor_id, uint64_t first, uint64_t n,
                              float stddev, float* d_out, void* stream);

/* ---- resident q-row GEMM (replaces reference_matmul_rows, runtime/domain/src/reference_kernels.cpp:24-30) */
typedef struct clm_b200_matrix clm_b200_matrix;
/* Upload a rows x cols row-major tensor in its stored representation and repack it for the tiled
 * kernels (lossless byte permutation for Q4_K / Q8_0; f32 / q8_0-fixture are decoded exactly to f32, as
 * the reference does at prepare, reference_domain.cpp:222-231).  Q4_K and Q8_0 need rows % 16 == 0 and
 * cols % 256 == 0.  `h_bytes` is host memory; `d_bytes` (the _device variant) is device memory, read after a
 * device synchronisation (so work of any stream that writes it completes first). */
CLM_API int clm_b200_matrix_upload(clm_b200_ctx* ctx, int quant, const void* h_bytes, uint64_t nbytes, uint32_t rows,
                           uint32_t cols, clm_b200_matrix** out);
CLM_API int clm_b200_matrix_upload_device(clm_b200_ctx* ctx, int quant, const void* d_bytes, uint64_t nbytes, uint32_t rows,
                                  uint32_t cols, clm_b200_matrix** out);
CLM_API int clm_b200_matrix_free(clm_b200_matrix* m);
CLM_API int clm_b200_matrix_info(const clm_b200_matrix* m, int* quant, uint32_t* rows, uint32_t* cols, uint64_t* device_bytes);
/* y[p][i] = W[i] . x[p] for p < positions (output position-major, as reference_matmul_rows).
 * 1 <= positions <= 16: the bandwidth-bound q-row GEMV (fp16 tensor-core products, f32 accumulation) for Q4_K /
 * Q8_0, f32 for f32.  17 <= positions <= 256 (Q4_K / Q8_0 only, d_x 16-byte aligned): a tcgen05 tensor-core GEMM
 * with TMEM accumulators (weights dequantised to fp16 in shared memory, activations rounded to fp16). */
CLM_API int clm_b200_matmul_rows(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x, uint32_t positions,
                         float* d_y, void* stream);
/* The same product with all of its scratch in a fixed CLM_B200_STATIC_SCRATCH_BYTES device array compiled into
 * the library: the call allocates no device memory (clm_b200_matmul_rows may grow the context's scratch with
 * cudaMalloc).  No reference counterpart: the reference's CPU matmul needs no device scratch.  For callers
 * that must not allocate once admitted, e.g. a domain whose device memory is fully leased at prepare.
 * CLM_RESOURCE_EXHAUSTED when the matrix/positions need more scratch than the array holds (then use
 * clm_b200_matmul_rows); CLM_OUT_OF_RANGE for more than 516,096 rows.  One array per device: calls whose kernels
 * overlap on one device race on it, so serialise them per device.  Every call first clears the array's reduction
 * counters; a row group whose bounded reduction wait gave up is written as NaN.  The first call on a device
 * resolves the array's address (set-up); make it before any stream capture meant to contain later calls. */
#define CLM_B200_STATIC_SCRATCH_BYTES (8u << 20)
CLM_API int clm_b200_matmul_rows_static(clm_b200_ctx* ctx, const clm_b200_matrix* w, const float* d_x,
                                        uint32_t positions, float* d_y, void* stream);

/* ---- sampling and speculative acceptance (runtime/domain/src/sampling.cpp:44-131) --------------- */
/* argmax per row, ties to the lowest index (sampling.cpp:44-49). */
CLM_API int clm_b200_argmax_rows(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab, int32_t* d_out,
                         void* stream);
/* distribution() per row (sampling.cpp:51-86): temperature <= 0 gives one-hot argmax; otherwise
 * exp(double(l - max)/T) normalised in double and rounded to f32.  With top_k > 0 or top_p < 1 the rows are
 * truncated exactly as the reference orders them (stable descending sort, ties by lower index; top-p
 * cumulative and kept sum in sorted order). */
CLM_API int clm_b200_distribution_rows(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab,
                               float temperature, uint32_t top_k, float top_p, float* d_probs, void* stream);
/* sample_from() per row with one caller-supplied uniform per row (sampling.cpp:88-101).  The result is
 * bit-identical to the serial double-precision reference: exact prefix sums locate the index and an
 * error bound proves the serial rounding cannot change it; otherwise the row is re-walked serially. */
CLM_API int clm_b200_sample_rows(clm_b200_ctx* ctx, const float* d_probs, uint32_t rows, uint32_t vocab,
                         const double* d_uniforms, int32_t* d_out, void* stream);
/* verify_speculative() for `batch` sequences (sampling.cpp:103-131).
 *   d_target      [batch][k+1][vocab] target probabilities
 *   d_drafts      [batch][k] drafted tokens
 *   d_draft_probs [batch][k][vocab] drafter probabilities, or NULL for a deterministic (one-hot) drafter
 *   d_uniforms    [batch][k+1] uniforms consumed in the reference's order (one per test with q > 0, then
 *                 one for the final sample), or NULL to draw them from Philox4x32-10 keyed by `seed` with
 *                 counter (draw, sequence, counter_base lo, counter_base hi)
 * Outputs d_accepted[batch] (0..k) and d_next[batch] (resampled or bonus token). */
CLM_API int clm_b200_verify_speculative(clm_b200_ctx* ctx, const float* d_target, const int32_t* d_drafts,
                                const float* d_draft_probs, uint32_t batch, uint32_t k, uint32_t vocab,
                                const double* d_uniforms, uint64_t seed, uint64_t counter_base, uint32_t* d_accepted,
                                int32_t* d_next, void* stream);
/* Fused acceptance straight from logits (no probability arrays written): P = distribution(target/T),
 * Q = distribution(draft/T) computed on the fly, then verify_speculative as above.
 *   d_target_logits [batch][k+1][vocab], d_draft_logits [batch][k][vocab] (NULL = one-hot drafter).
 * temperature > 0, no top-k / top-p. */
CLM_API int clm_b200_accept_logits(clm_b200_ctx* ctx, const float* d_target_logits, const float* d_draft_logits,
                           const int32_t* d_drafts, uint32_t batch, uint32_t k, uint32_t vocab, float temperature,
                           const double* d_uniforms, uint64_t seed, uint64_t counter_base, uint32_t* d_accepted,
                           int32_t* d_next, void* stream);
/* Vocab-sharded distribution rows (the LM head split by vocabulary over GPUs; no reference counterpart: the
 * reference computes distribution(), sampling.cpp:51-86, over whole rows).  A rank holds the logits of columns
 * [first_col, first_col + vocab_shard) of `rows` rows (first_col a multiple of 16384, the statistics chunk).
 * clm_b200_shard_stats writes, per row and 16384-column chunk of the shard (C = ceil(vocab_shard / 16384) per row),
 * the chunk's maximum (d_chunk_max, float[rows][C]) and the double sum of exp(double(l - chunk max) / T)
 * (d_chunk_sum, double[rows][C]): the same values as the whole-row statistics compute for those chunks. */
CLM_API int clm_b200_shard_stats(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab_shard,
                                 uint64_t first_col, float temperature, float* d_chunk_max, double* d_chunk_sum,
                                 void* stream);
/* The whole rows' maximum (d_max, float[rows]) and kept sum (d_kept, double[rows]) from every rank's chunk
 * statistics gathered as d_chunk_max / d_chunk_sum [world][rows][max_chunks] (rank w's first h_counts[w] chunks of
 * each row valid), combined in column order exactly as the whole-row statistics combine their chunks, so the
 * results equal those of clm_b200_distribution_rows over the gathered rows bit for bit.  world <= 64. */
CLM_API int clm_b200_shard_combine(clm_b200_ctx* ctx, const float* d_chunk_max, const double* d_chunk_sum,
                                   uint32_t world, const uint32_t* h_counts, uint32_t rows, uint32_t max_chunks,
                                   float temperature, float* d_max, double* d_kept, void* stream);
/* The shard's probabilities float(exp(double(l - max) / T) / kept) from the rows' global max and kept sum: the same
 * values clm_b200_distribution_rows writes for those columns of the whole rows. */
CLM_API int clm_b200_shard_probs(clm_b200_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t vocab_shard,
                                 float temperature, const float* d_global_max, const double* d_kept, float* d_probs,
                                 void* stream);
/* Philox4x32-10 uniforms: out[i] = top 53 bits of (o0:o1) * 2^-53 for counter (first+i lo, hi, c2, c3). */
CLM_API int clm_b200_philox_uniforms(clm_b200_ctx* ctx, uint64_t seed, uint64_t first, uint32_t c2, uint32_t c3, uint64_t n,
                             double* d_out, void* stream);

/* ---- execution engine: one stage (a contiguous layer range) of a model on one GPU ------------------
 * Replaces the CPU ReferenceDomain's compute (runtime/domain/src/reference_domain.cpp:376-585) behind
 * ExecutionDomain::run_prefix / run_window / run_tail / commit_window / abort_window
 * (runtime/domain/include/clusterlm/domain/execution_domain.hpp:143-174).  Admission (epochs, window IDs,
 * state versions) stays with the caller's WindowLedger; the engine checks positions and sizes. */
typedef struct clm_b200_engine clm_b200_engine;

/* StageRole (execution_domain.hpp:41) plus WHOLE = prefix and tail in one engine (tokens in, logits out). */
enum { CLM_ROLE_PREFIX = 0, CLM_ROLE_MIDDLE = 1, CLM_ROLE_TAIL = 2, CLM_ROLE_WHOLE = 3 };

/* Llama-shaped decoder: RMSNorm, GQA attention with RoPE, SwiGLU FFN; weights Q4_K or Q8_0; fp16 paged KV.
 * No reference implementation (the reference runs this family only through un-vendored llama.cpp; its
 * geometry mapping is runtime/backends/llama/include/clusterlm/backends/llama_manifest.hpp:5-9: hc = 1). */
typedef struct {
  uint32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
  float rope_theta, rms_eps;
  int quant;    /* CLM_QUANT_Q4_K or CLM_QUANT_Q8_0 */
  uint32_t mtp; /* 1: a one-layer MTP draft head (SwiGLU block over the previous token's embedding, shared LM head) */
} clm_b200_llama_geometry;

/* DomainSpec (execution_domain.hpp:44-58). */
typedef struct {
  uint32_t layer_begin, layer_end;
  int role;
  uint32_t max_context, max_window, max_sessions;
} clm_b200_stage_spec;

CLM_API int clm_b200_llama_create(clm_b200_ctx* ctx, const clm_b200_llama_geometry* geometry,
                                  const clm_b200_stage_spec* spec, clm_b200_engine** out);
CLM_API int clm_b200_engine_destroy(clm_b200_engine* e);
/* Counter-based synthetic weights for every tensor of this stage (clm_b200_generate_weights' generator,
 * tensor id 16*layer + {q,k,v,o,gate,up,down} = {0..6}; 1000 embedding, 1001 output head, 1002..1004 MTP
 * gate/up/down), encoded in the geometry's quant; norm weights are 1.  Replaces provisioning for tests and
 * benchmarks (random-init weights of the named architecture). */
CLM_API int clm_b200_engine_generate_weights(clm_b200_engine* e, uint64_t seed, float stddev);
/* One named host tensor: GGUF block bytes (quant = CLM_QUANT_Q4_K / CLM_QUANT_Q8_0) or f32 (CLM_QUANT_F32). */
typedef struct {
  const char* name;
  int quant;
  const void* data;
  uint64_t bytes;
} clm_b200_tensor;
/* Binds this stage's weights from tensors in llama.cpp's GGUF names and block layout (the weights of a GGUF file;
 * ClusterLM's GGUF manifests, runtime/objects/src/gguf_manifest.cpp, name the same tensors): token_embd.weight
 * (prefix / whole), blk.L.{attn_q,attn_k,attn_v,attn_output,ffn_gate,ffn_up,ffn_down}.weight in the geometry's
 * quant and blk.L.{attn_norm,ffn_norm}.weight in f32 for the stage's layers, output.weight + output_norm.weight
 * (tail / whole), and for mtp = 1 the head mtp.{ffn_gate,ffn_up,ffn_down}.weight + mtp.{ffn_norm,output_norm}.weight.
 * The host buffers are read during the call only.  CLM_NOT_FOUND names a missing tensor, CLM_DATA_LOSS a size
 * that does not match the geometry, CLM_UNIMPLEMENTED another quantisation (a file must be quantised uniformly,
 * e.g. llama-quantize --pure). */
CLM_API int clm_b200_llama_load_tensors(clm_b200_engine* e, const clm_b200_tensor* tensors, uint32_t n);
/* Allocates sequence state and window buffers (ExecutionDomain::prepare, execution_domain.hpp:150). */
CLM_API int clm_b200_engine_prepare(clm_b200_engine* e);
/* Resident weight bytes, per-session state bytes and boundary floats per position (hc*H + H + hc). */
CLM_API int clm_b200_engine_info(const clm_b200_engine* e, uint64_t* weight_bytes, uint64_t* state_bytes_per_session,
                                 uint32_t* floats_per_position);
CLM_API int clm_b200_session_open(clm_b200_engine* e, uint64_t session);
CLM_API int clm_b200_session_close(clm_b200_engine* e, uint64_t session);
/* One verification window of `positions` rows (1..max_window; max_window <= 256: windows of more than 16 rows,
 * prefill chunks and large trees, run on the tensor-core path) at committed position `base`.
 *   prefix / whole: h_tokens[positions]; middle / tail: h_in[positions][floats_per_position]
 *   prefix / middle: h_out[positions][floats_per_position]; tail / whole: h_logits[positions][vocab]
 * The window's state changes (KV rows) are tentative until clm_b200_commit. */
CLM_API int clm_b200_run_window(clm_b200_engine* e, uint64_t session, uint64_t base, uint32_t positions,
                                const int32_t* h_tokens, const float* h_in, float* h_out, float* h_logits);
/* Same with device buffers on the engine's GPU (stage hand-off by peer copies). */
CLM_API int clm_b200_run_window_device(clm_b200_engine* e, uint64_t session, uint64_t base, uint32_t positions,
                                       const int32_t* d_tokens, const float* d_in, float* d_out, float* d_logits,
                                       void* stream);
/* Keeps the first `accepted` positions of the outstanding window (1..q): commit_window, reference_domain.cpp:297-317. */
CLM_API int clm_b200_commit(clm_b200_engine* e, uint64_t session, uint32_t accepted);
/* Tree verification window (no reference counterpart: the reference's windows are linear,
 * coordinator.cpp:1244-1255).  Node i has parent h_parents[i] (an earlier node, or -1 for the committed
 * context); it is placed at KV slot base + i, rotated (RoPE) at position base + depth(i), and attends to the
 * committed context and its own ancestors.  Llama-family engines. */
CLM_API int clm_b200_run_tree_window(clm_b200_engine* e, uint64_t session, uint64_t base, uint32_t positions,
                                     const int32_t* h_parents, const int32_t* h_tokens, const float* h_in,
                                     float* h_out, float* h_logits);
/* Same with device buffers; the parent array is validated on the device (an entry that is not -1 or an earlier
 * node is replaced by -1 and the next commit reports CLM_INVALID_ARGUMENT). */
CLM_API int clm_b200_run_tree_window_device(clm_b200_engine* e, uint64_t session, uint64_t base, uint32_t positions,
                                            const int32_t* d_parents, const int32_t* d_tokens, const float* d_in,
                                            float* d_out, float* d_logits, void* stream);
/* Commits the accepted root-to-node path h_path[0..n) of the outstanding (tree or linear) window: the path's KV
 * rows move to slots base..base+n-1 and the committed position advances by n (commit_window's keep-prefix rule
 * for a tree). */
CLM_API int clm_b200_commit_path(clm_b200_engine* e, uint64_t session, const int32_t* h_path, uint32_t n);
/* One window over several sessions at once (no reference counterpart: the reference runs one window per
 * ExecutionDomain call, reference_domain.cpp:376-445): session sessions[b] verifies `positions` (<= 16) rows at
 * its committed position bases[b], as a tree with the shared parent array h_parents (see
 * clm_b200_run_tree_window) or linearly when h_parents is null.  Every weight matrix is read once for all
 * n_sessions * positions rows (17..max_window rows, the tensor-core path).  h_tokens[n_sessions][positions];
 * h_logits[n_sessions][positions][vocab] (optional).  Whole-model engines.  Each session then commits with
 * clm_b200_commit_path / clm_b200_commit (linear) or drops its window with clm_b200_abort. */
CLM_API int clm_b200_run_batch_window(clm_b200_engine* e, uint32_t n_sessions, const uint64_t* sessions,
                                      const uint64_t* bases, uint32_t positions, const int32_t* h_parents,
                                      const int32_t* h_tokens, float* h_logits);
/* A batched window on the q-row GEMV chain, for stages of any role: sessions[b] (n_sessions <= 4) verifies
 * `positions` (<= 8) linear rows at its committed position bases[b]; every weight matrix of the stage streams once for
 * all n_sessions * positions rows (<= 32, and <= max_window), with each session's KV rows and attention its own.
 * Device buffers on the engine's GPU, rows session-major:
 *   prefix / whole: d_tokens[n][positions]; middle / tail: d_in[n][positions][floats_per_position]
 *   prefix / middle: d_out[n][positions][floats_per_position]; tail / whole: d_logits[n][positions][vocab]
 * (no reference counterpart: the reference runs one window per ExecutionDomain call).  Each session then commits or
 * aborts on its own. */
CLM_API int clm_b200_run_batch_window_device(clm_b200_engine* e, uint32_t n_sessions, const uint64_t* sessions,
                                             const uint64_t* bases, uint32_t positions, const int32_t* d_tokens,
                                             const float* d_in, float* d_out, float* d_logits, void* stream);
/* Drops the outstanding window (abort_window, reference_domain.cpp:319-329). */
CLM_API int clm_b200_abort(clm_b200_engine* e, uint64_t session);
CLM_API int clm_b200_session_position(const clm_b200_engine* e, uint64_t session, uint64_t* committed);
/* Kernel launches in the last window or speculative round (the CUDA graph's kernel nodes). */
CLM_API int clm_b200_engine_last_launches(const clm_b200_engine* e, uint64_t* launches);

/* MTP draft head (tail / whole with mtp = 1): `count` chained draft tokens after `prev`
 * (MtpFixtureDrafter::draft / propose, runtime/domain/src/drafter.cpp:59-89): greedy argmax when
 * temperature <= 0, else sampled from distribution(logits, T) with Philox draws (seed, draw j, stream 1,
 * counter).  h_logits (optional) receives the [count][vocab] draft logits. */
CLM_API int clm_b200_mtp_draft(clm_b200_engine* e, int32_t prev, uint32_t count, float temperature, uint64_t seed,
                               uint64_t counter, int32_t* h_tokens, float* h_logits);

/* Stochastic MTP proposal (MtpFixtureDrafter::propose, runtime/domain/src/drafter.cpp:72-86): `count` chained drafts
 * after `prev`, draft j sampled from distribution(step logits, temperature, top_k, top_p) with the caller's uniform
 * h_uniforms[j] (the reference's sample_from draws one Rng uniform per draft, in this order).  h_probs (optional)
 * receives the [count][vocab] draft distributions, the Q rows of verify_speculative.  temperature <= 0: the greedy
 * draft with one-hot rows (h_uniforms unused). */
CLM_API int clm_b200_mtp_propose(clm_b200_engine* e, int32_t prev, uint32_t count, float temperature, uint32_t top_k,
                                 float top_p, const double* h_uniforms, int32_t* h_tokens, float* h_probs);

/* Device-resident speculative decoding on a WHOLE engine: one round = MTP draft of q-1 tokens, the q-row
 * verify window, acceptance (greedy prefix match, coordinator.cpp:1295-1298, or stochastic
 * verify_speculative with Philox draws keyed by (seed, session round)) and commit of accepted + 1
 * positions — one CUDA graph, no host round trip inside.  The round's parameters (16 bytes) are copied host
 * to device at every call. */
typedef struct {
  uint32_t q;
  float temperature;
  uint64_t seed;
} clm_b200_spec_params;
/* Prefills `n` prompt tokens (windows of max_window, each committed) and picks the first next token
 * (argmax, or a sample at temperature > 0). */
CLM_API int clm_b200_spec_begin(clm_b200_engine* e, uint64_t session, const int32_t* h_prompt, uint32_t n,
                                const clm_b200_spec_params* params);
/* One round; the emitted tokens (accepted drafts then the resampled/bonus token) go to h_tokens[0..*h_count). */
CLM_API int clm_b200_spec_round(clm_b200_engine* e, uint64_t session, const clm_b200_spec_params* params,
                                int32_t* h_tokens, uint32_t* h_count);
/* Same without host I/O: outputs stay in device memory (d_tokens[q], d_count). */
CLM_API int clm_b200_spec_round_device(clm_b200_engine* e, uint64_t session, const clm_b200_spec_params* params,
                                       int32_t* d_tokens, uint32_t* d_count, void* stream);

/* ---- stage pipeline across the GPUs of one node ----------------------------------------------------
 * Replaces the Father -> Node -> ... -> Father hops of a speculative window (RunWindow / StageResult over
 * TCP: orchestrator/coordinator/src/coordinator.cpp:736-832, runtime/transport) for stages placed on GPUs of
 * one box, one process (or context) per GPU.  A link is a one-way FIFO of `slots` messages of at most
 * `payload_bytes` between two GPUs: the sender's kernel stores each message into the receiver's memory over
 * NVLink and publishes it with a system-scope flag; the receiver's kernel waits for the flag (bounded by
 * `timeout_s`), copies the message out and returns a credit.  The two ends must be on different GPUs. */
typedef struct clm_b200_link clm_b200_link;
enum { CLM_LINK_SEND = 0, CLM_LINK_RECV = 1 };
#define CLM_B200_LINK_HANDLE_BYTES 128
CLM_API int clm_b200_link_create(clm_b200_ctx* ctx, int end, uint32_t slots, uint64_t payload_bytes, double timeout_s,
                                 clm_b200_link** out);
/* Writes this end's handle (CLM_B200_LINK_HANDLE_BYTES bytes) for the other end's process. */
CLM_API int clm_b200_link_export(const clm_b200_link* link, void* handle);
/* Maps the other end from its handle (a CUDA IPC mapping, or a peer pointer when both ends are in one process). */
CLM_API int clm_b200_link_connect(clm_b200_link* link, const void* peer_handle);
CLM_API int clm_b200_link_destroy(clm_b200_link* link);

/* Binds a stage engine into a speculative pipeline (Llama family, max_sessions sequences in flight):
 *   prefix: `in` receives window tokens from the tail, `out` sends boundary records to the next stage;
 *   middle: `in` receives records, `out` sends records;
 *   tail (with an MTP head): `in` receives records, `out` sends the next window's tokens to the prefix.
 * Every message carries the count of positions the receiver commits for the session before the window (the
 * tail's acceptance of the session's previous window: commit_window fan-out, coordinator.cpp:836-892). */
CLM_API int clm_b200_pipe_attach(clm_b200_engine* e, clm_b200_link* in, clm_b200_link* out);
/* One prompt chunk of `positions` (<= max_window) through this stage, committed at once (prefill with
 * auto_commit, coordinator.cpp:896-959).  The prefix takes h_tokens; the other stages receive records. */
CLM_API int clm_b200_pipe_prefill(clm_b200_engine* e, uint64_t session, const int32_t* h_tokens, uint32_t positions,
                                  void* stream);
/* Tail, after the prompt: the first next token from row `row` of the last prefill chunk's logits (argmax, or
 * a sample with Philox draw (0, stream 2, 0)), the first window's q-1 MTP drafts, sent to the prefix. */
CLM_API int clm_b200_pipe_begin(clm_b200_engine* e, uint64_t session, uint32_t row, const clm_b200_spec_params* params,
                                void* stream);
/* One speculative round of `session` on this stage, device-resident: wait for the input, commit the previous
 * round, run the window, forward.  The tail also accepts (as clm_b200_spec_round_device), commits, drafts the
 * next window and sends it to the prefix; its emitted tokens / count go to d_tokens / d_count (optional).
 * Every stage runs the same rounds of the same sessions in the same order.  A link delivers its messages in the
 * order they were sent, whatever their session: the prefix's rounds must come in the order of the tail's
 * clm_b200_pipe_begin / round calls that sent their windows. */
CLM_API int clm_b200_pipe_round(clm_b200_engine* e, uint64_t session, const clm_b200_spec_params* params,
                                int32_t* d_tokens, uint32_t* d_count, void* stream);
/* Synchronises the engine's stream; CLM_DEADLINE_EXCEEDED if a link wait gave up (a peer stage stopped). */
CLM_API int clm_b200_pipe_status(clm_b200_engine* e, void* stream);
/* Binds one session's messages to their own input / output links (NULL: the engine's, from
 * clm_b200_pipe_attach); the session's captured rounds are dropped.  Used by tail replicas: a plan may end in k
 * tail stages with the same layer range on k GPUs, replica j running the sessions s with s % k == j; the stage
 * before the replicas sends each session's records on the link to its replica and the prefix receives each
 * session's window tokens on the link from its replica.  The reference has one tail per plan (its Father's tail
 * domain, coordinator.cpp:736-892); replicas share the tail's LM head and MTP draft steps, the stage that no layer
 * split can make smaller. */
CLM_API int clm_b200_pipe_attach_session(clm_b200_engine* e, uint64_t session, clm_b200_link* in, clm_b200_link* out);

/* ---- clusterlm-fixture family: the reference's own model (hc gated residual streams, 3:1 recurrent /
 * attention layers without RoPE, top-K MoE with a shared SwiGLU expert, PLE n-gram lookup, injection gates;
 * runtime/domain/src/reference_domain.cpp:452-585).  Computed in f32 with the reference's ascending
 * reduction order and no FMA contraction. */
typedef struct {
  uint32_t n_layers, hidden, residual_streams, n_experts, n_active_experts, expert_ff, shared_expert_ff;
  uint32_t n_heads, n_kv_heads, head_dim, vocab, ple_layer, ple_ngram, ple_rows;
  const uint8_t* layer_kinds; /* n_layers entries: 0 recurrent, 1 full attention (geometry.hpp:16-19) */
} clm_b200_fixture_geometry;

CLM_API int clm_b200_fixture_create(clm_b200_ctx* ctx, const clm_b200_fixture_geometry* geometry,
                                    const clm_b200_stage_spec* spec, clm_b200_engine** out);
/* Binds one provisioned object by its manifest name ("blk.L.dense", "blk.L.shared", "blk.L.exp.E",
 * "token_embd", "ple_lookup", "output_head", "mtp_drafter"; runtime/objects/src/manifest.cpp:214-218) in its
 * stored representation (f32 or q8_0-fixture), decoded exactly on the device as the reference does at
 * prepare (reference_domain.cpp:191-245).  CLM_DATA_LOSS when the size does not match the geometry. */
CLM_API int clm_b200_engine_set_object(clm_b200_engine* e, const char* name, int quant, const void* h_bytes,
                                       uint64_t nbytes);

#ifdef __cplusplus
}
#endif
#endif
