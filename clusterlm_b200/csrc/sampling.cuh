// sampling.cuh — internal launchers of sampling.cu shared with the engines.
#pragma once
#include "common.cuh"

namespace clm {

// Sampling parameters read from device memory by graph-captured kernels (so a captured round can change
// its temperature value and seed without re-capture).
struct RoundCtl {
  float temperature;
  unsigned pad;
  unsigned long long seed;
};

constexpr uint32_t kSampleChunk = 2048;  // vocabulary entries per CTA
inline uint32_t sample_chunks(uint32_t V) { return (V + kSampleChunk - 1) / kSampleChunk; }

// Device scratch of the chunked row kernels for up to `rows` statistic rows and `seqs` sampled sequences.
// The first counter_bytes hold counters that must be zero before the first launch (every kernel leaves them
// zero).  One scratch must not be used by two launches that can run concurrently.
struct SampleScratch {
  uint32_t rows = 0, seqs = 0, chunks = 0;
  size_t counter_bytes = 0;
  int* rcnt = nullptr;               // [rows]
  int* scnt = nullptr;               // [seqs]
  float* cmax = nullptr;             // [rows][C]
  double* csum = nullptr;            // [rows][C]
  float* mx = nullptr;               // [rows]
  double* kept = nullptr;            // [rows]
  float* cval = nullptr;             // [rows][C] argmax chunks
  int32_t* cidx = nullptr;           // [rows][C]
  unsigned long long* c192 = nullptr;  // [seqs][2][C][3] exact chunk sums
  int32_t* clast = nullptr;          // [seqs][2][C]
  int* cflag = nullptr;              // [seqs][C]
  double* u = nullptr;               // [seqs]
  int32_t* sel = nullptr;            // [seqs]
  static size_t bytes(uint32_t rows, uint32_t seqs, uint32_t V);
  static SampleScratch carve(void* base, uint32_t rows, uint32_t seqs, uint32_t V);
};

// out[r] = argmax of row r (ties to the lowest index).
int launch_argmax_rows(const float* d_logits, uint32_t rows, uint32_t V, int32_t* d_out, const SampleScratch& s,
                       cudaStream_t st);
// Row statistics of distribution(logits[r], T) (max and kept) into scratch rows off + r.
int launch_row_stats(const float* d_logits, uint32_t rows, uint32_t V, float T, const RoundCtl* ctl, uint32_t off,
                     const SampleScratch& s, cudaStream_t st);
// probs[r] = distribution(logits[r], T) (temperature from ctl when given).
int launch_probs(const float* d_logits, uint32_t rows, uint32_t V, float T, const RoundCtl* ctl, float* d_probs,
                 const SampleScratch& s, cudaStream_t st);
// out[b] = sample_from(probs + b*row_stride, u_b): u_b = d_uniforms[b], or Philox(seed | ctl->seed, draw,
// stream_id, *d_counter) when d_uniforms is null.
int launch_sample_rows(const float* d_probs, uint32_t rows, uint64_t row_stride, uint32_t V, const double* d_uniforms,
                       uint64_t seed, uint32_t draw, uint32_t stream_id, const unsigned long long* d_counter,
                       const RoundCtl* ctl, int32_t* d_out, const SampleScratch& s, cudaStream_t st);
// One stochastic draft step: d_probs = distribution(d_logits, T, top_k, top_p) (T > 0; top-k / top-p truncation in
// the reference's exact order with scratch from the context), then *d_out = sample_from(d_probs, *d_u).
int launch_draft_sample(clm_b200_ctx* ctx, const float* d_logits, uint32_t V, float T, uint32_t top_k, float top_p,
                        const double* d_u, float* d_probs, int32_t* d_out, const SampleScratch& s, cudaStream_t st);
// The rows verify_speculative reads: target P [batch][k+1][V] and draft Q [batch][k][V] as probabilities, or as
// logits (LP / LQ) whose launch_row_stats statistics are at scratch rows 0.. (target) and q_stats_off.. (draft);
// the probabilities are then evaluated where they are used, bit-identical to launch_probs' output.  No Q and
// no LQ: one-hot drafts.
struct AcceptRows {
  const float* P = nullptr;
  const float* LP = nullptr;
  const float* Q = nullptr;
  const float* LQ = nullptr;
  uint32_t q_stats_off = 0;
  float T = 1.0f;  // logits-mode temperature (ctl's when given)
};
// verify_speculative for `batch` sequences.  Uniforms from d_uniforms [batch][k+1], else Philox(seed | ctl->seed,
// draw, sequence, counter_base | *d_counter).
int launch_accept(const AcceptRows& rows, const int32_t* d_drafts, uint32_t batch, uint32_t k, uint32_t V,
                  const double* d_uniforms, uint64_t seed, uint64_t counter_base,
                  const unsigned long long* d_counter, const RoundCtl* ctl, uint32_t* d_accepted, int32_t* d_next,
                  const SampleScratch& s, cudaStream_t st);
}  // namespace clm
