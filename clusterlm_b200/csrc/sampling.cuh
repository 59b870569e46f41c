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

int launch_argmax(const float* d_logits, uint32_t rows, uint32_t vocab, int32_t* d_out, cudaStream_t st);
// mx[r] = max of row r; kept[r] = sum exp(double(l - mx) / T)
int launch_row_stats(const float* d_logits, uint32_t rows, uint32_t vocab, float T, float* d_mx, double* d_kept,
                     cudaStream_t st, const RoundCtl* ctl = nullptr);
// Stats layout: target row j of sequence b at b*(k+1)+j; draft row j at batch*(k+1) + b*k + j.
// counter_base is read from *d_counter when d_counter is not null.
int launch_accept_logits(const float* d_tl, const float* d_dl, const int32_t* d_drafts, uint32_t batch, uint32_t k,
                         uint32_t vocab, float T, const float* d_mx, const double* d_kept, const double* d_uniforms,
                         uint64_t seed, uint64_t counter_base, const unsigned long long* d_counter,
                         uint32_t* d_accepted, int32_t* d_next, cudaStream_t st, const RoundCtl* ctl = nullptr);
// One logits row -> token: argmax for T <= 0, else an exact sample of distribution(row, T) with the Philox
// uniform (draw, stream_id, *d_counter lo, hi) under key `seed`.
int launch_sample_logits(const float* d_logits, uint32_t vocab, float T, uint64_t seed, uint32_t draw,
                         uint32_t stream_id, const unsigned long long* d_counter, int32_t* d_out, cudaStream_t st,
                         const RoundCtl* ctl = nullptr);
}  // namespace clm
