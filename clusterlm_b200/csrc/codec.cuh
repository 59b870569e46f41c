// codec.cuh — internal entry points of codec.cu shared with the engines.
#pragma once
#include "common.cuh"

namespace clm {

// One IEEE single multiply on the host (kept out of line of any expression so it rounds once).
inline float host_mul(float a, float b) {
  volatile float r = a * b;
  return r;
}

int launch_decode(int quant, const void* d_bytes, float* d_out, uint64_t n, cudaStream_t s);
// Generates n_elems synthetic weights of `tensor_id` (clm_b200_generate_weights' distribution) and writes them
// encoded as Q4_K or Q8_0 (GGUF block layout) into d_out.
int launch_gen_encode(int quant, uint64_t seed, uint32_t tensor_id, uint64_t n_elems, float stddev, void* d_out,
                      cudaStream_t s);

}  // namespace clm
