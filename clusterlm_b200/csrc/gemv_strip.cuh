// gemv_strip.cuh — the strip GEMV (gemv_strip.cu): q <= 8 window rows, K = 4096, every 16-row strip reduced inside
// one CTA.
#pragma once
#include "gemv2.cuh"

namespace clm {

// Whether the strip GEMV covers this matrix and window (16 superblocks per row, q <= 8, Q4_K / Q8_0).
bool gemv_strip_ok(const GemvShape& s, int q, int epi_kind);
// Ring stages of the strip GEMV for this matrix and epilogue (at least 2 when it is usable).
int strip_stages(const GemvShape& s, int epi_kind);
// y = W x with the fused epilogue `epi` (gemv2.cuh) over sm_count persistent CTAs.  The residual epilogue writes its
// sum-of-squares partials per 16 columns (the consumer's XBuf then has nss = cols / 16); the input's nss may be either
// granularity.  Dataflow counters (Epi::wait, ss_done, sig, done) count chunks of 512 input columns, and each strip
// signals once: 32 per chunk of the next input (8 per head for the QKV rows).
int launch_gemv_strip(const GemvShape& s, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi, int sm_count,
                      cudaStream_t st);

}  // namespace clm
