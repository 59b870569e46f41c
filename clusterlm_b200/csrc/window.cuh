// window.cuh — the verify-window megakernel of the Llama-shaped engine (window.cu).
//
// One cooperative launch runs a stage's whole layer range (and the LM head when the stage has one) for a q-row
// window as a sequence of phases separated by grid barriers:
//   per layer: QKV GEMV (RoPE + paged KV append) -> attention -> W_o GEMV (residual + ffn-norm preparation)
//              -> gate|up GEMV (SwiGLU + down preparation) -> down GEMV (residual + next-norm preparation)
//   then:      head GEMV (logits) for a tail / whole stage.
// The persistent CTAs (one per SM) keep one shared-memory ring of bulk-copy stages across all phases, so the
// producer warp streams the next phase's weights (and the committed KV pages) while the current phase finishes.
#pragma once
#include "gemv_core.cuh"

namespace clm {

enum { MK_GEMV = 0, MK_ATTN = 1 };

// One attention segment partial row (head dim 128): O[128], m, l, 2 floats of padding (16-byte aligned rows).
constexpr int kMkAttnRowFloats = 132;

struct MkGemv {
  const uint8_t* tiles = nullptr;
  uint32_t rows = 0;
  int ng = 0;
  G4Geom geo;
  int maxseg = 0;  // partial slots per row group in `part`
  XBuf in;
  Epi epi;
  int epi_kind = 0;
};

struct MkAttn {
  const __half* q16 = nullptr;
  const __half* kpool = nullptr;  // this layer's pools: K [page][nkv][64][hd], V^T [page][nkv][hd][64] (swizzled)
  const __half* vpool = nullptr;
  const int32_t* pages = nullptr;  // the session's page table
  int nh = 0, nkv = 0, mtiles = 0, maxseg = 0;
  float scale_log2 = 0.0f;
  float* part = nullptr;   // [mtiles*nkv][maxseg][16][kMkAttnRowFloats]
  int* counters = nullptr;  // [mtiles*nkv], zero
  XBuf out;                 // W_o's input fragments
  float hi_scale = 1.0f;
  int nt_out = 1;
};

struct MkPhase {
  int kind = MK_GEMV;
  MkGemv g;
  MkAttn a;
};

struct MkParams {
  const MkPhase* phases = nullptr;  // device array
  int nphases = 0;
  int q = 0;
  const long long* pos = nullptr;  // committed position = window base
  float* part = nullptr;           // GEMV segment partials
  int* counters = nullptr;         // GEMV row-group counters (zero)
  unsigned* barrier = nullptr;     // grid-barrier arrivals; zeroed before every launch
  int* err = nullptr;
  int stages = 0;
  int stage_bytes = 0;
};

// Shared memory of the megakernel for `stages` ring stages of `stage_bytes`.
size_t mk_smem_bytes(int stages, int stage_bytes);
// Ring stages that fit next to the megakernel's fixed shared memory.
int mk_stages(int stage_bytes);
// Persistent grid (co-resident CTAs) for the megakernel on `device`, or 0 if it cannot launch cooperatively.
int mk_grid(int device, int stages, int stage_bytes, int quant, int nt);
// Launches the megakernel (cooperative, `grid` CTAs); `p.barrier` must be zero (a memset is enqueued first).
int launch_window_mk(const MkParams& p, int quant, int nt, int grid, cudaStream_t st);

}  // namespace clm
