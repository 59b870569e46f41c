// flow.cuh — the verify-window dataflow kernel of the Llama-shaped engine (flow.cu).
//
// One cooperative launch runs a stage's whole layer range (and the LM head when the stage has one) for a q-row
// window (q <= 16) as a sequence of phases:
//   per layer: QKV GEMV (RoPE + paged KV append) -> attention -> W_o GEMV (residual + ffn-norm preparation)
//              -> gate|up GEMV (SwiGLU + down preparation) -> down GEMV (residual + next-norm preparation)
//   then:      head GEMV (logits) for a tail / whole stage.
// There is no barrier between phases.  Weights never depend on activations, so each CTA's producer warp streams
// the weights of its units of every phase through one shared-memory ring without waiting for anything but a free
// slot; only the activation part of a unit (and the KV page that holds the window's own rows) waits, on a
// readiness counter of exactly the data that unit reads:
//   * a GEMV unit covers 512 input columns (two superblocks): it waits until every output group of the previous
//     phase that writes those columns has finished its epilogue (4 row groups of a residual GEMV, 8 gate|up row
//     groups, or the attention outputs of the heads in those columns);
//   * an attention (m-tile, kv head) waits for the 6 QKV row groups of its heads (query heads, k head, v head);
//   * the row scale (folded rmsnorm) of the QKV, gate|up and head GEMVs needs every row group of the previous
//     residual phase: a CTA waits for that count only when it flushes its first row group of the phase.
// Every group signals with one release-add after its epilogue; readers acquire the counter (and fence the async
// proxy before bulk-copying what other CTAs wrote).  Every phase only waits on earlier phases and all CTAs are
// co-resident (cooperative launch, one CTA per SM), so every wait ends; each is bounded all the same.
#pragma once
#include "gemv_core.cuh"

namespace clm {

enum { FLOW_GEMV = 0, FLOW_ATTN = 1 };

// One attention segment partial row (head dim 128): O[128], m, l, 2 floats of padding (16-byte aligned rows).
constexpr int kFlowAttnRowFloats = 132;

struct FlowGemv {
  const uint8_t* tiles = nullptr;
  uint32_t rows = 0;
  int ng = 0;
  G4Geom geo;
  int maxseg = 0;  // partial slots per row group in `part`
  XBuf in;
  Epi epi;
  int epi_kind = 0;
  float* part = nullptr;   // stream-K segment partials [ng][maxseg][q][128] (one region per matrix kind)
  int* counters = nullptr;  // segment arrivals per row group (zero; reset by each group's first segment)
};

struct FlowAttn {
  const __half* q16 = nullptr;
  const __half* kpool = nullptr;  // this layer's pools: K [page][nkv][64][hd], V^T [page][nkv][hd][64] (swizzled)
  const __half* vpool = nullptr;
  const int32_t* pages = nullptr;  // the session's page table
  int nh = 0, nkv = 0, mtiles = 0, maxseg = 0;
  float scale_log2 = 0.0f;
  float* part = nullptr;    // [mtiles*nkv][maxseg][16][kFlowAttnRowFloats]
  int* counters = nullptr;  // [mtiles*nkv], zero (reset by the combining CTA)
  XBuf out;                 // W_o's input fragments
  float hi_scale = 1.0f;
  int nt_out = 1;
};

struct FlowPhase {
  int kind = FLOW_GEMV;
  FlowGemv g;
  FlowAttn a;
  // ---- dataflow (all counters zero at launch)
  int* wait = nullptr;     // readiness of the input: per 512-column chunk (GEMV) or per kv head (attention); null:
                           // the input was written before the launch
  int wait_target = 0;     // arrivals that make one chunk / kv head ready
  const int* ss_done = nullptr;  // row groups finished by the residual phase whose sums of squares give this phase's
  int ss_target = 0;             // row scale (null: no wait); its target
  int* sig = nullptr;      // counters this phase's finished groups signal (null: none)
  int sig_div = 1;         // GEMV: row group r signals sig[r / sig_div]
  int sig_qkv = 0;         // 1: QKV row group r (a head) signals its kv head
  int sig_span = 1;        // attention: a kv head's outputs cover sig_span chunks, signalled from kvh * sig_span
  int sig_kvh_div = 1;     //            (or kv heads share a chunk: chunk kvh / sig_kvh_div)
  int* done = nullptr;     // this phase's finished row groups (residual phases), or null
};

struct FlowParams {
  const FlowPhase* phases = nullptr;  // device array
  int nphases = 0;
  int q = 0;
  const long long* pos = nullptr;  // committed position = window base
  int* err = nullptr;
  int stages = 0;
  int stage_bytes = 0;
};

// Shared memory of the kernel for `stages` ring stages of `stage_bytes`.
size_t flow_smem_bytes(int stages, int stage_bytes);
// Ring stages that fit next to the kernel's fixed shared memory.
int flow_stages(int stage_bytes);
// Persistent grid (one co-resident CTA per SM) for the kernel on `device`, or 0 if it cannot launch cooperatively.
int flow_grid(int device, int stages, int stage_bytes, int quant, int nt);
// Zeroes the `ctr_bytes` of readiness counters at d_ctr, then launches the kernel (cooperative, `grid` CTAs).
int launch_flow(const FlowParams& p, int quant, int nt, int grid, int* d_ctr, size_t ctr_bytes, cudaStream_t st);

}  // namespace clm
