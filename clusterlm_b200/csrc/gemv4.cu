// gemv4.cu — persistent, warp-specialised, stream-K q-row GEMV with fused epilogues (sm_100a).
//
// y[p][row] = W[row] . x[p] for q <= 16 window rows, W in the group-major tile layout of gemv.cuh
// ([128-row group][superblock][8 row tiles]).  The work is the sequence of "units" (row group, superblock pair),
// U = ng * ceil(SB / 2) of them, split into gridDim.x contiguous ranges (stream-K): CTA c owns units
// [c*U/G, (c+1)*U/G).  Every unit is ~37 KB (Q4_K) / ~70 KB (Q8_0) of weights, so every CTA streams the same
// number of bytes whatever the matrix shape.
//
//  * Warp 16 is the producer: one lane keeps a ring of `stages` shared-memory slots (one unit each) full with
//    cp.async.bulk copies (no multicast) of the unit's weights, activation fragments and sub-block sums,
//    completing on the slot's "full" mbarrier.  The first `stages` weight copies are issued before
//    griddepcontrol.wait (weights are immutable), so under programmatic dependent launch they stream in while the
//    previous kernel finishes.
//  * Warps 0..15 consume in two groups of eight: group w / 8 takes the units at even / odd positions of the CTA's
//    range, warp w the row tile w % 8 of both superblocks of each.  A warp dequantises its tiles in registers
//    (gemv_tile.cuh), issues m16n8k16 tensor-core products against the staged fragments (even and odd k-steps on
//    separate accumulators, one min / bias mma pair per unit) and releases the slot ("empty" mbarrier, one
//    arrival per warp of the group).  The two groups run half a
//    unit apart, so their dequantisation bursts interleave and a slot is refilled as soon as its group is done.
//    The groups fold their accumulators through shared memory when the CTA flushes a row group.
//  * When a CTA's range leaves a row group it flushes the group: a group owned by one CTA goes straight to the
//    epilogue; otherwise the later segments publish their partials (release-add on the group's counter) and move
//    on, and the group's first segment, which reaches the group at the end of its range, waits for them (bounded
//    acquire spin), sums the segments in index order (deterministic) and runs the epilogue.
//  * Every mbarrier wait is bounded (bulk.cuh); a timeout raises the epilogue's error flag.
#include <cstdlib>

#include "gemv_core.cuh"
#include "pdl.cuh"

namespace clm {

template <typename Raw, int NT, int EPI>
__global__ void __launch_bounds__(kG4Threads, 1) gemv4_kernel(const uint8_t* __restrict__ tiles, uint32_t rows,
                                                             int ng, G4Geom geo, int stages, XBuf in, int q, Epi epi,
                                                             float* __restrict__ part, int* __restrict__ counters,
                                                             int maxseg, int ahead) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kG4MaxStages], empty[kG4MaxStages];
  __shared__ float s_scale[kSsRows];
  __shared__ float s_red[kG4Consumers];
  __shared__ int s_last;
  float* y = reinterpret_cast<float*>(smem + (size_t)stages * geo.stage_bytes);  // [16][128]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool linked = epi.wait != nullptr;
  const long long U = (long long)ng * geo.ppr;
  const int G = gridDim.x;
  const long long u0 = (long long)blockIdx.x * U / G, u1 = (long long)(blockIdx.x + 1) * U / G;
  const int n = (int)(u1 - u0);
  UnitCursor start;
  start.grp = (int)(u0 / geo.ppr);
  start.pr = (int)(u0 - (long long)start.grp * geo.ppr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvWarps);  // the eight warps of the group that consumes the slot's unit
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kG4Consumers / 32) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t policy = evict_first_policy();
      auto issue_weights = [&](const UnitCursor& c) {
        const int nsb = min(geo.usb, geo.sb - geo.usb * c.pr);
        uint8_t* st = smem + (size_t)c.slot * geo.stage_bytes;
        const uint32_t wb = (uint32_t)(nsb * geo.sb_bytes);
        const uint32_t ab = (uint32_t)(nsb * NT * kXfragSbBytes + nsb * 512 * sum_tiles(NT));
        mbar_expect_tx(&full[c.slot], wb + ab);
        bulk_g2s_stream(st, tiles + ((size_t)c.grp * geo.sb + geo.usb * c.pr) * geo.sb_bytes, wb, &full[c.slot], policy);
      };
      auto issue_acts = [&](const UnitCursor& c) {
        const int nsb = min(geo.usb, geo.sb - geo.usb * c.pr);
        uint8_t* st = smem + (size_t)c.slot * geo.stage_bytes;
        bulk_g2s(st + geo.frag_off, in.frag + (size_t)geo.usb * c.pr * NT * 512, (uint32_t)(nsb * NT * kXfragSbBytes),
                 &full[c.slot]);
        bulk_g2s(st + geo.sum_off, reinterpret_cast<const uint8_t*>(in.sum) + (size_t)geo.usb * c.pr * 512 * sum_tiles(NT),
                 (uint32_t)(nsb * 512 * sum_tiles(NT)), &full[c.slot]);
      };
      // dataflow: a unit's activation copies wait for its input chunk (a failed wait drops them from the stage's
      // barrier instead, so the consumers never wait for copies that will not come; the error flag is raised)
      auto acts_when_ready = [&](const UnitCursor& c) {
        if (linked) {
          if (!dep_wait(epi.wait + c.pr, epi.wait_target, epi.err)) {
            const int nsb = min(geo.usb, geo.sb - geo.usb * c.pr);
            mbar_complete_tx(&full[c.slot], (uint32_t)(nsb * NT * kXfragSbBytes + nsb * 512 * sum_tiles(NT)));
            return;
          }
          fence_proxy_async_global();  // the copies read what other CTAs' epilogues stored
        }
        issue_acts(c);
      };
      // L2 lookahead cursor: unit i + `ahead` is prefetched into L2 when unit i's copies are issued, so the ring's
      // copies find their bytes in L2 and the DRAM stream keeps more bytes in flight than the ring can hold
      UnitCursor l2 = start;
      int l2i = 0;
      auto l2_until = [&](int upto) {
        for (; l2i < n && l2i < upto; ++l2i, l2.next(geo.ppr, stages)) {
          const int nsb = min(geo.usb, geo.sb - geo.usb * l2.pr);
          const unsigned long long bytes = (unsigned long long)nsb * geo.sb_bytes;
          l2_prefetch_share(tiles + ((size_t)l2.grp * geo.sb + geo.usb * l2.pr) * geo.sb_bytes, bytes, 0, 1, bytes);
        }
      };
      const int pre = min(n, stages);
      l2i = pre;
      for (int i = 0; i < pre; ++i) l2.next(geo.ppr, stages);
      l2_until(pre + ahead);
      UnitCursor w = start, a = start;
      for (int i = 0; i < pre; ++i, w.next(geo.ppr, stages)) issue_weights(w);
      if (!linked) griddep_wait();
      griddep_launch();
      for (int i = 0; i < pre; ++i, a.next(geo.ppr, stages)) acts_when_ready(a);
      for (int i = pre; i < n; ++i, w.next(geo.ppr, stages)) {
        // the slot's previous use is consumed (sleeping between polls leaves the issue slots to the consumers)
        if (!mbar_wait_backoff(&empty[w.slot], w.phase ^ 1u, epi.err, 128)) break;
        issue_weights(w);
        acts_when_ready(w);
        if (ahead > 0) l2_until(i + 1 + ahead);  // (at 0 the cursor would prefetch the unit just issued)
      }
      // every copy of this CTA is issued: prefetch the next kernel's first bytes into L2 while this one drains
      if (EPI == EPI_ROPE_KV && epi.pf_kv) {
        const long long vis = *epi.pos + q;
        const long long npl = (vis + 63) / 64;
        const int np = (int)(npl < epi.pf_max_pages ? npl : epi.pf_max_pages);
        const size_t page_bytes = (size_t)epi.nkv * 64 * epi.hd * sizeof(__half);  // all kv heads of one page
        for (int item = blockIdx.x; item < 2 * np; item += G) {
          const __half* pool = (item & 1) ? epi.vpool : epi.kpool;
          const uint8_t* src = reinterpret_cast<const uint8_t*>(pool) + (size_t)epi.pages[item >> 1] * page_bytes;
          l2_prefetch_share(src, page_bytes, 0, 1, page_bytes);
        }
      } else {
        l2_prefetch_share(epi.pf, epi.pf_bytes, blockIdx.x, G, epi.pf_cap);
      }
    }
    griddep_launch();
    return;
  }

  // ---------------- consumers ----------------
  // linked: nothing this launch reads from its predecessor is touched before the unit data has arrived (the
  // producer waited for it), the row scale's partials are read after their own wait, and the epilogue's operands
  // are loaded by a group's first segment while it waits for the other segments, not at the group's start
  if (!linked) {
    griddep_wait();
    griddep_launch();
  }
  const int grp_of_warp = warp / kGemvWarps, rt = warp % kGemvWarps;
  const G4SsPre ss_pre = linked ? G4SsPre{} : g4_ss_load(in);
  bool scale_ready = false;
  G4Acc<NT> acc;
  acc.zero();
  int cur = n > 0 ? start.grp : -1;
  EpiPre pre;
  // 32-row launches keep no operands across the units (their accumulators already fill the register budget)
  const bool preload = !linked && NT < 4;
  const EpiPre* prep = preload ? &pre : nullptr;
  EpiPre* lazy = linked && NT < 4 ? &pre : nullptr;
  constexpr int kQm = NT >= 4 ? 32 : 16;
  if (cur >= 0 && preload) epi_preload<EPI, kQm>(pre, cur, rows, q, epi);
  UnitCursor c = start;
  // both groups walk every unit of the range, so they flush the same row groups at the same points
  for (int i = 0; i < n; ++i, c.next(geo.ppr, stages)) {
    if (c.grp != cur) {
      g4_flush<NT>(cur, acc, y, part, counters, maxseg, U, G, u0, geo.ppr, q, rows, EPI, epi, s_scale, &s_last, ss_pre,
                   in, scale_ready, s_red, prep, lazy);
      cur = c.grp;
      if (preload) epi_preload<EPI, kQm>(pre, cur, rows, q, epi);
      acc.zero();
    }
    if ((i & 1) != grp_of_warp) continue;
    mbar_wait(&full[c.slot], c.phase, epi.err);
    g4_consume_pair<Raw, NT>(smem + (size_t)c.slot * geo.stage_bytes, geo, min(geo.usb, geo.sb - geo.usb * c.pr), rt, lane, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[c.slot]);
  }
  if (cur >= 0) g4_flush<NT>(cur, acc, y, part, counters, maxseg, U, G, u0, geo.ppr, q, rows, EPI, epi, s_scale, &s_last, ss_pre,
                   in, scale_ready, s_red, prep, lazy);
}

// x[p][0:cols] (row stride ld) * w -> fragments / sums (+ sum-of-squares partials per 128 columns); one warp per
// (128-column group, row).  The partial is summed in the order of the residual epilogue (gemv_core.cuh: lane l
// adds columns l, l+32, l+64, l+96, then a butterfly over the warp), so a stage that starts from boundary records
// scales its first layer bit-identically to the same layer inside a whole-model engine.
__global__ void prep_rows_kernel(const float* __restrict__ x, long long ld, int q, int cols,
                                 const float* __restrict__ w, int nt, float hi_scale, uint2* __restrict__ frag,
                                 float* __restrict__ sum, float* __restrict__ ss) {
  griddep_wait();
  griddep_launch();
  const int groups = cols / 128;
  const int wid = (int)((blockIdx.x * blockDim.x + threadIdx.x) / 32), ln = threadIdx.x % 32;
  if (wid >= groups * 8 * nt) return;
  const int c = wid % groups, p = wid / groups;
  if (ln < 8) {
    const int col0 = 128 * c + 16 * ln;
    float vals[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float raw = p < q ? x[(size_t)p * ld + col0 + k] : 0.0f;
      vals[k] = w ? raw * w[col0 + k] : raw;
    }
    prep16(vals, nullptr, p, q, col0 / 16, nt, hi_scale, frag, sum, nullptr, cols);
  }
  float a = 0.0f;
  if (p < q) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float v = x[(size_t)p * ld + 128 * c + ln + 32 * k];
      a += v * v;
    }
  }
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  if (ss && ln == 0 && p < kSsRows) ss[(size_t)c * kSsRows + p] = a;
}

int launch_prep_rows(const float* d_x, long long ld, int q, int cols, const float* d_w, int nt, float hi_scale,
                     const XBuf& out, bool with_ss, cudaStream_t st) {
  CLM_CHECK(cols % 128 == 0, CLM_INTERNAL, "prep_rows needs a multiple of 128 columns");
  const int warps = cols / 128 * 8 * nt;
  return launch_pdl(prep_rows_kernel, dim3((warps + 3) / 4), dim3(128), 0, st, d_x, ld, q, cols, d_w, nt, hi_scale,
                    out.frag, out.sum, with_ss ? out.ss : nullptr);
}

// Units of L2 lookahead beyond the ring (CLM_B200_L2AHEAD, default kL2Ahead).
int gemv_l2_ahead() {
  static const int v = [] {
    const char* e = getenv("CLM_B200_L2AHEAD");
    return e ? atoi(e) : kL2Ahead;
  }();
  return v;
}

template <typename Raw, int NT, int EPI>
static int launch4(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q,
                   const Epi& epi, float* part, int* counters, cudaStream_t st) {
  auto kern = gemv4_kernel<Raw, NT, EPI>;
  CLM_TRY(ensure_smem(kern, p.smem));
  const G4Geom geo = g4_geom(s, NT, gemv_unit_sb(NT));
  return launch_pdl(kern, dim3((unsigned)p.grid), dim3(kG4Threads), p.smem, st, d_tiles, s.rows, (int)s.ng, geo,
                    p.stages, in, q, epi, part, counters, p.ksplit, gemv_l2_ahead());
}

template <typename Raw, int NT>
static int launch4_epi(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q,
                       const Epi& epi, float* part, int* counters, cudaStream_t st) {
  switch (epi.kind) {
    case EPI_STORE: return launch4<Raw, NT, EPI_STORE>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_RESID_PREP: return launch4<Raw, NT, EPI_RESID_PREP>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_ROPE_KV: return launch4<Raw, NT, EPI_ROPE_KV>(s, p, d_tiles, in, q, epi, part, counters, st);
    case EPI_SWIGLU_PREP: return launch4<Raw, NT, EPI_SWIGLU_PREP>(s, p, d_tiles, in, q, epi, part, counters, st);
  }
  return fail(CLM_INTERNAL, "unknown GEMV epilogue");
}

int launch_gemv(const GemvShape& s, const GemvPlan& p, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi,
                float* part, int* counters, cudaStream_t st) {
  CLM_CHECK(q >= 1 && q <= 8 * p.nt, CLM_INTERNAL, "GEMV plan does not cover the window width");
  if (s.quant == CLM_QUANT_Q4_K) {
    if (p.nt == 1) return launch4_epi<RawQ4k, 1>(s, p, d_tiles, in, q, epi, part, counters, st);
    if (p.nt == 2) return launch4_epi<RawQ4k, 2>(s, p, d_tiles, in, q, epi, part, counters, st);
    return launch4_epi<RawQ4k, 4>(s, p, d_tiles, in, q, epi, part, counters, st);
  }
  if (p.nt == 1) return launch4_epi<RawQ80, 1>(s, p, d_tiles, in, q, epi, part, counters, st);
  if (p.nt == 2) return launch4_epi<RawQ80, 2>(s, p, d_tiles, in, q, epi, part, counters, st);
  return launch4_epi<RawQ80, 4>(s, p, d_tiles, in, q, epi, part, counters, st);
}

}  // namespace clm
