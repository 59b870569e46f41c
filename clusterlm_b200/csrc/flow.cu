// flow.cu — the verify-window dataflow kernel (see flow.cuh for the phase sequence and the readiness counters).
//
// Persistent cooperative grid: one CTA per SM, 16 consumer warps + 1 producer warp (the layout of gemv4.cu).
//  * The producer lane walks the (phase, unit) sequence of its CTA with two cursors.  The first requests the
//    immutable part of a unit as soon as a ring slot is free: a GEMV unit's weights, or a KV page that holds only
//    committed positions.  The second follows it and requests what earlier phases produce (the unit's activation
//    fragments and sums, or the KV page that holds the window's own rows) once the unit's readiness counter says
//    it is complete.  Weight streaming therefore runs ahead across phase and layer boundaries as far as the ring
//    allows.
//  * GEMV phases are the stream-K GEMV of gemv_core.cuh (all 16 warps on one unit: row tile w % 8, superblock w / 8).
//    Attention phases stream-K over (m-tile, kv head, page) units: warps 0-7 compute S = Q K^T for 8 positions
//    each, every warp owns one row of the online softmax, and each warp accumulates 8 head dims of O = P V across
//    the CTA's pages of a head; a head split over several CTAs is combined by the last CTA to arrive (counter).
//  * A finished group (a GEMV row group's epilogue, an attention head's output fragments) is announced with one
//    release-add on the next phase's readiness counter; data other CTAs wrote is read with L1-bypassing loads or
//    bulk copies after an acquire and an async-proxy fence.
//  * Every wait is bounded (polls and %globaltimer).  The first one that gives up raises the error flag; from then
//    on every readiness and ring wait of every CTA returns at once, the producer balances the transaction bytes it
//    will no longer copy (mbarrier.complete_tx), and the consumers drain the ring without computing, so the kernel
//    ends promptly.  Every branch that skips work is taken by all consumer threads of a CTA alike (the flags it
//    tests are shared through shared memory), so no CTA barrier is ever left waiting.
#include "flow.cuh"
#include "pdl.cuh"

namespace clm {

namespace {

constexpr int kHd = 128;
constexpr int kRW = kFlowAttnRowFloats;
constexpr uint32_t kPageBytes = 64u * kHd * 2u;  // one K or V^T page of one kv head (16 KB)
constexpr int kMaxAttnSeg = 64;                  // attention segments per head combined in shared memory
// fixed shared memory after the ring: y / o [16][128] f32, S [16][64] f32, P [16][64] fp16, m/l/alpha [3][16],
// combine weights and sums [2][kMaxAttnSeg][16]
constexpr size_t kFixedBytes = 16 * 128 * 4 + 16 * 64 * 4 + 16 * 64 * 2 + 3 * 16 * 4 + 2 * kMaxAttnSeg * 16 * 4;


__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// One potentially blocking test of a barrier phase (mbarrier.try_wait: the thread may be suspended until the phase
// completes or a hardware time limit passes); true if the phase completed.
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// mbarrier wait of a consumer: bounded, and returns false at once once the error flag is raised.
__device__ bool flow_mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t a = smem_addr(bar);
  unsigned long long t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 255) {
      if (dep_failed(err)) return false;
      if (t0 == 0) {
        t0 = globaltimer();
      } else if (globaltimer() - t0 > kDepWaitNs) {
        dep_raise(err);
        return false;
      }
    }
  }
}

// Arrival with a count (a warp that stands for several of the barrier's expected arrivals).
__device__ __forceinline__ void mbar_arrive_n(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}


__device__ __forceinline__ uint32_t word_of4(const uint4 (&v)[4], int w) {
  const uint4& u = v[w / 4];
  return (w % 4 == 0) ? u.x : (w % 4 == 1) ? u.y : (w % 4 == 2) ? u.z : u.w;
}


// Units and this CTA's range of a phase.
struct PhaseRange {
  long long U = 0, u0 = 0;
  int n = 0;
  int per = 1;  // units per group (superblock pairs of a row group, or pages of a head)
};

__device__ __forceinline__ PhaseRange phase_range(const FlowPhase& ph, int npages) {
  PhaseRange r;
  if (ph.kind == FLOW_GEMV) {
    r.per = ph.g.geo.ppr;
    r.U = (long long)ph.g.ng * r.per;
  } else {
    r.per = npages;
    r.U = (long long)ph.a.mtiles * ph.a.nkv * npages;
  }
  const int G = gridDim.x;
  r.u0 = (long long)blockIdx.x * r.U / G;
  r.n = (int)((long long)(blockIdx.x + 1) * r.U / G - r.u0);
  return r;
}

// A position in the CTA's (phase, unit) sequence and its ring slot.
struct Cursor {
  int p = 0;       // phase
  int i = 0;       // unit of the phase's range
  int grp = 0, pr = 0;
  int slot = 0;
  uint32_t parity = 0;
  PhaseRange R;
  int rp = -1;  // phase whose range R holds
  __device__ __forceinline__ void settle(const FlowParams& P, int npages) {
    // skip phases in which this CTA owns no unit (the range is computed once per phase)
    while (p < P.nphases) {
      if (rp != p) {
        R = phase_range(P.phases[p], npages);
        rp = p;
      }
      if (i < R.n) break;
      ++p;
      i = 0;
    }
    if (p < P.nphases && i == 0) {
      grp = (int)(R.u0 / R.per);
      pr = (int)(R.u0 - (long long)grp * R.per);
    }
  }
  __device__ __forceinline__ void next(const FlowParams& P, int npages) {
    if (++slot == P.stages) {
      slot = 0;
      parity ^= 1u;
    }
    if (++pr == R.per) {
      pr = 0;
      ++grp;
    }
    if (++i == R.n) {
      ++p;
      i = 0;
    }
    settle(P, npages);
  }
  __device__ __forceinline__ bool done(const FlowParams& P) const { return p >= P.nphases; }
};

}  // namespace

size_t flow_smem_bytes(int stages, int stage_bytes) { return (size_t)stages * stage_bytes + kFixedBytes; }

int flow_stages(int stage_bytes) {
  int s = kG4MaxStages;
  while (s > 2 && flow_smem_bytes(s, stage_bytes) > 224 * 1024) --s;
  return flow_smem_bytes(s, stage_bytes) <= 224 * 1024 ? s : 0;
}

template <typename Raw, int NT>
__global__ void __launch_bounds__(kG4Threads, 1) flow_kernel(FlowParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kG4MaxStages], empty[kG4MaxStages];
  __shared__ float s_scale[kSsRows];
  __shared__ float s_red[kG4Consumers];
  __shared__ int s_last, s_ok;
  uint8_t* ring = smem;
  float* y = reinterpret_cast<float*>(smem + (size_t)P.stages * P.stage_bytes);  // [16][128]
  float* Ss = y + 16 * 128;                                                     // [16][64]
  __half* Ps = reinterpret_cast<__half*>(Ss + 16 * 64);                         // [16][64]
  float* m_run = reinterpret_cast<float*>(Ps + 16 * 64);                        // [16]
  float* l_run = m_run + 16;
  float* alpha = l_run + 16;
  float* cw = alpha + 16;             // [kMaxAttnSeg][16] combine weights
  float* cl = cw + kMaxAttnSeg * 16;  // [kMaxAttnSeg][16] segment sums

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int G = gridDim.x, q = P.q;
  int* err = P.err;
  if (tid == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kG4Consumers / 32);
    }
    mbar_fence_init();
  }
  __syncthreads();
  // the window base (committed position) is written only between windows
  const long long base = *P.pos;
  const int npages = (int)((base + q + 63) / 64);

  if (warp == kG4Consumers / 32) {
    // =============================== producer ===============================
    if (lane != 0) {
      griddep_wait();
      griddep_launch();
      return;
    }
    const uint64_t policy = evict_first_policy();
    auto committed = [&](int pr2) { return (long long)(pr2 + 1) * 64 <= base; };
    auto gemv_late_bytes = [&](const FlowGemv& m, int pr2) {
      const int nsb = min(2, m.geo.sb - 2 * pr2);
      return (uint32_t)(nsb * NT * kXfragSbBytes + nsb * 1024);
    };
    // the immutable part of a unit (and its barrier's whole transaction count)
    auto early = [&](const Cursor& c) {
      const FlowPhase& ph = P.phases[c.p];
      uint8_t* st = ring + (size_t)c.slot * P.stage_bytes;
      uint64_t* bar = &full[c.slot];
      if (ph.kind == FLOW_GEMV) {
        const FlowGemv& m = ph.g;
        const int nsb = min(2, m.geo.sb - 2 * c.pr);
        const uint32_t wb = (uint32_t)(nsb * m.geo.sb_bytes);
        mbar_expect_tx(bar, wb + gemv_late_bytes(m, c.pr));
        bulk_g2s_stream(st, m.tiles + ((size_t)c.grp * m.geo.sb + 2 * c.pr) * m.geo.sb_bytes, wb, bar, policy);
      } else {
        const FlowAttn& a = ph.a;
        mbar_expect_tx(bar, 2 * kPageBytes);
        if (committed(c.pr)) {
          const size_t off = ((size_t)a.pages[c.pr] * a.nkv + c.grp % a.nkv) * 64 * kHd;
          bulk_g2s(st, a.kpool + off, kPageBytes, bar);
          bulk_g2s(st + kPageBytes, a.vpool + off, kPageBytes, bar);
        }
      }
    };
    // whether the produced part of unit c is complete: a chunk (GEMV) or kv head (attention) seen complete once is
    // remembered for the rest of the phase, so the counter is acquired once per chunk, not once per unit; a newly
    // acquired counter asks for an async-proxy fence before the next copy
    uint64_t seen = 0;
    int seen_phase = -1;
    bool need_fence = false;
    auto late_ready = [&](const Cursor& c) {
      const FlowPhase& ph = P.phases[c.p];
      if (ph.wait == nullptr) return true;
      if (ph.kind != FLOW_GEMV && committed(c.pr)) return true;
      if (seen_phase != c.p) {
        seen = 0;
        seen_phase = c.p;
      }
      const int chunk = ph.kind == FLOW_GEMV ? c.pr : c.grp % ph.a.nkv;
      if (chunk < 64 && ((seen >> chunk) & 1ull)) return true;
      if (ld_acquire(ph.wait + chunk) < ph.wait_target) return false;
      if (chunk < 64) seen |= 1ull << chunk;
      need_fence = true;
      return true;
    };
    auto late = [&](const Cursor& c) {
      const FlowPhase& ph = P.phases[c.p];
      uint8_t* st = ring + (size_t)c.slot * P.stage_bytes;
      uint64_t* bar = &full[c.slot];
      if (ph.kind == FLOW_GEMV) {
        const FlowGemv& m = ph.g;
        const int nsb = min(2, m.geo.sb - 2 * c.pr);
        bulk_g2s(st + m.geo.frag_off, m.in.frag + (size_t)2 * c.pr * NT * 512, (uint32_t)(nsb * NT * kXfragSbBytes),
                 bar);
        bulk_g2s(st + m.geo.sum_off, reinterpret_cast<const uint8_t*>(m.in.sum) + (size_t)2 * c.pr * 1024,
                 (uint32_t)(nsb * 1024), bar);
      } else if (!committed(c.pr)) {
        const FlowAttn& a = ph.a;
        const size_t off = ((size_t)a.pages[c.pr] * a.nkv + c.grp % a.nkv) * 64 * kHd;
        bulk_g2s(st, a.kpool + off, kPageBytes, bar);
        bulk_g2s(st + kPageBytes, a.vpool + off, kPageBytes, bar);
      }
    };
    // transaction bytes of unit c's late part (balanced with complete_tx when it will not be copied)
    auto late_bytes = [&](const Cursor& c) -> uint32_t {
      const FlowPhase& ph = P.phases[c.p];
      if (ph.kind == FLOW_GEMV) return gemv_late_bytes(ph.g, c.pr);
      return committed(c.pr) ? 0u : 2 * kPageBytes;
    };

    // L2 lookahead: the immutable parts of the next kLookahead units beyond the ring are prefetched into L2 (no
    // shared memory, nothing to wait for), so HBM keeps streaming weights while the ring waits on a dependency
    auto prefetch = [&](const Cursor& c) {
      const FlowPhase& ph = P.phases[c.p];
      if (ph.kind == FLOW_GEMV) {
        const FlowGemv& m = ph.g;
        const int nsb = min(2, m.geo.sb - 2 * c.pr);
        const uint8_t* src = m.tiles + ((size_t)c.grp * m.geo.sb + 2 * c.pr) * m.geo.sb_bytes;
        const uint32_t bytes = (uint32_t)(nsb * m.geo.sb_bytes);
        for (uint32_t o = 0; o < bytes; o += 32768u) bulk_prefetch_l2(src + o, min(32768u, bytes - o));
      } else if (committed(c.pr)) {
        const FlowAttn& a = ph.a;
        const size_t off = ((size_t)a.pages[c.pr] * a.nkv + c.grp % a.nkv) * 64 * kHd;
        bulk_prefetch_l2(a.kpool + off, kPageBytes);
        bulk_prefetch_l2(a.vpool + off, kPageBytes);
      }
    };
    constexpr long long kLookahead = 4;
    Cursor W, A, F;
    W.settle(P, npages);
    A.settle(P, npages);
    F.settle(P, npages);
    long long nw = 0, na = 0, nf = 0;  // units whose immutable / produced parts are requested, units prefetched
    // the first stages' weights stream in while the previous kernel finishes; the stage input (phase 0's
    // activations) and every write are ordered after griddepcontrol.wait
    while (!W.done(P) && nw < P.stages && (P.phases[W.p].kind == FLOW_GEMV || committed(W.pr))) {
      early(W);
      W.next(P, npages);
      ++nw;
    }
    while (nf < nw) {  // the lookahead cursor starts where the ring stops
      F.next(P, npages);
      ++nf;
    }
    griddep_wait();
    griddep_launch();
    bool ok = true;
    unsigned long long idle_since = 0;
    uint32_t idle = 0;  // consecutive turns without progress
    while (ok && !A.done(P)) {
      bool progress = false;
      if (!W.done(P) && mbar_test(&empty[W.slot], W.parity ^ 1u)) {
        early(W);
        W.next(P, npages);
        ++nw;
        progress = true;
      }
      if (na < nw && late_ready(A)) {
        if (need_fence) {
          fence_proxy_async_global();
          need_fence = false;
        }
        late(A);
        A.next(P, npages);
        ++na;
        progress = true;
      }
      if (nf < nw) {  // units the ring requested itself need no prefetch
        F = W;
        nf = nw;
      }
      if (!F.done(P) && nf < nw + kLookahead) {
        prefetch(F);
        F.next(P, npages);
        ++nf;
        progress = true;
      }
      if (progress) {
        idle = 0;
        continue;
      }
      // idle: with every produced part requested the only thing to wait for is a free ring slot, so the producer
      // blocks on that slot's barrier (mbarrier.try_wait suspends until the slot is released or a short hardware
      // limit); while a produced part is outstanding it polls its counter.  The error flag and the clock are read
      // every 64th idle turn only (each is a global-memory round trip).
      if (na == nw && !W.done(P)) {
        mbar_try(&empty[W.slot], W.parity ^ 1u);
      } else {
        __nanosleep(32);
      }
      if ((++idle & 63) == 0) {
        if (dep_failed(err)) {
          ok = false;
          break;
        }
        const unsigned long long now = globaltimer();
        if (idle_since == 0 || idle == 64) {
          idle_since = now;
        } else if (now - idle_since > kDepWaitNs) {
          dep_raise(err);
          ok = false;
          break;
        }
      }
    }
    if (!ok) {
      // requested immutable parts whose produced part will not come: balance their barriers so the copies already
      // in flight still complete them, and the consumers (which stop computing) drain the ring
      while (na < nw) {
        const uint32_t b = late_bytes(A);
        if (b) mbar_complete_tx(&full[A.slot], b);
        A.next(P, npages);
        ++na;
      }
    }
    return;
  }

  // =============================== consumers ===============================
  griddep_wait();
  griddep_launch();
  const int t = lane % 4, g = lane / 4;
  int rs_slot = 0;
  uint32_t rs_parity = 0;
  auto ring_next = [&]() {
    if (++rs_slot == P.stages) {
      rs_slot = 0;
      rs_parity ^= 1u;
    }
  };
  // one thread waits for a counter; the result is shared with the consumer threads
  auto cta_wait = [&](const int* ctr, int target) -> bool {
    if (tid == 0) s_ok = dep_wait(ctr, target, err);
    consumer_sync();
    const bool r = s_ok;
    consumer_sync();
    return r;
  };
  // announce a finished group: all its writes are ordered before the release by the consumer barrier
  auto signal = [&](int* ctr) {
    if (tid == 0 && ctr != nullptr) {
      __threadfence();
      red_release_add(ctr, 1);
    }
  };

  for (int p = 0; p < P.nphases; ++p) {
    const FlowPhase& ph = P.phases[p];
    const PhaseRange R = phase_range(ph, npages);
    if (R.n == 0) continue;
    int grp = (int)(R.u0 / R.per), pr = (int)(R.u0 - (long long)grp * R.per);

    if (ph.kind == FLOW_GEMV) {
      const FlowGemv& m = ph.g;
      bool scale_ready = false;
      G4Acc<NT> acc;
      acc.zero();
      int cur = grp;
      const int my_group = warp / kGemvWarps, rt = warp % kGemvWarps;
      auto flush = [&](int gi) {
        if (!scale_ready) {
          // the row scale needs every row group of the previous residual phase
          bool ok = true;
          if (ph.ss_done != nullptr) ok = cta_wait(ph.ss_done, ph.ss_target);
          const G4SsPre ss_pre = ok ? g4_ss_load(m.in) : G4SsPre{};
          g4_ss_finish(ss_pre, m.in, m.epi, q, s_red, s_scale);
          scale_ready = true;
        }
        // the residual epilogue's operands (residual rows, next norm weights): every unit of the group is consumed,
        // so the rows other CTAs wrote before this phase are final; their loads overlap the segment reduction
        EpiPre pre;
        const bool resid = m.epi_kind == EPI_RESID_PREP;
        if (resid) epi_preload<EPI_RESID_PREP>(pre, gi, m.rows, q, m.epi);
        const bool ran = g4_flush<NT>(gi, acc, y, m.part, m.counters, m.maxseg, R.U, G, R.u0, R.per, q, m.rows,
                                      m.epi_kind, m.epi, s_scale, &s_last, G4SsPre{}, m.in, scale_ready, s_red,
                                      resid ? &pre : nullptr);
        if (ran) {
          if (ph.sig != nullptr) {
            int c = gi / ph.sig_div;
            if (ph.sig_qkv) {
              const int nh = m.epi.nh, nkv = m.epi.nkv;
              c = gi < nh ? gi / (nh / nkv) : (gi < nh + nkv ? gi - nh : gi - nh - nkv);
            }
            signal(ph.sig + c);
          }
          signal(ph.done);
        }
      };
      for (int i = 0; i < R.n; ++i) {
        if (grp != cur) {
          flush(cur);
          cur = grp;
          acc.zero();
        }
        // the two groups of 8 warps take alternate units (warp: row tile rt of both superblocks), so their
        // dequantisation bursts interleave; each warp's release stands for two of the slot's 16 arrivals
        if ((i & 1) == my_group) {
          const int nsb = min(2, m.geo.sb - 2 * pr);
          if (flow_mbar_wait(&full[rs_slot], rs_parity, err))
            g4_consume_pair<Raw, NT>(ring + (size_t)rs_slot * P.stage_bytes, m.geo, nsb, rt, lane, acc);
          __syncwarp();
          if (lane == 0) mbar_arrive_n(&empty[rs_slot], 2);
        }
        ring_next();
        if (++pr == R.per) {
          pr = 0;
          ++grp;
        }
      }
      flush(cur);
      continue;
    }

    // ---------------- attention phase ----------------
    const FlowAttn& a = ph.a;
    const int group = a.nh / a.nkv;
    uint4 qw0[4], qw1[4];
    float O[4];
    int cur = -1;
    bool live = true;
    // start a (m-tile, kv head): wait for its heads' QKV rows, Q fragments (S warps) and empty running state
    auto begin_group = [&](int gi) {
      const int mt = gi / a.nkv, kvh = gi % a.nkv;
      live = ph.wait == nullptr || cta_wait(ph.wait + kvh, ph.wait_target);
      if (warp < 8) {
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        const int i0 = r0 / group, i1 = r1 / group;
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4* pa =
            reinterpret_cast<const uint4*>(a.q16 + ((size_t)i0 * a.nh + kvh * group + r0 % group) * kHd + 32 * t);
        const uint4* pb =
            reinterpret_cast<const uint4*>(a.q16 + ((size_t)i1 * a.nh + kvh * group + r1 % group) * kHd + 32 * t);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          qw0[j] = (live && i0 < q) ? __ldcg(pa + j) : z;
          qw1[j] = (live && i1 < q) ? __ldcg(pb + j) : z;
        }
      }
      O[0] = O[1] = O[2] = O[3] = 0.0f;
      if (tid < 16) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
      }
      consumer_sync();
    };
    // finish a (m-tile, kv head): single segment -> output, else publish and let the last CTA combine
    auto end_group = [&](int gi) {
      const int mt = gi / a.nkv, kvh = gi % a.nkv;
      int seg = 0, nseg = 1;
      group_segments((long long)gi * R.per, (long long)gi * R.per + R.per - 1, R.U, G, R.u0, &seg, &nseg);
      if (nseg > a.maxseg) {  // never write past the partial slots
        if (tid == 0) atomicExch(err, kErrPartialSlots);
        consumer_sync();
        return;
      }
      float* o_s = y;  // [16][128]
      const int d0 = 8 * warp + 2 * t;
      if (nseg == 1) {
        const float inv0 = l_run[g] > 0.0f ? 1.0f / l_run[g] : 0.0f;
        const float inv1 = l_run[g + 8] > 0.0f ? 1.0f / l_run[g + 8] : 0.0f;
        o_s[g * kHd + d0] = O[0] * inv0;
        o_s[g * kHd + d0 + 1] = O[1] * inv0;
        o_s[(g + 8) * kHd + d0] = O[2] * inv1;
        o_s[(g + 8) * kHd + d0 + 1] = O[3] * inv1;
        consumer_sync();
      } else {
        float* mine = a.part + ((size_t)gi * a.maxseg + seg) * 16 * kRW;
        mine[g * kRW + d0] = O[0];
        mine[g * kRW + d0 + 1] = O[1];
        mine[(g + 8) * kRW + d0] = O[2];
        mine[(g + 8) * kRW + d0 + 1] = O[3];
        if (tid < 16) {
          mine[tid * kRW + kHd] = m_run[tid];
          mine[tid * kRW + kHd + 1] = l_run[tid];
        }
        __threadfence();
        consumer_sync();
        if (tid == 0) s_last = atomicAdd(&a.counters[gi], 1) == nseg - 1;
        consumer_sync();
        if (!s_last) return;
        __threadfence();
        const float* allp = a.part + (size_t)gi * a.maxseg * 16 * kRW;
        for (int i = tid; i < nseg * 16; i += kG4Consumers) {
          cw[i] = __ldcg(allp + (size_t)i * kRW + kHd);
          cl[i] = __ldcg(allp + (size_t)i * kRW + kHd + 1);
        }
        consumer_sync();
        if (tid < 16) {
          float M = -INFINITY;
          for (int s = 0; s < nseg; ++s) M = fmaxf(M, cw[s * 16 + tid]);
          float L = 0.0f;
          for (int s = 0; s < nseg; ++s) {
            const float mm = cw[s * 16 + tid];
            const float e = mm == -INFINITY ? 0.0f : exp2f(mm - M);
            L += cl[s * 16 + tid] * e;
            cw[s * 16 + tid] = e;
          }
          const float inv = L > 0.0f ? 1.0f / L : 0.0f;
          for (int s = 0; s < nseg; ++s) cw[s * 16 + tid] *= inv;
        }
        consumer_sync();
        {  // thread -> (row r, 4 columns); eight partials' loads in flight at a time, summed in segment order
          const int r = tid / 32, c4 = (tid % 32) * 4;
          float acc4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          const float4* src = reinterpret_cast<const float4*>(allp + (size_t)r * kRW + c4);
          const size_t seg_stride = (size_t)16 * kRW / 4;  // float4 units between segments
          for (int s0 = 0; s0 < nseg; s0 += 8) {
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = s0 + k < nseg ? __ldcg(src + (s0 + k) * seg_stride) : make_float4(0, 0, 0, 0);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              if (s0 + k >= nseg) break;
              const float w = cw[(s0 + k) * 16 + r];
              acc4[0] += v[k].x * w;
              acc4[1] += v[k].y * w;
              acc4[2] += v[k].z * w;
              acc4[3] += v[k].w * w;
            }
          }
          o_s[r * kHd + c4] = acc4[0];
          o_s[r * kHd + c4 + 1] = acc4[1];
          o_s[r * kHd + c4 + 2] = acc4[2];
          o_s[r * kHd + c4 + 3] = acc4[3];
        }
        if (tid == 0) a.counters[gi] = 0;
        consumer_sync();
      }
      // W_o input fragments of the 16 rows (query i = row / group, head kvh * group + row % group)
      const int qd = a.nh * kHd;
      if (tid < 16 * (kHd / 16)) {
        const int r = tid / (kHd / 16), gg = tid % (kHd / 16);
        const int i = (mt * 16 + r) / group, head = kvh * group + (mt * 16 + r) % group;
        if (i < q)
          prep16(&o_s[r * kHd + 16 * gg], nullptr, i, q, (head * kHd + 16 * gg) / 16, a.nt_out, a.hi_scale, a.out.frag,
                 a.out.sum, nullptr, qd);
      }
      consumer_sync();
      if (ph.sig != nullptr) {
        if (ph.sig_span > 1) {
          for (int c = 0; c < ph.sig_span; ++c) signal(ph.sig + kvh * ph.sig_span + c);
        } else {
          signal(ph.sig + kvh / ph.sig_kvh_div);
        }
      }
    };

    for (int i = 0; i < R.n; ++i) {
      if (grp != cur) {
        if (cur >= 0) end_group(cur);
        cur = grp;
        begin_group(grp);
      }
      const int mt = grp / a.nkv;
      const bool committed_page = (long long)(pr + 1) * 64 <= base;
      const bool have = flow_mbar_wait(&full[rs_slot], rs_parity, err) && live;
      const __half* ks = reinterpret_cast<const __half*>(ring + (size_t)rs_slot * P.stage_bytes);
      const __half* vs = ks + 64 * kHd;
      // S = Q K^T: warp j < 8 owns positions {16c + 2j + e}; row r of Ss = m-tile row, column = position
      if (warp < 8) {
        const int j = warp;
        float S[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int pos = 16 * (g / 2) + 2 * j + (g % 2);
        if (have) {
          const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)pos * kHd);
          uint4 kw[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) kw[u] = kr[kv_k_chunk(4 * t + u, pos)];
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma16816(S, word_of4(qw0, 2 * kk), word_of4(qw1, 2 * kk), word_of4(qw0, 2 * kk + 1),
                     word_of4(qw1, 2 * kk + 1), word_of4(kw, 2 * kk), word_of4(kw, 2 * kk + 1));
        }
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        const int i0 = r0 / group, i1 = r1 / group;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = 16 * t + 2 * j + e;
          const long long ap = (long long)pr * 64 + col;
          const bool vis0 = have && i0 < q && (committed_page || ap - base <= i0);
          const bool vis1 = have && i1 < q && (committed_page || ap - base <= i1);
          Ss[g * 64 + col] = vis0 ? S[e] * a.scale_log2 : -INFINITY;
          Ss[(g + 8) * 64 + col] = vis1 ? S[2 + e] * a.scale_log2 : -INFINITY;
        }
      }
      consumer_sync();
      // online softmax: warp r owns row r, lanes own positions 2*lane, 2*lane+1
      {
        const int r = warp;
        const float s0 = Ss[r * 64 + 2 * lane], s1 = Ss[r * 64 + 2 * lane + 1];
        float mx = fmaxf(s0, s1);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float m_old = m_run[r];
        const float m_new = fmaxf(m_old, mx);
        const float p0 = m_new == -INFINITY || s0 == -INFINITY ? 0.0f : exp2f(s0 - m_new);
        const float p1 = m_new == -INFINITY || s1 == -INFINITY ? 0.0f : exp2f(s1 - m_new);
        float ls = p0 + p1;
        for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        const float al = m_old == -INFINITY ? 0.0f : exp2f(m_old - m_new);
        reinterpret_cast<__half2*>(Ps)[(r * 64 + 2 * lane) / 2] = __floats2half2_rn(p0, p1);
        __syncwarp();
        if (lane == 0) {
          l_run[r] = l_run[r] * al + ls;
          m_run[r] = m_new;
          alpha[r] = al;
        }
      }
      consumer_sync();
      // O = alpha * O + P V: warp w owns head dims [8w, 8w+8)
      {
        const float al0 = alpha[g], al1 = alpha[g + 8];
        O[0] *= al0;
        O[1] *= al0;
        O[2] *= al1;
        O[3] *= al1;
        if (have) {
          const int dim = 8 * warp + g;
          const __half* vrow = vs + (size_t)dim * 64;
          const uint32_t* P32 = reinterpret_cast<const uint32_t*>(Ps);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int k0 = 16 * kk + 2 * t;
            const uint32_t a0 = P32[(g * 64 + k0) / 2], a1 = P32[((g + 8) * 64 + k0) / 2];
            const uint32_t a2 = P32[(g * 64 + k0 + 8) / 2], a3 = P32[((g + 8) * 64 + k0 + 8) / 2];
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(vrow + 8 * kv_v_chunk(k0 >> 3, dim) + (k0 & 7));
            const uint32_t b1 =
                *reinterpret_cast<const uint32_t*>(vrow + 8 * kv_v_chunk((k0 + 8) >> 3, dim) + ((k0 + 8) & 7));
            mma16816(O, a0, a1, a2, a3, b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[rs_slot]);
      ring_next();
      if (++pr == R.per) {
        pr = 0;
        ++grp;
      }
    }
    if (cur >= 0) end_group(cur);
  }
}

namespace {

template <typename Raw, int NT>
int launch_t(const FlowParams& p, int grid, int* d_ctr, size_t ctr_bytes, cudaStream_t st) {
  auto kern = flow_kernel<Raw, NT>;
  const size_t smem = flow_smem_bytes(p.stages, p.stage_bytes);
  CLM_TRY(ensure_smem(kern, smem));
  if (ctr_bytes) CLM_CUDA(cudaMemsetAsync(d_ctr, 0, ctr_bytes, st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kG4Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CLM_CUDA(cudaLaunchKernelEx(&cfg, kern, p));
  ++t_kernel_launches;
  return CLM_OK;
}

template <typename Raw, int NT>
int grid_t(int device, int stages, int stage_bytes) {
  auto kern = flow_kernel<Raw, NT>;
  const size_t smem = flow_smem_bytes(stages, stage_bytes);
  if (ensure_smem(kern, smem) != CLM_OK) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kG4Threads, smem) != cudaSuccess) return 0;
  int sms = 0, coop = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return 0;
  return per_sm >= 1 ? sms : 0;  // one CTA per SM
}

}  // namespace

int flow_grid(int device, int stages, int stage_bytes, int quant, int nt) {
  if (quant == CLM_QUANT_Q4_K)
    return nt == 1 ? grid_t<RawQ4k, 1>(device, stages, stage_bytes) : grid_t<RawQ4k, 2>(device, stages, stage_bytes);
  return nt == 1 ? grid_t<RawQ80, 1>(device, stages, stage_bytes) : grid_t<RawQ80, 2>(device, stages, stage_bytes);
}

int launch_flow(const FlowParams& p, int quant, int nt, int grid, int* d_ctr, size_t ctr_bytes, cudaStream_t st) {
  CLM_CHECK(grid > 0 && p.stages >= 2, CLM_INTERNAL, "flow kernel not configured");
  if (quant == CLM_QUANT_Q4_K)
    return nt == 1 ? launch_t<RawQ4k, 1>(p, grid, d_ctr, ctr_bytes, st) : launch_t<RawQ4k, 2>(p, grid, d_ctr, ctr_bytes, st);
  return nt == 1 ? launch_t<RawQ80, 1>(p, grid, d_ctr, ctr_bytes, st) : launch_t<RawQ80, 2>(p, grid, d_ctr, ctr_bytes, st);
}

}  // namespace clm
