// window.cu — the verify-window megakernel (see window.cuh for the phase sequence).
//
// Persistent cooperative grid: one CTA per SM, 16 consumer warps + 1 producer warp (the layout of gemv4.cu).
//  * The producer lane walks the same (phase, unit) sequence as the consumers and keeps the shared-memory ring
//    full.  For every phase it first requests the weights of the phase's first `stages` units (and the KV pages
//    that hold only committed positions, which no phase of this window writes), then waits for the grid barrier
//    that ends the previous phase before requesting anything the previous phase produced (activation fragments,
//    sums, the KV page that holds the window's own positions).
//  * GEMV phases are the stream-K GEMV of gemv_core.cuh.  Attention phases stream-K over (m-tile, kv head, page)
//    units: warps 0-7 compute S = Q K^T for 8 positions each, every warp owns one row of the online softmax, and
//    each warp accumulates 8 head dims of O = P V across the CTA's pages of a head; a head split over several CTAs
//    is combined by the last CTA to finish (counter), which writes W_o's input fragments.
//  * Grid barrier: one arrival per CTA on a counter zeroed before the launch; barrier k completes at k * grid
//    arrivals.  Every wait (barrier, mbarrier) is bounded and raises the error flag when it gives up.
#include "pdl.cuh"
#include "window.cuh"

namespace clm {

namespace {

constexpr int kHd = 128;
constexpr int kRW = kMkAttnRowFloats;  // O[128], m, l, padding: rows stay 16-byte aligned for the float4 reads
constexpr uint32_t kPageBytes = 64u * kHd * 2u;     // one K or V^T page of one kv head (16 KB)
constexpr int kMaxAttnSeg = 64;                     // attention segments per head combined in shared memory
constexpr uint32_t kBarrierSpin = 1u << 24;         // grid-barrier polls (each sleeps ~64 ns)
// fixed shared memory after the ring: y / o [16][128] f32, S [16][64] f32, P [16][64] fp16, m/l/alpha [3][16],
// combine weights and sums [2][kMaxAttnSeg][16]
constexpr size_t kFixedBytes = 16 * 128 * 4 + 16 * 64 * 4 + 16 * 64 * 2 + 3 * 16 * 4 + 2 * kMaxAttnSeg * 16 * 4;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until the barrier counter reaches `target`; false (error flag raised) when it gives up.
__device__ bool grid_wait(const unsigned* bar, unsigned target, int* err) {
  for (uint32_t i = 0; i < kBarrierSpin; ++i) {
    if (ld_acquire_u32(bar) >= target) return true;
    __nanosleep(64);
  }
  if (err != nullptr) atomicExch(err, kErrWaitTimeout);
  return false;
}

__device__ __forceinline__ uint32_t word_of4(const uint4 (&v)[4], int w) {
  const uint4& u = v[w / 4];
  return (w % 4 == 0) ? u.x : (w % 4 == 1) ? u.y : (w % 4 == 2) ? u.z : u.w;
}

// Bulk copies issued after this read global memory written by other CTAs' ordinary stores.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

struct RingPos {
  int slot = 0;
  uint32_t parity = 0;
  __device__ __forceinline__ void next(int stages) {
    if (++slot == stages) {
      slot = 0;
      parity ^= 1u;
    }
  }
};

// Units and this CTA's range of a phase.
struct PhaseRange {
  long long U = 0, u0 = 0;
  int n = 0;
  int per = 1;  // units per group (superblock pairs of a row group, or pages of a head)
};

__device__ __forceinline__ PhaseRange phase_range(const MkPhase& ph, int npages) {
  PhaseRange r;
  if (ph.kind == MK_GEMV) {
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

}  // namespace

size_t mk_smem_bytes(int stages, int stage_bytes) { return (size_t)stages * stage_bytes + kFixedBytes; }

int mk_stages(int stage_bytes) {
  int s = kG4MaxStages;
  while (s > 2 && mk_smem_bytes(s, stage_bytes) > 224 * 1024) --s;
  return mk_smem_bytes(s, stage_bytes) <= 224 * 1024 ? s : 0;
}

template <typename Raw, int NT>
__global__ void __launch_bounds__(kG4Threads, 1) window_mk_kernel(MkParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kG4MaxStages], empty[kG4MaxStages];
  __shared__ float s_scale[16];
  __shared__ float s_red[kG4Consumers];
  __shared__ int s_last;
  uint8_t* ring = smem;
  float* y = reinterpret_cast<float*>(smem + (size_t)P.stages * P.stage_bytes);  // [16][128]
  float* Ss = y + 16 * 128;                                                     // [16][64]
  __half* Ps = reinterpret_cast<__half*>(Ss + 16 * 64);                         // [16][64]
  float* m_run = reinterpret_cast<float*>(Ps + 16 * 64);                        // [16]
  float* l_run = m_run + 16;
  float* alpha = l_run + 16;
  float* cw = alpha + 16;                 // [kMaxAttnSeg][16] combine weights
  float* cl = cw + kMaxAttnSeg * 16;      // [kMaxAttnSeg][16] segment sums

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int G = gridDim.x, q = P.q;
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
    RingPos rp;
    for (int p = 0; p < P.nphases; ++p) {
      const MkPhase& ph = P.phases[p];
      const PhaseRange R = phase_range(ph, npages);
      int grp = (int)(R.u0 / R.per), pr = (int)(R.u0 - (long long)grp * R.per);
      // what unit i needs: bytes, immutable copies (before the barrier), produced copies (after it)
      auto early = [&](int g2, int pr2, uint8_t* st, uint64_t* bar) {
        if (ph.kind == MK_GEMV) {
          const MkGemv& m = ph.g;
          const int nsb = min(2, m.geo.sb - 2 * pr2);
          const uint32_t wb = (uint32_t)(nsb * m.geo.sb_bytes);
          mbar_expect_tx(bar, wb + (uint32_t)(nsb * NT * kXfragSbBytes + 2 * nsb * 512));
          bulk_g2s_stream(st, m.tiles + ((size_t)g2 * m.geo.sb + 2 * pr2) * m.geo.sb_bytes, wb, bar, policy);
        } else {
          const MkAttn& a = ph.a;
          mbar_expect_tx(bar, 2 * kPageBytes);
          if ((long long)(pr2 + 1) * 64 <= base) {
            const int kvh = g2 % a.nkv;
            const size_t off = ((size_t)a.pages[pr2] * a.nkv + kvh) * 64 * kHd;
            bulk_g2s(st, a.kpool + off, kPageBytes, bar);
            bulk_g2s(st + kPageBytes, a.vpool + off, kPageBytes, bar);
          }
        }
      };
      auto late = [&](int g2, int pr2, uint8_t* st, uint64_t* bar) {
        if (ph.kind == MK_GEMV) {
          const MkGemv& m = ph.g;
          const int nsb = min(2, m.geo.sb - 2 * pr2);
          bulk_g2s(st + m.geo.frag_off, m.in.frag + (size_t)2 * pr2 * NT * 512, (uint32_t)(nsb * NT * kXfragSbBytes),
                   bar);
          bulk_g2s(st + m.geo.sum_off, reinterpret_cast<const uint8_t*>(m.in.sum) + (size_t)2 * pr2 * 1024,
                   (uint32_t)(nsb * 1024), bar);
        } else if ((long long)(pr2 + 1) * 64 > base) {
          const MkAttn& a = ph.a;
          const int kvh = g2 % a.nkv;
          const size_t off = ((size_t)a.pages[pr2] * a.nkv + kvh) * 64 * kHd;
          bulk_g2s(st, a.kpool + off, kPageBytes, bar);
          bulk_g2s(st + kPageBytes, a.vpool + off, kPageBytes, bar);
        }
      };
      auto step = [&](int& g2, int& pr2) {
        if (++pr2 == R.per) {
          pr2 = 0;
          ++g2;
        }
      };
      const int pre = min(R.n, P.stages);
      RingPos r0 = rp;
      int g0 = grp, pr0 = pr;
      for (int i = 0; i < pre; ++i) {
        // the slot's previous use has been consumed (a fresh barrier passes the parity-1 wait at once)
        mbar_wait(&empty[rp.slot], rp.parity ^ 1u, P.err);
        early(grp, pr, ring + (size_t)rp.slot * P.stage_bytes, &full[rp.slot]);
        step(grp, pr);
        rp.next(P.stages);
      }
      // everything this phase reads that the previous phase wrote is complete once its barrier has passed
      if (p == 0) {
        griddep_wait();
        griddep_launch();
      } else {
        grid_wait(P.barrier, (unsigned)p * G, P.err);
        fence_proxy_async_global();
      }
      for (int i = 0; i < pre; ++i) {
        late(g0, pr0, ring + (size_t)r0.slot * P.stage_bytes, &full[r0.slot]);
        step(g0, pr0);
        r0.next(P.stages);
      }
      for (int i = pre; i < R.n; ++i) {
        mbar_wait(&empty[rp.slot], rp.parity ^ 1u, P.err);
        uint8_t* st = ring + (size_t)rp.slot * P.stage_bytes;
        early(grp, pr, st, &full[rp.slot]);
        late(grp, pr, st, &full[rp.slot]);
        step(grp, pr);
        rp.next(P.stages);
      }
    }
    return;
  }

  // =============================== consumers ===============================
  griddep_wait();
  griddep_launch();
  const int t = lane % 4, g = lane / 4;
  RingPos rc;
  for (int p = 0; p < P.nphases; ++p) {
    if (p > 0) {
      // grid barrier: every CTA has finished phase p-1 (epilogues included)
      consumer_sync();
      if (tid == 0) {
        __threadfence();
        atomicAdd(P.barrier, 1u);
        grid_wait(P.barrier, (unsigned)p * G, P.err);
        __threadfence();
      }
      consumer_sync();
    }
    const MkPhase& ph = P.phases[p];
    const PhaseRange R = phase_range(ph, npages);
    int grp = (int)(R.u0 / R.per), pr = (int)(R.u0 - (long long)grp * R.per);

    if (ph.kind == MK_GEMV) {
      const MkGemv& m = ph.g;
      const G4SsPre ss_pre = g4_ss_load(m.in);
      bool scale_ready = false;
      G4Acc<NT> acc;
      acc.zero();
      int cur = R.n > 0 ? grp : -1;
      for (int i = 0; i < R.n; ++i) {
        if (grp != cur) {
          g4_flush<NT>(cur, acc, y, P.part, P.counters, m.maxseg, R.U, G, R.u0, R.per, q, m.rows, m.epi_kind, m.epi, s_scale,
                       &s_last, ss_pre, m.in, scale_ready, s_red);
          cur = grp;
          acc.zero();
        }
        const int nsb = min(2, m.geo.sb - 2 * pr);
        mbar_wait(&full[rc.slot], rc.parity, P.err);
        g4_consume_unit<Raw, NT>(ring + (size_t)rc.slot * P.stage_bytes, m.geo, nsb, warp, lane, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[rc.slot]);
        rc.next(P.stages);
        if (++pr == R.per) {
          pr = 0;
          ++grp;
        }
      }
      if (cur >= 0)
        g4_flush<NT>(cur, acc, y, P.part, P.counters, m.maxseg, R.U, G, R.u0, R.per, q, m.rows, m.epi_kind, m.epi, s_scale,
                     &s_last, ss_pre, m.in, scale_ready, s_red);
      continue;
    }

    // ---------------- attention phase ----------------
    const MkAttn& a = ph.a;
    const int group = a.nh / a.nkv;
    uint4 qw0[4], qw1[4];
    float O[4];
    int cur = -1;
    // start a (m-tile, kv head): Q fragments (S warps) and empty running state
    auto begin_group = [&](int gi) {
      const int mt = gi / a.nkv, kvh = gi % a.nkv;
      if (warp < 8) {
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        const int i0 = r0 / group, i1 = r1 / group;
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4* pa = reinterpret_cast<const uint4*>(a.q16 + ((size_t)i0 * a.nh + kvh * group + r0 % group) * kHd + 32 * t);
        const uint4* pb = reinterpret_cast<const uint4*>(a.q16 + ((size_t)i1 * a.nh + kvh * group + r1 % group) * kHd + 32 * t);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          qw0[j] = i0 < q ? pa[j] : z;
          qw1[j] = i1 < q ? pb[j] : z;
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
        if (tid == 0 && P.err) atomicExch(P.err, kErrPartialSlots);
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
        // thread -> (row r, 4 columns)
        {
          const int r = tid / 32, c4 = (tid % 32) * 4;
          float acc4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int s = 0; s < nseg; ++s) {
            const float w = cw[s * 16 + r];
            const float4 v = __ldcg(reinterpret_cast<const float4*>(allp + ((size_t)s * 16 + r) * kRW + c4));
            acc4[0] += v.x * w;
            acc4[1] += v.y * w;
            acc4[2] += v.z * w;
            acc4[3] += v.w * w;
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
    };

    for (int i = 0; i < R.n; ++i) {
      if (grp != cur) {
        if (cur >= 0) end_group(cur);
        cur = grp;
        begin_group(grp);
      }
      const int mt = grp / a.nkv;
      const bool committed_page = (long long)(pr + 1) * 64 <= base;
      mbar_wait(&full[rc.slot], rc.parity, P.err);
      const __half* ks = reinterpret_cast<const __half*>(ring + (size_t)rc.slot * P.stage_bytes);
      const __half* vs = ks + 64 * kHd;
      // S = Q K^T: warp j < 8 owns positions {16c + 2j + e}; row r of Ss = m-tile row, column = position
      if (warp < 8) {
        const int j = warp;
        float S[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int pos = 16 * (g / 2) + 2 * j + (g % 2);
        const uint4* kr = reinterpret_cast<const uint4*>(ks + (size_t)pos * kHd);
        uint4 kw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) kw[u] = kr[kv_k_chunk(4 * t + u, pos)];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma16816(S, word_of4(qw0, 2 * kk), word_of4(qw1, 2 * kk), word_of4(qw0, 2 * kk + 1), word_of4(qw1, 2 * kk + 1),
                   word_of4(kw, 2 * kk), word_of4(kw, 2 * kk + 1));
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        const int i0 = r0 / group, i1 = r1 / group;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = 16 * t + 2 * j + e;
          const long long ap = (long long)pr * 64 + col;
          const bool vis0 = i0 < q && (committed_page || ap - base <= i0);
          const bool vis1 = i1 < q && (committed_page || ap - base <= i1);
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[rc.slot]);
      rc.next(P.stages);
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
int launch_t(const MkParams& p, int grid, cudaStream_t st) {
  auto kern = window_mk_kernel<Raw, NT>;
  const size_t smem = mk_smem_bytes(p.stages, p.stage_bytes);
  CLM_TRY(ensure_smem(kern, smem));
  CLM_CUDA(cudaMemsetAsync(p.barrier, 0, sizeof(unsigned), st));
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
  auto kern = window_mk_kernel<Raw, NT>;
  const size_t smem = mk_smem_bytes(stages, stage_bytes);
  if (ensure_smem(kern, smem) != CLM_OK) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kG4Threads, smem) != cudaSuccess) return 0;
  int sms = 0, coop = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return 0;
  return per_sm >= 1 ? sms : 0;  // one CTA per SM
}

}  // namespace

int mk_grid(int device, int stages, int stage_bytes, int quant, int nt) {
  if (quant == CLM_QUANT_Q4_K)
    return nt == 1 ? grid_t<RawQ4k, 1>(device, stages, stage_bytes) : grid_t<RawQ4k, 2>(device, stages, stage_bytes);
  return nt == 1 ? grid_t<RawQ80, 1>(device, stages, stage_bytes) : grid_t<RawQ80, 2>(device, stages, stage_bytes);
}

int launch_window_mk(const MkParams& p, int quant, int nt, int grid, cudaStream_t st) {
  CLM_CHECK(grid > 0 && p.stages >= 2, CLM_INTERNAL, "window megakernel not configured");
  if (quant == CLM_QUANT_Q4_K)
    return nt == 1 ? launch_t<RawQ4k, 1>(p, grid, st) : launch_t<RawQ4k, 2>(p, grid, st);
  return nt == 1 ? launch_t<RawQ80, 1>(p, grid, st) : launch_t<RawQ80, 2>(p, grid, st);
}

}  // namespace clm
