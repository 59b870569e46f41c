// gemv_strip.cu — q-row GEMV over 16-row strips with the activations resident in shared memory (sm_100a).
//
// y[p][row] = W[row] . x[p] for q <= 8 window rows and K = 4096 columns (16 superblocks), W in the group-major
// tile layout of gemv.cuh.  The work is the sequence of strips (16 rows x all 4096 columns, one row tile of every
// superblock; for the interleaved gate|up matrix a unit is the pair of row tiles r and r + 4 of a 128-row group,
// which hold the gate and up rows of the same 16 FFN indices).  Units are split into gridDim.x contiguous ranges;
// a unit is never split, so no CTA waits for another: each strip's dot products are complete inside one CTA,
// reduced across its warps in shared memory, and its epilogue runs at once.  This removes the cross-CTA partial
// exchange of the stream-K GEMV (gemv4.cu) from the end of every launch, which is what bounds the small matrices of
// a decode window (QKV, W_o, gate|up).
//
//  * Warp 16 is the producer.  One lane bulk-copies (cp.async.bulk, no multicast) the window's activation
//    fragments and sub-block sums for all 16 superblocks once (80 KB, one mbarrier per 512-column chunk) and keeps a
//    ring of stages full, one stage per half strip (8 tiles, superblocks 8h .. 8h + 7).  Weight copies of the first
//    stages are issued before the dependency wait.
//  * Warps 0..15 consume in two groups of eight; group w / 8 takes the units at even / odd positions of the CTA's
//    range, warp w % 8 the tile of superblock 8h + w % 8 of every stage of the unit (the same dequantising
//    tensor-core step as gemv4), so a warp uses the fragments of two fixed superblocks.
//  * At the end of a unit the group's eight warps store their accumulators, sum them in warp order (deterministic)
//    and run the fused epilogue on the strip's 16 rows: store, residual add + next-input preparation (sum-of-squares
//    partials per 16 columns), RoPE + paged KV append, or SwiGLU + next-input preparation.
//  * Dataflow (Epi::wait non-null): activation chunk c is copied once wait[c] reaches its target, the row scale is
//    read after *ss_done reaches its target, and each finished strip signals its chunk (Epi::sig) and *done.
//  * Every wait is bounded (bulk.cuh); a timeout raises the epilogue's error flag.
#include "gemv_core.cuh"
#include "gemv_strip.cuh"
#include "pdl.cuh"

namespace clm {

namespace {

constexpr int kStripSb = 16;                         // superblocks per row (K = 4096)
constexpr int kStripMaxStages = 8;
constexpr uint32_t kXFragBytes = kStripSb * kXfragSbBytes;  // 64 KB: fragments of all superblocks, one n-tile
constexpr uint32_t kXSumBytes = kStripSb * 1024;             // 16 KB: min / bias B fragments
constexpr uint32_t kChunkFrag = 2 * kXfragSbBytes, kChunkSum = 2 * 1024;
constexpr uint32_t kYBytes = 2 * 2 * 16 * 8 * 4;  // per group: y [16 rows][8 columns] (and the up rows)
constexpr size_t kStripSmemBudget = 220 * 1024;
// accumulator exchange: per group 8 warps x 32 lanes x one float4 (two for SwiGLU units: gate and up)
__host__ __device__ constexpr uint32_t red_bytes(int epi) { return 2 * 8 * 32 * (epi == EPI_SWIGLU_PREP ? 32 : 16); }
__host__ __device__ constexpr uint32_t fixed_bytes(int epi) { return kXFragBytes + kXSumBytes + red_bytes(epi) + kYBytes; }

__device__ __forceinline__ void group_sync(int g) { asm volatile("bar.sync %0, 256;" ::"r"(2 + g) : "memory"); }

}  // namespace

template <typename Raw, int EPI>
__global__ void __launch_bounds__(kG4Threads, 1) gemv_strip_kernel(const uint8_t* __restrict__ tiles, uint32_t rows,
                                                                  int tile_bytes, int stages, XBuf in, int q, Epi epi,
                                                                  int ahead) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStripMaxStages], empty[kStripMaxStages], xbar[kStripSb / 2];
  __shared__ float s_scale[2][8];
  __shared__ float s_ssp[2][256];  // row-scale partial sums: [group][thread]
  constexpr bool kSwiglu = EPI == EPI_SWIGLU_PREP;
  constexpr int kSpu = kSwiglu ? 4 : 2;  // stages per unit
  uint8_t* xfrag = smem;
  uint8_t* xsum = smem + kXFragBytes;
  constexpr int kAcc = kSwiglu ? 2 : 1;
  float4* red = reinterpret_cast<float4*>(smem + kXFragBytes + kXSumBytes);
  float* ybuf = reinterpret_cast<float*>(smem + kXFragBytes + kXSumBytes + red_bytes(EPI));
  uint8_t* ring = smem + fixed_bytes(EPI);
  const int stage_bytes = 8 * tile_bytes;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool linked = epi.wait != nullptr;
  const long long U = kSwiglu ? rows / 32 : rows / 16;
  const int G = gridDim.x;
  const long long u0 = (long long)blockIdx.x * U / G, u1 = (long long)(blockIdx.x + 1) * U / G;
  const int n = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvWarps);  // the eight warps of the group that consumes the stage
    }
    for (int c = 0; c < kStripSb / 2; ++c) mbar_init(&xbar[c], 1);
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kG4Consumers / 32) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t policy = evict_first_policy();
      const int nst = n * kSpu;
      // stage j: unit u0 + j / kSpu, part h = j % kSpu (SwiGLU: h / 2 = gate / up tile), superblocks 8 (h & 1) ..
      auto tile_of = [&](int j, int t) {
        const long long u = u0 + j / kSpu;
        const int h = j % kSpu;
        long long grp;
        int rt;
        if (kSwiglu) {
          grp = u / 4;
          rt = (int)(u % 4) + 4 * (h / 2);
        } else {
          grp = u / 8;
          rt = (int)(u % 8);
        }
        return tiles + (((size_t)grp * kStripSb + 8 * (h & 1) + t) * 8 + rt) * tile_bytes;
      };
      auto issue_stage = [&](int j) {
        const int slot = j % stages;
        uint8_t* dst = ring + (size_t)slot * stage_bytes;
        mbar_expect_tx(&full[slot], (uint32_t)stage_bytes);
        for (int t = 0; t < 8; ++t)
          bulk_g2s_stream(dst + (size_t)t * tile_bytes, tile_of(j, t), (uint32_t)tile_bytes, &full[slot], policy);
      };
      // L2 lookahead: stage j + `ahead` is prefetched into L2 when stage j is issued
      int l2j = 0;
      auto l2_until = [&](int upto) {
        for (; l2j < nst && l2j < upto; ++l2j)
          for (int t = 0; t < 8; ++t) bulk_prefetch_l2(tile_of(l2j, t), (uint32_t)tile_bytes);
      };
      const int pre = min(nst, stages);
      l2j = pre;
      l2_until(pre + ahead);
      for (int j = 0; j < pre; ++j) issue_stage(j);
      if (!linked) griddep_wait();
      griddep_launch();
      // the window's activations, chunk by chunk (a failed dataflow wait drops the chunk's bytes instead)
      for (int c = 0; c < kStripSb / 2; ++c) {
        mbar_expect_tx(&xbar[c], kChunkFrag + kChunkSum);
        if (linked) {
          if (!dep_wait(epi.wait + c, epi.wait_target, epi.err)) {
            mbar_complete_tx(&xbar[c], kChunkFrag + kChunkSum);
            continue;
          }
          fence_proxy_async_global();
        }
        bulk_g2s(xfrag + (size_t)c * kChunkFrag, reinterpret_cast<const uint8_t*>(in.frag) + (size_t)c * kChunkFrag,
                 kChunkFrag, &xbar[c]);
        bulk_g2s(xsum + (size_t)c * kChunkSum, reinterpret_cast<const uint8_t*>(in.sum) + (size_t)c * kChunkSum,
                 kChunkSum, &xbar[c]);
      }
      for (int j = pre; j < nst; ++j) {
        const int slot = j % stages;
        if (!mbar_wait_backoff(&empty[slot], ((j / stages) & 1) ^ 1u, epi.err, 128)) break;
        issue_stage(j);
        if (ahead > 0) l2_until(j + 1 + ahead);  // (at 0 the cursor would prefetch the stage just issued)
      }
      // every copy of this CTA is issued: the next kernel's first bytes into L2 while this one drains
      if (EPI == EPI_ROPE_KV && epi.pf_kv) {
        const long long vis = *epi.pos + q;
        const long long npl = (vis + 63) / 64;
        const int np = (int)(npl < epi.pf_max_pages ? npl : epi.pf_max_pages);
        const size_t page_bytes = (size_t)epi.nkv * 64 * epi.hd * sizeof(__half);
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
  if (!linked) {
    griddep_wait();
    griddep_launch();
  }
  const int grp_of_warp = warp / kGemvWarps, w = warp % kGemvWarps, tg = threadIdx.x % 256;
  const int t = lane % 4;
  float* y = ybuf + grp_of_warp * 2 * 128;  // [16 rows][8 columns], then the up rows (SwiGLU)
  // Row scale (folded rmsnorm) from the input's sum-of-squares partials: thread tg adds partials tg / 8 + 32 k
  // (k ascending) of row tg % 8, all of them independent loads; the first epilogue adds the 32 threads of a row in
  // order (for up to 32 partials the serial partial order).  Issued here, so the loads overlap the first strip,
  // unless the partials are still being written (dataflow mode, after the epilogue's readiness wait).
  auto ss_part = [&]() -> float {
    float a = 0.0f;
    if (in.ss && tg % 8 < q)
      for (int c = tg / 8; c < in.nss; c += 32) a += __ldcg(in.ss + (size_t)c * kSsRows + tg % 8);
    return a;
  };
  const float ss_pre = linked ? 0.0f : ss_part();
  bool scale_ready = false;
  uint32_t xready = 0;  // chunks of this warp's superblocks already waited for
  for (int i = grp_of_warp; i < n; i += 2) {
    const long long u = u0 + i;
    G4Acc<1> acc[kAcc];
#pragma unroll
    for (int a = 0; a < kAcc; ++a) acc[a].zero();
#pragma unroll
    for (int h = 0; h < kSpu; ++h) {
      const int j = i * kSpu + h;
      const int slot = j % stages;
      const int sb = 8 * (h & 1) + w;
      if (!(xready & (1u << (sb / 2)))) {
        mbar_wait(&xbar[sb / 2], 0, epi.err);
        xready |= 1u << (sb / 2);
      }
      mbar_wait(&full[slot], (uint32_t)((j / stages) & 1), epi.err);
      const uint8_t* tile = ring + (size_t)slot * stage_bytes + (size_t)w * tile_bytes;
      const uint2* xf = reinterpret_cast<const uint2*>(xfrag) + sb * 512;
      const uint4* sf = reinterpret_cast<const uint4*>(xsum) + sb * 64;
      G4Acc<1>& A = acc[kSwiglu ? h / 2 : 0];
      uint32_t mg, mg8;
      Raw r;
      load_raw_s(r, tile, lane);
      tile_mmas<1>(r, t, xf, lane, A.v, mg, mg8);
      const uint4 b = sf[lane];
      mma16816(A.v[0][0], mg, mg8, mg, mg8, b.x, b.y);
      mma16816(A.v[1][0], mg, mg8, mg, mg8, b.z, b.w);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // ---- the group's eight partial strips -> y (warp order), then the epilogue on the strip's 16 rows.  One
    // exchange buffer per group: a warp rewrites it only after the group's later barriers, when every read is done.
    float4* rb = red + (size_t)grp_of_warp * 8 * 32 * kAcc;
#pragma unroll
    for (int a = 0; a < kAcc; ++a) {
      const float(&v)[2][1][4] = acc[a].v;
      rb[(w * 32 + lane) * kAcc + a] =
          make_float4(v[0][0][0] + v[1][0][0], v[0][0][1] + v[1][0][1], v[0][0][2] + v[1][0][2], v[0][0][3] + v[1][0][3]);
    }
    if (!scale_ready) {
      // row scale (folded rmsnorm) from the input's sum-of-squares partials, summed in partial order
      if (epi.ss_done != nullptr && tg == 0) (void)dep_wait(epi.ss_done, epi.ss_target, epi.err);
      group_sync(grp_of_warp);
      s_ssp[grp_of_warp][tg] = linked ? ss_part() : ss_pre;
      group_sync(grp_of_warp);
      if (tg < 8) {
        float sc = 1.0f;
        if (in.ss && tg < q) {
          float tot = 0.0f;
          for (int c = 0; c < 32; ++c) tot += s_ssp[grp_of_warp][tg + 8 * c];
          sc = 1.0f / sqrtf(tot / epi.ss_n + epi.eps);
        }
        s_scale[grp_of_warp][tg] = sc;
      }
      scale_ready = true;
    }
    group_sync(grp_of_warp);
    if (tg < 128 * kAcc) {
      const int a = tg / 128, l = (tg % 128) / 4, e = tg % 4;
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 v = rb[(k * 32 + l) * kAcc + a];
        s += e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
      }
      const int row = l / 4 + 8 * (e >> 1), col = 2 * (l % 4) + (e & 1);
      y[a * 128 + row * 8 + col] = s * s_scale[grp_of_warp][col];
    }
    group_sync(grp_of_warp);
    const float* sc = s_scale[grp_of_warp];
    (void)sc;
    long long row0;
    if (kSwiglu) {
      row0 = (u / 4) * 64 + 16 * (u % 4);  // first FFN index of the unit
    } else {
      row0 = u * 16;
    }
    if (EPI == EPI_STORE) {
      const int r = tg / 8, p = tg % 8;
      if (tg < 128 && p < q && row0 + r < rows) epi.out[(size_t)p * epi.out_ld + row0 + r] = y[r * 8 + p];
    } else if (EPI == EPI_RESID_PREP) {
      if (tg < 16 * q) {
        const int r = tg % 16, p = tg / 16;
        float* hp = epi.h + (size_t)p * epi.H + row0 + r;
        const float hn = __ldcg(hp) + y[r * 8 + p];
        *hp = hn;
        y[r * 8 + p] = hn;
      }
      group_sync(grp_of_warp);
      if (tg < 8) {
        const int p = tg;
        float vals[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) vals[k] = p < q ? y[k * 8 + p] * epi.wnext[row0 + k] : 0.0f;
        prep16(vals, nullptr, p, q, (int)(row0 / 16), 1, epi.hi_scale, epi.next.frag, epi.next.sum, nullptr, epi.H);
      } else if (tg < 16 && epi.next.ss) {
        const int p = tg - 8;
        float a = 0.0f;
        if (p < q)
#pragma unroll
          for (int k = 0; k < 16; ++k) a += y[k * 8 + p] * y[k * 8 + p];
        epi.next.ss[(size_t)(row0 / 16) * kSsRows + p] = a;
      }
    } else if (EPI == EPI_ROPE_KV) {
      // rows row0 .. row0 + 15: dims d0 .. d0 + 15 of head row0 / hd (pairs d0 / 2 + i)
      const int hd = epi.hd, head = (int)(row0 / hd), d0 = (int)(row0 % hd);
      if (tg < 8 * q) {
        const int i = tg % 8, p = tg / 8, pr = d0 / 2 + i;
        const float a = y[(2 * i) * 8 + p], b = y[(2 * i + 1) * 8 + p];
        const long long base = *epi.pos, slot = base + p;
        const int32_t page = epi.pages[slot / 64];
        if (head < epi.nh + epi.nkv) {
          const long long rope_pos = epi.parent ? base + tree_depth4(epi.parent, p) : slot;
          const float2 cs = epi.rope[(size_t)rope_pos * (hd / 2) + pr];
          const float ra = a * cs.x - b * cs.y, rb2 = a * cs.y + b * cs.x;
          __half* dst;
          if (head < epi.nh) {
            dst = epi.q16 + ((size_t)p * epi.nh + head) * hd + 2 * pr;
          } else {
            const int pos = (int)(slot % 64), dd = 2 * pr;
            dst = epi.kpool + (((size_t)page * epi.nkv + (head - epi.nh)) * 64 + pos) * hd + 8 * kv_k_chunk(dd >> 3, pos) +
                  (dd & 7);
          }
          dst[0] = __float2half_rn(ra);
          dst[1] = __float2half_rn(rb2);
        } else {
          const int pos = (int)(slot % 64), dd = 2 * pr;
          __half* vt = epi.vpool + (((size_t)page * epi.nkv + (head - epi.nh - epi.nkv)) * hd + dd) * 64;
          vt[8 * kv_v_chunk(pos >> 3, dd) + (pos & 7)] = __float2half_rn(a);
          vt[64 + 8 * kv_v_chunk(pos >> 3, dd + 1) + (pos & 7)] = __float2half_rn(b);
        }
      }
    } else if (EPI == EPI_SWIGLU_PREP) {
      if (tg < 16 * q) {
        const int k = tg % 16, p = tg / 16;
        const float gv = y[k * 8 + p], uv = y[128 + k * 8 + p];
        y[k * 8 + p] = gv / (1.0f + expf(-gv)) * uv;
      }
      group_sync(grp_of_warp);
      if (tg < 8) {
        const int p = tg;
        float vals[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) vals[k] = p < q ? y[k * 8 + p] : 0.0f;
        prep16(vals, nullptr, p, q, (int)(row0 / 16), 1, epi.hi_scale, epi.next.frag, epi.next.sum, nullptr, epi.ffn);
      }
    }
    if (epi.sig != nullptr || epi.done != nullptr) {
      group_sync(grp_of_warp);  // the strip's stores are all issued before the release
      if (tg == 0) {
        if (epi.sig != nullptr) {
          int c = (int)(row0 / 512);
          if (epi.sig_qkv) {
            const int head = (int)(row0 / epi.hd), group = epi.nh / epi.nkv;
            c = head < epi.nh ? head / group : (head < epi.nh + epi.nkv ? head - epi.nh : head - epi.nh - epi.nkv);
          }
          red_release_add(epi.sig + c, 1);
        }
        if (epi.done != nullptr) red_release_add(epi.done, 1);
      }
    }
  }
}

bool gemv_strip_ok(const GemvShape& s, int q, int epi_kind) {
  if (s.sb != kStripSb || q < 1 || q > 8 || s.rows % 16 != 0) return false;
  if (s.quant != CLM_QUANT_Q4_K && s.quant != CLM_QUANT_Q8_0) return false;
  if (epi_kind == EPI_SWIGLU_PREP && s.rows % 128 != 0) return false;
  return strip_stages(s, epi_kind) >= 2;
}

int strip_stages(const GemvShape& s, int epi_kind) {
  const size_t stage = (size_t)8 * s.tile_bytes;
  const size_t fit = (kStripSmemBudget - fixed_bytes(epi_kind)) / stage;
  return (int)(fit < (size_t)kStripMaxStages ? fit : kStripMaxStages);
}

template <typename Raw, int EPI>
static int launch_strip(const GemvShape& s, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi,
                        int sm_count, cudaStream_t st) {
  auto kern = gemv_strip_kernel<Raw, EPI>;
  const int stages = strip_stages(s, EPI);
  const size_t smem = fixed_bytes(EPI) + (size_t)stages * 8 * s.tile_bytes;
  CLM_TRY(ensure_smem(kern, smem));
  return launch_pdl(kern, dim3((unsigned)sm_count), dim3(kG4Threads), smem, st, d_tiles, s.rows, s.tile_bytes, stages,
                    in, q, epi, 2 * gemv_l2_ahead());
}

int launch_gemv_strip(const GemvShape& s, const uint8_t* d_tiles, const XBuf& in, int q, const Epi& epi, int sm_count,
                      cudaStream_t st) {
  CLM_CHECK(gemv_strip_ok(s, q, epi.kind), CLM_INTERNAL, "matrix or window outside the strip GEMV");
  const bool q4 = s.quant == CLM_QUANT_Q4_K;
  switch (epi.kind) {
    case EPI_STORE:
      return q4 ? launch_strip<RawQ4k, EPI_STORE>(s, d_tiles, in, q, epi, sm_count, st)
                : launch_strip<RawQ80, EPI_STORE>(s, d_tiles, in, q, epi, sm_count, st);
    case EPI_RESID_PREP:
      return q4 ? launch_strip<RawQ4k, EPI_RESID_PREP>(s, d_tiles, in, q, epi, sm_count, st)
                : launch_strip<RawQ80, EPI_RESID_PREP>(s, d_tiles, in, q, epi, sm_count, st);
    case EPI_ROPE_KV:
      return q4 ? launch_strip<RawQ4k, EPI_ROPE_KV>(s, d_tiles, in, q, epi, sm_count, st)
                : launch_strip<RawQ80, EPI_ROPE_KV>(s, d_tiles, in, q, epi, sm_count, st);
    case EPI_SWIGLU_PREP:
      return q4 ? launch_strip<RawQ4k, EPI_SWIGLU_PREP>(s, d_tiles, in, q, epi, sm_count, st)
                : launch_strip<RawQ80, EPI_SWIGLU_PREP>(s, d_tiles, in, q, epi, sm_count, st);
  }
  return fail(CLM_INTERNAL, "unknown GEMV epilogue");
}

}  // namespace clm
