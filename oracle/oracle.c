/*
 * oracle.c — CPU restatement of ClusterLM's speculative-window hot path.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, the smoke check and bench.py's cpu_baseline leg as the
 * checker.  The product library (clusterlm_b200/lib/libclm_b200.so) never links or calls this code.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math), matching the reference's
 * determinism flags (runtime/domain/CMakeLists.txt:9-14).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ============================ binary16 ============================ */

/* runtime/objects/src/tensor_codec.cpp:16-40 (half_to_float): exact widening incl. subnormals. */
float orc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      uint32_t e = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --e;
      }
      bits = sign | (e << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* tensor_codec.cpp:42-64 (float_to_half): round to nearest even, NaN -> quiet, overflow -> inf. */
uint16_t orc_float_to_half(float f) {
  uint32_t bits;
  memcpy(&bits, &f, sizeof bits);
  uint32_t sign = (bits >> 16) & 0x8000u;
  uint32_t a = bits & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);
  if (a >= 0x47800000u) return (uint16_t)(sign | 0x7C00u);
  if (a < 0x38800000u) {
    if (a < 0x33000000u) return (uint16_t)sign;
    uint32_t e = a >> 23;
    uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126 - e;
    uint32_t h = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = (((a >> 23) - 127 + 15) << 10) | ((a >> 13) & 0x3FFu);
  uint32_t rem = a & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

/* ============================ codecs ============================ */

static float load_f32le(const uint8_t* p) {
  uint32_t b = (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
  float v;
  memcpy(&v, &b, sizeof v);
  return v;
}

static void store_f32le(uint8_t* p, float v) {
  uint32_t b;
  memcpy(&b, &v, sizeof b);
  for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(b >> (8 * i));
}

/* tensor_codec.cpp:9-14 plus the ggml Q4_K block (256 elements, 144 bytes; ggml_types.cpp:26). */
uint64_t orc_tensor_bytes(int quant, uint64_t n) {
  switch (quant) {
    case ORC_F32: return n * 4;
    case ORC_Q8_FIXTURE: return n % 32 == 0 ? n / 32 * 36 : 0;
    case ORC_Q8_0: return n % 32 == 0 ? n / 32 * 34 : 0;
    case ORC_Q4_K: return n % 256 == 0 ? n / 256 * 144 : 0;
    default: return 0;
  }
}

/* Q4_K 6-bit scale/min of sub-block j from the 12 packed bytes (public ggml block layout). */
static void q4k_scale_min(const uint8_t* sc, int j, uint8_t* s, uint8_t* m) {
  if (j < 4) {
    *s = sc[j] & 63;
    *m = sc[j + 4] & 63;
  } else {
    *s = (uint8_t)((sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4));
    *m = (uint8_t)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
  }
}

static void decode_q4k_block(const uint8_t* b, float* y) {
  float d = orc_half_to_float((uint16_t)(b[0] | b[1] << 8));
  float dmin = orc_half_to_float((uint16_t)(b[2] | b[3] << 8));
  const uint8_t* sc = b + 4;
  const uint8_t* qs = b + 16;
  for (int j = 0; j < 8; ++j) {
    uint8_t s, m;
    q4k_scale_min(sc, j, &s, &m);
    float ds = d * (float)s;    /* d * sc in f32, as gguf-py's dequantize_blocks */
    float dm = dmin * (float)m; /* dmin * m in f32 */
    const uint8_t* q = qs + 32 * (j / 2);
    int shift = (j & 1) ? 4 : 0;
    for (int l = 0; l < 32; ++l) y[32 * j + l] = ds * (float)((q[l] >> shift) & 0xF) - dm;
  }
}

/* tensor_codec.cpp:75-99 (decode_tensor) for f32 / q8_0 / q8_0-fixture; Q4_K as decoded above. */
int orc_decode_tensor(int quant, const uint8_t* bytes, uint64_t nbytes, float* out, uint64_t n) {
  uint64_t want = orc_tensor_bytes(quant, n);
  if (want == 0 && n != 0) return 1;
  if (nbytes != want) return 7;
  if (quant == ORC_F32) {
    for (uint64_t i = 0; i < n; ++i) out[i] = load_f32le(bytes + 4 * i);
  } else if (quant == ORC_Q8_0) {
    for (uint64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = bytes + b * 34;
      float scale = orc_half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
      for (int i = 0; i < 32; ++i) out[b * 32 + i] = scale * (float)(int8_t)blk[2 + i];
    }
  } else if (quant == ORC_Q8_FIXTURE) {
    for (uint64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = bytes + b * 36;
      float scale = load_f32le(blk);
      for (int i = 0; i < 32; ++i) out[b * 32 + i] = scale * (float)(int8_t)blk[4 + i];
    }
  } else {
    for (uint64_t b = 0; b < n / 256; ++b) decode_q4k_block(bytes + b * 144, out + b * 256);
  }
  return 0;
}

/* tensor_codec.cpp:110-125 (encode_q8_fixture): scale = amax/127, q = nearbyint(v/scale) clamped. */
int orc_encode_q8_fixture(const float* v, uint64_t n, uint8_t* out) {
  if (n % 32 != 0) return 1;
  for (uint64_t b = 0; b < n; b += 32) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[b + i]));
    float scale = amax / 127.0f;
    uint8_t* o = out + (b / 32) * 36;
    store_f32le(o, scale);
    for (int i = 0; i < 32; ++i) {
      float q = scale == 0.0f ? 0.0f : nearbyintf(v[b + i] / scale);
      if (q < -127.0f) q = -127.0f;
      if (q > 127.0f) q = 127.0f;
      o[4 + i] = (uint8_t)(int8_t)q;
    }
  }
  return 0;
}

/* tensor_codec.cpp:127-141 (encode_q8_0_ggml): d = amax/127 stored as binary16, q = round(v * (1/d)). */
int orc_encode_q8_0(const float* v, uint64_t n, uint8_t* out) {
  if (n % 32 != 0) return 1;
  for (uint64_t b = 0; b < n; b += 32) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[b + i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t h = orc_float_to_half(d);
    uint8_t* o = out + (b / 32) * 34;
    o[0] = (uint8_t)(h & 0xFF);
    o[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)(int8_t)roundf(v[b + i] * id);
  }
  return 0;
}

static float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

/* Q4_K encoder (this project's own; the reference has none).  Per 32-element sub-block: range
 * [min(0,min x), max x] -> scale = range/15, mneg = -min; per 256-element superblock: d = max scale/63,
 * dmin = max mneg/63 rounded to binary16; 6-bit sc/m = rint(scale/d), rint(mneg/dmin); nibble
 * q = rint((x + dmin*m)/(d*sc)) clamped to [0,15].  Every step is a single IEEE operation so the
 * device encoder reproduces the bytes exactly. */
int orc_encode_q4_k(const float* v, uint64_t n, uint8_t* out) {
  if (n % 256 != 0) return 1;
  for (uint64_t sb = 0; sb < n / 256; ++sb) {
    const float* x = v + sb * 256;
    uint8_t* o = out + sb * 144;
    float scale[8], mneg[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
      float mn = x[32 * j], mx = x[32 * j];
      for (int l = 1; l < 32; ++l) {
        float t = x[32 * j + l];
        if (t < mn) mn = t;
        if (t > mx) mx = t;
      }
      if (mn > 0.0f) mn = 0.0f;
      scale[j] = (mx - mn) / 15.0f;
      mneg[j] = -mn;
      if (scale[j] > max_scale) max_scale = scale[j];
      if (mneg[j] > max_min) max_min = mneg[j];
    }
    uint16_t dh = orc_float_to_half(max_scale / 63.0f);
    uint16_t mh = orc_float_to_half(max_min / 63.0f);
    float df = orc_half_to_float(dh), mf = orc_half_to_float(mh);
    uint8_t sc[8], mq[8];
    for (int j = 0; j < 8; ++j) {
      sc[j] = df > 0.0f ? (uint8_t)clampf(rintf(scale[j] / df), 0.0f, 63.0f) : 0;
      mq[j] = mf > 0.0f ? (uint8_t)clampf(rintf(mneg[j] / mf), 0.0f, 63.0f) : 0;
    }
    o[0] = (uint8_t)(dh & 0xFF);
    o[1] = (uint8_t)(dh >> 8);
    o[2] = (uint8_t)(mh & 0xFF);
    o[3] = (uint8_t)(mh >> 8);
    uint8_t* s12 = o + 4;
    for (int j = 0; j < 4; ++j) {
      s12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      s12[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
      s12[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
      float es = df * (float)sc[j];
      float em = mf * (float)mq[j];
      for (int l = 0; l < 32; ++l) {
        float t = es > 0.0f ? clampf(rintf((x[32 * j + l] + em) / es), 0.0f, 15.0f) : 0.0f;
        q[32 * j + l] = (uint8_t)t;
      }
    }
    uint8_t* qs = o + 16;
    for (int p = 0; p < 4; ++p)
      for (int l = 0; l < 32; ++l) qs[32 * p + l] = (uint8_t)(q[64 * p + l] | (q[64 * p + 32 + l] << 4));
  }
  return 0;
}

/* ============================ reference math ============================ */

/* reference_math.hpp:12-16 */
float orc_dot(const float* a, const float* b, uint64_t n) {
  float acc = 0.0f;
  for (uint64_t i = 0; i < n; ++i) acc += a[i] * b[i];
  return acc;
}

/* reference_math.hpp:19-21 */
void orc_matvec(const float* w, uint64_t rows, uint64_t cols, const float* x, float* y) {
  for (uint64_t i = 0; i < rows; ++i) y[i] = orc_dot(w + i * cols, x, cols);
}

/* reference_math.hpp:24-29 (eps is 1e-6 there; the Llama-shaped family passes its own). */
void orc_rmsnorm(const float* x, const float* w, uint64_t n, float eps, float* out) {
  float ss = 0.0f;
  for (uint64_t i = 0; i < n; ++i) ss += x[i] * x[i];
  float denom = sqrtf(ss / (float)n + eps);
  for (uint64_t i = 0; i < n; ++i) out[i] = x[i] * w[i] / denom;
}

/* reference_math.hpp:31-32 */
float orc_sigmoid(float z) { return 1.0f / (1.0f + expf(-z)); }
float orc_silu(float z) { return z / (1.0f + expf(-z)); }

/* reference_kernels.cpp:24-30 */
void orc_matmul_rows(const float* w, uint64_t rows, uint64_t cols, const float* x, uint64_t positions, float* y) {
  for (uint64_t i = 0; i < rows; ++i) {
    const float* row = w + i * cols;
    for (uint64_t p = 0; p < positions; ++p) y[p * rows + i] = orc_dot(row, x + p * cols, cols);
  }
}

typedef struct {
  int quant;
  const uint8_t* w;
  uint64_t row_bytes, rows, cols, positions, r0, r1;
  const float* x;
  float* y;
  int status;
} mm_job;

static void* mm_worker(void* arg) {
  mm_job* j = (mm_job*)arg;
  float* row = (float*)malloc(j->cols * sizeof(float));
  if (!row) {
    j->status = 6;
    return NULL;
  }
  for (uint64_t i = j->r0; i < j->r1; ++i) {
    int st = orc_decode_tensor(j->quant, j->w + i * j->row_bytes, j->row_bytes, row, j->cols);
    if (st) {
      j->status = st;
      break;
    }
    for (uint64_t p = 0; p < j->positions; ++p) j->y[p * j->rows + i] = orc_dot(row, j->x + p * j->cols, j->cols);
  }
  free(row);
  return NULL;
}

int orc_matmul_rows_quant(int quant, const uint8_t* w, uint64_t rows, uint64_t cols, const float* x,
                          uint64_t positions, float* y, int threads) {
  uint64_t rb = orc_tensor_bytes(quant, cols);
  if (rb == 0) return 1;
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > rows) threads = (int)rows;
  mm_job* jobs = (mm_job*)calloc((size_t)threads, sizeof(mm_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !tids) {
    free(jobs);
    free(tids);
    return 6;
  }
  for (int t = 0; t < threads; ++t) {
    mm_job* j = &jobs[t];
    j->quant = quant;
    j->w = w;
    j->row_bytes = rb;
    j->rows = rows;
    j->cols = cols;
    j->positions = positions;
    j->r0 = rows * (uint64_t)t / (uint64_t)threads;
    j->r1 = rows * (uint64_t)(t + 1) / (uint64_t)threads;
    j->x = x;
    j->y = y;
  }
  int status = 0;
  if (threads == 1) {
    mm_worker(&jobs[0]);
  } else {
    for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, mm_worker, &jobs[t]);
    for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
  }
  for (int t = 0; t < threads; ++t)
    if (jobs[t].status) status = jobs[t].status;
  free(jobs);
  free(tids);
  return status;
}

/* ============================ RNG ============================ */

static uint64_t splitmix_step(uint64_t* x) {
  uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

/* sampling.cpp:20-22 (Rng::Rng) */
void orc_rng_seed(orc_rng* r, uint64_t seed) {
  for (int i = 0; i < 4; ++i) r->s[i] = splitmix_step(&seed);
}

/* sampling.cpp:24-35 (Rng::next, xoshiro256**) */
uint64_t orc_rng_next(orc_rng* r) {
  uint64_t* s = r->s;
  uint64_t result = rotl64(s[1] * 5, 7) * 9;
  uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
  return result;
}

/* sampling.cpp:33 */
double orc_rng_uniform(orc_rng* r) { return (double)(orc_rng_next(r) >> 11) * 0x1.0p-53; }

/* sampling.cpp:37-42 */
uint64_t orc_mix_seed(uint64_t a, uint64_t b) {
  uint64_t x = a;
  uint64_t h = splitmix_step(&x);
  x = b ^ 0xD1B54A32D192ED03ull;
  return h ^ (splitmix_step(&x) * 0x9E3779B97F4A7C15ull);
}

/* drafter.cpp:10-15 */
uint64_t orc_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Philox4x32-10, from the published round function (multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key
 * increments 0x9E3779B9 / 0xBB67AE85). */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
  uint32_t k0 = key[0], k1 = key[1];
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
    c0 = n0;
    c1 = n1;
    c2 = n2;
    c3 = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

double orc_philox_uniform(uint64_t key, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
  uint32_t ctr[4] = {c0, c1, c2, c3};
  uint32_t k[2] = {(uint32_t)key, (uint32_t)(key >> 32)};
  uint32_t o[4];
  orc_philox4x32_10(ctr, k, o);
  uint64_t bits = ((uint64_t)o[0] << 32) | o[1];
  return (double)(bits >> 11) * 0x1.0p-53;
}

/* ============================ sampling ============================ */

/* sampling.cpp:44-49: ties resolve to the lowest index. */
int32_t orc_argmax(const float* logits, uint64_t n) {
  uint64_t best = 0;
  for (uint64_t i = 1; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  return (int32_t)best;
}

/* Stable merge sort of indices by e[] descending (std::stable_sort with e[a] > e[b], sampling.cpp:70). */
static void stable_sort_desc(uint32_t* idx, uint32_t* tmp, uint64_t n, const double* e) {
  for (uint64_t width = 1; width < n; width *= 2) {
    for (uint64_t lo = 0; lo < n; lo += 2 * width) {
      uint64_t mid = lo + width < n ? lo + width : n;
      uint64_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      uint64_t a = lo, b = mid, o = lo;
      while (a < mid && b < hi) tmp[o++] = (e[idx[b]] > e[idx[a]]) ? idx[b++] : idx[a++];
      while (a < mid) tmp[o++] = idx[a++];
      while (b < hi) tmp[o++] = idx[b++];
    }
    memcpy(idx, tmp, n * sizeof(uint32_t));
  }
}

/* sampling.cpp:51-86 */
void orc_distribution(const float* logits, uint64_t n, float temperature, uint32_t top_k, float top_p, float* out) {
  for (uint64_t i = 0; i < n; ++i) out[i] = 0.0f;
  if (n == 0) return;
  if (temperature <= 0.0f) {
    out[orc_argmax(logits, n)] = 1.0f;
    return;
  }
  float mx = logits[0];
  for (uint64_t i = 1; i < n; ++i)
    if (logits[i] > mx) mx = logits[i];
  double* e = (double*)malloc(n * sizeof(double));
  uint32_t* order = (uint32_t*)malloc(n * sizeof(uint32_t));
  uint32_t* tmp = (uint32_t*)malloc(n * sizeof(uint32_t));
  double sum = 0;
  for (uint64_t i = 0; i < n; ++i) {
    e[i] = exp((double)(logits[i] - mx) / (double)temperature);
    sum += e[i];
  }
  for (uint64_t i = 0; i < n; ++i) order[i] = (uint32_t)i;
  stable_sort_desc(order, tmp, n, e);
  uint64_t keep = n;
  if (top_k > 0 && top_k < keep) keep = top_k;
  if (top_p < 1.0f) {
    double acc = 0;
    for (uint64_t i = 0; i < keep; ++i) {
      acc += e[order[i]] / sum;
      if (acc >= (double)top_p) {
        keep = i + 1;
        break;
      }
    }
  }
  double kept = 0;
  for (uint64_t i = 0; i < keep; ++i) kept += e[order[i]];
  for (uint64_t i = 0; i < keep; ++i) out[order[i]] = (float)(e[order[i]] / kept);
  free(e);
  free(order);
  free(tmp);
}

/* sampling.cpp:88-101 with the uniform supplied. */
int32_t orc_sample_from(const float* probs, uint64_t n, double u) {
  double total = 0;
  for (uint64_t i = 0; i < n; ++i) total += (double)probs[i];
  double r = u * total;
  double acc = 0;
  int32_t last_nonzero = 0;
  for (uint64_t i = 0; i < n; ++i) {
    if (probs[i] <= 0.0f) continue;
    acc += (double)probs[i];
    last_nonzero = (int32_t)i;
    if (r < acc) return last_nonzero;
  }
  return last_nonzero;
}

/* sampling.cpp:103-131 */
void orc_verify_speculative(const float* target, const int32_t* drafts, const float* draft_probs, uint32_t k,
                            uint64_t V, const double* uniforms, uint32_t* accepted, int32_t* next_token,
                            uint32_t* used) {
  uint32_t u = 0, acc = 0;
  int one_hot = draft_probs == NULL;
  for (uint32_t j = 0; j < k; ++j) {
    const float* P = target + (uint64_t)j * V;
    uint64_t d = (uint64_t)(uint32_t)drafts[j];
    double p = d < V ? (double)P[d] : 0.0;
    double qd = one_hot ? 1.0 : (d < V ? (double)draft_probs[(uint64_t)j * V + d] : 0.0);
    if (qd > 0.0) {
      double ratio = p / qd;
      double lim = ratio < 1.0 ? ratio : 1.0;
      if (uniforms[u++] < lim) {
        ++acc;
        continue;
      }
    }
    float* residual = (float*)malloc(V * sizeof(float));
    double mass = 0;
    for (uint64_t i = 0; i < V; ++i) {
      double qi = one_hot ? (i == d ? 1.0 : 0.0) : (double)draft_probs[(uint64_t)j * V + i];
      double r = (double)P[i] - qi;
      if (r < 0.0) r = 0.0;
      residual[i] = (float)r;
      mass += r;
    }
    *next_token = mass > 0 ? orc_sample_from(residual, V, uniforms[u]) : orc_sample_from(P, V, uniforms[u]);
    ++u;
    free(residual);
    *accepted = acc;
    *used = u;
    return;
  }
  *next_token = orc_sample_from(target + (uint64_t)k * V, V, uniforms[u]);
  ++u;
  *accepted = acc;
  *used = u;
}

/* ============================ drafters ============================ */

/* drafter.cpp:39-55 (MtpFixtureDrafter::step) with refmath rmsnorm eps 1e-6. */
int32_t orc_mtp_fixture_step(const float* embd, const float* norm, const float* head, uint32_t H, uint32_t V,
                             int32_t prev) {
  if (prev < 0 || (uint32_t)prev >= V) return 0;
  float* x = (float*)malloc(H * sizeof(float));
  orc_rmsnorm(embd + (uint64_t)prev * H, norm, H, 1e-6f, x);
  int32_t best = 0;
  float best_logit = orc_dot(head, x, H);
  for (uint32_t v = 1; v < V; ++v) {
    float l = orc_dot(head + (uint64_t)v * H, x, H);
    if (l > best_logit) {
      best_logit = l;
      best = (int32_t)v;
    }
  }
  free(x);
  return best;
}

/* drafter.cpp:91-109 (ScriptedDrafter::draft; corruption_rate only, no forced positions). */
void orc_scripted_draft(const int32_t* ref, uint64_t ref_len, uint32_t vocab, uint64_t seed, double rate,
                        uint64_t committed_len, uint32_t count, int32_t* out) {
  for (uint32_t j = 1; j <= count; ++j) {
    uint64_t pos = committed_len + j;
    int32_t tok = pos < ref_len ? ref[pos] : 0;
    uint64_t h = orc_mix64(seed ^ orc_mix64(pos));
    int corrupt = rate > 0.0 && (double)(h >> 11) / 9007199254740992.0 < rate;
    if (corrupt && vocab >= 2) tok = (int32_t)(((uint64_t)(uint32_t)tok + 1 + (h >> 8) % (vocab - 1)) % vocab);
    out[j - 1] = tok;
  }
}

/* ============================ synthetic weights ============================ */

void orc_gen_weights(uint64_t seed, uint32_t tensor_id, uint64_t first, uint64_t n, float stddev, float* out) {
  uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  float c = stddev * 1.7320508f; /* std of IH4/2^22 is 1/sqrt(3) */
  for (uint64_t i = 0; i < n; ++i) {
    uint64_t idx = first + i;
    uint32_t ctr[4] = {(uint32_t)idx, (uint32_t)(idx >> 32), tensor_id, 0x5747454Eu};
    uint32_t o[4];
    orc_philox4x32_10(ctr, key, o);
    int32_t s = (int32_t)((o[0] >> 10) + (o[1] >> 10) + (o[2] >> 10) + (o[3] >> 10)) - (1 << 23);
    float v = (float)s * 0x1.0p-22f;
    out[i] = v * c;
  }
}

/* ============================ Llama-shaped layer ============================ */

static void rope_inplace(float* v, uint32_t hd, uint64_t pos, float theta) {
  for (uint32_t i = 0; i < hd / 2; ++i) {
    double inv = pow((double)theta, -2.0 * (double)i / (double)hd);
    double ang = (double)pos * inv;
    float c = (float)cos(ang), s = (float)sin(ang);
    float a = v[2 * i], b = v[2 * i + 1];
    v[2 * i] = a * c - b * s;
    v[2 * i + 1] = a * s + b * c;
  }
}

/* The K and V rows one layer appends to its cache for q positions at base..base+q-1 (the prefill of a context
 * without the rest of the layer): rmsnorm(h[p]) with attn_norm, the k and v rows of the q|k|v matrix (rows qd ..
 * qd+2kvd of wqkv), RoPE on k at position base+p -- the same steps as the first half of orc_llama_layer. */
int orc_llama_kv_rows(const orc_llama_dims* d, int quant, const uint8_t* wqkv, const float* attn_norm,
                      const float* h, uint64_t base, uint32_t q, float* kc, float* vc, int threads) {
  const uint32_t H = d->hidden, nh = d->n_heads, nkv = d->n_kv_heads, hd = d->head_dim;
  const uint32_t qd = nh * hd, kvd = nkv * hd;
  float* xn = (float*)malloc((size_t)q * H * sizeof(float));
  float* kv = (float*)malloc((size_t)q * 2 * kvd * sizeof(float));
  int st = 0;
  if (!xn || !kv) {
    st = 6;
    goto done;
  }
  for (uint32_t p = 0; p < q; ++p) orc_rmsnorm(h + (size_t)p * H, attn_norm, H, d->rms_eps, xn + (size_t)p * H);
  if ((st = orc_matmul_rows_quant(quant, wqkv + orc_tensor_bytes(quant, (uint64_t)qd * H), 2 * kvd, H, xn, q, kv,
                                  threads)))
    goto done;
  for (uint32_t p = 0; p < q; ++p) {
    float* row = kv + (size_t)p * 2 * kvd;
    for (uint32_t hh = 0; hh < nkv; ++hh) rope_inplace(row + hh * hd, hd, base + p, d->rope_theta);
    memcpy(kc + (base + p) * kvd, row, kvd * sizeof(float));
    memcpy(vc + (base + p) * kvd, row + kvd, kvd * sizeof(float));
  }
done:
  free(xn);
  free(kv);
  return st;
}

int orc_llama_layer(const orc_llama_dims* d, int quant, const uint8_t* wqkv, const uint8_t* wo, const uint8_t* wgu,
                    const uint8_t* wd, const float* attn_norm, const float* ffn_norm, float* kc, float* vc,
                    uint64_t base, uint32_t q, const int32_t* parent, float* h, int threads) {
  const uint32_t H = d->hidden, nh = d->n_heads, nkv = d->n_kv_heads, hd = d->head_dim, F = d->ffn;
  const uint32_t qd = nh * hd, kvd = nkv * hd, group = nh / nkv;
  float* xn = (float*)malloc((size_t)q * H * sizeof(float));
  float* qkv = (float*)malloc((size_t)q * (qd + 2 * kvd) * sizeof(float));
  float* o = (float*)malloc((size_t)q * qd * sizeof(float));
  float* m = (float*)malloc((size_t)q * H * sizeof(float));
  float* gu = (float*)malloc((size_t)q * 2 * F * sizeof(float));
  float* a = (float*)malloc((size_t)q * F * sizeof(float));
  float* scores = (float*)malloc((size_t)(base + q) * sizeof(float));
  int st = 0;
  if (!xn || !qkv || !o || !m || !gu || !a || !scores) {
    st = 6;
    goto done;
  }
  for (uint32_t p = 0; p < q; ++p) orc_rmsnorm(h + (size_t)p * H, attn_norm, H, d->rms_eps, xn + (size_t)p * H);
  if ((st = orc_matmul_rows_quant(quant, wqkv, qd + 2 * kvd, H, xn, q, qkv, threads))) goto done;
  /* qkv is p-major [q][qd+2kvd] */
  for (uint32_t p = 0; p < q; ++p) {
    float* row = qkv + (size_t)p * (qd + 2 * kvd);
    uint64_t pos = parent ? base + 0 : base + p; /* tree: rope position = depth, set below */
    if (parent) {
      uint64_t depth = 0;
      for (int32_t a2 = parent[p]; a2 >= 0; a2 = parent[a2]) ++depth;
      pos = base + depth;
    }
    for (uint32_t hh = 0; hh < nh; ++hh) rope_inplace(row + hh * hd, hd, pos, d->rope_theta);
    for (uint32_t hh = 0; hh < nkv; ++hh) rope_inplace(row + qd + hh * hd, hd, pos, d->rope_theta);
    memcpy(kc + (base + p) * kvd, row + qd, kvd * sizeof(float));
    memcpy(vc + (base + p) * kvd, row + qd + kvd, kvd * sizeof(float));
  }
  {
    const float scale = 1.0f / sqrtf((float)hd);
    for (uint32_t p = 0; p < q; ++p) {
      const float* qrow = qkv + (size_t)p * (qd + 2 * kvd);
      for (uint32_t hh = 0; hh < nh; ++hh) {
        uint32_t kvh = hh / group;
        const float* qh = qrow + hh * hd;
        /* visible slots: committed 0..base-1, then window slots base+i for i visible to p */
        uint64_t nslot = 0;
        float mx = 0.0f;
        for (uint64_t t = 0; t < base + q; ++t) {
          int vis;
          if (t < base) {
            vis = 1;
          } else if (!parent) {
            vis = t <= base + p;
          } else {
            vis = 0;
            for (int32_t a2 = (int32_t)p; a2 >= 0; a2 = parent[a2])
              if ((uint64_t)a2 == t - base) vis = 1;
          }
          if (!vis) {
            scores[t] = -INFINITY;
            continue;
          }
          float sco = orc_dot(qh, kc + t * kvd + kvh * hd, hd) * scale;
          scores[t] = sco;
          if (nslot == 0 || sco > mx) mx = sco;
          ++nslot;
        }
        float sum = 0.0f;
        for (uint64_t t = 0; t < base + q; ++t) {
          if (scores[t] == -INFINITY) {
            scores[t] = 0.0f;
            continue;
          }
          scores[t] = expf(scores[t] - mx);
          sum += scores[t];
        }
        float* oh = o + (size_t)p * qd + hh * hd;
        for (uint32_t e = 0; e < hd; ++e) oh[e] = 0.0f;
        for (uint64_t t = 0; t < base + q; ++t) {
          if (scores[t] == 0.0f) continue;
          float wt = scores[t] / sum;
          const float* vt = vc + t * kvd + kvh * hd;
          for (uint32_t e = 0; e < hd; ++e) oh[e] += wt * vt[e];
        }
      }
    }
  }
  if ((st = orc_matmul_rows_quant(quant, wo, H, qd, o, q, m, threads))) goto done;
  for (size_t i = 0; i < (size_t)q * H; ++i) h[i] += m[i];
  for (uint32_t p = 0; p < q; ++p) orc_rmsnorm(h + (size_t)p * H, ffn_norm, H, d->rms_eps, xn + (size_t)p * H);
  if ((st = orc_matmul_rows_quant(quant, wgu, 2 * F, H, xn, q, gu, threads))) goto done;
  for (uint32_t p = 0; p < q; ++p)
    for (uint32_t i = 0; i < F; ++i) {
      float g = gu[(size_t)p * 2 * F + i], u = gu[(size_t)p * 2 * F + F + i];
      a[(size_t)p * F + i] = orc_silu(g) * u;
    }
  if ((st = orc_matmul_rows_quant(quant, wd, H, F, a, q, m, threads))) goto done;
  for (size_t i = 0; i < (size_t)q * H; ++i) h[i] += m[i];
done:
  free(xn);
  free(qkv);
  free(o);
  free(m);
  free(gu);
  free(a);
  free(scores);
  return st;
}
