// codec.cu — exact tensor decoding, deterministic encoders and counter-based synthetic weights.
//
// Decode follows runtime/objects/src/tensor_codec.cpp:75-99 (f32, q8_0, q8_0-fixture) and the public ggml
// Q4_K block (d, dmin as binary16; 12 bytes of 6-bit scales/mins; 128 bytes of nibbles).  Every product and
// difference uses the round-to-nearest intrinsics so no contraction into FMA changes a bit.
#include "codec.cuh"

namespace clm {

__device__ __forceinline__ float ld_f32le(const uint8_t* p) {
  const uint32_t b = (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
  return __uint_as_float(b);
}

__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__device__ __forceinline__ void q4k_scale_min(const uint8_t* sc, int j, int* s, int* m) {
  if (j < 4) {
    *s = sc[j] & 63;
    *m = sc[j + 4] & 63;
  } else {
    *s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
    *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
}

__global__ void decode_kernel(int quant, const uint8_t* __restrict__ b, float* __restrict__ out, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float y;
    if (quant == CLM_QUANT_F32) {
      y = ld_f32le(b + 4 * i);
    } else if (quant == CLM_QUANT_Q8_0) {
      const uint8_t* blk = b + (i / 32) * 34;
      y = __fmul_rn(ld_half(blk), (float)(int8_t)blk[2 + i % 32]);
    } else if (quant == CLM_QUANT_Q8_FIXTURE) {
      const uint8_t* blk = b + (i / 32) * 36;
      y = __fmul_rn(ld_f32le(blk), (float)(int8_t)blk[4 + i % 32]);
    } else {
      const uint8_t* blk = b + (i / 256) * 144;
      const int e = (int)(i % 256), j = e / 32, l = e % 32;
      int s, m;
      q4k_scale_min(blk + 4, j, &s, &m);
      const float ds = __fmul_rn(ld_half(blk), (float)s);
      const float dm = __fmul_rn(ld_half(blk + 2), (float)m);
      const int q = (blk[16 + 32 * (j / 2) + l] >> ((j & 1) ? 4 : 0)) & 0xF;
      y = __fsub_rn(__fmul_rn(ds, (float)q), dm);
    }
    out[i] = y;
  }
}

__device__ __forceinline__ float clamp_f(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

// One Q4_K superblock per thread; the arithmetic is the oracle's orc_encode_q4_k step by step.
__device__ void encode_q4k_block(const float* x, uint8_t* o) {
  float scale[8], mneg[8];
  float max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; ++j) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int l = 1; l < 32; ++l) {
      const float t = x[32 * j + l];
      if (t < mn) mn = t;
      if (t > mx) mx = t;
    }
    if (mn > 0.0f) mn = 0.0f;
    scale[j] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    mneg[j] = -mn;
    if (scale[j] > max_scale) max_scale = scale[j];
    if (mneg[j] > max_min) max_min = mneg[j];
  }
  const __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
  const __half mh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
  const float df = __half2float(dh), mf = __half2float(mh);
  int sc[8], mq[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = df > 0.0f ? (int)clamp_f(rintf(__fdiv_rn(scale[j], df)), 0.0f, 63.0f) : 0;
    mq[j] = mf > 0.0f ? (int)clamp_f(rintf(__fdiv_rn(mneg[j], mf)), 0.0f, 63.0f) : 0;
  }
  const unsigned short dbits = __half_as_ushort(dh), mbits = __half_as_ushort(mh);
  o[0] = (uint8_t)(dbits & 0xFF);
  o[1] = (uint8_t)(dbits >> 8);
  o[2] = (uint8_t)(mbits & 0xFF);
  o[3] = (uint8_t)(mbits >> 8);
  for (int j = 0; j < 4; ++j) {
    o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    o[8 + j] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
    o[12 + j] = (uint8_t)((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
  }
  for (int p = 0; p < 4; ++p) {
    const int ja = 2 * p, jb = 2 * p + 1;
    const float esa = __fmul_rn(df, (float)sc[ja]), ema = __fmul_rn(mf, (float)mq[ja]);
    const float esb = __fmul_rn(df, (float)sc[jb]), emb = __fmul_rn(mf, (float)mq[jb]);
    for (int l = 0; l < 32; ++l) {
      const int qa =
          esa > 0.0f ? (int)clamp_f(rintf(__fdiv_rn(__fadd_rn(x[32 * ja + l], ema), esa)), 0.0f, 15.0f) : 0;
      const int qb =
          esb > 0.0f ? (int)clamp_f(rintf(__fdiv_rn(__fadd_rn(x[32 * jb + l], emb), esb)), 0.0f, 15.0f) : 0;
      o[16 + 32 * p + l] = (uint8_t)(qa | (qb << 4));
    }
  }
}

// binary16 bits of f, round to nearest even, by integer arithmetic (the binary16 encoding rules; same
// results as tensor_codec.cpp:42-64 float_to_half).
__device__ __forceinline__ uint32_t f32_to_f16_bits(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const uint32_t a = bits & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return sign | 0x7E00u;
  if (a >= 0x47800000u) return sign | 0x7C00u;
  if (a < 0x38800000u) {
    if (a < 0x33000000u) return sign;
    const uint32_t e = a >> 23, m = (a & 0x7FFFFFu) | 0x800000u, sh = 126 - e;
    uint32_t h = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return sign | h;
  }
  uint32_t h = (((a >> 23) - 127 + 15) << 10) | ((a >> 13) & 0x3FFu);
  const uint32_t rem = a & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return sign | h;
}

// tensor_codec.cpp:127-141 (encode_q8_0_ggml).
__device__ void encode_q8_0_block(const float* x, uint8_t* o) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const uint32_t h = f32_to_f16_bits(d);
  o[0] = (uint8_t)(h & 0xFFu);
  o[1] = (uint8_t)((h >> 8) & 0xFFu);
  for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)(int8_t)roundf(__fmul_rn(x[i], id));
}

__global__ void encode_kernel(int quant, const float* __restrict__ x, uint8_t* __restrict__ out, uint64_t nblocks) {
  const uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  if (quant == CLM_QUANT_Q4_K)
    encode_q4k_block(x + b * 256, out + b * 144);
  else
    encode_q8_0_block(x + b * 32, out + b * 34);
}

__device__ __forceinline__ float gen_weight(uint32_t k0, uint32_t k1, uint32_t tensor_id, uint64_t idx, float c) {
  uint32_t o[4];
  philox4x32_10((uint32_t)idx, (uint32_t)(idx >> 32), tensor_id, 0x5747454Eu, k0, k1, o);
  const int32_t s = (int32_t)((o[0] >> 10) + (o[1] >> 10) + (o[2] >> 10) + (o[3] >> 10)) - (1 << 23);
  return __fmul_rn((float)s * 0x1.0p-22f, c);
}

__global__ void gen_kernel(uint64_t seed, uint32_t tensor_id, uint64_t first, uint64_t n, float c,
                           float* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = gen_weight((uint32_t)seed, (uint32_t)(seed >> 32), tensor_id, first + i, c);
}

// Generates one 256-element row chunk (a superblock) of tensor `tensor_id` and encodes it in place.
__global__ void gen_encode_kernel(int quant, uint64_t seed, uint32_t tensor_id, uint64_t nblocks, float c,
                                  uint8_t* __restrict__ out) {
  const uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const int be = quant == CLM_QUANT_Q4_K ? 256 : 32;
  float x[256];
  for (int i = 0; i < be; ++i) x[i] = gen_weight((uint32_t)seed, (uint32_t)(seed >> 32), tensor_id, b * be + i, c);
  if (quant == CLM_QUANT_Q4_K)
    encode_q4k_block(x, out + b * 144);
  else
    encode_q8_0_block(x, out + b * 34);
}

int launch_decode(int quant, const void* d_bytes, float* d_out, uint64_t n, cudaStream_t s) {
  if (n == 0) return CLM_OK;
  const uint64_t blocks = ceil_div(n, 256);
  decode_kernel<<<(unsigned)(blocks < 65535 * 16 ? blocks : 65535 * 16), 256, 0, s>>>(
      quant, static_cast<const uint8_t*>(d_bytes), d_out, n);
  CLM_LAUNCHED("decode_kernel");
  return CLM_OK;
}

int launch_gen_encode(int quant, uint64_t seed, uint32_t tensor_id, uint64_t n_elems, float stddev, void* d_out,
                      cudaStream_t s) {
  const uint64_t be = quant == CLM_QUANT_Q4_K ? 256 : 32;
  CLM_CHECK(quant == CLM_QUANT_Q4_K || quant == CLM_QUANT_Q8_0, CLM_INVALID_ARGUMENT, "generator quant must be Q4_K or Q8_0");
  CLM_CHECK(n_elems % be == 0, CLM_INVALID_ARGUMENT, "element count is not whole blocks");
  const uint64_t nb = n_elems / be;
  if (nb == 0) return CLM_OK;
  const float c = host_mul(stddev, 1.7320508f);
  gen_encode_kernel<<<(unsigned)ceil_div(nb, 128), 128, 0, s>>>(quant, seed, tensor_id, nb, c,
                                                                 static_cast<uint8_t*>(d_out));
  CLM_LAUNCHED("gen_encode_kernel");
  return CLM_OK;
}

}  // namespace clm

using namespace clm;

extern "C" {

uint64_t clm_b200_tensor_bytes(int quant, uint64_t n) {
  switch (quant) {
    case CLM_QUANT_F32: return n * 4;
    case CLM_QUANT_Q8_FIXTURE: return n % 32 == 0 ? n / 32 * 36 : 0;
    case CLM_QUANT_Q8_0: return n % 32 == 0 ? n / 32 * 34 : 0;
    case CLM_QUANT_Q4_K: return n % 256 == 0 ? n / 256 * 144 : 0;
    default: return 0;
  }
}

int clm_b200_decode_tensor(clm_b200_ctx* ctx, int quant, const void* d_bytes, uint64_t nbytes, float* d_out,
                           uint64_t n, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  const uint64_t want = clm_b200_tensor_bytes(quant, n);
  CLM_CHECK(want != 0 || n == 0, CLM_INVALID_ARGUMENT, "unsupported tensor representation or partial block");
  CLM_CHECK(nbytes == want, CLM_DATA_LOSS, "tensor byte size does not match representation");
  CLM_CHECK(n == 0 || (d_bytes != nullptr && d_out != nullptr), CLM_INVALID_ARGUMENT, "null buffer");
  return launch_decode(quant, d_bytes, d_out, n, pick_stream(ctx, stream));
}

int clm_b200_encode(clm_b200_ctx* ctx, int quant, const float* d_in, uint64_t n, void* d_out, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  CLM_CHECK(quant == CLM_QUANT_Q4_K || quant == CLM_QUANT_Q8_0, CLM_INVALID_ARGUMENT, "encoder quant must be Q4_K or Q8_0");
  const uint64_t be = quant == CLM_QUANT_Q4_K ? 256 : 32;
  CLM_CHECK(n % be == 0, CLM_INVALID_ARGUMENT, "element count is not whole blocks");
  const uint64_t nb = n / be;
  if (nb == 0) return CLM_OK;
  encode_kernel<<<(unsigned)ceil_div(nb, 128), 128, 0, pick_stream(ctx, stream)>>>(quant, d_in,
                                                                                  static_cast<uint8_t*>(d_out), nb);
  CLM_LAUNCHED("encode_kernel");
  return CLM_OK;
}

int clm_b200_generate_weights(clm_b200_ctx* ctx, uint64_t seed, uint32_t tensor_id, uint64_t first, uint64_t n,
                              float stddev, float* d_out, void* stream) {
  CLM_TRY(ctx_enter(ctx));
  if (n == 0) return CLM_OK;
  CLM_CHECK(d_out != nullptr, CLM_INVALID_ARGUMENT, "null output");
  const float c = host_mul(stddev, 1.7320508f);
  const uint64_t blocks = ceil_div(n, 256);
  gen_kernel<<<(unsigned)(blocks < 65535 * 16 ? blocks : 65535 * 16), 256, 0, pick_stream(ctx, stream)>>>(
      seed, tensor_id, first, n, c, d_out);
  CLM_LAUNCHED("gen_kernel");
  return CLM_OK;
}

}  // extern "C"
