/*
 * odi_oracle.c -- CPU restatement of ODIEngine's quantized matrix product.
 * TEST INFRASTRUCTURE ONLY (the checker; never linked into the product).
 * See odi_oracle.h for what is restated and where each piece comes from.
 */
#include "odi_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* fp16 <-> fp32                                                              */
/* ------------------------------------------------------------------------- */

static float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t f32_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* IEEE binary16 -> binary32, exact for every code. */
float orc_fp16_to_fp32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t mant = h & 0x3FFu;
  if (exp == 0) {
    /* zero or subnormal: value = mant * 2^-24, exact in fp32 */
    float v = (float)mant * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_f32(sign | 0x7F800000u | (mant << 13));
  return bits_to_f32(sign | ((exp + 112u) << 23) | (mant << 13));
}

/* The reference converter, cpu_backend.cpp:660-684: correct for normal
 * numbers, zeros, inf and NaN; subnormals take the normalisation loop but
 * skip the exponent rebias, so they come out wrong.  Restated so the oracle
 * reproduces the reference bit for bit on every code. */
float orc_fp16_to_fp32_ref(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (uint32_t)(h & 0x7C00u) >> 10;
  uint32_t mant = (uint32_t)(h & 0x03FFu);
  if (exp == 0) {
    if (mant == 0) return bits_to_f32(sign);
    exp = 1;
    while ((mant & 0x400u) == 0) {
      mant <<= 1;
      exp--;
    }
    mant &= 0x3FFu;
  } else if (exp == 31) {
    exp = 255;
  } else {
    exp = exp + 127 - 15;
  }
  return bits_to_f32(sign | (exp << 23) | (mant << 13));
}

/* binary32 -> binary16, round to nearest even (numpy astype(float16)). */
uint16_t orc_fp32_to_fp16(float f) {
  uint32_t x = f32_to_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t mant = x & 0x7FFFFFu;
  if (exp == 255) return (uint16_t)(sign | 0x7C00u | (mant ? (0x200u | (mant >> 13)) : 0));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    uint32_t m = mant | 0x800000u;
    int shift = 14 - e; /* 24-bit significand -> subnormal field */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t q = ((uint32_t)e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[1] = (uint8_t)(v >> 8);
}

typedef float (*cvt_fn)(uint16_t);

/* ------------------------------------------------------------------------- */
/* Type table: GGUF block sizes (gguf_types.hpp:167-223, tensor.cpp:42-62)    */
/* ------------------------------------------------------------------------- */

int orc_block_elems(int dtype) {
  switch (dtype) {
    case ORC_Q8_0: case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: return 32;
    case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: return 256;
    default: return 0;
  }
}

int orc_block_bytes(int dtype) {
  switch (dtype) {
    case ORC_Q8_0: return 34;
    case ORC_Q4_0: return 18;
    case ORC_Q4_1: return 20;
    case ORC_Q5_0: return 22;
    case ORC_Q5_1: return 24;
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 210;
    default: return 0;
  }
}

static int supported(int dtype) {
  return dtype == ORC_Q8_0 || dtype == ORC_Q4_0 || dtype == ORC_Q4_1 || dtype == ORC_Q5_0 ||
         dtype == ORC_Q5_1 || dtype == ORC_Q4_K || dtype == ORC_Q5_K || dtype == ORC_Q6_K;
}

int64_t orc_row_bytes(int dtype, int64_t K) {
  int be = orc_block_elems(dtype);
  if (!be) return -1;
  return ((K + be - 1) / be) * orc_block_bytes(dtype);
}

/* ------------------------------------------------------------------------- */
/* Block decoders.  One 32- or 256-element block -> fp32, in the arithmetic    */
/* order of the reference (Q4_0, Q8_0) or of gguf 0.19.0 dequantize (K-quants) */
/* ------------------------------------------------------------------------- */

/* Q4_0: value = (q - 8) * d   (cpu_backend.cpp:693-700, 808-811) */
static void dec_q4_0(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk));
  const uint8_t* qs = blk + 2;
  for (int j = 0; j < 16; ++j) {
    out[j] = (float)((qs[j] & 0x0F) - 8) * d;
    out[j + 16] = (float)((qs[j] >> 4) - 8) * d;
  }
}

/* Q8_0: value = q * d  (cpu_backend.cpp:776-778) */
static void dec_q8_0(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk));
  const int8_t* qs = (const int8_t*)(blk + 2);
  for (int j = 0; j < 32; ++j) out[j] = (float)qs[j] * d;
}

/* The fifth bit of element l of a Q5_0 / Q5_1 block: bit l of the
 * little-endian qh word. */
static int qh_bit(const uint8_t* qh, int l) { return (qh[l >> 3] >> (l & 7)) & 1; }

/* Q4_1: value = q * d + m  (cpu_backend.cpp:704-721; block d, m, qs[16]) */
static void dec_q4_1(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk)), m = cvt(rd16(blk + 2));
  const uint8_t* qs = blk + 4;
  for (int j = 0; j < 16; ++j) {
    out[j] = (float)(qs[j] & 0x0F) * d + m;
    out[j + 16] = (float)(qs[j] >> 4) * d + m;
  }
}

/* Q5_0: value = (q - 16) * d, q = nibble | qh bit << 4  (cpu_backend.cpp:723-745;
 * block d, qh[4], qs[16]) */
static void dec_q5_0(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk));
  const uint8_t* qh = blk + 2;
  const uint8_t* qs = blk + 6;
  for (int j = 0; j < 16; ++j) {
    out[j] = (float)(((qs[j] & 0x0F) | (qh_bit(qh, j) << 4)) - 16) * d;
    out[j + 16] = (float)(((qs[j] >> 4) | (qh_bit(qh, j + 16) << 4)) - 16) * d;
  }
}

/* Q5_1: value = q * d + m  (cpu_backend.cpp:747-767; block d, m, qh[4], qs[16]) */
static void dec_q5_1(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk)), m = cvt(rd16(blk + 2));
  const uint8_t* qh = blk + 4;
  const uint8_t* qs = blk + 8;
  for (int j = 0; j < 16; ++j) {
    out[j] = (float)((qs[j] & 0x0F) | (qh_bit(qh, j) << 4)) * d + m;
    out[j + 16] = (float)((qs[j] >> 4) | (qh_bit(qh, j + 16) << 4)) * d + m;
  }
}

/* K-quant 6-bit scale/min unpacking (GGML format, 12 bytes for 8 pairs). */
static void kq_scale_min(const uint8_t* s, int j, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

/* Q4_K block: d, dmin (fp16), scales[12], qs[128].  Sub-block j (32 values)
 * uses qs[32*(j/2) .. +32], low nibbles for even j, high for odd j.
 * value = (d*sc_j) * q - (dmin*m_j). */
static void dec_q4_k(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk)), dmin = cvt(rd16(blk + 2));
  const uint8_t* sc = blk + 4;
  const uint8_t* qs = blk + 16;
  for (int j = 0; j < 8; ++j) {
    int s, m;
    kq_scale_min(sc, j, &s, &m);
    float d1 = d * (float)s, m1 = dmin * (float)m;
    const uint8_t* q = qs + 32 * (j / 2);
    int sh = (j & 1) ? 4 : 0;
    for (int l = 0; l < 32; ++l) out[32 * j + l] = d1 * (float)((q[l] >> sh) & 0x0F) - m1;
  }
}

/* Q5_K block: d, dmin, scales[12], qh[32], qs[128]; the fifth bit of
 * sub-block j element l is bit j of qh[l]. */
static void dec_q5_k(const uint8_t* blk, float* out, cvt_fn cvt) {
  float d = cvt(rd16(blk)), dmin = cvt(rd16(blk + 2));
  const uint8_t* sc = blk + 4;
  const uint8_t* qh = blk + 16;
  const uint8_t* qs = blk + 48;
  for (int j = 0; j < 8; ++j) {
    int s, m;
    kq_scale_min(sc, j, &s, &m);
    float d1 = d * (float)s, m1 = dmin * (float)m;
    const uint8_t* q = qs + 32 * (j / 2);
    int sh = (j & 1) ? 4 : 0;
    for (int l = 0; l < 32; ++l) {
      int v = ((q[l] >> sh) & 0x0F) | (((qh[l] >> j) & 1) << 4);
      out[32 * j + l] = d1 * (float)v - m1;
    }
  }
}

/* Q6_K block: ql[128], qh[64], scales[16] (int8), d (fp16).  Element e of
 * half h (e in 0..127): l = e%32, group c = e/32 (0..3);
 * low 4 bits = ql[64h + l + 32*(c&1)] >> (4*(c>>1)), high 2 bits =
 * qh[32h + l] >> (2c); scale = scales[e_global/16].  value = (d*sc)*(q-32). */
static int q6_code(const uint8_t* blk, int e) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  int h = e / 128, r = e % 128, c = r / 32, l = r % 32;
  int lo = (ql[64 * h + l + 32 * (c & 1)] >> (4 * (c >> 1))) & 0x0F;
  int hi = (qh[32 * h + l] >> (2 * c)) & 3;
  return lo | (hi << 4);
}

static void dec_q6_k(const uint8_t* blk, float* out, cvt_fn cvt) {
  const int8_t* sc = (const int8_t*)(blk + 192);
  float d = cvt(rd16(blk + 208));
  for (int e = 0; e < 256; ++e) {
    float ds = d * (float)sc[e / 16];
    out[e] = ds * (float)(q6_code(blk, e) - 32);
  }
}

static void dec_block(int dtype, const uint8_t* blk, float* out, cvt_fn cvt) {
  switch (dtype) {
    case ORC_Q4_0: dec_q4_0(blk, out, cvt); break;
    case ORC_Q8_0: dec_q8_0(blk, out, cvt); break;
    case ORC_Q4_1: dec_q4_1(blk, out, cvt); break;
    case ORC_Q5_0: dec_q5_0(blk, out, cvt); break;
    case ORC_Q5_1: dec_q5_1(blk, out, cvt); break;
    case ORC_Q4_K: dec_q4_k(blk, out, cvt); break;
    case ORC_Q5_K: dec_q5_k(blk, out, cvt); break;
    case ORC_Q6_K: dec_q6_k(blk, out, cvt); break;
    default: break;
  }
}

int orc_dequantize(int dtype, const void* blocks, int64_t N, int64_t K, float* out, int ref_fp16) {
  if (!supported(dtype) || N < 0 || K < 0) return -1;
  int be = orc_block_elems(dtype), bb = orc_block_bytes(dtype);
  int64_t nb = (K + be - 1) / be;
  cvt_fn cvt = ref_fp16 ? orc_fp16_to_fp32_ref : orc_fp16_to_fp32;
  float tmp[256];
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nb; ++b) {
      dec_block(dtype, (const uint8_t*)blocks + (n * nb + b) * bb, tmp, cvt);
      for (int j = 0; j < be && b * be + j < K; ++j) out[n * K + b * be + j] = tmp[j];
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------- */
/* Quantisers                                                                 */
/* ------------------------------------------------------------------------- */

/* Round half away from zero (numpy np_roundf in gguf 0.19.0 == C roundf). */
static float round_away(float v) { return roundf(v); }

/* Q8_0 block, gguf 0.19.0 Q8_0.quantize_blocks: d = amax/127 (fp32),
 * id = d ? 1/d : 0, q = roundf(x*id), d stored as fp16 (RNE). */
static void quant_q8_0_block(const float* x, uint8_t* blk) {
  float amax = 0.0f;
  for (int j = 0; j < 32; ++j) {
    float a = fabsf(x[j]);
    if (a > amax) amax = a;
  }
  float d = amax / 127.0f;
  float id = (d == 0.0f) ? 0.0f : 1.0f / d;
  wr16(blk, orc_fp32_to_fp16(d));
  for (int j = 0; j < 32; ++j) blk[2 + j] = (uint8_t)(int8_t)round_away(x[j] * id);
}

/* Q4_0 block, gguf 0.19.0 Q4_0.quantize_blocks: max = the signed value of
 * largest magnitude (first on ties), d = max / -8, id = d ? 1/d : 0,
 * q = min(15, trunc(x*id + 8.5)); element j in the low nibble of byte j,
 * element j+16 in the high nibble. */
static void quant_q4_0_block(const float* x, uint8_t* blk) {
  float amax = -1.0f, mx = 0.0f;
  for (int j = 0; j < 32; ++j) {
    float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      mx = x[j];
    }
  }
  float d = mx / -8.0f;
  float id = (d == 0.0f) ? 0.0f : 1.0f / d;
  wr16(blk, orc_fp32_to_fp16(d));
  uint8_t q[32];
  for (int j = 0; j < 32; ++j) {
    float t = truncf(x[j] * id + 8.5f);
    int v = (int)t;
    if (v < 0) v = 0;
    if (v > 15) v = 15;
    q[j] = (uint8_t)v;
  }
  for (int j = 0; j < 16; ++j) blk[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q4_1 (levels 15) / Q5_1 (levels 31), gguf 0.19.0 Q4_1 / Q5_1.quantize_blocks:
 * d = (max - min) / levels, id = d ? 1/d : 0,
 * q = min(levels, trunc((x - min) * id + 0.5)); d and min stored as fp16;
 * element j in the low nibble of qs[j], element j+16 in the high nibble,
 * the fifth bits (Q5_1) packed little-endian into qh, element j at bit j. */
static void quant_qmin_block(const float* x, uint8_t* blk, int levels) {
  float mx = x[0], mn = x[0];
  for (int j = 1; j < 32; ++j) {
    if (x[j] > mx) mx = x[j];
    if (x[j] < mn) mn = x[j];
  }
  float d = (mx - mn) / (float)levels;
  float id = (d == 0.0f) ? 0.0f : 1.0f / d;
  wr16(blk, orc_fp32_to_fp16(d));
  wr16(blk + 2, orc_fp32_to_fp16(mn));
  uint8_t q[32];
  for (int j = 0; j < 32; ++j) q[j] = (uint8_t)clampi((int)truncf((x[j] - mn) * id + 0.5f), 0, levels);
  uint8_t* qs = blk + (levels == 31 ? 8 : 4);
  for (int j = 0; j < 16; ++j) qs[j] = (uint8_t)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
  if (levels == 31) {
    memset(blk + 4, 0, 4);
    for (int j = 0; j < 32; ++j) blk[4 + (j >> 3)] |= (uint8_t)((q[j] >> 4) << (j & 7));
  }
}

/* Q5_0, gguf 0.19.0 Q5_0.quantize_blocks: max = the signed value of largest
 * magnitude (first on ties), d = max / -16, id = d ? 1/d : 0,
 * q = min(31, trunc(x*id + 16.5)); nibbles and fifth bits as Q5_1. */
static void quant_q5_0_block(const float* x, uint8_t* blk) {
  float amax = -1.0f, mx = 0.0f;
  for (int j = 0; j < 32; ++j) {
    float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      mx = x[j];
    }
  }
  float d = mx / -16.0f;
  float id = (d == 0.0f) ? 0.0f : 1.0f / d;
  wr16(blk, orc_fp32_to_fp16(d));
  uint8_t q[32];
  for (int j = 0; j < 32; ++j) q[j] = (uint8_t)clampi((int)truncf(x[j] * id + 16.5f), 0, 31);
  memset(blk + 2, 0, 4);
  for (int j = 0; j < 32; ++j) blk[2 + (j >> 3)] |= (uint8_t)((q[j] >> 4) << (j & 7));
  for (int j = 0; j < 16; ++j) blk[6 + j] = (uint8_t)((q[j] & 0x0F) | ((q[j + 16] & 0x0F) << 4));
}

/* Q4_K / Q5_K quantiser (this project's own; the format is GGML's).
 * Per 32-value sub-block: min mn (clamped to <= 0) and range; scale =
 * range / levels.  The 8 scales and 8 mins are coded as 6-bit multiples of
 * the super-block d = max scale / 63 and dmin = max min / 63 (fp16), then
 * each value is coded against the decoded (fp16-exact) scale and min. */
static void quant_kq45_block(const float* x, uint8_t* blk, int levels, int five) {
  float scale[8], mins[8], maxs = 0.0f, maxm = 0.0f;
  for (int j = 0; j < 8; ++j) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int l = 1; l < 32; ++l) {
      float v = x[32 * j + l];
      if (v < mn) mn = v;
      if (v > mx) mx = v;
    }
    if (mn > 0.0f) mn = 0.0f;
    scale[j] = (mx - mn) / (float)levels;
    mins[j] = -mn;
    if (scale[j] > maxs) maxs = scale[j];
    if (mins[j] > maxm) maxm = mins[j];
  }
  uint16_t dh = orc_fp32_to_fp16(maxs / 63.0f), mh = orc_fp32_to_fp16(maxm / 63.0f);
  float dd = orc_fp16_to_fp32(dh), dm = orc_fp16_to_fp32(mh);
  int ls[8], lm[8];
  for (int j = 0; j < 8; ++j) {
    ls[j] = dd > 0.0f ? clampi((int)round_away(scale[j] / dd), 0, 63) : 0;
    lm[j] = dm > 0.0f ? clampi((int)round_away(mins[j] / dm), 0, 63) : 0;
  }
  memset(blk, 0, five ? 176 : 144);
  wr16(blk, dh);
  wr16(blk + 2, mh);
  uint8_t* s = blk + 4;
  for (int j = 0; j < 4; ++j) {
    s[j] = (uint8_t)(ls[j] | ((ls[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)(lm[j] | ((lm[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((ls[j + 4] & 0x0F) | ((lm[j + 4] & 0x0F) << 4));
  }
  uint8_t* qh = five ? blk + 16 : NULL;
  uint8_t* qs = blk + (five ? 48 : 16);
  for (int j = 0; j < 8; ++j) {
    float es = dd * (float)ls[j], em = dm * (float)lm[j];
    for (int l = 0; l < 32; ++l) {
      int q = 0;
      if (es > 0.0f) q = clampi((int)round_away((x[32 * j + l] + em) / es), 0, levels);
      qs[32 * (j / 2) + l] |= (uint8_t)((q & 0x0F) << ((j & 1) ? 4 : 0));
      if (five) qh[l] |= (uint8_t)(((q >> 4) & 1) << j);
    }
  }
}

/* Q6_K quantiser (own design; GGML format).  16 sub-blocks of 16 values;
 * per sub-block the signed value of largest magnitude v gives scale v/-32;
 * scales are coded as int8 multiples of d = max|scale|/127 (fp16); values
 * as q in [0,63] with value = d*sc*(q-32). */
static void quant_q6_k_block(const float* x, uint8_t* blk) {
  float scale[16], amax = 0.0f;
  for (int j = 0; j < 16; ++j) {
    float best = -1.0f, v = 0.0f;
    for (int l = 0; l < 16; ++l) {
      float a = fabsf(x[16 * j + l]);
      if (a > best) {
        best = a;
        v = x[16 * j + l];
      }
    }
    scale[j] = v / -32.0f;
    if (fabsf(scale[j]) > amax) amax = fabsf(scale[j]);
  }
  uint16_t dh = orc_fp32_to_fp16(amax / 127.0f);
  float d = orc_fp16_to_fp32(dh);
  memset(blk, 0, 210);
  int8_t* sc = (int8_t*)(blk + 192);
  uint8_t q[256];
  for (int j = 0; j < 16; ++j) {
    int s = d > 0.0f ? clampi((int)round_away(scale[j] / d), -128, 127) : 0;
    sc[j] = (int8_t)s;
    float es = d * (float)s;
    for (int l = 0; l < 16; ++l) {
      int v = 32;
      if (es != 0.0f) v = clampi((int)round_away(x[16 * j + l] / es), -32, 31) + 32;
      q[16 * j + l] = (uint8_t)v;
    }
  }
  uint8_t* ql = blk;
  uint8_t* qh = blk + 128;
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 32; ++l) {
      int q1 = q[128 * h + l], q2 = q[128 * h + l + 32], q3 = q[128 * h + l + 64],
          q4 = q[128 * h + l + 96];
      ql[64 * h + l] = (uint8_t)((q1 & 0x0F) | ((q3 & 0x0F) << 4));
      ql[64 * h + l + 32] = (uint8_t)((q2 & 0x0F) | ((q4 & 0x0F) << 4));
      qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  wr16(blk + 208, dh);
}

int orc_quantize(int dtype, const float* w, int64_t N, int64_t K, void* out) {
  if (!supported(dtype) || N < 0 || K < 0) return -1;
  int be = orc_block_elems(dtype), bb = orc_block_bytes(dtype);
  if (be == 256 && K % 256) return -2; /* K-quant rows are whole super-blocks */
  int64_t nb = (K + be - 1) / be;
  float tmp[256];
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nb; ++b) {
      for (int j = 0; j < be; ++j) {
        int64_t k = b * be + j;
        tmp[j] = k < K ? w[n * K + k] : 0.0f;
      }
      uint8_t* blk = (uint8_t*)out + (n * nb + b) * bb;
      switch (dtype) {
        case ORC_Q4_0: quant_q4_0_block(tmp, blk); break;
        case ORC_Q8_0: quant_q8_0_block(tmp, blk); break;
        case ORC_Q4_1: quant_qmin_block(tmp, blk, 15); break;
        case ORC_Q5_0: quant_q5_0_block(tmp, blk); break;
        case ORC_Q5_1: quant_qmin_block(tmp, blk, 31); break;
        case ORC_Q4_K: quant_kq45_block(tmp, blk, 15, 0); break;
        case ORC_Q5_K: quant_kq45_block(tmp, blk, 31, 1); break;
        case ORC_Q6_K: quant_q6_k_block(tmp, blk); break;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------- */
/* Reference-order fp32 matmul                                                */
/* ------------------------------------------------------------------------- */

typedef struct {
  int dtype;
  float* out;
  const float* a;
  const uint8_t* b;
  int64_t M, K, N, n0, n1;
} mm_job;

/* For each (m, n): sum over blocks kb of sequential sum += a[k] * w[k], with
 * the block decoded to fp32 first (matmul_q4_0, cpu_backend.cpp:800-822).
 * Q8_0 keeps its own expression a * q * d (cpu_backend.cpp:846). */
static void* mm_worker(void* arg) {
  mm_job* j = (mm_job*)arg;
  int be = orc_block_elems(j->dtype), bb = orc_block_bytes(j->dtype);
  int64_t nb = (j->K + be - 1) / be;
  float temp[256];
  for (int64_t m = 0; m < j->M; ++m) {
    const float* am = j->a + m * j->K;
    for (int64_t n = j->n0; n < j->n1; ++n) {
      float sum = 0.0f;
      for (int64_t kb = 0; kb < nb; ++kb) {
        const uint8_t* blk = j->b + (n * nb + kb) * bb;
        int64_t k0 = kb * be, k1 = k0 + be < j->K ? k0 + be : j->K;
        if (j->dtype == ORC_Q8_0) {
          float d = orc_fp16_to_fp32_ref(rd16(blk));
          const int8_t* qs = (const int8_t*)(blk + 2);
          for (int64_t k = k0; k < k1; ++k) sum += am[k] * (float)qs[k - k0] * d;
        } else {
          /* The 32-value block types use the reference's own converter; the
           * K-quants have no reference code, so their semantics are gguf's
           * IEEE decode.  (The reference itself runs Q4_1 / Q5_0 / Q5_1
           * through dequantize + matmul_f32 with a layout bug,
           * cpu_backend.cpp:211-216; this is the product the format defines.) */
          dec_block(j->dtype, blk, temp, be == 32 ? orc_fp16_to_fp32_ref : orc_fp16_to_fp32);
          for (int64_t k = k0; k < k1; ++k) sum += am[k] * temp[k - k0];
        }
      }
      j->out[m * j->N + n] = sum;
    }
  }
  return NULL;
}

int orc_matmul_ref(int dtype, float* out, const float* a, const void* b, int64_t M, int64_t K,
                   int64_t N, int nthreads) {
  if (!supported(dtype) || M < 0 || N < 0 || K < 0) return -1;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > N) nthreads = (int)(N > 0 ? N : 1);
  mm_job jobs[256];
  pthread_t th[256];
  for (int t = 0; t < nthreads; ++t) {
    jobs[t] = (mm_job){dtype, out, a, (const uint8_t*)b, M, K, N, N * t / nthreads,
                       N * (t + 1) / nthreads};
  }
  if (nthreads == 1) {
    mm_worker(&jobs[0]);
    return 0;
  }
  for (int t = 0; t < nthreads; ++t) pthread_create(&th[t], NULL, mm_worker, &jobs[t]);
  for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
  return 0;
}

/* ------------------------------------------------------------------------- */
/* Activation quantisation (Q8_0)                                             */
/* ------------------------------------------------------------------------- */

void orc_quantize_q8_0_act(const float* x, int64_t M, int64_t K, void* blocks) {
  int64_t nb = (K + 31) / 32;
  float tmp[32];
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t b = 0; b < nb; ++b) {
      for (int j = 0; j < 32; ++j) {
        int64_t k = b * 32 + j;
        tmp[j] = k < K ? x[m * K + k] : 0.0f;
      }
      quant_q8_0_block(tmp, (uint8_t*)blocks + (m * nb + b) * 34);
    }
  }
}

typedef struct {
  float d;
  int16_t s_lo;
  int16_t s_hi;
} act_rec;

void orc_quantize_act_planes(const float* x, int64_t M, int64_t K, int8_t* xq, void* xs) {
  int64_t Kp = (K + 255) / 256 * 256, nb = Kp / 32;
  act_rec* rec = (act_rec*)xs;
  float tmp[32];
  uint8_t blk[34];
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t b = 0; b < nb; ++b) {
      for (int j = 0; j < 32; ++j) {
        int64_t k = b * 32 + j;
        tmp[j] = k < K ? x[m * K + k] : 0.0f;
      }
      quant_q8_0_block(tmp, blk);
      int slo = 0, shi = 0;
      for (int j = 0; j < 32; ++j) {
        int8_t q = (int8_t)blk[2 + j];
        xq[m * Kp + b * 32 + j] = q;
        if (j < 16) slo += q; else shi += q;
      }
      rec[m * nb + b].d = orc_fp16_to_fp32(rd16(blk));
      rec[m * nb + b].s_lo = (int16_t)slo;
      rec[m * nb + b].s_hi = (int16_t)shi;
    }
  }
}

/* ------------------------------------------------------------------------- */
/* Q8-activation product and bounds                                           */
/* ------------------------------------------------------------------------- */

/* Integer codes and fp32 scale/min factors of one weight block, as the CUDA
 * kernels see them: for each 32-value group g (16-value group for Q6_K) the
 * value is  A_g * q - B_g  with integer q. */
typedef struct {
  int q[256];
  float A[16];  /* per group scale factor (d, d*sc) */
  float B[16];  /* per group min factor (8*d for Q4_0, dmin*m for Q4_K/Q5_K) */
  int gsize;    /* 32 or 16 */
  int ngroups;
  int has_min;  /* B term present */
} wcodes;

static void block_codes(int dtype, const uint8_t* blk, wcodes* c) {
  memset(c, 0, sizeof(*c));
  switch (dtype) {
    case ORC_Q4_0: {
      float d = orc_fp16_to_fp32(rd16(blk));
      for (int j = 0; j < 16; ++j) {
        c->q[j] = blk[2 + j] & 0x0F;
        c->q[j + 16] = blk[2 + j] >> 4;
      }
      c->A[0] = d;
      c->B[0] = 8.0f * d; /* (q-8)*d = d*q - 8d */
      c->gsize = 32; c->ngroups = 1; c->has_min = 1;
      break;
    }
    case ORC_Q8_0: {
      c->A[0] = orc_fp16_to_fp32(rd16(blk));
      for (int j = 0; j < 32; ++j) c->q[j] = (int8_t)blk[2 + j];
      c->gsize = 32; c->ngroups = 1; c->has_min = 0;
      break;
    }
    case ORC_Q4_1:
    case ORC_Q5_0:
    case ORC_Q5_1: {
      /* Q4_1 / Q5_1: d*q + m = d*q - (-m); Q5_0: (q-16)*d = d*q - 16d */
      float d = orc_fp16_to_fp32(rd16(blk));
      const uint8_t* qh = blk + (dtype == ORC_Q5_1 ? 4 : 2);
      const uint8_t* qs = blk + (dtype == ORC_Q4_1 ? 4 : dtype == ORC_Q5_0 ? 6 : 8);
      for (int j = 0; j < 16; ++j) {
        c->q[j] = qs[j] & 0x0F;
        c->q[j + 16] = qs[j] >> 4;
        if (dtype != ORC_Q4_1) {
          c->q[j] |= qh_bit(qh, j) << 4;
          c->q[j + 16] |= qh_bit(qh, j + 16) << 4;
        }
      }
      c->A[0] = d;
      c->B[0] = dtype == ORC_Q5_0 ? 16.0f * d : -orc_fp16_to_fp32(rd16(blk + 2));
      c->gsize = 32; c->ngroups = 1; c->has_min = 1;
      break;
    }
    case ORC_Q4_K:
    case ORC_Q5_K: {
      float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
      int five = dtype == ORC_Q5_K;
      const uint8_t* qh = blk + 16;
      const uint8_t* qs = blk + (five ? 48 : 16);
      for (int j = 0; j < 8; ++j) {
        int s, m;
        kq_scale_min(blk + 4, j, &s, &m);
        c->A[j] = d * (float)s;
        c->B[j] = dmin * (float)m;
        for (int l = 0; l < 32; ++l) {
          int v = (qs[32 * (j / 2) + l] >> ((j & 1) ? 4 : 0)) & 0x0F;
          if (five) v |= ((qh[l] >> j) & 1) << 4;
          c->q[32 * j + l] = v;
        }
      }
      c->gsize = 32; c->ngroups = 8; c->has_min = 1;
      break;
    }
    case ORC_Q6_K: {
      const int8_t* sc = (const int8_t*)(blk + 192);
      float d = orc_fp16_to_fp32(rd16(blk + 208));
      for (int j = 0; j < 16; ++j) c->A[j] = d * (float)sc[j];
      for (int e = 0; e < 256; ++e) c->q[e] = q6_code(blk, e) - 32;
      c->gsize = 16; c->ngroups = 16; c->has_min = 0;
      break;
    }
  }
}

/* Per-element term magnitude T = |A_g * q| + |B_g| of the decomposition
 * value = A_g * q - B_g above (>= |value|; = |value| without a min term).
 * Rounding the two factors to fp16 before combining them errs by at most
 * 2^-11 * T per factor, so T is the scale of the fp16 decoding error of the
 * tensor-core path.  out is [N][K]. */
int orc_term_magnitude(int dtype, const void* blocks, int64_t N, int64_t K, float* out) {
  if (!supported(dtype) || N < 0 || K < 0) return -1;
  int be = orc_block_elems(dtype), bb = orc_block_bytes(dtype);
  int64_t nb = (K + be - 1) / be;
  wcodes c;
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nb; ++b) {
      block_codes(dtype, (const uint8_t*)blocks + (n * nb + b) * bb, &c);
      for (int j = 0; j < be && b * be + j < K; ++j) {
        int g = j / c.gsize;
        float t = fabsf(c.A[g] * (float)c.q[j]) + (c.has_min ? fabsf(c.B[g]) : 0.0f);
        out[n * K + b * be + j] = t;
      }
    }
  }
  return 0;
}

/* Per-element factors of value = A * q - B (A, B fp32 as computed from the
 * block's fp16 fields; B = 0 without a min term).  Out arrays are [N][K]. */
int orc_block_factors(int dtype, const void* blocks, int64_t N, int64_t K, float* A, float* B, int32_t* q) {
  if (!supported(dtype) || N < 0 || K < 0) return -1;
  int be = orc_block_elems(dtype), bb = orc_block_bytes(dtype);
  int64_t nb = (K + be - 1) / be;
  wcodes c;
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nb; ++b) {
      block_codes(dtype, (const uint8_t*)blocks + (n * nb + b) * bb, &c);
      for (int j = 0; j < be && b * be + j < K; ++j) {
        int g = j / c.gsize;
        int64_t o = n * K + b * be + j;
        A[o] = c.A[g];
        B[o] = c.has_min ? c.B[g] : 0.0f;
        q[o] = c.q[j];
      }
    }
  }
  return 0;
}

/* Rows [n0, n1) of the Q8-activation product: each weight block is decoded
 * once per row and applied to every token.  For each (m, n) the terms are
 * added in block order (kb, then group g), as the kernels order them. */
typedef struct {
  int dtype;
  const void* b;
  const int8_t* xq;
  const act_rec* xs;
  int64_t M, K, N, n0, n1;
  float *out, *bound, *mag_out;
  const float* a;
  int rc;
} q8_job;

static void* q8act_rows(void* arg) {
  q8_job* j = (q8_job*)arg;
  const int dtype = j->dtype;
  const int be = orc_block_elems(dtype), bb = orc_block_bytes(dtype);
  const int64_t M = j->M, K = j->K, N = j->N, nb = (K + be - 1) / be, Kp = (K + 255) / 256 * 256;
  const double u = 1.0 / 16777216.0;
  float* y = (float*)calloc((size_t)M + 1, sizeof(float));
  double* mag = (double*)calloc((size_t)M + 1, sizeof(double));
  double* act_err = (double*)calloc((size_t)M + 1, sizeof(double));
  if (!y || !mag || !act_err) {
    free(y); free(mag); free(act_err);
    j->rc = -3;
    return NULL;
  }
  wcodes c;
  for (int64_t n = j->n0; n < j->n1; ++n) {
    for (int64_t m = 0; m < M; ++m) { y[m] = 0.0f; mag[m] = 0.0; act_err[m] = 0.0; }
    int64_t terms = 0;
    for (int64_t kb = 0; kb < nb; ++kb) {
      block_codes(dtype, (const uint8_t*)j->b + (n * nb + kb) * bb, &c);
      for (int g = 0; g < c.ngroups; ++g) {
        const int64_t k0 = kb * be + (int64_t)g * c.gsize;
        const int64_t xb = k0 / 32;
        double dsum = 0.0; /* sum of |w| over the group, for the activation error */
        if (j->bound) {
          for (int l = 0; l < c.gsize && k0 + l < K; ++l) {
            double w = (double)c.A[g] * c.q[g * c.gsize + l] - (c.has_min ? (double)c.B[g] : 0.0);
            dsum += fabs(w);
          }
        }
        for (int64_t m = 0; m < M; ++m) {
          const act_rec* r = &j->xs[m * (Kp / 32) + xb];
          const int8_t* xm = j->xq + m * Kp + k0;
          int isum = 0, xsum = 0;
          for (int h0 = 0; h0 < c.gsize; h0 += 16) {
            /* The kernels convert each 16-value partial dot separately, so
             * the reordering magnitude is summed over 16-value halves. */
            int ih = 0, xh = 0;
            for (int l = h0; l < h0 + 16; ++l) {
              int xv = xm[l];
              ih += c.q[g * c.gsize + l] * xv;
              xh += xv;
            }
            isum += ih;
            xsum += xh;
            mag[m] += fabs((double)ih * c.A[g] * r->d) + (c.has_min ? fabs((double)xh * c.B[g] * r->d) : 0.0);
          }
          float t1 = (float)isum * (c.A[g] * r->d);
          float t2 = c.has_min ? (float)xsum * (c.B[g] * r->d) : 0.0f;
          y[m] += t1;
          y[m] -= t2;
          /* activation error: |x - q*d_x| <= 0.5*d32 + 127*|d32 - d16|
           * where d32 is the unrounded scale; bounded by 0.5625*d16. */
          if (j->bound) act_err[m] += 0.5625 * (double)r->d * dsum;
        }
        terms += 2;
      }
    }
    for (int64_t m = 0; m < M; ++m) {
      j->out[m * N + n] = y[m];
      if (j->mag_out) j->mag_out[m * N + n] = (float)mag[m];
      if (j->bound) j->bound[m * N + n] = (float)(act_err[m] + 2.0 * (double)(terms + 8) * u * mag[m] + 1e-30);
    }
  }
  free(y); free(mag); free(act_err);
  j->rc = 0;
  return NULL;
}

/* Run `fn` over nthreads row ranges of [0, N) (jobs: an array of job
 * structs of `size` bytes whose n0/n1 fields are filled in by `set`). */
static int run_rows(void* (*fn)(void*), void* jobs, size_t size, int nthreads, int64_t N,
                    void (*set)(void*, int64_t, int64_t), int (*rc_of)(void*)) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > N) nthreads = (int)(N > 0 ? N : 1);
  pthread_t th[256];
  for (int t = 0; t < nthreads; ++t) set((char*)jobs + t * size, N * t / nthreads, N * (t + 1) / nthreads);
  if (nthreads == 1) {
    fn(jobs);
  } else {
    for (int t = 0; t < nthreads; ++t) pthread_create(&th[t], NULL, fn, (char*)jobs + t * size);
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
  }
  for (int t = 0; t < nthreads; ++t)
    if (rc_of((char*)jobs + t * size)) return rc_of((char*)jobs + t * size);
  return 0;
}

static void q8_set(void* p, int64_t n0, int64_t n1) { ((q8_job*)p)->n0 = n0; ((q8_job*)p)->n1 = n1; }
static int q8_rc(void* p) { return ((q8_job*)p)->rc; }

int orc_matmul_q8act_mt(int dtype, float* out, const float* a, const void* b, int64_t M, int64_t K,
                        int64_t N, float* bound, float* mag_out, int nthreads) {
  if (!supported(dtype) || M < 0 || N < 0 || K < 0) return -1;
  int64_t Kp = (K + 255) / 256 * 256;
  int8_t* xq = (int8_t*)calloc((size_t)(M * Kp + 1), 1);
  act_rec* xs = (act_rec*)calloc((size_t)(M * (Kp / 32) + 1), sizeof(act_rec));
  if (!xq || !xs) {
    free(xq);
    free(xs);
    return -3;
  }
  orc_quantize_act_planes(a, M, K, xq, xs);
  q8_job jobs[256];
  for (int t = 0; t < 256; ++t)
    jobs[t] = (q8_job){dtype, b, xq, xs, M, K, N, 0, 0, out, bound, mag_out, a, 0};
  int rc = run_rows(q8act_rows, jobs, sizeof(q8_job), nthreads, N, q8_set, q8_rc);
  free(xq);
  free(xs);
  return rc;
}

int orc_matmul_q8act(int dtype, float* out, const float* a, const void* b, int64_t M, int64_t K,
                     int64_t N, float* bound, float* mag_out) {
  return orc_matmul_q8act_mt(dtype, out, a, b, M, K, N, bound, mag_out, 1);
}

typedef struct {
  int dtype;
  const float* a;
  const void* b;
  int64_t M, K, N, n0, n1;
  float* bound;
  int rc;
} b32_job;

/* Rows [n0, n1) of the fp32 reordering bound; each block decoded once per row. */
static void* fp32_bound_rows(void* arg) {
  b32_job* j = (b32_job*)arg;
  const int be = orc_block_elems(j->dtype), bb = orc_block_bytes(j->dtype);
  const int64_t M = j->M, K = j->K, N = j->N, nb = (K + be - 1) / be;
  const double u = 1.0 / 16777216.0;
  double* mag = (double*)calloc((size_t)M + 1, sizeof(double));
  if (!mag) {
    j->rc = -3;
    return NULL;
  }
  wcodes c;
  double w[256];
  for (int64_t n = j->n0; n < j->n1; ++n) {
    for (int64_t m = 0; m < M; ++m) mag[m] = 0.0;
    for (int64_t kb = 0; kb < nb; ++kb) {
      block_codes(j->dtype, (const uint8_t*)j->b + (n * nb + kb) * bb, &c);
      int ne = 0;
      for (int e = 0; e < be && kb * be + e < K; ++e, ++ne) {
        int g = e / c.gsize;
        w[e] = fabs((double)c.A[g] * c.q[e]) + (c.has_min ? fabs((double)c.B[g]) : 0.0);
      }
      for (int64_t m = 0; m < M; ++m) {
        const float* am = j->a + m * K + kb * be;
        double s = mag[m];
        for (int e = 0; e < ne; ++e) s += fabs((double)am[e]) * w[e];
        mag[m] = s;
      }
    }
    for (int64_t m = 0; m < M; ++m) j->bound[m * N + n] = (float)(2.0 * (double)(K + 16) * u * mag[m] + 1e-30);
  }
  free(mag);
  j->rc = 0;
  return NULL;
}

static void b32_set(void* p, int64_t n0, int64_t n1) { ((b32_job*)p)->n0 = n0; ((b32_job*)p)->n1 = n1; }
static int b32_rc(void* p) { return ((b32_job*)p)->rc; }

int orc_fp32_bound_mt(int dtype, const float* a, const void* b, int64_t M, int64_t K, int64_t N, float* bound,
                      int nthreads) {
  if (!supported(dtype) || M < 0 || N < 0 || K < 0) return -1;
  b32_job jobs[256];
  for (int t = 0; t < 256; ++t) jobs[t] = (b32_job){dtype, a, b, M, K, N, 0, 0, bound, 0};
  return run_rows(fp32_bound_rows, jobs, sizeof(b32_job), nthreads, N, b32_set, b32_rc);
}

int orc_fp32_bound(int dtype, const float* a, const void* b, int64_t M, int64_t K, int64_t N,
                   float* bound) {
  return orc_fp32_bound_mt(dtype, a, b, M, K, N, bound, 1);
}

/* ------------------------------------------------------------------------- */
/* Tiled device layout                                                        */
/*                                                                            */
/* Rows are grouped in tiles of 64, columns in spans of 256.  One unit =      */
/* (row tile g, span kb) = 64 row slices of S bytes, then a tail plane.       */
/* Units are stored g-major: offset = (g * KBu + kb) * unit_bytes.            */
/*   Q4_0 slice (144 B): d[8] fp16, then qs[8][16]                            */
/*   Q8_0 slice (272 B): d[8] fp16, then qs[8][32]                            */
/*   Q4_1 slice (176 B): d[8], m[8] fp16, qs[8][16], 16 B pad                 */
/*   Q5_0 slice (176 B): d[8] fp16, qh[8][4], qs[8][16]                       */
/*   Q5_1 slice (208 B): d[8], m[8] fp16, qh[8][4], qs[8][16], 16 B pad       */
/*   Q4_K slice (144 B): the GGUF block verbatim                              */
/*   Q5_K slice (176 B): the GGUF block verbatim                              */
/*   Q6_K slice (208 B): scales[16], ql[128], qh[64]; tail: d[64] fp16        */
/* Rows >= N and blocks past the row end are zero bytes.                      */
/* ------------------------------------------------------------------------- */

static int slice_bytes(int dtype) {
  switch (dtype) {
    case ORC_Q4_0: return 144;
    case ORC_Q8_0: return 272;
    case ORC_Q4_1: return 176;
    case ORC_Q5_0: return 176;
    case ORC_Q5_1: return 208;
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 208;
    default: return 0;
  }
}

int64_t orc_unit_bytes(int dtype) {
  if (!supported(dtype)) return -1;
  return (int64_t)slice_bytes(dtype) * ORC_UNIT_ROWS + (dtype == ORC_Q6_K ? 2 * ORC_UNIT_ROWS : 0);
}

int64_t orc_tiled_bytes(int dtype, int64_t N, int64_t K) {
  if (!supported(dtype) || N < 0 || K < 0) return -1;
  int64_t G = (N + ORC_UNIT_ROWS - 1) / ORC_UNIT_ROWS;
  int64_t KB = (K + ORC_UNIT_COLS - 1) / ORC_UNIT_COLS;
  return G * KB * orc_unit_bytes(dtype);
}

/* Copy one row slice between GGUF order (row n, span kb) and the tile.
 * dir = 0: gguf -> tile, dir = 1: tile -> gguf. */
static void move_slice(int dtype, uint8_t* row_gguf, int64_t nb_row, int64_t kb, uint8_t* slice,
                       uint8_t* tail_d, int dir) {
  int bb = orc_block_bytes(dtype);
  if (orc_block_elems(dtype) == 32) {
    /* fields [d][m][qh][qs] of each block, field-major over the 8 blocks:
     * {block offset, size, slice offset} */
    int has_m = dtype == ORC_Q4_1 || dtype == ORC_Q5_1, has_h = dtype == ORC_Q5_0 || dtype == ORC_Q5_1;
    int f[4][3], nf = 0;
    int boff = 2, soff = 16;
    f[nf][0] = 0, f[nf][1] = 2, f[nf][2] = 0, ++nf;
    if (has_m) f[nf][0] = boff, f[nf][1] = 2, f[nf][2] = soff, ++nf, boff += 2, soff += 16;
    if (has_h) f[nf][0] = boff, f[nf][1] = 4, f[nf][2] = soff, ++nf, boff += 4, soff += 32;
    f[nf][0] = boff, f[nf][1] = bb - boff, f[nf][2] = soff, ++nf;
    for (int j = 0; j < 8; ++j) {
      int64_t b = kb * 8 + j;
      if (b >= nb_row) break;
      uint8_t* blk = row_gguf + b * bb;
      for (int i = 0; i < nf; ++i) {
        uint8_t* sp = slice + f[i][2] + f[i][1] * j;
        if (dir == 0) memcpy(sp, blk + f[i][0], (size_t)f[i][1]);
        else memcpy(blk + f[i][0], sp, (size_t)f[i][1]);
      }
    }
    return;
  }
  uint8_t* blk = row_gguf + kb * bb;
  if (dtype == ORC_Q4_K || dtype == ORC_Q5_K) {
    if (dir == 0) memcpy(slice, blk, (size_t)bb);
    else memcpy(blk, slice, (size_t)bb);
    return;
  }
  /* Q6_K: gguf ql 0..127, qh 128..191, scales 192..207, d 208..209 */
  if (dir == 0) {
    memcpy(slice, blk + 192, 16);
    memcpy(slice + 16, blk, 128);
    memcpy(slice + 144, blk + 128, 64);
    memcpy(tail_d, blk + 208, 2);
  } else {
    memcpy(blk + 192, slice, 16);
    memcpy(blk, slice + 16, 128);
    memcpy(blk + 128, slice + 144, 64);
    memcpy(blk + 208, tail_d, 2);
  }
}

static int tile_walk(int dtype, uint8_t* gguf, uint8_t* tiled, int64_t N, int64_t K, int dir) {
  if (!supported(dtype) || N < 0 || K < 0) return -1;
  int be = orc_block_elems(dtype);
  if (be == 256 && K % 256) return -2;
  int64_t nb_row = (K + be - 1) / be;
  int64_t row_bytes = nb_row * orc_block_bytes(dtype);
  int64_t G = (N + 63) / 64, KB = (K + 255) / 256, ub = orc_unit_bytes(dtype);
  int sb = slice_bytes(dtype);
  if (dir == 0) memset(tiled, 0, (size_t)(G * KB * ub));
  for (int64_t g = 0; g < G; ++g) {
    for (int64_t kb = 0; kb < KB; ++kb) {
      uint8_t* unit = tiled + (g * KB + kb) * ub;
      for (int r = 0; r < 64; ++r) {
        int64_t n = g * 64 + r;
        if (n >= N) break;
        move_slice(dtype, gguf + n * row_bytes, nb_row, kb, unit + (int64_t)r * sb,
                   unit + 64 * (int64_t)sb + 2 * r, dir);
      }
    }
  }
  return 0;
}

int orc_repack(int dtype, const void* gguf, void* tiled, int64_t N, int64_t K) {
  return tile_walk(dtype, (uint8_t*)gguf, (uint8_t*)tiled, N, K, 0);
}

int orc_unpack(int dtype, const void* tiled, void* gguf, int64_t N, int64_t K) {
  return tile_walk(dtype, (uint8_t*)gguf, (uint8_t*)tiled, N, K, 1);
}
