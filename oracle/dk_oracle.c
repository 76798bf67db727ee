/*
 * dk_oracle.c -- CPU restatement of decode-kernel's W4A16 format and its
 * fp32 dequantize-then-matmul reference.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library; it is never linked into, called by, or used as a fallback for the
 * product path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline load it.
 *
 * What it restates (reference paths are inside RohanDisa/decode-kernel):
 *   dko_quantize_pack  <- python/decode_kernel/quantize.py:26-51
 *                         scale32 = max(amax/7, 1e-8) in fp32 (true IEEE
 *                         division, as torch does on CPU); q = round-half-even
 *                         (w / scale32) clamped to [-7, 7]; nibble = q & 0xF
 *                         at bit 4n of the word (low nibble first); stored
 *                         scale = fp16(scale32), round-to-nearest-even.
 *   dko_unpack_to_int  <- quantize.py:54-63 (sign-extend each nibble)
 *   dko_dequantize     <- quantize.py:66-78 (q * float(scale16) in fp32)
 *   dko_linear_fp32    <- python/decode_kernel/reference.py:17-26
 *                         y[b, m] = sum_k float(x16[b,k]) * w32[m,k].  The
 *                         products are formed in fp32 as in the reference;
 *                         the sum is carried in double so the oracle is at
 *                         least as accurate as the reference's fp32 BLAS.
 *
 * Parity is pinned against vectors produced by the reference package itself
 * (tests/golden/make_golden.py writes the fixtures in tests/golden): the quantizer must be
 * bit-exact, the linear output within 1e-4 absolute.
 *
 * Build: make -C oracle  (plain gcc, no -ffast-math: IEEE division and
 * round-half-even are part of the format).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define DKO_GROUP 128
#define DKO_NIBBLES 8
#define DKO_QMIN (-7)
#define DKO_QMAX 7

/* ---- IEEE binary16 <-> binary32, written from the format definitions ---- */

uint16_t dko_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFFu) { /* inf / nan */
    return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u));
  }
  const int e = (int)exp - 127 + 15; /* rebiased exponent */
  if (e >= 31) return (uint16_t)(sign | 0x7C00u); /* overflow -> inf */
  if (e <= 0) {
    /* subnormal half (or zero): value = man24 * 2^(exp-150), target unit
     * 2^-24, so shift right by (126 - exp) = 1 - e + 13 bits. */
    if (e < -10) return (uint16_t)sign; /* below half of min subnormal */
    man |= 0x800000u;                   /* implicit bit */
    const int shift = 14 - e;           /* in [14, 24] */
    uint32_t h = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h); /* carry into exponent is correct */
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u; /* may carry to inf */
  return (uint16_t)(sign | h);
}

float dko_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
  uint32_t man = (uint32_t)h & 0x3FFu;
  uint32_t x;
  if (exp == 0x1Fu) {
    x = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    x = sign | ((exp - 15u + 127u) << 23) | (man << 13);
  } else if (man == 0) {
    x = sign;
  } else { /* subnormal: normalise */
    int e = -1;
    do {
      man <<= 1;
      ++e;
    } while (!(man & 0x400u));
    x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* ---- format ---- */

/* Returns 0 on success, -1 on a shape the format rejects
 * (quantize.py:31-36: 2-D, K % 128 == 0, K % 8 == 0). */
int dko_quantize_pack(const float* w, int64_t M, int64_t K, int32_t* packed,
                      uint16_t* scales) {
  if (M < 0 || K <= 0 || K % DKO_GROUP != 0) return -1;
  const int64_t groups = K / DKO_GROUP;
  const int64_t words = K / DKO_NIBBLES;
  for (int64_t m = 0; m < M; ++m) {
    const float* row = w + m * K;
    uint32_t* prow = (uint32_t*)(packed + m * words);
    memset(prow, 0, (size_t)words * 4);
    for (int64_t g = 0; g < groups; ++g) {
      const float* grp = row + g * DKO_GROUP;
      float amax = 0.0f;
      int has_nan = 0;
      for (int i = 0; i < DKO_GROUP; ++i) {
        const float a = fabsf(grp[i]);
        if (isnan(a)) has_nan = 1;
        if (a > amax) amax = a;
      }
      float s = has_nan ? NAN : amax / (float)DKO_QMAX;
      if (s < 1e-8f) s = 1e-8f; /* clamp(min=1e-8); NaN passes through */
      scales[m * groups + g] = dko_f32_to_f16(s);
      for (int i = 0; i < DKO_GROUP; ++i) {
        float r = nearbyintf(grp[i] / s); /* round half to even */
        if (r < (float)DKO_QMIN) r = (float)DKO_QMIN;
        if (r > (float)DKO_QMAX) r = (float)DKO_QMAX;
        /* torch casts NaN to int32 as INT_MIN; its low nibble is 0. */
        const int32_t q = isnan(r) ? 0 : (int32_t)r;
        const int64_t k = g * DKO_GROUP + i;
        prow[k / DKO_NIBBLES] |= ((uint32_t)q & 0xFu) << (4 * (k % DKO_NIBBLES));
      }
    }
  }
  return 0;
}

void dko_unpack_to_int(const int32_t* packed, int64_t M, int64_t K, int8_t* q) {
  const int64_t words = K / DKO_NIBBLES;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t j = 0; j < words; ++j) {
      const uint32_t wd = (uint32_t)packed[m * words + j];
      for (int n = 0; n < DKO_NIBBLES; ++n) {
        const int v = (int)((wd >> (4 * n)) & 0xFu);
        q[m * K + j * DKO_NIBBLES + n] = (int8_t)(v >= 8 ? v - 16 : v);
      }
    }
  }
}

void dko_dequantize(const int32_t* packed, const uint16_t* scales, int64_t M,
                    int64_t K, float* w) {
  const int64_t words = K / DKO_NIBBLES;
  const int64_t groups = K / DKO_GROUP;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t j = 0; j < words; ++j) {
      const uint32_t wd = (uint32_t)packed[m * words + j];
      const int64_t k0 = j * DKO_NIBBLES;
      const float s = dko_f16_to_f32(scales[m * groups + k0 / DKO_GROUP]);
      for (int n = 0; n < DKO_NIBBLES; ++n) {
        const int v = (int)((wd >> (4 * n)) & 0xFu);
        w[m * K + k0 + n] = (float)(v >= 8 ? v - 16 : v) * s;
      }
    }
  }
}

/* y[B, M] fp32 = x[B, K] (fp16 bits) . dequant(W)[M, K]^T.
 * Rows [m0, m1) only, so callers can check a sample of a large matrix. */
void dko_linear_fp32_rows(const uint16_t* x, const int32_t* packed,
                          const uint16_t* scales, int64_t M, int64_t K,
                          int64_t B, int64_t m0, int64_t m1, float* y) {
  const int64_t words = K / DKO_NIBBLES;
  const int64_t groups = K / DKO_GROUP;
  (void)M;
  for (int64_t m = m0; m < m1; ++m) {
    for (int64_t b = 0; b < B; ++b) {
      const uint16_t* xb = x + b * K;
      double acc = 0.0;
      for (int64_t j = 0; j < words; ++j) {
        const uint32_t wd = (uint32_t)packed[m * words + j];
        const int64_t k0 = j * DKO_NIBBLES;
        const float s = dko_f16_to_f32(scales[m * groups + k0 / DKO_GROUP]);
        for (int n = 0; n < DKO_NIBBLES; ++n) {
          const int v = (int)((wd >> (4 * n)) & 0xFu);
          const float wv = (float)(v >= 8 ? v - 16 : v) * s;
          acc += (double)(wv * dko_f16_to_f32(xb[k0 + n]));
        }
      }
      y[b * M + m] = (float)acc;
    }
  }
}

void dko_linear_fp32(const uint16_t* x, const int32_t* packed,
                     const uint16_t* scales, int64_t M, int64_t K, int64_t B,
                     float* y) {
  dko_linear_fp32_rows(x, packed, scales, M, K, B, 0, M, y);
}
