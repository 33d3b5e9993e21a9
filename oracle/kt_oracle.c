/*
 * kt_oracle.c — CPU restatement of the reference's GGUF hot-expert MoE arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product links or calls this file: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg
 * load it, as the checker and as the timed CPU baseline.
 *
 * What it restates (paths relative to the reference project root):
 *   - GGUF block layouts and dequantization for Q8_0, Q4_K, Q6_K, IQ3_S
 *     (hot/kt_gguf_moe_multi/ggml-common.h:55-69, 88-94, 105-112, 145-154; ggml's
 *     dequantize_row_* order, which gguf-py 0.19.0 follows as well), and for the 32-value
 *     blocks Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL of the GEMV's wider type switch.
 *   - vec_dot_q4_0/q4_1/q5_0/q5_1_q8_1 (vecdotq.cuh:48-160 and their wrappers, 637-650,
 *     729-745, 850-865) and vec_dot_iq4_nl_q8_1 (vecdotq.cuh:1995-2015): chunk = 2 ints of
 *     nibbles (8 low + 8 high codes), the Q4_1 / Q5_1 products d*d8 and m*s8 rounded to
 *     half precision as the reference's __hmul2 does.
 *   - the K-quants Q2_K, Q3_K, Q5_K and IQ4_XS (ggml-common.h block_q2_K / q3_K / q5_K /
 *     iq4_xs; ggml's dequantize_row order): vec_dot_q2_K_q8_1 (vecdotq.cuh:211-241,
 *     1057-1076), vec_dot_q3_K_q8_1 (282-317, 1175-1198), vec_dot_q5_K_q8_1 (413-445,
 *     1467-1509), vec_dot_iq4_xs_q8_1 (2019-2040); and the reference's own Q2_0 block and
 *     vec_dot_q2_0_q8_1 (kt_gguf_moe_multi.cu:33-64).
 *   - the i-quants with a code book, IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ1_S / IQ1_M:
 *     ggml's dequantize_row order and vec_dot_*_q8_1 (vecdotq.cuh:1755-1977); code books
 *     from iquant_grids.h.
 *   - the q8_1 activation quantizer quantize_q8_1 (hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu:600-650),
 *     including the lane order of its 32-lane butterfly sum that produces ds.y.
 *   - the per-chunk integer dot products vec_dot_q8_0_q8_1 (vecdotq.cuh:969-982),
 *     vec_dot_q4_K_q8_1 (vecdotq.cuh:1326-1367, 349-376), vec_dot_q6_K_q8_1
 *     (vecdotq.cuh:1625-1646, 485-507), vec_dot_iq3_s_q8_1 (vecdotq.cuh:1875-1900).
 *   - the GEMV reduction of moe_vec_q_rows (kt_gguf_moe_multi.cu:74-130): lane t of a
 *     warp accumulates chunks t, t+32, ... of a row in order, then an xor butterfly
 *     (16, 8, 4, 2, 1) whose lane-0 value is the row's result; ids < 0 give zero rows
 *     (kt_gguf_moe_multi.cu:151-162).
 *   - silu_and_mul + the fused combine of KTGGUFHotExpertsMethod.apply
 *     (hot/kt_gguf_hot.py:43-71, 240-304).
 *   - an fp32 dequant-then-matmul oracle (the pattern of the streamer's
 *     _reference_check) with double accumulation.
 *
 * Parity status: integer parts (q8_1 bytes, dp4a sums, dequantized values) are exact.
 * The fp32 combination follows the reference's expression order without FMA
 * contraction; where the reference build contracts a multiply-add the fp32 results can
 * differ in the last bit, which the tests bound explicitly.
 *
 * Built by oracle/Makefile with -ffp-contract=off and OpenMP.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include "../kt-prefill-lend_b200/csrc/iq3s_grid.h"
#include "../kt-prefill-lend_b200/csrc/iquant_grids.h"

#define KO_Q4_0 2
#define KO_Q4_1 3
#define KO_Q5_0 6
#define KO_Q5_1 7
#define KO_IQ4_NL 20
#define KO_Q8_0 8
#define KO_Q4_K 12
#define KO_Q6_K 14
#define KO_IQ3_S 21
#define KO_Q2_K 10
#define KO_Q3_K 11
#define KO_Q5_K 13
#define KO_IQ4_XS 23
#define KO_Q2_0 42
#define KO_IQ2_XXS 16
#define KO_IQ2_XS 17
#define KO_IQ3_XXS 18
#define KO_IQ1_S 19
#define KO_IQ2_S 22
#define KO_IQ1_M 29
#define KO_IQ1_DELTA 0.125f

/* ---------------------------------------------------------------- numbers */

static float ko_h2f(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023, u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else { /* subnormal: normalise */
      int sh = 0;
      while (!(m & 1024)) { m <<= 1; ++sh; }
      m &= 1023;
      u = s | ((uint32_t)(113 - sh) << 23) | (m << 13);
    }
  } else if (e == 31) {
    u = s | 0x7f800000u | (m << 13);
  } else {
    u = s | ((e + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t ko_f2h(float f) { /* round to nearest even, like __float2half */
  _Float16 h = (_Float16)f;
  uint16_t r;
  memcpy(&r, &h, 2);
  return r;
}

static float ko_bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t ko_f2bf(float f) { /* round to nearest even, like __float2bfloat16 */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float ko_round_bf(float f) { return ko_bf2f(ko_f2bf(f)); }

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static int32_t rd32(const uint8_t* p) {
  return (int32_t)((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24));
}

/* __dp4a(a, b, c) with signed bytes */
static int32_t dp4a(int32_t a, int32_t b, int32_t c) {
  for (int i = 0; i < 4; ++i) c += (int32_t)(int8_t)(a >> (8 * i)) * (int32_t)(int8_t)(b >> (8 * i));
  return c;
}

int ko_block_info(int type, int* blck, int* bytes) {
  switch (type) {
    case KO_Q8_0: *blck = 32; *bytes = 34; return 0;
    case KO_Q4_K: *blck = 256; *bytes = 144; return 0;
    case KO_Q6_K: *blck = 256; *bytes = 210; return 0;
    case KO_IQ3_S: *blck = 256; *bytes = 110; return 0;
    case KO_Q4_0: *blck = 32; *bytes = 18; return 0;
    case KO_Q4_1: *blck = 32; *bytes = 20; return 0;
    case KO_Q5_0: *blck = 32; *bytes = 22; return 0;
    case KO_Q5_1: *blck = 32; *bytes = 24; return 0;
    case KO_IQ4_NL: *blck = 32; *bytes = 18; return 0;
    case KO_Q2_K: *blck = 256; *bytes = 84; return 0;
    case KO_Q3_K: *blck = 256; *bytes = 110; return 0;
    case KO_Q5_K: *blck = 256; *bytes = 176; return 0;
    case KO_IQ4_XS: *blck = 256; *bytes = 136; return 0;
    case KO_Q2_0: *blck = 64; *bytes = 18; return 0;
    case KO_IQ2_XXS: *blck = 256; *bytes = 66; return 0;
    case KO_IQ2_XS: *blck = 256; *bytes = 74; return 0;
    case KO_IQ3_XXS: *blck = 256; *bytes = 98; return 0;
    case KO_IQ1_S: *blck = 256; *bytes = 50; return 0;
    case KO_IQ2_S: *blck = 256; *bytes = 82; return 0;
    case KO_IQ1_M: *blck = 256; *bytes = 56; return 0;
    default: return -1;
  }
}

/* the IQ4_NL code book (ggml-common.h kvalues_iq4nl) */
static const int8_t ko_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* ---------------------------------------------------------------- dequant */

/* ggml get_scale_min_k4: 6-bit scale and min of sub-block j of a Q4_K block */
static void q4k_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

static void dq_q8_0(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
}

static void dq_q4_k(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b)), dmin = ko_h2f(rd16(b + 2));
  const uint8_t* scales = b + 4;
  const uint8_t* q = b + 16;
  int is = 0;
  for (int j = 0; j < 256; j += 64) {
    uint8_t sc, m;
    q4k_scale_min(is + 0, scales, &sc, &m);
    float d1 = d * sc, m1 = dmin * m;
    q4k_scale_min(is + 1, scales, &sc, &m);
    float d2 = d * sc, m2 = dmin * m;
    for (int l = 0; l < 32; ++l) *y++ = d1 * (float)(q[l] & 0xF) - m1;
    for (int l = 0; l < 32; ++l) *y++ = d2 * (float)(q[l] >> 4) - m2;
    q += 32;
    is += 2;
  }
}

/* Q2_K: scales[16] (low nibble scale, high nibble min), qs[64], d, dmin; 128-value halves,
 * four 2-bit planes each, 16 values per scale */
static void dq_q2_k(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b + 80)), dmin = ko_h2f(rd16(b + 82));
  const uint8_t* q = b + 16;
  int is = 0;
  for (int n = 0; n < 256; n += 128) {
    for (int shift = 0; shift < 8; shift += 2) {
      for (int h = 0; h < 2; ++h) {
        uint8_t sc = b[is++];
        float dl = d * (float)(sc & 0xF), ml = dmin * (float)(sc >> 4);
        for (int l = 0; l < 16; ++l) *y++ = dl * (float)((q[16 * h + l] >> shift) & 3) - ml;
      }
    }
    q += 32;
  }
}

/* Q3_K scale i (0..15): 4 low bits from byte i%8 (nibble i/8), 2 high bits from byte 8+i%4
 * (pair i/4), minus 32 */
static int q3k_scale(const uint8_t* s, int i) {
  return (((s[i % 8] >> (4 * (i / 8))) & 0xF) | (((s[8 + i % 4] >> (2 * (i / 4))) & 3) << 4)) - 32;
}

/* Q3_K: hmask[32], qs[64], scales[12], d; as Q2_K's planes, the hmask bit (clear: -4) */
static void dq_q3_k(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b + 108));
  const uint8_t* q = b + 32;
  const uint8_t* hm = b;
  int is = 0;
  uint8_t m = 1;
  for (int n = 0; n < 256; n += 128) {
    for (int shift = 0; shift < 8; shift += 2) {
      for (int h = 0; h < 2; ++h) {
        float dl = d * (float)q3k_scale(b + 96, is++);
        for (int l = 0; l < 16; ++l)
          *y++ = dl * (float)(((q[16 * h + l] >> shift) & 3) - ((hm[16 * h + l] & m) ? 0 : 4));
      }
      m <<= 1;
    }
    q += 32;
  }
}

/* Q5_K: d, dmin, Q4_K's 12-byte scales, qh[32], qs[128]; fifth bit from qh, planes 2j / 2j+1 */
static void dq_q5_k(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b)), dmin = ko_h2f(rd16(b + 2));
  const uint8_t* ql = b + 48;
  const uint8_t* qh = b + 16;
  int is = 0;
  uint8_t u1 = 1, u2 = 2;
  for (int j = 0; j < 256; j += 64) {
    uint8_t sc, m;
    q4k_scale_min(is + 0, b + 4, &sc, &m);
    float d1 = d * sc, m1 = dmin * m;
    q4k_scale_min(is + 1, b + 4, &sc, &m);
    float d2 = d * sc, m2 = dmin * m;
    for (int l = 0; l < 32; ++l) *y++ = d1 * (float)((ql[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
    for (int l = 0; l < 32; ++l) *y++ = d2 * (float)((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
    ql += 32;
    is += 2;
    u1 <<= 2;
    u2 <<= 2;
  }
}

/* IQ4_XS: d, scales_h (2 bits per sub-block), scales_l[4] (4 bits), qs[128]; IQ4_NL levels */
static void dq_iq4_xs(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  uint16_t scales_h = rd16(b + 2);
  const uint8_t* qs = b + 8;
  for (int ib = 0; ib < 8; ++ib) {
    int ls = ((b[4 + ib / 2] >> (4 * (ib % 2))) & 0xf) | (((scales_h >> (2 * ib)) & 3) << 4);
    float dl = d * (float)(ls - 32);
    for (int j = 0; j < 16; ++j) {
      y[j] = dl * (float)ko_iq4nl[qs[j] & 0xf];
      y[j + 16] = dl * (float)ko_iq4nl[qs[j] >> 4];
    }
    y += 32;
    qs += 16;
  }
}

/* Q2_0 (kt_gguf_moe_multi.cu:33-46): fp16 d, qs[16]; element 4j+s = code s of byte j
 * (bits 2s); value (code - 1) * d */
static void dq_q2_0(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int e = 0; e < 64; ++e) y[e] = (float)(((b[2 + e / 4] >> (2 * (e % 4))) & 3) - 1) * d;
}

/* ---- i-quants with a code book (ggml's dequantize_row_iq2_xxs / iq2_xs / iq2_s / iq3_xxs /
 * iq1_s / iq1_m order, which gguf-py restates). Code books: iquant_grids.h (byte j of an
 * IQ2 entry e is byte j%4 of word 2e + j/4; IQ3_XXS entries are one word; IQ1 entries hold
 * v + 1 in nibbles, element j<4 in the low nibble of byte j, j>=4 in the high nibble of
 * byte j-4). Sign bytes: 7 stored bits + an even-parity eighth (ksigns_iq2xs). */
static uint32_t ko_signs8(uint32_t s7) {
  uint32_t p = 0;
  for (int i = 0; i < 7; ++i) p ^= (s7 >> i) & 1u;
  return s7 | (p << 7);
}
static int ko_iq2_mag(const uint32_t* grid, int entry, int j) { return (int)((grid[2 * entry + j / 4] >> (8 * (j % 4))) & 0xffu); }
static int ko_iq1_val(int entry, int j) {
  return (int)((kt_iq1s_grid_host[entry] >> (8 * (j % 4) + 4 * (j / 4))) & 0xfu) - 1;
}
static uint32_t rd32u(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }

static void dq_iq2_xxs(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int ib = 0; ib < 8; ++ib) {
    const uint8_t* q2 = b + 2 + 8 * ib;
    uint32_t aux = rd32u(q2 + 4);
    float db = d * (0.5f + (float)(aux >> 28)) * 0.25f;
    for (int l = 0; l < 4; ++l) {
      uint32_t s = ko_signs8((aux >> (7 * l)) & 127u);
      for (int j = 0; j < 8; ++j) *y++ = db * (float)ko_iq2_mag(kt_iq2xxs_grid_host, q2[l], j) * ((s >> j) & 1 ? -1.0f : 1.0f);
    }
  }
}
static void dq_iq2_xs(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int ib = 0; ib < 8; ++ib) {
    const uint8_t* q2 = b + 2 + 8 * ib;
    float db[2] = {d * (0.5f + (float)(b[66 + ib] & 0xf)) * 0.25f, d * (0.5f + (float)(b[66 + ib] >> 4)) * 0.25f};
    for (int l = 0; l < 4; ++l) {
      uint32_t code = rd16(q2 + 2 * l), s = ko_signs8(code >> 9);
      for (int j = 0; j < 8; ++j)
        *y++ = db[l / 2] * (float)ko_iq2_mag(kt_iq2xs_grid_host, (int)(code & 511u), j) * ((s >> j) & 1 ? -1.0f : 1.0f);
    }
  }
}
static void dq_iq2_s(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int ib = 0; ib < 8; ++ib) {
    float db[2] = {d * (0.5f + (float)(b[74 + ib] & 0xf)) * 0.25f, d * (0.5f + (float)(b[74 + ib] >> 4)) * 0.25f};
    for (int l = 0; l < 4; ++l) {
      int idx = b[2 + 4 * ib + l] | ((b[66 + ib] << (8 - 2 * l)) & 0x300);
      uint32_t s = b[34 + 4 * ib + l];
      for (int j = 0; j < 8; ++j)
        *y++ = db[l / 2] * (float)ko_iq2_mag(kt_iq2s_grid_host, idx, j) * ((s >> j) & 1 ? -1.0f : 1.0f);
    }
  }
}
static void dq_iq3_xxs(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int ib = 0; ib < 8; ++ib) {
    const uint8_t* q3 = b + 2 + 8 * ib;
    uint32_t aux = rd32u(b + 66 + 4 * ib);
    float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
    for (int l = 0; l < 4; ++l) {
      uint32_t s = ko_signs8((aux >> (7 * l)) & 127u);
      for (int j = 0; j < 8; ++j) {
        int mag = (int)((kt_iq3xxs_grid_host[q3[2 * l + j / 4]] >> (8 * (j % 4))) & 0xffu);
        *y++ = db * (float)mag * ((s >> j) & 1 ? -1.0f : 1.0f);
      }
    }
  }
}
static void dq_iq1_s(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  for (int ib = 0; ib < 8; ++ib) {
    int qh = rd16(b + 34 + 2 * ib);
    float dl = d * (float)(2 * ((qh >> 12) & 7) + 1);
    float delta = (qh & 0x8000) ? -KO_IQ1_DELTA : KO_IQ1_DELTA;
    for (int l = 0; l < 4; ++l) {
      int e = b[2 + 4 * ib + l] | (((qh >> (3 * l)) & 7) << 8);
      for (int j = 0; j < 8; ++j) *y++ = dl * ((float)ko_iq1_val(e, j) + delta);
    }
  }
}
static void dq_iq1_m(const uint8_t* b, float* y) {
  uint16_t sc[4];
  for (int k = 0; k < 4; ++k) sc[k] = rd16(b + 48 + 2 * k);
  float d = ko_h2f((uint16_t)((sc[0] >> 12) | ((sc[1] >> 8) & 0x00F0) | ((sc[2] >> 4) & 0x0F00) | (sc[3] & 0xF000)));
  for (int ib = 0; ib < 8; ++ib) {
    int tmp = sc[ib / 2] >> (6 * (ib % 2));
    float dl[2] = {d * (float)(2 * (tmp & 7) + 1), d * (float)(2 * ((tmp >> 3) & 7) + 1)};
    for (int l = 0; l < 4; ++l) {
      int qhl = b[32 + 2 * ib + l / 2] >> (4 * (l % 2));
      int e = b[4 * ib + l] | ((qhl & 7) << 8);
      float delta = (qhl & 8) ? -KO_IQ1_DELTA : KO_IQ1_DELTA;
      for (int j = 0; j < 8; ++j) *y++ = dl[l / 2] * ((float)ko_iq1_val(e, j) + delta);
    }
  }
}

static void dq_q6_k(const uint8_t* b, float* y) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = (const int8_t*)(b + 192);
  float d = ko_h2f(rd16(b + 208));
  for (int n = 0; n < 256; n += 128) {
    for (int l = 0; l < 32; ++l) {
      int is = l / 16;
      int q1 = (int)((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
      int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
      int q3 = (int)((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      y[l + 0] = d * (float)sc[is + 0] * (float)q1;
      y[l + 32] = d * (float)sc[is + 2] * (float)q2;
      y[l + 64] = d * (float)sc[is + 4] * (float)q3;
      y[l + 96] = d * (float)sc[is + 6] * (float)q4;
    }
    y += 128;
    ql += 64;
    qh += 32;
    sc += 8;
  }
}

static void dq_iq3_s(const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  const uint8_t* qs = b + 2;
  const uint8_t* qh = b + 66;
  const uint8_t* signs = b + 74;
  const uint8_t* scales = b + 106;
  for (int ib32 = 0; ib32 < 8; ib32 += 2) {
    float db1 = d * (float)(1 + 2 * (scales[ib32 / 2] & 0xf));
    float db2 = d * (float)(1 + 2 * (scales[ib32 / 2] >> 4));
    for (int half = 0; half < 2; ++half) {
      float db = half ? db2 : db1;
      for (int l = 0; l < 4; ++l) {
        uint32_t g1 = kt_iq3s_grid_host[qs[2 * l + 0] | ((qh[half] << (8 - 2 * l)) & 256)];
        uint32_t g2 = kt_iq3s_grid_host[qs[2 * l + 1] | ((qh[half] << (7 - 2 * l)) & 256)];
        for (int j = 0; j < 4; ++j) {
          float v1 = db * (float)((g1 >> (8 * j)) & 0xff);
          float v2 = db * (float)((g2 >> (8 * j)) & 0xff);
          y[j + 0] = (signs[l] & (1u << j)) ? -v1 : v1;
          y[j + 4] = (signs[l] & (1u << (j + 4))) ? -v2 : v2;
        }
        y += 8;
      }
      qs += 8;
      signs += 4;
    }
    qh += 2;
  }
}

/* 32-value blocks: code j < 16 is the low nibble of qs[j], j >= 16 the high nibble of
 * qs[j - 16]; Q5 adds bit j of qh as the fifth bit. ggml: (q-8)*d, q*d+m, (q-16)*d, q*d+m,
 * level(q)*d */
static void dq_legacy(int type, const uint8_t* b, float* y) {
  float d = ko_h2f(rd16(b));
  float m = (type == KO_Q4_1 || type == KO_Q5_1) ? ko_h2f(rd16(b + 2)) : 0.0f;
  int qs_off = (type == KO_Q4_0 || type == KO_IQ4_NL) ? 2 : type == KO_Q4_1 ? 4 : type == KO_Q5_0 ? 6 : 8;
  uint32_t qh = type == KO_Q5_0 ? (uint32_t)rd32(b + 2) : type == KO_Q5_1 ? (uint32_t)rd32(b + 4) : 0u;
  for (int j = 0; j < 32; ++j) {
    int nib = (b[qs_off + (j & 15)] >> (j < 16 ? 0 : 4)) & 0xF;
    int q = nib | (int)(((qh >> j) & 1) << 4);
    switch (type) {
      case KO_Q4_0: y[j] = (float)(nib - 8) * d; break;
      case KO_Q4_1: case KO_Q5_1: y[j] = (float)q * d + m; break;
      case KO_Q5_0: y[j] = (float)(q - 16) * d; break;
      case KO_IQ4_NL: y[j] = (float)ko_iq4nl[nib] * d; break;
    }
  }
}

int ko_dequant_rows(int type, const uint8_t* w, int64_t nrows, int64_t cols, float* out) {
  int blck, bs;
  if (ko_block_info(type, &blck, &bs) || cols % blck) return -1;
  int64_t nb = cols / blck;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < nrows; ++r) {
    for (int64_t i = 0; i < nb; ++i) {
      const uint8_t* b = w + (r * nb + i) * bs;
      float* y = out + r * cols + i * blck;
      switch (type) {
        case KO_Q8_0: dq_q8_0(b, y); break;
        case KO_Q4_K: dq_q4_k(b, y); break;
        case KO_Q6_K: dq_q6_k(b, y); break;
        case KO_IQ3_S: dq_iq3_s(b, y); break;
        case KO_Q2_K: dq_q2_k(b, y); break;
        case KO_Q3_K: dq_q3_k(b, y); break;
        case KO_Q5_K: dq_q5_k(b, y); break;
        case KO_IQ4_XS: dq_iq4_xs(b, y); break;
        case KO_Q2_0: dq_q2_0(b, y); break;
        case KO_IQ2_XXS: dq_iq2_xxs(b, y); break;
        case KO_IQ2_XS: dq_iq2_xs(b, y); break;
        case KO_IQ2_S: dq_iq2_s(b, y); break;
        case KO_IQ3_XXS: dq_iq3_xxs(b, y); break;
        case KO_IQ1_S: dq_iq1_s(b, y); break;
        case KO_IQ1_M: dq_iq1_m(b, y); break;
        default: dq_legacy(type, b, y); break;
      }
    }
  }
  return 0;
}

/* ---------------------------------------------------------------- q8_1 */

int64_t ko_q8_1_row_bytes(int64_t cols) { return (cols + 511) / 512 * 512 / 32 * 36; }

/* One row: blocks of 36 bytes (half d, half s, 32 x int8), zero-padded to a multiple of 512. */
static void q8_1_row(const float* x, int64_t cols, uint8_t* y) {
  int64_t kpad = (cols + 511) / 512 * 512;
  for (int64_t ib = 0; ib < kpad / 32; ++ib) {
    float v[32], s[32], amax = 0.0f;
    for (int t = 0; t < 32; ++t) {
      int64_t ix = ib * 32 + t;
      v[t] = ix < cols ? x[ix] : 0.0f;
      s[t] = v[t];
      amax = fmaxf(amax, fabsf(v[t]));
    }
    /* lane-0 value of the xor butterfly: each step adds the partner's partial sum */
    for (int mask = 16; mask > 0; mask >>= 1) {
      float n[32];
      for (int t = 0; t < 32; ++t) n[t] = s[t] + s[t ^ mask];
      memcpy(s, n, sizeof n);
    }
    float d = amax / 127;
    uint8_t* blk = y + ib * 36;
    for (int t = 0; t < 32; ++t) blk[4 + t] = (uint8_t)(int8_t)(amax == 0.0f ? 0 : (int)roundf(v[t] / d));
    uint16_t hd = ko_f2h(d), hs = ko_f2h(s[0]);
    blk[0] = hd & 0xff; blk[1] = hd >> 8;
    blk[2] = hs & 0xff; blk[3] = hs >> 8;
  }
}

int ko_quantize_q8_1(const float* x, int64_t rows, int64_t cols, uint8_t* qx) {
  int64_t rb = ko_q8_1_row_bytes(cols);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) q8_1_row(x + r * cols, cols, qx + r * rb);
  return 0;
}

/* ---------------------------------------------------------------- per-chunk dot products */

static float q8_1_d(const uint8_t* blk) { return ko_h2f(rd16(blk)); }

/* vec_dot_q8_0_q8_1: chunk = 8 values, iqs in {0, 2, 4, 6} */
static float vd_q8_0(const uint8_t* bx, const uint8_t* by, int iqs) {
  int32_t sumi = 0;
  for (int i = 0; i < 2; ++i) sumi = dp4a(rd32(bx + 2 + 4 * (iqs + i)), rd32(by + 4 + 4 * (iqs + i)), sumi);
  float d80 = ko_h2f(rd16(bx)), d81 = q8_1_d(by);
  return d80 * d81 * (float)sumi;
}

/* vec_dot_q4_K_q8_1: chunk = 16 values from two sub-blocks, iqs in {0, 2, ..., 30} */
static float vd_q4_k(const uint8_t* bx, const uint8_t* by0, int iqs) {
  const int bq8_offset = 2 * ((iqs / 2) / 4);
  const uint8_t* q4 = bx + 16 + 16 * bq8_offset + 4 * ((iqs / 2) % 4);
  uint32_t v0 = (uint32_t)rd32(q4), v1 = (uint32_t)rd32(q4 + 16);
  const uint8_t* s = bx + 4;
  uint16_t s16[6];
  for (int i = 0; i < 6; ++i) s16[i] = rd16(s + 2 * i);
  uint16_t aux0, aux1;
  const int j = bq8_offset / 2;
  if (j < 2) {
    aux0 = s16[j + 0] & 0x3f3f;
    aux1 = s16[j + 2] & 0x3f3f;
  } else {
    aux0 = (uint16_t)(((s16[j + 2] >> 0) & 0x0f0f) | ((s16[j - 2] & 0xc0c0) >> 2));
    aux1 = (uint16_t)(((s16[j + 2] >> 4) & 0x0f0f) | ((s16[j - 0] & 0xc0c0) >> 2));
  }
  uint8_t sc[2] = {(uint8_t)(aux0 & 0xff), (uint8_t)(aux0 >> 8)};
  uint8_t m[2] = {(uint8_t)(aux1 & 0xff), (uint8_t)(aux1 >> 8)};
  float sumf_d = 0.0f, sumf_m = 0.0f;
  for (int i = 0; i < 2; ++i) {
    const uint8_t* b8 = by0 + 36 * (bq8_offset + i);
    float d8 = q8_1_d(b8);
    int32_t u0 = rd32(b8 + 4 + 4 * ((iqs / 2) % 4)), u1 = rd32(b8 + 4 + 4 * ((iqs / 2) % 4) + 16);
    int32_t v0i = (int32_t)((v0 >> (4 * i)) & 0x0F0F0F0Fu), v1i = (int32_t)((v1 >> (4 * i)) & 0x0F0F0F0Fu);
    int32_t dot1 = dp4a(v1i, u1, dp4a(v0i, u0, 0));
    int32_t dot2 = dp4a(0x01010101, u1, dp4a(0x01010101, u0, 0));
    sumf_d += d8 * (float)(dot1 * sc[i]);
    sumf_m += d8 * (float)(dot2 * m[i]);
  }
  float dmx = ko_h2f(rd16(bx)), dmy = ko_h2f(rd16(bx + 2));
  return dmx * sumf_d - dmy * sumf_m;
}

/* vec_dot_q6_K_q8_1: chunk = 8 values, iqs in 0..31 */
static float vd_q6_k(const uint8_t* bx, const uint8_t* by0, int iqs) {
  const int bq8_offset = 4 * (iqs / 16) + (iqs % 16) / 8;
  const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
  const int vh_shift = 2 * ((iqs % 16) / 8);
  uint32_t vl = (uint32_t)rd32(bx + 4 * iqs);
  uint32_t vh = (uint32_t)rd32(bx + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift;
  const int8_t* scales = (const int8_t*)(bx + 192 + scale_offset);
  float sumf = 0.0f;
  for (int i = 0; i < 2; ++i) {
    const uint8_t* b8 = by0 + 36 * (bq8_offset + 2 * i);
    int32_t u = rd32(b8 + 4 + 4 * (iqs % 8));
    float d8 = q8_1_d(b8);
    int sc = scales[4 * i];
    uint32_t vil = (vl >> (4 * i)) & 0x0F0F0F0Fu;
    uint32_t vih = ((vh >> (4 * i)) << 4) & 0x30303030u;
    uint32_t x = vil | vih, vi = 0;
    for (int k = 0; k < 4; ++k) vi |= (uint32_t)(uint8_t)((int)((x >> (8 * k)) & 0xff) - 32) << (8 * k);
    sumf += d8 * (float)(dp4a((int32_t)vi, u, 0) * sc);
  }
  return ko_h2f(rd16(bx + 208)) * sumf;
}

/* vec_dot_iq3_s_q8_1: chunk = one 32-value sub-block, iqs = ib32 in 0..7 */
static float vd_iq3_s(const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* qs = bx + 2 + 8 * ib32;
  const uint8_t qh = bx[66 + ib32];
  const uint8_t* signs = bx + 74 + 4 * ib32;
  const uint8_t* b8 = by0 + 36 * ib32;
  const uint8_t* q8 = b8 + 4;
  int32_t sumi = 0;
  for (int l = 0; l < 4; ++l) {
    uint32_t g1 = kt_iq3s_grid_host[qs[2 * l + 0] | ((qh << (8 - 2 * l)) & 256)];
    uint32_t g2 = kt_iq3s_grid_host[qs[2 * l + 1] | ((qh << (7 - 2 * l)) & 256)];
    uint32_t gl = 0, gh = 0;
    for (int j = 0; j < 4; ++j) {
      int a = (int)((g1 >> (8 * j)) & 0xff), b = (int)((g2 >> (8 * j)) & 0xff);
      if (signs[l] & (1u << j)) a = -a;
      if (signs[l] & (1u << (j + 4))) b = -b;
      gl |= (uint32_t)(uint8_t)a << (8 * j);
      gh |= (uint32_t)(uint8_t)b << (8 * j);
    }
    sumi = dp4a((int32_t)gl, rd32(q8 + 0), sumi);
    sumi = dp4a((int32_t)gh, rd32(q8 + 4), sumi);
    q8 += 8;
  }
  const float d = ko_h2f(rd16(bx)) * (float)(1 + 2 * ((bx[106 + ib32 / 2] >> 4 * (ib32 % 2)) & 0xf)) * q8_1_d(b8);
  return d * (float)sumi;
}

/* legacy blocks, chunk iqs in {0, 2}: ints iqs, iqs+1 of the nibble bytes against q8_1 ints
 * iqs+i (low codes) and iqs+i+4 (high codes) */
static float ko_h2f_product(uint16_t a, uint16_t b) { return ko_h2f(ko_f2h(ko_h2f(a) * ko_h2f(b))); }

static int32_t q5_lo(uint32_t ql, uint32_t h) {
  return (int32_t)((ql & 0x0F0F0F0Fu) | ((h << 4) & 0x10u) | ((h << 11) & 0x1000u) | ((h << 18) & 0x100000u) |
                   ((h << 25) & 0x10000000u));
}
static int32_t q5_hi(uint32_t ql, uint32_t h) {
  return (int32_t)(((ql >> 4) & 0x0F0F0F0Fu) | ((h >> 12) & 0x10u) | ((h >> 5) & 0x1000u) | ((h << 2) & 0x100000u) |
                   ((h << 9) & 0x10000000u));
}

static float vd_legacy(int type, const uint8_t* bx, const uint8_t* b8, int iqs) {
  const uint8_t* q8 = b8 + 4;
  int32_t sumi = 0, sumi2 = 0;
  int qs_off = (type == KO_Q4_0 || type == KO_IQ4_NL) ? 2 : type == KO_Q4_1 ? 4 : type == KO_Q5_0 ? 6 : 8;
  int32_t qh = type == KO_Q5_0 ? rd32(bx + 2) : type == KO_Q5_1 ? rd32(bx + 4) : 0;
  for (int i = 0; i < 2; ++i) {
    uint32_t v = (uint32_t)rd32(bx + qs_off + 4 * (iqs + i));
    int32_t u0 = rd32(q8 + 4 * (iqs + i)), u1 = rd32(q8 + 4 * (iqs + i + 4));
    if (type == KO_Q5_0 || type == KO_Q5_1) {
      uint32_t h = (uint32_t)(qh >> (4 * (iqs + i))); /* arithmetic shift, as the reference's int */
      sumi = dp4a(q5_lo(v, h), u0, sumi);
      sumi = dp4a(q5_hi(v, h), u1, sumi);
    } else if (type == KO_IQ4_NL) {
      uint32_t lo = 0, hi = 0;
      for (int k = 0; k < 4; ++k) {
        lo |= (uint32_t)(uint8_t)ko_iq4nl[(v >> (8 * k)) & 0xF] << (8 * k);
        hi |= (uint32_t)(uint8_t)ko_iq4nl[(v >> (8 * k + 4)) & 0xF] << (8 * k);
      }
      sumi = dp4a((int32_t)lo, u0, sumi);
      sumi2 = dp4a((int32_t)hi, u1, sumi2);
    } else {
      sumi = dp4a((int32_t)(v & 0x0F0F0F0Fu), u0, sumi);
      sumi = dp4a((int32_t)((v >> 4) & 0x0F0F0F0Fu), u1, sumi);
    }
  }
  const float d8 = ko_h2f(rd16(b8)), s8 = ko_h2f(rd16(b8 + 2));
  switch (type) {
    case KO_Q4_0: return ko_h2f(rd16(bx)) * ((float)sumi * d8 - 4.0f * s8);
    case KO_Q5_0: return ko_h2f(rd16(bx)) * ((float)sumi * d8 - 8.0f * s8);
    case KO_Q4_1:
    case KO_Q5_1: {
      float dd = ko_h2f_product(rd16(bx), rd16(b8)), ms = ko_h2f_product(rd16(bx + 2), rd16(b8 + 2));
      return (float)sumi * dd + ms / 2.0f;
    }
    default: { /* IQ4_NL */
      float d = ko_h2f(rd16(bx)) * d8;
      return d * (float)(sumi + sumi2);
    }
  }
}

/* vec_dot_q2_K_q8_1: iqs 0..15; int iqs of qs has 4 codes of 4 groups (bit pairs), against
 * int iqs%8 of q8_1 blocks 4(iqs/8) + i; group scales at 2i past scale_offset */
static float vd_q2_k(const uint8_t* bx, const uint8_t* by0, int iqs) {
  const int bq8_offset = 4 * (iqs / 8);
  const uint8_t* scales = bx + iqs - iqs % 8 + (iqs % 8) / 4;
  const uint32_t v = (uint32_t)rd32(bx + 16 + 4 * iqs);
  float sumf_d = 0.0f, sumf_m = 0.0f;
  for (int i = 0; i < 4; ++i) {
    const uint8_t* b8 = by0 + 36 * (bq8_offset + i);
    const int32_t u = rd32(b8 + 4 + 4 * (iqs % 8));
    const float d8 = q8_1_d(b8);
    const int sc = scales[2 * i];
    sumf_d += d8 * (float)(dp4a((int32_t)((v >> (2 * i)) & 0x03030303u), u, 0) * (sc & 0xF));
    sumf_m += d8 * (float)dp4a((sc >> 4) * 0x01010101, u, 0);
  }
  const float dmx = ko_h2f(rd16(bx + 80)), dmy = ko_h2f(rd16(bx + 82));
  return dmx * sumf_d - dmy * sumf_m;
}

/* vec_dot_q3_K_q8_1: as Q2_K, the code's third bit from hmask int iqs%8 (clear: subtract 4,
 * a per-byte saturating subtraction that never saturates for 0..3 - 0/4) */
static float vd_q3_k(const uint8_t* bx, const uint8_t* by0, int iqs) {
  const int bq8_offset = 4 * (iqs / 8);
  const int scale_offset = iqs - iqs % 8 + (iqs % 8) / 4;
  const uint32_t vl = (uint32_t)rd32(bx + 32 + 4 * iqs);
  const int32_t vh = ~rd32(bx + 4 * (iqs % 8)) >> bq8_offset;
  float sumf = 0.0f;
  for (int i = 0; i < 4; ++i) {
    const int sc = q3k_scale(bx + 96, scale_offset + 2 * i);
    const uint32_t lo = (vl >> (2 * i)) & 0x03030303u;
    const uint32_t hi = ((uint32_t)(vh >> i) << 2) & 0x04040404u;
    uint32_t vi = 0;
    for (int k = 0; k < 4; ++k) {
      int8_t a = (int8_t)(lo >> (8 * k)), c = (int8_t)(hi >> (8 * k));
      vi |= (uint32_t)(uint8_t)(int8_t)(a - c) << (8 * k);
    }
    const uint8_t* b8 = by0 + 36 * (bq8_offset + i);
    const int32_t u = rd32(b8 + 4 + 4 * (iqs % 8));
    sumf += q8_1_d(b8) * (float)(dp4a((int32_t)vi, u, 0) * sc);
  }
  return ko_h2f(rd16(bx + 108)) * sumf;
}

/* vec_dot_q5_K_q8_1: Q4_K's chunk (iqs even 0..30) with the fifth bit of each code from qh */
static float vd_q5_k(const uint8_t* bx, const uint8_t* by0, int iqs) {
  const int bq8_offset = 2 * ((iqs / 2) / 4);
  const uint8_t* ql = bx + 48 + 16 * bq8_offset + 4 * ((iqs / 2) % 4);
  const uint8_t* qh = bx + 16 + 4 * ((iqs / 2) % 4);
  const uint32_t vl0 = (uint32_t)rd32(ql), vl1 = (uint32_t)rd32(ql + 16);
  const int32_t vh0 = rd32(qh) >> bq8_offset, vh1 = rd32(qh + 16) >> bq8_offset;
  uint16_t s16[6];
  for (int i = 0; i < 6; ++i) s16[i] = rd16(bx + 4 + 2 * i);
  uint16_t aux0, aux1;
  const int j = bq8_offset / 2;
  if (j < 2) {
    aux0 = s16[j + 0] & 0x3f3f;
    aux1 = s16[j + 2] & 0x3f3f;
  } else {
    aux0 = (uint16_t)(((s16[j + 2] >> 0) & 0x0f0f) | ((s16[j - 2] & 0xc0c0) >> 2));
    aux1 = (uint16_t)(((s16[j + 2] >> 4) & 0x0f0f) | ((s16[j - 0] & 0xc0c0) >> 2));
  }
  float sumf_d = 0.0f, sumf_m = 0.0f;
  for (int i = 0; i < 2; ++i) {
    const uint8_t* b8 = by0 + 36 * (bq8_offset + i);
    const int32_t u0 = rd32(b8 + 4 + 4 * ((iqs / 2) % 4)), u1 = rd32(b8 + 4 + 4 * ((iqs / 2) % 4) + 16);
    const int32_t v0 = (int32_t)(((vl0 >> (4 * i)) & 0x0F0F0F0Fu) | (((uint32_t)(vh0 >> i) << 4) & 0x10101010u));
    const int32_t v1 = (int32_t)(((vl1 >> (4 * i)) & 0x0F0F0F0Fu) | (((uint32_t)(vh1 >> i) << 4) & 0x10101010u));
    const int32_t dot1 = dp4a(v0, u0, dp4a(v1, u1, 0));
    const int32_t dot2 = dp4a(0x01010101, u0, dp4a(0x01010101, u1, 0));
    const float d8 = q8_1_d(b8);
    const int sc = (aux0 >> (8 * i)) & 0xff, m = (aux1 >> (8 * i)) & 0xff;
    sumf_d += d8 * (float)(dot1 * sc);
    sumf_m += d8 * (float)(dot2 * m);
  }
  const float dmx = ko_h2f(rd16(bx)), dmy = ko_h2f(rd16(bx + 2));
  return dmx * sumf_d - dmy * sumf_m;
}

/* vec_dot_iq4_xs_q8_1: chunk = sub-block ib32 (0..7) against q8_1 block ib32 */
static float vd_iq4_xs(const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* b8 = by0 + 36 * ib32;
  const uint8_t* q4 = bx + 8 + 16 * ib32;
  const int scales_h = rd16(bx + 2);
  const int ls = ((bx[4 + ib32 / 2] >> (4 * (ib32 % 2))) & 0xf) | (((scales_h >> (2 * ib32)) & 3) << 4);
  const float d = ko_h2f(rd16(bx)) * (float)(ls - 32) * q8_1_d(b8);
  int32_t sumi1 = 0, sumi2 = 0;
  for (int j = 0; j < 4; ++j) {
    uint32_t q = (uint32_t)rd32(q4 + 4 * j), lo = 0, hi = 0;
    for (int k = 0; k < 4; ++k) {
      lo |= (uint32_t)(uint8_t)ko_iq4nl[(q >> (8 * k)) & 0xF] << (8 * k);
      hi |= (uint32_t)(uint8_t)ko_iq4nl[(q >> (8 * k + 4)) & 0xF] << (8 * k);
    }
    sumi1 = dp4a((int32_t)lo, rd32(b8 + 4 + 4 * j), sumi1);
    sumi2 = dp4a((int32_t)hi, rd32(b8 + 20 + 4 * j), sumi2);
  }
  return d * (float)(sumi1 + sumi2);
}

/* vec_dot_q2_0_q8_1 (kt_gguf_moe_multi.cu:49-64): iqs 0..3, bytes 4iqs..4iqs+3 (16 values)
 * against half iqs&1 of q8_1 block iqs/2; d * d8 * (sum(code*u) - sum(u)) */
static float vd_q2_0(const uint8_t* bx, const uint8_t* by0, int iqs) {
  const uint8_t* b8 = by0 + 36 * (iqs >> 1);
  const uint8_t* u = b8 + 4 + 16 * (iqs & 1);
  int32_t sumi = 0, sumy = 0;
  for (int j = 0; j < 4; ++j) {
    const int c = bx[2 + 4 * iqs + j];
    uint32_t codes = 0;
    for (int s = 0; s < 4; ++s) codes |= (uint32_t)((c >> (2 * s)) & 3) << (8 * s);
    sumi = dp4a((int32_t)codes, rd32(u + 4 * j), sumi);
    sumy = dp4a(0x01010101, rd32(u + 4 * j), sumy);
  }
  return ko_h2f(rd16(bx)) * q8_1_d(b8) * (float)(sumi - sumy);
}

/* ---- i-quant dot products (vecdotq.cuh:1755-1776 iq2_xxs, 1778-1806 iq2_xs, 1809-1845 iq2_s,
 * 1848-1872 iq3_xxs, 1903-1932 iq1_s, 1935-1977 iq1_m): chunk = sub-block ib32 against q8_1
 * block ib32. The integer sums are exact whatever the evaluation; the fp32 combinations
 * follow the reference's expressions. */
static int32_t ko_sdot8(const uint8_t* q8, int mag_of_j[8], uint32_t s8) {
  int32_t sum = 0;
  for (int j = 0; j < 8; ++j) sum += (int32_t)(int8_t)q8[j] * mag_of_j[j] * ((s8 >> j) & 1 ? -1 : 1);
  return sum;
}
static float vd_iq2_xxs(const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* b8 = by0 + 36 * ib32;
  const uint8_t* q2 = bx + 2 + 8 * ib32;
  uint32_t aux = rd32u(q2 + 4);
  int32_t sumi = 0;
  for (int l = 0; l < 4; ++l) {
    int m[8];
    for (int j = 0; j < 8; ++j) m[j] = ko_iq2_mag(kt_iq2xxs_grid_host, q2[l], j);
    sumi += ko_sdot8(b8 + 4 + 8 * l, m, ko_signs8((aux >> (7 * l)) & 127u));
  }
  const float d = ko_h2f(rd16(bx)) * (0.5f + (float)(aux >> 28)) * q8_1_d(b8) * 0.25f;
  return d * (float)sumi;
}
static float vd_iq2_xs_s(int type, const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* b8 = by0 + 36 * ib32;
  const int ls = type == KO_IQ2_XS ? bx[66 + ib32] : bx[74 + ib32];
  int32_t sumi[2] = {0, 0};
  for (int l = 0; l < 4; ++l) {
    int m[8];
    uint32_t s;
    if (type == KO_IQ2_XS) {
      uint32_t code = rd16(bx + 2 + 8 * ib32 + 2 * l);
      for (int j = 0; j < 8; ++j) m[j] = ko_iq2_mag(kt_iq2xs_grid_host, (int)(code & 511u), j);
      s = ko_signs8(code >> 9);
    } else {
      int idx = bx[2 + 4 * ib32 + l] | ((bx[66 + ib32] << (8 - 2 * l)) & 0x300);
      for (int j = 0; j < 8; ++j) m[j] = ko_iq2_mag(kt_iq2s_grid_host, idx, j);
      s = bx[34 + 4 * ib32 + l];
    }
    sumi[l / 2] += ko_sdot8(b8 + 4 + 8 * l, m, s);
  }
  const float d = ko_h2f(rd16(bx)) * q8_1_d(b8) * 0.25f;
  return d * ((0.5f + (float)(ls & 0xf)) * (float)sumi[0] + (0.5f + (float)(ls >> 4)) * (float)sumi[1]);
}
static float vd_iq3_xxs(const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* b8 = by0 + 36 * ib32;
  const uint8_t* q3 = bx + 2 + 8 * ib32;
  uint32_t aux = rd32u(bx + 66 + 4 * ib32);
  int32_t sumi = 0;
  for (int l = 0; l < 4; ++l) {
    int m[8];
    for (int j = 0; j < 8; ++j) m[j] = (int)((kt_iq3xxs_grid_host[q3[2 * l + j / 4]] >> (8 * (j % 4))) & 0xffu);
    sumi += ko_sdot8(b8 + 4 + 8 * l, m, ko_signs8((aux >> (7 * l)) & 127u));
  }
  const float d = ko_h2f(rd16(bx)) * (0.5f + (float)(aux >> 28)) * q8_1_d(b8) * 0.5f;
  return d * (float)sumi;
}
/* IQ1: sum((v+1)*u) over a group, the book's stored values */
static int32_t ko_iq1_dot8(const uint8_t* q8, int e) {
  int32_t sum = 0;
  for (int j = 0; j < 8; ++j) sum += (int32_t)(int8_t)q8[j] * (ko_iq1_val(e, j) + 1);
  return sum;
}
static float vd_iq1_s(const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* b8 = by0 + 36 * ib32;
  const int qh = rd16(bx + 34 + 2 * ib32);
  int32_t sumi = 0;
  for (int l = 0; l < 4; ++l) sumi += ko_iq1_dot8(b8 + 4 + 8 * l, bx[2 + 4 * ib32 + l] | (((qh >> (3 * l)) & 7) << 8));
  const float d1q = ko_h2f(rd16(bx)) * (float)(((qh >> 11) & 0x0E) + 1);
  const float delta = (qh & 0x8000) ? -1.0f - KO_IQ1_DELTA : -1.0f + KO_IQ1_DELTA;
  const float dx = ko_h2f(rd16(b8)), dy = ko_h2f(rd16(b8 + 2));
  return d1q * (dx * (float)sumi + dy * delta);
}
static float vd_iq1_m(const uint8_t* bx, const uint8_t* by0, int ib32) {
  const uint8_t* b8 = by0 + 36 * ib32;
  int32_t sumi[2] = {0, 0};
  float sumf[2] = {0.0f, 0.0f};
  for (int l = 0; l < 4; ++l) {
    const int qhl = bx[32 + 2 * ib32 + l / 2] >> (4 * (l % 2));
    sumi[l / 2] += ko_iq1_dot8(b8 + 4 + 8 * l, bx[4 * ib32 + l] | ((qhl & 7) << 8));
    const float delta = (qhl & 8) ? -1.0f - KO_IQ1_DELTA : -1.0f + KO_IQ1_DELTA;
    int32_t sumy = 0;
    for (int j = 0; j < 8; ++j) sumy += (int8_t)b8[4 + 8 * l + j];
    sumf[l / 2] += delta * (float)sumy;
  }
  uint16_t sc[4];
  for (int k = 0; k < 4; ++k) sc[k] = rd16(bx + 48 + 2 * k);
  const float d = ko_h2f((uint16_t)((sc[0] >> 12) | ((sc[1] >> 8) & 0x00F0) | ((sc[2] >> 4) & 0x0F00) | (sc[3] & 0xF000))) *
                  q8_1_d(b8);
  const int tmp = sc[ib32 / 2] >> (6 * (ib32 % 2));
  const int sc0 = 2 * (tmp & 7) + 1, sc1 = 2 * ((tmp >> 3) & 7) + 1;
  return d * (((float)sumi[0] + sumf[0]) * (float)sc0 + ((float)sumi[1] + sumf[1]) * (float)sc1);
}

/* chunk geometry of the reference launchers: values per block, chunks per block, vdr */
static int chunk_geom(int type, int* qk, int* cpb, int* vdr) {
  switch (type) {
    case KO_Q8_0: *qk = 32; *cpb = 4; *vdr = 2; return 0;   /* qi 8, vdr 2 */
    case KO_Q4_K: *qk = 256; *cpb = 16; *vdr = 2; return 0; /* qi 32, vdr 2 */
    case KO_Q6_K: *qk = 256; *cpb = 32; *vdr = 1; return 0; /* qi 32, vdr 1 */
    case KO_IQ3_S: *qk = 256; *cpb = 8; *vdr = 1; return 0; /* qi 8, vdr 1 */
    case KO_Q2_K: case KO_Q3_K: *qk = 256; *cpb = 16; *vdr = 1; return 0; /* qi 16, vdr 1 */
    case KO_Q5_K: *qk = 256; *cpb = 16; *vdr = 2; return 0; /* qi 32, vdr 2 */
    case KO_IQ4_XS: *qk = 256; *cpb = 8; *vdr = 1; return 0; /* qi 8, vdr 1 */
    case KO_Q2_0: *qk = 64; *cpb = 4; *vdr = 1; return 0;   /* qi 4, vdr 1 */
    case KO_IQ2_XXS: case KO_IQ2_XS: case KO_IQ2_S: case KO_IQ3_XXS: case KO_IQ1_S: case KO_IQ1_M:
      *qk = 256; *cpb = 8; *vdr = 1; return 0;              /* qi 8, vdr 1 */
    case KO_Q4_0: case KO_Q4_1: case KO_Q5_0: case KO_Q5_1: case KO_IQ4_NL:
      *qk = 32; *cpb = 2; *vdr = 2; return 0;               /* qi 4, vdr 2 */
    default: return -1;
  }
}

/* One output row: lane t takes chunks t, t+32, ... in order; then the xor butterfly. */
static float row_dot(int type, const uint8_t* wrow, int bs, int nblocks, const uint8_t* yrow) {
  int qk = 32, cpb = 1, vdr = 1;
  chunk_geom(type, &qk, &cpb, &vdr);
  float lane[32];
  for (int t = 0; t < 32; ++t) lane[t] = 0.0f;
  const int nchunks = nblocks * cpb;
  for (int c = 0; c < nchunks; ++c) {
    const int i = c / cpb, iqs = vdr * (c % cpb);
    const uint8_t* bx = wrow + (int64_t)i * bs;
    const uint8_t* by = yrow + (int64_t)i * (qk / 32) * 36;
    float v = 0.0f;
    switch (type) {
      case KO_Q8_0: v = vd_q8_0(bx, by, iqs); break;
      case KO_Q4_K: v = vd_q4_k(bx, by, iqs); break;
      case KO_Q6_K: v = vd_q6_k(bx, by, iqs); break;
      case KO_IQ3_S: v = vd_iq3_s(bx, by, iqs); break;
      case KO_Q2_K: v = vd_q2_k(bx, by, iqs); break;
      case KO_Q3_K: v = vd_q3_k(bx, by, iqs); break;
      case KO_Q5_K: v = vd_q5_k(bx, by, iqs); break;
      case KO_IQ4_XS: v = vd_iq4_xs(bx, by, iqs); break;
      case KO_Q2_0: v = vd_q2_0(bx, by, iqs); break;
      case KO_IQ2_XXS: v = vd_iq2_xxs(bx, by, iqs); break;
      case KO_IQ2_XS: case KO_IQ2_S: v = vd_iq2_xs_s(type, bx, by, iqs); break;
      case KO_IQ3_XXS: v = vd_iq3_xxs(bx, by, iqs); break;
      case KO_IQ1_S: v = vd_iq1_s(bx, by, iqs); break;
      case KO_IQ1_M: v = vd_iq1_m(bx, by, iqs); break;
      default: v = vd_legacy(type, bx, by, iqs); break;
    }
    lane[c % 32] += v;
  }
  for (int mask = 16; mask > 0; mask >>= 1) {
    float n[32];
    for (int t = 0; t < 32; ++t) n[t] = lane[t] + lane[t ^ mask];
    memcpy(lane, n, sizeof n);
  }
  return lane[0];
}

/*
 * moe_vec_q: out[p, r] = row r of expert slot ids[p] against q8_1(X[p / top_k]); zero rows
 * for ids < 0. slots[s] points at slot s's [rows, row_bytes] GGUF matrix (the plain layout
 * and the pointer-table build read the same bytes).
 */
int ko_moe_vec(int type, const uint8_t* const* slots, int64_t n_slots, const uint8_t* qx, int64_t qx_row_bytes,
               const int32_t* ids, int64_t routes, int64_t top_k, int64_t rows, int64_t cols, float* out) {
  int blck, bs;
  if (ko_block_info(type, &blck, &bs) || cols % blck) return -1;
  const int nb = (int)(cols / blck);
  const int64_t rb = (int64_t)nb * bs;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t p = 0; p < routes; ++p) {
    const int32_t e = ids[p];
    float* o = out + p * rows;
    if (e < 0 || e >= n_slots) {
      for (int64_t r = 0; r < rows; ++r) o[r] = 0.0f;
      continue;
    }
    const uint8_t* y = qx + (p / top_k) * qx_row_bytes;
    for (int64_t r = 0; r < rows; ++r) o[r] = row_dot(type, slots[e] + r * rb, bs, nb, y);
  }
  return 0;
}

/* ---------------------------------------------------------------- bf16 helpers, SwiGLU, combine */

int ko_f32_to_bf16(const float* x, int64_t n, uint16_t* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = ko_f2bf(x[i]);
  return 0;
}

int ko_bf16_to_f32(const uint16_t* x, int64_t n, float* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = ko_bf2f(x[i]);
  return 0;
}

static float silu_f(float x) { return x / (1.0f + expf(-x)); }

/* silu_and_mul on a bf16 [rows, 2n] tensor: h = bf16(silu(g) * u) in fp32 */
int ko_silu_and_mul_bf16(const uint16_t* h13, int64_t rows, int64_t n, uint16_t* h) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < n; ++j)
      h[r * n + j] = ko_f2bf(silu_f(ko_bf2f(h13[r * 2 * n + j])) * ko_bf2f(h13[r * 2 * n + n + j]));
  return 0;
}

/* _combine: res[t] = bf16(sum_k fp32(bf16(out[t,k] * bf16(w[t,k])))) in k order */
int ko_combine_bf16(const uint16_t* out, const float* w, int64_t T, int64_t top_k, int64_t K, uint16_t* res) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t c = 0; c < K; ++c) {
      float acc = 0.0f;
      for (int64_t k = 0; k < top_k; ++k) {
        float o = ko_bf2f(out[(t * top_k + k) * K + c]);
        float wk = ko_round_bf(w[t * top_k + k]);
        acc += ko_round_bf(o * wk);
      }
      res[t * K + c] = ko_f2bf(acc);
    }
  }
  return 0;
}

/*
 * The reference's hot-expert MoE layer on bf16 activations (KTGGUFHotExpertsMethod.apply):
 * q8_1(x) -> gate/up GEMV (bf16) -> silu_and_mul (bf16) -> q8_1(h) -> down GEMV (bf16)
 * -> combine. x [T, K] bf16; ids [T, top_k] slot ids (-1 = not on this device);
 * w [T, top_k] fp32; w13 slots [2N, K] (type13), w2 slots [K, N] (type2); res [T, K] bf16.
 * This is also the timed CPU baseline (OpenMP over routes).
 */
int ko_moe_ref_bf16(const uint16_t* x, int64_t T, int64_t K, int64_t N, const int32_t* ids, const float* w,
                    int64_t top_k, int type13, const uint8_t* const* w13, int type2, const uint8_t* const* w2,
                    int64_t n_slots, uint16_t* res) {
  const int64_t R = T * top_k;
  const int64_t qxb = ko_q8_1_row_bytes(K), qhb = ko_q8_1_row_bytes(N);
  float* xf = (float*)malloc(sizeof(float) * T * K);
  uint8_t* qx = (uint8_t*)malloc(qxb * T);
  float* h13f = (float*)malloc(sizeof(float) * R * 2 * N);
  uint16_t* h13 = (uint16_t*)malloc(2 * R * 2 * N);
  uint16_t* h = (uint16_t*)malloc(2 * R * N);
  float* hf = (float*)malloc(sizeof(float) * R * N);
  uint8_t* qh = (uint8_t*)malloc(qhb * R);
  float* yf = (float*)malloc(sizeof(float) * R * K);
  uint16_t* y = (uint16_t*)malloc(2 * R * K);
  int rc = -1;
  if (!xf || !qx || !h13f || !h13 || !h || !hf || !qh || !yf || !y) goto done;
  ko_bf16_to_f32(x, T * K, xf);
  ko_quantize_q8_1(xf, T, K, qx);
  if (ko_moe_vec(type13, w13, n_slots, qx, qxb, ids, R, top_k, 2 * N, K, h13f)) goto done;
  ko_f32_to_bf16(h13f, R * 2 * N, h13);
  ko_silu_and_mul_bf16(h13, R, N, h);
  ko_bf16_to_f32(h, R * N, hf);
  ko_quantize_q8_1(hf, R, N, qh);
  if (ko_moe_vec(type2, w2, n_slots, qh, qhb, ids, R, 1, K, N, yf)) goto done;
  ko_f32_to_bf16(yf, R * K, y);
  ko_combine_bf16(y, w, T, top_k, K, res);
  rc = 0;
done:
  free(xf); free(qx); free(h13f); free(h13); free(h); free(hf); free(qh); free(yf); free(y);
  return rc;
}

/*
 * fp32 dequant-then-matmul oracle (double accumulation): out[t] = sum_k w[t,k] *
 * W2[e] (silu(W13g[e] x) * W13u[e] x) over routes with ids >= 0. x [T, K] bf16,
 * out fp32 [T, K]. Weights are dequantized per slot on first use.
 */
int ko_moe_fp32(const uint16_t* x, int64_t T, int64_t K, int64_t N, const int32_t* ids, const float* w,
                int64_t top_k, int type13, const uint8_t* const* w13, int type2, const uint8_t* const* w2,
                int64_t n_slots, float* out) {
  float** d13 = (float**)calloc(n_slots, sizeof(float*));
  float** d2 = (float**)calloc(n_slots, sizeof(float*));
  if (!d13 || !d2) return -1;
  int rc = 0;
  for (int64_t s = 0; s < n_slots && !rc; ++s) {
    int used = 0;
    for (int64_t p = 0; p < T * top_k; ++p) used |= ids[p] == s;
    if (!used) continue;
    d13[s] = (float*)malloc(sizeof(float) * 2 * N * K);
    d2[s] = (float*)malloc(sizeof(float) * K * N);
    if (!d13[s] || !d2[s]) { rc = -1; break; }
    rc |= ko_dequant_rows(type13, w13[s], 2 * N, K, d13[s]);
    rc |= ko_dequant_rows(type2, w2[s], K, N, d2[s]);
  }
  if (!rc) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t t = 0; t < T; ++t) {
      double* acc = (double*)calloc(K, sizeof(double));
      double* hh = (double*)malloc(sizeof(double) * N);
      double* xx = (double*)malloc(sizeof(double) * K);
      for (int64_t c = 0; c < K; ++c) xx[c] = ko_bf2f(x[t * K + c]);
      for (int64_t k = 0; k < top_k; ++k) {
        int32_t e = ids[t * top_k + k];
        if (e < 0 || e >= n_slots) continue;
        for (int64_t j = 0; j < N; ++j) {
          double g = 0.0, u = 0.0;
          const float* wg = d13[e] + j * K;
          const float* wu = d13[e] + (N + j) * K;
          for (int64_t c = 0; c < K; ++c) { g += wg[c] * xx[c]; u += wu[c] * xx[c]; }
          hh[j] = g / (1.0 + exp(-g)) * u;
        }
        double wk = w[t * top_k + k];
        for (int64_t c = 0; c < K; ++c) {
          const float* wd = d2[e] + c * N;
          double s = 0.0;
          for (int64_t j = 0; j < N; ++j) s += wd[j] * hh[j];
          acc[c] += wk * s;
        }
      }
      for (int64_t c = 0; c < K; ++c) out[t * K + c] = (float)acc[c];
      free(acc); free(hh); free(xx);
    }
  }
  for (int64_t s = 0; s < n_slots; ++s) { free(d13[s]); free(d2[s]); }
  free(d13); free(d2);
  return rc;
}
