/*
 * gguf_encode.c — host-side GGUF encoders for synthetic expert weights.
 *
 * The reference quantizes its experts with llama.cpp's quantizers, which are not part of
 * the hot path and are not available here. The benchmark and the tests need GGUF blocks
 * of the four hot-path types built from seeded fp32 weights, so this file writes them:
 *   Q8_0  — ggml's rounding rule exactly (d = amax/127, q = roundf(x / d)).
 *   Q4_K  — per 32-value sub-block min/max, 6-bit scales and mins under fp16 d / dmin.
 *   Q6_K  — per 16-value sub-block absmax, int8 scales under an fp16 d.
 *   IQ3_S — per 32-value sub-block scale d*(1+2s), each group of 4 magnitudes snapped
 *           to the nearest grid entry of the 512-word IQ3_S codebook, sign bits apart.
 *   Q2_0  — the reference's 64-value block (ggml type 42): d = amax/2, code =
 *           clamp(roundf(x / d) + 1, 0, 3), so the levels are -d, 0, d, 2d.
 * Any bytes these produce are valid blocks of their type; the decoders (GPU kernels and
 * the CPU oracle) do not depend on how the encoder chose them.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include "iq3s_grid.h"

static uint16_t f2h(float f) {
  _Float16 h = (_Float16)f;
  uint16_t r;
  memcpy(&r, &h, 2);
  return r;
}

static float h2f(uint16_t v) {
  _Float16 h;
  memcpy(&h, &v, 2);
  return (float)h;
}

static void put16(uint8_t* p, uint16_t v) { p[0] = v & 0xff; p[1] = v >> 8; }

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static void enc_q8_0(const float* x, uint8_t* b) {
  float amax = 0.0f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
  const float d = amax / 127;
  const float id = d ? 1.0f / d : 0.0f;
  put16(b, f2h(d));
  for (int j = 0; j < 32; ++j) b[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

static void enc_q2_0(const float* x, uint8_t* b) {
  float amax = 0.0f;
  for (int j = 0; j < 64; ++j) amax = fmaxf(amax, fabsf(x[j]));
  const float d = amax / 2;
  const float id = d ? 1.0f / d : 0.0f;
  put16(b, f2h(d));
  memset(b + 2, 0, 16);
  for (int j = 0; j < 64; ++j) b[2 + j / 4] |= (uint8_t)(clampi((int)roundf(x[j] * id) + 1, 0, 3) << (2 * (j % 4)));
}

static void enc_q4_k(const float* x, uint8_t* b) {
  float scale[8], mins[8], max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; ++j) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int l = 1; l < 32; ++l) {
      mn = fminf(mn, x[32 * j + l]);
      mx = fmaxf(mx, x[32 * j + l]);
    }
    if (mn > 0) mn = 0;
    scale[j] = (mx - mn) / 15;
    mins[j] = -mn;
    max_scale = fmaxf(max_scale, scale[j]);
    max_min = fmaxf(max_min, mins[j]);
  }
  const uint16_t hd = f2h(max_scale / 63), hm = f2h(max_min / 63);
  const float d = h2f(hd), dmin = h2f(hm);
  uint8_t sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = (uint8_t)(d > 0 ? clampi((int)lrintf(scale[j] / d), 0, 63) : 0);
    m[j] = (uint8_t)(dmin > 0 ? clampi((int)lrintf(mins[j] / dmin), 0, 63) : 0);
  }
  put16(b, hd);
  put16(b + 2, hm);
  uint8_t* s = b + 4;
  for (int j = 0; j < 4; ++j) {
    s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; ++j) {
    const float ds = d * sc[j], dm = dmin * m[j];
    for (int l = 0; l < 32; ++l) q[32 * j + l] = (uint8_t)(ds > 0 ? clampi((int)lrintf((x[32 * j + l] + dm) / ds), 0, 15) : 0);
  }
  uint8_t* qs = b + 16;
  for (int j = 0; j < 4; ++j)
    for (int l = 0; l < 32; ++l) qs[32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

static void enc_q6_k(const float* x, uint8_t* b) {
  float scale[16], max_abs = 0.0f;
  for (int j = 0; j < 16; ++j) {
    float amax = 0.0f;
    for (int l = 0; l < 16; ++l) amax = fmaxf(amax, fabsf(x[16 * j + l]));
    scale[j] = amax / 31;
    max_abs = fmaxf(max_abs, scale[j]);
  }
  const uint16_t hd = f2h(max_abs / 127);
  const float d = h2f(hd);
  int8_t sc[16];
  uint8_t L[256];
  for (int j = 0; j < 16; ++j) {
    sc[j] = (int8_t)(d > 0 ? clampi((int)lrintf(scale[j] / d), -128, 127) : 0);
    const float ds = d * sc[j];
    for (int l = 0; l < 16; ++l) {
      int q = ds != 0 ? clampi((int)lrintf(x[16 * j + l] / ds), -32, 31) : 0;
      L[16 * j + l] = (uint8_t)(q + 32);
    }
  }
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  for (int n = 0; n < 2; ++n) {
    for (int l = 0; l < 32; ++l) {
      const uint8_t q1 = L[128 * n + l], q2 = L[128 * n + l + 32], q3 = L[128 * n + l + 64], q4 = L[128 * n + l + 96];
      ql[64 * n + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[64 * n + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  memcpy(b + 192, sc, 16);
  put16(b + 208, hd);
}

/* nearest grid index for every combination of four 3-bit levels (magnitude = 2*level + 1) */
static uint16_t iq3s_nearest[4096];
static int iq3s_ready = 0;

static void iq3s_init(void) {
  for (int c = 0; c < 4096; ++c) {
    int best = 0, best_err = 1 << 30;
    for (int g = 0; g < 512; ++g) {
      int err = 0;
      for (int j = 0; j < 4; ++j) {
        const int lv = ((int)((kt_iq3s_grid_host[g] >> (8 * j)) & 0xff) - 1) / 2;
        const int dv = lv - ((c >> (3 * j)) & 7);
        err += dv * dv;
      }
      if (err < best_err) { best_err = err; best = g; }
    }
    iq3s_nearest[c] = (uint16_t)best;
  }
  iq3s_ready = 1;
}

static void enc_iq3_s(const float* x, uint8_t* b) {
  memset(b, 0, 110);
  float amax[8], top = 0.0f;
  for (int ib = 0; ib < 8; ++ib) {
    amax[ib] = 0.0f;
    for (int l = 0; l < 32; ++l) amax[ib] = fmaxf(amax[ib], fabsf(x[32 * ib + l]));
    top = fmaxf(top, amax[ib]);
  }
  const uint16_t hd = f2h(top / 15 / 31);
  const float d = h2f(hd);
  put16(b, hd);
  if (d <= 0) return;
  uint8_t* qs = b + 2;
  uint8_t* qh = b + 66;
  uint8_t* signs = b + 74;
  uint8_t* scales = b + 106;
  for (int ib = 0; ib < 8; ++ib) {
    const int s = clampi((int)lrintf((amax[ib] / 15 / d - 1) / 2), 0, 15);
    scales[ib / 2] |= (uint8_t)(s << (4 * (ib % 2)));
    const float db = d * (float)(1 + 2 * s);
    for (int grp = 0; grp < 8; ++grp) {
      const float* v = x + 32 * ib + 4 * grp;
      int code = 0;
      uint8_t sg = 0;
      for (int j = 0; j < 4; ++j) {
        const int lv = clampi((int)lrintf((fabsf(v[j]) / db - 1) / 2), 0, 7);
        code |= lv << (3 * j);
        if (v[j] < 0) sg |= (uint8_t)(1u << j);
      }
      const int g = iq3s_nearest[code];
      const int l = grp / 2, h = grp % 2;
      qs[8 * ib + 2 * l + h] = (uint8_t)(g & 255);
      qh[ib] |= (uint8_t)(((g >> 8) & 1) << (2 * l + h));
      signs[4 * ib + l] |= (uint8_t)(sg << (4 * h));
    }
  }
}

int kte_row_bytes(int type, int64_t cols, int64_t* out) {
  int blck, bs;
  switch (type) {
    case 8: blck = 32; bs = 34; break;
    case 12: blck = 256; bs = 144; break;
    case 14: blck = 256; bs = 210; break;
    case 21: blck = 256; bs = 110; break;
    case 42: blck = 64; bs = 18; break;
    default: return -1;
  }
  if (cols % blck) return -2;
  *out = cols / blck * bs;
  return 0;
}

/* x [rows, cols] fp32 -> out [rows, row_bytes] GGUF blocks of the given ggml type */
int kte_quantize(int type, const float* x, int64_t rows, int64_t cols, uint8_t* out) {
  int64_t rb;
  int rc = kte_row_bytes(type, cols, &rb);
  if (rc) return rc;
  if (type == 21 && !iq3s_ready) iq3s_init();
  const int blck = type == 8 ? 32 : (type == 42 ? 64 : 256);
  const int bs = (int)(rb / (cols / blck));
  const int64_t nb = cols / blck;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t i = 0; i < nb; ++i) {
      const float* xb = x + r * cols + i * blck;
      uint8_t* bb = out + r * rb + i * bs;
      switch (type) {
        case 8: enc_q8_0(xb, bb); break;
        case 12: enc_q4_k(xb, bb); break;
        case 14: enc_q6_k(xb, bb); break;
        case 21: enc_iq3_s(xb, bb); break;
        case 42: enc_q2_0(xb, bb); break;
      }
    }
  }
  return 0;
}
