/*
 * kt_cpu_simd.c — the timed CPU baseline: the reference's hot-expert layer arithmetic (q8_1
 * activations x GGUF integer dot products, per-block fp32 scales, bf16 intermediates) written
 * for the host's SIMD units — TEST AND BENCHMARK INFRASTRUCTURE ONLY (bench.py's CPU baseline
 * and reference arm, and the tests that pin it to the scalar oracle). Not the checker: the
 * scalar restatement in kt_oracle.c is, and this file's results differ from it only in the
 * fp32 summation order of the per-block terms.
 *
 * What the reference's CPU path (kt-kernel's llamafile MoE on AVX-512 VNNI; not vendored
 * here) does per expert, restated: the routes of each expert are gathered, each weight row is
 * decoded once per group of routes into unsigned bytes, and VPDPBUSD multiplies 64 weight
 * bytes by 64 q8_1 activation bytes at a time into 16 int32 lanes, which are scaled by the
 * per-block weight scale times the activation block's d8 and accumulated in fp32. Unsigned
 * weight codes carry their offset as an integer correction with the activation block sums
 * (Q4_K: the mins; Q6_K: 32; Q8_0: 128), exactly as the reference's dp4a kernels subtract
 * them. Types: Q4_K, Q6_K, Q8_0 (BASELINE configs 1 and 2); others return -1.
 *
 * Arithmetic per projection (restates vecdotq.cuh vec_dot_q4_K_q8_1 :1326-1367,
 * vec_dot_q6_K_q8_1 :1625-1646, vec_dot_q8_0_q8_1 :969-982 and quantize_q8_1 in
 * kt_gguf_moe_multi.cu:600-650; the layer follows hot/kt_gguf_hot.py:240-304).
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KC_Q8_0 8
#define KC_Q4_K 12
#define KC_Q6_K 14
#define KC_GROUP 8 /* routes that share one decode of a weight row */

/* from kt_oracle.c (same library) */
int64_t ko_q8_1_row_bytes(int64_t cols);
int ko_quantize_q8_1(const float* x, int64_t rows, int64_t cols, uint8_t* qx);
int ko_silu_and_mul_bf16(const uint16_t* h13, int64_t rows, int64_t n, uint16_t* h);
int ko_combine_bf16(const uint16_t* out, const float* w, int64_t T, int64_t top_k, int64_t K, uint16_t* res);
int ko_f32_to_bf16(const float* x, int64_t n, uint16_t* y);
int ko_bf16_to_f32(const uint16_t* x, int64_t n, float* y);

/* IEEE half -> float (exact) */
static float kc_h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else { /* subnormal: m * 2^-24 */
      float f = (float)m * 5.9604644775390625e-8f;
      memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* activation rows in the layout the dot products read: int8 values [rows][kpad], and per
 * 32-value block d8 spread over 8 floats (so 16 consecutive floats scale two blocks' lanes),
 * sd8 = d8 * (sum of the block's ints) and, per 16-value group, sd16 = d8 * (sum of its ints) */
typedef struct {
  int64_t rows, kpad;
  int8_t* q;
  float* d8x8;
  float* sd8;
  float* sd16;
} KcAct;

static void kc_act_free(KcAct* a) {
  free(a->q);
  free(a->d8x8);
  free(a->sd8);
  free(a->sd16);
}

static int kc_act_build(const float* x, int64_t rows, int64_t cols, KcAct* a) {
  const int64_t kpad = (cols + 511) / 512 * 512, rb = ko_q8_1_row_bytes(cols), nb = kpad / 32;
  uint8_t* qx = (uint8_t*)malloc(rb * rows);
  a->rows = rows;
  a->kpad = kpad;
  a->q = (int8_t*)malloc(rows * kpad);
  a->d8x8 = (float*)malloc(sizeof(float) * rows * nb * 8);
  a->sd8 = (float*)malloc(sizeof(float) * rows * nb);
  a->sd16 = (float*)malloc(sizeof(float) * rows * nb * 2);
  if (!qx || !a->q || !a->d8x8 || !a->sd8 || !a->sd16) {
    free(qx);
    return -1;
  }
  ko_quantize_q8_1(x, rows, cols, qx); /* the reference's rounding: d = amax/127, roundf, fp16 d */
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < nb; ++b) {
      const uint8_t* blk = qx + r * rb + b * 36;
      const float d8 = kc_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
      int s0 = 0, s1 = 0;
      for (int t = 0; t < 32; ++t) {
        const int8_t v = (int8_t)blk[4 + t];
        a->q[r * kpad + b * 32 + t] = v;
        if (t < 16) s0 += v; else s1 += v;
      }
      for (int j = 0; j < 8; ++j) a->d8x8[(r * nb + b) * 8 + j] = d8;
      a->sd8[r * nb + b] = d8 * (float)(s0 + s1);
      a->sd16[(r * nb + b) * 2 + 0] = d8 * (float)s0;
      a->sd16[(r * nb + b) * 2 + 1] = d8 * (float)s1;
    }
  }
  free(qx);
  return 0;
}

__attribute__((target("avx512f,avx512bw,avx512vl,avx512dq,avx512vnni,fma"))) static float kc_hsum(__m512 v) {
  return _mm512_reduce_add_ps(v);
}

/* One weight row against n <= KC_GROUP activation rows (act row indices arows): out[i]. */
__attribute__((target("avx512f,avx512bw,avx512vl,avx512dq,avx512vnni,fma")))
static void kc_row_q4_k(const uint8_t* row, int64_t nsb, const KcAct* a, const int64_t* arows, int n, float* out) {
  __m512 acc[KC_GROUP];
  __m256 accm[KC_GROUP];
  for (int i = 0; i < n; ++i) {
    acc[i] = _mm512_setzero_ps();
    accm[i] = _mm256_setzero_ps();
  }
  const __m512i m4 = _mm512_set1_epi8(0x0F);
  const int64_t nb = a->kpad / 32;
  for (int64_t sb = 0; sb < nsb; ++sb) {
    const uint8_t* b = row + sb * 144;
    const float d = kc_h2f((uint16_t)(b[0] | (b[1] << 8))), dmin = kc_h2f((uint16_t)(b[2] | (b[3] << 8)));
    const uint8_t* q = b + 4;
    float sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
      int s, m;
      if (j < 4) {
        s = q[j] & 63;
        m = q[j + 4] & 63;
      } else {
        s = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
      }
      sc[j] = d * (float)s;
      mn[j] = dmin * (float)m;
    }
    const __m256 vmn = _mm256_loadu_ps(mn);
    for (int g = 0; g < 4; ++g) { /* 64 values: sub-blocks 2g (low nibbles) and 2g+1 (high) */
      const __m256i raw = _mm256_loadu_si256((const __m256i*)(b + 16 + 32 * g));
      const __m512i both = _mm512_inserti64x4(_mm512_castsi256_si512(raw), raw, 1);
      const __m512i sh = _mm512_mask_srli_epi16(both, 0xFFFF0000u, both, 4);
      const __m512i w = _mm512_and_si512(_mm512_mask_mov_epi16(both, 0xFFFF0000u, sh), m4);
      const __m512 wsc = _mm512_insertf32x8(_mm512_set1_ps(sc[2 * g]), _mm256_set1_ps(sc[2 * g + 1]), 1);
      for (int i = 0; i < n; ++i) {
        const int64_t blk = sb * 8 + 2 * g;
        const __m512i act = _mm512_loadu_si512((const void*)(a->q + arows[i] * a->kpad + blk * 32));
        const __m512i dot = _mm512_dpbusd_epi32(_mm512_setzero_si512(), w, act);
        const __m512 s = _mm512_mul_ps(wsc, _mm512_loadu_ps(a->d8x8 + (arows[i] * nb + blk) * 8));
        acc[i] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(dot), s, acc[i]);
      }
    }
    for (int i = 0; i < n; ++i)
      accm[i] = _mm256_fmadd_ps(vmn, _mm256_loadu_ps(a->sd8 + arows[i] * nb + sb * 8), accm[i]);
  }
  for (int i = 0; i < n; ++i) {
    __m256 m = accm[i];
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(m), _mm256_extractf128_ps(m, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    h = _mm_add_ss(h, _mm_shuffle_ps(h, h, 1));
    out[i] = kc_hsum(acc[i]) - _mm_cvtss_f32(h);
  }
}

__attribute__((target("avx512f,avx512bw,avx512vl,avx512dq,avx512vnni,fma")))
static void kc_row_q6_k(const uint8_t* row, int64_t nsb, const KcAct* a, const int64_t* arows, int n, float* out) {
  __m512 acc[KC_GROUP], accc[KC_GROUP];
  for (int i = 0; i < n; ++i) acc[i] = accc[i] = _mm512_setzero_ps();
  const __m512i m4 = _mm512_set1_epi8(0x0F), m2 = _mm512_set1_epi8(0x03);
  const int64_t nb = a->kpad / 32;
  for (int64_t sb = 0; sb < nsb; ++sb) {
    const uint8_t* b = row + sb * 210;
    const float d = kc_h2f((uint16_t)(b[208] | (b[209] << 8)));
    const int8_t* scales = (const int8_t*)(b + 192);
    float dsc[16];
    for (int g = 0; g < 16; ++g) dsc[g] = d * (float)scales[g];
    for (int nh = 0; nh < 2; ++nh) { /* 128 values: codes q1 q2 (low nibbles), q3 q4 (high) */
      const __m512i ql = _mm512_loadu_si512((const void*)(b + 64 * nh));
      const __m256i qh256 = _mm256_loadu_si256((const __m256i*)(b + 128 + 32 * nh));
      const __m512i qh = _mm512_inserti64x4(_mm512_castsi256_si512(qh256), _mm256_srli_epi16(qh256, 2), 1);
      const __m512i lo = _mm512_or_si512(_mm512_and_si512(ql, m4),
                                         _mm512_slli_epi16(_mm512_and_si512(qh, m2), 4));
      const __m512i hi = _mm512_or_si512(_mm512_and_si512(_mm512_srli_epi16(ql, 4), m4),
                                         _mm512_slli_epi16(_mm512_and_si512(_mm512_srli_epi16(qh, 4), m2), 4));
      /* lo: values [128nh, +64) (scale groups 8nh + 0..3), hi: [128nh + 64, +64) (8nh + 4..7);
       * scale of value v: group v / 16 (scales[8nh + (l/16) + 2*part] in ggml's indexing) */
      for (int part = 0; part < 2; ++part) {
        const __m512i w = part ? hi : lo;
        const int g0 = 8 * nh + 4 * part; /* first 16-value group of these 64 values */
        const __m512 wsc = _mm512_set_ps(dsc[g0 + 3], dsc[g0 + 3], dsc[g0 + 3], dsc[g0 + 3], dsc[g0 + 2],
                                         dsc[g0 + 2], dsc[g0 + 2], dsc[g0 + 2], dsc[g0 + 1], dsc[g0 + 1],
                                         dsc[g0 + 1], dsc[g0 + 1], dsc[g0], dsc[g0], dsc[g0], dsc[g0]);
        const int64_t blk = sb * 8 + 4 * nh + 2 * part; /* first 32-value q8_1 block */
        for (int i = 0; i < n; ++i) {
          const __m512i act = _mm512_loadu_si512((const void*)(a->q + arows[i] * a->kpad + blk * 32));
          const __m512i dot = _mm512_dpbusd_epi32(_mm512_setzero_si512(), w, act);
          const __m512 s = _mm512_mul_ps(wsc, _mm512_loadu_ps(a->d8x8 + (arows[i] * nb + blk) * 8));
          acc[i] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(dot), s, acc[i]);
        }
      }
    }
    /* the codes' offset: -32 * d * sc[g] * d8 * (sum of the group's ints), 16 groups at once */
    const __m512 vdsc = _mm512_loadu_ps(dsc);
    for (int i = 0; i < n; ++i)
      accc[i] = _mm512_fmadd_ps(vdsc, _mm512_loadu_ps(a->sd16 + (arows[i] * nb + sb * 8) * 2), accc[i]);
  }
  for (int i = 0; i < n; ++i) out[i] = kc_hsum(acc[i]) - 32.0f * kc_hsum(accc[i]);
}

__attribute__((target("avx512f,avx512bw,avx512vl,avx512dq,avx512vnni,fma")))
static void kc_row_q8_0(const uint8_t* row, int64_t nblk, const KcAct* a, const int64_t* arows, int n, float* out) {
  __m512 acc[KC_GROUP], accc[KC_GROUP];
  for (int i = 0; i < n; ++i) acc[i] = accc[i] = _mm512_setzero_ps();
  const __m512i bias = _mm512_set1_epi8((char)0x80);
  const int64_t nb = a->kpad / 32;
  for (int64_t bk = 0; bk < nblk; bk += 2) { /* two 34-byte blocks: 64 values */
    const uint8_t* b0 = row + bk * 34;
    const uint8_t* b1 = b0 + 34;
    const float d0 = kc_h2f((uint16_t)(b0[0] | (b0[1] << 8)));
    const float d1 = bk + 1 < nblk ? kc_h2f((uint16_t)(b1[0] | (b1[1] << 8))) : 0.0f;
    __m256i lo = _mm256_loadu_si256((const __m256i*)(b0 + 2));
    __m256i hi = bk + 1 < nblk ? _mm256_loadu_si256((const __m256i*)(b1 + 2)) : _mm256_setzero_si256();
    /* signed codes + 128 as unsigned bytes; the 128 * sum(activations) comes off below */
    const __m512i w = _mm512_xor_si512(_mm512_inserti64x4(_mm512_castsi256_si512(lo), hi, 1), bias);
    const __m512 wsc = _mm512_insertf32x8(_mm512_set1_ps(d0), _mm256_set1_ps(d1), 1);
    for (int i = 0; i < n; ++i) {
      const __m512i act = _mm512_loadu_si512((const void*)(a->q + arows[i] * a->kpad + bk * 32));
      const __m512i dot = _mm512_dpbusd_epi32(_mm512_setzero_si512(), w, act);
      const __m512 s = _mm512_mul_ps(wsc, _mm512_loadu_ps(a->d8x8 + (arows[i] * nb + bk) * 8));
      acc[i] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(dot), s, acc[i]);
      /* lanes 0 and 8 carry the two blocks' corrections */
      const __m512 corr = _mm512_maskz_mov_ps(0x0101, _mm512_set_ps(0, 0, 0, 0, 0, 0, 0, d1 * a->sd8[arows[i] * nb + bk + 1],
                                                                    0, 0, 0, 0, 0, 0, 0, d0 * a->sd8[arows[i] * nb + bk]));
      accc[i] = _mm512_add_ps(accc[i], corr);
    }
  }
  for (int i = 0; i < n; ++i) out[i] = kc_hsum(acc[i]) - 128.0f * kc_hsum(accc[i]);
}

static int kc_supported(void) {
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
         __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512vnni");
}

/* 1 if this host has the SIMD units the baseline is written for (AVX-512 with VNNI) */
int kc_simd_available(void) { return kc_supported(); }

/* One projection over all routes: out[p, r] = row r of slot ids[p] . act[p / top_k] (fp32),
 * zero rows for ids outside [0, n_slots). Routes of a slot share each decoded row. */
static int kc_project(int type, const uint8_t* const* slots, int64_t n_slots, const KcAct* a, const int32_t* ids,
                      int64_t routes, int64_t top_k, int64_t rows, int64_t cols, float* out) {
  const int64_t rb = type == KC_Q4_K ? cols / 256 * 144 : type == KC_Q6_K ? cols / 256 * 210 : cols / 32 * 34;
  const int64_t nunits = type == KC_Q8_0 ? cols / 32 : cols / 256;
  /* routes grouped by slot */
  int64_t* cnt = (int64_t*)calloc(n_slots + 1, sizeof(int64_t));
  int64_t* order = (int64_t*)malloc(sizeof(int64_t) * (routes > 0 ? routes : 1));
  if (!cnt || !order) {
    free(cnt);
    free(order);
    return -1;
  }
  for (int64_t p = 0; p < routes; ++p) {
    const int32_t e = ids[p];
    if (e >= 0 && e < n_slots) ++cnt[e + 1];
    else memset(out + p * rows, 0, sizeof(float) * rows);
  }
  for (int64_t e = 0; e < n_slots; ++e) cnt[e + 1] += cnt[e];
  int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (n_slots + 1));
  memcpy(fill, cnt, sizeof(int64_t) * (n_slots + 1));
  for (int64_t p = 0; p < routes; ++p) {
    const int32_t e = ids[p];
    if (e >= 0 && e < n_slots) order[fill[e]++] = p;
  }
  free(fill);
  /* work items: (slot, group of KC_GROUP routes, block of 64 rows) */
  const int64_t RB = 64;
  int64_t n_items = 0;
  for (int64_t e = 0; e < n_slots; ++e)
    n_items += (cnt[e + 1] - cnt[e] + KC_GROUP - 1) / KC_GROUP * ((rows + RB - 1) / RB);
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t it = 0; it < n_items; ++it) {
    int64_t rem = it, e = 0;
    for (; e < n_slots; ++e) {
      const int64_t here = (cnt[e + 1] - cnt[e] + KC_GROUP - 1) / KC_GROUP * ((rows + RB - 1) / RB);
      if (rem < here) break;
      rem -= here;
    }
    const int64_t rblocks = (rows + RB - 1) / RB;
    const int64_t grp = rem / rblocks, r0 = (rem % rblocks) * RB;
    const int64_t first = cnt[e] + grp * KC_GROUP;
    const int n = (int)((cnt[e + 1] - first) < KC_GROUP ? (cnt[e + 1] - first) : KC_GROUP);
    int64_t arows[KC_GROUP], prt[KC_GROUP];
    for (int i = 0; i < n; ++i) {
      prt[i] = order[first + i];
      arows[i] = prt[i] / top_k;
    }
    float res[KC_GROUP];
    for (int64_t r = r0; r < r0 + RB && r < rows; ++r) {
      const uint8_t* wrow = slots[e] + r * rb;
      if (type == KC_Q4_K) kc_row_q4_k(wrow, nunits, a, arows, n, res);
      else if (type == KC_Q6_K) kc_row_q6_k(wrow, nunits, a, arows, n, res);
      else kc_row_q8_0(wrow, nunits, a, arows, n, res);
      for (int i = 0; i < n; ++i) out[prt[i] * rows + r] = res[i];
    }
  }
  free(cnt);
  free(order);
  return 0;
}

/*
 * The hot-expert layer of the reference on bf16 activations with the SIMD dot products:
 * q8_1(x) -> gate/up (bf16) -> silu_and_mul (bf16) -> q8_1(h) -> down (bf16) -> combine, the
 * same steps and roundings as ko_moe_ref_bf16. Returns -2 when the host lacks AVX-512 VNNI and
 * -1 for a type without a SIMD dot product here.
 */
int kc_moe_layer(const uint16_t* x, int64_t T, int64_t K, int64_t N, const int32_t* ids, const float* w,
                 int64_t top_k, int type13, const uint8_t* const* w13, int type2, const uint8_t* const* w2,
                 int64_t n_slots, uint16_t* res) {
  if (!kc_supported()) return -2;
  const int ok13 = type13 == KC_Q4_K || type13 == KC_Q6_K || type13 == KC_Q8_0;
  const int ok2 = type2 == KC_Q4_K || type2 == KC_Q6_K || type2 == KC_Q8_0;
  if (!ok13 || !ok2 || K % 256 || N % 256) return -1;
  const int64_t R = T * top_k;
  float* xf = (float*)malloc(sizeof(float) * T * K);
  float* h13f = (float*)malloc(sizeof(float) * R * 2 * N);
  uint16_t* h13 = (uint16_t*)malloc(2 * R * 2 * N);
  uint16_t* h = (uint16_t*)malloc(2 * R * N);
  float* hf = (float*)malloc(sizeof(float) * R * N);
  float* yf = (float*)malloc(sizeof(float) * R * K);
  uint16_t* y = (uint16_t*)malloc(2 * R * K);
  KcAct ax = {0}, ah = {0};
  int rc = -1;
  if (!xf || !h13f || !h13 || !h || !hf || !yf || !y) goto done;
  ko_bf16_to_f32(x, T * K, xf);
  if (kc_act_build(xf, T, K, &ax)) goto done;
  if (kc_project(type13, w13, n_slots, &ax, ids, R, top_k, 2 * N, K, h13f)) goto done;
  ko_f32_to_bf16(h13f, R * 2 * N, h13);
  ko_silu_and_mul_bf16(h13, R, N, h);
  ko_bf16_to_f32(h, R * N, hf);
  if (kc_act_build(hf, R, N, &ah)) goto done;
  if (kc_project(type2, w2, n_slots, &ah, ids, R, 1, K, N, yf)) goto done;
  ko_f32_to_bf16(yf, R * K, y);
  ko_combine_bf16(y, w, T, top_k, K, res);
  rc = 0;
done:
  kc_act_free(&ax);
  kc_act_free(&ah);
  free(xf); free(h13f); free(h13); free(h); free(hf); free(yf); free(y);
  return rc;
}
