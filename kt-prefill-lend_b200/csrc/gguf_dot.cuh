// gguf_dot.cuh — per-chunk integer dot products of one GGUF weight block against q8_1
// activations, and the scalar/vector dequantizers of the four hot-path types.
//
// A "chunk" is the unit one lane handles in the decode GEMV: the same split of a block
// that the reference's vec_dot_*_q8_1 functions use (Q8_0: 8 values, Q4_K: 16 values from
// two sub-blocks, Q6_K: 8 values, IQ3_S: one 32-value sub-block). The integer part of
// every chunk (dp4a sums, scale unpacking, grid lookups, sign handling) is exact; the
// fp32 combination is written in the same expression order as the reference
// (hot/kt_gguf_moe_multi/vecdotq.cuh:969-982, 1326-1367, 1625-1646, 1875-1900).
#pragma once
#include "kt_common.cuh"

template <int TYPE>
struct KtChunk;

// chunks per block and value/byte geometry of the GEMV split
template <>
struct KtChunk<KT_Q8_0> {
  static constexpr int QK = 32, BYTES = 34, CPB = 4, VDR = 2;
};
// 32-value blocks of the legacy family and IQ4_NL: two chunks of 8 nibble pairs per block
// (the reference's VDR 2 over QI 4 ints: values [8c, 8c+8) and [16+8c, 16+8c+8) of chunk c)
template <>
struct KtChunk<KT_Q4_0> {
  static constexpr int QK = 32, BYTES = 18, CPB = 2, VDR = 2;
};
template <>
struct KtChunk<KT_Q4_1> {
  static constexpr int QK = 32, BYTES = 20, CPB = 2, VDR = 2;
};
template <>
struct KtChunk<KT_Q5_0> {
  static constexpr int QK = 32, BYTES = 22, CPB = 2, VDR = 2;
};
template <>
struct KtChunk<KT_Q5_1> {
  static constexpr int QK = 32, BYTES = 24, CPB = 2, VDR = 2;
};
template <>
struct KtChunk<KT_IQ4_NL> {
  static constexpr int QK = 32, BYTES = 18, CPB = 2, VDR = 2;
};
template <>
struct KtChunk<KT_Q4_K> {
  static constexpr int QK = 256, BYTES = 144, CPB = 16, VDR = 2;
};
// K-quants and IQ4_XS with the reference's split: Q2_K / Q3_K one int of 2-bit codes per
// chunk (QI 16, VDR 1), Q5_K two ints (QI 32, VDR 2), IQ4_XS one 32-value sub-block (QI 8)
template <>
struct KtChunk<KT_Q2_K> {
  static constexpr int QK = 256, BYTES = 84, CPB = 16, VDR = 1;
};
template <>
struct KtChunk<KT_Q3_K> {
  static constexpr int QK = 256, BYTES = 110, CPB = 16, VDR = 1;
};
template <>
struct KtChunk<KT_Q5_K> {
  static constexpr int QK = 256, BYTES = 176, CPB = 16, VDR = 2;
};
template <>
struct KtChunk<KT_IQ4_XS> {
  static constexpr int QK = 256, BYTES = 136, CPB = 8, VDR = 1;
};
// Q2_0: 4 bytes of codes (16 values) per chunk against half a q8_1 block (QI 4, VDR 1)
template <>
struct KtChunk<KT_Q2_0> {
  static constexpr int QK = 64, BYTES = 18, CPB = 4, VDR = 1;
};
// the i-quants with a code book: one 32-value sub-block per chunk (QI 8, VDR 1)
template <>
struct KtChunk<KT_IQ2_XXS> {
  static constexpr int QK = 256, BYTES = 66, CPB = 8, VDR = 1;
};
template <>
struct KtChunk<KT_IQ2_XS> {
  static constexpr int QK = 256, BYTES = 74, CPB = 8, VDR = 1;
};
template <>
struct KtChunk<KT_IQ2_S> {
  static constexpr int QK = 256, BYTES = 82, CPB = 8, VDR = 1;
};
template <>
struct KtChunk<KT_IQ3_XXS> {
  static constexpr int QK = 256, BYTES = 98, CPB = 8, VDR = 1;
};
template <>
struct KtChunk<KT_IQ1_S> {
  static constexpr int QK = 256, BYTES = 50, CPB = 8, VDR = 1;
};
template <>
struct KtChunk<KT_IQ1_M> {
  static constexpr int QK = 256, BYTES = 56, CPB = 8, VDR = 1;
};
template <>
struct KtChunk<KT_Q6_K> {
  static constexpr int QK = 256, BYTES = 210, CPB = 32, VDR = 1;
};
template <>
struct KtChunk<KT_IQ3_S> {
  static constexpr int QK = 256, BYTES = 110, CPB = 8, VDR = 1;
};

// Activations reach the dot products in the GEMV's split q8_1 layout: per token row, the
// int8 values of all 32-value blocks (block b at byte 32*b, 16-byte aligned rows), then the
// (d, s) half2 of every block (block b at byte kpad + 4*b). Values and scales are those of
// the reference's q8_1 blocks; only their placement differs. yq / yd point at the first
// q8_1 block a chunk uses.
__device__ __forceinline__ float kt_q8_1_dd(const uint8_t* yd) { return __low2float(*reinterpret_cast<const half2*>(yd)); }

// ---- Q8_0: d_w * d_a * sum(q_w * q_a) over 8 values (iqs in {0,2,4,6})
__device__ __forceinline__ float kt_vd_q8_0(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  int sumi = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) sumi = __dp4a(kt_ld_b2(bx + 2 + 4 * (iqs + i)), kt_ld_b4(yq + 4 * (iqs + i)), sumi);
  const float d80 = kt_h2f(*reinterpret_cast<const uint16_t*>(bx));
  const float d81 = kt_q8_1_dd(yd);
  return d80 * d81 * sumi;
}

// ---- legacy 32-value blocks: chunk iqs in {0, 2} covers the nibble bytes [4iqs, 4iqs+8):
// low nibbles are values 4iqs.., high nibbles values 16+4iqs.. (q8_1 ints iqs+i and iqs+i+4)
__device__ __forceinline__ float2 kt_ds8(const uint8_t* yd) { return __half22float2(*reinterpret_cast<const half2*>(yd)); }

// Q4_0 (d, qs[16]): d * (sum(q * u) * d8 - 4 * s8); the 4 is 8 (the code offset) times this
// chunk's share of the block's sum of activations s8 (2 of 4 ints)
__device__ __forceinline__ float kt_vd_q4_0(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  int sumi = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int v = kt_ld_b2(bx + 2 + 4 * (iqs + i));
    sumi = __dp4a(v & 0x0F0F0F0F, kt_ld_b4(yq + 4 * (iqs + i)), sumi);
    sumi = __dp4a((v >> 4) & 0x0F0F0F0F, kt_ld_b4(yq + 4 * (iqs + i + 4)), sumi);
  }
  const float2 ds8 = kt_ds8(yd);
  return kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (sumi * ds8.x - 4 * ds8.y);
}

// Q4_1 (half2 (d, m), qs[16]): the products d*d8 and m*s8 are formed in half precision, like
// the reference (__hmul2), then sum(q * u) * (d*d8) + (m*s8) / 2 (this chunk's half of m*s8)
__device__ __forceinline__ float kt_vd_q4_1(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  int sumi = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int v = kt_ld_b4(bx + 4 + 4 * (iqs + i));
    sumi = __dp4a(v & 0x0F0F0F0F, kt_ld_b4(yq + 4 * (iqs + i)), sumi);
    sumi = __dp4a((v >> 4) & 0x0F0F0F0F, kt_ld_b4(yq + 4 * (iqs + i + 4)), sumi);
  }
  const float2 t = __half22float2(__hmul2(*reinterpret_cast<const half2*>(bx), *reinterpret_cast<const half2*>(yd)));
  return sumi * t.x + t.y / 2;
}

// fifth bits of the 4 low-nibble (vl) and 4 high-nibble (vh) codes of int i of a Q5 block:
// qh bit 4i+j -> bit 8j+4 of the low word, bit 16+4i+j -> bit 8j+4 of the high word
__device__ __forceinline__ void kt_q5_codes(int ql, int qh, int i, int& lo, int& hi) {
  const int h = qh >> (4 * i);
  lo = (ql & 0x0F0F0F0F) | ((h << 4) & 0x10) | ((h << 11) & 0x1000) | ((h << 18) & 0x100000) | ((h << 25) & 0x10000000);
  hi = ((ql >> 4) & 0x0F0F0F0F) | ((h >> 12) & 0x10) | ((h >> 5) & 0x1000) | ((h << 2) & 0x100000) |
       ((h << 9) & 0x10000000);
}

// Q5_0 (d, qh[4], qs[16]): d * (sum(q * u) * d8 - 8 * s8)
__device__ __forceinline__ float kt_vd_q5_0(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int qh = kt_ld_b2(bx + 2);
  int sumi = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    int lo, hi;
    kt_q5_codes(kt_ld_b2(bx + 6 + 4 * (iqs + i)), qh, iqs + i, lo, hi);
    sumi = __dp4a(lo, kt_ld_b4(yq + 4 * (iqs + i)), sumi);
    sumi = __dp4a(hi, kt_ld_b4(yq + 4 * (iqs + i + 4)), sumi);
  }
  const float2 ds8 = kt_ds8(yd);
  return kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (sumi * ds8.x - 8 * ds8.y);
}

// Q5_1 (half2 (d, m), qh[4], qs[16]): as Q4_1 with 5-bit codes
__device__ __forceinline__ float kt_vd_q5_1(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int qh = kt_ld_b4(bx + 4);
  int sumi = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    int lo, hi;
    kt_q5_codes(kt_ld_b4(bx + 8 + 4 * (iqs + i)), qh, iqs + i, lo, hi);
    sumi = __dp4a(lo, kt_ld_b4(yq + 4 * (iqs + i)), sumi);
    sumi = __dp4a(hi, kt_ld_b4(yq + 4 * (iqs + i + 4)), sumi);
  }
  const float2 t = __half22float2(__hmul2(*reinterpret_cast<const half2*>(bx), *reinterpret_cast<const half2*>(yd)));
  return sumi * t.x + t.y / 2;
}

// the IQ4_NL code book, 16 signed levels (-127 ... 113), four per word as bytes
#define KT_IQ4NL_W0 0xBFAD9881u
#define KT_IQ4NL_W1 0xF6EADDCFu
#define KT_IQ4NL_W2 0x26190D01u
#define KT_IQ4NL_W3 0x71594535u
__device__ __forceinline__ int kt_iq4nl_level(int code) {
  const uint32_t w = code < 4 ? KT_IQ4NL_W0 : code < 8 ? KT_IQ4NL_W1 : code < 12 ? KT_IQ4NL_W2 : KT_IQ4NL_W3;
  return (int)(int8_t)(w >> (8 * (code & 3)));
}
// four codes (the low nibbles of the bytes of n, high nibbles zero) mapped through the code
// book into bytes: the low 3 bits of each code select a byte among the first or the last
// eight levels (two byte permutes), bit 3 picks between them
__device__ __forceinline__ int kt_iq4nl_bytes(uint32_t n) {
  const uint32_t x = n & 0x07070707u, y = x | (x >> 4);
  const uint32_t sel = (y & 0xffu) | ((y >> 8) & 0xff00u);
  const uint32_t lo = __byte_perm(KT_IQ4NL_W0, KT_IQ4NL_W1, sel), hi = __byte_perm(KT_IQ4NL_W2, KT_IQ4NL_W3, sel);
  const uint32_t m = ((n >> 3) & 0x01010101u) * 0xffu;
  return (int)((lo & ~m) | (hi & m));
}

// IQ4_NL (d, qs[16]): d * d8 * (sum over the low-nibble levels + sum over the high ones)
__device__ __forceinline__ float kt_vd_iq4_nl(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  int sumi1 = 0, sumi2 = 0;
#pragma unroll
  for (int l = 0; l < 2; ++l) {
    const uint32_t q = (uint32_t)kt_ld_b2(bx + 2 + 4 * (iqs + l));
    sumi1 = __dp4a(kt_iq4nl_bytes(q & 0x0F0F0F0Fu), kt_ld_b4(yq + 4 * (iqs + l)), sumi1);
    sumi2 = __dp4a(kt_iq4nl_bytes((q >> 4) & 0x0F0F0F0Fu), kt_ld_b4(yq + 4 * (iqs + l + 4)), sumi2);
  }
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * kt_q8_1_dd(yd);
  return d * (sumi1 + sumi2);
}

// ---- Q4_K: 16 values from sub-blocks (bq8_offset, bq8_offset + 1); iqs in {0,2,...,30}
__device__ __forceinline__ float kt_vd_q4_k(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 2 * ((iqs / 2) / 4);
  const uint8_t* q4 = bx + 16 + 16 * bq8_offset + 4 * ((iqs / 2) % 4);
  const int v0 = kt_ld_b4(q4), v1 = kt_ld_b4(q4 + 16);
  const uint16_t* s16 = reinterpret_cast<const uint16_t*>(bx + 4);
  uint16_t aux0, aux1;
  const int j = bq8_offset / 2;
  if (j < 2) {
    aux0 = s16[j + 0] & 0x3f3f;
    aux1 = s16[j + 2] & 0x3f3f;
  } else {
    aux0 = ((s16[j + 2] >> 0) & 0x0f0f) | ((s16[j - 2] & 0xc0c0) >> 2);
    aux1 = ((s16[j + 2] >> 4) & 0x0f0f) | ((s16[j - 0] & 0xc0c0) >> 2);
  }
  float sumf_d = 0.0f, sumf_m = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint8_t* q8 = yq + 32 * (bq8_offset + i);
    const float d8 = kt_q8_1_dd(yd + 4 * (bq8_offset + i));
    const int u0 = kt_ld_b4(q8 + 4 * ((iqs / 2) % 4));
    const int u1 = kt_ld_b4(q8 + 4 * ((iqs / 2) % 4) + 16);
    const int v0i = (v0 >> (4 * i)) & 0x0F0F0F0F;
    const int v1i = (v1 >> (4 * i)) & 0x0F0F0F0F;
    const int dot1 = __dp4a(v1i, u1, __dp4a(v0i, u0, 0));
    const int dot2 = __dp4a(0x01010101, u1, __dp4a(0x01010101, u0, 0));
    const int sc = (i ? (aux0 >> 8) : aux0) & 0xff;
    const int m = (i ? (aux1 >> 8) : aux1) & 0xff;
    sumf_d += d8 * (dot1 * sc);
    sumf_m += d8 * (dot2 * m);
  }
  const float2 dm = __half22float2(*reinterpret_cast<const half2*>(bx));
  return dm.x * sumf_d - dm.y * sumf_m;
}

// ---- Q2_K (scales[16] (scale | min << 4), qs[64], half2 (d, dmin)); iqs in 0..15: int iqs of
// qs holds 4 codes of each of the groups 8(iqs/8) + 2i + (iqs%8)/4 (i = 0..3, bits 2i),
// against int iqs%8 of q8_1 blocks 4(iqs/8) + i
__device__ __forceinline__ float kt_vd_q2_k(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 4 * (iqs / 8);
  const uint8_t* scales = bx + iqs - iqs % 8 + (iqs % 8) / 4;
  const int v = kt_ld_b4(bx + 16 + 4 * iqs);
  float sumf_d = 0.0f, sumf_m = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int u = kt_ld_b4(yq + 32 * (bq8_offset + i) + 4 * (iqs % 8));
    const float d8 = kt_q8_1_dd(yd + 4 * (bq8_offset + i));
    const int sc = scales[2 * i];
    sumf_d += d8 * (__dp4a((v >> (2 * i)) & 0x03030303, u, 0) * (sc & 0xF));
    sumf_m += d8 * __dp4a((sc >> 4) * 0x01010101, u, 0);  // the min in every byte
  }
  const float2 dm = __half22float2(*reinterpret_cast<const half2*>(bx + 80));
  return dm.x * sumf_d - dm.y * sumf_m;
}

// ---- Q3_K (hmask[32], qs[64], scales[12] (16 6-bit scales), d); iqs in 0..15: low 2 bits
// from int iqs of qs, the third bit (inverted: 0 -> -4) from int iqs%8 of hmask
__device__ __forceinline__ float kt_vd_q3_k(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 4 * (iqs / 8);
  const int scale_offset = iqs - iqs % 8 + (iqs % 8) / 4;
  const uint8_t* scales = bx + 96;
  const int vl = kt_ld_b2(bx + 32 + 4 * iqs);
  const int vh = ~kt_ld_b2(bx + 4 * (iqs % 8)) >> bq8_offset;
  float sumf = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int isc = scale_offset + 2 * i;
    const int sc_low = (scales[isc % 8] >> (4 * (isc / 8))) & 0xF;
    const int sc_high = ((scales[8 + isc % 4] >> (2 * (isc / 4))) & 3) << 4;
    const int sc = (sc_low | sc_high) - 32;
    const int vi = __vsubss4((vl >> (2 * i)) & 0x03030303, ((vh >> i) << 2) & 0x04040404);
    const int u = kt_ld_b4(yq + 32 * (bq8_offset + i) + 4 * (iqs % 8));
    sumf += kt_q8_1_dd(yd + 4 * (bq8_offset + i)) * (__dp4a(vi, u, 0) * sc);
  }
  return kt_h2f(*reinterpret_cast<const uint16_t*>(bx + 108)) * sumf;
}

// ---- Q5_K (half2 (d, dmin), scales[12], qh[32], qs[128]): as Q4_K, with the fifth bit of
// each code from qh (bit bq8_offset + i of the byte of the code's position)
__device__ __forceinline__ float kt_vd_q5_k(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 2 * ((iqs / 2) / 4);
  const uint8_t* ql = bx + 48 + 16 * bq8_offset + 4 * ((iqs / 2) % 4);
  const uint8_t* qh = bx + 16 + 4 * ((iqs / 2) % 4);
  const int vl0 = kt_ld_b4(ql), vl1 = kt_ld_b4(ql + 16);
  const int vh0 = kt_ld_b4(qh) >> bq8_offset, vh1 = kt_ld_b4(qh + 16) >> bq8_offset;
  const uint16_t* s16 = reinterpret_cast<const uint16_t*>(bx + 4);
  uint16_t aux0, aux1;
  const int j = bq8_offset / 2;
  if (j < 2) {
    aux0 = s16[j + 0] & 0x3f3f;
    aux1 = s16[j + 2] & 0x3f3f;
  } else {
    aux0 = ((s16[j + 2] >> 0) & 0x0f0f) | ((s16[j - 2] & 0xc0c0) >> 2);
    aux1 = ((s16[j + 2] >> 4) & 0x0f0f) | ((s16[j - 0] & 0xc0c0) >> 2);
  }
  float sumf_d = 0.0f, sumf_m = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint8_t* q8 = yq + 32 * (bq8_offset + i) + 4 * ((iqs / 2) % 4);
    const int u0 = kt_ld_b4(q8), u1 = kt_ld_b4(q8 + 16);
    const int v0 = ((vl0 >> (4 * i)) & 0x0F0F0F0F) | (((vh0 >> i) << 4) & 0x10101010);
    const int v1 = ((vl1 >> (4 * i)) & 0x0F0F0F0F) | (((vh1 >> i) << 4) & 0x10101010);
    const int dot1 = __dp4a(v0, u0, __dp4a(v1, u1, 0));
    const int dot2 = __dp4a(0x01010101, u0, __dp4a(0x01010101, u1, 0));
    const float d8 = kt_q8_1_dd(yd + 4 * (bq8_offset + i));
    const int sc = (aux0 >> (8 * i)) & 0xff, m = (aux1 >> (8 * i)) & 0xff;
    sumf_d += d8 * (dot1 * sc);
    sumf_m += d8 * (dot2 * m);
  }
  const float2 dm = __half22float2(*reinterpret_cast<const half2*>(bx));
  return dm.x * sumf_d - dm.y * sumf_m;
}

// ---- IQ4_XS (d, scales_h (2 bits per sub-block), scales_l[4] (4 bits), qs[128]); chunk =
// sub-block ib32: d * (ls - 32) * d8 * (sum over the low-nibble levels + the high ones)
__device__ __forceinline__ float kt_vd_iq4_xs(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32) {
  const uint8_t* q8 = yq + 32 * ib32;
  const uint8_t* q4 = bx + 8 + 16 * ib32;
  const int scales_h = bx[2] | (bx[3] << 8);
  const int ls = ((bx[4 + ib32 / 2] >> (4 * (ib32 % 2))) & 0xf) | (((scales_h >> (2 * ib32)) & 3) << 4);
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (ls - 32) * kt_q8_1_dd(yd + 4 * ib32);
  int sumi1 = 0, sumi2 = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t q = (uint32_t)kt_ld_b4(q4 + 4 * j);
    sumi1 = __dp4a(kt_iq4nl_bytes(q & 0x0F0F0F0Fu), kt_ld_b4(q8 + 4 * j), sumi1);
    sumi2 = __dp4a(kt_iq4nl_bytes((q >> 4) & 0x0F0F0F0Fu), kt_ld_b4(q8 + 16 + 4 * j), sumi2);
  }
  return d * (sumi1 + sumi2);
}

// ---- Q2_0 (fp16 d, qs[16]: byte b holds elements 4b..4b+3, code s at bits 2s; value
// d*(code-1)); chunk iqs 0..3 = bytes 4iqs..4iqs+3 against half iqs&1 of q8_1 block iqs/2.
// The -1 is taken as sum(code*u) - sum(u) so that no byte of a packed int borrows.
__device__ __forceinline__ float kt_vd_q2_0(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const uint8_t* q = bx + 2 + 4 * iqs;
  const uint8_t* u = yq + 32 * (iqs >> 1) + 16 * (iqs & 1);
  int sumi = 0, sumy = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int c = q[b];
    const int codes = (c | (c << 6) | (c << 12) | (c << 18)) & 0x03030303;  // code s -> byte s
    const int ub = kt_ld_b4(u + 4 * b);
    sumi = __dp4a(codes, ub, sumi);
    sumy = __dp4a(0x01010101, ub, sumy);
  }
  return kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * kt_q8_1_dd(yd + 4 * (iqs >> 1)) * (float)(sumi - sumy);
}

// ---- i-quants with a code book (grid: the type's book staged in shared memory)

// 7 stored sign bits + the parity bit that makes the count of minus signs even (ggml's
// ksigns_iq2xs table, computed)
__device__ __forceinline__ uint32_t kt_signs8(uint32_t s7) { return s7 | ((__popc(s7) & 1u) << 7); }
// four magnitudes (one per byte) with the signs of bits 0..3 of s4 applied
__device__ __forceinline__ int kt_signed4(uint32_t mag, uint32_t s4) {
  const uint32_t m = __vcmpne4((s4 * 0x01010101u) & 0x08040201u, 0u);  // 0xff where negative
  return (int)__vsub4(mag ^ m, m);
}

// IQ2_XXS (d, qs[32] u16): sub-block ib32 = 4 grid bytes + a word of 4x7 sign bits and a
// 4-bit scale: d * (0.5 + s) * d8 / 4 * sum(+-grid * u)
__device__ __forceinline__ float kt_vd_iq2_xxs(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                               const uint32_t* grid) {
  const uint8_t* q2 = bx + 2 + 8 * ib32;
  const uint8_t* q8 = yq + 32 * ib32;
  const uint32_t aux32 = (uint32_t)kt_ld_b2(q2 + 4);
  int sumi = 0;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t* g = grid + 2 * q2[l];
    const uint32_t s = kt_signs8((aux32 >> (7 * l)) & 127u);
    sumi = __dp4a(kt_signed4(g[0], s & 15u), kt_ld_b4(q8 + 8 * l), sumi);
    sumi = __dp4a(kt_signed4(g[1], s >> 4), kt_ld_b4(q8 + 8 * l + 4), sumi);
  }
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (0.5f + (aux32 >> 28)) * kt_q8_1_dd(yd + 4 * ib32) *
                  0.25f;
  return d * sumi;
}

// IQ2_XS (d, qs[32] u16: 9-bit grid index | 7 sign bits << 9, scales[8] two 4-bit scales)
__device__ __forceinline__ float kt_vd_iq2_xs(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                              const uint32_t* grid) {
  const uint8_t* q2 = bx + 2 + 8 * ib32;
  const uint8_t* q8 = yq + 32 * ib32;
  const uint8_t ls1 = bx[66 + ib32] & 0xf, ls2 = bx[66 + ib32] >> 4;
  int sumi1 = 0, sumi2 = 0;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t code = q2[2 * l] | (q2[2 * l + 1] << 8);
    const uint32_t* g = grid + 2 * (code & 511u);
    const uint32_t s = kt_signs8(code >> 9);
    int& sumi = l < 2 ? sumi1 : sumi2;
    sumi = __dp4a(kt_signed4(g[0], s & 15u), kt_ld_b4(q8 + 8 * l), sumi);
    sumi = __dp4a(kt_signed4(g[1], s >> 4), kt_ld_b4(q8 + 8 * l + 4), sumi);
  }
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * kt_q8_1_dd(yd + 4 * ib32) * 0.25f;
  return d * ((0.5f + ls1) * sumi1 + (0.5f + ls2) * sumi2);
}

// IQ2_S (d, qs[32] grid low bits, signs[32], qh[8] 2 high bits per group, scales[8])
__device__ __forceinline__ float kt_vd_iq2_s(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                             const uint32_t* grid) {
  const uint8_t* qs = bx + 2 + 4 * ib32;
  const uint8_t* signs = bx + 34 + 4 * ib32;
  const uint8_t* q8 = yq + 32 * ib32;
  const int qh = bx[66 + ib32];
  const uint8_t ls1 = bx[74 + ib32] & 0xf, ls2 = bx[74 + ib32] >> 4;
  int sumi1 = 0, sumi2 = 0;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t* g = grid + 2 * (qs[l] | ((qh << (8 - 2 * l)) & 0x300));
    const uint32_t s = signs[l];
    int& sumi = l < 2 ? sumi1 : sumi2;
    sumi = __dp4a(kt_signed4(g[0], s & 15u), kt_ld_b4(q8 + 8 * l), sumi);
    sumi = __dp4a(kt_signed4(g[1], s >> 4), kt_ld_b4(q8 + 8 * l + 4), sumi);
  }
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * kt_q8_1_dd(yd + 4 * ib32) * 0.25f;
  return d * ((0.5f + ls1) * sumi1 + (0.5f + ls2) * sumi2);
}

// IQ3_XXS (d, qs[64] grid indices, 8 words of 4x7 sign bits | 4-bit scale << 28)
__device__ __forceinline__ float kt_vd_iq3_xxs(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                               const uint32_t* grid) {
  const uint8_t* q3 = bx + 2 + 8 * ib32;
  const uint8_t* q8 = yq + 32 * ib32;
  const uint32_t aux32 = (uint32_t)kt_ld_b2(bx + 66 + 4 * ib32);
  int sumi = 0;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t s = kt_signs8((aux32 >> (7 * l)) & 127u);
    sumi = __dp4a(kt_signed4(grid[q3[2 * l]], s & 15u), kt_ld_b4(q8 + 8 * l), sumi);
    sumi = __dp4a(kt_signed4(grid[q3[2 * l + 1]], s >> 4), kt_ld_b4(q8 + 8 * l + 4), sumi);
  }
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (0.5f + (aux32 >> 28)) * kt_q8_1_dd(yd + 4 * ib32) *
                  0.5f;
  return d * sumi;
}

// IQ1 delta: values are grid + delta, delta = +-1/8 by a sign bit
#define KT_IQ1_DELTA 0.125f

// IQ1_S (d, qs[32], qh[8] u16: 3 high index bits per group, 3-bit scale, delta sign). The
// book holds v + 1 in nibbles, so sum(v*u) = sum((v+1)*u) - sum(u): the q8_1 block's s
// (sum of the unquantized activations) times delta - 1 stands for the -sum(u) + delta*sum(u)
__device__ __forceinline__ float kt_vd_iq1_s(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                             const uint32_t* grid) {
  const uint8_t* qs = bx + 2 + 4 * ib32;
  const uint8_t* q8 = yq + 32 * ib32;
  const int qh = bx[34 + 2 * ib32] | (bx[35 + 2 * ib32] << 8);
  int sumi = 0;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t w = grid[qs[l] | (((qh >> (3 * l)) & 7) << 8)];
    sumi = __dp4a((int)(w & 0x0F0F0F0Fu), kt_ld_b4(q8 + 8 * l), sumi);
    sumi = __dp4a((int)((w >> 4) & 0x0F0F0F0Fu), kt_ld_b4(q8 + 8 * l + 4), sumi);
  }
  const float d1q = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (((qh >> 11) & 0x0E) + 1);
  const float delta = -1.0f + KT_IQ1_DELTA - (qh & 0x8000) * (2.0f * KT_IQ1_DELTA / 0x8000);
  const float2 ds = __half22float2(*reinterpret_cast<const half2*>(yd + 4 * ib32));
  return d1q * (ds.x * sumi + ds.y * delta);
}

// IQ1_M (qs[32], qh[16]: per group 3 high index bits + delta sign, scales[8]: 3-bit scales
// per 16 values, and the fp16 d spread over the top nibbles of the four scale words)
__device__ __forceinline__ float kt_vd_iq1_m(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                             const uint32_t* grid) {
  const uint8_t* qs = bx + 4 * ib32;
  const uint8_t* q8 = yq + 32 * ib32;
  int sumi[2] = {0, 0};
  float sumf[2] = {0.0f, 0.0f};
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const int qhl = bx[32 + 2 * ib32 + l / 2] >> (4 * (l % 2));
    const uint32_t w = grid[qs[l] | ((qhl & 7) << 8)];
    const int u0 = kt_ld_b4(q8 + 8 * l), u1 = kt_ld_b4(q8 + 8 * l + 4);
    sumi[l / 2] = __dp4a((int)(w & 0x0F0F0F0Fu), u0, sumi[l / 2]);
    sumi[l / 2] = __dp4a((int)((w >> 4) & 0x0F0F0F0Fu), u1, sumi[l / 2]);
    const float delta = -1.0f + KT_IQ1_DELTA - (qhl & 0x08) * (2.0f * KT_IQ1_DELTA / 0x08);
    int sumy = 0;
    sumy = __dp4a(u0, 0x01010101, sumy);
    sumy = __dp4a(u1, 0x01010101, sumy);
    sumf[l / 2] += delta * sumy;
  }
  const uint8_t* s8 = bx + 48;
  uint16_t sc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) sc[k] = (uint16_t)(s8[2 * k] | (s8[2 * k + 1] << 8));
  const uint16_t dbits = (sc[0] >> 12) | ((sc[1] >> 8) & 0x00F0) | ((sc[2] >> 4) & 0x0F00) | (sc[3] & 0xF000);
  const float d = kt_h2f(dbits) * kt_q8_1_dd(yd + 4 * ib32);
  const int tmp = sc[ib32 / 2] >> (6 * (ib32 % 2));
  const int sc0 = 2 * ((tmp >> 0) & 0x07) + 1;
  const int sc1 = 2 * ((tmp >> 3) & 0x07) + 1;
  return d * ((sumi[0] + sumf[0]) * sc0 + (sumi[1] + sumf[1]) * sc1);
}

// ---- Q6_K: 8 values; iqs in 0..31. The reference's per-byte (code - 32) with __vsubss4
// never saturates (codes are 0..63), so the integer dot is dp4a(code, u) - 32 * sum(u),
// computed here with two dp4a instead of the emulated SIMD subtract.
__device__ __forceinline__ float kt_vd_q6_k(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 4 * (iqs / 16) + (iqs % 16) / 8;
  const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
  const int vh_shift = 2 * ((iqs % 16) / 8);
  const int vl = kt_ld_b2(bx + 4 * iqs);
  const int vh = kt_ld_b2(bx + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift;
  const int8_t* scales = reinterpret_cast<const int8_t*>(bx + 192 + scale_offset);
  float sumf = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int u = kt_ld_b4(yq + 32 * (bq8_offset + 2 * i) + 4 * (iqs % 8));
    const float d8 = kt_q8_1_dd(yd + 4 * (bq8_offset + 2 * i));
    const int sc = scales[4 * i];
    const int vil = (vl >> (4 * i)) & 0x0F0F0F0F;
    const int vih = ((vh >> (4 * i)) << 4) & 0x30303030;
    const int dot = __dp4a(vil | vih, u, 0) - 32 * __dp4a(0x01010101, u, 0);
    sumf += d8 * (dot * sc);
  }
  return kt_h2f(*reinterpret_cast<const uint16_t*>(bx + 208)) * sumf;
}

// byte j of the result is 0xFF when bit j of the nibble n is set (n < 16): the multiply
// moves bit j to bit 8j, no carries
__device__ __forceinline__ uint32_t kt_nibble_mask(uint32_t n) { return ((n * 0x00204081u) & 0x01010101u) * 0xffu; }

// ---- IQ3_S: one 32-value sub-block (ib32 = iqs in 0..7); `grid` is the 512-entry codebook
// in shared memory. The reference applies the signs per byte ((g ^ s) - s) before one dp4a
// chain; the same integer is sum(g * q) - 2 * sum((g & s) * q), two plain dp4a chains
// (grid magnitudes are < 128), with the byte masks s built from the sign bits in registers.
__device__ __forceinline__ float kt_vd_iq3_s(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int ib32,
                                             const uint32_t* grid) {
  yq += 32 * ib32;
  yd += 4 * ib32;
  const uint32_t qs0 = (uint32_t)kt_ld_b2(bx + 2 + 8 * ib32), qs1 = (uint32_t)kt_ld_b2(bx + 6 + 8 * ib32);
  const uint32_t qh = bx[66 + ib32];
  const uint32_t sg = (uint32_t)kt_ld_b2(bx + 74 + 4 * ib32);
  const int4 a0 = *reinterpret_cast<const int4*>(yq);
  const int4 a1 = *reinterpret_cast<const int4*>(yq + 16);
  const int q[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  int sum_all = 0, sum_neg = 0;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t w = l < 2 ? qs0 : qs1;
    const uint32_t b1 = (w >> (16 * (l & 1))) & 0xff, b2 = (w >> (16 * (l & 1) + 8)) & 0xff;
    const int g1 = (int)grid[b1 | ((qh << (8 - 2 * l)) & 256)];
    const int g2 = (int)grid[b2 | ((qh << (7 - 2 * l)) & 256)];
    const uint32_t sb = sg >> (8 * l);
    const int m1 = (int)kt_nibble_mask(sb & 15), m2 = (int)kt_nibble_mask((sb >> 4) & 15);
    sum_all = __dp4a(g1, q[2 * l], sum_all);
    sum_all = __dp4a(g2, q[2 * l + 1], sum_all);
    sum_neg = __dp4a(g1 & m1, q[2 * l], sum_neg);
    sum_neg = __dp4a(g2 & m2, q[2 * l + 1], sum_neg);
  }
  const int sumi = sum_all - 2 * sum_neg;
  const float d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (1 + 2 * ((bx[106 + ib32 / 2] >> 4 * (ib32 % 2)) & 0xf)) *
                  kt_q8_1_dd(yd);
  return d * sumi;
}

template <int TYPE>
__device__ __forceinline__ float kt_vec_dot(const uint8_t* bx, const uint8_t* yq, const uint8_t* yd, int iqs,
                                            const uint32_t* grid) {
  if constexpr (TYPE == KT_Q8_0) return kt_vd_q8_0(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q4_0) return kt_vd_q4_0(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q4_1) return kt_vd_q4_1(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q5_0) return kt_vd_q5_0(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q5_1) return kt_vd_q5_1(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_IQ4_NL) return kt_vd_iq4_nl(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q2_K) return kt_vd_q2_k(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q3_K) return kt_vd_q3_k(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q5_K) return kt_vd_q5_k(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_IQ4_XS) return kt_vd_iq4_xs(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q2_0) return kt_vd_q2_0(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_IQ2_XXS) return kt_vd_iq2_xxs(bx, yq, yd, iqs, grid);
  if constexpr (TYPE == KT_IQ2_XS) return kt_vd_iq2_xs(bx, yq, yd, iqs, grid);
  if constexpr (TYPE == KT_IQ2_S) return kt_vd_iq2_s(bx, yq, yd, iqs, grid);
  if constexpr (TYPE == KT_IQ3_XXS) return kt_vd_iq3_xxs(bx, yq, yd, iqs, grid);
  if constexpr (TYPE == KT_IQ1_S) return kt_vd_iq1_s(bx, yq, yd, iqs, grid);
  if constexpr (TYPE == KT_IQ1_M) return kt_vd_iq1_m(bx, yq, yd, iqs, grid);
  if constexpr (TYPE == KT_Q4_K) return kt_vd_q4_k(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_Q6_K) return kt_vd_q6_k(bx, yq, yd, iqs);
  if constexpr (TYPE == KT_IQ3_S) return kt_vd_iq3_s(bx, yq, yd, iqs, grid);
  return 0.0f;
}

// ------------------------------------------------------------------ member-stationary split
// The chunk dot products of the north-star types cut in two: KtAct<TYPE> holds a chunk's
// activation side for one member (q8_1 ints, the block scale, and the integer sums of the
// q8_1 values that do not depend on the weights), KtWgt<TYPE> a chunk's weight side for one
// row (codes, scales). kt_dot_split(w, a) evaluates the chunk's fp32 expression exactly as
// kt_vec_dot does, so a kernel can load each member's side once for all its rows and each
// row's side once for all its members and still produce the reference's sums bit for bit.
template <int TYPE>
struct KtAct;
template <int TYPE>
struct KtWgt;

template <>
struct KtAct<KT_Q8_0> {
  int u[2];
  float d;
};
template <>
struct KtWgt<KT_Q8_0> {
  int v[2];
  float d;
};
__device__ __forceinline__ void kt_act_load(KtAct<KT_Q8_0>& a, const uint8_t* yq, const uint8_t* yd, int iqs) {
#pragma unroll
  for (int i = 0; i < 2; ++i) a.u[i] = kt_ld_b4(yq + 4 * (iqs + i));
  a.d = kt_q8_1_dd(yd);
}
__device__ __forceinline__ void kt_wgt_load(KtWgt<KT_Q8_0>& w, const uint8_t* bx, int iqs, const uint32_t*) {
#pragma unroll
  for (int i = 0; i < 2; ++i) w.v[i] = kt_ld_b2(bx + 2 + 4 * (iqs + i));
  w.d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx));
}
__device__ __forceinline__ float kt_dot_split(const KtWgt<KT_Q8_0>& w, const KtAct<KT_Q8_0>& a) {
  int sumi = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) sumi = __dp4a(w.v[i], a.u[i], sumi);
  return w.d * a.d * sumi;  // kt_vd_q8_0: d80 * d81 * sumi
}

template <>
struct KtAct<KT_Q4_K> {
  int u0[2], u1[2], s[2];  // s: sum of the chunk's 8 q8_1 values of block bq8_offset + i
  float d8[2];
};
template <>
struct KtWgt<KT_Q4_K> {
  int v0[2], v1[2], sc[2], m[2];
  float dx, dy;
};
__device__ __forceinline__ void kt_act_load(KtAct<KT_Q4_K>& a, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 2 * ((iqs / 2) / 4);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint8_t* q8 = yq + 32 * (bq8_offset + i);
    a.d8[i] = kt_q8_1_dd(yd + 4 * (bq8_offset + i));
    a.u0[i] = kt_ld_b4(q8 + 4 * ((iqs / 2) % 4));
    a.u1[i] = kt_ld_b4(q8 + 4 * ((iqs / 2) % 4) + 16);
    a.s[i] = __dp4a(0x01010101, a.u1[i], __dp4a(0x01010101, a.u0[i], 0));
  }
}
__device__ __forceinline__ void kt_wgt_load(KtWgt<KT_Q4_K>& w, const uint8_t* bx, int iqs, const uint32_t*) {
  const int bq8_offset = 2 * ((iqs / 2) / 4);
  const uint8_t* q4 = bx + 16 + 16 * bq8_offset + 4 * ((iqs / 2) % 4);
  const int v0 = kt_ld_b4(q4), v1 = kt_ld_b4(q4 + 16);
  const uint16_t* s16 = reinterpret_cast<const uint16_t*>(bx + 4);
  uint16_t aux0, aux1;
  const int j = bq8_offset / 2;
  if (j < 2) {
    aux0 = s16[j + 0] & 0x3f3f;
    aux1 = s16[j + 2] & 0x3f3f;
  } else {
    aux0 = ((s16[j + 2] >> 0) & 0x0f0f) | ((s16[j - 2] & 0xc0c0) >> 2);
    aux1 = ((s16[j + 2] >> 4) & 0x0f0f) | ((s16[j - 0] & 0xc0c0) >> 2);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    w.v0[i] = (v0 >> (4 * i)) & 0x0F0F0F0F;
    w.v1[i] = (v1 >> (4 * i)) & 0x0F0F0F0F;
    w.sc[i] = (i ? (aux0 >> 8) : aux0) & 0xff;
    w.m[i] = (i ? (aux1 >> 8) : aux1) & 0xff;
  }
  const float2 dm = __half22float2(*reinterpret_cast<const half2*>(bx));
  w.dx = dm.x;
  w.dy = dm.y;
}
__device__ __forceinline__ float kt_dot_split(const KtWgt<KT_Q4_K>& w, const KtAct<KT_Q4_K>& a) {
  float sumf_d = 0.0f, sumf_m = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int dot1 = __dp4a(w.v1[i], a.u1[i], __dp4a(w.v0[i], a.u0[i], 0));
    sumf_d += a.d8[i] * (dot1 * w.sc[i]);
    sumf_m += a.d8[i] * (a.s[i] * w.m[i]);
  }
  return w.dx * sumf_d - w.dy * sumf_m;
}

template <>
struct KtAct<KT_Q6_K> {
  int u[2], s[2];
  float d8[2];
};
template <>
struct KtWgt<KT_Q6_K> {
  int q[2], sc[2];
  float d;
};
__device__ __forceinline__ void kt_act_load(KtAct<KT_Q6_K>& a, const uint8_t* yq, const uint8_t* yd, int iqs) {
  const int bq8_offset = 4 * (iqs / 16) + (iqs % 16) / 8;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    a.u[i] = kt_ld_b4(yq + 32 * (bq8_offset + 2 * i) + 4 * (iqs % 8));
    a.d8[i] = kt_q8_1_dd(yd + 4 * (bq8_offset + 2 * i));
    a.s[i] = __dp4a(0x01010101, a.u[i], 0);
  }
}
__device__ __forceinline__ void kt_wgt_load(KtWgt<KT_Q6_K>& w, const uint8_t* bx, int iqs, const uint32_t*) {
  const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
  const int vh_shift = 2 * ((iqs % 16) / 8);
  const int vl = kt_ld_b2(bx + 4 * iqs);
  const int vh = kt_ld_b2(bx + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift;
  const int8_t* scales = reinterpret_cast<const int8_t*>(bx + 192 + scale_offset);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    w.q[i] = ((vl >> (4 * i)) & 0x0F0F0F0F) | (((vh >> (4 * i)) << 4) & 0x30303030);
    w.sc[i] = scales[4 * i];
  }
  w.d = kt_h2f(*reinterpret_cast<const uint16_t*>(bx + 208));
}
__device__ __forceinline__ float kt_dot_split(const KtWgt<KT_Q6_K>& w, const KtAct<KT_Q6_K>& a) {
  float sumf = 0.0f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int dot = __dp4a(w.q[i], a.u[i], 0) - 32 * a.s[i];
    sumf += a.d8[i] * (dot * w.sc[i]);
  }
  return w.d * sumf;
}

template <>
struct KtAct<KT_IQ3_S> {
  int q[8];
  float d8;
};
template <>
struct KtWgt<KT_IQ3_S> {
  int g[8], m[8];
  float dsc;  // d * (1 + 2 * scale)
};
__device__ __forceinline__ void kt_act_load(KtAct<KT_IQ3_S>& a, const uint8_t* yq, const uint8_t* yd, int ib32) {
  const int4 a0 = *reinterpret_cast<const int4*>(yq + 32 * ib32);
  const int4 a1 = *reinterpret_cast<const int4*>(yq + 32 * ib32 + 16);
  a.q[0] = a0.x, a.q[1] = a0.y, a.q[2] = a0.z, a.q[3] = a0.w;
  a.q[4] = a1.x, a.q[5] = a1.y, a.q[6] = a1.z, a.q[7] = a1.w;
  a.d8 = kt_q8_1_dd(yd + 4 * ib32);
}
__device__ __forceinline__ void kt_wgt_load(KtWgt<KT_IQ3_S>& w, const uint8_t* bx, int ib32, const uint32_t* grid) {
  const uint32_t qs0 = (uint32_t)kt_ld_b2(bx + 2 + 8 * ib32), qs1 = (uint32_t)kt_ld_b2(bx + 6 + 8 * ib32);
  const uint32_t qh = bx[66 + ib32];
  const uint32_t sg = (uint32_t)kt_ld_b2(bx + 74 + 4 * ib32);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t wd = l < 2 ? qs0 : qs1;
    const uint32_t b1 = (wd >> (16 * (l & 1))) & 0xff, b2 = (wd >> (16 * (l & 1) + 8)) & 0xff;
    w.g[2 * l] = (int)grid[b1 | ((qh << (8 - 2 * l)) & 256)];
    w.g[2 * l + 1] = (int)grid[b2 | ((qh << (7 - 2 * l)) & 256)];
    const uint32_t sb = sg >> (8 * l);
    w.m[2 * l] = (int)kt_nibble_mask(sb & 15);
    w.m[2 * l + 1] = (int)kt_nibble_mask((sb >> 4) & 15);
  }
  w.dsc = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (1 + 2 * ((bx[106 + ib32 / 2] >> 4 * (ib32 % 2)) & 0xf));
}
__device__ __forceinline__ float kt_dot_split(const KtWgt<KT_IQ3_S>& w, const KtAct<KT_IQ3_S>& a) {
  int sum_all = 0, sum_neg = 0;
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    sum_all = __dp4a(w.g[l], a.q[l], sum_all);
    sum_neg = __dp4a(w.g[l] & w.m[l], a.q[l], sum_neg);
  }
  const int sumi = sum_all - 2 * sum_neg;
  const float d = w.dsc * a.d8;
  return d * sumi;
}

// IQ3_S weight side that reads a 32 KB signed code book in shared memory instead of the 512-word
// grid plus sign masks built per lookup. It produces each chunk's signed codes, whose dp4a chain
// is the same integer as the reference's ((g ^ s) - s) chain, so the chunk's fp32 expression and
// every route's result are unchanged bit for bit. (Grid bytes are odd, 1..15, so the bytewise
// negation (g ^ m) + (m & 0x01010101) never carries.)
//
// KtWgtS3, the signed book: entry (q | nib << 8 | h << 12) = the grid word of the 9-bit index
// (q | h << 8) with byte j negated where bit j of the sign nibble nib is set. The eight 13-bit
// entry indices come from the chunk's bytes with byte permutes: the sign nibbles and the ninth
// index bits are merged into one byte per lookup, then paired with the code bytes into 16-bit
// halves. One lookup per 4 values and no sign work. (A 512-word grid replicated for 16 lane
// columns, with conflict-free lookups and the signs applied in registers, measured no faster than
// the plain grid on config 3.)
constexpr int kIq3sBookWords = 8192;
__device__ __forceinline__ void kt_stage_iq3s_signed(uint32_t* tab, int tid, int nthreads) {
  for (int e = tid; e < kIq3sBookWords; e += nthreads) {
    const uint32_t g = kt_iq3s_grid_dev[(e & 255) | ((e >> 12) << 8)];
    const uint32_t m = kt_nibble_mask((e >> 8) & 15);
    tab[e] = (g ^ m) + (m & 0x01010101u);
  }
}
struct KtWgtS3 {
  int g[8];   // signed codes of the chunk's eight 4-value groups
  float dsc;  // d * (1 + 2 * scale)
};
__device__ __forceinline__ void kt_wgt_load(KtWgtS3& w, const uint8_t* bx, int ib32, const uint32_t* tab) {
  const uint32_t qs0 = (uint32_t)kt_ld_b2(bx + 2 + 8 * ib32), qs1 = (uint32_t)kt_ld_b2(bx + 6 + 8 * ib32);
  const uint32_t qh = bx[66 + ib32];
  const uint32_t sg = (uint32_t)kt_ld_b2(bx + 74 + 4 * ib32);
  // byte l of ce / co: the sign nibble and the ninth index bit of lookup 2l / 2l+1 (bit 4 of the
  // byte = bit 2l / 2l+1 of qh, spread by one multiply; its stray carries land on odd bits that
  // the mask drops)
  const uint32_t he = ((qh & 0x55u) * 0x00410410u) & 0x10101010u;
  const uint32_t ho = (((qh >> 1) & 0x55u) * 0x00410410u) & 0x10101010u;
  const uint32_t ce = (sg & 0x0f0f0f0fu) | he;
  const uint32_t co = ((sg >> 4) & 0x0f0f0f0fu) | ho;
  const uint32_t x = __byte_perm(ce, co, 0x5140), y = __byte_perm(ce, co, 0x7362);  // [ce_l, co_l] pairs
  const uint32_t e[4] = {__byte_perm(qs0, x, 0x5140), __byte_perm(qs0, x, 0x7362), __byte_perm(qs1, y, 0x5140),
                         __byte_perm(qs1, y, 0x7362)};
#pragma unroll
  for (int l = 0; l < 4; ++l) {  // e[l]: the entries of lookups 2l (low half) and 2l+1 (high half)
    w.g[2 * l] = (int)tab[e[l] & 0xffffu];
    w.g[2 * l + 1] = (int)tab[e[l] >> 16];
  }
  w.dsc = kt_h2f(*reinterpret_cast<const uint16_t*>(bx)) * (1 + 2 * ((bx[106 + ib32 / 2] >> 4 * (ib32 % 2)) & 0xf));
}

template <typename W>
__device__ __forceinline__ float kt_dot_signed(const W& w, const KtAct<KT_IQ3_S>& a) {
  int sumi = 0;
#pragma unroll
  for (int l = 0; l < 8; ++l) sumi = __dp4a(w.g[l], a.q[l], sumi);
  const float d = w.dsc * a.d8;
  return d * sumi;
}
__device__ __forceinline__ float kt_dot_split(const KtWgtS3& w, const KtAct<KT_IQ3_S>& a) { return kt_dot_signed(w, a); }

// ------------------------------------------------------------------ dequantization
// Each function writes the fp32 values of 32 consecutive elements [32*sub, 32*sub + 32)
// of one block, with ggml's operation order (products that are exact in fp32 first, one
// rounding at the end), so the values are bit-identical to ggml / gguf-py.

__device__ __forceinline__ void kt_dq32_q8_0(const uint8_t* b, float* y) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
#pragma unroll
  for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
}

__device__ __forceinline__ void kt_q4k_scale_min(int j, const uint8_t* q, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

__device__ __forceinline__ void kt_dq32_q4_k(const uint8_t* b, int sub, float* y) {
  const float d = kt_h2f(b[0] | (b[1] << 8)), dmin = kt_h2f(b[2] | (b[3] << 8));
  int sc, m;
  kt_q4k_scale_min(sub, b + 4, sc, m);
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
  const uint8_t* q = b + 16 + 32 * (sub / 2);
  const int sh = 4 * (sub & 1);
#pragma unroll
  for (int l = 0; l < 32; ++l) y[l] = __fsub_rn(__fmul_rn(d1, (float)((q[l] >> sh) & 0xF)), m1);
}

__device__ __forceinline__ void kt_dq32_q6_k(const uint8_t* b, int sub, float* y) {
  // sub 0..7: half n = sub / 4, quarter (sub % 4) selects ql low/high nibble and qh bits
  const int n = sub / 4, qq = sub % 4;
  const uint8_t* ql = b + 64 * n + 32 * (qq & 1);
  const uint8_t* qh = b + 128 + 32 * n;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + 8 * n;
  const float d = kt_h2f(b[208] | (b[209] << 8));
  const int lsh = 4 * (qq >> 1), hsh = 2 * qq;
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    const int q = (int)(((ql[l] >> lsh) & 0xF) | (((qh[l] >> hsh) & 3) << 4)) - 32;
    y[l] = __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * qq]), (float)q);
  }
}

__device__ __forceinline__ void kt_dq32_iq3_s(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const int s = (b[106 + sub / 2] >> (4 * (sub % 2))) & 0xf;
  const float db = __fmul_rn(d, (float)(1 + 2 * s));
  const uint8_t* qs = b + 2 + 8 * sub;
  const int qh = b[66 + sub];
  const uint8_t* signs = b + 74 + 4 * sub;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t g1 = grid[qs[2 * l + 0] | ((qh << (8 - 2 * l)) & 256)];
    const uint32_t g2 = grid[qs[2 * l + 1] | ((qh << (7 - 2 * l)) & 256)];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v1 = __fmul_rn(db, (float)((g1 >> (8 * j)) & 0xff));
      const float v2 = __fmul_rn(db, (float)((g2 >> (8 * j)) & 0xff));
      y[8 * l + j] = (signs[l] >> j) & 1 ? -v1 : v1;
      y[8 * l + 4 + j] = (signs[l] >> (j + 4)) & 1 ? -v2 : v2;
    }
  }
}

// legacy 32-value blocks: value j < 16 from the low nibble of qs[j], j >= 16 from the high
// nibble of qs[j-16]; Q5 types add bit j of qh as the fifth bit. ggml: (q - 8) * d, q * d + m,
// (q - 16) * d, q * d + m, level(q) * d (every product exact in fp32)
template <int TYPE>
__device__ __forceinline__ void kt_dq32_legacy(const uint8_t* b, float* y) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const bool has_m = TYPE == KT_Q4_1 || TYPE == KT_Q5_1;
  const float m = has_m ? kt_h2f(b[2] | (b[3] << 8)) : 0.0f;
  const int qs_off = TYPE == KT_Q4_0 || TYPE == KT_IQ4_NL ? 2 : TYPE == KT_Q4_1 ? 4 : TYPE == KT_Q5_0 ? 6 : 8;
  uint32_t qh = 0;
  if constexpr (TYPE == KT_Q5_0) qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
  if constexpr (TYPE == KT_Q5_1) qh = (uint32_t)b[4] | ((uint32_t)b[5] << 8) | ((uint32_t)b[6] << 16) | ((uint32_t)b[7] << 24);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int nib = (b[qs_off + (j & 15)] >> (j < 16 ? 0 : 4)) & 0xF;
    const int q = nib | (int)(((qh >> j) & 1) << 4);
    if constexpr (TYPE == KT_Q4_0) y[j] = (float)(nib - 8) * d;
    if constexpr (TYPE == KT_Q4_1 || TYPE == KT_Q5_1) y[j] = __fadd_rn(__fmul_rn((float)q, d), m);
    if constexpr (TYPE == KT_Q5_0) y[j] = (float)(q - 16) * d;
    if constexpr (TYPE == KT_IQ4_NL) y[j] = (float)kt_iq4nl_level(nib) * d;
  }
}

// K-quant sub-block sub (32 values) of a 256-value block, ggml's order and roundings:
// Q2_K: half n = sub/4, shift pair j = sub%4; values 0-15 from q[32n + l] >> 2j with group
// scale 8n+2j, 16-31 from q[32n + 16 + l] with group 8n+2j+1: (d*sc)*q - dmin*m
__device__ __forceinline__ void kt_dq32_q2_k(const uint8_t* b, int sub, float* y) {
  const float d = kt_h2f(b[80] | (b[81] << 8)), dmin = kt_h2f(b[82] | (b[83] << 8));
  const int n = sub / 4, j = sub % 4;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int sc = b[8 * n + 2 * j + h];
    const float dl = __fmul_rn(d, (float)(sc & 0xF)), ml = __fmul_rn(dmin, (float)(sc >> 4));
    const uint8_t* q = b + 16 + 32 * n + 16 * h;
#pragma unroll
    for (int l = 0; l < 16; ++l) y[16 * h + l] = __fsub_rn(__fmul_rn(dl, (float)((q[l] >> (2 * j)) & 3)), ml);
  }
}
// Q3_K: as Q2_K's grouping; the third bit is bit 4n+j of hmask[l] / hmask[16+l] (clear: -4);
// 6-bit scales minus 32: (d*(s-32))*q
__device__ __forceinline__ void kt_dq32_q3_k(const uint8_t* b, int sub, float* y) {
  const float d = kt_h2f(b[108] | (b[109] << 8));
  const int n = sub / 4, j = sub % 4, m = 1 << (4 * n + j);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int is = 8 * n + 2 * j + h;
    const int sc = (((b[96 + is % 8] >> (4 * (is / 8))) & 0xF) | (((b[104 + is % 4] >> (2 * (is / 4))) & 3) << 4)) - 32;
    const float dl = __fmul_rn(d, (float)sc);
    const uint8_t* q = b + 32 + 32 * n + 16 * h;
    const uint8_t* hm = b + 16 * h;
#pragma unroll
    for (int l = 0; l < 16; ++l) {
      const int v = ((q[l] >> (2 * j)) & 3) - ((hm[l] & m) ? 0 : 4);
      y[16 * h + l] = __fmul_rn(dl, (float)v);
    }
  }
}
// Q5_K: group j = sub/2 of 64 values, low (sub even) or high nibbles of ql[32j + l], fifth bit
// sub of qh[l]: (d*sc)*q - dmin*m
__device__ __forceinline__ void kt_dq32_q5_k(const uint8_t* b, int sub, float* y) {
  const float d = kt_h2f(b[0] | (b[1] << 8)), dmin = kt_h2f(b[2] | (b[3] << 8));
  int sc, m;
  kt_q4k_scale_min(sub, b + 4, sc, m);
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
  const uint8_t* ql = b + 48 + 32 * (sub / 2);
  const uint8_t* qh = b + 16;
  const int sh = 4 * (sub & 1);
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    const int q = ((ql[l] >> sh) & 0xF) | (((qh[l] >> sub) & 1) << 4);
    y[l] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
  }
}
// IQ4_XS: sub-block ib = sub: (d*(ls-32)) * level(code)
__device__ __forceinline__ void kt_dq32_iq4_xs(const uint8_t* b, int sub, float* y) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const int scales_h = b[2] | (b[3] << 8);
  const int ls = ((b[4 + sub / 2] >> (4 * (sub % 2))) & 0xf) | (((scales_h >> (2 * sub)) & 3) << 4);
  const float dl = __fmul_rn(d, (float)(ls - 32));
  const uint8_t* qs = b + 8 + 16 * sub;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    y[j] = __fmul_rn(dl, (float)kt_iq4nl_level(qs[j] & 0xf));
    y[j + 16] = __fmul_rn(dl, (float)kt_iq4nl_level(qs[j] >> 4));
  }
}

// i-quant sub-block sub (32 values), gguf-py's / ggml's order: db = d * (0.5 + s) * 1/4 (1/2
// for IQ3_XXS), value = (db * grid) with the sign applied; IQ1: dl * (v + delta)
__device__ __forceinline__ float kt_signed_mul(float db, uint32_t mag, uint32_t neg) {
  const float v = __fmul_rn(db, (float)mag);
  return neg ? -v : v;
}
__device__ __forceinline__ float kt_iq_db(float d, int s, float quarter_or_half) {
  return __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)s)), quarter_or_half);
}
// 8 values from two book words (IQ2 families): element j = byte j%4 of word j/4
__device__ __forceinline__ void kt_dq8_iq2(float db, const uint32_t* g, uint32_t s8, float* y) {
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = kt_signed_mul(db, (g[j / 4] >> (8 * (j % 4))) & 0xffu, (s8 >> j) & 1u);
}
__device__ __forceinline__ void kt_dq32_iq2_xxs(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const uint8_t* q2 = b + 2 + 8 * sub;
  const uint32_t aux32 = (uint32_t)(q2[4] | (q2[5] << 8) | (q2[6] << 16)) | ((uint32_t)q2[7] << 24);
  const float db = kt_iq_db(d, (int)(aux32 >> 28), 0.25f);
#pragma unroll
  for (int l = 0; l < 4; ++l) kt_dq8_iq2(db, grid + 2 * q2[l], kt_signs8((aux32 >> (7 * l)) & 127u), y + 8 * l);
}
__device__ __forceinline__ void kt_dq32_iq2_xs(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const uint8_t* q2 = b + 2 + 8 * sub;
  const float db0 = kt_iq_db(d, b[66 + sub] & 0xf, 0.25f), db1 = kt_iq_db(d, b[66 + sub] >> 4, 0.25f);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t code = q2[2 * l] | (q2[2 * l + 1] << 8);
    kt_dq8_iq2(l < 2 ? db0 : db1, grid + 2 * (code & 511u), kt_signs8(code >> 9), y + 8 * l);
  }
}
__device__ __forceinline__ void kt_dq32_iq2_s(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const float db0 = kt_iq_db(d, b[74 + sub] & 0xf, 0.25f), db1 = kt_iq_db(d, b[74 + sub] >> 4, 0.25f);
  const int qh = b[66 + sub];
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const int idx = b[2 + 4 * sub + l] | ((qh << (8 - 2 * l)) & 0x300);
    kt_dq8_iq2(l < 2 ? db0 : db1, grid + 2 * idx, b[34 + 4 * sub + l], y + 8 * l);
  }
}
__device__ __forceinline__ void kt_dq32_iq3_xxs(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const uint8_t* q3 = b + 2 + 8 * sub;
  const uint8_t* a = b + 66 + 4 * sub;
  const uint32_t aux32 = (uint32_t)(a[0] | (a[1] << 8) | (a[2] << 16)) | ((uint32_t)a[3] << 24);
  const float db = kt_iq_db(d, (int)(aux32 >> 28), 0.5f);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t s8 = kt_signs8((aux32 >> (7 * l)) & 127u);
    const uint32_t g[2] = {grid[q3[2 * l]], grid[q3[2 * l + 1]]};
    kt_dq8_iq2(db, g, s8, y + 8 * l);
  }
}
// 8 values v + delta (v from the nibble book: element j<4 low nibble of byte j, j>=4 high
// nibble of byte j-4, stored as v + 1)
__device__ __forceinline__ void kt_dq8_iq1(float dl, uint32_t w, float delta, float* y) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int v = (int)((w >> (8 * (j % 4) + 4 * (j / 4))) & 0xfu) - 1;
    y[j] = __fmul_rn(dl, __fadd_rn((float)v, delta));
  }
}
__device__ __forceinline__ void kt_dq32_iq1_s(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  const float d = kt_h2f(b[0] | (b[1] << 8));
  const int qh = b[34 + 2 * sub] | (b[35 + 2 * sub] << 8);
  const float dl = __fmul_rn(d, (float)(2 * ((qh >> 12) & 7) + 1));
  const float delta = (qh & 0x8000) ? -KT_IQ1_DELTA : KT_IQ1_DELTA;
#pragma unroll
  for (int l = 0; l < 4; ++l) kt_dq8_iq1(dl, grid[b[2 + 4 * sub + l] | (((qh >> (3 * l)) & 7) << 8)], delta, y + 8 * l);
}
__device__ __forceinline__ void kt_dq32_iq1_m(const uint8_t* b, int sub, float* y, const uint32_t* grid) {
  uint16_t sc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) sc[k] = (uint16_t)(b[48 + 2 * k] | (b[49 + 2 * k] << 8));
  const float d = kt_h2f((sc[0] >> 12) | ((sc[1] >> 8) & 0x00F0) | ((sc[2] >> 4) & 0x0F00) | (sc[3] & 0xF000));
  const int tmp = sc[sub / 2] >> (6 * (sub % 2));
  const float dl0 = __fmul_rn(d, (float)(2 * (tmp & 7) + 1)), dl1 = __fmul_rn(d, (float)(2 * ((tmp >> 3) & 7) + 1));
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const int qhl = b[32 + 2 * sub + l / 2] >> (4 * (l % 2));
    kt_dq8_iq1(l < 2 ? dl0 : dl1, grid[b[4 * sub + l] | ((qhl & 7) << 8)], (qhl & 8) ? -KT_IQ1_DELTA : KT_IQ1_DELTA,
               y + 8 * l);
  }
}

// 32 consecutive values starting at element 32*sub32 of a row made of blocks of TYPE
template <int TYPE>
__device__ __forceinline__ void kt_dq32(const uint8_t* row, int sub32, float* y, const uint32_t* grid) {
  if constexpr (TYPE == KT_Q8_0) {
    kt_dq32_q8_0(row + sub32 * 34, y);
  } else if constexpr (KtChunk<TYPE>::QK == 32) {
    kt_dq32_legacy<TYPE>(row + sub32 * KtChunk<TYPE>::BYTES, y);
  } else if constexpr (TYPE == KT_Q2_0) {  // half sub32&1 of 64-value block sub32/2: (code-1)*d
    const uint8_t* b = row + (sub32 / 2) * 18;
    const float d = kt_h2f(b[0] | (b[1] << 8));
    const uint8_t* q = b + 2 + 8 * (sub32 & 1);
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = __fmul_rn((float)(((q[j / 4] >> (2 * (j % 4))) & 3) - 1), d);
  } else {
    constexpr int BS = KtChunk<TYPE>::BYTES;
    const uint8_t* b = row + (sub32 / 8) * BS;
    if constexpr (TYPE == KT_Q4_K) kt_dq32_q4_k(b, sub32 % 8, y);
    if constexpr (TYPE == KT_Q6_K) kt_dq32_q6_k(b, sub32 % 8, y);
    if constexpr (TYPE == KT_IQ3_S) kt_dq32_iq3_s(b, sub32 % 8, y, grid);
    if constexpr (TYPE == KT_Q2_K) kt_dq32_q2_k(b, sub32 % 8, y);
    if constexpr (TYPE == KT_Q3_K) kt_dq32_q3_k(b, sub32 % 8, y);
    if constexpr (TYPE == KT_Q5_K) kt_dq32_q5_k(b, sub32 % 8, y);
    if constexpr (TYPE == KT_IQ4_XS) kt_dq32_iq4_xs(b, sub32 % 8, y);
    if constexpr (TYPE == KT_IQ2_XXS) kt_dq32_iq2_xxs(b, sub32 % 8, y, grid);
    if constexpr (TYPE == KT_IQ2_XS) kt_dq32_iq2_xs(b, sub32 % 8, y, grid);
    if constexpr (TYPE == KT_IQ2_S) kt_dq32_iq2_s(b, sub32 % 8, y, grid);
    if constexpr (TYPE == KT_IQ3_XXS) kt_dq32_iq3_xxs(b, sub32 % 8, y, grid);
    if constexpr (TYPE == KT_IQ1_S) kt_dq32_iq1_s(b, sub32 % 8, y, grid);
    if constexpr (TYPE == KT_IQ1_M) kt_dq32_iq1_m(b, sub32 % 8, y, grid);
  }
}
