// gguf_tile.cuh — register-level GGUF dequantization for the prefill GEMM producers.
//
// Four producer threads share one weight row of the tile. For every 64-wide k-step each reads
// the raw bytes of its 16 values from the row's shared-memory slot with 16-byte loads
// (conflict-free across consecutive rows), re-aligns them in registers (GGUF blocks are only
// 2-byte aligned, so the unit can start at any even offset of its 16-byte aligned slot),
// decodes the codes with byte permutes into "magic" floats (2^23 + code, exact), and
// produces 16 bf16 values as 8 packed words.
//
// Arithmetic matches ggml's dequantize_row_* exactly: every product of a scale and a code
// is exact in fp32 (at most 25 significant bits are never needed: see per type), so
// fma(scale, code, -min) and scale * code round exactly like ggml's separately rounded
// operations; the bf16 values are the round-to-nearest-even of ggml's fp32 values.
#pragma once
#include "kt_common.cuh"

// NW 32-bit words starting at the byte offset p of a 16-byte aligned shared slot. p must be
// even (GGUF fields used here all start at even offsets of 2-byte aligned blocks).
template <int NW>
__device__ __forceinline__ void kt_ld_words(const uint8_t* slot, int p, uint32_t (&out)[NW]) {
  constexpr int NC = (NW * 4 + 14 + 15) / 16;  // 16-byte chunks covering any start in 0..14
  const uint4* c = reinterpret_cast<const uint4*>(slot + (p & ~15));
  uint32_t w[NC * 4];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const uint4 v = c[i];
    w[4 * i + 0] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
  const int q = (p >> 2) & 3;
#pragma unroll
  for (int i = 0; i < NC * 4 - 1; ++i) w[i] = (q & 1) ? w[i + 1] : w[i];
#pragma unroll
  for (int i = 0; i < NC * 4 - 2; ++i) w[i] = (q & 2) ? w[i + 2] : w[i];
  const uint32_t sel = (p & 2) ? 0x5432u : 0x3210u;
#pragma unroll
  for (int i = 0; i < NW; ++i) out[i] = __byte_perm(w[i], w[i + 1], sel);
}

// byte k of `word` as the float 2^23 + byte (exact)
__device__ __forceinline__ float kt_magic(uint32_t word, int k) {
  return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7440u | (uint32_t)k));
}
__device__ __forceinline__ uint32_t kt_byte(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xffu; }
__device__ __forceinline__ float kt_lo_half(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w & 0xffff))); }
__device__ __forceinline__ float kt_hi_half(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w >> 16))); }

template <int TYPE>
struct KtTileDq;

// Each kstep_quarter call produces the 16 values [16*qt, 16*qt + 16) of the 64-value k-step
// kk of the unit as 8 packed bf16 pairs (four producer threads share a weight row).

// Q4_K: unit = one 144-byte block (d, dmin, 12 scale bytes, 128 nibble bytes).
// k-step kk uses qs bytes [32kk, 32kk+32): low nibbles = sub-block 2kk (values 0-31), high
// nibbles = sub-block 2kk+1 (values 32-63); quarter qt reads the 16 bytes [16(qt&1), +16) of
// them, nibble half qt>>1. d*sc (11+6 bits) * q (4 bits) is exact; the subtraction of dmin*m
// rounds once.
template <>
struct KtTileDq<KT_Q4_K> {
  static constexpr int KPU = 4;
  uint32_t h[4];
  __device__ __forceinline__ void unit(const uint8_t* slot, int off) { kt_ld_words<4>(slot, off, h); }
  __device__ __forceinline__ void scale_min(int j, int& sc, int& m) const {
    const uint32_t* s = h + 1;  // the 12 scale bytes
    if (j < 4) {
      sc = kt_byte(s, j) & 63;
      m = kt_byte(s, j + 4) & 63;
    } else {
      sc = (kt_byte(s, j + 4) & 0xF) | ((kt_byte(s, j - 4) >> 6) << 4);
      m = (kt_byte(s, j + 4) >> 4) | ((kt_byte(s, j) >> 6) << 4);
    }
  }
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t*) {
    const int hf = qt >> 1;
    uint32_t q[4];
    kt_ld_words<4>(slot, off + 16 + 32 * kk + 16 * (qt & 1), q);
    const float d = kt_lo_half(h[0]), dmin = kt_hi_half(h[0]);
    int sc, m;
    scale_min(2 * kk + hf, sc, m);
    const float ds = d * (float)sc, dm = dmin * (float)m;
    constexpr float M = 8388608.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = (q[i] >> (4 * hf)) & 0x0F0F0F0Fu;
      pk[2 * i + 0] = kt_pack_bf2(fmaf(ds, kt_magic(v, 0) - M, -dm), fmaf(ds, kt_magic(v, 1) - M, -dm));
      pk[2 * i + 1] = kt_pack_bf2(fmaf(ds, kt_magic(v, 2) - M, -dm), fmaf(ds, kt_magic(v, 3) - M, -dm));
    }
  }
};

// Q6_K: unit = one 210-byte block (ql[128], qh[64], int8 scales[16], d). k-step kk covers
// values [64kk, 64kk+64): half n = kk/2 of the block, nibble part = kk%2. Values 32*hf + j
// (hf = qt>>1, j < 32) take their low 4 bits from ql[64n + 32hf + j] and their high 2 bits
// from qh[32n + j]; quarter qt covers j in [16(qt&1), +16), which share the int8 scale
// 8n + 4part + 2hf + (qt&1). d*sc (11+8 bits) times the 6-bit signed code rounds once, like
// ggml's (d*sc)*q.
template <>
struct KtTileDq<KT_Q6_K> {
  static constexpr int KPU = 4;
  float d;
  // k-steps 2n and 2n+1 read the same ql / qh / scale bytes (nibble part kk%2 picks the
  // bits): they are loaded and re-aligned once, at the even k-step (kk is a compile-time
  // constant in the producers' unrolled loop)
  uint32_t ql[4], qh[4], sc[2];
  __device__ __forceinline__ void unit(const uint8_t* slot, int off) {
    uint32_t w[1];
    kt_ld_words<1>(slot, off + 208, w);
    d = kt_lo_half(w[0]);
  }
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t*) {
    const int n = kk >> 1, part = kk & 1, hf = qt >> 1, sub = qt & 1;
    if (part == 0) {
      kt_ld_words<4>(slot, off + 64 * n + 32 * hf + 16 * sub, ql);
      kt_ld_words<4>(slot, off + 128 + 32 * n + 16 * sub, qh);
      kt_ld_words<2>(slot, off + 192 + 8 * n, sc);
    }
    const float sa = d * (float)(int8_t)(sc[part] >> (8 * (2 * hf + sub)));
    constexpr float M = 8388640.0f;  // 2^23 + 32: magic(code) - M = code - 32
    const int ls = 4 * part, hs = 4 * part + 2 * hf;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a = ((ql[i] >> ls) & 0x0F0F0F0Fu) | (((qh[i] >> hs) & 0x03030303u) << 4);
      pk[2 * i + 0] = kt_pack_bf2(sa * (kt_magic(a, 0) - M), sa * (kt_magic(a, 1) - M));
      pk[2 * i + 1] = kt_pack_bf2(sa * (kt_magic(a, 2) - M), sa * (kt_magic(a, 3) - M));
    }
  }
};

// IQ3_S: unit = one 110-byte block (d, qs[64], qh[8], signs[32], scales[4]). k-step kk, half
// hf = qt>>1 is sub-block ib = 2kk + hf; quarter qt takes its groups l = 2(qt&1), 2(qt&1)+1 of
// 8 values (two 4-value grid entries each). d*(1+2s) (11+5 bits) times a grid magnitude
// (4 bits) is exact.
template <>
struct KtTileDq<KT_IQ3_S> {
  static constexpr int KPU = 4;
  float d;
  uint32_t sc;
  __device__ __forceinline__ void unit(const uint8_t* slot, int off) {
    uint32_t w[1], s4[1];
    kt_ld_words<1>(slot, off, w);
    kt_ld_words<1>(slot, off + 106, s4);  // scales[0..3]
    d = kt_lo_half(w[0]);
    sc = s4[0];
  }
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t* grid) {
    const int hf = qt >> 1, ib = 2 * kk + hf, l0 = 2 * (qt & 1);
    uint32_t qs[2], qh[1], sg[1];
    kt_ld_words<2>(slot, off + 2 + 8 * ib, qs);
    kt_ld_words<1>(slot, off + 66 + 2 * kk, qh);  // qh[2kk], qh[2kk+1] (an even offset)
    kt_ld_words<1>(slot, off + 74 + 4 * ib, sg);
    constexpr float M = 8388736.0f;  // 2^23 + 128: signed bytes are stored biased by 128
    const float db = d * (float)(1 + 2 * ((sc >> (8 * kk + 4 * hf)) & 0xf));
    const uint32_t qhh = (qh[0] >> (8 * hf)) & 0xff;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int l = l0 + j;
      const uint32_t i1 = kt_byte(qs, 2 * l) | ((qhh << (8 - 2 * l)) & 256);
      const uint32_t i2 = kt_byte(qs, 2 * l + 1) | ((qhh << (7 - 2 * l)) & 256);
      const uint32_t s = kt_byte(sg, l);
      const uint32_t s0 = __vcmpeq4(((s & 0xf) * 0x01010101u) & 0x08040201u, 0x08040201u);
      const uint32_t s1 = __vcmpeq4(((s >> 4) * 0x01010101u) & 0x08040201u, 0x08040201u);
      const uint32_t v1 = __vsub4(grid[i1] ^ s0, s0) ^ 0x80808080u;
      const uint32_t v2 = __vsub4(grid[i2] ^ s1, s1) ^ 0x80808080u;
      pk[4 * j + 0] = kt_pack_bf2(db * (kt_magic(v1, 0) - M), db * (kt_magic(v1, 1) - M));
      pk[4 * j + 1] = kt_pack_bf2(db * (kt_magic(v1, 2) - M), db * (kt_magic(v1, 3) - M));
      pk[4 * j + 2] = kt_pack_bf2(db * (kt_magic(v2, 0) - M), db * (kt_magic(v2, 1) - M));
      pk[4 * j + 3] = kt_pack_bf2(db * (kt_magic(v2, 2) - M), db * (kt_magic(v2, 3) - M));
    }
  }
};

// Q8_0: unit = four 34-byte blocks (d, 32 x int8). k-step kk, half qt>>1 = block
// 2kk + (qt>>1), quarter qt its 16 bytes [16(qt&1), +16); d (11 bits) * q (8 bits) is exact.
template <>
struct KtTileDq<KT_Q8_0> {
  static constexpr int KPU = 2;
  __device__ __forceinline__ void unit(const uint8_t*, int) {}
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t*) {
    constexpr float M = 8388736.0f;
    const int bo = off + 34 * (2 * kk + (qt >> 1));
    uint32_t dw[1], q[4];
    kt_ld_words<1>(slot, bo, dw);
    kt_ld_words<4>(slot, bo + 2 + 16 * (qt & 1), q);
    const float d = kt_lo_half(dw[0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = q[i] ^ 0x80808080u;
      pk[2 * i + 0] = kt_pack_bf2(d * (kt_magic(v, 0) - M), d * (kt_magic(v, 1) - M));
      pk[2 * i + 1] = kt_pack_bf2(d * (kt_magic(v, 2) - M), d * (kt_magic(v, 3) - M));
    }
  }
};
