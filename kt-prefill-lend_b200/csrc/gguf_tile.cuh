// gguf_tile.cuh — register-level GGUF dequantization for the prefill GEMM producers.
//
// Two or four producer threads share one weight row of the tile. For every 64-wide k-step
// each reads the raw bytes of its 16-value quarters from the row's shared-memory slot with
// 16-byte loads (conflict-free across consecutive rows), re-aligns them in registers (GGUF
// blocks are only 2-byte aligned, so the unit can start at any even offset of its 16-byte
// aligned slot; Q4_K units, 9 x 16 bytes, start on the boundary whenever the weights do and
// skip the re-alignment), decodes the codes with byte permutes into "magic" floats (2^23 +
// code, exact), scales them with packed f32x2 arithmetic, and produces 16 bf16 values as 8
// packed words.
//
// Arithmetic matches ggml's dequantize_row_* exactly: every product of a scale and a code
// is exact in fp32 (at most 25 significant bits are never needed: see per type), so
// fma(scale, code, -min) and scale * code round exactly like ggml's separately rounded
// operations; the bf16 values are the round-to-nearest-even of ggml's fp32 values.
#pragma once
#include "kt_common.cuh"

// NW 32-bit words starting at the byte offset p of a 16-byte aligned shared slot. p must be
// even (GGUF fields used here all start at even offsets of 2-byte aligned blocks). With A16 the
// caller guarantees p % 16 == 0 and the words are read directly.
template <int NW, bool A16 = false>
__device__ __forceinline__ void kt_ld_words(const uint8_t* slot, int p, uint32_t (&out)[NW]) {
  if constexpr (A16) {
    static_assert(NW == 4, "aligned reads take one 16-byte chunk");
    const uint4 v = *reinterpret_cast<const uint4*>(slot + p);
    out[0] = v.x;
    out[1] = v.y;
    out[2] = v.z;
    out[3] = v.w;
    return;
  }
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

// Two fp32 lanes in one 64-bit register for sm_100's packed f32x2 add / mul / fma: each lane
// is an ordinary round-to-nearest fp32 operation, so results equal the scalar ones bit for bit
// while the FMA pipe issues half as many instructions.
__device__ __forceinline__ uint64_t kt_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t kt_f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t kt_f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t kt_f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// bf16 pair (round to nearest even) of the two lanes; the low lane goes to the low half
__device__ __forceinline__ uint32_t kt_f2_bf16(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return kt_pack_bf2(lo, hi);
}
// bytes k and k+1 of `word` as magic floats (2^23 + byte) minus the pair m: exact
__device__ __forceinline__ uint64_t kt_magic2(uint32_t word, int k, uint64_t m) {
  return kt_f2_sub(kt_f2(kt_magic(word, k), kt_magic(word, k + 1)), m);
}

template <int TYPE>
struct KtTileDq;

// Each kstep_quarter call produces the 16 values [16*qt, 16*qt + 16) of the 64-value k-step
// kk of the unit as 8 packed bf16 pairs (two or four producer threads share a weight row).
// unit() reads what the thread needs of the unit's header once per unit. A16 = true promises
// that the unit starts on a 16-byte boundary of its slot (off == 0); only types whose block
// size is a 16-byte multiple (kAlignable) are ever called with it.

// Q4_K: unit = one 144-byte block (d, dmin, 12 scale bytes, 128 nibble bytes).
// k-step kk uses qs bytes [32kk, 32kk+32): low nibbles = sub-block 2kk (values 0-31), high
// nibbles = sub-block 2kk+1 (values 32-63); quarter qt reads the 16 bytes [16(qt&1), +16) of
// them, nibble half hf = qt>>1, so its sub-block is j = 2kk + hf. d*sc (11+6 bits) * q (4 bits)
// is exact; the subtraction of dmin*m rounds once.
template <>
struct KtTileDq<KT_Q4_K> {
  static constexpr int KPU = 4;
  static constexpr bool kAlignable = true;  // 144 = 9 x 16 bytes
  uint64_t dsp[4], dmp[4];                  // per k-step: (d*sc, d*sc) and (-dmin*m, -dmin*m)
  template <bool A16>
  __device__ __forceinline__ void unit(const uint8_t* slot, int off, int qt) {
    uint32_t h[4];
    kt_ld_words<4, A16>(slot, off, h);
    const float d = kt_lo_half(h[0]), dmin = kt_hi_half(h[0]);
    // 6-bit scales and mins of sub-blocks 0-3 (bytes of sc_lo / m_lo) and 4-7 (sc_hi / m_hi):
    // j < 4: sc = q[j] & 63, m = q[j+4] & 63; j >= 4: the low 4 bits come from q[j+4], the
    // high 2 bits from bits 6-7 of q[j-4] (scale) or q[j] (min)
    const uint32_t sc_lo = h[1] & 0x3F3F3F3Fu, m_lo = h[2] & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (h[3] & 0x0F0F0F0Fu) | ((h[1] >> 2) & 0x30303030u);
    const uint32_t m_hi = ((h[3] >> 4) & 0x0F0F0F0Fu) | ((h[2] >> 2) & 0x30303030u);
    const int hf = qt >> 1;
    constexpr float M = 8388608.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int b = 2 * (kk & 1) + hf;  // sub-block 2kk + hf: byte b of the low (kk < 2) or high words
      const float ds = d * (kt_magic(kk < 2 ? sc_lo : sc_hi, b) - M);
      const float dm = dmin * (kt_magic(kk < 2 ? m_lo : m_hi, b) - M);
      dsp[kk] = kt_f2(ds, ds);
      dmp[kk] = kt_f2(-dm, -dm);
    }
  }
  template <bool A16>
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t*) {
    const int hf = qt >> 1;
    uint32_t q[4];
    kt_ld_words<4, A16>(slot, off + 16 + 32 * kk + 16 * (qt & 1), q);
    const uint64_t M2 = kt_f2(8388608.0f, 8388608.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = (q[i] >> (4 * hf)) & 0x0F0F0F0Fu;
      pk[2 * i + 0] = kt_f2_bf16(kt_f2_fma(dsp[kk], kt_magic2(v, 0, M2), dmp[kk]));
      pk[2 * i + 1] = kt_f2_bf16(kt_f2_fma(dsp[kk], kt_magic2(v, 2, M2), dmp[kk]));
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
  static constexpr bool kAlignable = false;
  float d;
  // k-steps 2n and 2n+1 read the same ql / qh / scale bytes (nibble part kk%2 picks the
  // bits): they are loaded and re-aligned once, at the even k-step (kk is a compile-time
  // constant in the producers' unrolled loop)
  uint32_t ql[4], qh[4], sc[2];
  template <bool>
  __device__ __forceinline__ void unit(const uint8_t* slot, int off, int) {
    uint32_t w[1];
    kt_ld_words<1>(slot, off + 208, w);
    d = kt_lo_half(w[0]);
  }
  template <bool>
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t*) {
    const int n = kk >> 1, part = kk & 1, hf = qt >> 1, sub = qt & 1;
    if (part == 0) {
      kt_ld_words<4>(slot, off + 64 * n + 32 * hf + 16 * sub, ql);
      kt_ld_words<4>(slot, off + 128 + 32 * n + 16 * sub, qh);
      kt_ld_words<2>(slot, off + 192 + 8 * n, sc);
    }
    const float sa = d * (float)(int8_t)(sc[part] >> (8 * (2 * hf + sub)));
    const uint64_t sa2 = kt_f2(sa, sa);
    const uint64_t M2 = kt_f2(8388640.0f, 8388640.0f);  // 2^23 + 32: magic(code) - M = code - 32
    const int ls = 4 * part, hs = 4 * part + 2 * hf;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t a = ((ql[i] >> ls) & 0x0F0F0F0Fu) | (((qh[i] >> hs) & 0x03030303u) << 4);
      pk[2 * i + 0] = kt_f2_bf16(kt_f2_mul(sa2, kt_magic2(a, 0, M2)));
      pk[2 * i + 1] = kt_f2_bf16(kt_f2_mul(sa2, kt_magic2(a, 2, M2)));
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
  static constexpr bool kAlignable = false;
  float d;
  uint32_t sc;
  template <bool>
  __device__ __forceinline__ void unit(const uint8_t* slot, int off, int) {
    uint32_t w[1], s4[1];
    kt_ld_words<1>(slot, off, w);
    kt_ld_words<1>(slot, off + 106, s4);  // scales[0..3]
    d = kt_lo_half(w[0]);
    sc = s4[0];
  }
  template <bool>
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t* grid) {
    const int hf = qt >> 1, ib = 2 * kk + hf, l0 = 2 * (qt & 1);
    uint32_t qs[2], qh[1], sg[1];
    kt_ld_words<2>(slot, off + 2 + 8 * ib, qs);
    kt_ld_words<1>(slot, off + 66 + 2 * kk, qh);  // qh[2kk], qh[2kk+1] (an even offset)
    kt_ld_words<1>(slot, off + 74 + 4 * ib, sg);
    const uint64_t M2 = kt_f2(8388736.0f, 8388736.0f);  // 2^23 + 128: signed bytes are stored biased by 128
    const float db = d * (float)(1 + 2 * ((sc >> (8 * kk + 4 * hf)) & 0xf));
    const uint64_t db2 = kt_f2(db, db);
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
      pk[4 * j + 0] = kt_f2_bf16(kt_f2_mul(db2, kt_magic2(v1, 0, M2)));
      pk[4 * j + 1] = kt_f2_bf16(kt_f2_mul(db2, kt_magic2(v1, 2, M2)));
      pk[4 * j + 2] = kt_f2_bf16(kt_f2_mul(db2, kt_magic2(v2, 0, M2)));
      pk[4 * j + 3] = kt_f2_bf16(kt_f2_mul(db2, kt_magic2(v2, 2, M2)));
    }
  }
};

// Q8_0: unit = four 34-byte blocks (d, 32 x int8). k-step kk, half qt>>1 = block
// 2kk + (qt>>1), quarter qt its 16 bytes [16(qt&1), +16); d (11 bits) * q (8 bits) is exact.
template <>
struct KtTileDq<KT_Q8_0> {
  static constexpr int KPU = 2;
  static constexpr bool kAlignable = false;
  template <bool>
  __device__ __forceinline__ void unit(const uint8_t*, int, int) {}
  template <bool>
  __device__ __forceinline__ void kstep_quarter(const uint8_t* slot, int off, int kk, int qt, uint32_t (&pk)[8],
                                                const uint32_t*) {
    const uint64_t M2 = kt_f2(8388736.0f, 8388736.0f);
    const int bo = off + 34 * (2 * kk + (qt >> 1));
    uint32_t dw[1], q[4];
    kt_ld_words<1>(slot, bo, dw);
    kt_ld_words<4>(slot, bo + 2 + 16 * (qt & 1), q);
    const float d = kt_lo_half(dw[0]);
    const uint64_t d2 = kt_f2(d, d);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t v = q[i] ^ 0x80808080u;
      pk[2 * i + 0] = kt_f2_bf16(kt_f2_mul(d2, kt_magic2(v, 0, M2)));
      pk[2 * i + 1] = kt_f2_bf16(kt_f2_mul(d2, kt_magic2(v, 2, M2)));
    }
  }
};
