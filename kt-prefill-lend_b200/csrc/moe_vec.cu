// moe_vec.cu — decode path: q8_1 activation quantizer, route grouping, and the
// multi-token GGUF MoE GEMV (window and per-route semantics of kt_moe_a8_vec_multi).
//
// Reference behaviour (hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu):
//   quantize_q8_1 (:600-650): per 32 values d = amax/127, q = roundf(x/d), s = sum(x);
//     rows padded with zeros to a multiple of 512 values.
//   moe_vec_q (:132-217) + moe_vec_q_rows (:74-130): Y[p, r] = sum over the row's chunks of
//     vec_dot(W[ids[p]] row r, q8_1(X[p / top_k])); lane t of a warp takes chunks t, t+32, ...
//     in order and an xor butterfly (16,8,4,2,1) reduces the lanes; ids < 0 give zero rows.
//
// B200 design: routes are first grouped by expert slot (one tiny kernel), so every CTA
// owns one expert and a tile of rows and reads that tile of raw GGUF bytes from HBM once,
// with 16-byte vector loads into shared memory, for all the expert's routes in the call
// (the reference's window build does this for up to 4 routes, its per-route build not
// at all). Each warp then walks rows with the reference's lane-to-chunk assignment and
// butterfly, so every route's sum has the reference's order.
#include <string.h>

#include "gguf_dot.cuh"
#include "kt_kernels.h"

// ------------------------------------------------------------------ q8_1 quantizer

// SPLIT = false: the reference's q8_1 blocks (half2 ds, 32 int8) back to back; SPLIT = true:
// the GEMV's split layout (a row's int8 values, then its half2 ds per block), same values.
template <int DT, bool SPLIT>
__global__ void __launch_bounds__(256) kt_quantize_q8_1_kernel(const void* __restrict__ x, uint8_t* __restrict__ qx,
                                                               int64_t rows, int64_t cols, int64_t kpad) {
  const int64_t ix = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // column in the padded row
  const int64_t row = blockIdx.y + (int64_t)blockIdx.z * 65535;
  if (row >= rows || ix >= kpad) return;
  const float xi = ix < cols ? kt_load_act<DT>(x, row * cols + ix) : 0.0f;
  float amax = fabsf(xi), sum = xi;
#pragma unroll
  for (int mask = 16; mask > 0; mask >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, mask, 32));
    sum += __shfl_xor_sync(0xffffffffu, sum, mask, 32);
  }
  const float d = amax / 127;
  const int8_t q = amax == 0.0f ? 0 : (int8_t)roundf(xi / d);
  uint8_t* rowp = qx + row * (kpad / 32 * KT_Q8_1_BYTES);
  const half2 ds = __halves2half2(__float2half(d), __float2half(sum));
  if constexpr (SPLIT) {
    rowp[ix] = (uint8_t)q;
    if (ix % 32 == 0) *reinterpret_cast<half2*>(rowp + kpad + 4 * (ix / 32)) = ds;
  } else {
    uint8_t* blk = rowp + (ix / 32) * KT_Q8_1_BYTES;
    blk[4 + (ix % 32)] = (uint8_t)q;
    if (ix % 32 == 0) *reinterpret_cast<half2*>(blk) = ds;
  }
}

template <bool SPLIT>
static int launch_quantize(const void* x, int dtype, int64_t rows, int64_t cols, void* qx, cudaStream_t s) {
  if (rows <= 0) return 0;
  const int64_t kpad = (cols + 511) / 512 * 512;
  const int64_t zr = (rows + 65534) / 65535;
  dim3 grid((unsigned)((kpad + 255) / 256), (unsigned)(rows < 65535 ? rows : 65535), (unsigned)zr);
  switch (dtype) {
    case KT_DT_F32: kt_quantize_q8_1_kernel<KT_DT_F32, SPLIT><<<grid, 256, 0, s>>>(x, (uint8_t*)qx, rows, cols, kpad); break;
    case KT_DT_F16: kt_quantize_q8_1_kernel<KT_DT_F16, SPLIT><<<grid, 256, 0, s>>>(x, (uint8_t*)qx, rows, cols, kpad); break;
    case KT_DT_BF16: kt_quantize_q8_1_kernel<KT_DT_BF16, SPLIT><<<grid, 256, 0, s>>>(x, (uint8_t*)qx, rows, cols, kpad); break;
    default: return -1;
  }
  return 0;
}

int kt_launch_quantize_q8_1(const void* x, int dtype, int64_t rows, int64_t cols, void* qx, cudaStream_t s) {
  return launch_quantize<false>(x, dtype, rows, cols, qx, s);
}


// ------------------------------------------------------------------ route grouping
// One CTA: counting sort of the routes by expert slot. Routes with an id outside
// [0, n_slots) form the "zero" group (slot -1). With piece > 0 (a power of two) a slot's c
// routes are cut into groups of `piece` routes and then the binary parts of the rest
// (c = 13, piece 8: 8, 4, 1), so that a kernel can run each group with a compile-time member
// count; the zero group stays whole. Outputs, in the workspace:
//   groups[0]            number of groups G
//   groups[1 + 3g + 0]   slot of group g (-1 for the zero group)
//   groups[1 + 3g + 1]   first position of the group in `order`
//   groups[1 + 3g + 2]   routes in the group
//   order[R]             route indices grouped by slot (a slot's groups are consecutive)
// Order inside a slot is not fixed (atomics); every route's result is independent of it.

__device__ __forceinline__ int kt_group_pieces(int i, int c, int piece) {
  if (c == 0) return 0;
  if (i == 0 || piece == 0) return 1;
  return c / piece + __popc(c % piece);
}

// The same grouping for at most 32 routes by the first warp alone (no block barriers): lane p
// holds route p; lanes of one slot find each other with __match_any_sync, the lowest is the
// group's leader, and shuffle scans give each group its first position and first group index.
// Groups come out in the order of their leaders' lanes instead of slot order, which no caller
// relies on.
__device__ __forceinline__ void kt_group_routes_warp(const int32_t* __restrict__ ids, int routes, int n_slots,
                                                     int piece, int32_t* __restrict__ groups,
                                                     int32_t* __restrict__ order) {
  const int lane = threadIdx.x & 31;
  const bool live = lane < routes;
  const int32_t e = live ? ids[lane] : -1;
  const int slot = (e >= 0 && e < n_slots) ? e : -1;
  const uint32_t peers = __match_any_sync(0xffffffffu, live ? slot : -2);
  const int leader = __ffs(peers) - 1;
  const bool lead = live && lane == leader;
  const int cnt = __popc(peers);
  const int pieces = lead ? (slot < 0 || piece == 0 ? 1 : cnt / piece + __popc(cnt % piece)) : 0;
  int c_inc = lead ? cnt : 0, g_inc = pieces;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int cy = __shfl_up_sync(0xffffffffu, c_inc, o), gy = __shfl_up_sync(0xffffffffu, g_inc, o);
    if (lane >= o) c_inc += cy, g_inc += gy;
  }
  const int first = c_inc - (lead ? cnt : 0), g_first = g_inc - pieces;
  const int start = __shfl_sync(0xffffffffu, first, leader);
  if (live) order[start + __popc(peers & ((1u << lane) - 1))] = lane;
  if (lead) {
    int g = g_first, pos = first, left = cnt;
    auto emit = [&](int k) {
      groups[1 + 3 * g + 0] = slot;
      groups[1 + 3 * g + 1] = pos;
      groups[1 + 3 * g + 2] = k;
      ++g;
      pos += k;
      left -= k;
    };
    if (slot < 0 || piece == 0) {
      emit(cnt);
    } else {
      while (left >= piece) emit(piece);
      for (int bit = piece >> 1; bit > 0; bit >>= 1)
        if (left & bit) emit(bit);
    }
  }
  if (lane == 31) groups[0] = g_inc;
}

// the whole CTA groups; cnt: 2 * (n_slots + 1) ints of shared memory
__device__ __forceinline__ void kt_group_routes_body(const int32_t* __restrict__ ids, int64_t routes, int n_slots,
                                                     int piece, int32_t* __restrict__ groups,
                                                     int32_t* __restrict__ order, int32_t* cnt) {
  __shared__ int32_t wsum[2][32];
  int32_t* cur = cnt + (n_slots + 1);
  const int n = n_slots + 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int64_t p = threadIdx.x; p < routes; p += blockDim.x) {
    const int32_t e = ids[p];
    atomicAdd(&cnt[(e >= 0 && e < n_slots) ? e + 1 : 0], 1);
  }
  __syncthreads();
  // each thread owns consecutive counters [b, e): local totals, then block-wide exclusive
  // scans of the route counts (order offsets) and of the group counts (group indices)
  const int per = (n + (int)blockDim.x - 1) / (int)blockDim.x;
  const int b = min(n, (int)threadIdx.x * per), e = min(n, b + per);
  int c_sum = 0, g_sum = 0;
  for (int i = b; i < e; ++i) {
    c_sum += cnt[i];
    g_sum += kt_group_pieces(i, cnt[i], piece);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int cx = c_sum, gx = g_sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int cy = __shfl_up_sync(0xffffffffu, cx, o), gy = __shfl_up_sync(0xffffffffu, gx, o);
    if (lane >= o) cx += cy, gx += gy;
  }
  if (lane == 31) wsum[0][wid] = cx, wsum[1][wid] = gx;
  __syncthreads();
  if (wid == 0) {
    int cw = wsum[0][lane], gw = wsum[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int cy = __shfl_up_sync(0xffffffffu, cw, o), gy = __shfl_up_sync(0xffffffffu, gw, o);
      if (lane >= o) cw += cy, gw += gy;
    }
    wsum[0][lane] = cw, wsum[1][lane] = gw;
  }
  __syncthreads();
  int c_off = cx - c_sum + (wid ? wsum[0][wid - 1] : 0);
  int g_off = gx - g_sum + (wid ? wsum[1][wid - 1] : 0);
  for (int i = b; i < e; ++i) {
    const int c = cnt[i];
    cur[i] = c_off;
    if (c) {
      int first = c_off, left = c;
      auto emit = [&](int k) {
        groups[1 + 3 * g_off + 0] = i - 1;
        groups[1 + 3 * g_off + 1] = first;
        groups[1 + 3 * g_off + 2] = k;
        ++g_off;
        first += k;
        left -= k;
      };
      if (i == 0 || piece == 0) {
        emit(c);
      } else {
        while (left >= piece) emit(piece);
        for (int bit = piece >> 1; bit > 0; bit >>= 1)
          if (left & bit) emit(bit);
      }
    }
    c_off += c;
  }
  if (threadIdx.x == blockDim.x - 1) groups[0] = g_off;
  __syncthreads();
  for (int64_t p = threadIdx.x; p < routes; p += blockDim.x) {
    const int32_t e2 = ids[p];
    const int k = (e2 >= 0 && e2 < n_slots) ? e2 + 1 : 0;
    order[atomicAdd(&cur[k], 1)] = (int32_t)p;
  }
}

// The GEMV's two preparation steps in one launch: blocks [0, nqb) quantize the activations
// into the split q8_1 layout (256 columns of a row each, as kt_quantize_q8_1_kernel), block nqb
// groups the routes. Saves a launch on the decode path, where the GEMV itself is short.
template <int DT>
__global__ void __launch_bounds__(256) kt_quantize_group_kernel(const void* __restrict__ x, uint8_t* __restrict__ qx,
                                                                int64_t rows, int64_t cols, int64_t kpad, int64_t nqb,
                                                                const int32_t* __restrict__ ids, int64_t routes,
                                                                int n_slots, int piece, int32_t* __restrict__ groups,
                                                                int32_t* __restrict__ order, int* __restrict__ status) {
  extern __shared__ int32_t cnt[];
  if ((int64_t)blockIdx.x == nqb) {
    if (threadIdx.x == 0 && status) *status = KT_DEV_OK;  // the call's status word, before the GEMV runs
    if (routes <= 32) {
      if (threadIdx.x < 32) kt_group_routes_warp(ids, (int)routes, n_slots, piece, groups, order);
    } else {
      kt_group_routes_body(ids, routes, n_slots, piece, groups, order, cnt);
    }
    return;
  }
  const int64_t cbx = kpad / 256;
  const int64_t row = (int64_t)blockIdx.x / cbx;
  const int64_t ix = ((int64_t)blockIdx.x % cbx) * 256 + threadIdx.x;
  if (row >= rows) return;
  const float xi = ix < cols ? kt_load_act<DT>(x, row * cols + ix) : 0.0f;
  float amax = fabsf(xi), sum = xi;
#pragma unroll
  for (int mask = 16; mask > 0; mask >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, mask, 32));
    sum += __shfl_xor_sync(0xffffffffu, sum, mask, 32);
  }
  const float d = amax / 127;
  const int8_t q = amax == 0.0f ? 0 : (int8_t)roundf(xi / d);
  uint8_t* rowp = qx + row * (kpad / 32 * KT_Q8_1_BYTES);
  rowp[ix] = (uint8_t)q;
  if (ix % 32 == 0) *reinterpret_cast<half2*>(rowp + kpad + 4 * (ix / 32)) = __halves2half2(__float2half(d), __float2half(sum));
}

int kt_launch_quantize_group(const void* x, int dtype, int64_t rows, int64_t cols, void* qx, const int32_t* ids,
                             int64_t routes, int n_slots, int piece, int32_t* groups, int32_t* order, int* status,
                             cudaStream_t s) {
  // the counters are only needed by the block-wide grouping (more than 32 routes)
  const size_t smem = routes <= 32 ? 0 : sizeof(int32_t) * 2 * (size_t)(n_slots + 1);
  if (rows <= 0 || sizeof(int32_t) * 2 * (size_t)(n_slots + 1) > 200 * 1024 || piece < 0 || (piece & (piece - 1)))
    return -1;
  const int64_t kpad = (cols + 511) / 512 * 512;
  const int64_t nqb = rows * (kpad / 256);
  if (nqb + 1 > 0x7fffffff) return -1;
  switch (dtype) {
#define KT_QG_LAUNCH(DT)                                                                                          \
  {                                                                                                               \
    auto k = kt_quantize_group_kernel<DT>;                                                                        \
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
    k<<<(unsigned)(nqb + 1), 256, smem, s>>>(x, (uint8_t*)qx, rows, cols, kpad, nqb, ids, routes, n_slots, piece, \
                                             groups, order, status);                                              \
    return 0;                                                                                                     \
  }
    case KT_DT_F32: KT_QG_LAUNCH(KT_DT_F32)
    case KT_DT_F16: KT_QG_LAUNCH(KT_DT_F16)
    case KT_DT_BF16: KT_QG_LAUNCH(KT_DT_BF16)
#undef KT_QG_LAUNCH
  }
  return -1;
}

// ------------------------------------------------------------------ GEMV

struct KtVecArgs {
  const uint8_t* w;            // slot base (plain layout) or int64 table of slot addresses
  int table;                   // 1: w is the table
  const uint8_t* qx;           // q8_1 activations [tokens, qrow] bytes
  int64_t qrow;                // bytes per q8_1 row (split layout: kpad int8, then kpad/32 half2)
  int64_t kpad;                // padded columns of a q8_1 row
  const int32_t* groups;       // from the route grouping (kt_launch_quantize_group)
  const int32_t* order;
  int top_k;
  int rows, cols;
  int64_t row_bytes;
  int rows_per_cta;
  int members_per_pass;
  void* y;                     // [routes, rows]
  int* status;                 // workspace status word (bounded waits)
  int tiles_per_group;         // pipelined kernel: row tiles of rows_per_cta rows per group
  int stages;                  // bulk-staged member-stationary kernel: shared-memory stages
};

// LPR lanes per row: 32, or 16 when a row has at most 16 chunks (two rows per warp).
template <int TYPE, int DT, int LPR>
__global__ void __launch_bounds__(256) kt_moe_vec_kernel(const KtVecArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  using C = KtChunk<TYPE>;
  const int g = blockIdx.y;
  const int ngroups = a.groups[0];
  if (g >= ngroups) return;
  const int slot = a.groups[1 + 3 * g + 0];
  const int start = a.groups[1 + 3 * g + 1];
  const int count = a.groups[1 + 3 * g + 2];
  const int r0 = blockIdx.x * a.rows_per_cta;
  if (r0 >= a.rows) return;
  const int nr = min(a.rows_per_cta, a.rows - r0);
  const int tid = threadIdx.x;

  if (slot < 0) {  // routes not on this device: zero rows
    for (int64_t i = tid; i < (int64_t)count * nr; i += blockDim.x) {
      const int p = a.order[start + i / nr];
      kt_store_act<DT>(a.y, (int64_t)p * a.rows + r0 + i % nr, 0.0f);
    }
    return;
  }
  kt_stage_grid<TYPE>(grid_s, tid, blockDim.x);
  // raw rows [r0, r0 + nr) of the slot into shared memory
  const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                 : a.w + (int64_t)slot * a.rows * a.row_bytes;
  const uint8_t* src = wbase + (int64_t)r0 * a.row_bytes;
  const int64_t tile_bytes = (int64_t)nr * a.row_bytes;
  uint8_t* wt = smem;
  if ((((uintptr_t)src) & 15) == 0 && (tile_bytes & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(wt);
    for (int64_t i = tid; i < tile_bytes / 16; i += blockDim.x) d4[i] = __ldg(s4 + i);
  } else {  // GGUF blocks are always 2-byte aligned
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(wt);
    for (int64_t i = tid; i < tile_bytes / 2; i += blockDim.x) d2[i] = __ldg(s2 + i);
  }
  const int64_t wt_bytes = (tile_bytes + 15) & ~(int64_t)15;
  uint8_t* act = smem + wt_bytes;
  const int nblocks = a.cols / C::QK;
  const int nchunks = nblocks * C::CPB;
  const int warp = tid / 32, lane = tid % 32;
  constexpr int RPW = 32 / LPR;  // rows per warp pass
  const int sub = lane / LPR, sl = lane % LPR;

  for (int m0 = 0; m0 < count; m0 += a.members_per_pass) {
    const int nm = min(a.members_per_pass, count - m0);
    __syncthreads();  // previous pass done with `act`; first pass: weights visible
    for (int m = 0; m < nm; ++m) {
      const int p = a.order[start + m0 + m];
      const uint4* s4 = reinterpret_cast<const uint4*>(a.qx + (int64_t)(p / a.top_k) * a.qrow);
      uint4* d4 = reinterpret_cast<uint4*>(act + (int64_t)m * a.qrow);
      for (int64_t i = tid; i < a.qrow / 16; i += blockDim.x) d4[i] = __ldg(s4 + i);
    }
    __syncthreads();
    for (int rr = warp * RPW; rr < nr; rr += (blockDim.x / 32) * RPW) {
      const int r = rr + sub;
      const bool live = r < nr;
      const uint8_t* wrow = wt + (int64_t)(live ? r : 0) * a.row_bytes;
      for (int mb = 0; mb < nm; mb += 8) {
        float acc[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) acc[m] = 0.0f;
        if (live) {
          for (int c = sl; c < nchunks; c += LPR) {
            const int i = c / C::CPB, iqs = C::VDR * (c % C::CPB);
            const uint8_t* bx = wrow + (int64_t)i * C::BYTES;
            const int64_t qb = (int64_t)i * (C::QK / 32);  // first q8_1 block of the chunk
#pragma unroll
            for (int m = 0; m < 8; ++m)
              if (mb + m < nm) {
                const uint8_t* yr = act + (int64_t)(mb + m) * a.qrow;
                acc[m] += kt_vec_dot<TYPE>(bx, yr + 32 * qb, yr + a.kpad + 4 * qb, iqs, grid_s);
              }
          }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          float t = acc[m];
#pragma unroll
          for (int mask = LPR / 2; mask > 0; mask >>= 1) t += __shfl_xor_sync(0xffffffffu, t, mask);
          if (live && sl == 0 && mb + m < nm) {
            const int p = a.order[start + m0 + mb + m];
            kt_store_act<DT>(a.y, (int64_t)p * a.rows + r0 + r, t);
          }
        }
      }
    }
  }
}

// q8_1 of one activation row into shared memory (split layout), one thread per 8 consecutive
// values, so a 32-value block is 4 adjacent lanes. The values equal the 32-lanes-per-block
// quantizer's (kt_quantize_q8_1_kernel): amax is exact in any order, and the block sum follows
// the same addition tree as that kernel's xor butterfly (partners 16, 8, 4, 2, 1: values 16
// apart, then 8 apart -- the lanes two and one apart here -- then 4, 2 and 1 apart inside the
// thread), so d, the codes and the half2 (d, sum) match bit for bit. One 16-byte load per
// thread instead of one 2-byte load and ten shuffles per value. Needs cols % 32 == 0 (every GGUF
// block size) and a 16-byte aligned row start; blockDim a multiple of 32.
template <int DT>
__device__ __forceinline__ void kt_quantize_row_split(const void* __restrict__ x, int64_t off, int cols, int64_t kpad,
                                                      uint8_t* act, int tid, int nthreads) {
  for (int64_t u = tid; u < kpad / 8; u += nthreads) {  // kpad / 8 is a multiple of 64: whole warps
    const int64_t c0 = u * 8;
    float v[8];
    if (c0 < cols) {
      if constexpr (DT == KT_DT_F32) {
        const float4* s4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off + c0);
        const float4 lo = __ldg(s4), hi = __ldg(s4 + 1);
        v[0] = lo.x, v[1] = lo.y, v[2] = lo.z, v[3] = lo.w, v[4] = hi.x, v[5] = hi.y, v[6] = hi.z, v[7] = hi.w;
      } else {
        const uint4 r = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + off + c0));
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] = DT == KT_DT_F16 ? kt_h2f((uint16_t)(w[j] & 0xffff)) : kt_bf2f((uint16_t)(w[j] & 0xffff));
          v[2 * j + 1] = DT == KT_DT_F16 ? kt_h2f((uint16_t)(w[j] >> 16)) : kt_bf2f((uint16_t)(w[j] >> 16));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.0f;
    }
    float amax = fabsf(v[0]);
#pragma unroll
    for (int j = 1; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = v[j] + __shfl_xor_sync(0xffffffffu, v[j], 2);  // values 16 apart
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = t[j] + __shfl_xor_sync(0xffffffffu, t[j], 1);  // 8 apart
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = t[j] + t[j + 4];
    t[0] = t[0] + t[2];
    t[1] = t[1] + t[3];
    const float sum = t[0] + t[1];
    const float d = amax / 127;
    uint32_t q[2] = {0u, 0u};
    if (amax != 0.0f) {
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j / 4] |= (uint32_t)(uint8_t)(int8_t)roundf(v[j] / d) << (8 * (j % 4));
    }
    *reinterpret_cast<uint2*>(act + c0) = make_uint2(q[0], q[1]);
    if ((u & 3) == 0) *reinterpret_cast<half2*>(act + kpad + 4 * (u / 4)) = __halves2half2(__float2half(d), __float2half(sum));
  }
}

// Fused path for a handful of routes (a decode step of up to a few tokens): one launch, one CTA
// per (route, tile of 8, 16 or 32 rows). One thread streams the tile's raw rows into shared memory with a
// single bulk copy while the CTA quantizes the route's activation row into shared memory (the
// reference's q8_1 rounding, in the split layout); then each row is the per-route arithmetic of
// kt_moe_vec_kernel (the reference's lane-to-chunk order and butterfly), so the sums are the
// same bit for bit. The separate quantize-and-group launch and its global round trip are gone,
// which is most of a one-token projection's time. Routes not on this device write zero rows.
// Route counts up to 40 take the one-launch path. Measured at four tokens (20-call graph replays,
// one-launch / grouped): config 2 Q4_K gate/up (31 routes) 18.5 / 17.9 us, Q6_K down (32 routes)
// 15.7 / 17.0 us, config 3 IQ3_S gate/up (40 routes) 23.9 / 25.5 us.
constexpr int kFusedMaxRoutes = 40;
constexpr int kFusedSmemBytes = 192 * 1024;  // dynamic: the tile and the q8_1 row (code books are static)

template <int TYPE, int DT, int LPR>
__global__ void __launch_bounds__(256) kt_moe_vec_fused_kernel(const KtVecArgs a, const void* __restrict__ x,
                                                               const int32_t* __restrict__ ids, int n_slots) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  __shared__ __align__(8) uint64_t full;
  using C = KtChunk<TYPE>;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int R = a.rows_per_cta;
  const int tiles = a.rows / R;
  const int64_t p = blockIdx.x / tiles;
  const int r0 = (blockIdx.x % tiles) * R;
  // the call's status word: block 0 clears it when it starts, long before any bounded wait of
  // this grid could run out
  if (blockIdx.x == 0 && tid == 0 && a.status) *a.status = KT_DEV_OK;
  const int32_t e = ids[p];
  if (e < 0 || e >= n_slots) {
    for (int i = tid; i < R; i += blockDim.x) kt_store_act<DT>(a.y, p * a.rows + r0 + i, 0.0f);
    return;
  }
  const int64_t tile_bytes = (int64_t)R * a.row_bytes;  // a 16-byte multiple (host check)
  uint8_t* wt = smem;
  uint8_t* act = smem + ((tile_bytes + 127) & ~(int64_t)127);
  const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[e])
                                 : a.w + (int64_t)e * a.rows * a.row_bytes;
  const uint8_t* src = wbase + (int64_t)r0 * a.row_bytes;
  // a slot table may hold any address: bulk copies only from 16-byte aligned tiles
  const bool bulk = (((uintptr_t)src) & 15) == 0;
  if (bulk && tid == 0) {
    kt_mbar_init(&full, 1);
    kt_fence_mbar_init();
    kt_mbar_arrive_expect_tx(&full, (uint32_t)tile_bytes);
    kt_bulk_g2s(wt, src, (uint32_t)tile_bytes, &full);
  }
  if (!bulk) {  // GGUF blocks are always 2-byte aligned
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(wt);
    for (int64_t i = tid; i < tile_bytes / 2; i += blockDim.x) d2[i] = __ldg(s2 + i);
  }
  kt_stage_grid<TYPE>(grid_s, tid, blockDim.x);
  kt_quantize_row_split<DT>(x, (p / a.top_k) * a.cols, a.cols, a.kpad, act, tid, blockDim.x);
  __syncthreads();
  if (bulk && !kt_mbar_wait(&full, 0, a.status, nullptr)) return;  // the one copy in flight never landed
  const int nchunks = (a.cols / C::QK) * C::CPB;
  constexpr int RPW = 32 / LPR;
  const int sub = lane / LPR, sl = lane % LPR;
  for (int rr = warp * RPW; rr < R; rr += (blockDim.x / 32) * RPW) {
    const int r = rr + sub;
    const uint8_t* wrow = wt + (int64_t)r * a.row_bytes;
    float acc = 0.0f;
    for (int c = sl; c < nchunks; c += LPR) {
      const int i = c / C::CPB, iqs = C::VDR * (c % C::CPB);
      const int64_t qb = (int64_t)i * (C::QK / 32);
      acc += kt_vec_dot<TYPE>(wrow + (int64_t)i * C::BYTES, act + 32 * qb, act + a.kpad + 4 * qb, iqs, grid_s);
    }
#pragma unroll
    for (int mask = LPR / 2; mask > 0; mask >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, mask);
    if (sl == 0) kt_store_act<DT>(a.y, p * a.rows + r0 + r, acc);
  }
}

// One row (this lane's share) against W consecutive members of a group: per-lane sums in the
// reference's chunk order, xor butterfly over the LPR lanes of the row, one store per member.
// W is a compile-time width so that no work is issued for absent members.
template <int TYPE, int DT, int LPR, int W>
__device__ __forceinline__ void kt_vec_row_members(const KtVecArgs& a, const uint8_t* wrow, bool live, int nchunks,
                                                   int sl, int start, int mb, int64_t out_row,
                                                   const uint32_t* grid) {
  using C = KtChunk<TYPE>;
  const uint8_t* yrow[W];
#pragma unroll
  for (int m = 0; m < W; ++m) yrow[m] = a.qx + (int64_t)(a.order[start + mb + m] / a.top_k) * a.qrow;
  float acc[W];
#pragma unroll
  for (int m = 0; m < W; ++m) acc[m] = 0.0f;
  if (live) {
    for (int c = sl; c < nchunks; c += LPR) {
      const int i = c / C::CPB, iqs = C::VDR * (c % C::CPB);
      const uint8_t* bx = wrow + (int64_t)i * C::BYTES;
      const int64_t qb = (int64_t)i * (C::QK / 32);  // first q8_1 block of the chunk
#pragma unroll
      for (int m = 0; m < W; ++m) acc[m] += kt_vec_dot<TYPE>(bx, yrow[m] + 32 * qb, yrow[m] + a.kpad + 4 * qb, iqs, grid);
    }
  }
#pragma unroll
  for (int m = 0; m < W; ++m) {
    float t = acc[m];
#pragma unroll
    for (int mask = LPR / 2; mask > 0; mask >>= 1) t += __shfl_xor_sync(0xffffffffu, t, mask);
    if (live && sl == 0) kt_store_act<DT>(a.y, (int64_t)a.order[start + mb + m] * a.rows + out_row, t);
  }
}

// Pipelined variant for bandwidth: a persistent grid walks (group, row tile) items; one
// thread streams each item's raw rows into a ring of kVecStages shared-memory stages with a
// single 1-D bulk copy (the rows of a tile are contiguous in HBM), so several tiles per SM
// are in flight while the warps compute. The per-row arithmetic (lane-to-chunk assignment,
// per-lane sums in chunk order, xor butterfly) is the kernel's above, so every route's sum is
// the same. Activations are read from the q8_1 buffer in global memory (L1/L2 resident).
constexpr int kVecStages = 4;

template <int TYPE, int DT, int LPR>
__global__ void __launch_bounds__(256) kt_moe_vec_pipe_kernel(const KtVecArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  __shared__ __align__(8) uint64_t full[kVecStages];
  using C = KtChunk<TYPE>;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int n_items = a.groups[0] * a.tiles_per_group;
  const int64_t tile_cap = ((int64_t)a.rows_per_cta * a.row_bytes + 127) & ~(int64_t)127;
  if (tid == 0) {
    for (int i = 0; i < kVecStages; ++i) kt_mbar_init(&full[i], 1);
    kt_fence_mbar_init();
  }
  kt_stage_grid<TYPE>(grid_s, tid, blockDim.x);
  __syncthreads();
  // stage the raw rows of the CTA's j-th item
  auto issue = [&](int j) {
    const int item = blockIdx.x + j * gridDim.x;
    if (item >= n_items) return;
    uint64_t* bar = &full[j % kVecStages];
    const int g = item / a.tiles_per_group, r0 = (item % a.tiles_per_group) * a.rows_per_cta;
    const int slot = a.groups[1 + 3 * g + 0];
    if (slot < 0) {
      kt_mbar_arrive(bar);
      return;
    }
    const int nr = min(a.rows_per_cta, a.rows - r0);
    const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                   : a.w + (int64_t)slot * a.rows * a.row_bytes;
    const uint32_t bytes = (uint32_t)((int64_t)nr * a.row_bytes);
    kt_mbar_arrive_expect_tx(bar, bytes);
    kt_bulk_g2s(smem + (j % kVecStages) * tile_cap, wbase + (int64_t)r0 * a.row_bytes, bytes, bar);
  };
  if (tid == 0)
    for (int j = 0; j < kVecStages; ++j) issue(j);
  const int nblocks = a.cols / C::QK;
  const int nchunks = nblocks * C::CPB;
  constexpr int RPW = 32 / LPR;
  const int sub = lane / LPR, sl = lane % LPR;
  bool ok = true;
  for (int j = 0; blockIdx.x + j * gridDim.x < n_items; ++j) {
    const int item = blockIdx.x + j * gridDim.x;
    const int g = item / a.tiles_per_group, r0 = (item % a.tiles_per_group) * a.rows_per_cta;
    const int slot = a.groups[1 + 3 * g + 0];
    const int start = a.groups[1 + 3 * g + 1];
    const int count = a.groups[1 + 3 * g + 2];
    const int nr = min(a.rows_per_cta, a.rows - r0);
    if (!kt_mbar_wait(&full[j % kVecStages], (j / kVecStages) & 1, a.status, nullptr)) {
      // a copy that never landed (recorded in the status word): wait, bounded, for the other
      // copies this CTA issued, then leave
      ok = false;
      if (tid == 0)
        for (int jj = j + 1; jj < j + kVecStages && blockIdx.x + jj * gridDim.x < n_items; ++jj)
          kt_mbar_wait(&full[jj % kVecStages], (jj / kVecStages) & 1, nullptr, nullptr);
      break;
    }
    if (slot < 0) {  // routes not on this device: zero rows
      for (int64_t i = tid; i < (int64_t)count * nr; i += blockDim.x) {
        const int p = a.order[start + i / nr];
        kt_store_act<DT>(a.y, (int64_t)p * a.rows + r0 + i % nr, 0.0f);
      }
    } else {
      const uint8_t* wt = smem + (j % kVecStages) * tile_cap;
      for (int rr = warp * RPW; rr < nr; rr += (blockDim.x / 32) * RPW) {
        const int r = rr + sub;
        const bool live = r < nr;
        const uint8_t* wrow = wt + (int64_t)(live ? r : 0) * a.row_bytes;
        for (int mb = 0; mb < count;) {
          const int left = count - mb;
          if (left >= 4) {
            kt_vec_row_members<TYPE, DT, LPR, 4>(a, wrow, live, nchunks, sl, start, mb, r0 + r, grid_s);
            mb += 4;
          } else if (left >= 2) {
            kt_vec_row_members<TYPE, DT, LPR, 2>(a, wrow, live, nchunks, sl, start, mb, r0 + r, grid_s);
            mb += 2;
          } else {
            kt_vec_row_members<TYPE, DT, LPR, 1>(a, wrow, live, nchunks, sl, start, mb, r0 + r, grid_s);
            mb += 1;
          }
        }
      }
    }
    __syncthreads();  // every warp is done with the stage
    if (tid == 0) issue(j + kVecStages);
  }
  (void)ok;
}

// Member-stationary kernel for the north-star types (Q8_0, Q4_K, Q6_K, IQ3_S): groups of 1, 2, 4 or 8
// routes of one slot (grouped in pieces of kt_vec_ms_piece()) times row tiles of 8R rows are the work
// items of a persistent grid. A warp owns R rows of the tile; its lanes walk the chunks of a
// row as the reference does (lane t: chunks t, t+32, ...), but for each chunk they load the
// members' activation side once (KtAct: q8_1 ints, scales and the row-independent integer
// sums) and each row's weight side once (KtWgt), and combine every (row, member) pair with the
// chunk's own fp32 expression (kt_dot_split). Per-lane sums run in chunk order and end in the
// same xor butterfly, so every route's result is the reference's bit for bit; the saving is
// the activation work per row and the weight work per member.
// `tile` holds the raw rows from r0 on, row_bytes apart (the slot in global memory, or a
// staged copy of the tile in shared memory)
template <int TYPE, int DT, int R, int WM, typename WT = KtWgt<TYPE>>
__device__ __forceinline__ void kt_ms_item(const KtVecArgs& a, const uint8_t* tile, int start, int r0,
                                           const uint32_t* grid) {
  using C = KtChunk<TYPE>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint8_t* yrow[WM];
#pragma unroll
  for (int m = 0; m < WM; ++m) yrow[m] = a.qx + (int64_t)(a.order[start + m] / a.top_k) * a.qrow;
  float acc[R][WM];
#pragma unroll
  for (int j = 0; j < R; ++j)
#pragma unroll
    for (int m = 0; m < WM; ++m) acc[j][m] = 0.0f;
  const int nchunks = (a.cols / C::QK) * C::CPB;
  const int rbase = r0 + warp * R;
  for (int c = lane; c < nchunks; c += 32) {
    const int i = c / C::CPB, iqs = C::VDR * (c % C::CPB);
    const int64_t qb = (int64_t)i * (C::QK / 32);  // first q8_1 block of the chunk
    KtAct<TYPE> act[WM];
#pragma unroll
    for (int m = 0; m < WM; ++m) kt_act_load(act[m], yrow[m] + 32 * qb, yrow[m] + a.kpad + 4 * qb, iqs);
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int r = rbase + j;
      if (r < a.rows) {
        WT w;
        kt_wgt_load(w, tile + (int64_t)(r - r0) * a.row_bytes + (int64_t)i * C::BYTES, iqs, grid);
#pragma unroll
        for (int m = 0; m < WM; ++m) acc[j][m] += kt_dot_split(w, act[m]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < R; ++j)
#pragma unroll
    for (int m = 0; m < WM; ++m) {
      float t = acc[j][m];
#pragma unroll
      for (int mask = 16; mask > 0; mask >>= 1) t += __shfl_xor_sync(0xffffffffu, t, mask);
      if (lane == 0 && rbase + j < a.rows) kt_store_act<DT>(a.y, (int64_t)a.order[start + m] * a.rows + rbase + j, t);
    }
}

// one group of `count` routes (1, 2, 4 or 8, from the grouping in pieces of WMAX) on one tile
template <int TYPE, int DT, int R, int WMAX, typename WT = KtWgt<TYPE>>
__device__ __forceinline__ void kt_ms_group(const KtVecArgs& a, const uint8_t* tile, int start, int count, int r0,
                                            const uint32_t* grid) {
  switch (count) {
    case 8:
      if constexpr (WMAX >= 8) {
        kt_ms_item<TYPE, DT, R, 8, WT>(a, tile, start, r0, grid);
      } else {  // not produced with piece WMAX; in parts of WMAX if it were
        for (int m = 0; m < 8; m += WMAX) kt_ms_item<TYPE, DT, R, WMAX, WT>(a, tile, start + m, r0, grid);
      }
      break;
    case 4:
      if constexpr (WMAX >= 4) {
        kt_ms_item<TYPE, DT, R, 4, WT>(a, tile, start, r0, grid);
      } else {
        kt_ms_item<TYPE, DT, R, 2, WT>(a, tile, start, r0, grid);
        kt_ms_item<TYPE, DT, R, 2, WT>(a, tile, start + 2, r0, grid);
      }
      break;
    case 2: kt_ms_item<TYPE, DT, R, 2, WT>(a, tile, start, r0, grid); break;
    default:  // 1 (any other count only if the groups were not cut in powers of two)
      for (int m = 0; m < count; ++m) kt_ms_item<TYPE, DT, R, 1, WT>(a, tile, start + m, r0, grid);
  }
}

// WMAX 8: two CTAs per SM (128 registers); WMAX 4: three (80), more warps to hide the loads
template <int TYPE, int DT, int R, int WMAX>
__global__ void __launch_bounds__(256, WMAX >= 8 ? 2 : 3) kt_moe_vec_ms_kernel(const KtVecArgs a) {
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  if constexpr (kt_grid_words(TYPE) > 0) {
    kt_stage_grid<TYPE>(grid_s, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  constexpr int kRows = 8 * R;
  const int tiles = (a.rows + kRows - 1) / kRows;
  const int n_items = a.groups[0] * tiles;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int g = item / tiles, r0 = (item % tiles) * kRows;
    const int slot = a.groups[1 + 3 * g + 0];
    const int start = a.groups[1 + 3 * g + 1];
    const int count = a.groups[1 + 3 * g + 2];
    if (slot < 0) {  // routes not on this device: zero rows
      const int nr = min(kRows, a.rows - r0);
      for (int64_t i = threadIdx.x; i < (int64_t)count * nr; i += blockDim.x) {
        const int p = a.order[start + i / nr];
        kt_store_act<DT>(a.y, (int64_t)p * a.rows + r0 + i % nr, 0.0f);
      }
      continue;
    }
    const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                   : a.w + (int64_t)slot * a.rows * a.row_bytes;
    kt_ms_group<TYPE, DT, R, WMAX>(a, wbase + (int64_t)r0 * a.row_bytes, start, count, r0, grid_s);
  }
}

// Member-stationary kernel with the weight tiles staged in shared memory: the same work items
// (a group of routes of one slot x a tile of 8R rows) and the same per-row arithmetic as
// kt_moe_vec_ms_kernel, so every route's sum is unchanged bit for bit, but each tile's raw rows
// (contiguous in HBM) arrive by one 1-D bulk copy into a ring of a.stages shared-memory stages,
// issued a.stages items ahead by one thread. Many copies of whole tiles stay in flight per SM,
// so HBM latency hides behind the previous tiles' arithmetic, and the warps read the weights
// from shared memory instead of issuing small global loads.
// BOOK (IQ3_S): 0 the 512-word grid and sign masks (KtWgt), 1 the signed code book (KtWgtS3,
// 32 KB of shared memory after the stages; the same integers with fewer instructions and shared
// loads per chunk).
constexpr int kMsbMaxStages = 4;

template <int TYPE, int DT, int R, int WMAX, int BOOK = 0>
__global__ void __launch_bounds__(256, 2) kt_moe_vec_msb_kernel(const KtVecArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t grid_s[BOOK ? 1 : KtGridSmem<TYPE>::WORDS];
  __shared__ __align__(8) uint64_t full[kMsbMaxStages];
  constexpr int kRows = 8 * R;
  const int tid = threadIdx.x;
  const int S = a.stages;
  const int tiles = (a.rows + kRows - 1) / kRows;
  const int n_items = a.groups[0] * tiles;
  const int64_t tile_cap = ((int64_t)kRows * a.row_bytes + 127) & ~(int64_t)127;
  uint32_t* book = grid_s;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) kt_mbar_init(&full[i], 1);
    kt_fence_mbar_init();
  }
  if constexpr (BOOK == 1) {
    book = reinterpret_cast<uint32_t*>(smem + S * tile_cap);
    kt_stage_iq3s_signed(book, tid, blockDim.x);
  } else {
    kt_stage_grid<TYPE>(grid_s, tid, blockDim.x);
  }
  __syncthreads();
  auto issue = [&](int j) {  // the raw rows of this CTA's j-th item into stage j % S
    const int item = blockIdx.x + j * gridDim.x;
    if (item >= n_items) return;
    uint64_t* bar = &full[j % S];
    const int g = item / tiles, r0 = (item % tiles) * kRows;
    const int slot = a.groups[1 + 3 * g + 0];
    if (slot < 0) {
      kt_mbar_arrive(bar);  // nothing to copy for routes that are not on this device
      return;
    }
    const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                   : a.w + (int64_t)slot * a.rows * a.row_bytes;
    const uint32_t bytes = (uint32_t)((int64_t)min(kRows, a.rows - r0) * a.row_bytes);
    const uint8_t* src = wbase + (int64_t)r0 * a.row_bytes;
    if (((uintptr_t)src) & 15) {  // a slot table may hold any address: copy such a tile with plain loads
      const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
      uint16_t* d2 = reinterpret_cast<uint16_t*>(smem + (j % S) * tile_cap);
      for (uint32_t i = 0; i < bytes / 2; ++i) d2[i] = __ldg(s2 + i);
      kt_mbar_arrive(bar);
      return;
    }
    kt_mbar_arrive_expect_tx(bar, bytes);
    kt_bulk_g2s(smem + (j % S) * tile_cap, src, bytes, bar);
  };
  if (tid == 0)
    for (int j = 0; j < S; ++j) issue(j);
  for (int j = 0; blockIdx.x + j * gridDim.x < n_items; ++j) {
    const int item = blockIdx.x + j * gridDim.x;
    const int g = item / tiles, r0 = (item % tiles) * kRows;
    const int slot = a.groups[1 + 3 * g + 0];
    const int start = a.groups[1 + 3 * g + 1];
    const int count = a.groups[1 + 3 * g + 2];
    if (!kt_mbar_wait(&full[j % S], (j / S) & 1, a.status, nullptr)) {
      // a copy that never landed (recorded in the status word): wait, bounded, for the other
      // copies this CTA has in flight, then leave
      if (tid == 0)
        for (int jj = j + 1; jj < j + S && blockIdx.x + jj * gridDim.x < n_items; ++jj)
          kt_mbar_wait(&full[jj % S], (jj / S) & 1, nullptr, nullptr);
      break;
    }
    if (slot < 0) {  // routes not on this device: zero rows
      const int nr = min(kRows, a.rows - r0);
      for (int64_t i = tid; i < (int64_t)count * nr; i += blockDim.x) {
        const int p = a.order[start + i / nr];
        kt_store_act<DT>(a.y, (int64_t)p * a.rows + r0 + i % nr, 0.0f);
      }
    } else if constexpr (BOOK == 1) {
      kt_ms_group<TYPE, DT, R, WMAX, KtWgtS3>(a, smem + (j % S) * tile_cap, start, count, r0, book);
    } else {
      kt_ms_group<TYPE, DT, R, WMAX>(a, smem + (j % S) * tile_cap, start, count, r0, book);
    }
    __syncthreads();  // every warp is done with the stage
    if (tid == 0) issue(j + S);
  }
}

static int vec_num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

template <int TYPE, int DT, int LPR>
static int launch_pipe(const KtVecArgs& a, int max_groups, cudaStream_t s) {
  const int64_t tile_cap = ((int64_t)a.rows_per_cta * a.row_bytes + 127) & ~(int64_t)127;
  const size_t smem = (size_t)(kVecStages * tile_cap);
  auto k = kt_moe_vec_pipe_kernel<TYPE, DT, LPR>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -3;
  const int64_t max_items = (int64_t)max_groups * a.tiles_per_group;
  const int64_t ctas = 3 * (int64_t)vec_num_sms();
  k<<<(unsigned)(max_items < ctas ? max_items : ctas), 256, smem, s>>>(a);
  return 0;
}

template <int TYPE, int DT>
static int launch_vec_t(const KtVecArgs& a, int max_groups, int lpr, size_t smem, cudaStream_t s) {
  if (a.tiles_per_group > 0) return lpr == 16 ? launch_pipe<TYPE, DT, 16>(a, max_groups, s)
                                              : launch_pipe<TYPE, DT, 32>(a, max_groups, s);
  dim3 grid((a.rows + a.rows_per_cta - 1) / a.rows_per_cta, max_groups);
  if (lpr == 16) {
    auto k = kt_moe_vec_kernel<TYPE, DT, 16>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, 256, smem, s>>>(a);
  } else {
    auto k = kt_moe_vec_kernel<TYPE, DT, 32>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, 256, smem, s>>>(a);
  }
  return 0;
}

// routes per group of the member-stationary kernel: 4 (KT_B200_VEC_MS_PIECE=8 for tuning runs).
// Measured on config 2's Q4_K gate/up (CUDA-graph replays, B200): groups of 4 at three CTAs per
// SM beat groups of 8 at two (M=64: 156 vs 186 us with eight rows per warp).
int kt_vec_ms_piece() {
  static const int p = [] {
    const char* e = getenv("KT_B200_VEC_MS_PIECE");
    return e && atoi(e) == 8 ? 8 : 4;
  }();
  return p;
}

// the member-stationary kernel's rows per warp: 8 from 64 routes, else 4 (KT_B200_VEC_MS_R=1|2|4|8
// for tuning runs). Measured on config 2's Q4_K gate/up against the reference kernel (graph
// replays): M=4 (31 routes) 22.6 us with 4 rows (24.7 reference), M=16 51.3 us and M=64 155.8 us
// with 8 (53.7 and 188.6); 16 rows spill and lose (187 us at M=64).
// Bulk-staged variant (kt_moe_vec_msb_kernel), for IQ3_S: tiles of 8R rows, R the largest of 4,
// 2, 1 whose tile fits kMsbTileBytes, at least two stages within kMsbSmemBytes (two CTAs per SM),
// tiles whose bytes are a 16-byte multiple covering the slot exactly, and a 16-byte aligned weight
// base (or slot table). Returns R, or 0 when the global-load kernel runs. Measured (B200, graph
// replays, config 3's IQ3_S gate/up): 82.2 / 244.2 us at 16 / 64 tokens against 96.2 / 299.5 for
// the global-load kernel; on config 2's Q4_K gate/up and Q6_K down (about 11 routes per slot at 64
// tokens) it was slower (168.8 vs 155.2, 147.7 vs 140.0 us), so those types keep the global-load
// kernel. KT_B200_VEC_MSB=0 turns it off, =all takes it for every type (tuning runs).
constexpr int64_t kMsbTileBytes = 36 * 1024;
constexpr int64_t kMsbSmemBytes = 100 * 1024;
// IQ3_S's code book in the bulk-staged kernel (see kt_moe_vec_msb_kernel): the signed book (32 KB
// of the shared-memory budget) unless KT_B200_VEC_IQ3S_BOOK=0. Config 3's gate/up (B200, L2
// flushed): 236 / 87 us at 64 / 16 tokens against 251 / 91 with the plain grid.
static int msb_book(int type) {
  static const int book = [] {
    const char* e = getenv("KT_B200_VEC_IQ3S_BOOK");
    return e && e[0] == '0' ? 0 : 1;
  }();
  return type == KT_IQ3_S ? book : 0;
}
static int pick_msb_rows(const KtVecArgs& a, int type, int* stages) {
  static const int mode = [] {  // 0 off, 1 IQ3_S, 2 every type
    const char* e = getenv("KT_B200_VEC_MSB");
    return !e ? 1 : e[0] == '0' ? 0 : strcmp(e, "all") == 0 ? 2 : 1;
  }();
  if (mode == 0 || (mode == 1 && type != KT_IQ3_S)) return 0;
  if (!a.table && (((uintptr_t)a.w) & 15)) return 0;
  const int64_t budget = kMsbSmemBytes - (msb_book(type) ? 4 * kIq3sBookWords : 0);
  for (int R = 4; R >= 1; R /= 2) {
    const int64_t rows = 8 * R, bytes = rows * a.row_bytes;
    if (bytes > kMsbTileBytes || bytes % 16 || a.rows % rows) continue;
    const int64_t cap = (bytes + 127) & ~(int64_t)127;
    const int64_t st = budget / cap;
    if (st < 2) continue;
    *stages = (int)(st < kMsbMaxStages ? st : kMsbMaxStages);
    return R;
  }
  return 0;
}

template <int TYPE, int DT, int R, int WM>
static int launch_msb_t(KtVecArgs a, int stages, int max_groups, cudaStream_t s) {
  a.stages = stages;
  const int64_t cap = ((int64_t)8 * R * a.row_bytes + 127) & ~(int64_t)127;
  constexpr bool kBooks = TYPE == KT_IQ3_S;
  const int book = kBooks ? msb_book(TYPE) : 0;
  const size_t smem = (size_t)(stages * cap) + (book ? 4 * kIq3sBookWords : 0);
  auto k = book ? kt_moe_vec_msb_kernel<TYPE, DT, R, WM, kBooks ? 1 : 0> : kt_moe_vec_msb_kernel<TYPE, DT, R, WM, 0>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -3;
  const int64_t tiles = (a.rows + 8 * R - 1) / (8 * R);
  const int64_t items = (int64_t)max_groups * tiles, cap_ctas = 2 * (int64_t)vec_num_sms();
  k<<<(unsigned)(items < cap_ctas ? (items > 0 ? items : 1) : cap_ctas), 256, smem, s>>>(a);
  return 0;
}

template <int TYPE, int DT>
static int launch_ms(const KtVecArgs& a, int max_groups, cudaStream_t s) {
  static const int forced = [] {
    const char* e = getenv("KT_B200_VEC_MS_R");
    return e ? atoi(e) : 0;
  }();
  int stages = 0;
  const int wmax = kt_vec_ms_piece();
  if (const int Rb = pick_msb_rows(a, TYPE, &stages)) {
    if (wmax == 4) {
      if (Rb == 4) return launch_msb_t<TYPE, DT, 4, 4>(a, stages, max_groups, s);
      if (Rb == 2) return launch_msb_t<TYPE, DT, 2, 4>(a, stages, max_groups, s);
      return launch_msb_t<TYPE, DT, 1, 4>(a, stages, max_groups, s);
    }
    if (Rb == 4) return launch_msb_t<TYPE, DT, 4, 8>(a, stages, max_groups, s);
    if (Rb == 2) return launch_msb_t<TYPE, DT, 2, 8>(a, stages, max_groups, s);
    return launch_msb_t<TYPE, DT, 1, 8>(a, stages, max_groups, s);
  }
  const int R = forced == 1 || forced == 2 || forced == 4 || forced == 8 ? forced : max_groups >= 64 ? 8 : 4;
  const int64_t tiles = (a.rows + 8 * R - 1) / (8 * R);
  const int64_t items = (int64_t)max_groups * tiles, cap = 8 * (int64_t)vec_num_sms();
  const unsigned grid = (unsigned)(items < cap ? (items > 0 ? items : 1) : cap);
#define KT_MS_LAUNCH(RR, WW) kt_moe_vec_ms_kernel<TYPE, DT, RR, WW><<<grid, 256, 0, s>>>(a)
#define KT_MS_ROWS(WW)            \
  if (R == 8) KT_MS_LAUNCH(8, WW);  \
  else if (R == 4) KT_MS_LAUNCH(4, WW); \
  else if (R == 2) KT_MS_LAUNCH(2, WW); \
  else KT_MS_LAUNCH(1, WW);
  if (wmax == 4) {
    KT_MS_ROWS(4)
  } else {
    KT_MS_ROWS(8)
  }
#undef KT_MS_ROWS
#undef KT_MS_LAUNCH
  return 0;
}

template <int TYPE>
static int launch_ms_dt(const KtVecArgs& a, int dtype, int max_groups, cudaStream_t s) {
  switch (dtype) {
    case KT_DT_F32: return launch_ms<TYPE, KT_DT_F32>(a, max_groups, s);
    case KT_DT_F16: return launch_ms<TYPE, KT_DT_F16>(a, max_groups, s);
    case KT_DT_BF16: return launch_ms<TYPE, KT_DT_BF16>(a, max_groups, s);
  }
  return -1;
}

// whether kt_launch_moe_vec runs the member-stationary kernel for this type, width and number
// of routes (then the routes are grouped in pieces of kt_vec_ms_piece()): the north-star types
// (Q8_0, Q4_K, Q6_K, IQ3_S), rows of more than 16 chunks (32 lanes per row), 16 routes or more, unless
// KT_B200_VEC_MS=0. Measured against the reference kernel (graph replays, B200): config 2's Q6_K
// down 45.2 / 141.4 us at 16 / 64 tokens (reference 56.0 / 202.9, the staged kernels 72.2 /
// 263.3), config 3's IQ3_S gate/up 30.8 / 96.2 / 299.5 us at 4 / 16 / 64 tokens (reference 40.0 /
// 99.5 / 362.6).
bool kt_vec_ms_ok(int type, int cols, int64_t routes) {
  static const int64_t min_routes = [] {  // KT_B200_VEC_MS_MIN_ROUTES for tuning runs
    const char* e = getenv("KT_B200_VEC_MS_MIN_ROUTES");
    return e ? (int64_t)atoll(e) : (int64_t)16;
  }();
  if (routes < min_routes) return false;  // fewer routes: the staged kernels are quicker (measured)
  static const bool on = [] {
    const char* e = getenv("KT_B200_VEC_MS");
    return !(e && e[0] == '0');
  }();
  if (!on) return false;
  static const bool all = [] {  // KT_B200_VEC_MS_ALL=0: Q6_K and IQ3_S on the staged kernels (tuning runs)
    const char* e = getenv("KT_B200_VEC_MS_ALL");
    return !(e && e[0] == '0');
  }();
  const int cpb = type == KT_Q8_0    ? KtChunk<KT_Q8_0>::CPB
                  : type == KT_Q4_K  ? KtChunk<KT_Q4_K>::CPB
                  : !all             ? 0
                  : type == KT_Q6_K  ? KtChunk<KT_Q6_K>::CPB
                  : type == KT_IQ3_S ? KtChunk<KT_IQ3_S>::CPB
                                     : 0;
  const KtBlockInfo bi = kt_block_info(type);
  return cpb > 0 && bi.qk > 0 && cols % bi.qk == 0 && (int64_t)cols / bi.qk * cpb > 16;
}

template <int TYPE>
static int launch_vec_dt(const KtVecArgs& a, int dtype, int max_groups, int lpr, size_t smem, cudaStream_t s) {
  switch (dtype) {
    case KT_DT_F32: return launch_vec_t<TYPE, KT_DT_F32>(a, max_groups, lpr, smem, s);
    case KT_DT_F16: return launch_vec_t<TYPE, KT_DT_F16>(a, max_groups, lpr, smem, s);
    case KT_DT_BF16: return launch_vec_t<TYPE, KT_DT_BF16>(a, max_groups, lpr, smem, s);
  }
  return -1;
}

// Rows per CTA: a power of two giving a tile of at most ~24 KB of raw rows, at least 8.
static int pick_rows_per_cta(int64_t row_bytes, int rows) {
  int rpc = 8;
  while (rpc < 64 && (int64_t)(rpc * 2) * row_bytes <= 24 * 1024) rpc *= 2;
  return rpc;
}

// Pipelined path: tiles of at most 16 KB whose bytes are a 16-byte multiple (1-D bulk copies
// need 16-byte aligned addresses and sizes), a whole number of tiles per slot, and a
// 16-byte aligned weight base (or slot table). Returns the rows per tile, or 0.
static int pick_pipe_rows(int64_t row_bytes, int rows, const void* w, int table) {
  if (!table && (((uintptr_t)w) & 15)) return 0;
  for (int rpt = 64; rpt >= 8; rpt /= 2)
    if ((int64_t)rpt * row_bytes <= 16 * 1024 && ((int64_t)rpt * row_bytes) % 16 == 0 && rows % rpt == 0) return rpt;
  return 0;
}

template <int TYPE, int DT>
static int launch_fused_t(const KtVecArgs& a, const void* x, const int32_t* ids, int64_t routes, int n_slots, int lpr,
                          size_t smem, cudaStream_t s) {
  const unsigned grid = (unsigned)(routes * (a.rows / a.rows_per_cta));
  // the shared-memory limit is raised once per instantiation to the most any call asks for
  static const bool ok16 = cudaFuncSetAttribute(kt_moe_vec_fused_kernel<TYPE, DT, 16>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kFusedSmemBytes) == cudaSuccess;
  static const bool ok32 = cudaFuncSetAttribute(kt_moe_vec_fused_kernel<TYPE, DT, 32>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kFusedSmemBytes) == cudaSuccess;
  if (smem > (size_t)kFusedSmemBytes || !(lpr == 16 ? ok16 : ok32)) return -3;
  if (lpr == 16)
    kt_moe_vec_fused_kernel<TYPE, DT, 16><<<grid, 256, smem, s>>>(a, x, ids, n_slots);
  else
    kt_moe_vec_fused_kernel<TYPE, DT, 32><<<grid, 256, smem, s>>>(a, x, ids, n_slots);
  return 0;
}

template <int TYPE>
static int launch_fused_dt(const KtVecArgs& a, int dtype, const void* x, const int32_t* ids, int64_t routes,
                           int n_slots, int lpr, size_t smem, cudaStream_t s) {
  switch (dtype) {
    case KT_DT_F32: return launch_fused_t<TYPE, KT_DT_F32>(a, x, ids, routes, n_slots, lpr, smem, s);
    case KT_DT_F16: return launch_fused_t<TYPE, KT_DT_F16>(a, x, ids, routes, n_slots, lpr, smem, s);
    case KT_DT_BF16: return launch_fused_t<TYPE, KT_DT_BF16>(a, x, ids, routes, n_slots, lpr, smem, s);
  }
  return -1;
}

static int vec_chunks_per_block(int type) {
  return type == KT_Q8_0     ? KtChunk<KT_Q8_0>::CPB
         : type == KT_Q4_K   ? KtChunk<KT_Q4_K>::CPB
         : type == KT_Q6_K   ? KtChunk<KT_Q6_K>::CPB
         : type == KT_IQ3_S  ? KtChunk<KT_IQ3_S>::CPB
         : type == KT_Q2_K   ? KtChunk<KT_Q2_K>::CPB
         : type == KT_Q3_K   ? KtChunk<KT_Q3_K>::CPB
         : type == KT_Q5_K   ? KtChunk<KT_Q5_K>::CPB
         : type == KT_IQ4_XS ? KtChunk<KT_IQ4_XS>::CPB
         : type == KT_Q2_0   ? KtChunk<KT_Q2_0>::CPB
         : kt_grid_words(type) > 0 ? 8  // the i-quants: one sub-block a chunk
                                   : KtChunk<KT_Q4_0>::CPB;  // the 32-value legacy blocks
}

// Rows per CTA of the fused single-launch path, or 0 when it does not take the call. It takes at
// most kFusedMaxRoutes routes with a 16-byte aligned weight base (or a slot table) and rows in
// whole tiles of 8, 16 or 32 whose bytes are a 16-byte multiple (one bulk copy per tile), the
// tile plus the activation row fitting in shared memory. Of those it picks the largest tile that
// still gives three CTAs per SM: a larger tile quantizes the activation row fewer times, a
// smaller one puts more bulk copies in flight. Measured (B200, 20-call graph replays, one token):
// config 2 Q4_K gate/up 8.5 / 7.8 / 7.8 us at 8 / 16 / 32 rows, Q6_K down 8.8 / 6.7 / 5.8 us,
// config 3 IQ3_S gate/up 10.8 / 9.3 / 10.0 us; the rule takes 16, 32 and 16. The activations'
// base must be 16-byte aligned (each thread of the quantizer loads 8 values at once).
// KT_B200_VEC_FUSED=0 turns the path off, KT_B200_VEC_FUSED_ROWS=8/16/32 fixes the tile and
// KT_B200_VEC_FUSED_MAX the largest route count it takes (tuning runs).
static int fused_rows(int type, const void* w, int table, const void* x, int64_t routes, int rows, int cols) {
  static const int mode = [] {
    const char* e = getenv("KT_B200_VEC_FUSED");
    const char* r = getenv("KT_B200_VEC_FUSED_ROWS");
    if (e && e[0] == '0') return 0;
    const int n = r ? atoi(r) : 0;
    return n == 8 || n == 16 || n == 32 ? n : 1;
  }();
  const KtBlockInfo bi = kt_block_info(type);
  static const int64_t max_routes = [] {
    const char* e = getenv("KT_B200_VEC_FUSED_MAX");
    const int n = e ? atoi(e) : 0;
    return (int64_t)(n > 0 && n <= 64 ? n : kFusedMaxRoutes);
  }();
  if (!mode || !bi.qk || routes < 1 || routes > max_routes || rows <= 0 || cols <= 0 || cols % bi.qk) return 0;
  if ((!table && (((uintptr_t)w) & 15)) || (((uintptr_t)x) & 15)) return 0;
  const int64_t row_bytes = (int64_t)cols / bi.qk * bi.bytes;
  int pick = 0;
  for (int R = 32; R >= 8; R /= 2) {
    const int64_t tile = (int64_t)R * row_bytes;
    const int64_t smem = ((tile + 127) & ~(int64_t)127) + kt_q8_1_row_bytes(cols);
    if (rows % R || tile % 16 || smem > kFusedSmemBytes || routes * (rows / R) >= 0x7fffffff) continue;
    pick = R;
    if (mode == R || (mode == 1 && routes * (rows / R) >= 3 * (int64_t)vec_num_sms())) break;
  }
  return pick;
}

bool kt_vec_fused_ok(int type, const void* w, int table, const void* x, int64_t routes, int rows, int cols) {
  return fused_rows(type, w, table, x, routes, rows, cols) != 0;
}

int kt_launch_moe_vec_fused(int type, const void* w, int table, int n_slots, const void* x, int dtype,
                            const int32_t* ids, int64_t routes, int top_k, int rows, int cols, void* y, int* status,
                            cudaStream_t s) {
  const int R = fused_rows(type, w, table, x, routes, rows, cols);
  if (!R) return -1;
  const KtBlockInfo bi = kt_block_info(type);
  KtVecArgs a{};
  a.w = (const uint8_t*)w;
  a.table = table;
  a.kpad = ((int64_t)cols + 511) / 512 * 512;
  a.qrow = kt_q8_1_row_bytes(cols);
  a.top_k = top_k;
  a.rows = rows;
  a.cols = cols;
  a.row_bytes = (int64_t)cols / bi.qk * bi.bytes;
  a.status = status;
  a.y = y;
  a.rows_per_cta = R;
  const size_t smem = (size_t)((((int64_t)R * a.row_bytes + 127) & ~(int64_t)127) + a.qrow);
  const int lpr = cols / bi.qk * vec_chunks_per_block(type) <= 16 ? 16 : 32;
  switch (type) {
#define KT_FUSED_CASE(T)   case T: return launch_fused_dt<T>(a, dtype, x, ids, routes, n_slots, lpr, smem, s);
    KT_FUSED_CASE(KT_Q8_0)
    KT_FUSED_CASE(KT_Q4_0)
    KT_FUSED_CASE(KT_Q4_1)
    KT_FUSED_CASE(KT_Q5_0)
    KT_FUSED_CASE(KT_Q5_1)
    KT_FUSED_CASE(KT_IQ4_NL)
    KT_FUSED_CASE(KT_Q2_K)
    KT_FUSED_CASE(KT_Q3_K)
    KT_FUSED_CASE(KT_Q5_K)
    KT_FUSED_CASE(KT_IQ4_XS)
    KT_FUSED_CASE(KT_Q2_0)
    KT_FUSED_CASE(KT_IQ2_XXS)
    KT_FUSED_CASE(KT_IQ2_XS)
    KT_FUSED_CASE(KT_IQ2_S)
    KT_FUSED_CASE(KT_IQ3_XXS)
    KT_FUSED_CASE(KT_IQ1_S)
    KT_FUSED_CASE(KT_IQ1_M)
    KT_FUSED_CASE(KT_Q4_K)
    KT_FUSED_CASE(KT_Q6_K)
    KT_FUSED_CASE(KT_IQ3_S)
#undef KT_FUSED_CASE
  }
  return -1;
}

int kt_launch_moe_vec(int type, const void* w, int table, const void* qx, int64_t qrow, const int32_t* groups,
                      const int32_t* order, int max_groups, int top_k, int rows, int cols, int dtype, void* y,
                      int* status, cudaStream_t s) {
  const KtBlockInfo bi = kt_block_info(type);
  if (!bi.qk || cols % bi.qk) return -1;
  KtVecArgs a{};
  a.w = (const uint8_t*)w;
  a.table = table;
  a.qx = (const uint8_t*)qx;
  a.qrow = qrow;
  a.kpad = (cols + 511) / 512 * 512;
  a.groups = groups;
  a.order = order;
  a.top_k = top_k;
  a.rows = rows;
  a.cols = cols;
  a.row_bytes = (int64_t)cols / bi.qk * bi.bytes;
  a.status = status;
  a.y = y;
  if (kt_vec_ms_ok(type, cols, max_groups)) {  // grouped with piece 8: max_groups = routes
    switch (type) {
      case KT_Q8_0: return launch_ms_dt<KT_Q8_0>(a, dtype, max_groups, s);
      case KT_Q4_K: return launch_ms_dt<KT_Q4_K>(a, dtype, max_groups, s);
      case KT_Q6_K: return launch_ms_dt<KT_Q6_K>(a, dtype, max_groups, s);
      case KT_IQ3_S: return launch_ms_dt<KT_IQ3_S>(a, dtype, max_groups, s);
    }
  }
  const int pipe_rows = pick_pipe_rows(a.row_bytes, rows, w, table);
  a.rows_per_cta = pipe_rows ? pipe_rows : pick_rows_per_cta(a.row_bytes, rows);
  a.tiles_per_group = pipe_rows ? rows / pipe_rows : 0;
  const int64_t wt_bytes = ((int64_t)a.rows_per_cta * a.row_bytes + 15) & ~(int64_t)15;
  int mpp = 8;
  while (mpp > 1 && wt_bytes + mpp * qrow > 200 * 1024) mpp /= 2;
  a.members_per_pass = mpp;
  const size_t smem = (size_t)(wt_bytes + mpp * qrow);
  if (smem + 4 * (size_t)kt_grid_words(type) > 222 * 1024) return -2;  // + the static code book
  const int nchunks = cols / bi.qk * vec_chunks_per_block(type);
  const int lpr = nchunks <= 16 ? 16 : 32;
  switch (type) {
    case KT_Q8_0: return launch_vec_dt<KT_Q8_0>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q4_0: return launch_vec_dt<KT_Q4_0>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q4_1: return launch_vec_dt<KT_Q4_1>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q5_0: return launch_vec_dt<KT_Q5_0>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q5_1: return launch_vec_dt<KT_Q5_1>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ4_NL: return launch_vec_dt<KT_IQ4_NL>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q2_K: return launch_vec_dt<KT_Q2_K>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q3_K: return launch_vec_dt<KT_Q3_K>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q5_K: return launch_vec_dt<KT_Q5_K>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ4_XS: return launch_vec_dt<KT_IQ4_XS>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q2_0: return launch_vec_dt<KT_Q2_0>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ2_XXS: return launch_vec_dt<KT_IQ2_XXS>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ2_XS: return launch_vec_dt<KT_IQ2_XS>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ2_S: return launch_vec_dt<KT_IQ2_S>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ3_XXS: return launch_vec_dt<KT_IQ3_XXS>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ1_S: return launch_vec_dt<KT_IQ1_S>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ1_M: return launch_vec_dt<KT_IQ1_M>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q4_K: return launch_vec_dt<KT_Q4_K>(a, dtype, max_groups, lpr, smem, s);
    case KT_Q6_K: return launch_vec_dt<KT_Q6_K>(a, dtype, max_groups, lpr, smem, s);
    case KT_IQ3_S: return launch_vec_dt<KT_IQ3_S>(a, dtype, max_groups, lpr, smem, s);
  }
  return -1;
}
