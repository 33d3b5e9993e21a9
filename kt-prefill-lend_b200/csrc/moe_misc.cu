// moe_misc.cu — the small kernels around the expert GEMMs:
//   dequant      GGUF rows -> fp32/f16/bf16 (bit-identical fp32 values to ggml / gguf-py)
//   silu_and_mul h = silu(g) * u on [rows, 2n] (the sgl-kernel op the reference calls,
//                hot/kt_gguf_hot.py:260)
//   combine      res[t] = bf16(sum_k fp32(bf16(out[t,k] * bf16(w[t,k])))) — the rounding
//                and order of the reference's fused combine (hot/kt_gguf_hot.py:43-71)
//   route        HotCache.route: slot / CPU ids by table lookup and route counts
//                (hot/kt_hot_cache.py:62-75, 121-143)
//   topk         router top-k: softmax, and DeepSeek-V3 grouped sigmoid routing
//   permute      counting sort of routes by slot into 256-token tiles for the prefill GEMM
#include <stdlib.h>

#include <type_traits>
#include "gguf_dot.cuh"
#include "gguf_tile.cuh"
#include "kt_kernels.h"

// ------------------------------------------------------------------ dequant

template <int TYPE, int DT>
__global__ void kt_dequant_kernel(const uint8_t* __restrict__ w, int64_t rows, int64_t cols, int64_t row_bytes,
                                  void* __restrict__ out) {
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  if constexpr (kt_grid_words(TYPE) > 0) {
    kt_stage_grid<TYPE>(grid_s, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  const int64_t subs = cols / 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * subs) return;
  const int64_t r = i / subs, sub = i % subs;
  float y[32];
  kt_dq32<TYPE>(w + r * row_bytes, (int)sub, y, grid_s);
#pragma unroll
  for (int j = 0; j < 32; ++j) kt_store_act<DT>(out, r * cols + sub * 32 + j, y[j]);
}

// 2-byte outputs through shared memory on both sides. Sub-block i (32 values) of the matrix
// lands at output values [32 i, 32 i + 32), and its GGUF bytes lie in block i / SPB (SPB
// sub-blocks per GGUF block, rows being whole blocks), so a CTA's 256 sub-blocks read one
// contiguous run of raw bytes and write one contiguous 16 KB run. The CTA copies the raw run
// into shared memory with 16-byte loads, each thread decodes its sub-block there with the same
// decoder as above (kt_dq32, the same values bit for bit), and the CTA stores the bf16 / f16
// run with coalesced 16-byte stores (512 contiguous bytes per warp instruction). Needs 16-byte
// aligned weights and output (every CTA's raw run then starts on a 16-byte boundary: 256 / SPB
// blocks of an even size).
template <int TYPE, int DT>
__global__ void __launch_bounds__(256) kt_dequant16_kernel(const uint8_t* __restrict__ w, int64_t rows, int64_t cols,
                                                           void* __restrict__ out) {
  constexpr int SPB = kt_block_info(TYPE).qk / 32, BS = kt_block_info(TYPE).bytes;
  constexpr int RAW = (256 / SPB) * BS;
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  __shared__ __align__(16) uint4 stage[256 * 4];
  __shared__ __align__(16) uint8_t raw[RAW];
  const int t = threadIdx.x;
  if constexpr (kt_grid_words(TYPE) > 0) kt_stage_grid<TYPE>(grid_s, t, blockDim.x);
  const int64_t n = rows * (cols / 32);
  const int64_t i0 = (int64_t)blockIdx.x * 256;
  const int nsub = (int)(n - i0 < 256 ? n - i0 : 256);  // a multiple of SPB
  const int raw_len = nsub / SPB * BS;
  const uint8_t* g = w + i0 / SPB * BS;
  for (int c = t; c < raw_len / 16; c += 256) reinterpret_cast<uint4*>(raw)[c] = __ldg(reinterpret_cast<const uint4*>(g) + c);
  for (int c = raw_len / 16 * 16 + 2 * t; c < raw_len; c += 512)  // the last CTA's ragged end (even sizes)
    *reinterpret_cast<uint16_t*>(raw + c) = __ldg(reinterpret_cast<const uint16_t*>(g + c));
  __syncthreads();
  if (t < nsub) {
    float y[32];
    kt_dq32<TYPE>(raw, t, y, grid_s);  // the run as one row: sub-block t of the CTA
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if constexpr (DT == KT_DT_BF16) {
        pk[j] = kt_pack_bf2(y[2 * j], y[2 * j + 1]);
      } else {
        const half2 hv = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
        pk[j] = *reinterpret_cast<const uint32_t*>(&hv);
      }
    }
    // chunk j of thread t at 4t + (j ^ ((t >> 1) & 3)): eight neighbouring threads' stores of
    // one j cover all eight 16-byte bank groups
#pragma unroll
    for (int j = 0; j < 4; ++j)
      stage[4 * t + (j ^ ((t >> 1) & 3))] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  }
  __syncthreads();
  uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + i0 * 32);
  for (int c = t; c < 4 * nsub; c += 256) {
    const int owner = c >> 2;
    o[c] = stage[4 * owner + ((c & 3) ^ ((owner >> 1) & 3))];
  }
}

// Persistent, pipelined form of the 2-byte pass for large matrices (the prefill layer's weight
// passes): the same work items (256 sub-blocks: one contiguous raw run in, one contiguous 16 KB
// run out) and the same decoder, so the values are the same bit for bit. Each CTA walks items
// blockIdx.x, +gridDim.x, ...; one thread keeps kDqStages raw runs in flight by 1-D bulk copies
// into a ring of shared-memory stages, and the decoded run leaves by one bulk store from one of
// two staging buffers. Several runs per SM stay in flight on both sides, where the one-shot
// kernel above held one load phase per CTA. The thread writes of a staging buffer are made
// conflict-free without a permuted layout: thread t writes its four 16-byte chunks in the order
// c ^ ((t >> 1) & 3), chosen by two conditional swaps in registers. Waits are bounded: a raw
// copy that never lands records KT_DEV_TIMEOUT in *status (when given) and the CTA stops after
// letting its other copies land. Needs 16-byte aligned weights and output.
constexpr int kDqStages = 3;
template <int TYPE>
struct DqRun {
  static constexpr int SPB = kt_block_info(TYPE).qk / 32, BS = kt_block_info(TYPE).bytes;
  static constexpr int RAW = (256 / SPB) * BS;           // a full item's raw run (a multiple of 16)
  static constexpr int RAWA = (RAW + 127) / 128 * 128;    // its stage, 128-byte aligned
  static constexpr int SMEM = kDqStages * RAWA + 2 * 256 * 64;
};
__device__ __forceinline__ void kt_swap4(uint32_t* a, uint32_t* b, bool c) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = a[i], y = b[i];
    a[i] = c ? y : x;
    b[i] = c ? x : y;
  }
}
__device__ __forceinline__ void kt_bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(kt_smem_addr(src)),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int TYPE, int DT>
__global__ void __launch_bounds__(256, 3) kt_dequant16p_kernel(const uint8_t* __restrict__ w, int64_t n_sub,
                                                               void* __restrict__ out, int* status) {
  using D = DqRun<TYPE>;
  extern __shared__ __align__(128) uint8_t dq_smem[];
  __shared__ uint32_t grid_s[KtGridSmem<TYPE>::WORDS];
  __shared__ __align__(8) uint64_t full[kDqStages];
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int t = threadIdx.x;
  const int64_t items = (n_sub + 255) / 256;
  if (t == 0) {
    for (int i = 0; i < kDqStages; ++i) kt_mbar_init(&full[i], 1);
    *abort_flag = 0;
    kt_fence_mbar_init();
  }
  kt_stage_grid<TYPE>(grid_s, t, blockDim.x);
  __syncthreads();
  auto run_len = [&](int64_t item) -> int {  // raw bytes of an item (the last one may be short)
    const int64_t nsub = n_sub - item * 256 < 256 ? n_sub - item * 256 : 256;
    return (int)(nsub / D::SPB * D::BS);
  };
  auto issue = [&](int j) {  // thread 0: the raw run of this CTA's j-th item into stage j % kDqStages
    const int64_t item = blockIdx.x + (int64_t)j * gridDim.x;
    if (item >= items) return;
    uint64_t* bar = &full[j % kDqStages];
    const int len = run_len(item);
    if (len % 16) {  // a short last run that is not a 16-byte multiple: the CTA loads it itself
      kt_mbar_arrive(bar);
      return;
    }
    kt_mbar_arrive_expect_tx(bar, (uint32_t)len);
    kt_bulk_g2s(dq_smem + (j % kDqStages) * D::RAWA, w + item * D::RAW, (uint32_t)len, bar);
  };
  if (t == 0)
    for (int j = 0; j < kDqStages; ++j) issue(j);
  int j = 0;
  for (;; ++j) {
    const int64_t item = blockIdx.x + (int64_t)j * gridDim.x;
    if (item >= items) break;
    uint8_t* raw = dq_smem + (j % kDqStages) * D::RAWA;
    uint64_t* bar = &full[j % kDqStages];
    const uint32_t parity = (j / kDqStages) & 1;
    // thread 0 alone runs the bounded wait, so the whole CTA takes one decision after the
    // barrier below; it also waits until staging buffer j & 1 is no longer read by the bulk
    // store of item j - 2
    if (t == 0 && kt_mbar_wait(bar, parity, status, abort_flag))
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncthreads();
    if (*abort_flag) break;
    kt_mbar_try_wait(bar, parity);  // the phase has completed: every thread acquires the copy
    const int nsub = (int)(n_sub - item * 256 < 256 ? n_sub - item * 256 : 256);
    const int len = run_len(item);
    if (len % 16) {
      const uint16_t* g = reinterpret_cast<const uint16_t*>(w + item * D::RAW);
      for (int c = t; c < len / 2; c += 256) reinterpret_cast<uint16_t*>(raw)[c] = __ldg(g + c);
      __syncthreads();
    }
    uint4* stage = reinterpret_cast<uint4*>(dq_smem + kDqStages * D::RAWA + (j & 1) * 256 * 64);
    if constexpr (TYPE == KT_Q4_K || TYPE == KT_Q6_K || TYPE == KT_IQ3_S) {
      static_assert(DT == KT_DT_BF16, "the tile decoders produce bf16");
      // the prefill GEMM producers' decoders (gguf_tile.cuh: the same bf16 values, with aligned
      // 16-byte reads and packed f32x2 arithmetic): task = (block u, quarter qt), the quarter's
      // 16 values of each of the block's four 64-value k-steps
      for (int task = t; task < (nsub / D::SPB) * 4; task += 256) {
        const int u = task >> 2, qt = task & 3;
        const int ub = u * D::BS;
        const uint8_t* slot = raw + (ub & ~15);
        const int off = ub & 15;
        KtTileDq<TYPE> dq;
        auto run = [&](auto a16) {
          constexpr bool A16 = decltype(a16)::value;
          dq.template unit<A16>(slot, off, qt);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            uint32_t pk[8];
            dq.template kstep_quarter<A16>(slot, off, kk, qt, pk, grid_s);
            uint4* d = stage + (u * 256 + kk * 64 + qt * 16) / 8;
            d[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            d[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        };
        if constexpr (KtTileDq<TYPE>::kAlignable) {  // Q4_K: 144-byte blocks, always on a boundary
          run(std::integral_constant<bool, true>());
        } else {
          run(std::integral_constant<bool, false>());
        }
      }
      kt_fence_proxy_async_smem();
    } else if (t < nsub) {
      float y[32];
      kt_dq32<TYPE>(raw, t, y, grid_s);
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if constexpr (DT == KT_DT_BF16) {
          pk[i] = kt_pack_bf2(y[2 * i], y[2 * i + 1]);
        } else {
          const half2 hv = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
          pk[i] = *reinterpret_cast<const uint32_t*>(&hv);
        }
      }
      // chunk c moves to register position c ^ sw: step i then writes chunk i ^ sw
      const int sw = (t >> 1) & 3;
      kt_swap4(pk + 0, pk + 4, sw & 1);
      kt_swap4(pk + 8, pk + 12, sw & 1);
      kt_swap4(pk + 0, pk + 8, sw & 2);
      kt_swap4(pk + 4, pk + 12, sw & 2);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        stage[4 * t + (i ^ sw)] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      kt_fence_proxy_async_smem();
    }
    __syncthreads();  // the run is staged; every thread is done with the raw stage
    if (t == 0) {
      kt_bulk_s2g(reinterpret_cast<uint16_t*>(out) + item * 256 * 32, stage, (uint32_t)nsub * 64);
      issue(j + kDqStages);
    }
  }
  if (*abort_flag) kt_drain_ns(200000);  // raw copies issued but never consumed land first
  if (t == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <int TYPE, int DT>
static int dequant16p_t(const void* w, int64_t rows, int64_t cols, void* out, int* status, cudaStream_t s) {
  static int grid_cap = 0;
  auto k = kt_dequant16p_kernel<TYPE, DT>;
  if (!grid_cap) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, DqRun<TYPE>::SMEM) != cudaSuccess) return -3;
    int dev = 0, sms = 148, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 256, DqRun<TYPE>::SMEM) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    grid_cap = sms * per_sm;
  }
  const int64_t n = rows * (cols / 32);
  const int64_t items = (n + 255) / 256;
  const unsigned grid = (unsigned)(items < grid_cap ? items : grid_cap);
  k<<<grid, 256, DqRun<TYPE>::SMEM, s>>>((const uint8_t*)w, n, out, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int TYPE>
static int dequant_t(const void* w, int64_t rows, int64_t cols, void* out, int dt, cudaStream_t s) {
  const KtBlockInfo bi = kt_block_info(TYPE);
  const int64_t rb = cols / bi.qk * bi.bytes;
  const int64_t n = rows * (cols / 32);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (n == 0) return 0;
  if ((dt == KT_DT_BF16 || dt == KT_DT_F16) && ((((uintptr_t)out) | ((uintptr_t)w)) & 15) == 0) {
    if (dt == KT_DT_BF16)
      kt_dequant16_kernel<TYPE, KT_DT_BF16><<<blocks, 256, 0, s>>>((const uint8_t*)w, rows, cols, out);
    else
      kt_dequant16_kernel<TYPE, KT_DT_F16><<<blocks, 256, 0, s>>>((const uint8_t*)w, rows, cols, out);
    return 0;
  }
  switch (dt) {
    case KT_DT_F32: kt_dequant_kernel<TYPE, KT_DT_F32><<<blocks, 256, 0, s>>>((const uint8_t*)w, rows, cols, rb, out); break;
    case KT_DT_F16: kt_dequant_kernel<TYPE, KT_DT_F16><<<blocks, 256, 0, s>>>((const uint8_t*)w, rows, cols, rb, out); break;
    case KT_DT_BF16: kt_dequant_kernel<TYPE, KT_DT_BF16><<<blocks, 256, 0, s>>>((const uint8_t*)w, rows, cols, rb, out); break;
    default: return -1;
  }
  return 0;
}

int kt_launch_dequant(int type, const void* w, int64_t rows, int64_t cols, void* out, int out_dtype, cudaStream_t s,
                      int* status) {
  const KtBlockInfo bi = kt_block_info(type);
  if (!bi.qk || cols % bi.qk) return -1;
  // large bf16 passes of the prefill types (the prefill layer's weight passes): the pipelined
  // kernel, from four items per SM on; KT_B200_DQ_PIPE=0 keeps the one-shot kernel
  static const bool pipe = [] {
    const char* e = getenv("KT_B200_DQ_PIPE");
    return !(e && e[0] == '0');
  }();
  if (pipe && out_dtype == KT_DT_BF16 && ((((uintptr_t)out) | ((uintptr_t)w)) & 15) == 0 &&
      rows * (cols / 32) >= (int64_t)4 * 148 * 256) {
    switch (type) {
      case KT_Q8_0: return dequant16p_t<KT_Q8_0, KT_DT_BF16>(w, rows, cols, out, status, s);
      case KT_Q4_K: return dequant16p_t<KT_Q4_K, KT_DT_BF16>(w, rows, cols, out, status, s);
      case KT_Q6_K: return dequant16p_t<KT_Q6_K, KT_DT_BF16>(w, rows, cols, out, status, s);
      case KT_IQ3_S: return dequant16p_t<KT_IQ3_S, KT_DT_BF16>(w, rows, cols, out, status, s);
    }
  }
  switch (type) {
    case KT_Q8_0: return dequant_t<KT_Q8_0>(w, rows, cols, out, out_dtype, s);
    case KT_Q4_0: return dequant_t<KT_Q4_0>(w, rows, cols, out, out_dtype, s);
    case KT_Q4_1: return dequant_t<KT_Q4_1>(w, rows, cols, out, out_dtype, s);
    case KT_Q5_0: return dequant_t<KT_Q5_0>(w, rows, cols, out, out_dtype, s);
    case KT_Q5_1: return dequant_t<KT_Q5_1>(w, rows, cols, out, out_dtype, s);
    case KT_IQ4_NL: return dequant_t<KT_IQ4_NL>(w, rows, cols, out, out_dtype, s);
    case KT_Q2_K: return dequant_t<KT_Q2_K>(w, rows, cols, out, out_dtype, s);
    case KT_Q3_K: return dequant_t<KT_Q3_K>(w, rows, cols, out, out_dtype, s);
    case KT_Q5_K: return dequant_t<KT_Q5_K>(w, rows, cols, out, out_dtype, s);
    case KT_IQ4_XS: return dequant_t<KT_IQ4_XS>(w, rows, cols, out, out_dtype, s);
    case KT_Q2_0: return dequant_t<KT_Q2_0>(w, rows, cols, out, out_dtype, s);
    case KT_IQ2_XXS: return dequant_t<KT_IQ2_XXS>(w, rows, cols, out, out_dtype, s);
    case KT_IQ2_XS: return dequant_t<KT_IQ2_XS>(w, rows, cols, out, out_dtype, s);
    case KT_IQ2_S: return dequant_t<KT_IQ2_S>(w, rows, cols, out, out_dtype, s);
    case KT_IQ3_XXS: return dequant_t<KT_IQ3_XXS>(w, rows, cols, out, out_dtype, s);
    case KT_IQ1_S: return dequant_t<KT_IQ1_S>(w, rows, cols, out, out_dtype, s);
    case KT_IQ1_M: return dequant_t<KT_IQ1_M>(w, rows, cols, out, out_dtype, s);
    case KT_Q4_K: return dequant_t<KT_Q4_K>(w, rows, cols, out, out_dtype, s);
    case KT_Q6_K: return dequant_t<KT_Q6_K>(w, rows, cols, out, out_dtype, s);
    case KT_IQ3_S: return dequant_t<KT_IQ3_S>(w, rows, cols, out, out_dtype, s);
  }
  return -1;
}

// ------------------------------------------------------------------ silu_and_mul

template <int DT>
__global__ void kt_silu_and_mul_kernel(const void* __restrict__ h13, int64_t rows, int64_t n, void* __restrict__ h) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * n) return;
  const int64_t r = i / n, j = i % n;
  const float g = kt_load_act<DT>(h13, r * 2 * n + j);
  const float u = kt_load_act<DT>(h13, r * 2 * n + n + j);
  kt_store_act<DT>(h, i, g / (1.0f + expf(-g)) * u);
}

int kt_launch_silu_and_mul(const void* h13, int dtype, int64_t rows, int64_t n, void* h, cudaStream_t s) {
  const int64_t tot = rows * n;
  if (tot == 0) return 0;
  const unsigned blocks = (unsigned)((tot + 255) / 256);
  switch (dtype) {
    case KT_DT_F32: kt_silu_and_mul_kernel<KT_DT_F32><<<blocks, 256, 0, s>>>(h13, rows, n, h); break;
    case KT_DT_F16: kt_silu_and_mul_kernel<KT_DT_F16><<<blocks, 256, 0, s>>>(h13, rows, n, h); break;
    case KT_DT_BF16: kt_silu_and_mul_kernel<KT_DT_BF16><<<blocks, 256, 0, s>>>(h13, rows, n, h); break;
    default: return -1;
  }
  return 0;
}

// ------------------------------------------------------------------ combine

template <int DT>
__device__ __forceinline__ float kt_round_dt(float v) {
  if constexpr (DT == KT_DT_F32) return v;
  if constexpr (DT == KT_DT_F16) return __half2float(__float2half_rn(v));
  return __bfloat162float(__float2bfloat16_rn(v));
}

// out [T, top_k, K] in DT; the route weight is cast to DT first (out.mul_(w.to(out.dtype)))
template <int DT>
__global__ void kt_combine_kernel(const void* __restrict__ out, const float* __restrict__ w, int64_t T, int top_k,
                                  int64_t K, void* __restrict__ res) {
  const int64_t t = blockIdx.x;
  for (int64_t c = threadIdx.x; c < K; c += blockDim.x) {
    float acc = 0.0f;
    for (int k = 0; k < top_k; ++k) {
      const float o = kt_load_act<DT>(out, (t * top_k + k) * K + c);
      const float wk = kt_round_dt<DT>(w[t * top_k + k]);
      acc += kt_round_dt<DT>(o * wk);
    }
    kt_store_act<DT>(res, t * K + c, acc);
  }
}

int kt_launch_combine(const void* out, int dtype, const float* w, int64_t T, int64_t top_k, int64_t K, void* res,
                      cudaStream_t s) {
  if (T == 0 || K == 0) return 0;
  if (T > 0x7fffffff) return -1;
  const unsigned grid = (unsigned)T;
  switch (dtype) {
    case KT_DT_F32: kt_combine_kernel<KT_DT_F32><<<grid, 256, 0, s>>>(out, w, T, (int)top_k, K, res); break;
    case KT_DT_F16: kt_combine_kernel<KT_DT_F16><<<grid, 256, 0, s>>>(out, w, T, (int)top_k, K, res); break;
    case KT_DT_BF16: kt_combine_kernel<KT_DT_BF16><<<grid, 256, 0, s>>>(out, w, T, (int)top_k, K, res); break;
    default: return -1;
  }
  return 0;
}

// The prefill finalize: route (t, k) lives at sorted row route_pos[t*top_k+k] of y [R, K] bf16,
// or is absent (-1: not on this device, contributes nothing). res[t] = bf16(sum_k w * y) with
// the fp32 router weight and fp32 accumulation in k order, rounded once (the finalize of the
// CUTLASS fused MoE that the reference's streamed prefill runs; the decode combine above keeps
// the hot method's per-route bf16 roundings). Each thread produces 8 consecutive columns.
// LOAD: the sum starts from acc[t] (fp32) instead of 0; STORE: the fp32 sum goes back to acc
// instead of bf16 into res. With both, a token none of whose routes is present keeps its acc
// untouched and is skipped (the expert-group loop of a streamed prefill).
template <int KMAX, bool LOAD, bool STORE>
__global__ void kt_combine_sorted_kernel(const uint16_t* __restrict__ y, const int32_t* __restrict__ route_pos,
                                         const float* __restrict__ w, int64_t T, int top_k, int64_t K,
                                         uint16_t* __restrict__ res, float* __restrict__ acc_f32,
                                         const int32_t* __restrict__ tokens_dev) {
  kt_pdl_wait();  // Y (the down kernel's output) is complete
  const int64_t t = blockIdx.x;
  if (tokens_dev && t >= *tokens_dev) return;  // past the tokens present in this call
  // the token's routes: positions and weights (KMAX >= top_k), then all row loads in flight
  int32_t pos[KMAX];
  float wk[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    pos[k] = k < top_k ? route_pos[t * top_k + k] : -1;
    wk[k] = k < top_k ? w[t * top_k + k] : 0.0f;
  }
  if constexpr (LOAD && STORE) {
    bool any = false;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) any |= pos[k] >= 0;
    if (!any) return;
  }
  for (int64_t c = (int64_t)threadIdx.x * 8; c < K; c += (int64_t)blockDim.x * 8) {
    uint4 v[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      v[k] = pos[k] >= 0 ? __ldcs(reinterpret_cast<const uint4*>(y + (int64_t)pos[k] * K + c)) : make_uint4(0, 0, 0, 0);
    float acc[8];
    if constexpr (LOAD) {
      const float4 a0 = *reinterpret_cast<const float4*>(acc_f32 + t * K + c);
      const float4 a1 = *reinterpret_cast<const float4*>(acc_f32 + t * K + c + 4);
      acc[0] = a0.x, acc[1] = a0.y, acc[2] = a0.z, acc[3] = a0.w;
      acc[4] = a1.x, acc[5] = a1.y, acc[6] = a1.z, acc[7] = a1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    }
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (pos[k] < 0) continue;  // bf16(0 * w) adds an exact zero
      const uint32_t u[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += kt_bf2f((uint16_t)(u[j] & 0xffff)) * wk[k];
        acc[2 * j + 1] += kt_bf2f((uint16_t)(u[j] >> 16)) * wk[k];
      }
    }
    if constexpr (STORE) {
      *reinterpret_cast<float4*>(acc_f32 + t * K + c) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(acc_f32 + t * K + c + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint4 o;
      o.x = kt_pack_bf2(acc[0], acc[1]);
      o.y = kt_pack_bf2(acc[2], acc[3]);
      o.z = kt_pack_bf2(acc[4], acc[5]);
      o.w = kt_pack_bf2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(res + t * K + c) = o;
    }
  }
}

template <bool LOAD, bool STORE>
static void launch_combine_sorted_mode(const uint16_t* y, const int32_t* route_pos, const float* w, int64_t T, int k,
                                       int64_t K, uint16_t* res, float* acc, int threads, cudaStream_t s,
                                       const int32_t* td) {
  const unsigned g = (unsigned)T;
  if (k <= 4)
    kt_launch_pdl(kt_combine_sorted_kernel<4, LOAD, STORE>, g, threads, 0, s, y, route_pos, w, T, k, K, res, acc, td);
  else if (k <= 8)
    kt_launch_pdl(kt_combine_sorted_kernel<8, LOAD, STORE>, g, threads, 0, s, y, route_pos, w, T, k, K, res, acc, td);
  else if (k <= 16)
    kt_launch_pdl(kt_combine_sorted_kernel<16, LOAD, STORE>, g, threads, 0, s, y, route_pos, w, T, k, K, res, acc, td);
  else
    kt_launch_pdl(kt_combine_sorted_kernel<32, LOAD, STORE>, g, threads, 0, s, y, route_pos, w, T, k, K, res, acc, td);
}

int kt_launch_combine_sorted(const uint16_t* y, const int32_t* route_pos, const float* w, int64_t T, int64_t top_k,
                             int64_t K, uint16_t* res, cudaStream_t s, float* acc, int acc_flags,
                             const int32_t* tokens_dev) {
  if (T == 0) return 0;
  if (K % 8 || T > 0x7fffffff || top_k > 32) return -1;
  const bool load = acc_flags & 1, store = acc_flags & 2;
  if ((load || store) && (!acc || ((uintptr_t)acc & 15))) return -1;
  const int64_t vec = K / 8;
  const int threads = (int)(vec < 256 ? (vec + 31) / 32 * 32 : 256);
  const int k = (int)top_k;
  if (load && store)
    launch_combine_sorted_mode<true, true>(y, route_pos, w, T, k, K, res, acc, threads, s, tokens_dev);
  else if (load)
    launch_combine_sorted_mode<true, false>(y, route_pos, w, T, k, K, res, acc, threads, s, tokens_dev);
  else if (store)
    launch_combine_sorted_mode<false, true>(y, route_pos, w, T, k, K, res, acc, threads, s, tokens_dev);
  else
    launch_combine_sorted_mode<false, false>(y, route_pos, w, T, k, K, res, acc, threads, s, tokens_dev);
  return 0;
}

bool kt_pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("KT_B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// ------------------------------------------------------------------ row gathers

// one warp per row, 16 bytes per lane per step
__global__ void kt_gather_rows_kernel(const uint16_t* __restrict__ src, int64_t cols, const int32_t* __restrict__ idx,
                                      int64_t n, const int32_t* __restrict__ n_limit, uint16_t* __restrict__ dst) {
  const int64_t lim = n_limit ? (int64_t)*n_limit : n;
  const int64_t end = lim < n ? lim : n;
  const int lane = threadIdx.x & 31;
  const int64_t vec = cols / 8;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; i < end;
       i += (int64_t)gridDim.x * blockDim.x / 32) {
    const int32_t j = idx[i];
    uint4* d = reinterpret_cast<uint4*>(dst + i * cols);
    if (j < 0) {
      for (int64_t c = lane; c < vec; c += 32) d[c] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* sr = reinterpret_cast<const uint4*>(src + (int64_t)j * cols);
      for (int64_t c = lane; c < vec; c += 32) d[c] = sr[c];
    }
  }
}

int kt_launch_gather_rows(const uint16_t* src, int64_t cols, const int32_t* idx, int64_t n, const int32_t* n_limit,
                          uint16_t* dst, cudaStream_t s) {
  if (n == 0) return 0;
  if (cols % 8 || (((uintptr_t)src | (uintptr_t)dst) & 15)) return -1;
  const int64_t warps = n < 148 * 64 ? n : 148 * 64;
  kt_gather_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(src, cols, idx, n, n_limit, dst);
  return 0;
}

// ------------------------------------------------------------------ route (HotCache.route)

__global__ void kt_route_kernel(const int32_t* __restrict__ ids, int64_t n, const int32_t* __restrict__ slot_tab,
                                const int32_t* __restrict__ cpu_tab, float* __restrict__ counts,
                                int32_t* __restrict__ slot_out, int32_t* __restrict__ cpu_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t e = ids[i];
  slot_out[i] = slot_tab[e];
  cpu_out[i] = cpu_tab[e];
  if (counts) atomicAdd(&counts[e], 1.0f);
}

int kt_launch_route(const int32_t* ids, int64_t n, const int32_t* slot_tab, const int32_t* cpu_tab, float* counts,
                    int32_t* slot_out, int32_t* cpu_out, cudaStream_t s) {
  if (n == 0) return 0;
  kt_route_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ids, n, slot_tab, cpu_tab, counts, slot_out, cpu_out);
  return 0;
}

// ------------------------------------------------------------------ router top-k
// One warp per token. Selection takes the largest score; ties go to the lower expert id.

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, m);
    const int oi = __shfl_xor_sync(0xffffffffu, i, m);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

constexpr int kMaxExpertsPerLane = 32;  // E <= 1024

__global__ void kt_topk_softmax_kernel(const float* __restrict__ logits, int64_t T, int E, int k, int renorm,
                                       float* __restrict__ weights, int32_t* __restrict__ ids) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float v[kMaxExpertsPerLane];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMaxExpertsPerLane; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? logits[t * E + e] : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxExpertsPerLane; ++j) {
    v[j] = (lane + 32 * j) < E ? expf(v[j] - mx) : -1.0f;
    sum += v[j] > 0.0f ? v[j] : 0.0f;
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
  float picked = 0.0f, mine_w = 0.0f;
  int mine_i = -1;
  for (int r = 0; r < k; ++r) {
    float bv = -1.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j)
      if (v[j] > bv) {
        bv = v[j];
        bi = lane + 32 * j;
      }
    warp_argmax(bv, bi);
    const float p = bv / sum;
    picked += p;
    if (lane == r) {
      mine_w = p;
      mine_i = bi;
    }
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j)
      if (lane + 32 * j == bi) v[j] = -2.0f;
  }
  if (lane < k) {
    weights[t * k + lane] = renorm ? mine_w / picked : mine_w;
    ids[t * k + lane] = mine_i;
  }
}

int kt_launch_topk_softmax(const float* logits, int64_t T, int E, int k, int renorm, float* weights, int32_t* ids,
                           cudaStream_t s) {
  if (E > 32 * kMaxExpertsPerLane || k > 32 || k > E) return -1;
  if (T == 0) return 0;
  kt_topk_softmax_kernel<<<(unsigned)((T + 7) / 8), 256, 0, s>>>(logits, T, E, k, renorm, weights, ids);
  return 0;
}

// DeepSeek-V3 routing: s = sigmoid(logit); selection score s + bias; group score = sum of the
// two best selection scores in the group; keep topk_group groups; top-k experts among them by
// selection score; weight = s (unbiased), renormalised over the k and multiplied by scale.
__global__ void kt_topk_grouped_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int64_t T, int E,
                                       int n_group, int topk_group, int k, int renorm, float scale,
                                       float* __restrict__ weights, int32_t* __restrict__ ids) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  const int gsize = E / n_group;
  float sc[kMaxExpertsPerLane], sel[kMaxExpertsPerLane];
#pragma unroll
  for (int j = 0; j < kMaxExpertsPerLane; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      sc[j] = 1.0f / (1.0f + expf(-logits[t * E + e]));
      sel[j] = sc[j] + (bias ? bias[e] : 0.0f);
    } else {
      sc[j] = 0.0f;
      sel[j] = -INFINITY;
    }
  }
  // group scores: top-2 selection scores of each group, summed (lane g computes group g)
  __shared__ float gs_all[8][64];
  float* gs = gs_all[threadIdx.x / 32];
  for (int g = 0; g < n_group; ++g) {
    float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < E && e / gsize == g) {
        const float x = sel[j];
        if (x > b1) {
          b2 = b1;
          b1 = x;
        } else if (x > b2) {
          b2 = x;
        }
      }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, b1, m), o2 = __shfl_xor_sync(0xffffffffu, b2, m);
      const float n1 = fmaxf(b1, o1);
      const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
      b1 = n1;
      b2 = n2;
    }
    if (lane == 0) gs[g] = b1 + b2;
  }
  __syncwarp();
  // keep the topk_group best groups
  uint64_t keep = 0;
  for (int r = 0; r < topk_group; ++r) {
    float bv = -INFINITY;
    int bg = 0;
    for (int g = 0; g < n_group; ++g)
      if (!((keep >> g) & 1) && gs[g] > bv) {
        bv = gs[g];
        bg = g;
      }
    keep |= 1ull << bg;
  }
#pragma unroll
  for (int j = 0; j < kMaxExpertsPerLane; ++j) {
    const int e = lane + 32 * j;
    if (e < E && !((keep >> (e / gsize)) & 1)) sel[j] = -INFINITY;
  }
  float picked = 0.0f, mine_w = 0.0f;
  int mine_i = -1;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    float bs = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j)
      if (sel[j] > bv) {
        bv = sel[j];
        bi = lane + 32 * j;
        bs = sc[j];
      }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      const float os = __shfl_xor_sync(0xffffffffu, bs, m);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bs = os;
      }
    }
    picked += bs;
    if (lane == r) {
      mine_w = bs;
      mine_i = bi;
    }
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; ++j)
      if (lane + 32 * j == bi) sel[j] = -INFINITY;
  }
  if (lane < k) {
    weights[t * k + lane] = (renorm ? mine_w / picked : mine_w) * scale;
    ids[t * k + lane] = mine_i;
  }
}

int kt_launch_topk_grouped(const float* logits, const float* bias, int64_t T, int E, int n_group, int topk_group, int k,
                           int renorm, float scale, float* weights, int32_t* ids, cudaStream_t s) {
  if (E > 32 * kMaxExpertsPerLane || k > 32 || n_group > 64 || n_group <= 0 || E % n_group || topk_group > n_group ||
      k > (E / n_group) * topk_group)
    return -1;
  if (T == 0) return 0;
  kt_topk_grouped_kernel<<<(unsigned)((T + 7) / 8), 256, 0, s>>>(logits, bias, T, E, n_group, topk_group, k, renorm,
                                                                scale, weights, ids);
  return 0;
}

// ------------------------------------------------------------------ permute for the prefill GEMM
// Three kernels, no global atomics:
//   hist     one block per kPermBlock routes: shared-memory histogram over slots with
//            warp-aggregated atomics; each route keeps its rank among the block's routes of
//            its slot (in route_pos, temporarily); the block's histogram goes to hist[b][*]
//   scan     one block: per slot, exclusive prefix over blocks (hist becomes each block's
//            first position per slot) plus the slot's base (exclusive prefix over slots);
//            counts[] and the token tiles (<= tile_tokens rows each, in slot order)
//   scatter  position = hist[b][slot] + rank: sorted_token[pos], route_pos[route]
constexpr int kPermBlock = 1024;

// routes at or past `lim` (the present routes, when a device token count limits them) are absent
__device__ __forceinline__ int64_t kt_perm_limit(int64_t routes, int top_k, const int32_t* tokens_dev) {
  if (!tokens_dev) return routes;
  const int64_t n = (int64_t)(*tokens_dev) * top_k;
  return n < routes ? (n > 0 ? n : 0) : routes;
}

__global__ void __launch_bounds__(kPermBlock) kt_perm_hist_kernel(const int32_t* __restrict__ ids, int64_t routes,
                                                                  int top_k, int n_slots, int id_base,
                                                                  const int32_t* __restrict__ tokens_dev,
                                                                  int32_t* __restrict__ hist,
                                                                  int32_t* __restrict__ rank) {
  extern __shared__ int32_t sh[];
  kt_pdl_trigger();  // the scan may launch; it waits for this grid before reading hist
  for (int e = threadIdx.x; e < n_slots; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int64_t lim = kt_perm_limit(routes, top_k, tokens_dev);
  const int64_t p = (int64_t)blockIdx.x * kPermBlock + threadIdx.x;
  const int32_t e0 = p < lim ? ids[p] : -1;
  const int32_t e = e0 >= id_base ? e0 - id_base : -1;  // slot of the id window [id_base, id_base + n_slots)
  const bool valid = e >= 0 && e < n_slots;
  const int lane = threadIdx.x & 31;
  const uint32_t peers = __match_any_sync(0xffffffffu, valid ? e : -1);
  const int leader = __ffs(peers) - 1;
  int base = 0;
  if (valid && lane == leader) base = atomicAdd(&sh[e], __popc(peers));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (p < routes) rank[p] = valid ? base + __popc(peers & ((1u << lane) - 1)) : -1;
  __syncthreads();
  for (int e2 = threadIdx.x; e2 < n_slots; e2 += blockDim.x) hist[(int64_t)blockIdx.x * n_slots + e2] = sh[e2];
}

// exclusive scan of v over the block (1024 threads); returns the total in *total
__device__ __forceinline__ int32_t kt_block_exclusive_scan(int32_t v, int32_t* warp_sums, int32_t* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int32_t w = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  const int32_t excl = x - v + (wid > 0 ? warp_sums[wid - 1] : 0);
  *total = warp_sums[(blockDim.x >> 5) - 1];
  __syncthreads();
  return excl;
}

// Up to 1024 slots: G threads per slot (G the largest power of two <= 32 with G * n_slots <=
// 1024), thread (slot e, run j) owning the blocks [j * ceil(nb / G), ...): its loads of one block
// row are coalesced with the other slots' threads, eight independent loads in flight, and the
// per-slot prefix over the G runs is taken in shared memory. More slots: warp w handles slots
// w, w + 32, ...; lanes walk the blocks. Both give hist[b][e] = base(e) + the routes of slot e
// in the blocks before b.
__device__ __forceinline__ int kt_scan_threads_per_slot(int n_slots) {
  if (n_slots > kPermBlock) return 0;
  int g = 32;
  while (g > 1 && g * n_slots > kPermBlock) g >>= 1;
  return g;
}
__global__ void __launch_bounds__(kPermBlock) kt_perm_scan_kernel(int32_t* __restrict__ hist, int n_blocks, int n_slots,
                                                                  int tile_tokens, int chunk_tiles,
                                                                  int32_t* __restrict__ counts,
                                                                  int32_t* __restrict__ tiles,
                                                                  int32_t* __restrict__ n_tiles,
                                                                  int32_t* __restrict__ chunks) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t sbase[kPermMaxSlots];
  __shared__ int32_t part[kPermBlock];  // [run j][slot e]: routes of the run, then its exclusive prefix
  kt_pdl_trigger();
  kt_pdl_wait();  // the block histograms are complete
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int G = kt_scan_threads_per_slot(n_slots);
  const int nbp = G ? (n_blocks + G - 1) / G : 0;  // blocks per run
  const int my_e = G ? (int)threadIdx.x % n_slots : 0, my_j = G ? (int)threadIdx.x / n_slots : 0;
  const bool runs = G && (int)threadIdx.x < G * n_slots;
  const int rb0 = my_j * nbp, rb1 = min(n_blocks, rb0 + nbp);
  constexpr int U = 8;
  // 1. per-slot totals
  if (G) {
    if (runs) {
      int32_t v = 0;
      for (int b = rb0; b < rb1; b += U) {
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (b + u < rb1) v += hist[(int64_t)(b + u) * n_slots + my_e];
      }
      part[my_j * n_slots + my_e] = v;
    }
    __syncthreads();
    if ((int)threadIdx.x < n_slots) {
      int32_t acc = 0;
      for (int j = 0; j < G; ++j) {
        const int32_t v = part[j * n_slots + threadIdx.x];
        part[j * n_slots + threadIdx.x] = acc;
        acc += v;
      }
      counts[threadIdx.x] = acc;
    }
  } else {
    for (int e = wid; e < n_slots; e += nw) {
      int32_t v = 0;
      for (int b = lane; b < n_blocks; b += 32) v += hist[(int64_t)b * n_slots + e];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) counts[e] = v;
    }
  }
  __syncthreads();
  // 2. slot bases and tile offsets: exclusive scans over the slots (thread t owns [e0, e1))
  const int per = (n_slots + blockDim.x - 1) / blockDim.x;
  const int e0 = min(n_slots, (int)threadIdx.x * per), e1 = min(n_slots, e0 + per);
  int32_t my_routes = 0, my_tiles = 0, my_chunks = 0;
  for (int e = e0; e < e1; ++e) {
    const int32_t nt = (counts[e] + tile_tokens - 1) / tile_tokens;
    my_routes += counts[e];
    my_tiles += nt;
    my_chunks += (nt + chunk_tiles - 1) / chunk_tiles;
  }
  int32_t total_routes, total_tiles, total_chunks;
  int32_t off = kt_block_exclusive_scan(my_routes, warp_sums, &total_routes);
  int32_t t = kt_block_exclusive_scan(my_tiles, warp_sums, &total_tiles);
  int32_t ch = kt_block_exclusive_scan(my_chunks, warp_sums, &total_chunks);
  for (int e = e0; e < e1; ++e) {
    const int32_t c = counts[e];
    const int32_t nt = (c + tile_tokens - 1) / tile_tokens;
    for (int32_t k = 0; k < nt; k += chunk_tiles, ++ch) {
      chunks[3 * ch + 0] = e;
      chunks[3 * ch + 1] = off + k * tile_tokens;
      chunks[3 * ch + 2] = min(chunk_tiles * tile_tokens, c - k * tile_tokens);
    }
    for (int32_t r = 0; r < c; r += tile_tokens, ++t) {
      tiles[3 * t + 0] = e;
      tiles[3 * t + 1] = off + r;
      tiles[3 * t + 2] = min(tile_tokens, c - r);
    }
    sbase[e] = off;
    off += c;
  }
  __syncthreads();
  // 3. hist[b][e] <- base(e) + routes of slot e in the blocks before b
  if (runs) {
    int32_t carry = sbase[my_e] + part[my_j * n_slots + my_e];
    for (int b = rb0; b < rb1; b += U) {
      int32_t v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = b + u < rb1 ? hist[(int64_t)(b + u) * n_slots + my_e] : 0;
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (b + u < rb1) {
          hist[(int64_t)(b + u) * n_slots + my_e] = carry;
          carry += v[u];
        }
    }
  }
  for (int e = wid; !G && e < n_slots; e += nw) {
    int32_t carry = sbase[e];
    for (int b0 = 0; b0 < n_blocks; b0 += 32) {
      const int b = b0 + lane;
      const int32_t v = b < n_blocks ? hist[(int64_t)b * n_slots + e] : 0;
      int32_t x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (b < n_blocks) hist[(int64_t)b * n_slots + e] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
  if (threadIdx.x == 0) {
    n_tiles[0] = total_tiles;
    n_tiles[1] = total_routes;
    n_tiles[2] = total_chunks;
  }
}

__global__ void __launch_bounds__(kPermBlock) kt_perm_scatter_kernel(const int32_t* __restrict__ ids, int64_t routes,
                                                                     int top_k, int n_slots, int id_base,
                                                                     const int32_t* __restrict__ tokens_dev,
                                                                     const int32_t* __restrict__ hist,
                                                                     int32_t* __restrict__ sorted_token,
                                                                     int32_t* __restrict__ route_pos) {
  kt_pdl_trigger();
  kt_pdl_wait();  // the scan's bases are complete
  const int64_t p = (int64_t)blockIdx.x * kPermBlock + threadIdx.x;
  if (p >= routes) return;
  const int64_t lim = kt_perm_limit(routes, top_k, tokens_dev);
  const int32_t e = p < lim && ids[p] >= id_base ? ids[p] - id_base : -1;
  if (e >= 0 && e < n_slots) {
    const int32_t pos = hist[(int64_t)blockIdx.x * n_slots + e] + route_pos[p];
    sorted_token[pos] = (int32_t)(p / top_k);
    route_pos[p] = pos;
  } else {
    route_pos[p] = -1;
  }
}

int64_t kt_permute_hist_ints(int64_t routes, int n_slots) { return ((routes + kPermBlock - 1) / kPermBlock) * n_slots; }

int kt_launch_permute(const int32_t* ids, int64_t routes, int top_k, int n_slots, int tile_tokens, int chunk_tiles,
                      int32_t* counts, int32_t* hist, int32_t* tiles, int32_t* n_tiles, int32_t* chunks,
                      int32_t* sorted_token, int32_t* route_pos, cudaStream_t s, int id_base,
                      const int32_t* tokens_dev) {
  if (n_slots <= 0 || n_slots > kPermMaxSlots || chunk_tiles <= 0 || id_base < 0) return -1;
  const int nb = (int)((routes + kPermBlock - 1) / kPermBlock);
  if (nb > 0)
    kt_perm_hist_kernel<<<nb, kPermBlock, n_slots * sizeof(int32_t), s>>>(ids, routes, top_k, n_slots, id_base,
                                                                          tokens_dev, hist, route_pos);
  if (kt_launch_pdl(kt_perm_scan_kernel, 1, kPermBlock, 0, s, (int32_t*)hist, nb, n_slots, tile_tokens, chunk_tiles,
                    counts, tiles, n_tiles, chunks))
    return -4;
  if (nb > 0 && kt_launch_pdl(kt_perm_scatter_kernel, nb, kPermBlock, 0, s, ids, routes, top_k, n_slots, id_base,
                              tokens_dev, (const int32_t*)hist, sorted_token, route_pos))
    return -4;
  return 0;
}
