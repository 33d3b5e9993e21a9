// moe_gemm.cu — prefill path: persistent, warp-specialised tcgen05 grouped GEMM over the
// hot experts with in-kernel GGUF dequantization.
//
// Replaces the reference's streamed-prefill pair "dequant experts to bf16 in HBM (Triton),
// then FlashInfer's bf16 CUTLASS fused MoE" (trees/flash-next-gguf patch, kt_stream_prefill_gguf
// _group_body; kt_gguf_dequant.py) and, at prefill sizes, the per-route GEMV build of
// kt_moe_a8_vec_multi (hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu:653). Weights stay in their
// GGUF bytes in HBM; each tile's raw super-blocks are copied into shared memory by the bulk
// copy engine and dequantized there to bf16, so HBM sees 4.5-6.6 bits per weight instead of a
// bf16 round trip.
//
// Problem, per expert slot e with M_e routed tokens (sorted by slot):
//   phase 1: H[M_e, N]  = silu(X_e W_gate^T) * (X_e W_up^T)    (W13 rows [gate; up], K = hidden)
//   phase 2: Y[M_e, K]  = H W_down^T                             (W2 [K, N])
// Swap-AB: the MMA's M dimension is weight rows (two 128-row halves per tile, sharing the
// token operand), its N dimension is tokens (up to 256 per tile), reduction along K.
//
// Warp roles (480 threads):
//   warps 0-7   dequant producers: thread r owns A row r of the tile; per 64-wide k-step it
//               decodes 64 values from the raw stage and writes them as bf16 into the A stage
//               in the UMMA K-major 128-byte swizzle layout
//   warp 8      raw loader: per 256-value super-block column, one 1-D bulk copy per row of the
//               16-byte aligned span holding that row's block (cp.async.bulk, no multicast)
//   warp 9      B loader: phase 1 gathers token rows of X with TMA tile::gather4 (4 rows per
//               instruction); phase 2 loads H rows with a 2-D TMA tile (rows are contiguous)
//   warp 10     MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> fp32 in TMEM), commits
//   warps 11-14 epilogue: tcgen05.ld of the accumulators; phase 1 applies SwiGLU and writes H
//               (bf16), phase 2 writes Y (bf16); both transposed through shared memory
// TMEM: 512 columns = two fp32 accumulators of up to 256 columns (gate/up, or the two
// 128-row halves of the down tile).
#include "gguf_dot.cuh"
#include "kt_kernels.h"

namespace {

constexpr int kProducers = 256;
constexpr int kThreads = 480;
constexpr int kWarpRaw = 8, kWarpB = 9, kWarpMma = 10, kWarpEpi0 = 11;
constexpr int kTN = 256;           // tokens per tile (MMA N), at most
constexpr int kStages = 2;         // A/B stages
constexpr int kAStageBytes = 256 * 128;
constexpr int kBStageBytes = kTN * 128;
constexpr int kFixedSmem = 2 * kStages * 128 * 256 /* A and B */ + 4 * 32 * 32 * 2 /* epilogue transpose */ +
                           2048 /* grid */ + 512 /* barriers */ + 1024 /* alignment slack */;

// Raw staging: a "unit" is UV consecutive values of one weight row (a 256-value super-block,
// or four 32-value Q8_0 blocks); a raw stage holds one unit for one half (128 rows) of the
// tile. Each row's slot holds the 16-byte aligned span around its unit (bulk copies need
// 16-byte aligned addresses and sizes; GGUF blocks are only 2-byte aligned).
template <int TYPE>
struct Raw {
  static constexpr int UV = TYPE == KT_Q8_0 ? 128 : 256;
  static constexpr int UNIT_BYTES = TYPE == KT_Q8_0 ? 4 * 34 : kt_block_info(TYPE).bytes;
  static constexpr int SLOT = (UNIT_BYTES + 14 + 15) / 16 * 16;  // unit starts at an even offset <= 14
  static constexpr int STAGE_BYTES = 128 * SLOT;
  static constexpr int NRAW_FIT = (227 * 1024 - kFixedSmem) / STAGE_BYTES;
  static constexpr int NRAW = NRAW_FIT > 4 ? 4 : NRAW_FIT;  // ring of half-tile stages
  static constexpr int KPU = UV / 64;                        // k-steps per unit
  static_assert(NRAW >= 3, "raw ring too small");
};

struct Smem {
  static constexpr int A = 0;
  static constexpr int B = A + kStages * kAStageBytes;
  static constexpr int RAW = B + kStages * kBStageBytes;
};

template <int TYPE>
constexpr int smem_bytes() {
  return kFixedSmem + Raw<TYPE>::NRAW * Raw<TYPE>::STAGE_BYTES;
}

// 32 values (sub-unit `sub` of 8) of one row's raw unit -> fp32
template <int TYPE>
__device__ __forceinline__ void dq_unit(const uint8_t* unit, int sub, float* y, const uint32_t* grid) {
  if constexpr (TYPE == KT_Q8_0) kt_dq32_q8_0(unit + 34 * sub, y);
  if constexpr (TYPE == KT_Q4_K) kt_dq32_q4_k(unit, sub, y);
  if constexpr (TYPE == KT_Q6_K) kt_dq32_q6_k(unit, sub, y);
  if constexpr (TYPE == KT_IQ3_S) kt_dq32_iq3_s(unit, sub, y, grid);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

}  // namespace

template <int TYPE, int PHASE>
__global__ void __launch_bounds__(kThreads, 1) kt_moe_gemm_kernel(const __grid_constant__ CUtensorMap bmap, const KtGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  using R = Raw<TYPE>;
  uint8_t* sA = smem + Smem::A;
  uint8_t* sB = smem + Smem::B;
  uint8_t* sRaw = smem + Smem::RAW;
  uint16_t* sEpi = reinterpret_cast<uint16_t*>(sRaw + R::NRAW * R::STAGE_BYTES);
  uint32_t* sGrid = reinterpret_cast<uint32_t*>(sEpi + 4 * 32 * 32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGrid + 512);
  uint64_t* full_ab = bars;                      // [kStages]
  uint64_t* empty_ab = bars + kStages;           // [kStages]
  uint64_t* raw_full = bars + 2 * kStages;       // [NRAW]
  uint64_t* raw_empty = raw_full + R::NRAW;      // [NRAW]
  uint64_t* acc_full = raw_empty + R::NRAW;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* done_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      kt_mbar_init(&full_ab[s], kProducers + 1);
      kt_mbar_init(&empty_ab[s], 1);
    }
    for (int s = 0; s < R::NRAW; ++s) {
      kt_mbar_init(&raw_full[s], 1);
      kt_mbar_init(&raw_empty[s], 128);
    }
    kt_mbar_init(acc_full, 1);
    kt_mbar_init(acc_empty, 128);
    kt_mbar_init(done_bar, 1);
    *abort_flag = 0;
    kt_fence_mbar_init();
  }
  if constexpr (TYPE == KT_IQ3_S) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) sGrid[i] = kt_iq3s_grid_dev[i];
  }
  if (warp == kWarpMma) kt_tmem_alloc(tmem_slot, 512);
  kt_tc_fence_before();
  __syncthreads();
  kt_tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int n_tiles = *a.n_tiles;
  const int n_wt = a.n_wtiles;
  const int n_items = n_tiles * n_wt;
  const int ksteps = a.K / 64;
  const int units = a.K / R::UV;

  if (warp < 8) {
    // ---------------------------------------------------------------- dequant producers
    const int r = threadIdx.x;  // A row in the tile
    uint32_t kit = 0, uit = 0;
    for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
      const int tile = item / n_wt, wt = item % n_wt;
      const int slot = a.tiles[3 * tile + 0];
      const int64_t grow = PHASE == 1 ? (r < 128 ? (int64_t)wt * 128 + r : (int64_t)a.N + (int64_t)wt * 128 + (r - 128))
                                      : (int64_t)wt * 256 + r;
      const int64_t rows_total = PHASE == 1 ? 2 * (int64_t)a.N : (int64_t)a.K_out;
      const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                     : a.w + (int64_t)slot * rows_total * a.row_bytes;
      const uint8_t* grow_ptr = wbase + grow * a.row_bytes;
      const int hh = r / 128, rh = r % 128;  // tile half and row within it
      for (int u = 0; u < units && !*abort_flag; ++u, ++uit) {
        const uint32_t hit = 2 * uit + hh;
        const int su = hit % R::NRAW;
        if (!kt_mbar_wait(&raw_full[su], (hit / R::NRAW) & 1, a.status, abort_flag)) break;
        // the loader copied the 16-byte aligned span around this row's unit into the row's
        // slot; the unit starts at the alignment remainder of its global address
        const uintptr_t gaddr = (uintptr_t)(grow_ptr + (int64_t)u * R::UNIT_BYTES);
        const uint8_t* rowp = sRaw + su * R::STAGE_BYTES + rh * R::SLOT + (gaddr & 15);
        for (int kk = 0; kk < R::KPU && !*abort_flag; ++kk, ++kit) {
          const int s = kit % kStages;
          if (!kt_mbar_wait(&empty_ab[s], ((kit / kStages) & 1) ^ 1, a.status, abort_flag)) break;
          uint8_t* arow = sA + s * kAStageBytes;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[32];
            dq_unit<TYPE>(rowp, 2 * kk + h, v, sGrid);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint4 q;
              q.x = kt_pack_bf2(v[8 * c + 0], v[8 * c + 1]);
              q.y = kt_pack_bf2(v[8 * c + 2], v[8 * c + 3]);
              q.z = kt_pack_bf2(v[8 * c + 4], v[8 * c + 5]);
              q.w = kt_pack_bf2(v[8 * c + 6], v[8 * c + 7]);
              *reinterpret_cast<uint4*>(arow + kt_swz128(r, 32 * h + 8 * c)) = q;
            }
          }
          kt_fence_proxy_async_smem();
          kt_mbar_arrive(&full_ab[s]);
        }
        kt_mbar_arrive(&raw_empty[su]);
      }
    }
  } else if (warp == kWarpRaw) {
    // ---------------------------------------------------------------- raw loader
    uint32_t uit = 0;
    for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
      const int tile = item / n_wt, wt = item % n_wt;
      const int slot = a.tiles[3 * tile + 0];
      const int64_t rows_total = PHASE == 1 ? 2 * (int64_t)a.N : (int64_t)a.K_out;
      const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                     : a.w + (int64_t)slot * rows_total * a.row_bytes;
      for (int u = 0; u < units && !*abort_flag; ++u, ++uit) {
        for (int hh = 0; hh < 2 && !*abort_flag; ++hh) {
          const uint32_t hit = 2 * uit + hh;
          const int su = hit % R::NRAW;
          if (!kt_mbar_wait(&raw_empty[su], ((hit / R::NRAW) & 1) ^ 1, a.status, abort_flag)) break;
          uintptr_t src[4];
          uint32_t len[4], total = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = hh * 128 + lane + 32 * i;
            const int64_t grow = PHASE == 1 ? (r < 128 ? (int64_t)wt * 128 + r : (int64_t)a.N + (int64_t)wt * 128 + (r - 128))
                                            : (int64_t)wt * 256 + r;
            const uintptr_t g = (uintptr_t)(wbase + grow * a.row_bytes + (int64_t)u * R::UNIT_BYTES);
            src[i] = g & ~(uintptr_t)15;
            len[i] = (uint32_t)(((g + R::UNIT_BYTES + 15) & ~(uintptr_t)15) - src[i]);
            total += len[i];
          }
#pragma unroll
          for (int m = 16; m > 0; m >>= 1) total += __shfl_xor_sync(0xffffffffu, total, m);
          if (lane == 0) kt_mbar_arrive_expect_tx(&raw_full[su], total);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i)
            kt_bulk_g2s(sRaw + su * R::STAGE_BYTES + (lane + 32 * i) * R::SLOT, reinterpret_cast<const void*>(src[i]),
                        len[i], &raw_full[su]);
        }
      }
    }
  } else if (warp == kWarpB) {
    // ---------------------------------------------------------------- B loader
    uint32_t kit = 0;
    for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
      const int tile = item / n_wt;
      const int pos0 = a.tiles[3 * tile + 1], ntok = a.tiles[3 * tile + 2];
      const int nN = (ntok + 15) & ~15;
      for (int ks = 0; ks < ksteps && !*abort_flag; ++ks, ++kit) {
        const int s = kit % kStages;
        if (!kt_mbar_wait(&empty_ab[s], ((kit / kStages) & 1) ^ 1, a.status, abort_flag)) break;
        uint8_t* dst = sB + s * kBStageBytes;
        if constexpr (PHASE == 1) {
          if (lane == 0) kt_mbar_arrive_expect_tx(&full_ab[s], (uint32_t)nN * 128);
          __syncwarp();
          for (int q = lane; q < nN / 4; q += 32) {
            int rr[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int row = 4 * q + j;
              rr[j] = a.sorted_token[pos0 + (row < ntok ? row : 0)];
            }
            kt_tma_gather4(dst + q * 4 * 128, &bmap, ks * 64, rr[0], rr[1], rr[2], rr[3], &full_ab[s]);
          }
        } else {
          if (lane == 0) {
            kt_mbar_arrive_expect_tx(&full_ab[s], (uint32_t)kBStageBytes);
            kt_tma_2d(dst, &bmap, ks * 64, pos0, &full_ab[s]);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == kWarpMma) {
    // ---------------------------------------------------------------- MMA issuer
    uint32_t kit = 0, ait = 0;
    for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++ait) {
      const int tile = item / n_wt;
      const int ntok = a.tiles[3 * tile + 2];
      const int nN = (ntok + 15) & ~15;
      const uint32_t idesc = kt_idesc_bf16(128, nN);
      if (!kt_mbar_wait(acc_empty, (ait & 1) ^ 1, a.status, abort_flag)) break;
      kt_tc_fence_after();
      for (int ks = 0; ks < ksteps && !*abort_flag; ++ks, ++kit) {
        const int s = kit % kStages;
        if (!kt_mbar_wait(&full_ab[s], (kit / kStages) & 1, a.status, abort_flag)) break;
        kt_tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = kt_smem_addr(sA + s * kAStageBytes);
          const uint32_t b0 = kt_smem_addr(sB + s * kBStageBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t da0 = kt_desc_k128(a0) + 2 * kk;
            const uint64_t da1 = kt_desc_k128(a0 + 128 * 128) + 2 * kk;
            const uint64_t db = kt_desc_k128(b0) + 2 * kk;
            const uint32_t acc = (ks | kk) != 0;
            kt_mma_bf16_ss(tmem + 0, da0, db, idesc, acc);
            kt_mma_bf16_ss(tmem + 256, da1, db, idesc, acc);
          }
          kt_mma_commit(&empty_ab[s]);
        }
        __syncwarp();
      }
      if (lane == 0) kt_mma_commit(acc_full);
      __syncwarp();
    }
    if (lane == 0) {
      kt_mma_commit(done_bar);
      kt_mbar_wait(done_bar, 0, a.status, nullptr);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    uint16_t* stg = sEpi + (warp - kWarpEpi0) * 32 * 32;
    uint32_t ait = 0;
    for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++ait) {
      const int tile = item / n_wt, wt = item % n_wt;
      const int pos0 = a.tiles[3 * tile + 1], ntok = a.tiles[3 * tile + 2];
      if (!kt_mbar_wait(acc_full, ait & 1, a.status, abort_flag)) break;
      kt_tc_fence_after();
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
      for (int c0 = 0; c0 < ntok; c0 += 32) {
        if constexpr (PHASE == 1) {
          uint32_t g[32], u[32];
          kt_tmem_ld32(lane_base + c0, g);
          kt_tmem_ld32(lane_base + 256 + c0, u);
          kt_tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
            stg[j * 32 + lane] = kt_f2bf(silu(gv) * uv);
          }
          __syncwarp();
          const int tok = c0 + lane;
          if (tok < ntok) {
            uint16_t* dst = a.out + (int64_t)(pos0 + tok) * a.out_ld + (int64_t)wt * 128 + 32 * q;
            const uint4* src = reinterpret_cast<const uint4*>(stg + lane * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(dst)[i] = src[i];
          }
          __syncwarp();
        } else {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            uint32_t v[32];
            kt_tmem_ld32(lane_base + 256 * h + c0, v);
            kt_tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = kt_f2bf(__uint_as_float(v[j]));
            __syncwarp();
            const int tok = c0 + lane;
            if (tok < ntok) {
              uint16_t* dst = a.out + (int64_t)(pos0 + tok) * a.out_ld + (int64_t)wt * 256 + 128 * h + 32 * q;
              const uint4* src = reinterpret_cast<const uint4*>(stg + lane * 32);
#pragma unroll
              for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(dst)[i] = src[i];
            }
            __syncwarp();
          }
        }
      }
      kt_tc_fence_before();
      kt_mbar_arrive(acc_empty);
    }
  }

  kt_tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    kt_tc_fence_after();
    kt_tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                    const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_encodeTiled)p;
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box {64 cols, box_rows}, 128B swizzle
static int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <int TYPE, int PHASE>
static int launch_t(const CUtensorMap& m, const KtGemmArgs& a, int grid, cudaStream_t s) {
  constexpr int smem = smem_bytes<TYPE>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  auto k = kt_moe_gemm_kernel<TYPE, PHASE>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -3;
  k<<<grid, kThreads, smem, s>>>(m, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int PHASE>
static int launch_phase(int type, const CUtensorMap& m, const KtGemmArgs& a, int grid, cudaStream_t s) {
  switch (type) {
    case KT_Q8_0: return launch_t<KT_Q8_0, PHASE>(m, a, grid, s);
    case KT_Q4_K: return launch_t<KT_Q4_K, PHASE>(m, a, grid, s);
    case KT_Q6_K: return launch_t<KT_Q6_K, PHASE>(m, a, grid, s);
    case KT_IQ3_S: return launch_t<KT_IQ3_S, PHASE>(m, a, grid, s);
  }
  return -1;
}

// phase 1: X [T, K] bf16 gathered by sorted_token; W13 slots [2N, K]; out H [R, N]
int kt_launch_gemm_gate_up(int type, const void* x, int64_t T, int K, int N, const void* w13, int table,
                           const int32_t* tiles, const int32_t* n_tiles, const int32_t* sorted_token, void* h,
                           int* status, int grid, cudaStream_t s) {
  if (K % 256 || N % 128) return -1;
  CUtensorMap m;
  if (make_map(&m, x, T, K, 1)) return -2;
  KtGemmArgs a{};
  a.w = (const uint8_t*)w13;
  a.table = table;
  a.row_bytes = (int64_t)K / kt_block_info(type).qk * kt_block_info(type).bytes;
  a.K = K;
  a.N = N;
  a.K_out = K;
  a.tiles = tiles;
  a.n_tiles = n_tiles;
  a.n_wtiles = N / 128;
  a.sorted_token = sorted_token;
  a.out = (uint16_t*)h;
  a.out_ld = N;
  a.status = status;
  return launch_phase<1>(type, m, a, grid, s);
}

// phase 2: H [R, N] bf16 (sorted rows); W2 slots [K, N]; out Y [R, K]
int kt_launch_gemm_down(int type, const void* h, int64_t R, int K, int N, const void* w2, int table, const int32_t* tiles,
                        const int32_t* n_tiles, void* y, int* status, int grid, cudaStream_t s) {
  if (N % 256 || K % 256) return -1;
  CUtensorMap m;
  if (make_map(&m, h, R, N, kTN)) return -2;
  KtGemmArgs a{};
  a.w = (const uint8_t*)w2;
  a.table = table;
  a.row_bytes = (int64_t)N / kt_block_info(type).qk * kt_block_info(type).bytes;
  a.K = N;  // reduction length
  a.N = N;
  a.K_out = K;  // rows of W2
  a.tiles = tiles;
  a.n_tiles = n_tiles;
  a.n_wtiles = K / 256;
  a.sorted_token = nullptr;
  a.out = (uint16_t*)y;
  a.out_ld = K;
  a.status = status;
  return launch_phase<2>(type, m, a, grid, s);
}

int kt_gemm_tile_tokens() { return kTN; }
