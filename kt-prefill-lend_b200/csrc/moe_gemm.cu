// moe_gemm.cu — prefill path: persistent, warp-specialised tcgen05 grouped GEMM over the
// hot experts with in-kernel GGUF dequantization, on CTA pairs (cta_group::2).
//
// Replaces the reference's streamed-prefill pair "dequant experts to bf16 in HBM (Triton),
// then FlashInfer's bf16 CUTLASS fused MoE" (trees/flash-next-gguf patch, kt_stream_prefill_gguf
// _group_body; kt_gguf_dequant.py) and, at prefill sizes, the per-route GEMV build of
// kt_moe_a8_vec_multi (hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu:653). Weights stay in their
// GGUF bytes in HBM; each tile's raw super-blocks are copied into shared memory by TMA and
// dequantized there to bf16, so HBM sees 4.5-6.6 bits per weight instead of a bf16 round trip.
//
// Problem, per expert slot e with M_e routed tokens (sorted by slot):
//   phase 1: H[M_e, N]  = silu(X_e W_gate^T) * (X_e W_up^T)    (W13 rows [gate; up], K = hidden)
//   phase 2: Y[M_e, K]  = H W_down^T                             (W2 [K, N])
// Swap-AB: the MMA's M dimension is weight rows, N is tokens, reduction along K. A cluster of
// two CTAs (two SMs) computes one 256-row x 256-token tile with M=256 tcgen05 MMAs: each CTA
// holds 128 of the weight rows (A) and 128 of the tokens (B) in its shared memory and gets the
// accumulator of its 128 rows x 256 tokens in its own TMEM. Phase 1 gives each CTA 64 gate
// rows and the matching 64 up rows, so SwiGLU needs no data from the peer.
//
// Warp roles per CTA (P = 8 producer warps in phase 1, 16 in phase 2):
//   warps 0..P-1  dequant producers: two (phase 1) or four (phase 2) threads per A row, each
//                 decoding 16 values per k-step quarter from the raw stage and writing them as
//                 bf16 into the A stage in the UMMA K-major 128-byte swizzle layout
//   warp P        raw loader: per 256-value super-block column, 2G 2-D TMA loads of a tensor
//                 map that views G consecutive weight rows as one (G = rows whose bytes make a
//                 16-byte multiple); slot tables fall back to one 1-D bulk copy per row
//   warp P+1      B loader: phase 1 gathers this CTA's token rows of X with 16-byte cp.async
//                 copies into the swizzled stage, 32 rows each, together with warps P+7..P+9;
//                 phase 2 loads H rows with one 2-D TMA per k-step
//   warp P+2      even CTA: MMA issuer (tcgen05.mma.cta_group::2, commits multicast to both
//                 CTAs); odd CTA: forwards its stage completions to the even CTA's barrier
//   warps P+3..P+6 epilogue: tcgen05.ld of the accumulator; phase 1 SwiGLU -> H (bf16),
//                 phase 2 -> Y (bf16)
// The pair's two CTAs meet on the even CTA's stage barriers: the odd CTA's producers and B
// copies complete a local barrier, and one warp forwards each completed stage with a single
// remote arrival.
// TMEM (per CTA): two 256-column fp32 accumulators, so the epilogue of one tile overlaps the
// MMAs of the next. Every TMA and bulk copy lands in the issuing CTA only (no cluster-wide
// delivery of loaded data).
#include <stdlib.h>
#include <string.h>

#include "gguf_dot.cuh"
#include "gguf_tile.cuh"
#include "kt_kernels.h"

namespace {

// Warp roles per phase. Phase 1 runs 8 producer warps (two threads per A row) and four warps
// gathering token rows (32 rows each): the gather rate grows with the number of gathering
// warps, not with the copies per warp, and four outrun the dequant producers. Phase 2 loads B
// with one TMA per k-step and runs 16 producer warps (four threads per A row), which shortens
// each producer's per-k-step latency, the bound of phase 2. The epilogue warps' index modulo 4
// is the TMEM lane quadrant they may read.
template <int PHASE>
struct Roles {
  static constexpr int kProd = PHASE == 1 ? 8 : 16;  // producer warps
  static constexpr int kRaw = kProd, kMma = kProd + 2, kEpi0 = kProd + 3;
  static constexpr int kGather = PHASE == 1 ? 4 : 1;  // B loader warps: P+1, then P+7, P+8, ...
  static constexpr int kThreads = 32 * (kProd + 6 + kGather);
  static constexpr int kQuarters = 4 * 128 / (32 * kProd);  // k-step quarters per producer thread (2 or 1)
  static_assert(kQuarters == 1 || kQuarters == 2, "two or four producer threads per A row");
  // B loader index of a warp, or -1
  static __device__ __forceinline__ int gather_index(int warp) {
    if (warp == kProd + 1) return 0;
    if (warp >= kProd + 7 && warp < kProd + 6 + kGather) return warp - kProd - 6;
    return -1;
  }
};
template <bool B>
struct KtBool {
  static constexpr bool value = B;
};
constexpr int kTN = 256;           // tokens per tile (MMA N, split between the pair)
constexpr int kHalfN = kTN / 2;    // B rows held by each CTA
constexpr int kStages = 4;         // A/B stages
constexpr int kAStageBytes = 128 * 128;
constexpr int kBStageBytes = kHalfN * 128;
constexpr int kXchgBytes = 2 * 32 * 32 * 4;  // phase-1 epilogue: up values for the gate warps
constexpr int kEpiBytes = 4 * 32 * 32 * 2;   // per-warp transpose buffers
constexpr int kFixedSmem = kStages * (kAStageBytes + kBStageBytes) + kXchgBytes + kEpiBytes + 2048 /* grid */ +
                           1024 /* barriers */ + 1024 /* alignment slack */;
// A/B stages: 4 with the raw ring of the in-kernel dequant; 6 when A arrives as bf16 by TMA
// (PRE: no raw ring)
template <bool PRE>
struct Stages {
  static constexpr int N = PRE ? 6 : kStages;
  static constexpr int SMEM = N * (kAStageBytes + kBStageBytes) + kXchgBytes + kEpiBytes + 2048 + 1024 + 1024;
};

// Raw staging: a "unit" is UV consecutive values of one weight row (a 256-value super-block,
// or four 32-value Q8_0 blocks); a raw stage holds one unit for the CTA's 128 rows. Each
// row's slot holds the 16-byte aligned span around its unit (TMA needs 16-byte aligned
// addresses and sizes; GGUF blocks are only 2-byte aligned).
template <int TYPE, int AVAIL_ = 227 * 1024 - kFixedSmem, int MINRAW = 2>
struct Raw {
  static constexpr int UV = TYPE == KT_Q8_0 ? 128 : 256;
  static constexpr int UNIT_BYTES = TYPE == KT_Q8_0 ? 4 * 34 : kt_block_info(TYPE).bytes;
  static constexpr int SPAN = (UNIT_BYTES + 14 + 15) / 16 * 16;  // the unit starts at an even offset <= 14
  static constexpr int AVAIL = AVAIL_;
  // an odd number of 16-byte chunks per slot keeps 16-byte loads of 8 consecutive rows on
  // distinct bank groups; taken when the minimum number of stages still fits
  static constexpr int SLOT =
      ((SPAN / 16) % 2 == 0 && MINRAW * 128 * (SPAN + 16) + MINRAW * 2048 <= AVAIL) ? SPAN + 16 : SPAN;
  // a stage = two 64-row segments (gate / up rows in phase 1); a segment = G sub-tiles of
  // 64/G rows, one per TMA load, each starting on a 128-byte boundary (TMA destinations
  // must); producer thread l reads slot l%64 of its segment in this order
  static constexpr int SEG_BYTES = 64 * SLOT + 1024;
  static constexpr int STAGE_BYTES = 2 * SEG_BYTES;
  static constexpr int NRAW_FIT = AVAIL / STAGE_BYTES;
  static constexpr int NRAW = NRAW_FIT > 4 ? 4 : NRAW_FIT;
  static constexpr int KPU = UV / 64;  // k-steps per unit
  static_assert(NRAW >= MINRAW, "raw ring too small");
};

template <int TYPE>
constexpr int smem_bytes() {
  return kFixedSmem + Raw<TYPE>::NRAW * Raw<TYPE>::STAGE_BYTES;
}

// silu(x) = x * sigmoid(x), sigmoid(x) = 0.5 + 0.5 * tanh(x / 2): one hardware tanh
// (tanh.approx.f32, about 2^-11 relative error) per value; the result is rounded to bf16
__device__ __forceinline__ float kt_tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu(float x) { return x * fmaf(0.5f, kt_tanh_approx(0.5f * x), 0.5f); }

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// raw sub-tile pitch: 64/G slots of `slot` bytes rounded up to a 128-byte boundary
__device__ __forceinline__ int sub_pitch(int slot, int G) { return ((64 / G) * slot + 127) & ~127; }
// weight row (within a 64-row segment) held by slot position rr when the G sub-tiles hold
// rows j, j+G, j+2G, ...
__device__ __forceinline__ int wrow(int rr, int G) { return (rr % (64 / G)) * G + rr / (64 / G); }

// global row (within a slot) of A row `rh` of this CTA in weight tile `wt`
template <int PHASE>
__device__ __forceinline__ int64_t a_row(int rh, int wt, uint32_t cr, int N) {
  if constexpr (PHASE == 1)
    return rh < 64 ? (int64_t)wt * 128 + 64 * cr + rh : (int64_t)N + (int64_t)wt * 128 + 64 * cr + (rh - 64);
  return (int64_t)wt * 256 + 128 * cr + rh;
}

}  // namespace

// LINEAR (phase 1 only): the epilogue stores both halves of the projection as they are, with
// no activation (kt_moe_gemm_routes), instead of silu(gate) * up
template <int TYPE, int PHASE, bool LINEAR = false, bool PRE = false>
__global__ void __launch_bounds__(Roles<PHASE>::kThreads, 1) kt_moe_gemm_kernel(const __grid_constant__ CUtensorMap bmap,
                                                                  const __grid_constant__ CUtensorMap wmap,
                                                                  const KtGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  using RL = Roles<PHASE>;
  constexpr int kProdWarps = RL::kProd, kWarpRaw = RL::kRaw, kWarpMma = RL::kMma, kWarpEpi0 = RL::kEpi0,
                kGatherWarps = RL::kGather;
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  using R = Raw<TYPE>;
  constexpr int NS = Stages<PRE>::N;
  uint8_t* sA = smem;
  uint8_t* sB = sA + NS * kAStageBytes;
  uint8_t* sRaw = sB + NS * kBStageBytes;
  float* sX = reinterpret_cast<float*>(sRaw + (PRE ? 0 : R::NRAW * R::STAGE_BYTES));
  uint16_t* sEpi = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(sX) + kXchgBytes);
  uint32_t* sGrid = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sEpi) + kEpiBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGrid + 512);
  uint64_t* full = bars;                 // [NS] even CTA: A and B of both CTAs landed
  uint64_t* empty = full + NS;      // [NS] both CTAs: MMAs of the stage done
  uint64_t* bfull = empty + NS;     // [NS] odd CTA: its A and B of the stage landed
  uint64_t* raw_full = bfull + NS;  // [NRAW]
  uint64_t* raw_empty = raw_full + R::NRAW;
  uint64_t* acc_full = raw_empty + R::NRAW;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2] even CTA
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t cr = kt_cluster_rank();
  const bool leader = cr == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      // even CTA: its producer warps (PRE: the one thread that loads A), its B copies, and one
      // forwarded arrival for the odd CTA's producers and B copies (which arrive on its bfull)
      constexpr int kProdArrive = PRE ? 1 : kProdWarps;
      kt_mbar_init(&full[s], kProdArrive + (PHASE == 1 ? 32 * kGatherWarps : 1) + 1);
      kt_mbar_init(&empty[s], 1);
      kt_mbar_init(&bfull[s], kProdArrive + (PHASE == 1 ? 32 * kGatherWarps : 1));
    }
    for (int s = 0; s < R::NRAW; ++s) {
      kt_mbar_init(&raw_full[s], 1);
      kt_mbar_init(&raw_empty[s], kProdWarps);
    }
    for (int b = 0; b < 2; ++b) {
      kt_mbar_init(&acc_full[b], 1);
      kt_mbar_init(&acc_empty[b], 8);
    }
    kt_mbar_init(done_bar, 1);
    *abort_flag = 0;
    kt_fence_mbar_init();
  }
  if constexpr (TYPE == KT_IQ3_S && !PRE) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) sGrid[i] = kt_iq3s_grid_dev[i];
  }
  kt_cluster_sync();  // the peer's barriers are initialised before any remote arrival
  if (warp == kWarpMma) kt_tmem_alloc2(tmem_slot, 512);
  kt_tc_fence_before();
  __syncthreads();
  kt_tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  kt_pdl_trigger();  // the next kernel may set itself up on SMs this grid leaves
  kt_pdl_wait();     // the permutation (tiles, sorted tokens) and the inputs are complete

  const int n_tiles = *a.n_tiles;
  const int n_wt = a.n_wtiles;
  const int n_items = n_tiles * n_wt;
  const int ksteps = a.K / 64;
  const int units = a.K / R::UV;
  const int first_item = blockIdx.x >> 1, item_stride = gridDim.x >> 1;
  const int64_t rows_total = PHASE == 1 ? 2 * (int64_t)a.N : (int64_t)a.K_out;

  if (PRE && warp < kProdWarps) {
    // ---------------------------------------------------------------- A loader (PRE)
    // the weights were dequantized to bf16 [slots * rows, K] before this kernel: per k-step one
    // thread loads this CTA's 64 gate (or first) rows and 64 up (or next) rows with two 2-D TMA
    // loads in the 128-byte swizzle, the layout the dequant producers write
    if (warp == 0 && lane == 0) {
      uint64_t* stage_bar = leader ? full : bfull;
      uint32_t kit = 0;
      for (int item = first_item; item < n_items && !*abort_flag; item += item_stride) {
        const int tile = item / n_wt, wt = item % n_wt;
        const int64_t r0 = (int64_t)a.tiles[3 * tile + 0] * rows_total;
        for (int ks = 0; ks < ksteps; ++ks, ++kit) {
          const int s = kit % NS;
          if (!kt_mbar_wait(&empty[s], ((kit / NS) & 1) ^ 1, a.status, abort_flag)) break;
          uint8_t* dst = sA + s * kAStageBytes;
          kt_mbar_arrive_expect_tx(&stage_bar[s], (uint32_t)kAStageBytes);
#pragma unroll
          for (int sg = 0; sg < 2; ++sg)
            kt_tma_2d(dst + sg * (kAStageBytes / 2), &wmap, ks * 64, (int)(r0 + a_row<PHASE>(64 * sg, wt, cr, a.N)),
                      &stage_bar[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp < kProdWarps) {
    // ---------------------------------------------------------------- dequant producers
    // thread -> A row rh (= TMEM lane) -> raw slot in load order: the G sub-tiles of a
    // segment hold weight rows j, j+G, ...; lane rh holds weight row seg*64 + wrow(rh)
    const int rh = threadIdx.x & 127, qt0 = (threadIdx.x >> 7) * RL::kQuarters;
    const int G = a.raw_group > 0 ? a.raw_group : 1;
    const int seg = rh >> 6, rr = rh & 63;
    const int slot_off = seg * R::SEG_BYTES + (rr / (64 / G)) * sub_pitch(R::SLOT, G) + (rr % (64 / G)) * R::SLOT;
    const int wr = seg * 64 + wrow(rr, G);
    uint64_t* stage_bar = leader ? full : bfull;  // local; the odd CTA's forwarder warp relays
    uint32_t kit = 0, uit = 0;
    for (int item = first_item; item < n_items && !*abort_flag; item += item_stride) {
      const int tile = item / n_wt, wt = item % n_wt;
      const int slot = a.tiles[3 * tile + 0];
      const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                     : a.w + (int64_t)slot * rows_total * a.row_bytes;
      const uint8_t* grow_ptr = wbase + a_row<PHASE>(wr, wt, cr, a.N) * a.row_bytes;
      for (int u = 0; u < units && !*abort_flag; ++u, ++uit) {
        const int su = uit % R::NRAW;
        if (!kt_mbar_wait(&raw_full[su], (uit / R::NRAW) & 1, a.status, abort_flag)) break;
        // the loader copied the 16-byte aligned span around this row's unit into the row's
        // slot; the unit starts at the alignment remainder of its global address
        const int off = (int)(((uintptr_t)(grow_ptr + (int64_t)u * R::UNIT_BYTES)) & 15);
        const uint8_t* slotp = sRaw + su * R::STAGE_BYTES + slot_off;
        // the unit's k-steps; A16: the unit starts on a 16-byte boundary of its slot
        auto run_unit = [&](auto a16) -> bool {
          constexpr bool A16 = decltype(a16)::value;
          // one decoder per k-step quarter of this thread (decoders may keep bytes across k-steps)
          KtTileDq<TYPE> dq[RL::kQuarters];
#pragma unroll
          for (int j = 0; j < RL::kQuarters; ++j) dq[j].template unit<A16>(slotp, off, qt0 + j);
          bool ok = true;
#pragma unroll
          for (int kk = 0; kk < R::KPU; ++kk) {
            const int s = (kit + kk) % NS;
            if (ok && !kt_mbar_wait(&empty[s], (((kit + kk) / NS) & 1) ^ 1, a.status, abort_flag)) ok = false;
            if (ok) {
              uint8_t* arow = sA + s * kAStageBytes;
              // quarters beat one wider half per thread here: more independent loads in flight
#pragma unroll
              for (int j = 0; j < RL::kQuarters; ++j) {
                uint32_t pk[8];
                dq[j].template kstep_quarter<A16>(slotp, off, kk, qt0 + j, pk, sGrid);
#pragma unroll
                for (int c = 0; c < 2; ++c)
                  *reinterpret_cast<uint4*>(arow + kt_swz128(rh, 16 * (qt0 + j) + 8 * c)) =
                      make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
              }
              kt_fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) kt_mbar_arrive(&stage_bar[s]);
            }
          }
          return ok;
        };
        bool ok;
        if constexpr (KtTileDq<TYPE>::kAlignable) {
          ok = off == 0 ? run_unit(KtBool<true>()) : run_unit(KtBool<false>());
        } else {
          ok = run_unit(KtBool<false>());
        }
        kit += R::KPU;
        if (!ok) break;
        __syncwarp();
        if (lane == 0) kt_mbar_arrive(&raw_empty[su]);
      }
    }
  } else if (warp == kWarpRaw) {
    // ---------------------------------------------------------------- raw loader
    uint32_t uit = 0;
    for (int item = first_item; !PRE && item < n_items && !*abort_flag; item += item_stride) {  // idle with PRE
      const int tile = item / n_wt, wt = item % n_wt;
      const int slot = a.tiles[3 * tile + 0];
      const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                     : a.w + (int64_t)slot * rows_total * a.row_bytes;
      for (int u = 0; u < units && !*abort_flag; ++u, ++uit) {
        const int su = uit % R::NRAW;
        if (!kt_mbar_wait(&raw_empty[su], ((uit / R::NRAW) & 1) ^ 1, a.status, abort_flag)) break;
        uint8_t* stage = sRaw + su * R::STAGE_BYTES;
        if (a.raw_group > 0) {
          // per 64-row segment, G loads: sub-tile j holds rows j, j+G, ... (group rows)
          if (lane == 0) {
            const int G = a.raw_group;
            kt_mbar_arrive_expect_tx(&raw_full[su], 128u * R::SLOT);
            for (int sg = 0; sg < 2; ++sg) {
              const int64_t first = (int64_t)slot * rows_total + a_row<PHASE>(64 * sg, wt, cr, a.N);
              for (int j = 0; j < G; ++j) {
                const int x = (int)(((int64_t)j * a.row_bytes + (int64_t)u * R::UNIT_BYTES) & ~(int64_t)15);
                kt_tma_2d(stage + sg * R::SEG_BYTES + j * sub_pitch(R::SLOT, G), &wmap, x, (int)(first / G),
                          &raw_full[su]);
              }
            }
          }
          __syncwarp();
          continue;
        }
        uintptr_t src[4];
        uint32_t len[4], total = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rh = lane + 32 * i;
          const uintptr_t g = (uintptr_t)(wbase + a_row<PHASE>(rh, wt, cr, a.N) * a.row_bytes + (int64_t)u * R::UNIT_BYTES);
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
          kt_bulk_g2s(stage + ((lane + 32 * i) >> 6) * R::SEG_BYTES + ((lane + 32 * i) & 63) * R::SLOT,
                      reinterpret_cast<const void*>(src[i]), len[i], &raw_full[su]);
      }
    }
  } else if (RL::gather_index(warp) >= 0) {
    // ---------------------------------------------------------------- B loaders
    const int gw = RL::gather_index(warp);
    constexpr int NR = kHalfN / (4 * kGatherWarps);  // rows per lane per k-step (phase 1)
    uint32_t kit = 0;
    for (int item = first_item; item < n_items && !*abort_flag; item += item_stride) {
      const int tile = item / n_wt;
      const int pos0 = a.tiles[3 * tile + 1], ntok = a.tiles[3 * tile + 2];
      const int half = ((ntok + 31) & ~31) / 2;  // B rows of each CTA (the MMA N is 2*half)
      const int b0 = cr * half;                  // first tile row held by this CTA
      // phase 1: lane copies 16-byte chunk (lane % 8) of rows lane/8 + 4*(gw + 2i); the
      // token ids of those rows are kept in registers for the whole tile
      int tokr[NR];
      if constexpr (PHASE == 1) {
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          const int j = (lane >> 3) + 4 * (gw + kGatherWarps * i);
          tokr[i] = j < half ? a.sorted_token[pos0 + (b0 + j < ntok ? b0 + j : 0)] : 0;
        }
      }
      for (int ks = 0; ks < ksteps && !*abort_flag; ++ks, ++kit) {
        const int s = kit % NS;
        if (!kt_mbar_wait(&empty[s], ((kit / NS) & 1) ^ 1, a.status, abort_flag)) break;
        uint8_t* dst = sB + s * kBStageBytes;
        uint64_t* bar = leader ? &full[s] : &bfull[s];
        if constexpr (PHASE == 1) {
          const int c = lane & 7;
          const uint16_t* xk = a.x + (int64_t)ks * 64 + 8 * c;
#pragma unroll
          for (int i = 0; i < NR; ++i) {
            const int j = (lane >> 3) + 4 * (gw + kGatherWarps * i);
            if (j < half) kt_cp_async16(dst + kt_swz128(j, 8 * c), xk + (int64_t)tokr[i] * a.K);
          }
          kt_cp_async_arrive(bar);
        } else if (gw == 0) {
          if (lane == 0) {
            // 128 rows from the first row of this CTA's half; rows past the tile belong to the
            // next tile or lie past the end (zero fill) and only reach unused accumulator columns
            kt_mbar_arrive_expect_tx(bar, (uint32_t)kBStageBytes);
            kt_tma_2d(dst, &bmap, ks * 64, pos0 + b0, bar);
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == kWarpMma) {
    if (leader) {
      // -------------------------------------------------------------- MMA issuer (even CTA)
      // One lane runs the whole loop: a tcgen05.mma holds its issuing thread for most of its
      // execution, so the tensor pipe only stays busy if the work between one k-step's MMAs
      // and the next (stage wait, bookkeeping) stays short. Lanes 1-31 wait at the __syncwarp.
      if (lane == 0) {
        uint32_t s = 0, ph = 0, iit = 0;  // stage, its phase parity, items done
        const uint32_t sa0 = kt_smem_addr(sA), sb0 = kt_smem_addr(sB);
        // each item's token count is read one item ahead, off the MMA's path
        int ntok_next = first_item < n_items ? a.tiles[3 * (first_item / n_wt) + 2] : 0;
        bool ok = true;
        for (int item = first_item; ok && item < n_items; item += item_stride, ++iit) {
          const int ntok = ntok_next;
          const int next = item + item_stride;
          ntok_next = next < n_items ? a.tiles[3 * (next / n_wt) + 2] : 0;
          const uint32_t idesc = kt_idesc_bf16(256, (ntok + 31) & ~31);
          const int b = iit & 1;
          if (!kt_mbar_wait_cluster(&acc_empty[b], ((iit >> 1) & 1) ^ 1, a.status, abort_flag)) break;
          kt_tc_fence_after();
          const uint32_t d = tmem + 256 * b;
          for (int ks = 0; ks < ksteps; ++ks) {
            if (!kt_mbar_wait_cluster(&full[s], ph, a.status, abort_flag)) {
              ok = false;
              break;
            }
            kt_tc_fence_after();
            const uint64_t da = kt_desc_k128(sa0 + s * kAStageBytes);
            const uint64_t db = kt_desc_k128(sb0 + s * kBStageBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) kt_mma2_bf16_ss(d, da + 2 * kk, db + 2 * kk, idesc, (ks | kk) != 0);
            kt_mma2_commit_mc(&empty[s], 3);
            if (++s == NS) {
              s = 0;
              ph ^= 1;
            }
          }
          if (ok) kt_mma2_commit_mc(&acc_full[b], 3);
        }
        kt_mma2_commit_mc(done_bar, 3);
      }
      __syncwarp();
    } else {
      // -------------------------------------------------------------- stage forwarder (odd CTA):
      // one cluster-scope arrival per stage once this CTA's A rows and B rows have landed
      if (lane == 0) {
        uint32_t s = 0, ph = 0;
        const uint32_t full0 = kt_mapa(&full[0], 0);
        bool ok = true;
        for (int item = first_item; ok && item < n_items; item += item_stride) {
          for (int ks = 0; ks < ksteps; ++ks) {
            if (!kt_mbar_wait(&bfull[s], ph, a.status, abort_flag)) {
              ok = false;
              break;
            }
            kt_mbar_arrive_cluster(full0 + 8 * s);
            if (++s == NS) {
              s = 0;
              ph ^= 1;
            }
          }
        }
      }
      __syncwarp();
    }
    kt_mbar_wait(done_bar, 0, a.status, nullptr);  // every MMA of the pair has completed
  } else if (warp >= kWarpEpi0 && warp < kWarpEpi0 + 4) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int G = a.raw_group > 0 ? a.raw_group : 1;
    const int l = 32 * q + lane;                   // TMEM lane = A row of this CTA
    const int wr = (l >> 6) * 64 + wrow(l & 63, G);  // weight row (feature) it holds
    const uint32_t acc_empty0 = kt_mapa(&acc_empty[0], 0);
    uint32_t iit = 0;
    for (int item = first_item; item < n_items && !*abort_flag; item += item_stride, ++iit) {
      const int tile = item / n_wt, wt = item % n_wt;
      const int pos0 = a.tiles[3 * tile + 1], ntok = a.tiles[3 * tile + 2];
      const int b = iit & 1;
      if (!kt_mbar_wait(&acc_full[b], (iit >> 1) & 1, a.status, abort_flag)) break;
      kt_tc_fence_after();
      const uint32_t lane_base = tmem + 256 * b + ((uint32_t)(32 * q) << 16);
      for (int c0 = 0; c0 < ntok; c0 += 32) {
        uint32_t v[32];
        kt_tmem_ld32(lane_base + c0, v);
        kt_tmem_wait_ld();
        if constexpr (PHASE == 1 && LINEAR) {
          // lanes 0-63 hold rows [wt*128 + 64cr, +64) of the weight, lanes 64-127 the rows N
          // above them: staged [token][128 positions], then each half to its own output columns
#pragma unroll
          for (int j = 0; j < 32; ++j) sEpi[j * 128 + wr] = kt_f2bf(__uint_as_float(v[j]));
          epi_bar();
          const int t = l, c = t & 15;
          const int64_t col = (c < 8 ? 0 : (int64_t)a.N) + (int64_t)wt * 128 + 64 * cr + 8 * (c & 7);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int tok = (t >> 4) + 8 * i;
            if (c0 + tok < ntok)
              *reinterpret_cast<uint4*>(a.out + (int64_t)(pos0 + c0 + tok) * a.out_ld + col) =
                  *reinterpret_cast<const uint4*>(sEpi + tok * 128 + 8 * c);
          }
          epi_bar();
        } else if constexpr (PHASE == 1) {
          // lanes 0-63 hold gate rows, 64-127 the matching up rows: the up warps hand their
          // values to the gate warps through shared memory; h is staged [token][feature]
          float* xq = sX + (q & 1) * 32 * 32;
          if (q >= 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) xq[j * 32 + lane] = __uint_as_float(v[j]);
          }
          epi_bar();
          if (q < 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) sEpi[j * 64 + wr] = kt_f2bf(silu(__uint_as_float(v[j])) * xq[j * 32 + lane]);
          }
          epi_bar();
          // 32 tokens x 64 features (128 bytes per token): thread copies 16-byte chunk
          // (t % 8) of token t / 8 + 16 i
          const int t = l, c = t & 7;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int tok = (t >> 3) + 16 * i;
            if (c0 + tok < ntok)
              *reinterpret_cast<uint4*>(a.out + (int64_t)(pos0 + c0 + tok) * a.out_ld + (int64_t)wt * 128 + 64 * cr + 8 * c) =
                  *reinterpret_cast<const uint4*>(sEpi + tok * 64 + 8 * c);
          }
          epi_bar();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) sEpi[j * 128 + wr] = kt_f2bf(__uint_as_float(v[j]));
          epi_bar();
          // 32 tokens x 128 features (256 bytes per token): thread copies 16-byte chunk
          // (t % 16) of token t / 16 + 8 i
          const int t = l, c = t & 15;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int tok = (t >> 4) + 8 * i;
            if (c0 + tok < ntok)
              *reinterpret_cast<uint4*>(a.out + (int64_t)(pos0 + c0 + tok) * a.out_ld + (int64_t)wt * 256 + 128 * cr + 8 * c) =
                  *reinterpret_cast<const uint4*>(sEpi + tok * 128 + 8 * c);
          }
          epi_bar();
        }
      }
      kt_tc_fence_before();
      __syncwarp();
      if (lane == 0) kt_mbar_arrive_cluster(acc_empty0 + 8 * b);
    }
  }

  kt_tc_fence_before();
  __syncthreads();
  // after a timed-out wait the loaders may have copies (TMA, bulk, cp.async) in flight that no
  // role waited for: let them land in this CTA's shared memory before it can exit
  if (*abort_flag) kt_drain_ns(200000);
  kt_cluster_sync();  // neither CTA leaves while the pair's MMAs may read its shared memory
  if (warp == kWarpMma) {
    kt_tc_fence_after();
    kt_tmem_dealloc2(tmem, 512);
  }
}


// ------------------------------------------------------------------ down projection, resident A
//
// Phase 2 with a short reduction (N <= 512: at most kResSlices k-steps). Each CTA keeps the
// whole dequantized A strip of its 128 weight rows (one slice of 128 rows x 64 values per
// k-step, 16 KB each) in shared memory and runs it against every token tile of a chunk of up
// to kResChunk consecutive tiles, decoding again only when the slot (expert) changes. At
// config 2 (540 token tiles over 64 slots) this decodes each weight tile ~3x instead of ~8x.
// Work unit = (chunk, weight tile), chunk-major, so the pairs that share a chunk's H rows run
// side by side. Slices are refilled one at a time as the last tile that reads them finishes,
// so a refill overlaps the MMAs of the previous strip's last tile.
// Roles: warps 0-15 dequant producers (four threads per A row), 16 raw loader, 17 B loader
// (one 2-D TMA of H rows per k-step), 18 MMA issuer (even CTA) / stage forwarder (odd CTA),
// 19-22 epilogue (Y rows in bf16).
constexpr int kResSlices = 8;  // resident A slices: reduction length <= 512
constexpr int kResB = 3;       // B stages
constexpr int kResChunk = 4;   // token tiles per work unit
constexpr int kResFixed = kResSlices * kAStageBytes + kResB * kBStageBytes + kEpiBytes + 2048 /* grid */ +
                          1024 /* barriers */ + 1024 /* alignment slack */;
template <int TYPE>
using RawRes = Raw<TYPE, 227 * 1024 - kResFixed, 1>;
template <int TYPE>
constexpr int res_smem_bytes() {
  return kResFixed + RawRes<TYPE>::NRAW * RawRes<TYPE>::STAGE_BYTES;
}
struct ResRoles {
  static constexpr int kProd = 16, kRaw = 16, kB = 17, kMma = 18, kEpi0 = 19, kThreads = 32 * 23;
};

// One work unit: a chunk of at most kResChunk consecutive token tiles of one slot (from the
// permutation's chunk list: slot, first sorted row, rows) and a weight tile. Its tiles are
// full 256-row tiles but the last. Each role loads the next unit's entry when it starts the
// current one, so the load's latency is spent while it works.
struct ResUnit {
  int wt, slot, pos0, rows;
  __device__ __forceinline__ int n() const { return (rows + kTN - 1) / kTN; }
  __device__ __forceinline__ int tile_pos0(int i) const { return pos0 + kTN * i; }
  __device__ __forceinline__ int tile_rows(int i) const { return min(kTN, rows - kTN * i); }
};
__device__ __forceinline__ ResUnit res_unit(const int32_t* chunks, int n_wt, int n_units, int un) {
  ResUnit u{0, 0, 0, 0};
  if (un < n_units) {
    const int c = un / n_wt;
    u.wt = un % n_wt;
    u.slot = chunks[3 * c];
    u.pos0 = chunks[3 * c + 1];
    u.rows = chunks[3 * c + 2];
  }
  return u;
}

template <int TYPE>
__global__ void __launch_bounds__(ResRoles::kThreads, 1) kt_moe_down_res_kernel(const __grid_constant__ CUtensorMap bmap,
                                                                              const __grid_constant__ CUtensorMap wmap,
                                                                              const KtGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  using R = RawRes<TYPE>;
  using RL = ResRoles;
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = sA + kResSlices * kAStageBytes;
  uint8_t* sRaw = sB + kResB * kBStageBytes;
  uint16_t* sEpi = reinterpret_cast<uint16_t*>(sRaw + R::NRAW * R::STAGE_BYTES);
  uint32_t* sGrid = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sEpi) + kEpiBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGrid + 512);
  uint64_t* afull = bars;                   // [kResSlices] slice written (even CTA: by both CTAs)
  uint64_t* aempty = afull + kResSlices;    // [kResSlices] the strip's last MMAs on the slice done
  uint64_t* bfull = aempty + kResSlices;    // [kResB] H rows landed (even CTA: in both CTAs)
  uint64_t* bempty = bfull + kResB;         // [kResB]
  uint64_t* raw_full = bempty + kResB;      // [NRAW]
  uint64_t* raw_empty = raw_full + R::NRAW;
  uint64_t* acc_full = raw_empty + R::NRAW;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2] even CTA
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t cr = kt_cluster_rank();
  const bool leader = cr == 0;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kResSlices; ++j) {
      kt_mbar_init(&afull[j], RL::kProd + (leader ? 1 : 0));  // + the odd CTA's forwarded arrival
      kt_mbar_init(&aempty[j], 1);
    }
    for (int s = 0; s < kResB; ++s) {
      kt_mbar_init(&bfull[s], 1 + (leader ? 1 : 0));
      kt_mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < R::NRAW; ++s) {
      kt_mbar_init(&raw_full[s], 1);
      kt_mbar_init(&raw_empty[s], RL::kProd);
    }
    for (int b = 0; b < 2; ++b) {
      kt_mbar_init(&acc_full[b], 1);
      kt_mbar_init(&acc_empty[b], 8);
    }
    kt_mbar_init(done_bar, 1);
    *abort_flag = 0;
    kt_fence_mbar_init();
  }
  if constexpr (TYPE == KT_IQ3_S) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) sGrid[i] = kt_iq3s_grid_dev[i];
  }
  kt_cluster_sync();
  if (warp == RL::kMma) kt_tmem_alloc2(tmem_slot, 512);
  kt_tc_fence_before();
  __syncthreads();
  kt_tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  kt_pdl_trigger();
  kt_pdl_wait();  // H (the gate/up kernel's output) and the chunk list are complete

  const int n_wt = a.n_wtiles;
  const int n_units = a.n_tiles[2] * n_wt;  // chunks x weight tiles
  const int ksteps = a.K / 64;
  const int units = a.K / R::UV;  // raw units per strip
  const int first_unit = blockIdx.x >> 1, unit_stride = gridDim.x >> 1;
  const int64_t rows_total = a.K_out;

  if (warp < RL::kProd) {
    // ---------------------------------------------------------------- dequant producers
    const int rh = threadIdx.x & 127, qt = threadIdx.x >> 7;
    const int G = a.raw_group > 0 ? a.raw_group : 1;
    const int seg = rh >> 6, rr = rh & 63;
    const int slot_off = seg * R::SEG_BYTES + (rr / (64 / G)) * sub_pitch(R::SLOT, G) + (rr % (64 / G)) * R::SLOT;
    const int wr = seg * 64 + wrow(rr, G);
    uint64_t* const fill_bar = afull;  // local; the odd CTA's forwarder relays
    uint32_t uit = 0, strip = 0;
    ResUnit nxt = res_unit(a.chunks, n_wt, n_units, first_unit);
    for (int un = first_unit; un < n_units && !*abort_flag; un += unit_stride) {
      const ResUnit cur = nxt;
      nxt = res_unit(a.chunks, n_wt, n_units, un + unit_stride);
      const int wt = cur.wt;
      {  // one strip per unit
        const int slot = cur.slot;
        const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                       : a.w + (int64_t)slot * rows_total * a.row_bytes;
        const uint8_t* grow_ptr = wbase + a_row<2>(wr, wt, cr, a.N) * a.row_bytes;
        bool ok = true;
        for (int u = 0; u < units && ok; ++u, ++uit) {
          const int su = uit % R::NRAW;
          if (!kt_mbar_wait(&raw_full[su], (uit / R::NRAW) & 1, a.status, abort_flag)) {
            ok = false;
            break;
          }
          const int off = (int)(((uintptr_t)(grow_ptr + (int64_t)u * R::UNIT_BYTES)) & 15);
          const uint8_t* slotp = sRaw + su * R::STAGE_BYTES + slot_off;
          auto run_unit = [&](auto a16) -> bool {
            constexpr bool A16 = decltype(a16)::value;
            KtTileDq<TYPE> dq;
            dq.template unit<A16>(slotp, off, qt);
#pragma unroll
            for (int kk = 0; kk < R::KPU; ++kk) {
              const int j = u * R::KPU + kk;
              // the previous strip's last tile has finished reading slice j
              if (strip > 0 && !kt_mbar_wait(&aempty[j], (strip - 1) & 1, a.status, abort_flag)) return false;
              uint8_t* arow = sA + j * kAStageBytes;
              uint32_t pk[8];
              dq.template kstep_quarter<A16>(slotp, off, kk, qt, pk, sGrid);
#pragma unroll
              for (int c = 0; c < 2; ++c)
                *reinterpret_cast<uint4*>(arow + kt_swz128(rh, 16 * qt + 8 * c)) =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
              kt_fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) kt_mbar_arrive(&fill_bar[j]);
            }
            return true;
          };
          if constexpr (KtTileDq<TYPE>::kAlignable) {
            ok = off == 0 ? run_unit(KtBool<true>()) : run_unit(KtBool<false>());
          } else {
            ok = run_unit(KtBool<false>());
          }
          __syncwarp();
          if (ok && lane == 0) kt_mbar_arrive(&raw_empty[su]);
        }
        if (!ok) break;
        ++strip;
      }
    }
  } else if (warp == RL::kRaw) {
    // ---------------------------------------------------------------- raw loader
    uint32_t uit = 0;
    ResUnit nxt = res_unit(a.chunks, n_wt, n_units, first_unit);
    for (int un = first_unit; un < n_units && !*abort_flag; un += unit_stride) {
      const ResUnit cur = nxt;
      nxt = res_unit(a.chunks, n_wt, n_units, un + unit_stride);
      const int wt = cur.wt;
      {  // one strip per unit
        const int slot = cur.slot;
        const uint8_t* wbase = a.table ? reinterpret_cast<const uint8_t*>(reinterpret_cast<const int64_t*>(a.w)[slot])
                                       : a.w + (int64_t)slot * rows_total * a.row_bytes;
        for (int u = 0; u < units && !*abort_flag; ++u, ++uit) {
          const int su = uit % R::NRAW;
          if (!kt_mbar_wait(&raw_empty[su], ((uit / R::NRAW) & 1) ^ 1, a.status, abort_flag)) break;
          uint8_t* stage = sRaw + su * R::STAGE_BYTES;
          if (a.raw_group > 0) {
            if (lane == 0) {
              const int G = a.raw_group;
              kt_mbar_arrive_expect_tx(&raw_full[su], 128u * R::SLOT);
              for (int sg = 0; sg < 2; ++sg) {
                const int64_t fr = (int64_t)slot * rows_total + a_row<2>(64 * sg, wt, cr, a.N);
                for (int j = 0; j < G; ++j) {
                  const int x = (int)(((int64_t)j * a.row_bytes + (int64_t)u * R::UNIT_BYTES) & ~(int64_t)15);
                  kt_tma_2d(stage + sg * R::SEG_BYTES + j * sub_pitch(R::SLOT, G), &wmap, x, (int)(fr / G),
                            &raw_full[su]);
                }
              }
            }
            __syncwarp();
            continue;
          }
          uintptr_t src[4];
          uint32_t len[4], total = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rh = lane + 32 * i;
            const uintptr_t g = (uintptr_t)(wbase + a_row<2>(rh, wt, cr, a.N) * a.row_bytes + (int64_t)u * R::UNIT_BYTES);
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
            kt_bulk_g2s(stage + ((lane + 32 * i) >> 6) * R::SEG_BYTES + ((lane + 32 * i) & 63) * R::SLOT,
                        reinterpret_cast<const void*>(src[i]), len[i], &raw_full[su]);
        }
      }
    }
  } else if (warp == RL::kB) {
    // ---------------------------------------------------------------- B loader (H rows by TMA)
    uint32_t kit = 0;
    ResUnit nxt = res_unit(a.chunks, n_wt, n_units, first_unit);
    for (int un = first_unit; un < n_units && !*abort_flag; un += unit_stride) {
      const ResUnit cur = nxt;
      nxt = res_unit(a.chunks, n_wt, n_units, un + unit_stride);
      const int nt = cur.n();
      for (int i = 0; i < nt && !*abort_flag; ++i) {
        const int pos0 = cur.tile_pos0(i), ntok = cur.tile_rows(i);
        const int half = ((ntok + 31) & ~31) / 2;
        const int b0 = cr * half;
        for (int ks = 0; ks < ksteps && !*abort_flag; ++ks, ++kit) {
          const int s = kit % kResB;
          if (!kt_mbar_wait(&bempty[s], ((kit / kResB) & 1) ^ 1, a.status, abort_flag)) break;
          if (lane == 0) {
            // rows past the tile belong to the next tile or lie past the end (zero fill) and
            // only reach unused accumulator columns
            kt_mbar_arrive_expect_tx(&bfull[s], (uint32_t)kBStageBytes);
            kt_tma_2d(sB + s * kBStageBytes, &bmap, ks * 64, pos0 + b0, &bfull[s]);
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == RL::kMma) {
    if (leader) {
      // -------------------------------------------------------------- MMA issuer (even CTA)
      // one lane runs the loop (see the streaming kernel's issuer); lanes 1-31 wait at the
      // __syncwarp
      if (lane == 0) {
        uint32_t s = 0, ph = 0, iit = 0, strip = 0;  // B stage and parity, tiles, strips
        const uint32_t sa0 = kt_smem_addr(sA), sb0 = kt_smem_addr(sB);
        ResUnit nxt = res_unit(a.chunks, n_wt, n_units, first_unit);
        bool ok = true;
        for (int un = first_unit; ok && un < n_units; un += unit_stride, ++strip) {
          const ResUnit cur = nxt;
          nxt = res_unit(a.chunks, n_wt, n_units, un + unit_stride);
          const int nt = cur.n();
          for (int i = 0; ok && i < nt; ++i, ++iit) {
            const uint32_t idesc = kt_idesc_bf16(256, (cur.tile_rows(i) + 31) & ~31);
            const int b = iit & 1;
            if (!kt_mbar_wait_cluster(&acc_empty[b], ((iit >> 1) & 1) ^ 1, a.status, abort_flag)) {
              ok = false;
              break;
            }
            kt_tc_fence_after();
            const uint32_t d = tmem + 256 * b;
            const bool last = i == nt - 1;
            for (int ks = 0; ks < ksteps; ++ks) {
              // the strip's first tile waits for each slice; later tiles find them resident
              if ((i == 0 && !kt_mbar_wait_cluster(&afull[ks], strip & 1, a.status, abort_flag)) ||
                  !kt_mbar_wait_cluster(&bfull[s], ph, a.status, abort_flag)) {
                ok = false;
                break;
              }
              kt_tc_fence_after();
              const uint64_t da = kt_desc_k128(sa0 + ks * kAStageBytes);
              const uint64_t db = kt_desc_k128(sb0 + s * kBStageBytes);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) kt_mma2_bf16_ss(d, da + 2 * kk, db + 2 * kk, idesc, (ks | kk) != 0);
              kt_mma2_commit_mc(&bempty[s], 3);
              if (last) kt_mma2_commit_mc(&aempty[ks], 3);
              if (++s == kResB) {
                s = 0;
                ph ^= 1;
              }
            }
            if (ok) kt_mma2_commit_mc(&acc_full[b], 3);
          }
        }
        kt_mma2_commit_mc(done_bar, 3);
      }
      __syncwarp();
    } else {
      // -------------------------------------------------------------- forwarder (odd CTA): relays
      // its slice and B-stage completions to the even CTA's barriers in the MMA's order
      if (lane == 0) {
        uint32_t s = 0, ph = 0, strip = 0;
        const uint32_t afull0 = kt_mapa(&afull[0], 0), bfull0 = kt_mapa(&bfull[0], 0);
        ResUnit nxt = res_unit(a.chunks, n_wt, n_units, first_unit);
        bool ok = true;
        for (int un = first_unit; ok && un < n_units; un += unit_stride, ++strip) {
          const ResUnit cur = nxt;
          nxt = res_unit(a.chunks, n_wt, n_units, un + unit_stride);
          const int nt = cur.n();
          for (int i = 0; ok && i < nt; ++i) {
            for (int ks = 0; ks < ksteps; ++ks) {
              if (i == 0) {
                if (!kt_mbar_wait(&afull[ks], strip & 1, a.status, abort_flag)) {
                  ok = false;
                  break;
                }
                kt_mbar_arrive_cluster(afull0 + 8 * ks);
              }
              if (!kt_mbar_wait(&bfull[s], ph, a.status, abort_flag)) {
                ok = false;
                break;
              }
              kt_mbar_arrive_cluster(bfull0 + 8 * s);
              if (++s == kResB) {
                s = 0;
                ph ^= 1;
              }
            }
          }
        }
      }
      __syncwarp();
    }
    kt_mbar_wait(done_bar, 0, a.status, nullptr);  // every MMA of the pair has completed
  } else if (warp >= RL::kEpi0 && warp < RL::kEpi0 + 4) {
    // ---------------------------------------------------------------- epilogue: Y rows (bf16)
    const int q = warp & 3;
    const int G = a.raw_group > 0 ? a.raw_group : 1;
    const int l = 32 * q + lane;
    const int wr = (l >> 6) * 64 + wrow(l & 63, G);
    const uint32_t acc_empty0 = kt_mapa(&acc_empty[0], 0);
    uint16_t* const sE = sEpi;  // shared by the four warps: one 32-token chunk at a time
    uint32_t iit = 0;
    ResUnit nxt = res_unit(a.chunks, n_wt, n_units, first_unit);
    for (int un = first_unit; un < n_units && !*abort_flag; un += unit_stride) {
      const ResUnit cur = nxt;
      nxt = res_unit(a.chunks, n_wt, n_units, un + unit_stride);
      const int wt = cur.wt, nt = cur.n();
      for (int i = 0; i < nt && !*abort_flag; ++i, ++iit) {
        const int pos0 = cur.tile_pos0(i), ntok = cur.tile_rows(i);
        const int b = iit & 1;
        if (!kt_mbar_wait(&acc_full[b], (iit >> 1) & 1, a.status, abort_flag)) break;
        kt_tc_fence_after();
        const uint32_t lane_base = tmem + 256 * b + ((uint32_t)(32 * q) << 16);
        for (int c0 = 0; c0 < ntok; c0 += 32) {
          uint32_t v[32];
          kt_tmem_ld32(lane_base + c0, v);
          kt_tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) sE[j * 128 + wr] = kt_f2bf(__uint_as_float(v[j]));
          epi_bar();
          // 32 tokens x 128 features (256 bytes per token): thread copies 16-byte chunk
          // (t % 16) of token t / 16 + 8 i
          const int c = l & 15;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int tok = (l >> 4) + 8 * i;
            if (c0 + tok < ntok)
              *reinterpret_cast<uint4*>(a.out + (int64_t)(pos0 + c0 + tok) * a.out_ld + (int64_t)wt * 256 + 128 * cr + 8 * c) =
                  *reinterpret_cast<const uint4*>(sE + tok * 128 + 8 * c);
          }
          epi_bar();
        }
        kt_tc_fence_before();
        __syncwarp();
        if (lane == 0) kt_mbar_arrive_cluster(acc_empty0 + 8 * b);
      }
    }
  }

  kt_tc_fence_before();
  __syncthreads();
  // after a timed-out wait the loaders may have copies (TMA, bulk, cp.async) in flight that no
  // role waited for: let them land in this CTA's shared memory before it can exit
  if (*abort_flag) kt_drain_ns(200000);
  kt_cluster_sync();  // neither CTA leaves while the pair's MMAs may read its shared memory
  if (warp == RL::kMma) {
    kt_tc_fence_after();
    kt_tmem_dealloc2(tmem, 512);
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

template <int TYPE>
static int raw_slot() {
  return Raw<TYPE>::SLOT;
}

template <int TYPE>
static int res_raw_slot() {
  return RawRes<TYPE>::SLOT;
}

static int raw_slot_of(int type, bool res) {
  if (res) {
    switch (type) {
      case KT_Q8_0: return res_raw_slot<KT_Q8_0>();
      case KT_Q4_K: return res_raw_slot<KT_Q4_K>();
      case KT_Q6_K: return res_raw_slot<KT_Q6_K>();
      case KT_IQ3_S: return res_raw_slot<KT_IQ3_S>();
    }
    return 0;
  }
  switch (type) {
    case KT_Q8_0: return raw_slot<KT_Q8_0>();
    case KT_Q4_K: return raw_slot<KT_Q4_K>();
    case KT_Q6_K: return raw_slot<KT_Q6_K>();
    case KT_IQ3_S: return raw_slot<KT_IQ3_S>();
  }
  return 0;
}

// Raw weight map: G consecutive rows of `row_bytes` form one tensor row of G*row_bytes bytes
// (a 16-byte multiple, as TMA requires), box {slot bytes, 64/G group rows}. Returns G, or 0
// when the plain-layout base is not 16-byte aligned (per-row bulk copies are used then).
static int make_raw_map(CUtensorMap* m, const void* w, int64_t row_bytes, int64_t rows_total, int n_slots, int type,
                        bool res = false) {
  if (((uintptr_t)w) & 15) return 0;
  int64_t g = 16;
  while (row_bytes % g) g /= 2;
  const int G = (int)(16 / g);
  if (rows_total % G || 64 % G) return 0;
  PFN_encodeTiled enc = get_encode();
  if (!enc) return 0;
  const int slot = raw_slot_of(type, res);
  cuuint64_t dims[2] = {(cuuint64_t)(G * row_bytes), (cuuint64_t)(n_slots * rows_total / G)};
  cuuint64_t strides[1] = {(cuuint64_t)(G * row_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)slot, (cuuint32_t)(64 / G)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? G : 0;
}

template <int TYPE, int PHASE, bool LINEAR = false, bool PRE = false>
static int launch_t(const CUtensorMap& m, const CUtensorMap& wm, const KtGemmArgs& a, int grid, cudaStream_t s) {
  constexpr int smem = PRE ? Stages<true>::SMEM : smem_bytes<TYPE>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  auto k = kt_moe_gemm_kernel<TYPE, PHASE, LINEAR, PRE>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -3;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(grid & ~1), 1, 1);  // whole CTA pairs
  cfg.blockDim = dim3(Roles<PHASE>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = kt_pdl_enabled() ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, k, m, wm, a) != cudaSuccess) return -4;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int TYPE>
static int launch_res(const CUtensorMap& m, const CUtensorMap& wm, const KtGemmArgs& a, int grid, cudaStream_t s) {
  constexpr int smem = res_smem_bytes<TYPE>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  auto k = kt_moe_down_res_kernel<TYPE>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -3;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(grid & ~1), 1, 1);
  cfg.blockDim = dim3(ResRoles::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = kt_pdl_enabled() ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, k, m, wm, a) != cudaSuccess) return -4;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int PHASE, bool LINEAR = false>
static int launch_phase(int type, const CUtensorMap& m, const CUtensorMap& wm, const KtGemmArgs& a, int grid,
                        cudaStream_t s) {
  switch (type) {
    case KT_Q8_0: return launch_t<KT_Q8_0, PHASE, LINEAR>(m, wm, a, grid, s);
    case KT_Q4_K: return launch_t<KT_Q4_K, PHASE, LINEAR>(m, wm, a, grid, s);
    case KT_Q6_K: return launch_t<KT_Q6_K, PHASE, LINEAR>(m, wm, a, grid, s);
    case KT_IQ3_S: return launch_t<KT_IQ3_S, PHASE, LINEAR>(m, wm, a, grid, s);
  }
  return -1;
}

// phase 1: X [T, K] bf16 gathered by sorted_token; W13 slots [2N, K]; out H [R, N], or with
// linear the raw projection [R, 2N] (no activation)
int kt_launch_gemm_gate_up(int type, const void* x, int64_t T, int K, int N, const void* w13, int table, int n_slots,
                           const int32_t* tiles, const int32_t* n_tiles, const int32_t* sorted_token, void* h,
                           int* status, int grid, cudaStream_t s, int linear, const void* w13_bf16) {
  if (K % 256 || N % 128) return -1;
  if (((uintptr_t)x) & 15) return -1;
  CUtensorMap m, wm;
  memset(&m, 0, sizeof m);
  memset(&wm, 0, sizeof wm);
  KtGemmArgs a{};
  a.w = (const uint8_t*)w13;
  a.table = table;
  a.row_bytes = (int64_t)K / kt_block_info(type).qk * kt_block_info(type).bytes;
  if (w13_bf16) {  // the weights already dequantized to bf16 [n_slots * 2N, K]
    if (((uintptr_t)w13_bf16) & 15 || make_map(&wm, w13_bf16, (int64_t)n_slots * 2 * N, K, 64)) return -2;
    a.raw_group = 1;  // A rows in natural order (the epilogue's row map)
  } else {
    a.raw_group = table ? 0 : make_raw_map(&wm, w13, a.row_bytes, 2 * (int64_t)N, n_slots, type);
  }
  a.x = (const uint16_t*)x;
  a.K = K;
  a.N = N;
  a.K_out = K;
  a.tiles = tiles;
  a.n_tiles = n_tiles;
  a.n_wtiles = N / 128;
  a.sorted_token = sorted_token;
  a.out = (uint16_t*)h;
  a.out_ld = linear ? 2 * (int64_t)N : N;
  a.status = status;
  if (w13_bf16)  // the GGUF type no longer matters: one instance serves every type
    return linear ? launch_t<KT_Q8_0, 1, true, true>(m, wm, a, grid, s) : launch_t<KT_Q8_0, 1, false, true>(m, wm, a, grid, s);
  return linear ? launch_phase<1, true>(type, m, wm, a, grid, s) : launch_phase<1>(type, m, wm, a, grid, s);
}

// phase 2: H [R, N] bf16 (sorted rows); W2 slots [K, N]; out Y [R, K]
int kt_launch_gemm_down(int type, const void* h, int64_t R, int K, int N, const void* w2, int table, int n_slots,
                        const int32_t* tiles, const int32_t* n_tiles, const int32_t* chunks, void* y, int* status,
                        int grid, cudaStream_t s, const void* w2_bf16) {
  if (N % 256 || K % 256) return -1;
  CUtensorMap m, wm;
  memset(&wm, 0, sizeof wm);
  if (make_map(&m, h, R, N, kHalfN)) return -2;
  if (w2_bf16) {
    // the down weights already dequantized to bf16 [n_slots * K, N]: A rows by two 2-D TMA loads
    // per k-step, no producers; one instance for every GGUF type
    if (((uintptr_t)w2_bf16) & 15 || make_map(&wm, w2_bf16, (int64_t)n_slots * K, N, 64)) return -2;
    KtGemmArgs a{};
    a.w = (const uint8_t*)w2_bf16;
    a.raw_group = 1;  // A rows in natural order (the epilogue's row map)
    a.K = N;          // reduction length
    a.N = N;
    a.K_out = K;      // rows of W2
    a.tiles = tiles;
    a.n_tiles = n_tiles;
    a.chunks = chunks;
    a.n_wtiles = K / 256;
    a.out = (uint16_t*)y;
    a.out_ld = K;
    a.status = status;
    return launch_t<KT_Q8_0, 2, false, true>(m, wm, a, grid, s);
  }
  // reductions of up to kResSlices k-steps keep the dequantized weight strip resident
  const bool res = N / 64 <= kResSlices && getenv("KT_B200_DOWN_STREAM") == nullptr;
  KtGemmArgs a{};
  a.w = (const uint8_t*)w2;
  a.table = table;
  a.row_bytes = (int64_t)N / kt_block_info(type).qk * kt_block_info(type).bytes;
  a.raw_group = table ? 0 : make_raw_map(&wm, w2, a.row_bytes, (int64_t)K, n_slots, type, res);
  a.K = N;  // reduction length
  a.N = N;
  a.K_out = K;  // rows of W2
  a.tiles = tiles;
  a.n_tiles = n_tiles;
  a.chunks = chunks;
  a.n_wtiles = K / 256;
  a.sorted_token = nullptr;
  a.out = (uint16_t*)y;
  a.out_ld = K;
  a.status = status;
  if (res) {
    switch (type) {
      case KT_Q8_0: return launch_res<KT_Q8_0>(m, wm, a, grid, s);
      case KT_Q4_K: return launch_res<KT_Q4_K>(m, wm, a, grid, s);
      case KT_Q6_K: return launch_res<KT_Q6_K>(m, wm, a, grid, s);
      case KT_IQ3_S: return launch_res<KT_IQ3_S>(m, wm, a, grid, s);
    }
    return -1;
  }
  return launch_phase<2>(type, m, wm, a, grid, s);
}

// ------------------------------------------------------------------ self-test of the failure path
//
// One CTA pair that takes the GEMM kernels' set-up and exit path around a wait that cannot end:
// both CTAs allocate the pair's TMEM, one warp per CTA waits on a local barrier and one on the
// same barrier through the cluster-variant wait, and nothing ever arrives on it. The waits give
// up after limit_ns, record KT_DEV_TIMEOUT in *status and raise the CTA's abort flag; the CTA
// then drains as the GEMMs do after a timeout, meets its peer at the cluster barrier and frees
// TMEM. No copy or MMA is issued, so nothing is in flight when the kernel ends.
__global__ void __launch_bounds__(96, 1) kt_selftest_wait_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    kt_mbar_init(&bar, 1);  // one arrival expected, none made
    *abort_flag = 0;
    kt_fence_mbar_init();
  }
  kt_cluster_sync();
  if (warp == 0) kt_tmem_alloc2(&tmem_slot, 512);
  kt_tc_fence_before();
  __syncthreads();
  kt_tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (lane == 0) {
    if (warp == 1) kt_mbar_wait_for(&bar, 0, status, abort_flag, limit_ns);
    if (warp == 2) kt_mbar_wait_cluster_for(&bar, 0, status, abort_flag, limit_ns);
  }
  __syncwarp();
  kt_tc_fence_before();
  __syncthreads();
  if (*abort_flag) kt_drain_ns(200000);
  kt_cluster_sync();
  if (warp == 0) {
    kt_tc_fence_after();
    kt_tmem_dealloc2(tmem, 512);
  }
}

int kt_launch_selftest_wait(int* status, uint64_t limit_ns, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(96, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kt_selftest_wait_kernel, status, limit_ns) != cudaSuccess) return -4;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int kt_gemm_tile_tokens() { return kTN; }
int kt_gemm_chunk_tiles() { return kResChunk; }
