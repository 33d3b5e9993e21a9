// kt_common.cuh — shared device helpers for the B200 GGUF hot-expert MoE kernels.
//
// GGUF block layouts (byte offsets) of the four hot-path types, bf16 helpers, and thin
// inline-PTX wrappers for mbarriers, bulk/tensor copies and tcgen05 (TMEM allocation,
// MMA, commit, loads). Every spin on an mbarrier is bounded: after KT_WAIT_NS of wall time it
// records an error code in the caller-provided status word and returns false, so a lost
// arrival ends the kernel with an error instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "iq3s_grid.h"
#include "iquant_grids.h"

// the i-quant code books in global memory; kernels copy their type's book to shared memory
// before use (kt_stage_grid)
static __device__ const uint32_t kt_iq3s_grid_dev[512] = KT_IQ3S_GRID_INIT;
static __device__ const uint32_t kt_iq2xxs_grid_dev[KT_IQ2XXS_GRID_WORDS] = KT_IQ2XXS_GRID_INIT;
static __device__ const uint32_t kt_iq2xs_grid_dev[KT_IQ2XS_GRID_WORDS] = KT_IQ2XS_GRID_INIT;
static __device__ const uint32_t kt_iq2s_grid_dev[KT_IQ2S_GRID_WORDS] = KT_IQ2S_GRID_INIT;
static __device__ const uint32_t kt_iq3xxs_grid_dev[KT_IQ3XXS_GRID_WORDS] = KT_IQ3XXS_GRID_INIT;
static __device__ const uint32_t kt_iq1s_grid_dev[KT_IQ1S_GRID_WORDS] = KT_IQ1S_GRID_INIT;

#define KT_Q4_0 2
#define KT_Q4_1 3
#define KT_Q5_0 6
#define KT_Q5_1 7
#define KT_Q8_0 8
#define KT_Q2_K 10
#define KT_Q3_K 11
#define KT_Q4_K 12
#define KT_Q5_K 13
#define KT_Q6_K 14
#define KT_IQ4_NL 20
#define KT_IQ3_S 21
#define KT_IQ4_XS 23
#define KT_IQ2_XXS 16
#define KT_IQ2_XS 17
#define KT_IQ3_XXS 18
#define KT_IQ1_S 19
#define KT_IQ2_S 22
#define KT_IQ1_M 29
#define KT_Q2_0 42  // 64-value blocks: fp16 d, 2-bit codes, value d*(code-1)

// activation / output dtype codes of the C ABI
#define KT_DT_F32 0
#define KT_DT_F16 1
#define KT_DT_BF16 2

// device status word values (written by kernels, read by the host after a call)
#define KT_DEV_OK 0
#define KT_DEV_TIMEOUT 1
#define KT_DEV_BAD_INPUT 2

#ifndef KT_WAIT_NS
#define KT_WAIT_NS 2000000000ull  // 2 s: far above any legitimate wait inside one kernel
#endif

struct KtBlockInfo {
  int qk;     // values per block
  int bytes;  // bytes per block
};

__host__ __device__ constexpr KtBlockInfo kt_block_info(int type) {
  return type == KT_Q8_0     ? KtBlockInfo{32, 34}
         : type == KT_Q4_0   ? KtBlockInfo{32, 18}
         : type == KT_Q4_1   ? KtBlockInfo{32, 20}
         : type == KT_Q5_0   ? KtBlockInfo{32, 22}
         : type == KT_Q5_1   ? KtBlockInfo{32, 24}
         : type == KT_IQ4_NL ? KtBlockInfo{32, 18}
         : type == KT_Q2_K   ? KtBlockInfo{256, 84}
         : type == KT_Q3_K   ? KtBlockInfo{256, 110}
         : type == KT_Q5_K   ? KtBlockInfo{256, 176}
         : type == KT_IQ4_XS ? KtBlockInfo{256, 136}
         : type == KT_Q2_0   ? KtBlockInfo{64, 18}
         : type == KT_IQ2_XXS ? KtBlockInfo{256, 66}
         : type == KT_IQ2_XS ? KtBlockInfo{256, 74}
         : type == KT_IQ3_XXS ? KtBlockInfo{256, 98}
         : type == KT_IQ1_S  ? KtBlockInfo{256, 50}
         : type == KT_IQ2_S  ? KtBlockInfo{256, 82}
         : type == KT_IQ1_M  ? KtBlockInfo{256, 56}
         : type == KT_Q4_K   ? KtBlockInfo{256, 144}
         : type == KT_Q6_K ? KtBlockInfo{256, 210}
         : type == KT_IQ3_S ? KtBlockInfo{256, 110}
                            : KtBlockInfo{0, 0};
}

// q8_1 activation blocks: half d, half s (sum of the unquantized values), 32 x int8
#define KT_Q8_1_BYTES 36
__host__ __device__ inline int64_t kt_q8_1_row_bytes(int64_t cols) { return (cols + 511) / 512 * 512 / 32 * KT_Q8_1_BYTES; }

__device__ __forceinline__ float kt_h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ float kt_bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t kt_f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ uint32_t kt_pack_bf2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int DT>
__device__ __forceinline__ float kt_load_act(const void* p, int64_t i) {
  if constexpr (DT == KT_DT_F32) return reinterpret_cast<const float*>(p)[i];
  if constexpr (DT == KT_DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

template <int DT>
__device__ __forceinline__ void kt_store_act(void* p, int64_t i, float v) {
  if constexpr (DT == KT_DT_F32) reinterpret_cast<float*>(p)[i] = v;
  else if constexpr (DT == KT_DT_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// 32-bit little-endian word from a 2-byte aligned address (GGUF blocks of 34, 110 and
// 210 bytes leave 4-byte words only 2-byte aligned)
__device__ __forceinline__ int kt_ld_b2(const uint8_t* p) {
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return (int)((uint32_t)q[0] | ((uint32_t)q[1] << 16));
}
__device__ __forceinline__ int kt_ld_b4(const uint8_t* p) { return *reinterpret_cast<const int*>(p); }
// the decode GEMV's types (prefill GEMM: Q8_0, Q4_K, Q6_K, IQ3_S only)
__host__ __device__ constexpr bool kt_gemv_type(int t) {
  return t == KT_Q4_0 || t == KT_Q4_1 || t == KT_Q5_0 || t == KT_Q5_1 || t == KT_Q8_0 || t == KT_IQ4_NL ||
         t == KT_Q2_K || t == KT_Q3_K || t == KT_Q4_K || t == KT_Q5_K || t == KT_Q6_K || t == KT_IQ3_S ||
         t == KT_IQ4_XS || t == KT_Q2_0 || t == KT_IQ2_XXS || t == KT_IQ2_XS || t == KT_IQ3_XXS || t == KT_IQ1_S ||
         t == KT_IQ2_S || t == KT_IQ1_M;
}
// words of the code book a type's kernels stage in shared memory (0: none)
__host__ __device__ constexpr int kt_grid_words(int t) {
  return t == KT_IQ3_S     ? 512
         : t == KT_IQ2_XXS ? KT_IQ2XXS_GRID_WORDS
         : t == KT_IQ2_XS  ? KT_IQ2XS_GRID_WORDS
         : t == KT_IQ2_S   ? KT_IQ2S_GRID_WORDS
         : t == KT_IQ3_XXS ? KT_IQ3XXS_GRID_WORDS
         : (t == KT_IQ1_S || t == KT_IQ1_M) ? KT_IQ1S_GRID_WORDS
                                            : 0;
}
// size of a static shared array holding TYPE's code book (one word for types without one)
template <int TYPE>
struct KtGridSmem {
  static constexpr int WORDS = kt_grid_words(TYPE) > 0 ? kt_grid_words(TYPE) : 1;
};
// copies TYPE's code book into shared memory (nothing for types without one); the caller
// synchronises before the first read
template <int TYPE>
__device__ __forceinline__ void kt_stage_grid(uint32_t* dst, int tid, int nthreads) {
  constexpr int W = kt_grid_words(TYPE);
  if constexpr (W > 0) {
    const uint32_t* src = TYPE == KT_IQ3_S     ? kt_iq3s_grid_dev
                          : TYPE == KT_IQ2_XXS ? kt_iq2xxs_grid_dev
                          : TYPE == KT_IQ2_XS  ? kt_iq2xs_grid_dev
                          : TYPE == KT_IQ2_S   ? kt_iq2s_grid_dev
                          : TYPE == KT_IQ3_XXS ? kt_iq3xxs_grid_dev
                                               : kt_iq1s_grid_dev;
    for (int i = tid; i < W; i += nthreads) dst[i] = src[i];
  }
}
__host__ __device__ constexpr bool kt_prefill_type(int t) {
  return t == KT_Q8_0 || t == KT_Q4_K || t == KT_Q6_K || t == KT_IQ3_S;
}

__device__ __forceinline__ uint32_t kt_smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void kt_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(kt_smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void kt_fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void kt_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(kt_smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void kt_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(kt_smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool kt_mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(kt_smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t kt_globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after limit_ns of wall time (global timer), records KT_DEV_TIMEOUT
// in *status (global) and sets *abort (shared) so the CTA's other roles leave their loops
// too; returns false then. A wait also returns false once *abort is set. The kernels use
// kt_mbar_wait (limit KT_WAIT_NS); the library's self-test of this path passes a short limit.
__device__ __forceinline__ bool kt_mbar_wait_for(uint64_t* bar, uint32_t parity, int* status, volatile int* abort,
                                                 uint64_t limit_ns) {
  if (kt_mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = kt_globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (kt_mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if ((i & 255) == 0 && kt_globaltimer_ns() - t0 > limit_ns) break;
  }
  if (status) atomicExch(status, KT_DEV_TIMEOUT);
  if (abort) *abort = 1;
  return false;
}
__device__ __forceinline__ bool kt_mbar_wait(uint64_t* bar, uint32_t parity, int* status, volatile int* abort) {
  return kt_mbar_wait_for(bar, parity, status, abort, KT_WAIT_NS);
}

// spin for `ns` nanoseconds of wall time (the global timer), bounded by construction
__device__ __forceinline__ void kt_drain_ns(uint64_t ns) {
  const uint64_t t0 = kt_globaltimer_ns();
  while (kt_globaltimer_ns() - t0 < ns) {
  }
}

// ------------------------------------------------------------------ programmatic dependent launch
// The prefill layer's kernels are launched with programmatic stream serialization: a kernel may
// start (and run its prologue: barriers, TMEM, code books) while the previous kernel of the
// stream is still finishing, and waits here before it reads anything that kernel wrote.
// kt_pdl_trigger lets the next kernel of the stream launch early; both are no-ops for a kernel
// launched without the attribute or with no dependent.
__device__ __forceinline__ void kt_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void kt_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ clusters (CTA pairs)

__device__ __forceinline__ uint32_t kt_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t kt_mapa(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(kt_smem_addr(p)), "r"(rank));
  return r;
}
// arrive on an mbarrier of either CTA of the pair, given by its shared::cluster address.
// Default semantics (release at CTA scope), as CUTLASS's cluster barrier uses for peer
// arrivals: what an arrival publishes is shared memory of the arriving CTA that the arriving
// thread has already observed complete (it acquired the local barrier guarding it). A
// release at cluster scope makes every such arrival wait for a cluster-wide fence; on the
// pair's stage-forwarding path that fence cost more than an MMA k-step.
__device__ __forceinline__ void kt_mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool kt_mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(kt_smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait on a barrier that also receives arrivals from the peer CTA
__device__ __forceinline__ bool kt_mbar_wait_cluster_for(uint64_t* bar, uint32_t parity, int* status,
                                                         volatile int* abort, uint64_t limit_ns) {
  if (kt_mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = kt_globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (kt_mbar_try_wait_cluster(bar, parity)) return true;
    if (abort && *abort) return false;
    if ((i & 255) == 0 && kt_globaltimer_ns() - t0 > limit_ns) break;
  }
  if (status) atomicExch(status, KT_DEV_TIMEOUT);
  if (abort) *abort = 1;
  return false;
}
__device__ __forceinline__ bool kt_mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status, volatile int* abort) {
  return kt_mbar_wait_cluster_for(bar, parity, status, abort, KT_WAIT_NS);
}
__device__ __forceinline__ void kt_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ------------------------------------------------------------------ bulk / tensor copies

__device__ __forceinline__ void kt_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   kt_smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(kt_smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void kt_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          kt_smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(kt_smem_addr(bar))
      : "memory");
}

// 16-byte global -> shared copy through L2 (cp.async.cg); completion is tracked by
// kt_cp_async_arrive on an mbarrier
__device__ __forceinline__ void kt_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(kt_smem_addr(dst)), "l"(src) : "memory");
}
// arrive on the mbarrier once all of this thread's earlier cp.async copies have landed; the
// arrival counts against the barrier's expected count (noinc)
__device__ __forceinline__ void kt_cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(kt_smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void kt_fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05

// CTA-pair (cta_group::2) forms: allocation and release are executed by the same warp of
// both CTAs; MMAs are issued by the even CTA and read A and B halves from both CTAs' shared
// memory; commits arrive on the barrier at the same offset in every CTA of `mask`.
__device__ __forceinline__ void kt_tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(kt_smem_addr(dst_smem)), "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void kt_tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void kt_mma2_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void kt_mma2_commit_mc(uint64_t* bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   kt_smem_addr(bar)),
               "h"(mask)
               : "memory");
}

__device__ __forceinline__ void kt_tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void kt_tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns starting at taddr (lane field = warp's quadrant)
__device__ __forceinline__ void kt_tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void kt_tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major bf16 tile stored in the 128-byte swizzle
// layout: rows of 128 bytes (64 elements), 8-row groups 1024 bytes apart, tile base
// 1024-byte aligned. Bits: [0,14) address>>4, [16,30) leading offset>>4 (unused for
// swizzled K-major), [32,46) stride offset>>4, [46,48) version 1, [61,64) layout 2 = 128B.
__device__ __forceinline__ uint64_t kt_desc_k128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: D f32, A and B bf16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t kt_idesc_bf16(int M, int N) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A format bf16
         | (1u << 10)                   // B format bf16
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// byte offset of element (row, k) in a K-major 128B-swizzled tile (64 bf16 per row)
__device__ __forceinline__ uint32_t kt_swz128(int row, int k) {
  const uint32_t chunk = (uint32_t)(k >> 3) ^ (uint32_t)(row & 7);
  return (uint32_t)row * 128u + chunk * 16u + (uint32_t)(k & 7) * 2u;
}
