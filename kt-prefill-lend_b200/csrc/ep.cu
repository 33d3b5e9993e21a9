// ep.cu — expert-parallel plumbing around the NCCL all-to-all: the dispatch plan, the row
// packing and the combine of the partial outputs, as three small kernels so that a layer
// call needs no sort, no nonzero and no index arithmetic in PyTorch.
//
// Plan (for P <= 8 ranks): route (t, j) with logical expert e = ids[t, j] >= 0 goes to rank
// owner[e] (< 0: no rank, dropped) as local slot local[e]. A token is sent once to every rank
// that owns at least one of its experts. Send rows are grouped by destination rank, tokens
// ascending within a rank (deterministic). Outputs:
//   counts[r]          rows for rank r
//   send_token[row]    source token of each send row
//   meta[row][2k]      the row's k local slots (int32, -1 where the expert is on another
//                      rank or nowhere), then its k weights (fp32 bits, 0 where the slot is -1)
//   row_of[t][r]       send row of token t for rank r, or -1 (used by the combine)
// Two passes over blocks of kEpBlock tokens: per-block counts per rank, then (after one scan
// block) the rows, each token's rank-r row at base(r) + rows of rank r in earlier blocks +
// rows of rank r for earlier tokens of the same block.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace {

constexpr int kEpBlock = 256;
constexpr int kEpMaxRanks = 8;

__device__ __forceinline__ uint32_t kt_ep_mask(const int32_t* ids, int k, const int32_t* owner, int n_experts) {
  uint32_t m = 0;
  for (int j = 0; j < k; ++j) {
    const int32_t e = ids[j];
    if (e >= 0 && e < n_experts) {
      const int32_t r = owner[e];
      if (r >= 0 && r < kEpMaxRanks) m |= 1u << r;
    }
  }
  return m;
}

// per block and rank: tokens of the block sent to the rank (warp ballots, shared counters)
__global__ void __launch_bounds__(kEpBlock) kt_ep_count_kernel(const int32_t* __restrict__ ids, int64_t T, int k,
                                                               const int32_t* __restrict__ owner, int n_experts,
                                                               int P, int32_t* __restrict__ block_counts) {
  __shared__ int32_t cnt[kEpMaxRanks];
  if (threadIdx.x < kEpMaxRanks) cnt[threadIdx.x] = 0;
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * kEpBlock + threadIdx.x;
  const uint32_t m = t < T ? kt_ep_mask(ids + t * k, k, owner, n_experts) : 0u;
  const int lane = threadIdx.x & 31;
  for (int r = 0; r < P; ++r) {
    const uint32_t b = __ballot_sync(0xffffffffu, (m >> r) & 1u);
    if (lane == 0 && b) atomicAdd(&cnt[r], __popc(b));
  }
  __syncthreads();
  if (threadIdx.x < P) block_counts[(int64_t)blockIdx.x * P + threadIdx.x] = cnt[threadIdx.x];
}

// one block: block_counts[b][r] -> first row of block b for rank r; counts[r]
__global__ void kt_ep_scan_kernel(int32_t* __restrict__ block_counts, int n_blocks, int P,
                                  int32_t* __restrict__ counts) {
  __shared__ int32_t tot[kEpMaxRanks];
  const int r = threadIdx.x;
  if (r < P) {
    int32_t run = 0;
    for (int b = 0; b < n_blocks; ++b) {
      const int32_t c = block_counts[(int64_t)b * P + r];
      block_counts[(int64_t)b * P + r] = run;
      run += c;
    }
    tot[r] = run;
    counts[r] = run;
  }
  __syncthreads();
  if (r < P) {
    int32_t base = 0;
    for (int q = 0; q < r; ++q) base += tot[q];
    for (int b = 0; b < n_blocks; ++b) block_counts[(int64_t)b * P + r] += base;
  }
}

__global__ void __launch_bounds__(kEpBlock) kt_ep_rows_kernel(const int32_t* __restrict__ ids,
                                                              const float* __restrict__ w, int64_t T, int k,
                                                              const int32_t* __restrict__ owner,
                                                              const int32_t* __restrict__ local, int n_experts, int P,
                                                              const int32_t* __restrict__ block_first,
                                                              int32_t* __restrict__ send_token,
                                                              int32_t* __restrict__ meta, int32_t* __restrict__ row_of) {
  __shared__ int32_t warp_cnt[kEpBlock / 32][kEpMaxRanks];
  const int64_t t = (int64_t)blockIdx.x * kEpBlock + threadIdx.x;
  const uint32_t m = t < T ? kt_ep_mask(ids + t * k, k, owner, n_experts) : 0u;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint32_t below[kEpMaxRanks];
#pragma unroll
  for (int r = 0; r < kEpMaxRanks; ++r) {
    below[r] = 0;
    if (r < P) {
      const uint32_t b = __ballot_sync(0xffffffffu, (m >> r) & 1u);
      below[r] = __popc(b & ((1u << lane) - 1u));
      if (lane == 0) warp_cnt[wid][r] = __popc(b);
    }
  }
  __syncthreads();
  if (t >= T) return;
#pragma unroll
  for (int r = 0; r < kEpMaxRanks; ++r) {
    if (r >= P) break;
    int32_t row = -1;
    if ((m >> r) & 1u) {
      int32_t pre = 0;
      for (int q = 0; q < wid; ++q) pre += warp_cnt[q][r];
      row = block_first[(int64_t)blockIdx.x * P + r] + pre + (int32_t)below[r];
      send_token[row] = (int32_t)t;
      int32_t* mr = meta + (int64_t)row * 2 * k;
      for (int j = 0; j < k; ++j) {
        const int32_t e = ids[t * k + j];
        const bool here = e >= 0 && e < n_experts && owner[e] == r;
        mr[j] = here ? local[e] : -1;
        mr[k + j] = __float_as_int(here ? w[t * k + j] : 0.0f);
      }
    }
    row_of[t * P + r] = row;
  }
}

// rows[i] = x[send_token[i]] for i < n: one warp per row, 16-byte copies
__global__ void kt_ep_pack_kernel(const uint16_t* __restrict__ x, int64_t K, const int32_t* __restrict__ send_token,
                                  int64_t n, uint16_t* __restrict__ rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t chunks = K / 8;
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; i < n; i += warps) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)send_token[i] * K);
    uint4* dst = reinterpret_cast<uint4*>(rows + i * K);
    for (int64_t c = lane; c < chunks; c += 32) dst[c] = __ldg(src + c);
  }
}

// out[t] = bf16(shared[t] + sum over r in rank order of back[row_of[t][r]]), fp32 sums; one
// block per token, 8 columns per thread
__global__ void kt_ep_combine_kernel(const uint16_t* __restrict__ back, const int32_t* __restrict__ row_of, int P,
                                     const uint16_t* __restrict__ shared, int64_t K, uint16_t* __restrict__ out) {
  const int64_t t = blockIdx.x;
  int32_t rows[kEpMaxRanks];
  for (int r = 0; r < kEpMaxRanks; ++r) rows[r] = r < P ? row_of[t * P + r] : -1;
  for (int64_t c = (int64_t)threadIdx.x * 8; c < K; c += (int64_t)blockDim.x * 8) {
    float acc[8];
    if (shared) {
      const uint4 v = *reinterpret_cast<const uint4*>(shared + t * K + c);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = kt_bf2f((uint16_t)(u[j] & 0xffff));
        acc[2 * j + 1] = kt_bf2f((uint16_t)(u[j] >> 16));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    }
#pragma unroll
    for (int r = 0; r < kEpMaxRanks; ++r) {
      if (rows[r] < 0) continue;
      const uint4 v = __ldcs(reinterpret_cast<const uint4*>(back + (int64_t)rows[r] * K + c));
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += kt_bf2f((uint16_t)(u[j] & 0xffff));
        acc[2 * j + 1] += kt_bf2f((uint16_t)(u[j] >> 16));
      }
    }
    uint4 o;
    o.x = kt_pack_bf2(acc[0], acc[1]);
    o.y = kt_pack_bf2(acc[2], acc[3]);
    o.z = kt_pack_bf2(acc[4], acc[5]);
    o.w = kt_pack_bf2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * K + c) = o;
  }
}

// ---- exchange over peer memory (rows written into, and partials read from, the other ranks'
// buffers mapped into this process by CUDA IPC)
//
// counts_all [P][P]: counts_all[s][d] = rows rank s sends to rank d (every rank's plan counts,
// gathered). Rank s's rows for rank d land in d's receive buffers at rows
// base(s, d) + j, base(s, d) = sum over s' < s of counts_all[s'][d], j the row's index within
// s's send segment for d; d's layer writes its output row for receive row i at row i of its y.

struct KtEpOffsets {
  int32_t seg[kEpMaxRanks + 1];  // this rank's send segment starts (rank-major send rows)
  int32_t base[kEpMaxRanks];     // this rank's first row in each destination's receive buffers
};

__device__ __forceinline__ void kt_ep_offsets(const int32_t* counts_all, int me, int P, KtEpOffsets& o) {
  int32_t run = 0;
  for (int d = 0; d < P; ++d) {
    o.seg[d] = run;
    run += counts_all[me * P + d];
    int32_t b = 0;
    for (int s2 = 0; s2 < me; ++s2) b += counts_all[s2 * P + d];
    o.base[d] = b;
  }
  o.seg[P] = run;
}

// one warp per send row: the token's K bf16 values, then the row's k slot ids and k weights,
// stored into the destination rank's buffers (16-byte stores, over NVLink for other ranks)
__global__ void __launch_bounds__(256) kt_ep_dispatch_p2p_kernel(
    const uint16_t* __restrict__ x, int64_t K, const int32_t* __restrict__ send_token,
    const int32_t* __restrict__ meta, int k, const int32_t* __restrict__ counts_all, int me, int P,
    const int64_t* __restrict__ peer_x, const int64_t* __restrict__ peer_ids, const int64_t* __restrict__ peer_w,
    int64_t rows_cap, int32_t* __restrict__ recv_total) {
  __shared__ KtEpOffsets o;
  if (threadIdx.x == 0) kt_ep_offsets(counts_all, me, P, o);
  if (blockIdx.x == 0 && threadIdx.x == 1) {  // rows this rank receives (its layer's token count)
    int32_t r = 0;
    for (int s2 = 0; s2 < P; ++s2) r += counts_all[s2 * P + me];
    *recv_total = r;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t n = o.seg[P];
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t chunks = K / 8;
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; i < n; i += warps) {
    int d = 0;
    while (d + 1 < P && i >= o.seg[d + 1]) ++d;
    const int64_t row = (int64_t)o.base[d] + (i - o.seg[d]);
    if (row >= rows_cap) continue;  // cannot happen with buffers of the planned capacity
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)send_token[i] * K);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(peer_x[d]) + row * K);
    // a lane's loads of up to 8 chunks are all in flight before its (remote) stores
    constexpr int U = 8;
    for (int64_t c0 = lane; c0 < chunks; c0 += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (c0 + 32 * u < chunks) v[u] = __ldg(src + c0 + 32 * u);
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (c0 + 32 * u < chunks) dst[c0 + 32 * u] = v[u];
    }
    if (lane < k) {
      reinterpret_cast<int32_t*>(peer_ids[d])[row * k + lane] = meta[i * 2 * k + lane];
      reinterpret_cast<int32_t*>(peer_w[d])[row * k + lane] = meta[i * 2 * k + k + lane];
    }
  }
  __threadfence_system();  // the stores reach the other GPUs before the barrier that follows
}

// out[t] = bf16(shared[t] + sum over ranks d in rank order of d's y row for token t), fp32
// sums; the rows are read from the other ranks' y buffers (one CTA per token, 8 columns a thread)
__global__ void kt_ep_combine_p2p_kernel(const int32_t* __restrict__ row_of, const int32_t* __restrict__ counts_all,
                                         int me, int P, const int64_t* __restrict__ peer_y,
                                         const uint16_t* __restrict__ shared, int64_t K, uint16_t* __restrict__ out) {
  __shared__ KtEpOffsets o;
  if (threadIdx.x == 0) kt_ep_offsets(counts_all, me, P, o);
  __syncthreads();
  const int64_t t = blockIdx.x;
  const uint16_t* src[kEpMaxRanks];
#pragma unroll
  for (int d = 0; d < kEpMaxRanks; ++d) {
    const int32_t r = d < P ? row_of[t * P + d] : -1;
    src[d] = r >= 0 ? reinterpret_cast<const uint16_t*>(peer_y[d]) + ((int64_t)o.base[d] + (r - o.seg[d])) * K
                    : nullptr;
  }
  for (int64_t c = (int64_t)threadIdx.x * 8; c < K; c += (int64_t)blockDim.x * 8) {
    uint4 v[kEpMaxRanks];
#pragma unroll
    for (int d = 0; d < kEpMaxRanks; ++d)  // every rank's load in flight before the sums
      v[d] = src[d] ? __ldcg(reinterpret_cast<const uint4*>(src[d] + c)) : make_uint4(0, 0, 0, 0);
    float acc[8];
    if (shared) {
      const uint4 sv = *reinterpret_cast<const uint4*>(shared + t * K + c);
      const uint32_t u[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = kt_bf2f((uint16_t)(u[j] & 0xffff));
        acc[2 * j + 1] = kt_bf2f((uint16_t)(u[j] >> 16));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    }
#pragma unroll
    for (int d = 0; d < kEpMaxRanks; ++d) {
      if (!src[d]) continue;
      const uint32_t u[4] = {v[d].x, v[d].y, v[d].z, v[d].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += kt_bf2f((uint16_t)(u[j] & 0xffff));
        acc[2 * j + 1] += kt_bf2f((uint16_t)(u[j] >> 16));
      }
    }
    uint4 ov;
    ov.x = kt_pack_bf2(acc[0], acc[1]);
    ov.y = kt_pack_bf2(acc[2], acc[3]);
    ov.z = kt_pack_bf2(acc[4], acc[5]);
    ov.w = kt_pack_bf2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * K + c) = ov;
  }
}

}  // namespace

int kt_launch_ep_dispatch_p2p(const void* x, int64_t K, const int32_t* send_token, const int32_t* meta, int k,
                              const int32_t* counts_all, int me, int P, const int64_t* peer_x, const int64_t* peer_ids,
                              const int64_t* peer_w, int64_t rows_cap, int32_t* recv_total, cudaStream_t s) {
  if (K % 8 || P < 1 || P > kEpMaxRanks || me < 0 || me >= P || k < 1 || k > 32 || (((uintptr_t)x) & 15)) return -1;
  kt_ep_dispatch_p2p_kernel<<<148 * 4, 256, 0, s>>>((const uint16_t*)x, K, send_token, meta, k, counts_all, me, P,
                                                    peer_x, peer_ids, peer_w, rows_cap, recv_total);
  return 0;
}

int kt_launch_ep_combine_p2p(const int32_t* row_of, const int32_t* counts_all, int me, int P, const int64_t* peer_y,
                             const void* shared, int64_t T, int64_t K, void* out, cudaStream_t s) {
  if (K % 8 || P < 1 || P > kEpMaxRanks || me < 0 || me >= P || T > 0x7fffffff) return -1;
  if (T == 0) return 0;
  const int64_t vec = K / 8;
  const int threads = (int)(vec < 256 ? (vec + 31) / 32 * 32 : 256);
  kt_ep_combine_p2p_kernel<<<(unsigned)T, threads, 0, s>>>(row_of, counts_all, me, P, peer_y, (const uint16_t*)shared,
                                                          K, (uint16_t*)out);
  return 0;
}

int64_t kt_ep_plan_ints(int64_t T, int P) { return ((T + kEpBlock - 1) / kEpBlock) * P; }

int kt_launch_ep_plan(const int32_t* ids, const float* w, int64_t T, int k, const int32_t* owner, const int32_t* local,
                      int n_experts, int P, int32_t* block_scratch, int32_t* counts, int32_t* send_token, int32_t* meta,
                      int32_t* row_of, cudaStream_t s) {
  if (P < 1 || P > kEpMaxRanks || k < 1 || T < 0 || n_experts < 1) return -1;
  const int nb = (int)((T + kEpBlock - 1) / kEpBlock);
  if (nb > 0) kt_ep_count_kernel<<<nb, kEpBlock, 0, s>>>(ids, T, k, owner, n_experts, P, block_scratch);
  kt_ep_scan_kernel<<<1, 32, 0, s>>>(block_scratch, nb, P, counts);
  if (nb > 0)
    kt_ep_rows_kernel<<<nb, kEpBlock, 0, s>>>(ids, w, T, k, owner, local, n_experts, P, block_scratch, send_token, meta,
                                              row_of);
  return 0;
}

int kt_launch_ep_pack(const void* x, int64_t K, const int32_t* send_token, int64_t n, void* rows, cudaStream_t s) {
  if (K % 8 || (((uintptr_t)x | (uintptr_t)rows) & 15)) return -1;
  if (n <= 0) return 0;
  const int64_t want = (n + 7) / 8;
  kt_ep_pack_kernel<<<(unsigned)(want < 148 * 16 ? want : 148 * 16), 256, 0, s>>>(
      (const uint16_t*)x, K, send_token, n, (uint16_t*)rows);
  return 0;
}

int kt_launch_ep_combine(const void* back, const int32_t* row_of, int P, const void* shared, int64_t T, int64_t K,
                         void* out, cudaStream_t s) {
  if (K % 8 || P < 1 || P > kEpMaxRanks || T > 0x7fffffff) return -1;
  if (T == 0) return 0;
  const int64_t vec = K / 8;
  const int threads = (int)(vec < 256 ? (vec + 31) / 32 * 32 : 256);
  kt_ep_combine_kernel<<<(unsigned)T, threads, 0, s>>>((const uint16_t*)back, row_of, P, (const uint16_t*)shared, K,
                                                      (uint16_t*)out);
  return 0;
}
