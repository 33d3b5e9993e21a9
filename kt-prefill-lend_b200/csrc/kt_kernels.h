// kt_kernels.h — internal launcher declarations shared by the .cu files of the library.
// The public C ABI is include/kt_gguf_b200.h; nothing here is exported.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

struct KtGemmArgs {
  const uint8_t* w;             // slot base (plain layout) or int64 table of per-slot addresses
  int table;
  int raw_group;                // rows per raw tensor-map row (1, 2, 4, 8); 0: per-row bulk copies
  const uint16_t* x;            // phase 1: bf16 activations [T, K], gathered by sorted_token
  int64_t row_bytes;            // bytes of one GGUF weight row
  int K;                        // reduction length of this phase
  int N;                        // expert intermediate size
  int K_out;                    // rows of W2 (hidden size); phase 1: unused
  const int32_t* tiles;         // [n_tiles][3]: slot, first sorted position, tokens (<= 256)
  const int32_t* n_tiles;       // device scalars: tiles, resident routes, chunks
  const int32_t* chunks;        // [n_chunks][3]: slot, first sorted row, rows (down projection, resident A)
  int n_wtiles;                 // weight tiles per token tile
  const int32_t* sorted_token;  // token of each sorted position (phase 1)
  uint16_t* out;                // bf16 output rows (H or Y), row = sorted position
  int64_t out_ld;
  int* status;                  // device status word
};

// whether the prefill layer's kernels are launched with programmatic stream serialization
// (KT_B200_PDL=0: plain stream order, for comparison runs)
bool kt_pdl_enabled();

// launch with programmatic stream serialization (the kernel calls kt_pdl_wait before it reads
// what the previous kernel of the stream wrote); 0 on success
template <typename... KArgs, typename... Args>
inline int kt_launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t s,
                         Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(block, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = kt_pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) == cudaSuccess ? 0 : -4;
}

int kt_launch_quantize_q8_1(const void* x, int dtype, int64_t rows, int64_t cols, void* qx, cudaStream_t s);
// the GEMV runs its member-stationary kernel for this type, width and route count (routes grouped
// in pieces of kt_vec_ms_piece(); kt_launch_moe_vec then takes max_groups = routes)
bool kt_vec_ms_ok(int type, int cols, int64_t routes);
int kt_vec_ms_piece();
// q8_1 quantization in the GEMV's split layout (a row's int8 values, then its half2 (d, s) per
// block) and route grouping in one launch; also resets *status
int kt_launch_quantize_group(const void* x, int dtype, int64_t rows, int64_t cols, void* qx, const int32_t* ids,
                             int64_t routes, int n_slots, int piece, int32_t* groups, int32_t* order, int* status,
                             cudaStream_t s);
// the decode GEMV in one launch for at most 40 routes (quantization fused, one CTA per route and
// tile of 8, 16 or 32 rows); kt_vec_fused_ok says whether a call qualifies
bool kt_vec_fused_ok(int type, const void* w, int table, const void* x, int64_t routes, int rows, int cols);
int kt_launch_moe_vec_fused(int type, const void* w, int table, int n_slots, const void* x, int dtype,
                            const int32_t* ids, int64_t routes, int top_k, int rows, int cols, void* y, int* status,
                            cudaStream_t s);
int kt_launch_moe_vec(int type, const void* w, int table, const void* qx, int64_t qrow, const int32_t* groups,
                      const int32_t* order, int max_groups, int top_k, int rows, int cols, int dtype, void* y,
                      int* status, cudaStream_t s);

// status (optional): the workspace status word for the bounded waits of the pipelined pass
int kt_launch_dequant(int type, const void* w, int64_t rows, int64_t cols, void* out, int out_dtype, cudaStream_t s,
                      int* status = nullptr);
int kt_launch_silu_and_mul(const void* h13, int dtype, int64_t rows, int64_t n, void* h, cudaStream_t s);
int kt_launch_combine(const void* out, int dtype, const float* w, int64_t T, int64_t top_k, int64_t K, void* res,
                      cudaStream_t s);
// acc_flags bit 0: start each token's sum from acc (fp32 [T, K]); bit 1: write the fp32 sum to
// acc instead of bf16 to res (tokens with no present route are then skipped)
// tokens_dev (optional): the number of tokens, read on the device (T is then a capacity; tokens
// at or past *tokens_dev are not written)
int kt_launch_combine_sorted(const uint16_t* y, const int32_t* route_pos, const float* w, int64_t T, int64_t top_k,
                             int64_t K, uint16_t* res, cudaStream_t s, float* acc = nullptr, int acc_flags = 0,
                             const int32_t* tokens_dev = nullptr);
// dst[i] = src[idx[i]] (rows of `cols` bf16, 16-byte aligned) for i < n, zero rows where
// idx[i] < 0; with n_limit, rows i >= *n_limit (a device count) are left untouched
int kt_launch_gather_rows(const uint16_t* src, int64_t cols, const int32_t* idx, int64_t n, const int32_t* n_limit,
                          uint16_t* dst, cudaStream_t s);
int kt_launch_route(const int32_t* ids, int64_t n, const int32_t* slot_tab, const int32_t* cpu_tab, float* counts,
                    int32_t* slot_out, int32_t* cpu_out, cudaStream_t s);
int kt_launch_topk_softmax(const float* logits, int64_t T, int E, int k, int renorm, float* weights, int32_t* ids,
                           cudaStream_t s);
int kt_launch_topk_grouped(const float* logits, const float* bias, int64_t T, int E, int n_group, int topk_group, int k,
                           int renorm, float scale, float* weights, int32_t* ids, cudaStream_t s);

// prefill permutation: routes sorted by slot, token tiles of kt_gemm_tile_tokens() rows;
// hist holds kt_permute_hist_ints() ints; n_tiles[0] = tiles, n_tiles[1] = resident routes,
// n_tiles[2] = chunks: runs of at most chunk_tiles consecutive tiles of one slot, as
// chunks[3c..3c+2] = slot, first sorted row, rows (capacity: that of the tile list)
constexpr int kPermMaxSlots = 8192;
int64_t kt_permute_hist_ints(int64_t routes, int n_slots);
// ids outside [id_base, id_base + n_slots) (and negative ids) are not present; slot = id - id_base
// tokens_dev (optional): routes at or past *tokens_dev * top_k are not present
int kt_launch_permute(const int32_t* ids, int64_t routes, int top_k, int n_slots, int tile_tokens, int chunk_tiles,
                      int32_t* counts, int32_t* hist, int32_t* tiles, int32_t* n_tiles, int32_t* chunks,
                      int32_t* sorted_token, int32_t* route_pos, cudaStream_t s, int id_base = 0,
                      const int32_t* tokens_dev = nullptr);

// linear = 1: no activation, the raw projection [R, 2N] (rows of w13 in order) instead of H [R, N];
// w13_bf16: the slots' weights already dequantized to bf16 [n_slots * 2N, K] (A tiles by TMA, no
// in-kernel dequantization), or null
int kt_launch_gemm_gate_up(int type, const void* x, int64_t T, int K, int N, const void* w13, int table, int n_slots,
                           const int32_t* tiles, const int32_t* n_tiles, const int32_t* sorted_token, void* h,
                           int* status, int grid, cudaStream_t s, int linear = 0, const void* w13_bf16 = nullptr);
// w2_bf16: the slots' down weights already dequantized to bf16 [n_slots * K, N] (A tiles by TMA, the
// streaming kernel's instance without producers), or null
int kt_launch_gemm_down(int type, const void* h, int64_t R, int K, int N, const void* w2, int table, int n_slots,
                        const int32_t* tiles, const int32_t* n_tiles, const int32_t* chunks, void* y, int* status,
                        int grid, cudaStream_t s, const void* w2_bf16 = nullptr);
int kt_gemm_tile_tokens();
// the GEMM kernels' bounded-wait and exit path around a barrier nothing arrives on (one CTA
// pair); writes KT_DEV_TIMEOUT to *status after limit_ns
int kt_launch_selftest_wait(int* status, uint64_t limit_ns, cudaStream_t s);
int kt_gemm_chunk_tiles();  // tiles per chunk of the down projection's work units

// expert-parallel plumbing (ep.cu): dispatch plan, row packing, combine of partials (bf16 rows)
int64_t kt_ep_plan_ints(int64_t T, int P);
int kt_launch_ep_plan(const int32_t* ids, const float* w, int64_t T, int k, const int32_t* owner, const int32_t* local,
                      int n_experts, int P, int32_t* block_scratch, int32_t* counts, int32_t* send_token, int32_t* meta,
                      int32_t* row_of, cudaStream_t s);
int kt_launch_ep_pack(const void* x, int64_t K, const int32_t* send_token, int64_t n, void* rows, cudaStream_t s);
int kt_launch_ep_combine(const void* back, const int32_t* row_of, int P, const void* shared, int64_t T, int64_t K,
                         void* out, cudaStream_t s);
// the exchange over peer memory: peer_* are device arrays of P addresses (this rank's own
// buffers at index me), counts_all [P][P] every rank's plan counts
int kt_launch_ep_dispatch_p2p(const void* x, int64_t K, const int32_t* send_token, const int32_t* meta, int k,
                              const int32_t* counts_all, int me, int P, const int64_t* peer_x, const int64_t* peer_ids,
                              const int64_t* peer_w, int64_t rows_cap, int32_t* recv_total, cudaStream_t s);
int kt_launch_ep_combine_p2p(const int32_t* row_of, const int32_t* counts_all, int me, int P, const int64_t* peer_y,
                             const void* shared, int64_t T, int64_t K, void* out, cudaStream_t s);
