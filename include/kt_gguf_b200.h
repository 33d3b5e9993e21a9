/*
 * kt_gguf_b200.h — C ABI of the B200 (sm_100a) GGUF hot-expert MoE library
 * (libkt_gguf_b200.so).
 *
 * Plain pointers and sizes only: every device pointer is a CUDA device address on the
 * current device, `stream` is a cudaStream_t passed as void*, and nothing here allocates
 * device memory: outputs and scratch ("workspace") come from the caller, sized by the
 * *_workspace_size queries. All calls are asynchronous on `stream` and never synchronize
 * the host, so they can be captured into CUDA graphs.
 *
 * Return value: KT_OK, or a KT_ERR_* code for arguments rejected on the host (nothing is
 * launched then). Kernels that wait on on-chip barriers bound every wait; if one runs out
 * they write KT_DEV_TIMEOUT into the workspace's status word, which kt_workspace_status()
 * reads after the stream has finished.
 *
 * Types (ggml type ids, KT_GGML_* below): the prefill layer takes Q8_0 (8), Q4_K (12),
 * Q6_K (14) and IQ3_S (21). The decode GEMV, the dense GEMV and the dequantizer take those and
 * every other type of the reference kernel's switch (kt_gguf_moe_multi.cu:671-932): the
 * 32-value blocks Q4_0 (2), Q4_1 (3), Q5_0 (6), Q5_1 (7), IQ4_NL (20); the K-quants Q2_K (10),
 * Q3_K (11), Q5_K (13); the i-quants IQ2_XXS (16), IQ2_XS (17), IQ3_XXS (18), IQ1_S (19),
 * IQ2_S (22), IQ4_XS (23), IQ1_M (29); and the reference's own 64-value 2-bit Q2_0 (42)
 * (kt_gguf_moe_multi.cu:33-46). The prefill layer returns KT_ERR_TYPE for the GEMV-only types.
 * Activation dtypes: KT_DTYPE_F32 (0), KT_DTYPE_F16 (1), KT_DTYPE_BF16 (2).
 *
 * Weight layout (as the reference's KTGGUFHotExpertsMethod, hot/kt_gguf_hot.py:17-20):
 *   w13  uint8 [n_slots, 2*inter, row_bytes(hidden)]   rows [gate; up]
 *   w2   uint8 [n_slots, hidden,  row_bytes(inter)]
 * or, with w_is_table = 1, w points at an int64 device table of n_slots per-slot addresses
 * (the reference's KT_PTR_TABLE build, kt_gguf_moe_multi.cu:184-189). Slot addresses in a
 * table must be 16-byte aligned.
 * Slot ids: route p uses slot ids[p]; ids outside [0, n_slots) (the reference uses -1 for
 * experts on the CPU) produce zero rows / contribute nothing.
 */
#ifndef KT_GGUF_B200_H
#define KT_GGUF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KT_OK 0
#define KT_ERR_ARG 1       /* invalid argument (null pointer, bad shape, unsupported size) */
#define KT_ERR_TYPE 2      /* ggml type without a kernel here */
#define KT_ERR_WORKSPACE 3 /* workspace smaller than the *_workspace_size query */
#define KT_ERR_CUDA 4      /* a CUDA call or launch failed */
#define KT_ERR_DEVICE 5    /* the GPU is not an sm_100 part */

#define KT_DEV_OK 0
#define KT_DEV_TIMEOUT 1

#define KT_GGML_Q4_0 2
#define KT_GGML_Q4_1 3
#define KT_GGML_Q5_0 6
#define KT_GGML_Q5_1 7
#define KT_GGML_Q8_0 8
#define KT_GGML_Q2_K 10
#define KT_GGML_Q3_K 11
#define KT_GGML_Q4_K 12
#define KT_GGML_Q5_K 13
#define KT_GGML_Q6_K 14
#define KT_GGML_IQ2_XXS 16
#define KT_GGML_IQ2_XS 17
#define KT_GGML_IQ3_XXS 18
#define KT_GGML_IQ1_S 19
#define KT_GGML_IQ4_NL 20
#define KT_GGML_IQ3_S 21
#define KT_GGML_IQ2_S 22
#define KT_GGML_IQ4_XS 23
#define KT_GGML_IQ1_M 29
#define KT_GGML_Q2_0 42

#define KT_DTYPE_F32 0
#define KT_DTYPE_F16 1
#define KT_DTYPE_BF16 2

/* Library version (major * 10000 + minor * 100 + patch). */
int kt_version(void);
/* Static description of a status code. */
const char* kt_status_string(int status);
/* 1 if the current device is an sm_100 GPU this library was built for, else 0. */
int kt_device_supported(void);

/* Bytes of one row of `cols` values in GGUF blocks of `ggml_type`.
 * Replaces BLOCK_INFO / _row_bytes (hot/kt_gguf_hot.py:62-93). */
int kt_gguf_row_bytes(int ggml_type, int64_t cols, int64_t* row_bytes);

/* Reads the device status word of a workspace used by a previous call (synchronizes the
 * stream first). *status = KT_DEV_OK or KT_DEV_TIMEOUT. */
int kt_workspace_status(const void* workspace, void* stream, int* status);

/* q8_1 activation quantizer: x [rows, cols] (dtype) -> qx [rows, qrow] bytes, with
 * qrow = ceil(cols / 512) * 512 / 32 * 36. Replaces quantize_row_q8_1_cuda
 * (hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu:600-650); bit-identical blocks. */
int kt_quantize_q8_1(const void* x, int x_dtype, int64_t rows, int64_t cols, void* qx, void* stream);

/* Decode GEMV workspace for kt_moe_a8_vec_multi / _routes / kt_dense_a8_vec. */
size_t kt_moe_a8_vec_workspace_size(int64_t tokens, int64_t cols, int64_t routes, int n_slots);

/* Y[p, r] = row r of slot topk_ids[p] . q8_1(X[p / top_k]) for p < tokens*top_k, in X's dtype;
 * zero rows for ids outside [0, n_slots). x [tokens, cols], y [tokens*top_k, rows].
 * Replaces the torch op kt_moe_a8_vec_multi (hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu:653-935,
 * bound at hot/kt_gguf_moe_multi.py:81-82): same sums, every route of a slot sharing one read
 * of its weights, at any token count. */
int kt_moe_a8_vec_multi(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w, int w_is_table,
                        int n_slots, const int32_t* topk_ids, int64_t top_k, int ggml_type, int64_t rows, void* y,
                        void* workspace, size_t workspace_bytes, void* stream);

/* The per-route contract of the reference's KT_PER_ROUTE build (hot/kt_gguf_moe_multi.py:85-87).
 * Sums are identical to kt_moe_a8_vec_multi per route. */
int kt_moe_a8_vec_routes(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w, int w_is_table,
                         int n_slots, const int32_t* topk_ids, int64_t top_k, int ggml_type, int64_t rows, void* y,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Size of the library's own scratch area used by kt_moe_a8_vec_multi_static (2 MiB). */
#define KT_STATIC_SCRATCH_BYTES (2u << 20)

/* kt_moe_a8_vec_multi without a caller workspace, for callers that cannot allocate device
 * memory per call (graph capture under a frozen pool, host frameworks that own all device
 * memory, C callers without an allocator). No counterpart in the reference: its op always
 * allocated through torch.
 * Scratch comes from a fixed KT_STATIC_SCRATCH_BYTES array inside the library, held on every
 * GPU that loads it until the process exits; calls whose scratch need
 * (kt_moe_a8_vec_workspace_size) exceeds it return KT_ERR_WORKSPACE. The first call on a
 * device looks up the array's address, so make it before any stream capture. All calls on a
 * device share the array: calls that can overlap on the GPU (other streams, concurrent
 * graphs) race and must be serialised by the caller. Nothing is allocated or freed. */
int kt_moe_a8_vec_multi_static(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w, int w_is_table,
                               int n_slots, const int32_t* topk_ids, int64_t top_k, int ggml_type, int64_t rows,
                               void* y, void* stream);

/* The device status word of the most recent kt_moe_a8_vec_multi_static call on the current
 * device (the counterpart of kt_workspace_status for the library's own scratch): synchronizes
 * `stream`, then *status = KT_DEV_OK or KT_DEV_TIMEOUT (meaningful once a static call has run
 * on the device). No counterpart in the reference. */
int kt_static_scratch_status(void* stream, int* status);

/* Workspace for kt_dense_a8_vec. */
size_t kt_dense_a8_vec_workspace_size(int64_t tokens, int64_t cols);

/* y [tokens, rows] = x [tokens, cols] . W^T for a dense GGUF weight w [rows, row_bytes]
 * (hot/kt_gguf_moe_multi.py:103-112). */
int kt_dense_a8_vec(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w, int ggml_type,
                    int64_t rows, void* y, void* workspace, size_t workspace_bytes, void* stream);

/* GGUF rows [rows, row_bytes] -> out [rows, cols] in out_dtype. The fp32 values are
 * bit-identical to ggml's dequantize_row_* (and gguf-py); f16/bf16 are those rounded to
 * nearest even. Replaces dequant_experts (flash-next-gguf patch, kt_gguf_dequant.py). */
int kt_gguf_dequantize(const void* w, int ggml_type, int64_t rows, int64_t cols, void* out, int out_dtype,
                       void* stream);

/* h [rows, n] = silu(h13[:, :n]) * h13[:, n:] in fp32, stored in dtype (sgl-kernel
 * silu_and_mul, called at hot/kt_gguf_hot.py:260). */
int kt_silu_and_mul(const void* h13, int dtype, int64_t rows, int64_t n, void* h, void* stream);

/* res [tokens, cols] = sum over k of dtype(out[t, k] * dtype(w[t, k])), accumulated in fp32
 * in k order and rounded once (the reference's _combine, hot/kt_gguf_hot.py:43-71). */
int kt_moe_combine(const void* out, int dtype, const float* w, int64_t tokens, int64_t top_k, int64_t cols, void* res,
                   void* stream);

/* HotCache.route (hot/kt_hot_cache.py:62-75, 121-143): slot_out[i] = log2slot[ids[i]],
 * cpu_out[i] = log2cpu[ids[i]], counts[ids[i]] += 1 (counts may be NULL). */
int kt_hot_route(const int32_t* ids, int64_t n, const int32_t* log2slot, const int32_t* log2cpu, float* counts,
                 int32_t* slot_out, int32_t* cpu_out, void* stream);

/* Router top-k over logits [tokens, n_experts] fp32: softmax, then the k largest
 * probabilities (ties to the lower id), optionally renormalised to sum 1. */
int kt_topk_softmax(const float* logits, int64_t tokens, int n_experts, int k, int renormalize, float* weights,
                    int32_t* ids, void* stream);

/* DeepSeek-V3 grouped routing: sigmoid scores, selection by score + bias (bias may be
 * NULL), group score = sum of the group's two best, keep topk_group groups, k experts;
 * weights = unbiased scores, optionally renormalised, times scale. */
int kt_topk_grouped(const float* logits, const float* bias, int64_t tokens, int n_experts, int n_group, int topk_group,
                    int k, int renormalize, float scale, float* weights, int32_t* ids, void* stream);

/* Prefill MoE layer workspace (permutation, H and Y staging, status word; and, for the shapes
 * kt_moe_prefill_predequant accepts, room for the expert weights in bf16). */
size_t kt_moe_prefill_workspace_size(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter, int n_slots);

/* Which expert weights a kt_moe_prefill / kt_moe_prefill_counted call of this shape
 * dequantizes to bf16 in one pass before the GEMMs (A tiles then arrive by TMA, with no
 * decoding in the GEMMs): bit 0 the gate/up weights, bit 1 the down weights; 0 if the GEMMs
 * decode the GGUF bytes themselves. The passes are taken when the slots average four 256-token
 * tiles or more and the bf16 copies are at most 4 GiB together, for contiguous 16-byte aligned
 * slots (not a table), when the workspace holds them (the size above); KT_B200_PREDQ=0 turns
 * them off, =1 on for every shape, KT_B200_PREDQ_DOWN=0 keeps the down weights in the GEMM's
 * decoding. Either way the outputs are the same bit for bit. No counterpart in the reference
 * (its streamed prefill dequantizes every group). */
int kt_moe_prefill_predequant(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter, int n_slots);

/* Byte offsets inside a kt_moe_prefill workspace, for inspection after a call:
 * offsets[0] status word (int), [1] per-slot route counts (int32 [n_slots]),
 * [2] tile list (int32 [n_tiles][3]: slot, first sorted row, rows), [3] n_tiles and the
 * number of resident routes (int32 [2]),
 * [4] token of each sorted row (int32 [tokens*top_k]; sorted rows of one slot are in no
 * particular order), [5] sorted row of each route
 * (int32 [tokens*top_k], -1 if not resident), [6] H (bf16 [tokens*top_k, inter]),
 * [7] per-route outputs Y (bf16 [tokens*top_k, hidden]). Rows past the resident routes are
 * unused. Returns KT_OK. */
int kt_moe_prefill_workspace_layout(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter, int n_slots,
                                    size_t offsets[8]);

/* One MoE layer on the GPU-resident slots, for prefill chunks:
 *   out[t] = sum_k w[t,k] * W2[s] (silu(W13g[s] x_t) * W13u[s] x_t),  s = topk_ids[t, k]
 * with bf16 activations x/out [tokens, hidden], fp32 topk_weights, slot ids as above.
 * The expert GEMMs run on tcgen05 with the GGUF weights dequantized to bf16 (in shared memory,
 * or in one pass first: kt_moe_prefill_predequant; fp32 accumulation);
 * H and the per-route outputs are rounded to bf16, and the
 * weighted sum over k is accumulated in fp32 with the fp32 router weights and rounded once
 * (the finalize of the fused MoE the reference's streamed prefill uses). Replaces the hot
 * method's apply (hot/kt_gguf_hot.py:240-304) at prefill sizes and the streamer's
 * dequant + cutlass_fused_moe group body. hidden % 256 == 0, inter % 256 == 0,
 * 1 <= top_k <= 32, 1 <= n_slots <= 8192. */
int kt_moe_prefill(const void* x, int64_t tokens, int64_t hidden, int64_t inter, const int32_t* topk_ids,
                   const float* topk_weights, int64_t top_k, const void* w13, int type13, const void* w2, int type2,
                   int w_is_table, int n_slots, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* kt_moe_prefill over an expert group, for the streamed prefill of experts that are not
 * resident (the reference's KTStreamPrefillGGUF._group_body, kt_stream_prefill_gguf.py in
 * its SGLang tree: dequant to bf16 + cutlass_fused_moe on the group, acc += out per group).
 * Routes whose id lies in [id_base, id_base + n_slots) run on slot id - id_base of w13 / w2
 * (the group's staged experts); every other route contributes nothing. acc_flags:
 *   KT_ACC_LOAD   each token's weighted sum starts from acc[t] (fp32 [tokens, hidden]);
 *   KT_ACC_STORE  the fp32 sum is written to acc (out unused, may be NULL); tokens with no
 *                 route in the group are skipped when KT_ACC_LOAD is set too;
 *   neither       as kt_moe_prefill: out = bf16(sum).
 * A group loop runs the first group with KT_ACC_STORE, the middle ones with both flags and
 * the last with KT_ACC_LOAD, so the sum over all groups is rounded to bf16 once. acc is
 * 16-byte aligned. Errors as kt_moe_prefill, and KT_ERR_ARG for id_base < 0 or unknown
 * flags. */
#define KT_ACC_LOAD 1
#define KT_ACC_STORE 2
int kt_moe_prefill_ex(const void* x, int64_t tokens, int64_t hidden, int64_t inter, const int32_t* topk_ids,
                      const float* topk_weights, int64_t top_k, const void* w13, int type13, const void* w2, int type2,
                      int w_is_table, int n_slots, int32_t id_base, float* acc, int acc_flags, void* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* kt_moe_prefill that also records four caller-created CUDA events (cudaEvent_t as void*)
 * on `stream` after its stages: [0] routing permutation, [1] gate/up GEMM, [2] down GEMM,
 * [3] combine. For per-stage timing; stage_events may be NULL. */
int kt_moe_prefill_timed(const void* x, int64_t tokens, int64_t hidden, int64_t inter, const int32_t* topk_ids,
                         const float* topk_weights, int64_t top_k, const void* w13, int type13, const void* w2, int type2,
                         int w_is_table, int n_slots, void* out, void* workspace, size_t workspace_bytes, void* stream,
                         void* const* stage_events);

/* Workspace for kt_moe_gemm_routes. */
size_t kt_moe_gemm_routes_workspace_size(int64_t tokens, int64_t top_k, int64_t cols, int64_t rows, int n_slots);

/* The per-route projection of kt_moe_a8_vec_routes on tensor cores:
 *   y[p] = bf16(W[ids[p]] . x[p / top_k])   for p < tokens*top_k, zero rows for ids outside
 *   [0, n_slots),
 * with bf16 activations x [tokens, cols], the GGUF weights (w [n_slots, rows, row_bytes(cols)]
 * or a slot table) dequantized in shared memory to bf16 exactly as kt_gguf_dequantize rounds
 * them, fp32 accumulation, y [tokens*top_k, rows] bf16. The prefill layer's own GEMM kernels
 * run it: reductions of at most 512 the down projection's, longer ones the gate/up
 * projection's without the SwiGLU, so a one-hot x reads back the dequantized weights those
 * kernels multiply with. Replaces, at prefill sizes, the reference's per-route GEMV build
 * (hot/kt_gguf_moe_multi.py:85-87) for a single projection. Types as kt_moe_prefill;
 * cols % 256 == 0, rows % 256 == 0; x and y 16-byte aligned. */
int kt_moe_gemm_routes(const void* x, int64_t tokens, int64_t cols, const int32_t* topk_ids, int64_t top_k,
                       const void* w, int ggml_type, int64_t rows, int w_is_table, int n_slots, void* y,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Self-test of the failure path the prefill GEMMs rely on: one CTA pair sets up as they do
 * (barriers, the pair's TMEM), waits on a barrier that nothing arrives on with the library's
 * bounded wait (limit_ns, 1 ms to 2 s, instead of the GEMMs' 2 s), then drains, meets its peer
 * and frees TMEM as the GEMMs do after a timeout. Clears the status word (the first int of
 * `workspace`) first; after the stream has finished, kt_workspace_status reports
 * KT_DEV_TIMEOUT and the context stays usable. No counterpart in the reference. */
int kt_selftest_bounded_wait(void* workspace, size_t workspace_bytes, int64_t limit_ns, void* stream);

/* ---- Expert-parallel plumbing (no counterpart in the reference, which runs the hot experts on
 * one GPU per tensor-parallel rank). Around an all-to-all of bf16 rows over n_ranks <= 8
 * ranks: owner[e] / local[e] give, for each of n_experts logical experts, its rank (< 0: none)
 * and its slot there. */

/* Scratch for kt_ep_plan (per block of 256 tokens and rank). */
size_t kt_ep_plan_workspace_size(int64_t tokens, int n_ranks);

/* Dispatch plan: each token goes once to every rank owning at least one of its experts; send
 * rows are grouped by destination rank, tokens ascending. Writes counts [n_ranks],
 * send_token [rows] (rows <= tokens*n_ranks), meta [rows][2*top_k] (the row's local slots,
 * -1 where the expert is elsewhere, then its weights as fp32 bits, 0 there) and
 * row_of [tokens][n_ranks] (send row of token t for rank r, or -1). */
int kt_ep_plan(const int32_t* topk_ids, const float* topk_weights, int64_t tokens, int64_t top_k, const int32_t* owner,
               const int32_t* local, int n_experts, int n_ranks, int32_t* counts, int32_t* send_token, int32_t* meta,
               int32_t* row_of, void* workspace, size_t workspace_bytes, void* stream);

/* out[i] = x[send_token[i]] for i < rows; x, out bf16 rows of `hidden` values, 16-byte aligned. */
int kt_ep_pack(const void* x, int64_t hidden, const int32_t* send_token, int64_t rows, void* out, void* stream);

/* out[t] = bf16(shared[t] + sum over r = 0..n_ranks-1 of back[row_of[t][r]]) with fp32 sums in
 * rank order; rows of -1 are skipped; shared may be NULL. bf16 rows of `hidden` values. */
int kt_ep_combine(const void* back, const int32_t* row_of, int n_ranks, const void* shared, int64_t tokens,
                  int64_t hidden, void* out, void* stream);

/* ---- The exchange over peer memory (no counterpart in the reference). Instead of moving rows
 * with NCCL all-to-alls, each rank writes its rows straight into the other ranks' receive
 * buffers and reads its partial outputs straight from their output buffers, over NVLink, with
 * plain loads and stores from these kernels (no TMA, no multicast). The buffers are mapped into
 * every rank's process by CUDA IPC (kt_ipc_*); the caller orders the steps with barriers (any
 * collective on the stream): every rank's dispatch before any rank's layer, every layer before
 * any combine. counts_all [n_ranks][n_ranks] int32 on the device: row counts of every rank's
 * kt_ep_plan (counts_all[s][d]: rows s sends to d). peer_* are device arrays of n_ranks buffer
 * addresses (this rank's own at index rank). Rank s's rows for rank d land in d's receive
 * buffers at rows base(s, d) + j, base(s, d) = sum over s' < s of counts_all[s'][d], j the
 * row's index among s's rows for d. */

/* 64-byte handle and offset of the allocation holding ptr, for kt_ipc_import in another
 * process on this node. */
int kt_ipc_export(const void* ptr, void* handle, size_t* offset);
/* *ptr = the exported buffer mapped into this process (peer access enabled). */
int kt_ipc_import(const void* handle, size_t offset, void** ptr);
/* Unmaps a buffer mapped by kt_ipc_import (ptr and offset as returned / passed there). */
int kt_ipc_close(void* ptr, size_t offset);

/* Dispatch: send row i of kt_ep_plan (token send_token[i], meta[i] = its k slot ids then k
 * weights) goes to its destination rank d's buffers: x rows peer_x[d] bf16 [rows_cap, hidden],
 * slot ids peer_ids[d] int32 [rows_cap, top_k], weights peer_w[d] fp32 [rows_cap, top_k].
 * *recv_total = the rows this rank receives (sum over s of counts_all[s][rank]). */
int kt_ep_dispatch_p2p(const void* x, int64_t hidden, const int32_t* send_token, const int32_t* meta, int64_t top_k,
                       const int32_t* counts_all, int rank, int n_ranks, const int64_t* peer_x, const int64_t* peer_ids,
                       const int64_t* peer_w, int64_t rows_cap, int32_t* recv_total, void* stream);

/* Combine: out[t] = bf16(shared[t] + sum over ranks d, in rank order, of d's output row for
 * this rank's row row_of[t][d]) with fp32 sums; the rows are read from peer_y[d] (each rank's
 * layer output over its receive rows). shared may be NULL. */
int kt_ep_combine_p2p(const int32_t* row_of, const int32_t* counts_all, int rank, int n_ranks, const int64_t* peer_y,
                      const void* shared, int64_t tokens, int64_t hidden, void* out, void* stream);

/* kt_moe_prefill over a device-resident token count: x, topk_ids, topk_weights and out have
 * room for tokens_cap tokens, the call processes the first *tokens_dev of them (read on the
 * device, so the host needs no copy of it) and writes only their output rows. For the rows an
 * expert-parallel rank receives. */
int kt_moe_prefill_counted(const void* x, int64_t tokens_cap, const int32_t* tokens_dev, int64_t hidden, int64_t inter,
                           const int32_t* topk_ids, const float* topk_weights, int64_t top_k, const void* w13,
                           int type13, const void* w2, int type2, int w_is_table, int n_slots, void* out,
                           void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KT_GGUF_B200_H */
