// capi.cu — the exported C ABI (include/kt_gguf_b200.h): argument checks, workspace
// carving, and the launch sequences of the decode GEMV and the prefill layer.
#include <string.h>

#include <stdlib.h>

#include <mutex>

#include "kt_gguf_b200.h"
#include "kt_common.cuh"
#include "kt_kernels.h"

#define KT_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool type_ok(int t) { return kt_gemv_type(t); }  // decode GEMV, dequantization, row sizes
inline bool dtype_ok(int d) { return d == KT_DT_F32 || d == KT_DT_F16 || d == KT_DT_BF16; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// bump allocator over a caller workspace
struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base((uint8_t*)b) {}
  template <typename T>
  T* take(size_t count, size_t align = 256) {
    off = align_up(off, align);
    T* p = reinterpret_cast<T*>(reinterpret_cast<uintptr_t>(base) + off);  // base 0: offsets
    off += sizeof(T) * count;
    return p;
  }
};

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int launch_rc(int rc) {
  if (rc) return rc == -1 ? KT_ERR_ARG : KT_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? KT_OK : KT_ERR_CUDA;
}

// decode GEMV workspace layout
struct VecWs {
  int* status;
  uint8_t* qx;
  int32_t* groups;
  int32_t* order;
  size_t bytes;
};

VecWs vec_ws(void* ws, int64_t tokens, int64_t cols, int64_t routes, int n_slots) {
  Carve c(ws);
  VecWs v;
  v.status = c.take<int>(4);
  v.qx = c.take<uint8_t>((size_t)tokens * kt_q8_1_row_bytes(cols));
  // groups: at most one per route once slots are cut into pieces, else one per slot (+ zero)
  v.groups = c.take<int32_t>(1 + 3 * (size_t)(n_slots + 1 + routes));
  v.order = c.take<int32_t>((size_t)routes);
  v.bytes = align_up(c.off, 256);
  return v;
}

int moe_vec(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w, int table, int n_slots,
            const int32_t* ids, int64_t top_k, int type, int64_t rows, void* y, void* ws, size_t ws_bytes, void* stream) {
  if (!type_ok(type)) return KT_ERR_TYPE;
  if (!dtype_ok(x_dtype) || tokens < 0 || cols <= 0 || rows <= 0 || top_k <= 0 || n_slots <= 0) return KT_ERR_ARG;
  if (cols % kt_block_info(type).qk || rows > (1 << 30)) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  if (!x || !w || !ids || !y || !ws) return KT_ERR_ARG;
  const int64_t routes = tokens * top_k;
  VecWs v = vec_ws(ws, tokens, cols, routes, n_slots);
  if (ws_bytes < v.bytes) return KT_ERR_WORKSPACE;
  cudaStream_t s = S(stream);
  if (cols <= (1 << 24) && kt_vec_fused_ok(type, w, table, x, routes, (int)rows, (int)cols))  // a few tokens
    return launch_rc(kt_launch_moe_vec_fused(type, w, table, n_slots, x, x_dtype, ids, routes, (int)top_k, (int)rows,
                                             (int)cols, y, v.status, s));
  const int piece = kt_vec_ms_ok(type, (int)cols, routes) ? kt_vec_ms_piece() : 0;
  int rc = kt_launch_quantize_group(x, x_dtype, tokens, cols, v.qx, ids, routes, n_slots, piece, v.groups, v.order,
                                    v.status, s);  // the first launch also resets the status word
  if (rc) return launch_rc(rc);
  const int max_groups = (int)(piece || routes < (int64_t)n_slots + 1 ? routes : (int64_t)n_slots + 1);
  rc = kt_launch_moe_vec(type, w, table, v.qx, kt_q8_1_row_bytes(cols), v.groups, v.order, max_groups, (int)top_k,
                         (int)rows, (int)cols, x_dtype, y, v.status, s);
  return launch_rc(rc);
}

// prefill workspace layout
struct PreWs {
  int* status;
  int32_t* counts;
  int32_t* hist;  // per permute block and slot: route count, then first sorted position
  int32_t* tiles;
  int32_t* n_tiles;
  int32_t* chunks;
  int32_t* sorted_token;
  int32_t* route_pos;
  uint16_t* h;
  uint16_t* y;
  uint16_t* w13b;  // gate/up weights dequantized to bf16 [n_slots * 2 inter, hidden] (when pre_dequant)
  uint16_t* w2b;   // down weights dequantized to bf16 [n_slots * hidden, inter] (when pre_dequant has kPreDown)
  size_t bytes;
  size_t bytes_min;  // without w13b and w2b
};

// Whether a prefill call of this shape dequantizes the expert weights to bf16 once, before the
// GEMMs, instead of in the GEMMs' producers for every token tile (gate/up) or chunk of four
// tiles (down). Worth it when the slots average four token tiles or more: each weight tile is
// then decoded once instead of ~8 (gate/up) or ~2-3 (down) times, for a pass that costs about
// (raw + bf16 bytes) / HBM bandwidth. Both copies together stay under 4 GiB. KT_B200_PREDQ=0
// turns it off, =1 on for every shape; KT_B200_PREDQ_DOWN=0 keeps the down weights in the
// GEMM's own decoding. Returns kPreGateUp | kPreDown bits.
constexpr int kPreGateUp = 1, kPreDown = 2;
int pre_dequant(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter, int n_slots) {
  static const int mode = [] {
    const char* e = getenv("KT_B200_PREDQ");
    return !e ? 2 : e[0] == '0' ? 0 : 1;
  }();
  static const bool down = [] {
    const char* e = getenv("KT_B200_PREDQ_DOWN");
    return !(e && e[0] == '0');
  }();
  const int64_t bytes = (int64_t)n_slots * 3 * inter * hidden * 2;
  if (mode == 0 || bytes > ((int64_t)4 << 30)) return 0;
  if (mode == 2 && tokens * top_k < 4 * (int64_t)kt_gemm_tile_tokens() * n_slots) return 0;
  return kPreGateUp | (down ? kPreDown : 0);
}

PreWs pre_ws(void* ws, int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter, int n_slots) {
  Carve c(ws);
  PreWs p;
  const int64_t R = tokens * top_k;
  const int tn = kt_gemm_tile_tokens();
  p.status = c.take<int>(4);
  p.counts = c.take<int32_t>(n_slots);
  p.hist = c.take<int32_t>((size_t)kt_permute_hist_ints(R, n_slots));
  p.tiles = c.take<int32_t>(3 * (size_t)(R / tn + n_slots + 1));
  p.n_tiles = c.take<int32_t>(4);
  p.chunks = c.take<int32_t>(3 * (size_t)(R / tn + n_slots + 1));
  p.sorted_token = c.take<int32_t>(R);
  p.route_pos = c.take<int32_t>(R);
  p.h = c.take<uint16_t>((size_t)R * inter, 1024);
  p.y = c.take<uint16_t>((size_t)R * hidden, 1024);
  p.bytes_min = align_up(c.off, 256);
  const int pre = pre_dequant(tokens, top_k, hidden, inter, n_slots);
  p.w13b = pre & kPreGateUp ? c.take<uint16_t>((size_t)n_slots * 2 * inter * hidden, 1024) : nullptr;
  p.w2b = pre & kPreDown ? c.take<uint16_t>((size_t)n_slots * hidden * inter, 1024) : nullptr;
  p.bytes = align_up(c.off, 256);
  return p;
}

// per-route expert GEMM workspace layout (kt_moe_gemm_routes)
struct RouteWs {
  int* status;
  int32_t* counts;
  int32_t* hist;
  int32_t* tiles;
  int32_t* n_tiles;
  int32_t* chunks;
  int32_t* sorted_token;
  int32_t* route_pos;
  uint16_t* xs;  // activation rows in slot order (reductions <= 512 only)
  uint16_t* ys;  // outputs in slot order
  size_t bytes;
};

constexpr int64_t kRouteShortReduction = 512;  // reductions up to this run the down kernels

RouteWs route_ws(void* ws, int64_t tokens, int64_t top_k, int64_t cols, int64_t rows, int n_slots) {
  Carve c(ws);
  RouteWs r;
  const int64_t R = tokens * top_k;
  const int tn = kt_gemm_tile_tokens();
  r.status = c.take<int>(4);
  r.counts = c.take<int32_t>(n_slots);
  r.hist = c.take<int32_t>((size_t)kt_permute_hist_ints(R, n_slots));
  r.tiles = c.take<int32_t>(3 * (size_t)(R / tn + n_slots + 1));
  r.n_tiles = c.take<int32_t>(4);
  r.chunks = c.take<int32_t>(3 * (size_t)(R / tn + n_slots + 1));
  r.sorted_token = c.take<int32_t>(R);
  r.route_pos = c.take<int32_t>(R);
  r.xs = c.take<uint16_t>(cols <= kRouteShortReduction ? (size_t)R * cols : 0, 1024);
  r.ys = c.take<uint16_t>((size_t)R * rows, 1024);
  r.bytes = align_up(c.off, 256);
  return r;
}

}  // namespace

KT_EXPORT int kt_version(void) { return 100; }

KT_EXPORT const char* kt_status_string(int status) {
  switch (status) {
    case KT_OK: return "ok";
    case KT_ERR_ARG: return "invalid argument";
    case KT_ERR_TYPE: return "unsupported ggml type";
    case KT_ERR_WORKSPACE: return "workspace too small";
    case KT_ERR_CUDA: return "CUDA error";
    case KT_ERR_DEVICE: return "device is not sm_100";
  }
  return "unknown status";
}

KT_EXPORT int kt_device_supported(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

KT_EXPORT int kt_gguf_row_bytes(int ggml_type, int64_t cols, int64_t* row_bytes) {
  if (!type_ok(ggml_type)) return KT_ERR_TYPE;
  const KtBlockInfo bi = kt_block_info(ggml_type);
  if (!row_bytes || cols < 0 || cols % bi.qk) return KT_ERR_ARG;
  *row_bytes = cols / bi.qk * bi.bytes;
  return KT_OK;
}

KT_EXPORT int kt_workspace_status(const void* workspace, void* stream, int* status) {
  if (!workspace || !status) return KT_ERR_ARG;
  if (cudaStreamSynchronize(S(stream)) != cudaSuccess) return KT_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return KT_ERR_CUDA;
  *status = v;
  return KT_OK;
}

KT_EXPORT int kt_quantize_q8_1(const void* x, int x_dtype, int64_t rows, int64_t cols, void* qx, void* stream) {
  if (!dtype_ok(x_dtype) || rows < 0 || cols <= 0) return KT_ERR_ARG;
  if (rows == 0) return KT_OK;
  if (!x || !qx) return KT_ERR_ARG;
  return launch_rc(kt_launch_quantize_q8_1(x, x_dtype, rows, cols, qx, S(stream)));
}

KT_EXPORT size_t kt_moe_a8_vec_workspace_size(int64_t tokens, int64_t cols, int64_t routes, int n_slots) {
  return vec_ws(nullptr, tokens, cols, routes, n_slots).bytes;
}

KT_EXPORT int kt_moe_a8_vec_multi(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w,
                                  int w_is_table, int n_slots, const int32_t* topk_ids, int64_t top_k, int ggml_type,
                                  int64_t rows, void* y, void* workspace, size_t workspace_bytes, void* stream) {
  return moe_vec(x, x_dtype, tokens, cols, w, w_is_table, n_slots, topk_ids, top_k, ggml_type, rows, y, workspace,
                 workspace_bytes, stream);
}

KT_EXPORT int kt_moe_a8_vec_routes(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w,
                                   int w_is_table, int n_slots, const int32_t* topk_ids, int64_t top_k, int ggml_type,
                                   int64_t rows, void* y, void* workspace, size_t workspace_bytes, void* stream) {
  return moe_vec(x, x_dtype, tokens, cols, w, w_is_table, n_slots, topk_ids, top_k, ggml_type, rows, y, workspace,
                 workspace_bytes, stream);
}

KT_EXPORT size_t kt_dense_a8_vec_workspace_size(int64_t tokens, int64_t cols) {
  return align_up(kt_moe_a8_vec_workspace_size(tokens, cols, tokens, 1), 256) + align_up(sizeof(int32_t) * (size_t)tokens, 256);
}

KT_EXPORT int kt_dense_a8_vec(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w, int ggml_type,
                              int64_t rows, void* y, void* workspace, size_t workspace_bytes, void* stream) {
  // a dense weight is a one-slot MoE whose routes all use slot 0; the route ids live in
  // the workspace tail (zeroed here)
  const size_t need = kt_moe_a8_vec_workspace_size(tokens, cols, tokens, 1);
  const size_t ids_off = align_up(need, 256);
  if (workspace_bytes < ids_off + sizeof(int32_t) * (size_t)tokens) return KT_ERR_WORKSPACE;
  if (tokens <= 0) return tokens == 0 ? KT_OK : KT_ERR_ARG;
  int32_t* ids = reinterpret_cast<int32_t*>((uint8_t*)workspace + ids_off);
  if (cudaMemsetAsync(ids, 0, sizeof(int32_t) * tokens, S(stream)) != cudaSuccess) return KT_ERR_CUDA;
  return moe_vec(x, x_dtype, tokens, cols, w, 0, 1, ids, 1, ggml_type, rows, y, workspace, need, stream);
}

KT_EXPORT int kt_gguf_dequantize(const void* w, int ggml_type, int64_t rows, int64_t cols, void* out, int out_dtype,
                                 void* stream) {
  if (!type_ok(ggml_type)) return KT_ERR_TYPE;
  if (!dtype_ok(out_dtype) || rows < 0 || cols < 0 || cols % kt_block_info(ggml_type).qk) return KT_ERR_ARG;
  if (rows == 0 || cols == 0) return KT_OK;
  if (!w || !out) return KT_ERR_ARG;
  return launch_rc(kt_launch_dequant(ggml_type, w, rows, cols, out, out_dtype, S(stream)));
}

KT_EXPORT int kt_silu_and_mul(const void* h13, int dtype, int64_t rows, int64_t n, void* h, void* stream) {
  if (!dtype_ok(dtype) || rows < 0 || n < 0) return KT_ERR_ARG;
  if (rows == 0 || n == 0) return KT_OK;
  if (!h13 || !h) return KT_ERR_ARG;
  return launch_rc(kt_launch_silu_and_mul(h13, dtype, rows, n, h, S(stream)));
}

KT_EXPORT int kt_moe_combine(const void* out, int dtype, const float* w, int64_t tokens, int64_t top_k, int64_t cols,
                             void* res, void* stream) {
  if (!dtype_ok(dtype) || tokens < 0 || top_k <= 0 || cols < 0) return KT_ERR_ARG;
  if (tokens == 0 || cols == 0) return KT_OK;
  if (!out || !w || !res) return KT_ERR_ARG;
  return launch_rc(kt_launch_combine(out, dtype, w, tokens, top_k, cols, res, S(stream)));
}

KT_EXPORT int kt_hot_route(const int32_t* ids, int64_t n, const int32_t* log2slot, const int32_t* log2cpu, float* counts,
                           int32_t* slot_out, int32_t* cpu_out, void* stream) {
  if (n < 0) return KT_ERR_ARG;
  if (n == 0) return KT_OK;
  if (!ids || !log2slot || !log2cpu || !slot_out || !cpu_out) return KT_ERR_ARG;
  return launch_rc(kt_launch_route(ids, n, log2slot, log2cpu, counts, slot_out, cpu_out, S(stream)));
}

KT_EXPORT int kt_topk_softmax(const float* logits, int64_t tokens, int n_experts, int k, int renormalize, float* weights,
                              int32_t* ids, void* stream) {
  if (tokens < 0 || n_experts <= 0 || k <= 0) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  if (!logits || !weights || !ids) return KT_ERR_ARG;
  return launch_rc(kt_launch_topk_softmax(logits, tokens, n_experts, k, renormalize, weights, ids, S(stream)));
}

KT_EXPORT int kt_topk_grouped(const float* logits, const float* bias, int64_t tokens, int n_experts, int n_group,
                              int topk_group, int k, int renormalize, float scale, float* weights, int32_t* ids,
                              void* stream) {
  if (tokens < 0 || n_experts <= 0 || k <= 0) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  if (!logits || !weights || !ids) return KT_ERR_ARG;
  return launch_rc(kt_launch_topk_grouped(logits, bias, tokens, n_experts, n_group, topk_group, k, renormalize, scale,
                                          weights, ids, S(stream)));
}

KT_EXPORT size_t kt_moe_prefill_workspace_size(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter,
                                               int n_slots) {
  return pre_ws(nullptr, tokens, top_k, hidden, inter, n_slots).bytes;
}

KT_EXPORT int kt_moe_prefill_predequant(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter, int n_slots) {
  return pre_dequant(tokens, top_k, hidden, inter, n_slots);
}

KT_EXPORT int kt_moe_prefill_workspace_layout(int64_t tokens, int64_t top_k, int64_t hidden, int64_t inter,
                                              int n_slots, size_t offsets[8]) {
  if (!offsets) return KT_ERR_ARG;
  PreWs p = pre_ws(nullptr, tokens, top_k, hidden, inter, n_slots);
  const void* ptrs[8] = {p.status, p.counts, p.tiles, p.n_tiles, p.sorted_token, p.route_pos, p.h, p.y};
  for (int i = 0; i < 8; ++i) offsets[i] = (size_t)(uintptr_t)ptrs[i];
  return KT_OK;
}

static int prefill_run(const void* x, int64_t tokens, int64_t hidden, int64_t inter, const int32_t* topk_ids,
                       const float* topk_weights, int64_t top_k, const void* w13, int type13, const void* w2, int type2,
                       int w_is_table, int n_slots, int32_t id_base, float* acc, int acc_flags, void* out,
                       void* workspace, size_t workspace_bytes, void* stream, void* const* stage_events,
                       const int32_t* tokens_dev = nullptr) {
  if (!kt_prefill_type(type13) || !kt_prefill_type(type2)) return KT_ERR_TYPE;
  if (tokens < 0 || top_k <= 0 || top_k > 32 || n_slots <= 0 || n_slots > kPermMaxSlots || hidden <= 0 || inter <= 0)
    return KT_ERR_ARG;
  if (hidden % 256 || inter % 256 || hidden > (1 << 20) || inter > (1 << 20)) return KT_ERR_ARG;
  if (tokens * top_k > (int64_t)1 << 30) return KT_ERR_ARG;
  if (id_base < 0 || (acc_flags & ~(KT_ACC_LOAD | KT_ACC_STORE))) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  const bool to_acc = acc_flags & KT_ACC_STORE;
  if (!x || !topk_ids || !topk_weights || !w13 || !w2 || !workspace || (!to_acc && !out)) return KT_ERR_ARG;
  if (acc_flags && (!acc || ((uintptr_t)acc & 15))) return KT_ERR_ARG;
  if (((uintptr_t)x | (uintptr_t)(to_acc ? nullptr : out)) & 15) return KT_ERR_ARG;
  PreWs p = pre_ws(workspace, tokens, top_k, hidden, inter, n_slots);
  if (workspace_bytes < p.bytes_min) return KT_ERR_WORKSPACE;
  // the one-pass bf16 dequantization of the expert weights: plain calls (not an expert group of
  // a streamed layer, which has few tokens per expert) with contiguous slots and the room for it
  const bool pre_ok = workspace_bytes >= p.bytes && !w_is_table && id_base == 0 && !acc_flags &&
                      !(((uintptr_t)w13) & 15) && !(((uintptr_t)w2) & 15);
  const void* w13b = pre_ok ? p.w13b : nullptr;
  const void* w2b = pre_ok ? p.w2b : nullptr;
  cudaStream_t s = S(stream);
  auto mark = [&](int i) {
    if (stage_events && stage_events[i]) cudaEventRecord(reinterpret_cast<cudaEvent_t>(stage_events[i]), s);
  };
  const int64_t R = tokens * top_k;
  if (cudaMemsetAsync(p.status, 0, sizeof(int), s) != cudaSuccess) return KT_ERR_CUDA;
  int rc = kt_launch_permute(topk_ids, R, (int)top_k, n_slots, kt_gemm_tile_tokens(), kt_gemm_chunk_tiles(), p.counts,
                             p.hist, p.tiles, p.n_tiles, p.chunks, p.sorted_token, p.route_pos, s, id_base, tokens_dev);
  if (rc) return launch_rc(rc);
  // the weight passes, timed with the permutation (stage 0) so the GEMM stages are the GEMMs alone
  if (w13b) {
    rc = kt_launch_dequant(type13, w13, (int64_t)n_slots * 2 * inter, hidden, (void*)w13b, KT_DT_BF16, s, p.status);
    if (rc) return launch_rc(rc);
  }
  if (w2b) {
    rc = kt_launch_dequant(type2, w2, (int64_t)n_slots * hidden, inter, (void*)w2b, KT_DT_BF16, s, p.status);
    if (rc) return launch_rc(rc);
  }
  mark(0);
  // SMs left to concurrent kernels (e.g. NCCL's while an expert-parallel layer overlaps its
  // all-to-alls with these GEMMs): KT_B200_RESERVE_SMS, read once; the GEMMs are persistent
  // grids and would otherwise hold every SM until they end
  static const int reserve = [] {
    const char* e = getenv("KT_B200_RESERVE_SMS");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : 0;
  }();
  const int grid = num_sms() - reserve >= 2 ? num_sms() - reserve : 2;
  rc = kt_launch_gemm_gate_up(type13, x, tokens, (int)hidden, (int)inter, w13, w_is_table, n_slots, p.tiles, p.n_tiles,
                              p.sorted_token, p.h, p.status, grid, s, 0, w13b);
  if (rc) return launch_rc(rc);
  mark(1);
  rc = kt_launch_gemm_down(type2, p.h, R, (int)hidden, (int)inter, w2, w_is_table, n_slots, p.tiles, p.n_tiles,
                           p.chunks, p.y, p.status, grid, s, w2b);
  if (rc) return launch_rc(rc);
  mark(2);
  rc = kt_launch_combine_sorted(p.y, p.route_pos, topk_weights, tokens, top_k, hidden, (uint16_t*)out, s, acc,
                                acc_flags, tokens_dev);
  if (rc) return launch_rc(rc);
  mark(3);
  return launch_rc(0);
}

KT_EXPORT int kt_moe_prefill_timed(const void* x, int64_t tokens, int64_t hidden, int64_t inter,
                                   const int32_t* topk_ids, const float* topk_weights, int64_t top_k, const void* w13,
                                   int type13, const void* w2, int type2, int w_is_table, int n_slots, void* out,
                                   void* workspace, size_t workspace_bytes, void* stream, void* const* stage_events) {
  return prefill_run(x, tokens, hidden, inter, topk_ids, topk_weights, top_k, w13, type13, w2, type2, w_is_table,
                     n_slots, 0, nullptr, 0, out, workspace, workspace_bytes, stream, stage_events);
}

KT_EXPORT int kt_moe_prefill(const void* x, int64_t tokens, int64_t hidden, int64_t inter, const int32_t* topk_ids,
                             const float* topk_weights, int64_t top_k, const void* w13, int type13, const void* w2,
                             int type2, int w_is_table, int n_slots, void* out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  return prefill_run(x, tokens, hidden, inter, topk_ids, topk_weights, top_k, w13, type13, w2, type2, w_is_table,
                     n_slots, 0, nullptr, 0, out, workspace, workspace_bytes, stream, nullptr);
}

KT_EXPORT int kt_moe_prefill_ex(const void* x, int64_t tokens, int64_t hidden, int64_t inter, const int32_t* topk_ids,
                                const float* topk_weights, int64_t top_k, const void* w13, int type13, const void* w2,
                                int type2, int w_is_table, int n_slots, int32_t id_base, float* acc, int acc_flags,
                                void* out, void* workspace, size_t workspace_bytes, void* stream) {
  return prefill_run(x, tokens, hidden, inter, topk_ids, topk_weights, top_k, w13, type13, w2, type2, w_is_table,
                     n_slots, id_base, acc, acc_flags, out, workspace, workspace_bytes, stream, nullptr);
}

KT_EXPORT int kt_selftest_bounded_wait(void* workspace, size_t workspace_bytes, int64_t limit_ns, void* stream) {
  if (!workspace || workspace_bytes < sizeof(int)) return KT_ERR_ARG;
  if (limit_ns < 1000000 || limit_ns > 2000000000) return KT_ERR_ARG;  // 1 ms .. 2 s
  if (cudaMemsetAsync(workspace, 0, sizeof(int), S(stream)) != cudaSuccess) return KT_ERR_CUDA;
  return launch_rc(kt_launch_selftest_wait((int*)workspace, (uint64_t)limit_ns, S(stream)));
}

// ------------------------------------------------------------------ per-route expert GEMM

KT_EXPORT size_t kt_moe_gemm_routes_workspace_size(int64_t tokens, int64_t top_k, int64_t cols, int64_t rows,
                                                   int n_slots) {
  return route_ws(nullptr, tokens, top_k, cols, rows, n_slots).bytes;
}

KT_EXPORT int kt_moe_gemm_routes(const void* x, int64_t tokens, int64_t cols, const int32_t* topk_ids, int64_t top_k,
                                 const void* w, int ggml_type, int64_t rows, int w_is_table, int n_slots, void* y,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  if (!kt_prefill_type(ggml_type)) return KT_ERR_TYPE;
  if (tokens < 0 || top_k <= 0 || n_slots <= 0 || n_slots > kPermMaxSlots || cols <= 0 || rows <= 0) return KT_ERR_ARG;
  if (cols % 256 || rows % 256 || cols > (1 << 20) || rows > (1 << 20)) return KT_ERR_ARG;
  if (tokens * top_k > (int64_t)1 << 30) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  if (!x || !topk_ids || !w || !y || !workspace || (((uintptr_t)x | (uintptr_t)y) & 15)) return KT_ERR_ARG;
  RouteWs r = route_ws(workspace, tokens, top_k, cols, rows, n_slots);
  if (workspace_bytes < r.bytes) return KT_ERR_WORKSPACE;
  cudaStream_t s = S(stream);
  const int64_t R = tokens * top_k;
  if (cudaMemsetAsync(r.status, 0, sizeof(int), s) != cudaSuccess) return KT_ERR_CUDA;
  int rc = kt_launch_permute(topk_ids, R, (int)top_k, n_slots, kt_gemm_tile_tokens(), kt_gemm_chunk_tiles(), r.counts,
                             r.hist, r.tiles, r.n_tiles, r.chunks, r.sorted_token, r.route_pos, s, 0);
  if (rc) return launch_rc(rc);
  const int grid = num_sms();
  if (cols <= kRouteShortReduction) {
    // short reductions: the activation rows in slot order, then the down projection's kernels
    // (the resident-strip kernel; KT_B200_DOWN_STREAM selects the streaming one)
    rc = kt_launch_gather_rows((const uint16_t*)x, cols, r.sorted_token, R, r.n_tiles + 1, r.xs, s);
    if (rc) return launch_rc(rc);
    rc = kt_launch_gemm_down(ggml_type, r.xs, R, (int)rows, (int)cols, w, w_is_table, n_slots, r.tiles, r.n_tiles,
                             r.chunks, r.ys, r.status, grid, s);
  } else {
    // longer ones: the gate/up kernel (token rows gathered in the kernel) without the activation
    rc = kt_launch_gemm_gate_up(ggml_type, x, tokens, (int)cols, (int)(rows / 2), w, w_is_table, n_slots, r.tiles,
                                r.n_tiles, r.sorted_token, r.ys, r.status, grid, s, 1);
  }
  if (rc) return launch_rc(rc);
  // back to route order, zero rows for routes without a resident slot
  return launch_rc(kt_launch_gather_rows(r.ys, rows, r.route_pos, R, nullptr, (uint16_t*)y, s));
}

KT_EXPORT int kt_moe_prefill_counted(const void* x, int64_t tokens_cap, const int32_t* tokens_dev, int64_t hidden,
                                     int64_t inter, const int32_t* topk_ids, const float* topk_weights, int64_t top_k,
                                     const void* w13, int type13, const void* w2, int type2, int w_is_table,
                                     int n_slots, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!tokens_dev) return KT_ERR_ARG;
  return prefill_run(x, tokens_cap, hidden, inter, topk_ids, topk_weights, top_k, w13, type13, w2, type2, w_is_table,
                     n_slots, 0, nullptr, 0, out, workspace, workspace_bytes, stream, nullptr, tokens_dev);
}

// ------------------------------------------------------------------ expert-parallel plumbing

KT_EXPORT size_t kt_ep_plan_workspace_size(int64_t tokens, int n_ranks) {
  if (tokens < 0 || n_ranks < 1) return 0;
  return align_up((size_t)kt_ep_plan_ints(tokens, n_ranks) * sizeof(int32_t) + 256, 256);
}

KT_EXPORT int kt_ep_plan(const int32_t* topk_ids, const float* topk_weights, int64_t tokens, int64_t top_k,
                         const int32_t* owner, const int32_t* local, int n_experts, int n_ranks, int32_t* counts,
                         int32_t* send_token, int32_t* meta, int32_t* row_of, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (tokens < 0 || top_k < 1 || top_k > 64 || n_experts < 1 || n_ranks < 1 || n_ranks > 8) return KT_ERR_ARG;
  if (!counts || !owner || !local || !workspace) return KT_ERR_ARG;
  if (tokens > 0 && (!topk_ids || !topk_weights || !send_token || !meta || !row_of)) return KT_ERR_ARG;
  if (workspace_bytes < kt_ep_plan_workspace_size(tokens, n_ranks)) return KT_ERR_WORKSPACE;
  return launch_rc(kt_launch_ep_plan(topk_ids, topk_weights, tokens, (int)top_k, owner, local, n_experts, n_ranks,
                                     (int32_t*)workspace, counts, send_token, meta, row_of, S(stream)));
}

KT_EXPORT int kt_ep_pack(const void* x, int64_t hidden, const int32_t* send_token, int64_t rows, void* out,
                         void* stream) {
  if (hidden <= 0 || rows < 0) return KT_ERR_ARG;
  if (rows == 0) return KT_OK;
  if (!x || !send_token || !out) return KT_ERR_ARG;
  return launch_rc(kt_launch_ep_pack(x, hidden, send_token, rows, out, S(stream)));
}

KT_EXPORT int kt_ep_combine(const void* back, const int32_t* row_of, int n_ranks, const void* shared, int64_t tokens,
                            int64_t hidden, void* out, void* stream) {
  if (tokens < 0 || hidden <= 0 || n_ranks < 1 || n_ranks > 8) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  if (!row_of || !out || (!back && !shared)) return KT_ERR_ARG;
  return launch_rc(kt_launch_ep_combine(back, row_of, n_ranks, shared, tokens, hidden, out, S(stream)));
}

KT_EXPORT int kt_ep_dispatch_p2p(const void* x, int64_t hidden, const int32_t* send_token, const int32_t* meta,
                                 int64_t top_k, const int32_t* counts_all, int rank, int n_ranks, const int64_t* peer_x,
                                 const int64_t* peer_ids, const int64_t* peer_w, int64_t rows_cap,
                                 int32_t* recv_total, void* stream) {
  if (hidden <= 0 || hidden % 8 || top_k < 1 || top_k > 32 || n_ranks < 1 || n_ranks > 8 || rank < 0 ||
      rank >= n_ranks || rows_cap < 0)
    return KT_ERR_ARG;
  if (!x || !send_token || !meta || !counts_all || !peer_x || !peer_ids || !peer_w || !recv_total) return KT_ERR_ARG;
  return launch_rc(kt_launch_ep_dispatch_p2p(x, hidden, send_token, meta, (int)top_k, counts_all, rank, n_ranks, peer_x,
                                             peer_ids, peer_w, rows_cap, recv_total, S(stream)));
}

KT_EXPORT int kt_ep_combine_p2p(const int32_t* row_of, const int32_t* counts_all, int rank, int n_ranks,
                                const int64_t* peer_y, const void* shared, int64_t tokens, int64_t hidden, void* out,
                                void* stream) {
  if (tokens < 0 || hidden <= 0 || hidden % 8 || n_ranks < 1 || n_ranks > 8 || rank < 0 || rank >= n_ranks)
    return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  if (!row_of || !counts_all || !peer_y || !out) return KT_ERR_ARG;
  return launch_rc(
      kt_launch_ep_combine_p2p(row_of, counts_all, rank, n_ranks, peer_y, shared, tokens, hidden, out, S(stream)));
}

// ------------------------------------------------------------------ CUDA IPC of exchange buffers

typedef CUresult (*PFN_getAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

static PFN_getAddressRange get_address_range() {
  static PFN_getAddressRange fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return (PFN_getAddressRange)p;
    return (PFN_getAddressRange) nullptr;
  }();
  return fn;
}

KT_EXPORT int kt_ipc_export(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) return KT_ERR_ARG;
  PFN_getAddressRange range = get_address_range();
  CUdeviceptr base = 0;
  size_t size = 0;
  if (!range || range(&base, &size, (CUdeviceptr)(uintptr_t)ptr) != CUDA_SUCCESS) return KT_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return KT_ERR_CUDA;
  memcpy(handle, &h, sizeof h);
  *offset = (size_t)((uintptr_t)ptr - (uintptr_t)base);
  return KT_OK;
}

KT_EXPORT int kt_ipc_import(const void* handle, size_t offset, void** ptr) {
  if (!handle || !ptr) return KT_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return KT_ERR_CUDA;
  *ptr = static_cast<uint8_t*>(base) + offset;
  return KT_OK;
}

KT_EXPORT int kt_ipc_close(void* ptr, size_t offset) {
  if (!ptr) return KT_ERR_ARG;
  return cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset) == cudaSuccess ? KT_OK : KT_ERR_CUDA;
}

// ------------------------------------------------------------------ allocation-free decode GEMV
// Some callers cannot hand this library device memory on every call: code that runs while a
// CUDA graph is being captured under a frozen memory pool, plugins whose host framework owns
// all of the GPU's memory, or plain C callers with no device allocator at all. For them the
// decode GEMV can use a fixed scratch area that lives in the library itself: a file-scope
// __device__ array of KT_STATIC_SCRATCH_BYTES, which every GPU that loads the library holds
// until the process exits. All calls on a device share it (see the header for the rules).

static __device__ __align__(256) uint8_t kt_static_scratch[KT_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_scratch_mu;
void* g_static_scratch_ptr[256] = {};  // device address of kt_static_scratch, per device ordinal
}  // namespace

KT_EXPORT int kt_moe_a8_vec_multi_static(const void* x, int x_dtype, int64_t tokens, int64_t cols, const void* w,
                                         int w_is_table, int n_slots, const int32_t* topk_ids, int64_t top_k,
                                         int ggml_type, int64_t rows, void* y, void* stream) {
  if (tokens < 0 || cols <= 0 || top_k <= 0 || n_slots <= 0) return KT_ERR_ARG;
  if (tokens == 0) return KT_OK;
  // the scratch this call needs must fit the fixed area
  if (kt_moe_a8_vec_workspace_size(tokens, cols, tokens * top_k, n_slots) > (size_t)KT_STATIC_SCRATCH_BYTES)
    return KT_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return KT_ERR_CUDA;
  void* scratch = nullptr;
  {
    // first call on this device: look up the array's device address with the device current
    // (the host-side name is only a stand-in, not a device address)
    std::lock_guard<std::mutex> lock(g_static_scratch_mu);
    if (!g_static_scratch_ptr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, kt_static_scratch) != cudaSuccess || !p) return KT_ERR_CUDA;
      g_static_scratch_ptr[dev] = p;
    }
    scratch = g_static_scratch_ptr[dev];
  }
  // moe_vec clears the status word at the start of every call; every other scratch byte it
  // reads is written earlier in the same call
  return moe_vec(x, x_dtype, tokens, cols, w, w_is_table, n_slots, topk_ids, top_k, ggml_type, rows, y, scratch,
                 (size_t)KT_STATIC_SCRATCH_BYTES, stream);
}

// The device status word of the last kt_moe_a8_vec_multi_static call on the current device: the
// first int of the static scratch (the GEMV's workspace layout starts with it). Reading it goes
// through the symbol itself, so it needs no address lookup and allocates nothing. The word only
// means something once a static call has run on the device.
KT_EXPORT int kt_static_scratch_status(void* stream, int* status) {
  if (!status) return KT_ERR_ARG;
  if (cudaStreamSynchronize(S(stream)) != cudaSuccess) return KT_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, kt_static_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost) != cudaSuccess)
    return KT_ERR_CUDA;
  *status = v;
  return KT_OK;
}
