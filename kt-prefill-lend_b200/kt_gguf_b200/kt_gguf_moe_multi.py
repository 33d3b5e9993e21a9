"""Multi-token GGUF MoE GEMV for the KT hot experts — B200 (sm_100a) implementation.

Drop-in for the reference module sglang.srt.layers.moe.kt_gguf_moe_multi
(hot/kt_gguf_moe_multi.py): same public names, signatures and return shapes.

`moe_a8_vec_multi(X, W, ids, top_k, type, rows, tokens)`: Y [tokens*top_k, rows] in X's
dtype; route p is row block `ids[p]` of W against q8_1(X[p // top_k]); ids < 0 (experts on
the CPU) give zero rows. The routes of one slot share one read of its weights at any token
count (the reference shares it within windows of up to KT_GGUF_MOE_MAXM tokens).

`moe_a8_vec_routes(...)`: the reference's per-route build. Here both names run the same
kernel and give identical sums per route.

With table=True, W is an int64 device table of per-slot weight addresses (the reference's
KT_PTR_TABLE build for KV-lent slots, hot/kt_gguf_moe_multi.py:20-24); addresses must be
16-byte aligned.

`dense_a8_vec(X, W, type)`: a dense GGUF linear [rows, row_bytes] as a one-slot MoE.

`moe_prefill(...)`: the whole expert layer for prefill chunks on tcgen05 (no counterpart
name in the reference module; it replaces the streamer's dequant + CUTLASS group body for
resident slots).

Everything reaches CUDA through libkt_gguf_b200.so (include/kt_gguf_b200.h). There is no
CPU path: CPU tensors and non-sm_100 devices raise.
"""
import os

import torch

from . import _native as N

MAX_TOKENS = int(os.environ.get("KT_GGUF_MOE_MAXM", "4"))
MMV_Y = int(os.environ.get("KT_GGUF_MOE_MMV_Y", "2"))  # kept for compatibility; the B200 kernel sizes its own CTAs
RPW = int(os.environ.get("KT_GGUF_MOE_RPW", "4"))
DENSE = os.environ.get("KT_GGUF_DENSE_MULTI", "1") == "1"
DENSE_MMV_Y = int(os.environ.get("KT_GGUF_DENSE_MMV_Y", "4"))
DENSE_RPW = int(os.environ.get("KT_GGUF_DENSE_RPW", "1"))
DENSE_MIN_ROWS = 513
ROUTES = os.environ.get("KT_GGUF_MOE_ROUTES", "1") == "1"
# types the dense path is offered for (dense_ok), as the reference lists them
# (hot/kt_gguf_moe_multi.py:48): the K-quants and i-quants of dense GGUF shards. dense_a8_vec
# itself runs any GEMV type (SUPPORTED_TYPES), IQ2_XS, IQ1_M and Q2_0 included.
DENSE_TYPES = {2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 16, 18, 19, 20, 21, 22, 23}
# types with a decode GEMV here: every type of the reference kernel's switch
# (kt_gguf_moe_multi.cu:671-932) and its Q2_0
SUPPORTED_TYPES = set(N.SUPPORTED_TYPES)
# types of the tcgen05 prefill layer (Q8_0, Q4_K, Q6_K, IQ3_S)
PREFILL_TYPES = set(N.PREFILL_TYPES)


class _Op:
    """One build configuration of the reference's extension, as `_load` returns it
    (hot/kt_gguf_moe_multi.py:55-74): an object whose kt_moe_a8_vec_multi has the torch op's
    signature and allocation contract (kt_gguf_moe_multi.cu:653-668): X [tokens, K] fp32 /
    fp16 / bf16, W uint8 [E, row, row_bytes] (or, for a table build, the int64 table of slot
    addresses), topk_ids int32 [tokens*top_k], returning a new Y [tokens*top_k, row] in X's
    dtype. The window sizes of the reference's builds (mmv_y, rpw, KT_MAXM) have no meaning
    here: one kernel serves every configuration with the same sums per route."""

    def __init__(self, per_route: bool, table: bool):
        self.per_route, self.table = per_route, table
        self.lib = N.load()  # the C ABI library behind the op

    def kt_moe_a8_vec_multi(self, X, W, topk_ids, top_k, type, row, tokens):  # noqa: A002 (the op's argument name)
        entry = "kt_moe_a8_vec_routes" if self.per_route else "kt_moe_a8_vec_multi"
        return _vec(entry, X, W, topk_ids, int(top_k), int(type), int(row), int(tokens), self.table)


_ops: dict = {}


def _load(mmv_y=None, rpw=None, per_route=False, table=False):
    """The op of one build configuration (the reference JIT-builds one extension per
    (MAX_TOKENS, mmv_y, rpw, per_route, table); here one prebuilt library serves them all)."""
    key = (bool(per_route), bool(table))
    op = _ops.get(key)
    if op is None:
        op = _ops[key] = _Op(*key)
    return op


def enabled() -> bool:
    return os.environ.get("KT_GGUF_MOE_MULTI", "1") == "1"


def _check_common(X, W, ids, qtype, table):
    N.require_device(X)
    if qtype not in SUPPORTED_TYPES:
        raise ValueError(f"ggml type {qtype} has no B200 kernel (supported: {sorted(SUPPORTED_TYPES)})")
    if X.dim() != 2:
        raise ValueError(f"X must be [tokens, cols], got {tuple(X.shape)}")
    if ids.dtype != torch.int32:
        raise TypeError(f"topk ids must be int32 (got {ids.dtype})")
    if table:
        if W.dtype != torch.int64 or W.dim() != 1:
            raise TypeError("with table=True, W must be a 1-D int64 table of slot addresses")
    elif W.dtype != torch.uint8 or W.dim() != 3 or not W.is_contiguous():
        raise TypeError("W must be a contiguous uint8 [slots, rows, row_bytes] tensor")
    for t in (W, ids):
        if t.device != X.device:
            raise ValueError("X, W and ids must be on the same device")


_ws_sizes: dict = {}
_entries: dict = {}


def _vec(entry, X, W, ids, top_k, qtype, rows, tokens, table):
    _check_common(X, W, ids, qtype, table)
    X = X.contiguous()
    ids = ids.contiguous()
    cols = X.shape[1]
    if tokens > X.shape[0] or ids.numel() < tokens * top_k:
        raise ValueError("tokens / top_k exceed X or ids")
    if not table and W.shape[1] != rows:
        raise ValueError(f"W has {W.shape[1]} rows per slot, expected {rows}")
    if not table and W.shape[2] != N.row_bytes(qtype, cols):
        raise ValueError(f"W row bytes {W.shape[2]} do not match type {qtype} at {cols} columns")
    n_slots = W.numel() if table else W.shape[0]
    if tokens == 0:
        return torch.empty((0, rows), dtype=X.dtype, device=X.device)
    lib = N.load()
    key = (tokens, cols, tokens * top_k, n_slots)
    ws_bytes = _ws_sizes.get(key)
    if ws_bytes is None:
        ws_bytes = _ws_sizes[key] = max(256, int(lib.kt_moe_a8_vec_workspace_size(tokens, cols, tokens * top_k,
                                                                                 n_slots)))
    # Y and the call's scratch in one allocation (Y first, the scratch 256-byte aligned after it)
    y_bytes = tokens * top_k * rows * X.element_size()
    y_pad = (y_bytes + 255) & ~255
    buf = torch.empty(y_pad + ws_bytes, dtype=torch.uint8, device=X.device)
    Y = buf[:y_bytes].view(X.dtype).view(tokens * top_k, rows)
    fn = _entries.get(entry)
    if fn is None:
        fn = _entries[entry] = getattr(lib, entry)
    base = buf.data_ptr()
    N.check(fn(X.data_ptr(), N.dtype_code(X), tokens, cols, W.data_ptr(), int(table), n_slots, ids.data_ptr(), top_k,
               qtype, rows, base, base + y_pad, ws_bytes, N.stream_of(X)), entry)
    return Y


def moe_a8_vec_multi(X, W, ids, top_k, qtype, rows, tokens, table=False):
    return _vec("kt_moe_a8_vec_multi", X, W, ids, top_k, qtype, rows, tokens, table)


def moe_a8_vec_routes(X, W, ids, top_k, qtype, rows, tokens, table=False):
    """ggml_moe_a8_vec's contract at any token count: route p's rows from expert ids[p], zeros for ids < 0."""
    return _vec("kt_moe_a8_vec_routes", X, W, ids, top_k, qtype, rows, tokens, table)


def reads_table(tokens: int) -> bool:
    """Whether the hot method's kernel for a window of this many tokens reads the slot
    weights through the pointer table. Every B200 kernel does (GEMV and prefill GEMM)."""
    return enabled()


def dense_ok(x, qweight, qtype) -> bool:
    return (DENSE and 2 <= x.shape[0] <= MAX_TOKENS and qtype in DENSE_TYPES and qweight.dim() == 2
            and qweight.shape[0] >= DENSE_MIN_ROWS and qweight.dtype == torch.uint8 and qweight.is_contiguous())


def dense_a8_vec(x, qweight, qtype):
    """y = x @ W^T for a GGUF weight [rows, row_bytes], each row read once for all tokens."""
    N.require_device(x)
    if qtype not in SUPPORTED_TYPES:
        raise ValueError(f"ggml type {qtype} has no B200 kernel")
    x = x.contiguous()
    T, cols = x.shape
    rows = qweight.shape[0]
    if qweight.dtype != torch.uint8 or qweight.dim() != 2 or qweight.shape[1] != N.row_bytes(qtype, cols):
        raise TypeError("qweight must be a uint8 [rows, row_bytes] GGUF matrix matching x")
    y = torch.empty((T, rows), dtype=x.dtype, device=x.device)
    if T == 0:
        return y
    lib = N.load()
    ws = N.workspace(lib.kt_dense_a8_vec_workspace_size(T, cols), x.device)
    N.check(lib.kt_dense_a8_vec(N.ptr(x), N.dtype_code(x), T, cols, N.ptr(qweight.contiguous()), qtype, rows, N.ptr(y),
                                N.ptr(ws), ws.numel(), N.stream_of(x)), "kt_dense_a8_vec")
    return y


def moe_prefill(x, w13, w2, topk_ids, topk_weights, type13, type2, inter, table=False, out=None, workspace=None):
    """out [T, K] bf16 = sum_k w[t,k] * down(silu(gate x) * up x) over resident slots, on tcgen05.

    x [T, K] bf16; w13 [S, 2*inter, row_bytes] / w2 [S, K, row_bytes] uint8 (or int64 slot
    address tables with table=True); topk_ids [T, k] int32 slot ids (-1: not resident);
    topk_weights [T, k] float32. `workspace` (uint8, optional) is reused when large enough.
    """
    return moe_prefill_ex(x, w13, w2, topk_ids, topk_weights, type13, type2, inter, table=table, out=out,
                          workspace=workspace)


def moe_prefill_ex(x, w13, w2, topk_ids, topk_weights, type13, type2, inter, table=False, id_base=0, acc=None,
                   acc_flags=0, out=None, workspace=None):
    """moe_prefill over the expert group [id_base, id_base + S) (C ABI kt_moe_prefill_ex):
    routes with other ids contribute nothing. acc (fp32 [T, K]) with acc_flags N.KT_ACC_LOAD
    (start from acc) / N.KT_ACC_STORE (write the fp32 sum to acc, out not written) carries the
    sum across groups; returns out (bf16) or, with KT_ACC_STORE, acc."""
    N.require_device(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("the prefill path takes bf16 activations")
    if type13 not in PREFILL_TYPES or type2 not in PREFILL_TYPES:
        raise ValueError(f"ggml types {type13}/{type2}: the prefill layer takes {sorted(PREFILL_TYPES)}")
    if topk_ids.dtype != torch.int32 or topk_weights.dtype != torch.float32:
        raise TypeError("topk ids must be int32 and weights float32")
    x = x.contiguous()
    T, K = x.shape
    top_k = topk_ids.shape[1]
    n_slots = w13.numel() if table else w13.shape[0]
    if not table:
        if w13.shape[1] != 2 * inter or w13.shape[2] != N.row_bytes(type13, K):
            raise ValueError("w13 shape does not match [S, 2*inter, row_bytes(K)]")
        if w2.shape[1] != K or w2.shape[2] != N.row_bytes(type2, inter):
            raise ValueError("w2 shape does not match [S, K, row_bytes(inter)]")
    to_acc = bool(acc_flags & N.KT_ACC_STORE)
    if acc_flags:
        if acc is None or acc.dtype != torch.float32 or tuple(acc.shape) != (T, K) or not acc.is_contiguous():
            raise ValueError("acc must be a contiguous float32 [tokens, hidden] tensor")
    if out is None and not to_acc:
        out = torch.empty((T, K), dtype=torch.bfloat16, device=x.device)
    lib = N.load()
    need = lib.kt_moe_prefill_workspace_size(T, top_k, K, inter, n_slots)
    if workspace is None or workspace.numel() < need:
        workspace = N.workspace(need, x.device)
    ids, wts = topk_ids.contiguous(), topk_weights.contiguous()
    N.check(lib.kt_moe_prefill_ex(N.ptr(x), T, K, inter, N.ptr(ids), N.ptr(wts), top_k, N.ptr(w13), type13, N.ptr(w2),
                                  type2, int(table), n_slots, int(id_base), N.ptr(acc) if acc is not None else None,
                                  int(acc_flags), None if to_acc else N.ptr(out), N.ptr(workspace), workspace.numel(),
                                  N.stream_of(x)), "kt_moe_prefill_ex")
    return acc if to_acc else out


def moe_gemm_routes(X, W, ids, top_k, qtype, rows, tokens, table=False, workspace=None):
    """moe_a8_vec_routes' contract on tensor cores (C ABI kt_moe_gemm_routes): Y [tokens*top_k,
    rows] bf16, route p = W[ids[p]] . X[p // top_k] with bf16 activations, the GGUF weights
    dequantized in shared memory to bf16 and fp32 accumulation; zero rows for ids < 0. Runs the
    prefill layer's GEMM kernels for a single projection (prefill types; cols and rows
    multiples of 256)."""
    N.require_device(X)
    if X.dtype != torch.bfloat16:
        raise TypeError("moe_gemm_routes takes bf16 activations")
    if qtype not in PREFILL_TYPES:
        raise ValueError(f"ggml type {qtype}: the tensor-core path takes {sorted(PREFILL_TYPES)}")
    if ids.dtype != torch.int32:
        raise TypeError(f"topk ids must be int32 (got {ids.dtype})")
    X = X.contiguous()
    ids = ids.contiguous()
    cols = X.shape[1]
    if tokens > X.shape[0] or ids.numel() < tokens * top_k:
        raise ValueError("tokens / top_k exceed X or ids")
    if table:
        if W.dtype != torch.int64 or W.dim() != 1:
            raise TypeError("with table=True, W must be a 1-D int64 table of slot addresses")
        n_slots = W.numel()
    else:
        if W.dtype != torch.uint8 or W.dim() != 3 or W.shape[1] != rows or W.shape[2] != N.row_bytes(qtype, cols):
            raise TypeError("W must be a uint8 [slots, rows, row_bytes(cols)] GGUF tensor")
        n_slots = W.shape[0]
    Y = torch.empty((tokens * top_k, rows), dtype=torch.bfloat16, device=X.device)
    if tokens == 0:
        return Y
    lib = N.load()
    need = lib.kt_moe_gemm_routes_workspace_size(tokens, top_k, cols, rows, n_slots)
    if workspace is None or workspace.numel() < need:
        workspace = N.workspace(need, X.device)
    N.check(lib.kt_moe_gemm_routes(N.ptr(X), tokens, cols, N.ptr(ids), top_k, N.ptr(W.contiguous()), qtype, rows,
                                   int(table), n_slots, N.ptr(Y), N.ptr(workspace), workspace.numel(), N.stream_of(X)),
            "kt_moe_gemm_routes")
    return Y
