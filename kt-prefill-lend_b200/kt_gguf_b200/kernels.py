"""Torch-tensor wrappers of the small C ABI entry points: GGUF dequantization, the q8_1
activation quantizer, silu_and_mul, the reference combine, HotCache route lookups and
router top-k. All run on the current CUDA stream; none has a CPU path."""
import torch

from . import _native as N


def gguf_dequantize(qweight: torch.Tensor, qtype: int, cols: int, dtype=torch.float32) -> torch.Tensor:
    """[..., rows, row_bytes] GGUF bytes -> [..., rows, cols] values (fp32 bit-identical to ggml)."""
    N.require_device(qweight)
    if qweight.dtype != torch.uint8:
        raise TypeError("qweight must be uint8")
    rb = N.row_bytes(qtype, cols)
    if qweight.shape[-1] != rb:
        raise ValueError(f"row bytes {qweight.shape[-1]} != {rb} for type {qtype} at {cols} columns")
    q = qweight.contiguous()
    rows = q.numel() // rb
    out = torch.empty((*q.shape[:-1], cols), dtype=dtype, device=q.device)
    N.check(N.load().kt_gguf_dequantize(N.ptr(q), qtype, rows, cols, N.ptr(out), N.DTYPE_CODES[dtype], N.stream_of(q)),
            "kt_gguf_dequantize")
    return out


def quantize_q8_1(x: torch.Tensor) -> torch.Tensor:
    """x [rows, cols] -> q8_1 blocks as uint8 [rows, ceil(cols/512)*512/32*36]."""
    N.require_device(x)
    x = x.contiguous()
    rows, cols = x.shape
    qrow = (cols + 511) // 512 * 512 // 32 * 36
    qx = torch.empty((rows, qrow), dtype=torch.uint8, device=x.device)
    N.check(N.load().kt_quantize_q8_1(N.ptr(x), N.dtype_code(x), rows, cols, N.ptr(qx), N.stream_of(x)), "kt_quantize_q8_1")
    return qx


def silu_and_mul(h13: torch.Tensor) -> torch.Tensor:
    """[rows, 2n] -> [rows, n]: silu(h13[:, :n]) * h13[:, n:] in fp32, stored in h13's dtype."""
    N.require_device(h13)
    h13 = h13.contiguous()
    rows, two_n = h13.shape
    n = two_n // 2
    h = torch.empty((rows, n), dtype=h13.dtype, device=h13.device)
    N.check(N.load().kt_silu_and_mul(N.ptr(h13), N.dtype_code(h13), rows, n, N.ptr(h), N.stream_of(h13)), "kt_silu_and_mul")
    return h


def combine(out: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """out [T, top_k, K], w [T, top_k] -> [T, K]: sum_k dtype(out * dtype(w)) in fp32, rounded once."""
    N.require_device(out)
    T, top_k, K = out.shape
    out = out.contiguous()
    w = w.to(torch.float32).contiguous()
    res = torch.empty((T, K), dtype=out.dtype, device=out.device)
    N.check(N.load().kt_moe_combine(N.ptr(out), N.dtype_code(out), N.ptr(w), T, top_k, K, N.ptr(res), N.stream_of(out)),
            "kt_moe_combine")
    return res


def hot_route(ids: torch.Tensor, log2slot: torch.Tensor, log2cpu: torch.Tensor, counts=None):
    """HotCache.route's table lookups and count update; ids int32 logical expert ids."""
    N.require_device(ids)
    if ids.dtype != torch.int32 or log2slot.dtype != torch.int32 or log2cpu.dtype != torch.int32:
        raise TypeError("route ids and tables must be int32")
    flat = ids.contiguous().view(-1)
    slot = torch.empty_like(flat)
    cpu = torch.empty_like(flat)
    N.check(N.load().kt_hot_route(N.ptr(flat), flat.numel(), N.ptr(log2slot), N.ptr(log2cpu), N.ptr(counts), N.ptr(slot),
                                  N.ptr(cpu), N.stream_of(flat)), "kt_hot_route")
    return slot.view_as(ids), cpu.view_as(ids)


def topk_softmax(logits: torch.Tensor, k: int, renormalize: bool = False):
    N.require_device(logits)
    logits = logits.to(torch.float32).contiguous()
    T, E = logits.shape
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    N.check(N.load().kt_topk_softmax(N.ptr(logits), T, E, k, int(renormalize), N.ptr(w), N.ptr(ids), N.stream_of(logits)),
            "kt_topk_softmax")
    return w, ids


def topk_grouped(logits: torch.Tensor, bias, n_group: int, topk_group: int, k: int, renormalize=True, scale=1.0):
    N.require_device(logits)
    logits = logits.to(torch.float32).contiguous()
    T, E = logits.shape
    b = None if bias is None else bias.to(torch.float32).contiguous()
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    N.check(N.load().kt_topk_grouped(N.ptr(logits), N.ptr(b), T, E, n_group, topk_group, k, int(renormalize), float(scale),
                                     N.ptr(w), N.ptr(ids), N.stream_of(logits)), "kt_topk_grouped")
    return w, ids
