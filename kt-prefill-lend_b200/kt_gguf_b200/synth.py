"""Seeded synthetic inputs for the benchmark configurations and the tests.

The reference is measured on real GGUF checkpoints; no checkpoint or dataset is available
here, so every input is generated from a seed with the shapes and value distributions of
the benchmark configurations: expert weights fp32 N(0, 0.02) quantized to the config's
GGUF types with gguf_encode.c (lib/libkt_gguf_encode.so), activations N(0, 1), router
logits N(0, 1) (plus a log-space Zipf(1.1) per-expert bias where the config asks for a
skewed load).
"""
import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np
import torch

ENC_PATH = Path(__file__).resolve().parent / "lib" / "libkt_gguf_encode.so"
BLOCK = {8: (32, 34), 12: (256, 144), 14: (256, 210), 21: (256, 110),
         2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 20: (32, 18),
         10: (256, 84), 11: (256, 110), 13: (256, 176), 23: (256, 136), 42: (64, 18),
         16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 22: (256, 82), 29: (256, 56)}
_enc = None


def _encoder():
    global _enc
    if _enc is None:
        if not ENC_PATH.exists():
            raise ImportError(f"{ENC_PATH} is missing; build it with `python -m kt_gguf_b200.build`")
        _enc = ctypes.CDLL(str(ENC_PATH))
        _enc.kte_quantize.restype = ctypes.c_int
        _enc.kte_quantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    return _enc


def row_bytes(qtype: int, cols: int) -> int:
    qk, bs = BLOCK[qtype]
    assert cols % qk == 0, (qtype, cols)
    return cols // qk * bs


def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    """fp32 [..., cols] -> uint8 [..., row_bytes] GGUF blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.empty((*x.shape[:-1], row_bytes(qtype, cols)), dtype=np.uint8)
    rc = _encoder().kte_quantize(qtype, x.ctypes.data, rows, cols, out.ctypes.data)
    if rc:
        raise ValueError(f"kte_quantize({qtype}) failed: {rc}")
    return out


def random_blocks(rng: np.random.Generator, qtype: int, rows: int, cols: int) -> np.ndarray:
    """Arbitrary bytes that are valid blocks of the type, with finite fp16 scales in a
    realistic range; exercises every bit pattern of the codes, not only encoder output."""
    qk, bs = BLOCK[qtype]
    nb = rows * cols // qk
    b = rng.integers(0, 256, size=(nb, bs), dtype=np.uint8)
    def put_f16(off, lo, hi):
        v = rng.uniform(lo, hi, size=nb).astype(np.float16)
        b[:, off:off + 2] = v.view(np.uint8).reshape(nb, 2)
    if qtype == 8:
        put_f16(0, -1e-3, 1e-3)
    elif qtype == 12:
        put_f16(0, 0, 2e-3)
        put_f16(2, 0, 2e-3)
    elif qtype == 14:
        put_f16(208, -2e-4, 2e-4)
    elif qtype == 21:
        put_f16(0, 0, 2e-4)
    elif qtype in (2, 6, 20, 42):  # d
        put_f16(0, -2e-3, 2e-3)
    elif qtype in (3, 7):  # d, m
        put_f16(0, 0, 2e-3)
        put_f16(2, -2e-2, 2e-2)
    elif qtype == 10:  # d, dmin at the block's end
        put_f16(80, 0, 2e-3)
        put_f16(82, 0, 2e-3)
    elif qtype == 11:  # d
        put_f16(108, -2e-3, 2e-3)
    elif qtype == 13:  # d, dmin
        put_f16(0, 0, 2e-3)
        put_f16(2, 0, 2e-3)
    elif qtype == 23:  # d
        put_f16(0, -2e-4, 2e-4)
    elif qtype in (16, 17, 22):  # d of the IQ2 families
        put_f16(0, 0, 5e-4)
    elif qtype == 18:
        put_f16(0, 0, 3e-4)
    elif qtype == 19:
        put_f16(0, 0, 3e-3)
    elif qtype == 29:  # the fp16 d spread over the top nibbles of the four scale words
        d = rng.uniform(0, 3e-3, size=nb).astype(np.float16).view(np.uint16).astype(np.uint16)
        for k in range(4):
            hi = ((d >> (4 * k)) & 0xF).astype(np.uint8) << 4
            b[:, 49 + 2 * k] = (b[:, 49 + 2 * k] & 0x0F) | hi
    return b.reshape(rows, cols // qk * bs)


@dataclass
class MoELayer:
    """One MoE layer's inputs: slots [S, ...] of GGUF weights, activations and routing."""
    hidden: int
    inter: int
    type13: int
    type2: int
    w13: np.ndarray           # uint8 [S, 2*inter, row_bytes(hidden)]
    w2: np.ndarray            # uint8 [S, hidden, row_bytes(inter)]
    x: torch.Tensor           # bf16 [T, hidden] (CPU)
    topk_ids: torch.Tensor    # int32 [T, k] slot ids, -1 where the expert is not resident
    topk_weights: torch.Tensor  # float32 [T, k]
    logical_ids: Optional[torch.Tensor] = None  # int32 [T, k] router ids before the slot map


def expert_weights(rng, n, hidden, inter, type13, type2, scale=0.02):
    w13 = np.empty((n, 2 * inter, row_bytes(type13, hidden)), dtype=np.uint8)
    w2 = np.empty((n, hidden, row_bytes(type2, inter)), dtype=np.uint8)
    for e in range(n):
        w13[e] = quantize(rng.standard_normal((2 * inter, hidden), dtype=np.float32) * scale, type13)
        w2[e] = quantize(rng.standard_normal((hidden, inter), dtype=np.float32) * scale, type2)
    return w13, w2


def softmax_topk(logits: torch.Tensor, k: int, renormalize: bool = False):
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w.float(), ids.to(torch.int32)


def zipf_bias(rng: np.random.Generator, n_experts: int, s: float = 1.1) -> np.ndarray:
    """b_e = -s * ln(r_e) with r = 1 + a seeded permutation of 0..E-1 (log-space Zipf(s))."""
    r = 1 + rng.permutation(n_experts)
    return (-s * np.log(r)).astype(np.float32)


def make_layer(seed: int, tokens: int, hidden: int, inter: int, n_experts: int, top_k: int, type13: int, type2: int,
               n_hot: Optional[int] = None, zipf: Optional[float] = None, renormalize: bool = False,
               token_seed: Optional[int] = None) -> MoELayer:
    """Config generator: router logits N(0,1) (+ Zipf bias), softmax top-k; the n_hot experts
    with the largest bias (or the first n_hot) are resident in slots 0..n_hot-1 (hottest
    first); the others map to -1 like HotCache.route's slot ids. Weights and the bias come
    from `seed`, activations and logits from `token_seed` (default: seed), so ranks can share
    the experts and differ in tokens."""
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed if token_seed is None else token_seed)
    logits = torch.randn((tokens, n_experts), generator=g)
    hot = np.arange(n_experts) if n_hot is None else None
    if zipf is not None:
        bias = zipf_bias(rng, n_experts, zipf)
        logits = logits + torch.from_numpy(bias)
        if n_hot is not None:
            hot = np.argsort(-bias, kind="stable")[:n_hot]
    elif n_hot is not None:
        hot = np.arange(n_hot)
    w, ids = softmax_topk(logits, top_k, renormalize)
    log2slot = np.full(n_experts, -1, dtype=np.int32)
    log2slot[hot] = np.arange(len(hot), dtype=np.int32)
    slot_ids = torch.from_numpy(log2slot)[ids.long()].to(torch.int32)
    w13, w2 = expert_weights(rng, len(hot), hidden, inter, type13, type2)
    x = torch.randn((tokens, hidden), generator=g).to(torch.bfloat16)
    return MoELayer(hidden, inter, type13, type2, w13, w2, x, slot_ids.contiguous(), w.contiguous(), ids.contiguous())


# the benchmark configurations (BASELINE.json "configs")
CONFIGS = {
    1: dict(tokens=256, hidden=2048, inter=768, n_experts=16, top_k=4, type13=8, type2=8),
    2: dict(tokens=16384, hidden=2048, inter=512, n_experts=256, top_k=8, type13=12, type2=14, n_hot=64, zipf=1.1),
    3: dict(tokens=16384, hidden=2048, inter=512, n_experts=512, top_k=10, type13=21, type2=21),
}
