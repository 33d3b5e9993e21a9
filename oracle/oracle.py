"""CPU oracle for the GGUF hot-expert MoE path — TEST INFRASTRUCTURE ONLY.

numpy/ctypes front of libkt_oracle.so (kt_oracle.c, a C restatement of the reference's
arithmetic; see its header for the reference lines each function follows). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference leg use it, as the
checker; the product (kt_gguf_b200) never imports it.

Parity pin: the dequantizers are checked bit-for-bit against gguf-py 0.19.0 on the
committed golden vectors (tests/golden/gguf_dequant.npz, made by
tests/golden/make_golden.py), and the IQ3_S codebook against the reference's own table.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libkt_oracle.so"
BLOCK = {8: (32, 34), 12: (256, 144), 14: (256, 210), 21: (256, 110),
         2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 20: (32, 18),
         10: (256, 84), 11: (256, 110), 13: (256, 176), 23: (256, 136), 42: (64, 18),
         16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 22: (256, 82), 29: (256, 56)}

_lib = None


def build(force: bool = False) -> Path:
    newest = max((HERE / f).stat().st_mtime for f in ("kt_oracle.c", "kt_cpu_simd.c"))
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
        subprocess.run(["make", "-C", str(HERE), "-B" if force else "libkt_oracle.so"], check=True,
                       capture_output=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.ko_block_info.argtypes = [I, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.ko_dequant_rows.argtypes = [I, P, I64, I64, P]
        L.ko_q8_1_row_bytes.argtypes = [I64]
        L.ko_q8_1_row_bytes.restype = I64
        L.ko_quantize_q8_1.argtypes = [P, I64, I64, P]
        L.ko_moe_vec.argtypes = [I, P, I64, P, I64, P, I64, I64, I64, I64, P]
        L.ko_silu_and_mul_bf16.argtypes = [P, I64, I64, P]
        L.ko_combine_bf16.argtypes = [P, P, I64, I64, I64, P]
        L.ko_moe_ref_bf16.argtypes = [P, I64, I64, I64, P, P, I64, I, P, I, P, I64, P]
        L.ko_moe_fp32.argtypes = [P, I64, I64, I64, P, P, I64, I, P, I, P, I64, P]
        L.kc_moe_layer.argtypes = [P, I64, I64, I64, P, P, I64, I, P, I, P, I64, P]
        L.kc_simd_available.argtypes = []
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    os.environ["OMP_NUM_THREADS"] = str(n)


# ---------------------------------------------------------------- bf16 helpers (numpy)

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """round to nearest even, as uint16 bit patterns"""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def row_bytes(qtype: int, cols: int) -> int:
    qk, bs = BLOCK[qtype]
    return cols // qk * bs


# ---------------------------------------------------------------- restated reference arithmetic

def dequant(qtype: int, w: np.ndarray, cols: int) -> np.ndarray:
    """GGUF rows [..., row_bytes] -> fp32 [..., cols] (ggml order, bit-exact)."""
    w = _c(w, np.uint8)
    rows = w.size // row_bytes(qtype, cols)
    out = np.empty((*w.shape[:-1], cols), dtype=np.float32)
    if lib().ko_dequant_rows(qtype, _p(w), rows, cols, _p(out)):
        raise ValueError("ko_dequant_rows failed")
    return out


def q8_1_row_bytes(cols: int) -> int:
    return int(lib().ko_q8_1_row_bytes(cols))


def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    rows, cols = x.shape
    out = np.empty((rows, q8_1_row_bytes(cols)), dtype=np.uint8)
    lib().ko_quantize_q8_1(_p(x), rows, cols, _p(out))
    return out


def _slot_ptrs(w: np.ndarray):
    w = _c(w, np.uint8)
    ptrs = (ctypes.c_void_p * w.shape[0])(*[w.ctypes.data + i * w[0].nbytes for i in range(w.shape[0])])
    return w, ptrs


def moe_vec(qtype: int, w: np.ndarray, qx: np.ndarray, ids: np.ndarray, top_k: int, rows: int, cols: int) -> np.ndarray:
    """moe_vec_q in the reference's lane order: fp32 [routes, rows] before the output cast."""
    w, ptrs = _slot_ptrs(w)
    qx = _c(qx, np.uint8)
    ids = _c(ids, np.int32).reshape(-1)
    out = np.empty((ids.size, rows), dtype=np.float32)
    if lib().ko_moe_vec(qtype, ctypes.cast(ptrs, ctypes.c_void_p), w.shape[0], _p(qx), qx.shape[1], _p(ids), ids.size,
                        top_k, rows, cols, _p(out)):
        raise ValueError("ko_moe_vec failed")
    return out


def silu_and_mul_bf16(h13: np.ndarray) -> np.ndarray:
    h13 = _c(h13, np.uint16)
    rows, two_n = h13.shape
    out = np.empty((rows, two_n // 2), dtype=np.uint16)
    lib().ko_silu_and_mul_bf16(_p(h13), rows, two_n // 2, _p(out))
    return out


def combine_bf16(out: np.ndarray, w: np.ndarray) -> np.ndarray:
    """out [T, top_k, K] bf16 bits, w [T, top_k] fp32 -> [T, K] bf16 bits (the reference combine)."""
    out = _c(out, np.uint16)
    w = _c(w, np.float32)
    T, top_k, K = out.shape
    res = np.empty((T, K), dtype=np.uint16)
    lib().ko_combine_bf16(_p(out), _p(w), T, top_k, K, _p(res))
    return res


def moe_ref_bf16(x_bf16: np.ndarray, ids: np.ndarray, w: np.ndarray, type13: int, w13: np.ndarray, type2: int,
                 w2: np.ndarray, inter: int) -> np.ndarray:
    """The reference hot-expert layer (q8_1 GEMVs, bf16 intermediates, reference combine)."""
    x = _c(x_bf16, np.uint16)
    T, K = x.shape
    ids = _c(ids, np.int32)
    w = _c(w, np.float32)
    w13, p13 = _slot_ptrs(w13)
    w2, p2 = _slot_ptrs(w2)
    res = np.empty((T, K), dtype=np.uint16)
    rc = lib().ko_moe_ref_bf16(_p(x), T, K, inter, _p(ids), _p(w), ids.shape[1], type13, ctypes.cast(p13, ctypes.c_void_p),
                               type2, ctypes.cast(p2, ctypes.c_void_p), w13.shape[0], _p(res))
    if rc:
        raise ValueError("ko_moe_ref_bf16 failed")
    return res


def moe_fp32(x_bf16: np.ndarray, ids: np.ndarray, w: np.ndarray, type13: int, w13: np.ndarray, type2: int,
             w2: np.ndarray, inter: int) -> np.ndarray:
    """fp32 dequant-then-matmul oracle with double accumulation: [T, K] fp32."""
    x = _c(x_bf16, np.uint16)
    T, K = x.shape
    ids = _c(ids, np.int32)
    w = _c(w, np.float32)
    w13, p13 = _slot_ptrs(w13)
    w2, p2 = _slot_ptrs(w2)
    out = np.empty((T, K), dtype=np.float32)
    rc = lib().ko_moe_fp32(_p(x), T, K, inter, _p(ids), _p(w), ids.shape[1], type13, ctypes.cast(p13, ctypes.c_void_p),
                           type2, ctypes.cast(p2, ctypes.c_void_p), w13.shape[0], _p(out))
    if rc:
        raise ValueError("ko_moe_fp32 failed")
    return out


def simd_available() -> bool:
    """whether this host runs the SIMD CPU baseline (AVX-512 with VNNI)"""
    return bool(lib().kc_simd_available())


def moe_cpu_simd(x_bf16: np.ndarray, ids: np.ndarray, w: np.ndarray, type13: int, w13: np.ndarray, type2: int,
                 w2: np.ndarray, inter: int) -> np.ndarray:
    """The reference hot-expert layer with the SIMD dot products of kt_cpu_simd.c (the timed
    CPU baseline; Q4_K / Q6_K / Q8_0): bf16 bits [T, K], as moe_ref_bf16 up to the fp32
    summation order of the per-block terms."""
    x = _c(x_bf16, np.uint16)
    T, K = x.shape
    ids = _c(ids, np.int32)
    w = _c(w, np.float32)
    w13, p13 = _slot_ptrs(w13)
    w2, p2 = _slot_ptrs(w2)
    res = np.empty((T, K), dtype=np.uint16)
    rc = lib().kc_moe_layer(_p(x), T, K, inter, _p(ids), _p(w), ids.shape[1], type13, ctypes.cast(p13, ctypes.c_void_p),
                            type2, ctypes.cast(p2, ctypes.c_void_p), w13.shape[0], _p(res))
    if rc:
        raise ValueError("kc_moe_layer failed (%s)" % ("no AVX-512 VNNI" if rc == -2 else "unsupported type"))
    return res


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
