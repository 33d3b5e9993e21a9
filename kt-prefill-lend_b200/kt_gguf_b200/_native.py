"""ctypes binding of libkt_gguf_b200.so (the C ABI in include/kt_gguf_b200.h).

The library is built in-tree (python -m kt_gguf_b200.build) and loaded from
kt_gguf_b200/lib/. There is no fallback: if the library is missing, or the GPU is not an
sm_100 part, every entry point raises.
"""
import ctypes
import threading
from pathlib import Path

import torch

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIB_PATH = LIB_DIR / "libkt_gguf_b200.so"

KT_OK, KT_ERR_ARG, KT_ERR_TYPE, KT_ERR_WORKSPACE, KT_ERR_CUDA, KT_ERR_DEVICE = range(6)
KT_DEV_OK, KT_DEV_TIMEOUT = 0, 1
KT_ACC_LOAD, KT_ACC_STORE = 1, 2  # kt_moe_prefill_ex accumulator flags
GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_IQ4_NL = 2, 3, 6, 7, 20
GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_IQ3_S = 8, 12, 14, 21
GGML_Q2_K, GGML_Q3_K, GGML_Q5_K, GGML_IQ4_XS = 10, 11, 13, 23
GGML_Q2_0 = 42  # the reference's 64-value 2-bit block (kt_gguf_moe_multi.cu:33-46)
GGML_IQ2_XXS, GGML_IQ2_XS, GGML_IQ3_XXS, GGML_IQ1_S, GGML_IQ2_S, GGML_IQ1_M = 16, 17, 18, 19, 22, 29
# types of the prefill layer (tcgen05 GEMMs) ...
PREFILL_TYPES = (GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_IQ3_S)
# ... and of the decode GEMV, the dense GEMV and the dequantizer
SUPPORTED_TYPES = PREFILL_TYPES + (GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q5_1, GGML_IQ4_NL,
                                   GGML_Q2_K, GGML_Q3_K, GGML_Q5_K, GGML_IQ4_XS, GGML_Q2_0,
                                   GGML_IQ2_XXS, GGML_IQ2_XS, GGML_IQ3_XXS, GGML_IQ1_S, GGML_IQ2_S, GGML_IQ1_M)
DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_P, _I, _I64, _SZ, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
# name -> (restype, argtypes); every function declared in include/kt_gguf_b200.h
SIGNATURES = {
    "kt_version": (_I, []),
    "kt_status_string": (ctypes.c_char_p, [_I]),
    "kt_device_supported": (_I, []),
    "kt_gguf_row_bytes": (_I, [_I, _I64, ctypes.POINTER(_I64)]),
    "kt_workspace_status": (_I, [_P, _P, ctypes.POINTER(_I)]),
    "kt_quantize_q8_1": (_I, [_P, _I, _I64, _I64, _P, _P]),
    "kt_moe_a8_vec_workspace_size": (_SZ, [_I64, _I64, _I64, _I]),
    "kt_moe_a8_vec_multi": (_I, [_P, _I, _I64, _I64, _P, _I, _I, _P, _I64, _I, _I64, _P, _P, _SZ, _P]),
    "kt_moe_a8_vec_routes": (_I, [_P, _I, _I64, _I64, _P, _I, _I, _P, _I64, _I, _I64, _P, _P, _SZ, _P]),
    "kt_moe_a8_vec_multi_static": (_I, [_P, _I, _I64, _I64, _P, _I, _I, _P, _I64, _I, _I64, _P, _P]),
    "kt_static_scratch_status": (_I, [_P, ctypes.POINTER(_I)]),
    "kt_selftest_bounded_wait": (_I, [_P, _SZ, _I64, _P]),
    "kt_moe_gemm_routes_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _I]),
    "kt_moe_gemm_routes": (_I, [_P, _I64, _I64, _P, _I64, _P, _I, _I64, _I, _I, _P, _P, _SZ, _P]),
    "kt_ep_plan_workspace_size": (_SZ, [_I64, _I]),
    "kt_ep_plan": (_I, [_P, _P, _I64, _I64, _P, _P, _I, _I, _P, _P, _P, _P, _P, _SZ, _P]),
    "kt_ep_pack": (_I, [_P, _I64, _P, _I64, _P, _P]),
    "kt_ep_combine": (_I, [_P, _P, _I, _P, _I64, _I64, _P, _P]),
    "kt_ep_dispatch_p2p": (_I, [_P, _I64, _P, _P, _I64, _P, _I, _I, _P, _P, _P, _I64, _P, _P]),
    "kt_ep_combine_p2p": (_I, [_P, _P, _I, _I, _P, _P, _I64, _I64, _P, _P]),
    "kt_ipc_export": (_I, [_P, _P, ctypes.POINTER(_SZ)]),
    "kt_ipc_import": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "kt_ipc_close": (_I, [_P, _SZ]),
    "kt_moe_prefill_counted": (_I, [_P, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I, _I, _I, _P, _P, _SZ,
                                    _P]),
    "kt_dense_a8_vec_workspace_size": (_SZ, [_I64, _I64]),
    "kt_dense_a8_vec": (_I, [_P, _I, _I64, _I64, _P, _I, _I64, _P, _P, _SZ, _P]),
    "kt_gguf_dequantize": (_I, [_P, _I, _I64, _I64, _P, _I, _P]),
    "kt_silu_and_mul": (_I, [_P, _I, _I64, _I64, _P, _P]),
    "kt_moe_combine": (_I, [_P, _I, _P, _I64, _I64, _I64, _P, _P]),
    "kt_hot_route": (_I, [_P, _I64, _P, _P, _P, _P, _P, _P]),
    "kt_topk_softmax": (_I, [_P, _I64, _I, _I, _I, _P, _P, _P]),
    "kt_topk_grouped": (_I, [_P, _P, _I64, _I, _I, _I, _I, _I, _F, _P, _P, _P]),
    "kt_moe_prefill_workspace_size": (_SZ, [_I64, _I64, _I64, _I64, _I]),
    "kt_moe_prefill_predequant": (_I, [_I64, _I64, _I64, _I64, _I]),
    "kt_moe_prefill_workspace_layout": (_I, [_I64, _I64, _I64, _I64, _I, ctypes.POINTER(_SZ)]),
    "kt_moe_prefill": (_I, [_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "kt_moe_prefill_timed": (_I, [_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I, _I, _I, _P, _P, _SZ, _P,
                                  ctypes.POINTER(_P)]),
    "kt_moe_prefill_ex": (_I, [_P, _I64, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I, _I, _I, _I, _P, _I, _P, _P, _SZ,
                               _P]),
}

_lib = None
_lock = threading.Lock()
_device_checked = set()


def load(path=None) -> ctypes.CDLL:
    """Loads the library (once) and declares every C ABI signature."""
    global _lib
    if _lib is not None and path is None:  # the per-call path: no lock once loaded
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise ImportError(f"{p} is missing; build it with `python -m kt_gguf_b200.build`")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


class KtError(RuntimeError):
    def __init__(self, code: int, where: str):
        super().__init__(f"{where}: {load().kt_status_string(code).decode()} (status {code})")
        self.code = code


def check(code: int, where: str) -> None:
    if code != KT_OK:
        raise KtError(code, where)


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """cudaStream_t of the current stream on t's device"""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def require_device(t: torch.Tensor) -> None:
    """The tensor must live on an sm_100 GPU; the library has no CPU path."""
    if not t.is_cuda:
        raise ValueError("kt_gguf_b200 runs on CUDA tensors only (no CPU path)")
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if dev not in _device_checked:
        with torch.cuda.device(dev):
            if not load().kt_device_supported():
                raise RuntimeError(f"cuda:{dev} is not an sm_100 GPU; libkt_gguf_b200 is built for sm_100a only")
        _device_checked.add(dev)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"activation dtype {t.dtype} is not float32/float16/bfloat16") from None


_row_bytes_cache: dict = {}


def row_bytes(qtype: int, cols: int) -> int:
    key = (qtype, cols)
    v = _row_bytes_cache.get(key)
    if v is None:
        out = ctypes.c_int64(0)
        check(load().kt_gguf_row_bytes(qtype, cols, ctypes.byref(out)), "kt_gguf_row_bytes")
        v = _row_bytes_cache[key] = out.value
    return v


def workspace(nbytes: int, device) -> torch.Tensor:
    """Scratch from torch's caching allocator (graph-capture safe, like the reference's
    torch::empty in kt_moe_a8_vec_multi)."""
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def workspace_status(ws: torch.Tensor) -> int:
    st = ctypes.c_int(0)
    check(load().kt_workspace_status(ptr(ws), stream_of(ws), ctypes.byref(st)), "kt_workspace_status")
    return st.value
