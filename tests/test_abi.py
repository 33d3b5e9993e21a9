"""The C ABI library loads and exports every symbol include/kt_gguf_b200.h declares; the
host-side argument checks answer without a GPU (no kernel is launched here)."""
import ctypes
import re
from pathlib import Path

import pytest

from kt_gguf_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "kt_gguf_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(kt_\w+)\s*\(", text, flags=re.M)))


def test_header_and_binding_agree():
    names = declared_functions()
    assert len(names) >= 20
    assert set(names) == set(N.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(N.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_host_only_queries():
    lib = N.load()
    assert lib.kt_version() >= 100
    assert lib.kt_status_string(N.KT_ERR_WORKSPACE) == b"workspace too small"
    assert N.row_bytes(12, 2048) == 1152 and N.row_bytes(14, 512) == 420 and N.row_bytes(21, 2048) == 880
    out = ctypes.c_int64()
    assert lib.kt_gguf_row_bytes(1, 256, ctypes.byref(out)) == N.KT_ERR_TYPE  # F16: not a GGUF block type here
    assert lib.kt_gguf_row_bytes(11, 256, ctypes.byref(out)) == 0 and out.value == 110
    assert lib.kt_gguf_row_bytes(12, 100, ctypes.byref(out)) == N.KT_ERR_ARG
    assert lib.kt_moe_a8_vec_workspace_size(4, 2048, 40, 512) > 4 * 2304
    offs = (ctypes.c_size_t * 8)()
    assert lib.kt_moe_prefill_workspace_layout(16384, 8, 2048, 512, 64, offs) == 0
    assert list(offs) == sorted(offs) and offs[6] % 1024 == 0 and offs[7] % 1024 == 0
    assert offs[7] - offs[6] >= 16384 * 8 * 512 * 2
    assert lib.kt_moe_prefill_workspace_size(16384, 8, 2048, 512, 64) >= offs[7] + 16384 * 8 * 2048 * 2


def test_argument_errors_before_any_launch():
    lib = N.load()
    P = ctypes.c_void_p
    # unsupported ggml type, bad dtype, bad shapes, tiny workspace: rejected on the host
    assert lib.kt_moe_a8_vec_multi(P(16), 2, 1, 2048, P(16), 0, 4, P(16), 1, 1, 64, P(16), P(16), 1 << 20,
                                   None) == N.KT_ERR_TYPE
    assert lib.kt_moe_a8_vec_multi(P(16), 7, 1, 2048, P(16), 0, 4, P(16), 1, 12, 64, P(16), P(16), 1 << 20,
                                   None) == N.KT_ERR_ARG
    assert lib.kt_moe_a8_vec_multi(P(16), 2, 1, 100, P(16), 0, 4, P(16), 1, 12, 64, P(16), P(16), 1 << 20,
                                   None) == N.KT_ERR_ARG
    assert lib.kt_moe_a8_vec_multi(P(16), 2, 1, 2048, P(16), 0, 4, P(16), 1, 12, 64, P(16), P(16), 16,
                                   None) == N.KT_ERR_WORKSPACE
    # zero tokens is a no-op
    assert lib.kt_moe_a8_vec_multi(None, 2, 0, 2048, None, 0, 4, None, 1, 12, 64, None, None, 0, None) == N.KT_OK
    assert lib.kt_moe_prefill(P(16), 16, 2048, 500, P(16), P(16), 8, P(16), 12, P(16), 14, 0, 64, P(16), P(16), 1 << 40,
                              None) == N.KT_ERR_ARG
    assert lib.kt_moe_prefill(P(16), 16, 2048, 512, P(16), P(16), 8, P(16), 12, P(16), 99, 0, 64, P(16), P(16), 1 << 40,
                              None) == N.KT_ERR_TYPE
    # the 32-value legacy blocks, Q2_K / Q3_K / Q5_K / IQ4_XS and Q2_0 have a decode GEMV but no
    # prefill GEMM
    for t in (2, 10, 11, 13, 23, 42, 16, 17, 18, 19, 22, 29):
        assert lib.kt_moe_prefill(P(16), 16, 2048, 512, P(16), P(16), 8, P(16), t, P(16), 14, 0, 64, P(16), P(16),
                                  1 << 40, None) == N.KT_ERR_TYPE
    # the group call: negative id_base, unknown flags, a missing or misaligned accumulator
    ex = lambda id_base, acc, flags, out: lib.kt_moe_prefill_ex(  # noqa: E731
        P(16), 16, 2048, 512, P(16), P(16), 8, P(16), 12, P(16), 14, 0, 8, id_base, acc, flags, out, P(16), 1 << 40,
        None)
    assert ex(-1, None, 0, P(16)) == N.KT_ERR_ARG
    assert ex(0, P(16), 4, P(16)) == N.KT_ERR_ARG
    assert ex(0, None, N.KT_ACC_LOAD, P(16)) == N.KT_ERR_ARG
    assert ex(0, P(8), N.KT_ACC_STORE, None) == N.KT_ERR_ARG
    assert ex(0, None, 0, None) == N.KT_ERR_ARG  # no accumulator to write: out is needed
    rb = ctypes.c_int64()
    assert lib.kt_gguf_row_bytes(2, 2048, ctypes.byref(rb)) == N.KT_OK and rb.value == 64 * 18
    assert lib.kt_gguf_row_bytes(7, 512, ctypes.byref(rb)) == N.KT_OK and rb.value == 16 * 24
    assert lib.kt_moe_prefill(P(16), 16, 2048, 512, P(16), P(16), 8, P(16), 12, P(16), 14, 0, 64, P(16), P(16), 64,
                              None) == N.KT_ERR_WORKSPACE
    # the permute keeps a shared-memory histogram over slots: at most 8192 slots
    assert lib.kt_moe_prefill(P(16), 16, 2048, 512, P(16), P(16), 8, P(16), 12, P(16), 14, 0, 8193, P(16), P(16),
                              1 << 40, None) == N.KT_ERR_ARG
    assert lib.kt_topk_softmax(None, 0, 256, 8, 0, None, None, None) == N.KT_OK
    # the per-route tensor-core projection: prefill types only, sizes in multiples of 256
    assert lib.kt_moe_gemm_routes(P(16), 4, 2048, P(16), 2, P(16), 10, 512, 0, 4, P(16), P(16), 1 << 40,
                                  None) == N.KT_ERR_TYPE
    assert lib.kt_moe_gemm_routes(P(16), 4, 2000, P(16), 2, P(16), 12, 512, 0, 4, P(16), P(16), 1 << 40,
                                  None) == N.KT_ERR_ARG
    assert lib.kt_moe_gemm_routes(P(16), 4, 2048, P(16), 2, P(16), 12, 500, 0, 4, P(16), P(16), 1 << 40,
                                  None) == N.KT_ERR_ARG
    assert lib.kt_moe_gemm_routes(P(16), 4, 2048, P(16), 2, P(16), 12, 512, 0, 4, P(16), P(16), 64,
                                  None) == N.KT_ERR_WORKSPACE
    assert lib.kt_moe_gemm_routes(None, 0, 2048, None, 2, None, 12, 512, 0, 4, None, None, 0, None) == N.KT_OK
    assert lib.kt_moe_gemm_routes_workspace_size(64, 2, 512, 512, 4) >= 128 * (512 + 512) * 2
    # the bounded-wait self-test: limits from 1 ms to 2 s, a workspace for the status word
    assert lib.kt_selftest_bounded_wait(None, 256, 5_000_000, None) == N.KT_ERR_ARG
    assert lib.kt_selftest_bounded_wait(P(256), 256, 10, None) == N.KT_ERR_ARG
    assert lib.kt_selftest_bounded_wait(P(256), 256, 3_000_000_000, None) == N.KT_ERR_ARG
    # the static scratch's status word needs somewhere to go
    assert lib.kt_static_scratch_status(None, None) == N.KT_ERR_ARG


def test_load_and_dense_types_follow_the_reference_module():
    from kt_gguf_b200 import kt_gguf_moe_multi as M

    # hot/kt_gguf_moe_multi.py:48
    assert M.DENSE_TYPES == {2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 16, 18, 19, 20, 21, 22, 23}
    assert M.DENSE_TYPES <= M.SUPPORTED_TYPES and M.PREFILL_TYPES <= M.SUPPORTED_TYPES
    op = M._load()
    assert op is M._load(2, 4) and op is not M._load(per_route=True) and M._load(table=True).table
    assert callable(op.kt_moe_a8_vec_multi) and hasattr(op.lib, "kt_moe_a8_vec_multi")


def test_python_front_rejects_cpu_tensors():
    import torch

    from kt_gguf_b200 import kt_gguf_moe_multi as M

    x = torch.zeros((2, 256), dtype=torch.bfloat16)
    W = torch.zeros((1, 8, 144), dtype=torch.uint8)
    ids = torch.zeros((2,), dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        M.moe_a8_vec_multi(x, W, ids, 1, 12, 8, 2)
    with pytest.raises(ValueError, match="CUDA"):
        M._load().kt_moe_a8_vec_multi(x, W, ids, 1, 12, 8, 2)
