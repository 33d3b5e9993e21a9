"""The allocation-free decode GEMV entry point (kt_moe_a8_vec_multi_static).

It exists for callers that cannot give the library device memory on each call — code inside
a CUDA graph capture with a frozen memory pool, host frameworks that own all of the GPU's
memory, C callers without an allocator — and runs on a fixed 2 MiB scratch array inside the
library instead of a caller workspace. Checked through the C ABI against the workspace entry
point on two calls in a row (the second with different inputs, so stale scratch from the
first call would show), at route counts on both sides of the one-warp route grouping (up to
32 routes) and the block-wide grouping above it, plus the size limit and the status word
(kt_static_scratch_status). Collected last so that a run stopping at the first failure has run
every other test already.
"""
import ctypes

import numpy as np
import pytest
import torch

from kt_gguf_b200 import _native as Nt
from kt_gguf_b200 import synth

pytestmark = pytest.mark.gpu


def _call_static(lib, x, w, ids, top_k, qtype, rows, n_slots, y):
    return lib.kt_moe_a8_vec_multi_static(Nt.ptr(x), Nt.dtype_code(x), x.shape[0], x.shape[1], Nt.ptr(w), 0, n_slots,
                                          Nt.ptr(ids), top_k, qtype, rows, Nt.ptr(y),
                                          torch.cuda.current_stream().cuda_stream)


def _call_workspace(lib, x, w, ids, top_k, qtype, rows, n_slots, y):
    T, cols = x.shape
    ws = torch.empty(lib.kt_moe_a8_vec_workspace_size(T, cols, T * top_k, n_slots), dtype=torch.uint8, device=x.device)
    return lib.kt_moe_a8_vec_multi(Nt.ptr(x), Nt.dtype_code(x), T, cols, Nt.ptr(w), 0, n_slots, Nt.ptr(ids), top_k, qtype,
                                   rows, Nt.ptr(y), Nt.ptr(ws), ws.numel(), torch.cuda.current_stream().cuda_stream)


def _static_status(lib):
    st = ctypes.c_int(-1)
    assert lib.kt_static_scratch_status(torch.cuda.current_stream().cuda_stream, ctypes.byref(st)) == Nt.KT_OK
    return st.value


# (4, 3) tokens x top_k 8 = 32 / 24 routes: one-warp grouping; (16, 12) x 8 = 128 / 96 routes:
# the block-wide grouping with its shared-memory counters
@pytest.mark.parametrize("token_counts", [(4, 3), (16, 12)])
@pytest.mark.parametrize("qtype,cols,rows", [(12, 2048, 1024), (21, 512, 2048)])
def test_static_scratch_matches_workspace_entry_point(cuda_device, qtype, cols, rows, token_counts):
    lib = Nt.load()
    rng = np.random.default_rng(qtype)
    slots, top_k = 8, 8
    W = torch.from_numpy(np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype)
                                   for _ in range(slots)])).to(cuda_device)
    for call, tokens in enumerate(token_counts):  # two calls in a row, different inputs and sizes
        x = torch.randn((tokens, cols), generator=torch.Generator().manual_seed(call)).to(torch.bfloat16).to(cuda_device)
        ids = torch.from_numpy(np.stack([rng.permutation(slots)[:top_k] for _ in range(tokens)]).astype(np.int32))
        ids[0, 0] = -1  # a route on the CPU: zero row
        ids = ids.reshape(-1).to(cuda_device)
        y_static = torch.full((tokens * top_k, rows), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        y_ws = torch.empty_like(y_static)
        assert _call_static(lib, x, W, ids, top_k, qtype, rows, slots, y_static) == Nt.KT_OK
        assert _call_workspace(lib, x, W, ids, top_k, qtype, rows, slots, y_ws) == Nt.KT_OK
        torch.cuda.synchronize()
        # same kernels, same arithmetic: bit-identical (the GEMV tests bound it vs the oracle)
        assert torch.equal(y_static, y_ws), f"call {call}"
        assert torch.all(y_static[0] == 0)
        assert _static_status(lib) == Nt.KT_DEV_OK


def test_static_scratch_rejects_oversized_calls(cuda_device):
    lib = Nt.load()
    cols, rows, top_k, slots = 2048, 64, 8, 4
    tokens = 2048  # q8_1 rows alone need 2048 x 2304 bytes > 2 MiB
    assert lib.kt_moe_a8_vec_workspace_size(tokens, cols, tokens * top_k, slots) > (2 << 20)
    x = torch.zeros((tokens, cols), dtype=torch.bfloat16, device=cuda_device)
    W = torch.zeros((slots, rows, 8 * 144), dtype=torch.uint8, device=cuda_device)
    ids = torch.zeros((tokens * top_k,), dtype=torch.int32, device=cuda_device)
    y = torch.empty((tokens * top_k, rows), dtype=torch.bfloat16, device=cuda_device)
    assert _call_static(lib, x, W, ids, top_k, 12, rows, slots, y) == Nt.KT_ERR_WORKSPACE
    assert lib.kt_status_string(Nt.KT_ERR_WORKSPACE) == b"workspace too small"
