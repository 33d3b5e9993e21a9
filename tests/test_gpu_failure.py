"""The failure path of the bounded device waits, exercised without a GPU fault.

Every mbarrier wait in the tcgen05 GEMMs gives up after a time limit, records KT_DEV_TIMEOUT in
the call's status word, and the kernel drains, frees its TMEM and returns. kt_selftest_bounded_wait
runs that set-up and exit path in one CTA pair around a barrier nothing arrives on, with a
short limit; the host then reads the status word, and the context must still run a layer."""
import time

import pytest
import torch

from kt_gguf_b200 import _native as Nt
from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("limit_ms", [5, 50])
def test_bounded_wait_times_out_and_the_context_survives(cuda_device, limit_ms):
    lib = Nt.load()
    ws = torch.zeros(256, dtype=torch.uint8, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    Nt.check(lib.kt_selftest_bounded_wait(Nt.ptr(ws), ws.numel(), limit_ms * 1_000_000, Nt.stream_of(ws)),
             "kt_selftest_bounded_wait")
    assert Nt.workspace_status(ws) == Nt.KT_DEV_TIMEOUT
    elapsed = time.perf_counter() - t0
    assert limit_ms * 1e-3 <= elapsed < 5.0, elapsed
    # the context is intact: a layer afterwards runs clean and reports KT_DEV_OK
    L = synth.make_layer(seed=3, tokens=256, hidden=512, inter=256, n_experts=6, top_k=2, type13=12, type2=14)
    dev = cuda_device
    w13, w2 = torch.from_numpy(L.w13).to(dev), torch.from_numpy(L.w2).to(dev)
    need = lib.kt_moe_prefill_workspace_size(256, 2, 512, 256, w13.shape[0])
    lws = Nt.workspace(need, dev)
    out = M.moe_prefill(L.x.to(dev), w13, w2, L.topk_ids.to(dev), L.topk_weights.to(dev), 12, 14, L.inter,
                        workspace=lws)
    assert Nt.workspace_status(lws) == Nt.KT_DEV_OK
    assert bool(torch.isfinite(out).all())
