"""Per-layer weight return (kt_gguf_b200.lend.LayerStreamer): every layer computes with its own
weights although they come back through two device slots on a side stream, over several
passes, and the copy statistics add up."""
import pytest
import torch

from kt_gguf_b200 import lend

pytestmark = pytest.mark.gpu


def test_layer_streamer_serves_each_layer_its_weights(cuda_device):
    g = torch.Generator().manual_seed(0)
    n, rows, cols = 7, 512, 1024
    host = [torch.randn((rows, cols), generator=g).to(torch.bfloat16).pin_memory() for _ in range(n)]
    x = torch.randn((2048, cols), generator=g).to(torch.bfloat16).to(cuda_device)
    s = lend.LayerStreamer(host, cuda_device, timing=True)
    for _ in range(3):  # passes
        outs = []
        for i in range(n):
            w = s.enter(i)
            outs.append((x @ w.t()).float().sum(dim=0))  # work on the compute stream while i+1 copies
        s.finish()
        torch.cuda.synchronize()
        for i in range(n):
            want = (x @ host[i].to(cuda_device).t()).float().sum(dim=0)
            assert torch.equal(outs[i], want), i
    st = s.stats()
    assert st["copies"] == 3 * n and st["bytes"] == 3 * n * rows * cols * 2
    assert st["copy_ms"] > 0 and st["wait_ms"] >= 0


def test_layer_streamer_rejects_pageable_host_memory(cuda_device):
    with pytest.raises(ValueError):
        lend.LayerStreamer([torch.zeros((4, 4), dtype=torch.bfloat16)], cuda_device)
