"""The CPU restatement of the reference arithmetic, checked against independent numpy
math (no GPU): the integer GEMV equals W_deq . deq(q8_1(x)) to fp32 rounding, the fused
combine equals mul_ + moe_sum, and the reference layer's distance to the fp32 oracle."""
import numpy as np
import pytest
import torch

from kt_gguf_b200 import synth
from oracle import oracle as O


def q8_1_dequant(qx: np.ndarray, cols: int) -> np.ndarray:
    nb = qx.shape[1] // 36
    b = qx.reshape(qx.shape[0], nb, 36)
    d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, :, 4:].view(np.int8).astype(np.float32)
    return (q * d).reshape(qx.shape[0], -1)[:, :cols]


@pytest.mark.parametrize("qtype,cols,rows", [(8, 2048, 96), (8, 768, 40), (12, 2048, 64), (14, 512, 64),
                                             (21, 2048, 48), (21, 512, 40)])
def test_gemv_integer_path_equals_dequant_matmul(qtype, cols, rows):
    rng = np.random.default_rng(qtype * 1000 + cols)
    x = rng.standard_normal((5, cols), dtype=np.float32)
    W = np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype) for _ in range(3)])
    qx = O.quantize_q8_1(x)
    ids = np.array([0, 2, -1, 1, 2, 0, 1, 1, 2, 0], dtype=np.int32)  # top_k 2, a CPU route, repeats
    y = O.moe_vec(qtype, W, qx, ids, 2, rows, cols)
    xd = q8_1_dequant(qx, cols)
    Wd = O.dequant(qtype, W, cols)
    exp = np.stack([Wd[e] @ xd[p // 2] if e >= 0 else np.zeros(rows, np.float32) for p, e in enumerate(ids)])
    assert O.rel_l2(y, exp) < 2e-6
    assert np.all(y[2] == 0)


def test_fused_combine_equals_mul_and_sum():
    # hot/kt_gguf_hot.py:297-304: the fused kernel and out.mul_(w) + moe_sum give identical bits
    g = torch.Generator().manual_seed(3)
    T, k, K = 7, 8, 96
    out = torch.randn((T, k, K), generator=g).to(torch.bfloat16)
    w = torch.rand((T, k), generator=g)
    ref = out.clone().mul_(w.view(T, k, 1).to(torch.bfloat16)).float().sum(1).to(torch.bfloat16)
    got = O.combine_bf16(out.view(torch.int16).numpy().view(np.uint16), w.numpy())
    assert np.array_equal(got, ref.view(torch.int16).numpy().view(np.uint16))


def test_silu_and_mul_bf16():
    g = torch.Generator().manual_seed(4)
    h13 = torch.randn((5, 64), generator=g).to(torch.bfloat16)
    want = (torch.nn.functional.silu(h13[:, :32].float()) * h13[:, 32:].float()).to(torch.bfloat16)
    got = O.silu_and_mul_bf16(h13.view(torch.int16).numpy().view(np.uint16))
    diff = np.abs(O.bf16_to_f32(got) - want.float().numpy())
    assert np.max(diff / (np.abs(want.float().numpy()) + 1e-6)) <= 2 ** -7


def test_reference_layer_vs_fp32_oracle_gap():
    # the reference's double int8 activation quantization keeps it about 1% (rel-L2) from
    # the fp32 dequant-then-matmul oracle on N(0,1) activations; recorded, not a target
    L = synth.make_layer(0, 32, 2048, 768, 16, 4, 8, 8)
    xb = L.x.view(torch.int16).numpy().view(np.uint16)
    ref = O.moe_ref_bf16(xb, L.topk_ids.numpy(), L.topk_weights.numpy(), 8, L.w13, 8, L.w2, 768)
    f = O.moe_fp32(xb, L.topk_ids.numpy(), L.topk_weights.numpy(), 8, L.w13, 8, L.w2, 768)
    gap = O.rel_l2(O.bf16_to_f32(ref), f)
    assert 1e-3 < gap < 3e-2


def test_masked_routes_contribute_nothing():
    L = synth.make_layer(1, 8, 512, 256, 8, 2, 14, 14, n_hot=4)
    xb = L.x.view(torch.int16).numpy().view(np.uint16)
    ids = L.topk_ids.numpy().copy()
    ids[:] = -1
    f = O.moe_fp32(xb, ids, L.topk_weights.numpy(), 14, L.w13, 14, L.w2, 256)
    r = O.moe_ref_bf16(xb, ids, L.topk_weights.numpy(), 14, L.w13, 14, L.w2, 256)
    assert np.all(f == 0) and np.all(O.bf16_to_f32(r) == 0)
