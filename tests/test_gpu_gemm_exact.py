"""The tcgen05 GEMM kernels' in-register GGUF decoders, pinned bit for bit through the C ABI.

kt_moe_gemm_routes runs the prefill layer's own GEMM kernels on a single projection: the down
projection's kernels for reductions of at most 512 (the resident-strip kernel, or the
streaming one with KT_B200_DOWN_STREAM=1) and the gate/up kernel without its SwiGLU for longer
ones. With one-hot activation rows (x_t = e_j) every output is one product w * 1.0 accumulated
in fp32 with exact zeros, so y[p, r] must equal the bf16 dequantized weight W[slot][r, j]: the
round-to-nearest-even of ggml's fp32 dequantization (the oracle's, pinned to gguf-py's golden
vectors). This is the north-star "dequantized weights bit for bit" for the weights the tensor
cores actually multiply. Random activations are checked against torch fp32 math on the same
bf16 operands."""
import numpy as np
import pytest
import torch

from kt_gguf_b200 import kernels as Kn
from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
TOL_STAGE = 4e-3  # vs fp32 math on the same bf16 operands: the bf16 output rounding

# (cols = reduction, kernel selection): 512 -> down kernels, 2048 -> gate/up kernel
PATHS = [(512, "resident"), (512, "streaming"), (2048, "gate_up")]


def _weights(qtype, slots, rows, cols, seed):
    rng = np.random.default_rng(seed)
    # arbitrary valid blocks: every code and scale bit pattern, not only encoder output
    return np.stack([synth.random_blocks(rng, qtype, rows, cols) for _ in range(slots)])


@pytest.mark.parametrize("cols,path", PATHS)
@pytest.mark.parametrize("qtype", [8, 12, 14, 21])
def test_in_gemm_dequant_bit_exact(cuda_device, monkeypatch, qtype, cols, path):
    if path == "streaming":
        monkeypatch.setenv("KT_B200_DOWN_STREAM", "1")
    else:
        monkeypatch.delenv("KT_B200_DOWN_STREAM", raising=False)
    slots, rows, top_k = 5, 512, 2
    W = _weights(qtype, slots, rows, cols, seed=qtype * 100 + cols)
    T = cols  # token j is the one-hot row e_j: together they read every column
    x = torch.zeros((T, cols), dtype=torch.bfloat16)
    x[torch.arange(T), torch.arange(T)] = 1.0
    rng = np.random.default_rng(cols + qtype)
    ids = np.stack([rng.permutation(slots)[:top_k] for _ in range(T)]).astype(np.int32)
    ids[rng.random(ids.shape) < 0.1] = -1
    Wd = torch.from_numpy(W).to(cuda_device)
    y = M.moe_gemm_routes(x.to(cuda_device), Wd, torch.from_numpy(ids.reshape(-1)).to(cuda_device), top_k, qtype, rows,
                          T)
    torch.cuda.synchronize()
    deq = O.bf16_to_f32(O.f32_to_bf16(O.dequant(qtype, W, cols)))  # [slots, rows, cols]
    flat = ids.reshape(-1)
    tok = np.arange(T * top_k) // top_k
    want = np.where((flat >= 0)[:, None], deq[np.clip(flat, 0, None), :, tok], 0.0).astype(np.float32)
    got = y.float().cpu().numpy()
    bad = got != want  # values compared (a -0 from the decoder accumulates to +0)
    assert not bad.any(), f"{bad.mean():.2e} of the outputs differ from the bf16 dequantized weights"


@pytest.mark.parametrize("cols,path", PATHS)
@pytest.mark.parametrize("qtype", [8, 12, 14, 21])
def test_gemm_routes_random_activations(cuda_device, monkeypatch, qtype, cols, path):
    if path == "streaming":
        monkeypatch.setenv("KT_B200_DOWN_STREAM", "1")
    else:
        monkeypatch.delenv("KT_B200_DOWN_STREAM", raising=False)
    slots, rows, T, top_k = 6, 768, 700, 4
    rng = np.random.default_rng(qtype + cols)
    W = np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype)
                  for _ in range(slots)])
    x = torch.randn((T, cols), generator=torch.Generator().manual_seed(cols)).to(torch.bfloat16)
    ids = torch.from_numpy(rng.integers(-1, slots, size=(T, top_k)).astype(np.int32))
    Wd = torch.from_numpy(W).to(cuda_device)
    xd, idd = x.to(cuda_device), ids.reshape(-1).to(cuda_device)
    y = M.moe_gemm_routes(xd, Wd, idd, top_k, qtype, rows, T)
    Wf = Kn.gguf_dequantize(Wd, qtype, cols, torch.bfloat16).float()
    flat = idd.long()
    tok = torch.arange(T * top_k, device=cuda_device) // top_k
    want = torch.einsum("prc,pc->pr", Wf[flat.clamp(min=0)], xd.float()[tok])
    want[flat < 0] = 0
    assert bool((y[flat < 0] == 0).all())
    assert O.rel_l2(y.float().cpu().numpy(), want.cpu().numpy()) < TOL_STAGE
    # slot tables read the same weights
    copies = [Wd[s].clone() for s in range(slots)]
    table = torch.tensor([c.data_ptr() for c in copies], dtype=torch.int64, device=cuda_device)
    yt = M.moe_gemm_routes(xd, table, idd, top_k, qtype, rows, T, table=True)
    assert torch.equal(y, yt)
