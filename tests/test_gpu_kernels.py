"""GPU parity of the decode-path kernels against the CPU oracle (restated reference
arithmetic), through the C ABI (ctypes -> libkt_gguf_b200.so)."""
import numpy as np
import pytest
import torch

from kt_gguf_b200 import kernels as Kn
from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = np.load(__import__("pathlib").Path(__file__).with_name("golden") / "gguf_dequant.npz")
TYPES = (8, 12, 14, 21)
# decode GEMV and dequantizer only: 32-value blocks and the K-quants Q2_K / Q3_K / Q5_K / IQ4_XS
LEGACY = (2, 3, 6, 7, 20, 10, 11, 13, 23, 42, 16, 17, 18, 19, 22, 29)  # Q2_0 and the code-book i-quants too


def bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """distance in bf16 units in the last place between two bf16 bit arrays (same sign)"""
    ia = a.astype(np.int32)
    ib = b.astype(np.int32)
    ia = np.where(ia & 0x8000, 0x8000 - ia, ia)
    ib = np.where(ib & 0x8000, 0x8000 - ib, ib)
    return np.abs(ia - ib)


@pytest.mark.parametrize("qtype", TYPES + LEGACY)
def test_dequant_bit_exact_vs_golden(cuda_device, qtype):
    blocks = torch.from_numpy(GOLDEN[f"{qtype}_blocks"]).to(cuda_device)
    want = GOLDEN[f"{qtype}_values"]
    got = Kn.gguf_dequantize(blocks, qtype, 512, torch.float32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    gb = Kn.gguf_dequantize(blocks, qtype, 512, torch.bfloat16)
    assert np.array_equal(bits(gb), O.f32_to_bf16(want))
    gh = Kn.gguf_dequantize(blocks, qtype, 512, torch.float16).cpu().numpy()
    assert np.array_equal(gh, want.astype(np.float16))


# sizes that take the pipelined bf16 pass (four 256-sub-block items per SM or more): whole items,
# and a short last item whose raw run is not a 16-byte multiple (loaded by the CTA itself)
@pytest.mark.parametrize("qtype,rows,cols", [(12, 640, 8192), (14, 607, 8448), (8, 2401, 2080), (21, 600, 8192),
                                             (14, 1200, 4096)])
def test_dequant_bf16_pass_matches_fp32(cuda_device, qtype, rows, cols):
    rng = np.random.default_rng(qtype * 7 + rows)
    blocks = torch.from_numpy(synth.random_blocks(rng, qtype, rows, cols)).to(cuda_device)
    want = Kn.gguf_dequantize(blocks, qtype, cols, torch.float32).cpu().numpy()
    got = Kn.gguf_dequantize(blocks, qtype, cols, torch.bfloat16)
    torch.cuda.synchronize()
    assert np.array_equal(bits(got), O.f32_to_bf16(want).reshape(rows, cols))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("cols", [2048, 512, 768, 100])
def test_quantize_q8_1_bit_exact(cuda_device, dtype, cols):
    g = torch.Generator().manual_seed(cols)
    x = (torch.randn((7, cols), generator=g) * 3).to(dtype)
    x[3] = 0  # all-zero row: d = 0, codes 0
    got = Kn.quantize_q8_1(x.to(cuda_device)).cpu().numpy()
    want = O.quantize_q8_1(x.float().numpy())
    assert np.array_equal(got, want)


def close_enough(got_bits: np.ndarray, want: np.ndarray) -> None:
    """bf16 results vs fp32 sums computed in another order: within one bf16 ulp of the value,
    plus a slack of 1e-5 of the row's largest magnitude for rows whose sum cancels (there
    the fp32 order differences are large relative to the result)"""
    got = O.bf16_to_f32(got_bits).reshape(want.shape)
    slack = 1e-5 * np.abs(want).max(axis=-1, keepdims=True)
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + slack)


def _gemv_case(qtype, cols, rows, slots, tokens, top_k, seed, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    if qtype in LEGACY:  # no encoder here for these: arbitrary valid blocks
        W = np.stack([synth.random_blocks(rng, qtype, rows, cols) for _ in range(slots)])
    else:
        W = np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype)
                      for _ in range(slots)])
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((tokens, cols), generator=g).to(dtype)
    ids = torch.from_numpy(rng.integers(-1, slots, size=(tokens, top_k)).astype(np.int32))
    return W, x, ids


def _oracle_gemv(qtype, W, x, ids, top_k, rows, cols):
    qx = O.quantize_q8_1(x.float().numpy())
    return O.moe_vec(qtype, W, qx, ids.numpy().reshape(-1), top_k, rows, cols)


@pytest.mark.parametrize("qtype,cols,rows", [(8, 2048, 96), (8, 768, 2048), (12, 2048, 1024), (14, 512, 2048),
                                             (21, 2048, 1024), (21, 512, 2048), (12, 7168, 64),
                                             (2, 2048, 256), (3, 2048, 256), (6, 512, 512), (7, 2048, 256),
                                             (20, 2048, 256), (10, 2048, 256), (11, 512, 512), (13, 2048, 256),
                                             (23, 2048, 256), (42, 2048, 256), (42, 512, 1024),
                                             (16, 2048, 256), (17, 2048, 256), (18, 2048, 256), (19, 2048, 256),
                                             (22, 2048, 256), (29, 2048, 256), (22, 7168, 64)])
@pytest.mark.parametrize("tokens,top_k", [(1, 8), (4, 10), (16, 3)])
def test_gemv_matches_reference_arithmetic(cuda_device, qtype, cols, rows, tokens, top_k):
    slots = 6
    W, x, ids = _gemv_case(qtype, cols, rows, slots, tokens, top_k, seed=qtype + cols + tokens)
    want = _oracle_gemv(qtype, W, x, ids, top_k, rows, cols)
    Wd = torch.from_numpy(W).to(cuda_device)
    y = M.moe_a8_vec_multi(x.to(cuda_device), Wd, ids.reshape(-1).to(cuda_device), top_k, qtype, rows, tokens)
    yr = M.moe_a8_vec_routes(x.to(cuda_device), Wd, ids.reshape(-1).to(cuda_device), top_k, qtype, rows, tokens)
    assert y.shape == (tokens * top_k, rows) and y.dtype == torch.bfloat16
    assert torch.equal(y, yr)  # window and per-route contracts: identical sums per route
    got = bits(y)
    exp = O.f32_to_bf16(want)
    # same lane order and butterfly as the reference: results agree bit for bit except where
    # a multiply-add contraction differs in the last fp32 bit and that flips a bf16 rounding
    d = ulp_diff_bf16(got, exp)
    assert (d > 0).mean() < 2e-3
    close_enough(got, want)
    zero = (ids.reshape(-1) < 0).numpy()
    assert np.all(got[zero] == 0)


@pytest.mark.parametrize("qtype", TYPES + LEGACY)
def test_gemv_f32_output_and_table_mode(cuda_device, qtype):
    cols, rows, slots, tokens, top_k = (2048 if qtype != 14 else 512), 256, 5, 3, 4
    W, x, ids = _gemv_case(qtype, cols, rows, slots, tokens, top_k, seed=7 + qtype, dtype=torch.float32)
    want = _oracle_gemv(qtype, W, x, ids, top_k, rows, cols)
    Wd = torch.from_numpy(W).to(cuda_device)
    idd = ids.reshape(-1).to(cuda_device)
    y = M.moe_a8_vec_multi(x.to(cuda_device), Wd, idd, top_k, qtype, rows, tokens).cpu().numpy()
    assert np.max(np.abs(y - want)) <= 2e-6 * np.max(np.abs(want)) + 1e-12
    # pointer-table build: slots live anywhere (here: reversed copies); same sums
    copies = [Wd[s].clone() for s in range(slots)][::-1]
    table = torch.tensor([c.data_ptr() for c in copies[::-1]], dtype=torch.int64, device=cuda_device)
    yt = M.moe_a8_vec_multi(x.to(cuda_device), table, idd, top_k, qtype, rows, tokens, table=True).cpu().numpy()
    assert np.array_equal(yt.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("qtype,tokens,top_k", [(12, 1, 8), (14, 2, 8), (21, 1, 8), (21, 6, 8), (8, 2, 4)])
def test_gemv_table_slots_at_odd_addresses(cuda_device, qtype, tokens, top_k):
    # slot addresses 2 bytes past a 16-byte boundary: the kernels that stage weight tiles with bulk
    # copies (the one-launch decode path at 40 routes or fewer, the staged IQ3_S kernel) take plain
    # loads for such tiles; the sums stay those of the plain layout bit for bit
    cols, rows, slots = (2048 if qtype != 14 else 512), 256, 9
    W, x, ids = _gemv_case(qtype, cols, rows, slots, tokens, top_k, seed=5 + qtype + tokens)
    Wd = torch.from_numpy(W).to(cuda_device)
    idd = ids.reshape(-1).to(cuda_device)
    y = M.moe_a8_vec_multi(x.to(cuda_device), Wd, idd, top_k, qtype, rows, tokens)
    slot_bytes = W[0].nbytes
    buf = torch.zeros(2 + slots * slot_bytes + 64, dtype=torch.uint8, device=cuda_device)
    flat = Wd.reshape(-1)
    buf[2:2 + slots * slot_bytes] = flat
    base = buf.data_ptr() + 2
    assert base % 16 == 2
    table = torch.tensor([base + s * slot_bytes for s in range(slots)], dtype=torch.int64, device=cuda_device)
    yt = M.moe_a8_vec_multi(x.to(cuda_device), table, idd, top_k, qtype, rows, tokens, table=True)
    assert np.array_equal(bits(yt), bits(y))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("qtype", (8, 12, 14, 21, 2, 16, 42))
def test_gemv_one_launch_path_matches_grouped_path(cuda_device, qtype, dtype):
    # up to 40 routes take the one-launch path (the activation row quantized inside each CTA,
    # 8 values per thread); more routes take the quantize-and-group launch and the grouped GEMV
    # (32 values per warp). The same routes give the same bits either way; zero and negative-zero
    # blocks and large values included.
    cols, rows, slots, top_k = (2048 if qtype != 14 else 512), 256, 6, 8
    W, x, ids = _gemv_case(qtype, cols, rows, slots, 6, top_k, seed=19 + qtype, dtype=dtype)
    x[0, :32] = 0.0
    x[1, 32:64] = -0.0
    x[1, 64:96] *= 300.0
    Wd = torch.from_numpy(W).to(cuda_device)
    y6 = M.moe_a8_vec_multi(x.to(cuda_device), Wd, ids.reshape(-1).to(cuda_device), top_k, qtype, rows, 6)
    y2 = M.moe_a8_vec_multi(x[:2].contiguous().to(cuda_device), Wd, ids[:2].reshape(-1).contiguous().to(cuda_device),
                            top_k, qtype, rows, 2)
    assert y2.shape[0] == 2 * top_k
    assert torch.equal(y2.view(torch.uint8), y6[:2 * top_k].view(torch.uint8))


def test_gemv_many_routes_per_slot(cuda_device):
    # a decode window where one slot gets far more routes than the reference's window (4)
    qtype, cols, rows = 12, 2048, 512
    W, x, _ = _gemv_case(qtype, cols, rows, 2, 40, 1, seed=11)
    ids = torch.zeros((40, 1), dtype=torch.int32)
    ids[::7] = 1
    want = _oracle_gemv(qtype, W, x, ids, 1, rows, cols)
    y = M.moe_a8_vec_multi(x.to(cuda_device), torch.from_numpy(W).to(cuda_device), ids.reshape(-1).to(cuda_device), 1,
                           qtype, rows, 40)
    d = ulp_diff_bf16(bits(y), O.f32_to_bf16(want))
    assert (d > 0).mean() < 2e-3
    close_enough(bits(y), want)


# every type dense_ok offers (the reference's DENSE_TYPES) and the three the GEMV adds
# (IQ2_XS, IQ1_M, Q2_0: dense_a8_vec runs them, dense_ok does not offer them)
@pytest.mark.parametrize("qtype", sorted(M.DENSE_TYPES) + [17, 29, 42])
@pytest.mark.parametrize("tokens", [2, 4])
def test_dense_a8_vec(cuda_device, qtype, tokens):
    cols, rows = (512 if qtype in (6, 11, 14) else 2048), 640
    rng = np.random.default_rng(5 + qtype)
    if qtype in TYPES:
        W = synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype)
    else:
        W = synth.random_blocks(rng, qtype, rows, cols)
    x = torch.randn((tokens, cols), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    want = _oracle_gemv(qtype, W[None], x, torch.zeros(tokens, dtype=torch.int32), 1, rows, cols)
    assert M.dense_ok(x, torch.from_numpy(W), qtype) == (qtype in M.DENSE_TYPES)
    y = M.dense_a8_vec(x.to(cuda_device), torch.from_numpy(W).to(cuda_device), qtype)
    assert y.shape == (tokens, rows)
    close_enough(bits(y), want)
    # the reference's own route to it: the one-slot MoE op of the dense build
    # (hot/kt_gguf_moe_multi.py:103-112)
    zero_ids = torch.zeros(tokens, dtype=torch.int32, device=cuda_device)
    Wd = torch.from_numpy(W).to(cuda_device)
    y_op = M._load(M.DENSE_MMV_Y, M.DENSE_RPW).kt_moe_a8_vec_multi(x.to(cuda_device), Wd.view(1, rows, -1), zero_ids,
                                                                    1, qtype, rows, tokens)
    assert torch.equal(y_op.view(tokens, rows), y)


@pytest.mark.parametrize("per_route,table", [(False, False), (True, False), (False, True)])
def test_load_returns_the_reference_op(cuda_device, per_route, table):
    # _load(...).kt_moe_a8_vec_multi(X, W, ids, top_k, type, row, tokens): the op signature of
    # kt_gguf_moe_multi.cu:653-660, a new Y per call, the same sums as the module functions
    qtype, cols, rows, slots, tokens, top_k = 12, 2048, 512, 6, 3, 8
    W, x, ids = _gemv_case(qtype, cols, rows, slots, tokens, top_k, seed=21)
    Wd = torch.from_numpy(W).to(cuda_device)
    xd, idd = x.to(cuda_device), ids.reshape(-1).to(cuda_device)
    want = M.moe_a8_vec_multi(xd, Wd, idd, top_k, qtype, rows, tokens)
    Warg = torch.tensor([Wd[s].data_ptr() for s in range(slots)], dtype=torch.int64, device=cuda_device) if table \
        else Wd
    op = M._load(per_route=per_route, table=table)
    y1 = op.kt_moe_a8_vec_multi(xd, Warg, idd, top_k, qtype, rows, tokens)
    y2 = op.kt_moe_a8_vec_multi(xd, Warg, idd, top_k, qtype, rows, tokens)
    assert y1.shape == (tokens * top_k, rows) and y1.dtype == xd.dtype
    assert y1.data_ptr() != y2.data_ptr()  # a new output per call, as the op allocates one
    assert torch.equal(y1, want) and torch.equal(y2, want)


def test_silu_and_mul_and_combine(cuda_device):
    g = torch.Generator().manual_seed(9)
    h13 = torch.randn((33, 2 * 96), generator=g).to(torch.bfloat16)
    h = Kn.silu_and_mul(h13.to(cuda_device))
    want = O.silu_and_mul_bf16(bits(h13))
    assert ulp_diff_bf16(bits(h), want).max() <= 1
    out = torch.randn((9, 8, 200), generator=g).to(torch.bfloat16)
    w = torch.rand((9, 8), generator=g)
    res = Kn.combine(out.to(cuda_device), w.to(cuda_device))
    assert np.array_equal(bits(res), O.combine_bf16(bits(out), w.numpy()))


def test_hot_route(cuda_device):
    E = 32
    g = torch.Generator().manual_seed(2)
    log2slot = torch.full((E,), -1, dtype=torch.int32)
    log2slot[torch.randperm(E, generator=g)[:12]] = torch.arange(12, dtype=torch.int32)
    log2cpu = torch.where(log2slot >= 0, torch.tensor(-1, dtype=torch.int32), torch.arange(E, dtype=torch.int32))
    ids = torch.randint(0, E, (6, 8), generator=g, dtype=torch.int32)
    counts = torch.zeros(E, device=cuda_device)
    s, c = Kn.hot_route(ids.to(cuda_device), log2slot.to(cuda_device), log2cpu.to(cuda_device), counts)
    assert torch.equal(s.cpu(), log2slot[ids.long()]) and torch.equal(c.cpu(), log2cpu[ids.long()])
    assert torch.equal(counts.cpu(), torch.bincount(ids.reshape(-1).long(), minlength=E).float())


@pytest.mark.parametrize("E,k", [(16, 4), (256, 8), (512, 10)])
def test_topk_softmax(cuda_device, E, k):
    g = torch.Generator().manual_seed(E)
    logits = torch.randn((70, E), generator=g)
    w, ids = Kn.topk_softmax(logits.to(cuda_device), k)
    p = torch.softmax(logits, -1)
    rw, rids = torch.topk(p, k, -1)
    assert torch.equal(ids.cpu().long(), rids)
    assert torch.allclose(w.cpu(), rw, rtol=1e-5, atol=1e-7)
    w2, ids2 = Kn.topk_softmax(logits.to(cuda_device), k, renormalize=True)
    assert torch.allclose(w2.cpu().sum(-1), torch.ones(70), atol=1e-5)


def test_topk_grouped_deepseek(cuda_device):
    T, E, G, TG, k = 50, 256, 8, 4, 8
    g = torch.Generator().manual_seed(1)
    logits = torch.randn((T, E), generator=g)
    bias = torch.randn((E,), generator=g) * 0.1
    w, ids = Kn.topk_grouped(logits.to(cuda_device), bias.to(cuda_device), G, TG, k, True, 2.5)
    s = torch.sigmoid(logits)
    sel = s + bias
    gs = sel.view(T, G, -1).topk(2, -1).values.sum(-1)
    keep = torch.zeros((T, G), dtype=torch.bool).scatter_(1, gs.topk(TG, -1).indices, True)
    sel = sel.masked_fill(~keep.repeat_interleave(E // G, 1), float("-inf"))
    rids = sel.topk(k, -1).indices
    rw = s.gather(1, rids)
    rw = rw / rw.sum(-1, keepdim=True) * 2.5
    assert torch.equal(ids.cpu().long(), rids)
    assert torch.allclose(w.cpu(), rw, rtol=1e-5, atol=1e-6)
