"""Pins the oracle and the B200 GEMV to the reference kernel itself: the reference's
kt_gguf_moe_multi.cu, compiled for sm_100a from the reference tree by oracle/build_ref.py
(window and per-route builds), run on the same seeded inputs.

Skipped when the reference modules were not built (no reference tree where build() ran).
"""
import numpy as np
import pytest
import torch

from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import synth
from oracle import build_ref
from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (build_ref.available("kt_ref_window") and build_ref.available("kt_ref_routes")),
                                 reason="reference kernel not built (oracle/build_ref.py)")]

CASES = [(8, 2048, 768), (8, 768, 2048), (12, 2048, 1024), (14, 512, 2048), (21, 2048, 1024), (21, 512, 2048)]


def bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def ref_mods():
    return build_ref.load_module("kt_ref_window"), build_ref.load_module("kt_ref_routes")


@pytest.mark.parametrize("qtype,cols,rows", CASES)
@pytest.mark.parametrize("tokens,top_k", [(1, 8), (3, 10), (4, 4)])
def test_window_kernel_vs_reference(cuda_device, ref_mods, qtype, cols, rows, tokens, top_k):
    win, routes = ref_mods
    slots = 12
    rng = np.random.default_rng(qtype * 7 + tokens)
    W = np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype)
                  for _ in range(slots)])
    x = torch.randn((tokens, cols), generator=torch.Generator().manual_seed(tokens + cols)).to(torch.bfloat16)
    # distinct ids within a token (router top-k), some routes on the CPU (-1)
    ids = np.stack([rng.permutation(slots)[:top_k] for _ in range(tokens)]).astype(np.int32)
    ids[rng.random(ids.shape) < 0.2] = -1
    ids_t = torch.from_numpy(ids.reshape(-1)).to(cuda_device)
    Wd = torch.from_numpy(W).to(cuda_device)
    xd = x.to(cuda_device)
    y_ref = win.kt_moe_a8_vec_multi(xd, Wd, ids_t, top_k, qtype, rows, tokens)
    y_ref_routes = routes.kt_moe_a8_vec_multi(xd, Wd, ids_t, top_k, qtype, rows, tokens)
    y = M.moe_a8_vec_multi(xd, Wd, ids_t, top_k, qtype, rows, tokens)
    torch.cuda.synchronize()
    # the reference's own claim: window and per-route builds give identical sums
    assert torch.equal(y_ref, y_ref_routes)
    # oracle pinned to the reference kernel
    want = O.moe_vec(qtype, W, O.quantize_q8_1(x.float().numpy()), ids.reshape(-1), top_k, rows, cols)
    ob = O.f32_to_bf16(want)
    rb = bits(y_ref)
    assert (ob != rb).mean() < 2e-3
    assert O.rel_l2(O.bf16_to_f32(rb), O.bf16_to_f32(ob)) < 2e-4
    # the B200 kernel against the reference kernel
    gb = bits(y)
    mismatch = (gb != rb).mean()
    print(f"\nREFPIN type={qtype} cols={cols} rows={rows} tokens={tokens} top_k={top_k}: "
          f"oracle!=ref {(ob != rb).mean():.2e}  b200!=ref {mismatch:.2e}  b200!=oracle {(gb != ob).mean():.2e}")
    # the B200 GEMV keeps the reference's per-chunk arithmetic, lane order and butterfly:
    # every output bit-identical to the reference kernel's
    assert torch.equal(y, y_ref), f"{mismatch:.2e} of the outputs differ"


@pytest.mark.parametrize("qtype,cols,rows", [(2, 2048, 512), (3, 2048, 512), (6, 512, 1024), (7, 2048, 512),
                                             (20, 2048, 512), (10, 2048, 512), (11, 512, 1024), (13, 2048, 512),
                                             (23, 2048, 512), (42, 2048, 512), (42, 512, 2048),
                                             (16, 2048, 512), (17, 2048, 512), (18, 2048, 512), (19, 2048, 512),
                                             (22, 2048, 512), (29, 2048, 512)])
@pytest.mark.parametrize("tokens,top_k", [(1, 8), (4, 4)])
def test_legacy_blocks_vs_reference(cuda_device, ref_mods, qtype, cols, rows, tokens, top_k):
    # the 32-value block types and the K-quants Q2_K / Q3_K / Q5_K / IQ4_XS of the reference's
    # switch (kt_gguf_moe_multi.cu:672-749, 880-892), on arbitrary valid blocks
    win, _ = ref_mods
    slots = 8
    rng = np.random.default_rng(qtype * 11 + tokens)
    W = np.stack([synth.random_blocks(rng, qtype, rows, cols) for _ in range(slots)])
    x = torch.randn((tokens, cols), generator=torch.Generator().manual_seed(tokens * 3 + cols)).to(torch.bfloat16)
    ids = np.stack([rng.permutation(slots)[:top_k] for _ in range(tokens)]).astype(np.int32)
    ids[rng.random(ids.shape) < 0.2] = -1
    ids_t = torch.from_numpy(ids.reshape(-1)).to(cuda_device)
    Wd, xd = torch.from_numpy(W).to(cuda_device), x.to(cuda_device)
    y_ref = win.kt_moe_a8_vec_multi(xd, Wd, ids_t, top_k, qtype, rows, tokens)
    y = M.moe_a8_vec_multi(xd, Wd, ids_t, top_k, qtype, rows, tokens)
    torch.cuda.synchronize()
    want = O.moe_vec(qtype, W, O.quantize_q8_1(x.float().numpy()), ids.reshape(-1), top_k, rows, cols)
    ob, rb, gb = O.f32_to_bf16(want), bits(y_ref), bits(y)
    print(f"\nREFPIN type={qtype} cols={cols} rows={rows} tokens={tokens} top_k={top_k}: "
          f"oracle!=ref {(ob != rb).mean():.2e}  b200!=ref {(gb != rb).mean():.2e}")
    assert (ob != rb).mean() < 2e-3  # the oracle: multiply-add contraction in the last fp32 bit
    assert torch.equal(y, y_ref), f"{(gb != rb).mean():.2e} of the outputs differ"


@pytest.mark.parametrize("qtype,cols,rows", [(12, 2048, 1024), (21, 512, 2048)])
def test_per_route_build_at_prefill_size(cuda_device, ref_mods, qtype, cols, rows):
    _, routes = ref_mods
    rng = np.random.default_rng(3)
    slots, tokens, top_k = 8, 96, 8
    W = np.stack([synth.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, qtype)
                  for _ in range(slots)])
    x = torch.randn((tokens, cols), generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    ids = torch.from_numpy(np.stack([rng.permutation(slots)[:top_k] for _ in range(tokens)]).astype(np.int32))
    xd, Wd, idd = x.to(cuda_device), torch.from_numpy(W).to(cuda_device), ids.reshape(-1).to(cuda_device)
    y_ref = routes.kt_moe_a8_vec_multi(xd, Wd, idd, top_k, qtype, rows, tokens)
    y = M.moe_a8_vec_routes(xd, Wd, idd, top_k, qtype, rows, tokens)
    assert torch.equal(y, y_ref), f"{(bits(y) != bits(y_ref)).mean():.2e} of the outputs differ"


# (name, ggml type of the projection, layer) for the decode timing: config 2's gate/up (Q4_K) and
# down (Q6_K, one route per row of the silu output), config 3's gate/up (IQ3_S, 512 experts)
SPEED_CASES = [("config2 gate/up Q4_K", "gate_up", 2), ("config2 down Q6_K", "down", 2),
               ("config3 gate/up IQ3_S", "gate_up", 3)]


@pytest.mark.parametrize("case", SPEED_CASES, ids=[c[0] for c in SPEED_CASES])
@pytest.mark.parametrize("tokens", [1, 4, 16, 64])
def test_decode_speed_vs_reference_kernel(cuda_device, ref_mods, tokens, case):
    # A decode projection of the benchmark layers timed for the reference kernel (its window
    # build up to 4 rows of activations, the per-route build above, as hot/kt_gguf_hot.py picks
    # them) and for the B200 kernel on the same inputs, warm L2, CUDA events over 50 calls each,
    # eager and as CUDA-graph replays of 20 calls (the serving engine captures decode in graphs).
    # Printed as REFSPEED; the bound only catches a gross regression.
    win, routes = ref_mods
    name, proj, cfg = case
    if cfg == 2:
        L = synth.make_layer(0, tokens, 2048, 512, 256, 8, 12, 14, n_hot=64, zipf=1.1)
    else:
        L = synth.make_layer(0, tokens, 2048, 512, 512, 10, 21, 21)
    top_k = L.topk_ids.shape[1]
    if proj == "gate_up":
        Wd, qtype, rows = torch.from_numpy(L.w13).to(cuda_device), L.type13, 2 * L.inter
        xd = L.x.to(cuda_device)
        ids, k, n = L.topk_ids.reshape(-1).contiguous().to(cuda_device), top_k, tokens
    else:  # the down GEMV: one route per row of h
        Wd, qtype, rows = torch.from_numpy(L.w2).to(cuda_device), L.type2, L.hidden
        g = torch.Generator().manual_seed(tokens)
        xd = torch.randn((tokens * top_k, L.inter), generator=g).to(torch.bfloat16).to(cuda_device)
        ids, k, n = L.topk_ids.reshape(-1).contiguous().to(cuda_device), 1, tokens * top_k
    ref = win if n <= 4 else routes

    def timed(fn, reps=50):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    def graph_timed(fn, calls=20, reps=10):
        # `calls` calls captured in one graph, so the host's launch of a replay is not what is
        # timed (a single-call graph replays no faster than the host submits it)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(calls):
                fn()
        return timed(gr.replay, reps) / calls

    # the reference kernel indexes by id and reads ids < 0 as CPU routes (skipped)
    f_ref = lambda: ref.kt_moe_a8_vec_multi(xd, Wd, ids, k, qtype, rows, n)  # noqa: E731
    f_b200 = lambda: M.moe_a8_vec_multi(xd, Wd, ids, k, qtype, rows, n)  # noqa: E731
    us_ref, us_b200 = timed(f_ref), timed(f_b200)
    g_ref, g_b200 = graph_timed(f_ref), graph_timed(f_b200)
    y_ref, y = f_ref(), f_b200()
    torch.cuda.synchronize()
    live = (ids >= 0).cpu().numpy()
    assert np.array_equal(bits(y)[live], bits(y_ref)[live])
    print(f"\nREFSPEED {name} tokens={tokens} routes={int(live.sum())}: "
          f"reference {us_ref:.1f} us  b200 {us_b200:.1f} us  ratio {us_ref / us_b200:.2f} | "
          f"graph replay: reference {g_ref:.1f} us  b200 {g_b200:.1f} us  ratio {g_ref / g_b200:.2f}")
    assert us_b200 < 3.0 * us_ref
