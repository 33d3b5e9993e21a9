"""The expert-parallel layer on one GPU (world of one rank): dispatch, the tcgen05 layer on the
rank's slots and the combine must reproduce kt_moe_prefill exactly (one partial per token, so
the fp32 combine adds a single bf16 value)."""
import pytest
import torch

from kt_gguf_b200 import ep as EP
from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import synth

pytestmark = pytest.mark.gpu


def test_single_rank_ep_equals_prefill_layer(cuda_device):
    L = synth.make_layer(3, 512, 2048, 512, 64, 8, 12, 14, n_hot=16, zipf=1.1)
    w13 = torch.from_numpy(L.w13).to(cuda_device)
    w2 = torch.from_numpy(L.w2).to(cuda_device)
    x, ids, w = L.x.to(cuda_device), L.topk_ids.to(cuda_device), L.topk_weights.to(cuda_device)
    owner, local = EP.snake_placement(w13.shape[0], 1)
    layer = EP.ExpertParallelMoE(owner, local, EP.prefill_expert_fn(w13, w2, 12, 14, 512))
    out = layer(x, ids, w)
    ref = M.moe_prefill(x, w13, w2, ids, w, 12, 14, 512)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("P", [2, 3, 8])
def test_plan_pack_combine_kernels_match_torch_plan(cuda_device, P):
    from kt_gguf_b200 import _native as Nt

    g = torch.Generator().manual_seed(P)
    T, k, E, K = 1000, 8, 64, 256
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    ids[::5, 2] = -1
    w = torch.rand((T, k), generator=g)
    owner, local = EP.snake_placement(E, P)
    owner[7] = -1  # an expert no rank owns
    tok, dest, lid, lw, counts = EP.plan_dispatch(ids, w, owner, local, P)
    layer = EP.ExpertParallelMoE(owner, local, None)
    layer.world = P  # plan for P ranks inside one process
    x = torch.randn((T, K), generator=g).to(torch.bfloat16).to(cuda_device)
    plan = layer._plan(x, ids.to(cuda_device), w.to(cuda_device))
    send_token, meta, counts_d, row_of = plan["send_token"], plan["meta"], plan["counts"], plan["row_of"]
    n = int(counts.sum())
    assert torch.equal(counts_d.cpu().long(), counts)
    assert torch.equal(send_token[:n].cpu().long(), tok)
    assert torch.equal(meta[:n, :k].cpu(), lid)
    assert torch.equal(meta[:n, k:].cpu().view(torch.float32), lw)
    for r in range(P):
        rows = row_of[:, r].cpu()
        sel = rows >= 0
        assert torch.equal(tok[rows[sel].long()], torch.arange(T)[sel])
    lib = Nt.load()
    packed = torch.empty((n, K), dtype=torch.bfloat16, device=cuda_device)
    assert lib.kt_ep_pack(Nt.ptr(x), K, Nt.ptr(send_token), n, Nt.ptr(packed), Nt.stream_of(x)) == 0
    assert torch.equal(packed.cpu(), x.cpu()[tok])
    back = torch.randn((n, K), generator=g).to(torch.bfloat16).to(cuda_device)
    shared = torch.randn((T, K), generator=g).to(torch.bfloat16).to(cuda_device)
    out = torch.empty((T, K), dtype=torch.bfloat16, device=cuda_device)
    assert lib.kt_ep_combine(Nt.ptr(back), Nt.ptr(row_of), P, Nt.ptr(shared), T, K, Nt.ptr(out), Nt.stream_of(x)) == 0
    acc = shared.float().cpu()
    start = 0
    for c in counts.tolist():  # rank order, fp32
        idx = tok[start:start + c]
        acc[idx] += back[start:start + c].float().cpu()
        start += c
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), acc.to(torch.bfloat16))
