"""Expert-parallel dispatch / combine (kt_gguf_b200.ep) on CPU: the routing plan in one
process, and the full layer on two gloo ranks against a direct per-route computation. The
expert function is a stand-in (an exact fp32 function of the expert id), so these tests
check the exchange, not the GEMMs (those are the GPU parity tests)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kt_gguf_b200 import ep

E, K, T, TOPK = 8, 16, 40, 3


def fake_expert(gid: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """[n] expert ids, [n, K] rows -> [n, K]: a distinct affine map per expert"""
    g = gid.to(torch.float32).unsqueeze(1)
    return x * (g + 1.0) + g * 0.25


def reference(x, ids, w, owner):
    out = torch.zeros_like(x)
    for j in range(ids.shape[1]):
        e = ids[:, j].long()
        ok = (e >= 0) & (owner[e.clamp(min=0)] >= 0)
        out[ok] += w[ok, j:j + 1] * fake_expert(e[ok], x[ok])
    return out


def make_inputs(rank):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn((T, K), generator=g)
    ids = torch.stack([torch.randperm(E, generator=g)[:TOPK] for _ in range(T)]).to(torch.int32)
    ids[::7, 0] = -1  # some routes on the CPU
    w = torch.rand((T, TOPK), generator=g)
    return x, ids, w


def test_plan_groups_rows_by_rank_and_dedups():
    owner, local = ep.contiguous_placement(E, 2)
    ids = torch.tensor([[0, 1, 5], [4, 6, 7], [-1, 2, 3]], dtype=torch.int32)
    w = torch.tensor([[0.1, 0.2, 0.3], [0.4, 0.5, 0.6], [0.7, 0.8, 0.9]])
    tok, dest, lid, lw, counts = ep.plan_dispatch(ids, w, owner, local, 2)
    # rank 0 gets tokens 0 (experts 0,1) and 2 (experts 2,3); rank 1 gets tokens 0 (5) and 1 (4,6,7)
    assert counts.tolist() == [2, 2]
    assert tok.tolist() == [0, 2, 0, 1] and dest.tolist() == [0, 0, 1, 1]
    assert lid.tolist() == [[0, 1, -1], [-1, 2, 3], [-1, -1, 1], [0, 2, 3]]
    assert torch.allclose(lw, torch.tensor([[0.1, 0.2, 0], [0, 0.8, 0.9], [0, 0, 0.3], [0.4, 0.5, 0.6]]))


def test_round_robin_placement():
    hot = torch.tensor([5, 2, 7, 0], dtype=torch.int32)
    owner, local = ep.round_robin_placement(hot, 8, 2)
    # hot[i] -> rank i % 2, slot i // 2: 5 -> (0, 0), 2 -> (1, 0), 7 -> (0, 1), 0 -> (1, 1)
    assert owner.tolist() == [1, -1, 1, -1, -1, 0, -1, 0]
    assert local.tolist() == [1, -1, 0, -1, -1, 0, -1, 1]


def test_snake_placement():
    owner, local = ep.snake_placement(8, 3)
    assert owner.tolist() == [0, 1, 2, 2, 1, 0, 0, 1]
    assert local.tolist() == [0, 0, 0, 1, 1, 1, 2, 2]


def test_single_rank_layer_matches_reference():
    owner, local = ep.contiguous_placement(E, 1)
    x, ids, w = make_inputs(0)
    layer = ep.ExpertParallelMoE(owner, local, lambda xr, lid, lw: sum(
        lw[:, j:j + 1] * torch.where((lid[:, j:j + 1] >= 0), fake_expert(lid[:, j].clamp(min=0), xr), torch.zeros_like(xr))
        for j in range(lid.shape[1])))
    out = layer(x, ids, w)
    assert torch.allclose(out, reference(x, ids, w, owner), rtol=1e-5, atol=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, placement, q, chunks=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if placement == "contiguous":
            owner, local = ep.contiguous_placement(E, world)
        else:
            owner, local = ep.round_robin_placement(torch.tensor([6, 1, 3, 4, 0, 7], dtype=torch.int32), E, world)
        mine = (owner == rank).nonzero().flatten()
        gid_of_slot = torch.full((E,), -1, dtype=torch.long)
        gid_of_slot[local[mine].long()] = mine

        def expert_fn(xr, lid, lw):
            out = torch.zeros_like(xr)
            for j in range(lid.shape[1]):
                ok = lid[:, j] >= 0
                out[ok] += lw[ok, j:j + 1] * fake_expert(gid_of_slot[lid[ok, j].long()], xr[ok])
            return out

        x, ids, w = make_inputs(rank)
        layer = ep.ExpertParallelMoE(owner, local, expert_fn, shared_fn=lambda xx: 0.5 * xx, chunks=chunks)
        out = layer(x, ids, w)
        want = reference(x, ids, w, owner) + 0.5 * x
        q.put((rank, float((out - want).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("placement,chunks", [("contiguous", 1), ("round_robin", 1), ("contiguous", 3)])
def test_two_gloo_ranks_match_reference(placement, chunks):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, placement, q, chunks)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) < 1e-4, res
