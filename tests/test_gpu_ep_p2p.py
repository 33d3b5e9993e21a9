"""The expert-parallel exchange over peer memory on real GPUs.

kt_moe_prefill_counted (the layer over a device-resident row count) runs on one GPU. The
exchange itself needs two GPUs or more: two ranks (NCCL, one process each) run the config-2-like
layer with the 16 hot experts dealt in snake order; the peer-memory exchange (rows written into
the other rank's buffers, partials read from them, CUDA IPC) must equal the NCCL all-to-all
exchange bit for bit (the same rows reach the same layer, and the partials are summed in the same
rank order), over several calls (the alternating output buffers), and stay within the bf16
rounding of the partials of the whole layer on one GPU. Skipped with fewer than two GPUs."""
import datetime
import os
import socket

import pytest
import torch

from kt_gguf_b200 import _native as Nt
from kt_gguf_b200 import ep as EP
from kt_gguf_b200 import kt_gguf_moe_multi as M
from kt_gguf_b200 import synth

pytestmark = pytest.mark.gpu


def test_counted_prefill_equals_prefill_on_the_counted_rows(cuda_device):
    L = synth.make_layer(4, 600, 2048, 512, 32, 8, 12, 14, n_hot=16, zipf=1.1)
    dev = cuda_device
    w13, w2 = torch.from_numpy(L.w13).to(dev), torch.from_numpy(L.w2).to(dev)
    x, ids, w = L.x.to(dev), L.topk_ids.to(dev), L.topk_weights.to(dev)
    fn = EP.prefill_expert_fn(w13, w2, 12, 14, 512)
    for n in (0, 1, 257, 600):
        ref = M.moe_prefill(x[:n].contiguous(), w13, w2, ids[:n].contiguous(), w[:n].contiguous(), 12, 14, 512) \
            if n else None
        out = torch.full((600, 2048), 7.0, dtype=torch.bfloat16, device=dev)
        fn.counted(x, torch.tensor([n], dtype=torch.int32, device=dev), ids, w, out)
        torch.cuda.synchronize()
        if n:
            assert torch.equal(out[:n], ref)
        assert bool((out[n:] == 7.0).all())  # rows past the count are not written


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        L = synth.make_layer(0, 1024, 2048, 512, 64, 8, 12, 14, n_hot=16, zipf=1.1, token_seed=10 + rank)
        S = L.w13.shape[0]
        owner, local = EP.snake_placement(S, world)
        mine = (owner == rank).nonzero().flatten()
        mine = mine[torch.argsort(local[mine])]
        w13_all, w2_all = torch.from_numpy(L.w13).to(dev), torch.from_numpy(L.w2).to(dev)
        w13, w2 = w13_all[mine.to(dev)].contiguous(), w2_all[mine.to(dev)].contiguous()
        x, ids, w = L.x.to(dev), L.topk_ids.to(dev), L.topk_weights.to(dev)
        fn = EP.prefill_expert_fn(w13, w2, 12, 14, 512)
        p2p = EP.ExpertParallelMoE(owner, local, fn, p2p=True)
        nccl = EP.ExpertParallelMoE(owner, local, fn, p2p=False)
        whole = M.moe_prefill(x, w13_all, w2_all, ids, w, 12, 14, 512)
        results = []
        for call in range(3):
            n = 1024 - 100 * call  # token counts change between calls
            a = p2p(x[:n].contiguous(), ids[:n].contiguous(), w[:n].contiguous())
            b = nccl(x[:n].contiguous(), ids[:n].contiguous(), w[:n].contiguous())
            torch.cuda.synchronize()
            err = float((a.float() - whole[:n].float()).norm() / whole[:n].float().norm())
            results.append((bool(torch.equal(a, b)), err))
        p2p.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        q.put((rank, results, None))
    except Exception as e:  # reported to the test
        import traceback

        q.put((rank, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_exchange_equals_nccl_exchange_on_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, results, err in got:
        assert err is None, f"rank {rank}:\n{err}"
        for same, rel in results:
            assert same
            assert rel < 5e-3, rel
